"""The reference-facing API: logit_processors mirror and the sampler entry
points.  Structure follows the reference's tests/test_logit_processors.py and
tests/test_optimized_single_logits_migration.py."""

import enum

import numpy as np
import pytest
import torch

from mapperatorinator_b200 import _native as N
from mapperatorinator_b200 import logit_processors as LP
from mapperatorinator_b200 import sampling as S
from tests import _golden as G


class EventType(enum.Enum):
    TIME_SHIFT = "t"
    BEAT = "beat"
    MEASURE = "measure"
    TIMING_POINT = "timing_point"
    CIRCLE = "circle"
    HOLD_NOTE = "hold_note"
    HOLD_NOTE_END = "hold_note_end"
    SCROLL_SPEED = "scroll_speed"


class _FakeTokenizer:
    sos_id = 1
    context_sos = {}
    event_start = {EventType.TIME_SHIFT: 10}
    event_end = {EventType.TIME_SHIFT: 20}


def _apply(processor, input_ids, scores):
    return processor(input_ids.clone(), scores.clone())


# ---------------------------------------------------------------- CPU: construction and errors
def test_rejects_optimized_stateful_mode():
    with pytest.raises(ValueError, match="moved to optimized single inference"):
        LP.MonotonicTimeShiftLogitsProcessor(_FakeTokenizer(), stateful_batch1=True)


def test_lookback_warper_constructs_from_tokenizer():
    m = G.case("lookback_renorm")["meta"]
    w = LP.LookbackBiasLogitsWarper(m["lookback_time"], G.lookback_tokenizer(m), True, "cpu")
    assert (w.lookback_start, w.lookback_end, w.eos_ids) == (16, 66, (2, 4, 5))
    lst = LP.build_logits_processor_list(G.lookback_tokenizer(m), types_first=False, lookback_time=100.0)
    assert lst[0].lookback["mode"] == N.LOOKBACK_MASK and lst[0].lookback["end"] == 16 + 20 + 10
    with pytest.raises(ValueError):
        LP.LookbackBiasLogitsWarper(5000.0, G.lookback_tokenizer(m), True, "cpu")


def test_token_helpers():
    class Tok:
        event_start = {EventType.BEAT: 130, EventType.MEASURE: 131, EventType.TIMING_POINT: 132,
                       EventType.CIRCLE: 140, EventType.HOLD_NOTE: 141, EventType.HOLD_NOTE_END: 142,
                       EventType.SCROLL_SPEED: 150, EventType.TIME_SHIFT: 0}
        event_end = {EventType.SCROLL_SPEED: 153, EventType.TIME_SHIFT: 100}

    assert LP.get_beat_type_tokens(Tok) == (130, 131, 132)
    assert LP.get_mania_type_tokens(Tok) == (140, 141, 142)
    assert LP.get_scroll_speed_tokens(Tok) == (150, 151, 152)
    assert LP.get_mania_type_tokens(_FakeTokenizer) == ()


def test_cpu_tensors_rejected():
    p = LP.MonotonicTimeShiftLogitsProcessor(_FakeTokenizer())
    with pytest.raises(ValueError, match="CUDA"):
        p(torch.tensor([[1, 12]]), torch.zeros(1, 64))


def test_bad_warper_params():
    with pytest.raises(ValueError):
        LP.FusedLogitsProcessor(top_p=0.0)
    with pytest.raises(ValueError):
        LP.FusedLogitsProcessor(temperature=0.0)


# ---------------------------------------------------------------- GPU: reference test vectors
@pytest.mark.gpu
def test_v32_monotonic_full_scan_masks_earlier_time_shifts(cuda_device):
    processor = LP.MonotonicTimeShiftLogitsProcessor(_FakeTokenizer())
    input_ids = torch.tensor([[1, 12, 5, 15, 3]], dtype=torch.long, device=cuda_device)
    scores = (torch.arange(64, dtype=torch.float32).reshape(1, 64) / 10).to(cuda_device)
    result = _apply(processor, input_ids, scores)
    assert torch.isneginf(result[0, 10:15]).all()
    assert torch.equal(result[0, 15:], scores[0, 15:])


@pytest.mark.gpu
def test_conditional_temperature_is_batch_correct_with_first_match_precedence(cuda_device):
    processor = LP.ConditionalTemperatureLogitsWarper(
        temperature=1.0, timing_temperature=2.0, mania_column_temperature=4.0, taiko_hit_temperature=8.0,
        types_first=True, beat_type_tokens=(10, 11), mania_type_tokens=(20,), scroll_speed_tokens=(30,))
    input_ids = torch.tensor([[0, 0, 10], [20, 0, 0], [0, 0, 30], [20, 0, 10], [0, 0, 0]], device=cuda_device)
    scores = torch.full((5, 64), 8.0, device=cuda_device)
    result = processor(input_ids, scores)
    assert torch.equal(result[:, 0].cpu(), torch.tensor([4.0, 2.0, 1.0, 4.0, 8.0]))


@pytest.mark.gpu
def test_conditional_temperature_preserves_batch1_calculation(cuda_device):
    processor = LP.ConditionalTemperatureLogitsWarper(1.0, 2.0, 1.0, 1.0, True, (10,), (), ())
    scores = torch.tensor([[3.0, 5.0] + [0.0] * 30], device=cuda_device)
    assert torch.equal(processor(torch.tensor([[0, 10]], device=cuda_device), scores), scores / 2.0)


@pytest.mark.gpu
def test_stateful_monotonic_matches_full_scan_for_growing_prefixes(cuda_device):
    tok = _FakeTokenizer()
    full_scan = LP.MonotonicTimeShiftLogitsProcessor(tok)
    stateful = LP.StatefulMonotonicTimeShiftLogitsProcessor(tok)
    tokens = torch.tensor([[1, 12, 5, 11, 7, 15, 3, 1, 14, 9]], device=cuda_device)
    ref = G.case("ref_stateful_prefixes")["out"]
    for length in range(1, tokens.shape[1] + 1):
        scores = (torch.arange(64, dtype=torch.float32).reshape(1, 64) / 10).to(cuda_device)
        a = _apply(full_scan, tokens[:, :length], scores)
        b = _apply(stateful, tokens[:, :length], scores)
        assert torch.equal(a, b)
        assert np.array_equal(b.cpu().numpy()[0], ref[length - 1])


@pytest.mark.gpu
def test_stateful_monotonic_reinitializes_after_sequence_jump(cuda_device):
    tok = _FakeTokenizer()
    full_scan = LP.MonotonicTimeShiftLogitsProcessor(tok)
    stateful = LP.StatefulMonotonicTimeShiftLogitsProcessor(tok)
    scores = (torch.arange(64, dtype=torch.float32).reshape(1, 64) / 10).to(cuda_device)
    _apply(stateful, torch.tensor([[1, 12, 5, 13]], device=cuda_device), scores)
    second = torch.tensor([[1, 18, 4]], device=cuda_device)
    assert torch.equal(_apply(full_scan, second, scores), _apply(stateful, second, scores))


@pytest.mark.gpu
@pytest.mark.parametrize("batch_size", [1, 2, 5])
def test_monotonic_random_trials_match_reference(cuda_device, batch_size):
    c = G.case(f"ref_random_b{batch_size}")
    full_scan = LP.MonotonicTimeShiftLogitsProcessor(_FakeTokenizer())
    for t in range(c["input_ids"].shape[0]):
        L = int(c["lens"][t])
        ids = torch.from_numpy(np.ascontiguousarray(c["input_ids"][t, :, :L])).to(cuda_device)
        sc = torch.from_numpy(c["scores"][t]).to(cuda_device)
        candidate = LP.StatefulMonotonicTimeShiftLogitsProcessor(_FakeTokenizer())
        assert np.array_equal(_apply(full_scan, ids, sc).cpu().numpy(), c["out"][t])
        assert np.array_equal(_apply(candidate, ids, sc).cpu().numpy(), c["out"][t])


# ---------------------------------------------------------------- GPU: full chain vs reference fixtures
def _tokenizer_for(meta):
    class Tok:
        pass

    t = Tok()
    t.sos_id = meta["sos"][0]
    t.context_sos = {i: s for i, s in enumerate(meta["sos"][1:])}
    t.event_start = {EventType.TIME_SHIFT: meta["ts"][0]}
    t.event_end = {EventType.TIME_SHIFT: meta["ts"][1]}
    for name, (a, b) in meta.get("extra", {}).items():
        t.event_start[EventType[name]] = a
        t.event_end[EventType[name]] = b
    return t


def _chain(name, **kw):
    c = G.case(name)
    m = c["meta"]
    t = m["temps"]
    procs = LP.build_logits_processor_list(
        _tokenizer_for(m), cfg_scale=m["cfg"], timeshift_bias=m["bias"], types_first=m["types_first"],
        temperature=t[0], timing_temperature=t[1], mania_column_temperature=t[2], taiko_hit_temperature=t[3], **kw)
    return c, m, procs


@pytest.mark.gpu
@pytest.mark.parametrize("name", G.CHAIN_CASES)
def test_build_logits_processor_list_matches_reference(cuda_device, name):
    c, m, procs = _chain(name)
    x = torch.from_numpy(c["logits"]).to(cuda_device)
    if m.get("dtype") == "bf16":
        x = x.to(torch.bfloat16)
    ids = torch.from_numpy(c["input_ids"]).to(cuda_device)
    out = procs(ids, x).cpu().numpy()
    assert np.array_equal(out.view(np.uint32), c["processed"].view(np.uint32))


@pytest.mark.gpu
@pytest.mark.parametrize("name", G.CHAIN_CASES)
@pytest.mark.parametrize("stateful", [False, True])
def test_fused_warpers_match_reference_keep_sets(cuda_device, name, stateful):
    factory = LP.StatefulMonotonicTimeShiftLogitsProcessor if stateful else LP.MonotonicTimeShiftLogitsProcessor
    c, m, procs = _chain(name, top_k=m_topk(name), top_p=G.case(name)["meta"]["top_p"],
                         monotonic_processor_factory=factory)
    x = torch.from_numpy(c["logits"]).to(cuda_device)
    ids = torch.from_numpy(c["input_ids"]).to(cuda_device)
    out = procs(ids, x).cpu().numpy()
    ref = c["final_hf"]
    for row in range(out.shape[0]):
        kg, kr = np.isfinite(out[row]), np.isfinite(ref[row])
        if not np.array_equal(kg, kr):
            # documented tie rule (lowest id first) or a sub-1e-5 mass margin
            assert G.explain_keep_mismatch(c["processed"][row], kr, kg, m["top_p"]), row
        else:
            assert np.array_equal(out[row][kg], ref[row][kr])


def m_topk(name):
    return G.case(name)["meta"]["top_k"]


@pytest.mark.gpu
@pytest.mark.parametrize("name", G.CHAIN_CASES)
def test_sample_entry_point_greedy_and_keep_set(cuda_device, name):
    c = G.case(name)
    m = c["meta"]
    proc = torch.from_numpy(c["processed"]).to(cuda_device)
    greedy = S._sample(proc, False, m["top_p"], m["top_k"], 1.0)
    assert greedy.shape == (proc.shape[0], 1)
    assert np.array_equal(greedy.cpu().numpy(), c["greedy"])
    keep = c["sample_fn_probs"] > 0
    gen = torch.Generator(cuda_device).manual_seed(3)
    for _ in range(64):
        ids = S._sample(proc, True, m["top_p"], m["top_k"], 1.0, generator=gen).cpu().numpy()[:, 0]
        for r, t in enumerate(ids):
            # a token outside the reference keep set may only come from a tie at the cut
            if not keep[r, t]:
                x = c["processed"][r]
                assert x[t] == x[keep[r]].min(), (r, t)


@pytest.mark.gpu
@pytest.mark.parametrize("top_k,top_p", [(0, 1.0), (20, 0.9)])
def test_sample_distribution_matches_multinomial(cuda_device, top_k, top_p):
    """Inverse-CDF draws from uniforms against torch.multinomial, 2^20 draws each:
    a goodness-of-fit chi-square of our draws against the exact renormalised
    probabilities, and a two-sample chi-square of our histogram against
    torch.multinomial's (the reference's sampler) on the same probabilities."""
    torch.manual_seed(0)
    V = 64
    logits = torch.randn(1, V, device=cuda_device) * 1.5
    n = 1 << 20
    u = torch.rand(n, device=cuda_device)
    rows = logits.expand(n, V).contiguous()
    ours = S._sample(rows, True, top_p, top_k, 1.0, uniforms=u).view(-1)
    counts = torch.bincount(ours, minlength=V).double().cpu()
    # the reference's probabilities: HF top-k then the _sample top-p rule, softmax
    x = logits.double().cpu()[0]
    if top_k:
        x = torch.where(x < torch.topk(x, top_k).values[-1], torch.tensor(float("-inf"), dtype=x.dtype), x)
    if top_p < 1.0:
        sx, si = torch.sort(x, descending=True)
        cum = torch.softmax(sx, -1).cumsum(-1)
        rm = cum > top_p
        rm[1:] = rm[:-1].clone()
        rm[0] = False
        x = x.scatter(0, si, sx.masked_fill(rm, float("-inf")))
    p = torch.softmax(x, -1)
    expected = p * n
    mask = expected > 5
    chi2 = (((counts - expected) ** 2) / expected)[mask].sum().item()
    dof = int(mask.sum()) - 1
    assert chi2 < dof + 6 * (2 * dof) ** 0.5, (chi2, dof)
    assert counts[p == 0].sum() == 0  # nothing outside the keep set
    theirs = torch.bincount(torch.multinomial(p.float().to(cuda_device), n, replacement=True), minlength=V)
    theirs = theirs.double().cpu()
    both = (counts + theirs) > 0
    chi2b = (((counts - theirs) ** 2) / (counts + theirs))[both].sum().item()
    dofb = int(both.sum()) - 1
    assert chi2b < dofb + 6 * (2 * dofb) ** 0.5, (chi2b, dofb)


@pytest.mark.gpu
def test_fused_sampler_public_api_matches_oracle(cuda_device):
    from tests.harness import workloads as W
    from oracle import oracle

    s = W.batched_decode(seed=5, pairs=32)
    class_of = torch.from_numpy(s.grammar_class_of).to(cuda_device)
    allow = torch.from_numpy(s.grammar_allow.view(np.int32)).to(cuda_device)
    fs = S.FusedSampler(vocab_size=4096, num_rows=32, device=cuda_device, cfg_scale=1.5, time_shift_range=(0, 2000),
                        sos_ids=s.sos_ids, grammar=S.GrammarTable(class_of, allow),
                        column_temperatures=s.col_ranges, top_p=0.9, return_scores=True)
    fs.mono_state.copy_(torch.from_numpy(s.mono_state))
    fs.prev_token.copy_(torch.from_numpy(s.prev_token))
    fs._scan_next = fs._prev_from_ids_next = False
    host = s.with_(flags=N.FLAG_MONO_UPDATE_FROM_SAMPLE | N.FLAG_GRAMMAR_UPDATE_FROM_SAMPLE, want_scores=True)
    rng = np.random.default_rng(1)
    for _ in range(5):
        x = rng.normal(0, 1.5, size=(64, 4096)).astype(np.float32)
        u = rng.random(32, dtype=np.float32)
        host = host.with_(logits=W.bf16_bits(x), uniforms=u)
        ref = oracle.run(host)
        logits = torch.from_numpy(x).to(cuda_device).to(torch.bfloat16)
        ids = fs.step(logits, uniforms=torch.from_numpy(u).to(cuda_device))
        torch.cuda.synchronize()
        assert np.array_equal(ids.cpu().numpy(), ref["out_ids"])
        assert np.array_equal(fs.mono_state.cpu().numpy(), ref["mono_state"])
        assert np.array_equal(fs.scores.cpu().numpy().view(np.uint32), ref["out_scores"].view(np.uint32))
        host = host.with_(mono_state=ref["mono_state"], prev_token=ref["prev_token"])


@pytest.mark.gpu
@pytest.mark.parametrize("name", ["ref_decode_pad", "ref_decode_pad_random"])
def test_fused_sampler_pads_finished_rows_like_the_reference_loop(cuda_device, name):
    """FusedSampler(track_finished=True), greedy, against the tokens the
    reference's active_prefix_decode_generate emits for the same scripted
    logits: finished rows get pad 0 and the loop state follows the EOS 2."""
    import torch

    from mapperatorinator_b200.sampling import FusedSampler

    c = G.case(name)
    sched, want = c["schedule"], c["generated"]
    steps, rows = sched.shape
    s = FusedSampler(vocab_size=8, num_rows=rows, device=cuda_device, do_sample=False, eos_token_ids=(2,),
                     pad_token_id=0, track_finished=True)
    for t in range(steps):
        x = torch.full((rows, 8), -1000.0, device=cuda_device)
        x[torch.arange(rows), torch.from_numpy(sched[t]).to(cuda_device)] = 1000.0
        ids = s.step(x)
        assert torch.equal(ids.cpu(), torch.from_numpy(want[:, t])), t
    assert not s.unfinished.any().item()


# ---------------------------------------------------------------- GPU: lookback bias
@pytest.mark.gpu
@pytest.mark.parametrize("name", ["lookback_renorm", "lookback_mask"])
def test_lookback_warper_matches_reference(cuda_device, name):
    c = G.case(name)
    m = c["meta"]
    w = LP.LookbackBiasLogitsWarper(m["lookback_time"], G.lookback_tokenizer(m), m["types_first"], cuda_device)
    for t in range(m["steps"]):
        ids = torch.from_numpy(c["input_ids"][:, : m["prefix"] + t + 1]).to(cuda_device)
        x = torch.from_numpy(c["scores"][t]).to(cuda_device)
        x0 = x.clone()
        out = w(ids, x).cpu().numpy()
        assert torch.equal(x, x0)  # the reference returns a new tensor when it changes scores
        assert G.lookback_close(out, c["out"][t], 16) == [], t
    w.reset()  # forgets the previous scores: the next call is a first call again
    ids = torch.from_numpy(c["input_ids"][:, : m["prefix"] + 1]).to(cuda_device)
    out = w(ids, torch.from_numpy(c["scores"][0]).to(cuda_device)).cpu().numpy()
    assert G.lookback_close(out, c["out"][0], 16) == []


@pytest.mark.gpu
def test_build_logits_processor_list_with_lookback_matches_reference(cuda_device):
    c = G.case("lookback_chain")
    m = c["meta"]
    procs = LP.build_logits_processor_list(G.lookback_tokenizer(m), cfg_scale=m["cfg"], timeshift_bias=m["bias"],
                                           types_first=True, temperature=m["temps"][0],
                                           timing_temperature=m["temps"][1], lookback_time=m["lookback_time"])
    for t in range(m["steps"]):
        ids = torch.from_numpy(c["input_ids"][:, : m["prefix"] + t + 1]).to(cuda_device)
        out = procs(ids, torch.from_numpy(c["logits"][t]).to(cuda_device)).cpu().numpy()
        assert G.lookback_close(out, c["processed"][t], 16) == [], t


@pytest.mark.gpu
def test_fused_sampler_with_lookback_matches_oracle(cuda_device):
    from tests.harness import workloads as W
    from oracle import oracle

    s0 = W.lookback_decode(seed=21, pairs=48, vocab=4096, dtype="bf16")
    timed = [t for t in range(4096) if (s0.lb_timed_bits[t >> 5] >> (t & 31)) & 1]
    spec = {"mode": N.LOOKBACK_RENORM, "start": s0.lb_start, "end": s0.lb_end, "eos_ids": s0.lb_eos_ids,
            "timed": timed}
    fs = S.FusedSampler(vocab_size=4096, num_rows=48, device=cuda_device, cfg_scale=1.5, temperature=0.9, top_k=40,
                        top_p=0.9, lookback=spec, return_logprobs=True)
    state = np.full(48, np.nan, dtype=np.float32)
    with pytest.raises(ValueError):
        fs.step(torch.zeros((96, 4096), device=cuda_device))  # the bias needs input_ids
    for step in range(4):
        host = W.lookback_decode(seed=21, pairs=48, vocab=4096, dtype="bf16", step=step, lb_state=state)
        host = host.with_(mono_mode=N.MONO_OFF, mono_state=None, want_logprobs=True)
        ref = oracle.run(host)
        logits = torch.from_numpy(W.bf16_to_f32(host.logits)).to(cuda_device).to(torch.bfloat16)
        ids = fs.step(logits, torch.from_numpy(host.input_ids).to(cuda_device),
                      uniforms=torch.from_numpy(host.uniforms).to(cuda_device))
        torch.cuda.synchronize()
        assert np.array_equal(ids.cpu().numpy(), ref["out_ids"]), step
        got_state = fs.lb_state.cpu().numpy()
        assert np.array_equal(got_state.view(np.uint32), ref["lb_state"].view(np.uint32)) or \
            np.array_equal(got_state, ref["lb_state"], equal_nan=True)
        state = ref["lb_state"]
    fs.reset()
    assert torch.isnan(fs.lb_state).all()


@pytest.mark.gpu
def test_fused_sampler_graph_step_appends_and_stops(cuda_device):
    """A whole token step in one CUDA graph: a stand-in decoder (embedding of the
    previous token -> lm_head matmul) and FusedSampler.step appending at a
    device-side cur_len that the graph advances; compared with eager steps."""
    from mapperatorinator_b200.sampling import FusedSampler

    B, V, d, steps = 16, 512, 64, 12
    g = torch.Generator(device=cuda_device).manual_seed(3)
    emb = torch.randn((V, d), device=cuda_device, generator=g)
    head = torch.randn((V, d), device=cuda_device, generator=g) * 0.5

    def make():
        return FusedSampler(vocab_size=V, num_rows=B, device=cuda_device, top_p=0.9, eos_token_ids=(3,),
                            pad_token_id=0, track_finished=True)

    uniforms = torch.rand((steps, B), device=cuda_device, generator=g)
    # eager
    eager = make()
    buf_e = torch.full((B, steps + 4), -1, dtype=torch.int64, device=cuda_device)
    buf_e[:, :2] = 1
    for t in range(steps):
        logits = emb[buf_e[:, 1 + t]] @ head.T
        eager.step(logits, buf_e[:, : 2 + t], uniforms=uniforms[t], id_buffer=buf_e, cur_len=2 + t)
    # graph: one capture of the whole step, replayed `steps` times
    fs = make()
    buf = torch.full((B, steps + 4), -1, dtype=torch.int64, device=cuda_device)
    buf[:, :2] = 1
    cur = torch.tensor([2], dtype=torch.int32, device=cuda_device)
    u = torch.empty(B, device=cuda_device)
    prev = torch.empty(B, dtype=torch.int64, device=cuda_device)

    def one_step():
        prev.copy_(buf.gather(1, (cur.long() - 1).expand(B, 1)).squeeze(1))
        logits = emb[prev] @ head.T
        fs.step(logits, None, uniforms=u, id_buffer=buf, cur_len=cur)
        cur.add_(1)

    s = torch.cuda.Stream(cuda_device)
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        u.copy_(uniforms[0])
        one_step()  # warm-up outside the capture
    torch.cuda.current_stream().wait_stream(s)
    torch.cuda.synchronize()
    buf[:, 2:] = -1
    cur.fill_(2)
    fs.reset()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        one_step()
    torch.cuda.synchronize()
    buf[:, 2:] = -1
    cur.fill_(2)
    fs.reset()
    for t in range(steps):
        u.copy_(uniforms[t])
        graph.replay()
    torch.cuda.synchronize()
    assert torch.equal(buf, buf_e)
    assert torch.equal(fs.stop_counts, eager.stop_counts)
    assert torch.equal(fs.unfinished, eager.unfinished)
    assert fs.all_finished() == eager.all_finished()
    assert int(cur.item()) == 2 + steps
    del graph


def test_row_status_report_reads_the_contract():
    # a hand-built step: row 1 non-finite, row 4 and every later row of its CTA lost
    # their staged copy (header: MTR_ROW_COPY_TIMEOUT), row 2 a tie at the cut (info only)
    status = np.zeros(8, dtype=np.uint32)
    status[1] = N.ROW_NONFINITE
    status[2] = N.ROW_TIE_AT_CUT
    status[4] = N.ROW_COPY_TIMEOUT | N.ROW_SLOW_PATH
    status[6] = N.ROW_COPY_TIMEOUT
    ids = np.array([5, 7, 9, 11, 7, 13, 7, 2], dtype=np.int64)
    rep = S.row_status_report(status, ids, pad_id=7)
    assert rep["padded"] == [1, 4, 6]
    assert rep["copy_timeout"] == [4, 6] and rep["tie_at_cut"] == [2] and rep["nonfinite"] == [1]
    assert "bad_id" not in rep
    ids[6] = 3  # a timed-out row that kept another token breaks the contract
    with pytest.raises(ValueError):
        S.row_status_report(status, ids, pad_id=7)
    # int32 tensors (FusedSampler.status) read the same way
    assert S.row_status_report(torch.from_numpy(status.view(np.int32)))["padded"] == [1, 4, 6]

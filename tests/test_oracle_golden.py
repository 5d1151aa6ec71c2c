"""Pin the CPU oracle to the reference: fixtures produced by running the
reference's own processors (tests/golden/make_golden.py).  CPU only."""

import numpy as np
import pytest

from mapperatorinator_b200 import _native as N
from oracle import oracle
from tests import _golden as G


def test_reference_monotonic_vector():
    # tests/test_logit_processors.py:43-51: ids [1,12,5,15,3], TS 10..19 -> -inf on 10..14
    c = G.case("ref_mono_vector")
    s = G.StepInputs(logits=c["scores"], dtype="f32", num_rows=1, input_ids=c["input_ids"], mono_mode=N.MONO_SCAN,
                     ts_start=10, ts_end=20, sos_ids=(1,), select_mode=N.SELECT_NONE, want_scores=True)
    out = oracle.run(s)["out_scores"]
    assert np.array_equal(out, c["out"])
    assert np.isneginf(out[0, 10:15]).all()
    assert np.array_equal(out[0, 15:], c["scores"][0, 15:])


def test_reference_conditional_temperature_batch():
    # tests/test_logit_processors.py:63-91: first-match precedence -> [4, 2, 1, 4, 8]
    c = G.case("ref_condtemp_batch")
    conds = [(2.0, 1, G.bits_for([10, 11], 64)), (4.0, 3, G.bits_for([20], 64)), (8.0, 1, G.bits_for([30], 64))]
    logits = np.zeros((5, 64), dtype=np.float32)
    logits[:, :4] = c["scores"]
    s = G.StepInputs(logits=logits, dtype="f32", num_rows=5, input_ids=c["input_ids"], temp_mode=N.TEMP_ROW_CONDITIONAL,
                     temperature=1.0, cond=conds, select_mode=N.SELECT_NONE, want_scores=True)
    out = oracle.run(s)["out_scores"][:, :4]
    assert np.array_equal(out, c["out"])
    assert np.array_equal(out[:, 0], np.array([4.0, 2.0, 1.0, 4.0, 8.0], dtype=np.float32))


def test_reference_stateful_prefixes_match_state_mode():
    # optimized/single/logits.py stateful processor over growing prefixes
    c = G.case("ref_stateful_prefixes")
    seq = c["input_ids"]
    scores = (np.arange(64, dtype=np.float32) / 10).reshape(1, 64)
    state = np.array([-1], dtype=np.int32)
    for n in range(1, seq.shape[1] + 1):
        ids = seq[:, :n]
        mode, flags = (N.MONO_SCAN, 0) if n == 1 else (N.MONO_STATE, N.FLAG_MONO_UPDATE_FROM_IDS)
        s = G.StepInputs(logits=scores, dtype="f32", num_rows=1, input_ids=ids, mono_mode=mode, flags=flags,
                         ts_start=10, ts_end=20, sos_ids=(1,), mono_state=state, select_mode=N.SELECT_NONE,
                         want_scores=True)
        r = oracle.run(s)
        state = r["mono_state"]
        assert np.array_equal(r["out_scores"][0], c["out"][n - 1]), n


@pytest.mark.parametrize("bsz", [1, 2, 5])
def test_reference_random_full_scan_trials(bsz):
    # test_optimized_single_logits_migration.py:59-78 inputs, reference full-scan outputs
    c = G.case(f"ref_random_b{bsz}")
    for t in range(c["input_ids"].shape[0]):
        L = int(c["lens"][t])
        ids = np.ascontiguousarray(c["input_ids"][t, :, :L])
        s = G.StepInputs(logits=c["scores"][t], dtype="f32", num_rows=bsz, input_ids=ids, mono_mode=N.MONO_SCAN,
                         ts_start=10, ts_end=20, sos_ids=(1,), select_mode=N.SELECT_NONE, want_scores=True)
        assert np.array_equal(oracle.run(s)["out_scores"], c["out"][t]), t


@pytest.mark.parametrize("name", G.CHAIN_CASES)
def test_chain_processed_scores_bit_exact(name):
    # CFG -> monotonic -> [bias] -> temperature, exactly as build_logits_processor_list
    c = G.case(name)
    out = oracle.run(G.chain_step(name))["out_scores"]
    ref = c["processed"]
    assert out.view(np.uint32).tolist() == ref.view(np.uint32).tolist() or np.array_equal(out, ref)


@pytest.mark.parametrize("name", G.CHAIN_CASES)
def test_chain_hf_warpers_keep_set(name):
    c = G.case(name)
    m = c["meta"]
    r = oracle.run(G.chain_step(name, top_k=m["top_k"], top_p=m["top_p"], top_p_mode=N.TOPP_HF))
    out, ref = r["out_scores"], c["final_hf"]
    for row in range(out.shape[0]):
        kg, kr = np.isfinite(out[row]), np.isfinite(ref[row])
        if not np.array_equal(kg, kr):
            assert G.explain_keep_mismatch(c["processed"][row], kr, kg, m["top_p"], int(r["out_status"][row])), row
        else:
            assert np.array_equal(out[row][kg], ref[row][kr])


@pytest.mark.parametrize("name", G.CHAIN_CASES)
def test_chain_sample_fn_keep_set(name):
    # compiled_decode._sample: top-k then descending-cumsum top-p (shifted by one)
    c = G.case(name)
    m = c["meta"]
    r = oracle.run(G.chain_step(name, top_k=m["top_k"], top_p=m["top_p"], top_p_mode=N.TOPP_SAMPLE_FN))
    for row in range(r["out_scores"].shape[0]):
        kg = np.isfinite(r["out_scores"][row])
        kr = c["sample_fn_probs"][row] > 0
        if not np.array_equal(kg, kr):
            assert G.explain_keep_mismatch(c["processed"][row], kr, kg, m["top_p"], int(r["out_status"][row])), row


@pytest.mark.parametrize("name", G.CHAIN_CASES)
def test_chain_greedy_ids(name):
    c = G.case(name)
    r = oracle.run(G.chain_step(name, select_mode=N.SELECT_ARGMAX))
    assert np.array_equal(r["out_ids"], c["greedy"].reshape(-1))


def test_hf_repetition_penalty_then_warpers():
    c = G.case("hf_repetition")
    x = c["logits"]
    s = G.StepInputs(logits=G.bf16_bits(x), dtype="bf16", num_rows=x.shape[0], input_ids=c["input_ids"],
                     repetition_penalty=1.1, select_mode=N.SELECT_NONE, want_scores=True)
    assert np.array_equal(oracle.run(s)["out_scores"], c["processed"])
    r = oracle.run(s.with_(top_k=50, top_p=0.95))
    out, ref = r["out_scores"], c["final_hf"]
    for row in range(out.shape[0]):
        kg, kr = np.isfinite(out[row]), np.isfinite(ref[row])
        if not np.array_equal(kg, kr):
            assert G.explain_keep_mismatch(c["processed"][row], kr, kg, 0.95, int(r["out_status"][row])), row


# ---------------------------------------------------------------- the CPU port used by bench.py
@pytest.mark.parametrize("name", ["chain_cfg_mono_temp", "chain_bias_cfg2", "chain_c0_shape", "chain_c1_bf16",
                                  "hf_repetition"])
def test_torch_chain_port_matches_reference(name):
    """oracle/torch_chain.py (the CPU chain bench.py falls back to) reproduces the
    reference's processed scores and HF-warped scores bit for bit."""
    import torch

    from oracle import torch_chain as TC

    c = G.case(name)
    m = c["meta"]
    logits = torch.from_numpy(c["logits"].astype(np.float32))
    ids = torch.from_numpy(c["input_ids"].astype(np.int64))
    if name == "hf_repetition":
        prm = TC.ChainParams(repetition_penalty=m["penalty"])
    else:
        prm = TC.ChainParams(cfg_scale=m["cfg"], ts_range=tuple(m["ts"]), sos_ids=tuple(m["sos"]),
                             timeshift_bias=m["bias"], temperature=m["temps"][0])
    got = TC.processed_scores(logits, ids, prm).numpy()
    assert np.array_equal(got.view(np.uint32), c["processed"].view(np.uint32))
    prm.top_k, prm.top_p = m["top_k"], m["top_p"]
    got = TC.processed_scores(logits, ids, prm).numpy()
    assert np.array_equal(got.view(np.uint32), c["final_hf"].view(np.uint32))


@pytest.mark.parametrize("name", ["ref_decode_pad", "ref_decode_pad_random"])
def test_oracle_decode_loop_pad_and_finished(name):
    """Pad-on-finished and EOS tracking step by step, pinned to the reference's
    own decode loop (active_prefix_decode_generate on scripted one-hot logits)."""
    from tests.harness.workloads import StepInputs

    c = G.case(name)
    sched, want = c["schedule"], c["generated"]
    steps, rows = sched.shape
    unf = np.ones(rows, dtype=np.uint8)
    prompt = 3
    buf = np.full((rows, prompt + steps + 2), -1, dtype=np.int64)
    counts = np.zeros(2, dtype=np.uint32)
    for t in range(steps):
        x = np.full((rows, 8), -1000.0, dtype=np.float32)
        x[np.arange(rows), sched[t]] = 1000.0
        s = StepInputs(logits=x, dtype="f32", num_rows=rows, select_mode=N.SELECT_ARGMAX, unfinished=unf,
                       pad_id=0, eos_ids=(2,), id_buffer=buf, cur_len=prompt + t, stop_counts=counts)
        r = oracle.run(s)
        assert np.array_equal(r["out_ids"], want[:, t]), t
        unf, buf, counts = r["unfinished"], r["id_buffer"], r["stop_counts"]
        # the reference loop runs until every row has finished: [1] == rows exactly at its last step
        assert (counts[1] == rows) == (t == steps - 1), t
        assert counts[1] == rows - int(unf.sum())
    assert not unf.any()
    # the appended columns are the reference loop's generated tokens (torch.cat at cur_len)
    assert np.array_equal(buf[:, prompt: prompt + steps], want)
    assert (buf[:, :prompt] == -1).all() and (buf[:, prompt + steps:] == -1).all()
    # [0] counts live rows that emitted an EOS: one per row here
    assert counts[0] == rows


def test_oracle_append_skips_out_of_range_column():
    from tests.harness.workloads import StepInputs

    x = np.zeros((2, 8), dtype=np.float32)
    buf = np.full((2, 4), -1, dtype=np.int64)
    r = oracle.run(StepInputs(logits=x, dtype="f32", num_rows=2, select_mode=N.SELECT_ARGMAX, id_buffer=buf,
                              cur_len_dev=np.array([4], dtype=np.int32)))
    assert (r["out_status"] & N.ROW_APPEND_SKIPPED).all() and (r["id_buffer"] == -1).all()
    r = oracle.run(StepInputs(logits=x, dtype="f32", num_rows=2, select_mode=N.SELECT_ARGMAX, id_buffer=buf,
                              cur_len_dev=np.array([3], dtype=np.int32), cur_len=99))
    assert (r["out_status"] == 0).all() and (r["id_buffer"][:, 3] == 0).all()


def test_lookback_spec_from_tokenizer():
    # logit_processors.py:127-141 on the fixture's layout: TIME_SHIFT values from -20,
    # lookback 300 ms -> value 30 -> ids [16, 16 + 20 + 30); eos + context eos; timed ids
    from mapperatorinator_b200.logit_processors import lookback_spec

    m = G.case("lookback_renorm")["meta"]
    tok = G.lookback_tokenizer(m)
    spec = lookback_spec(m["lookback_time"], tok, True)
    assert (spec["start"], spec["end"]) == (16, 66)
    assert spec["eos_ids"] == (2, 4, 5)
    assert spec["mode"] == N.LOOKBACK_RENORM
    assert sorted(spec["timed"]) == sorted(t for k, (a, b) in m["extra"].items() if k != "SCROLL_SPEED"
                                           for t in range(a, b))
    assert lookback_spec(m["lookback_time"], tok, False)["mode"] == N.LOOKBACK_MASK
    with pytest.raises(ValueError):
        lookback_spec(2000.0, tok, True)  # value 200 > max 79


@pytest.mark.parametrize("name", G.LOOKBACK_CASES)
def test_lookback_oracle_matches_reference(name):
    # consecutive calls carry the previous EOS probability; step 0 has none (no bias)
    c = G.case(name)
    steps, B = c["meta"]["steps"], c["input_ids"].shape[0]
    state = np.full(B, np.nan, dtype=np.float32)
    transformed = 0
    for t in range(steps):
        r = oracle.run(G.lookback_step(name, t, state))
        ref = G.lookback_reference(name, t)
        assert G.lookback_close(r["out_scores"], ref, 16) == [], t
        if c["meta"]["types_first"]:
            state = r["lb_state"]
            assert np.isfinite(state).all()
            transformed += int(np.isneginf(ref[:, 17:66]).all(axis=1).sum())
    if c["meta"]["types_first"]:
        assert transformed >= 8  # the fixture exercises the bias on many rows


def test_lookback_state_nan_rows_and_edge_values():
    # a row with NaN stores NaN and is left alone; p = 1 gives a NaN lb_start score (reference: 0/0)
    from mapperatorinator_b200.logit_processors import lookback_spec

    m = G.case("lookback_renorm")["meta"]
    spec = lookback_spec(m["lookback_time"], G.lookback_tokenizer(m), True)
    rng = np.random.default_rng(5)
    x = rng.normal(size=(3, 256)).astype(np.float32)
    x[1, 7] = np.nan
    ids = np.full((3, 2), 140, dtype=np.int64)
    s = G.StepInputs(logits=x, dtype="f32", num_rows=3, input_ids=ids, select_mode=N.SELECT_NONE, want_scores=True,
                     lookback_mode=N.LOOKBACK_RENORM, lb_start=spec["start"], lb_end=spec["end"],
                     lb_eos_ids=spec["eos_ids"], lb_timed_bits=G.bits_for(spec["timed"], 256),
                     lb_state=np.array([0.25, 0.25, 1.0], dtype=np.float32))
    r = oracle.run(s)
    assert np.isnan(r["lb_state"][1]) and np.isfinite(r["lb_state"][[0, 2]]).all()
    out = r["out_scores"]
    assert np.array_equal(out[1], x[1], equal_nan=True)
    assert np.isfinite(out[0, spec["start"]]) and np.isneginf(out[0, spec["start"] + 1: spec["end"]]).all()
    assert np.isnan(out[2, spec["start"]])


def test_log_d_accuracy():
    import math

    rng = np.random.default_rng(0)
    xs = np.concatenate([rng.uniform(0, 4, 2000), np.exp(rng.uniform(-700, 700, 2000)), [1.0, 0.5, 2.0, 5e-324]])
    for x in xs:
        got, want = oracle.log_d(float(x)), math.log(float(x))
        assert abs(got - want) <= 4e-16 * max(abs(want), 1e-300) + (0.0 if want else 0.0), x
    assert oracle.log_d(0.0) == -math.inf and math.isnan(oracle.log_d(-1.0))


@pytest.mark.parametrize("name", ["lookback_renorm", "lookback_chain"])
def test_lookback_extra_mass_against_float64(name):
    # the EOS mass moved to lb_start, evaluated in float64 from the unbiased
    # scores (bit-exact to the reference chain): within 2e-8 of it
    c = G.case(name)
    B = c["input_ids"].shape[0]
    state, prev = np.full(B, np.nan, dtype=np.float32), None
    checked = 0
    for t in range(c["meta"]["steps"]):
        s = G.lookback_step(name, t, state)
        pre = oracle.run(s.with_(lookback_mode=N.LOOKBACK_OFF))["out_scores"].astype(np.float64)
        r = oracle.run(s)
        P = np.exp(pre - pre.max(axis=1, keepdims=True))
        P /= P.sum(axis=1, keepdims=True)
        if prev is not None:
            p = prev[:, [2, 4, 5]].sum(axis=1)
            O = P[:, np.r_[0:16, 66:256]].sum(axis=1)
            sv = 1.0 / (O * (1.0 - p) + p)
            extra = np.clip((sv - 1.0) * p / (1.0 - p), 0.0, 1.0)
            on = np.isneginf(r["out_scores"][:, 17:66]).all(axis=1)
            got = np.exp(r["out_scores"][on, 16].astype(np.float64))
            assert np.abs(got - extra[on]).max(initial=0.0) <= 2e-8, t
            checked += int(on.sum())
        prev, state = P, r["lb_state"]
    assert checked >= 8

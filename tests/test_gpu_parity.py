"""Kernel vs CPU oracle through the C ABI (bit-exact ids, keep sets, states;
log-probs within 1e-5 relative + 1e-6 absolute)."""

import numpy as np
import pytest

from mapperatorinator_b200 import _native as N
from tests.harness import workloads as W
from tests.harness.stepargs import DeviceStep, fill_args, host_arrays
from oracle import oracle
from tests import _golden as G

pytestmark = pytest.mark.gpu

_KERNEL_FLAGS = {"cta": N.FLAG_KERNEL_ROW_CTA, "warp": N.FLAG_KERNEL_ROW_WARP, "stream": N.FLAG_KERNEL_STREAM}
_ALL_KERNEL_FLAGS = N.FLAG_KERNEL_ROW_CTA | N.FLAG_KERNEL_ROW_WARP | N.FLAG_KERNEL_STREAM
_kernel = {"name": "cta"}


@pytest.fixture(autouse=True, params=["cta", "warp", "stream"])
def kernel(request):
    """Every parity case runs on every kernel that serves it (the row-per-warp
    kernel takes vocabularies up to 4096; the streaming kernel a top-k in
    [1, 64] with sampling or processor output)."""
    _kernel["name"] = request.param
    yield request.param
    _kernel["name"] = "cta"


def forced(s):
    """`s` with the current kernel forced; skips requests the kernel does not serve."""
    if _kernel["name"] == "warp" and s.vocab > 4096:
        pytest.skip("row-per-warp kernel: vocab <= 4096")
    s = s.with_(flags=(s.flags & ~_ALL_KERNEL_FLAGS) | _KERNEL_FLAGS[_kernel["name"]])
    if _kernel["name"] != "cta":
        arrays = host_arrays(s)
        args = fill_args(N.new_args(), s, lambda k: arrays[k].ctypes.data if k in arrays else 0)
        if N.validate(args) == N.ERR_UNSUPPORTED:
            pytest.skip(f"{_kernel['name']} kernel does not serve this request")
    return s


def run_both(s, device):
    import torch

    s = forced(s)
    ref = oracle.run(s)
    dev = DeviceStep(s, device)
    dev.launch()
    torch.cuda.synchronize(device)
    return ref, dev.results()


def assert_parity(s, device):
    ref, got = run_both(s, device)
    errs = oracle.compare(ref, got)
    assert not errs, "\n".join(errs)
    return ref, got


# ---------------------------------------------------------------- workloads
@pytest.mark.parametrize("want", [(False, False), (True, True)])
def test_cfg_pair_fp32(cuda_device, want):
    for seed in range(8):
        s = W.cfg_pair_fp32(seed).with_(want_scores=want[0], want_logprobs=want[1])
        assert_parity(s, cuda_device)


@pytest.mark.parametrize("dtype", ["bf16", "f32"])
def test_batched_decode(cuda_device, dtype):
    s = W.batched_decode(seed=11, pairs=64, dtype=dtype).with_(want_scores=True, want_logprobs=True)
    assert_parity(s, cuda_device)


def test_penalty_sweep(cuda_device):
    s = W.penalty_sweep(seed=12, rows=1024).with_(want_scores=True, want_logprobs=True)
    assert_parity(s, cuda_device)


def test_sharded_decode_full_size(cuda_device):
    s = W.sharded_decode(seed=13, pairs=4096)
    ref, got = assert_parity(s, cuda_device)
    assert (got["out_status"] & (N.ROW_NONFINITE | N.ROW_ALL_MASKED) == 0).all()


@pytest.mark.parametrize("vocab", [8192, 16384, 32768, 65536, 131072])
def test_vocab_sweep_clusters(cuda_device, vocab):
    rows = 256 if vocab <= 65536 else 64
    s = W.penalty_sweep(seed=vocab, rows=rows, vocab=vocab, history=256).with_(want_scores=True)
    assert_parity(s, cuda_device)
    s2 = W.batched_decode(seed=vocab + 1, pairs=rows // 2, vocab=vocab).with_(want_scores=True, want_logprobs=True)
    assert_parity(s2, cuda_device)


# ---------------------------------------------------------------- modes
@pytest.mark.parametrize("mode", [N.SELECT_NONE, N.SELECT_ARGMAX, N.SELECT_SAMPLE])
@pytest.mark.parametrize("topp_mode", [N.TOPP_HF, N.TOPP_SAMPLE_FN])
def test_select_modes(cuda_device, mode, topp_mode):
    s = W.batched_decode(seed=21, pairs=96).with_(select_mode=mode, top_p_mode=topp_mode, top_k=40,
                                                   want_scores=True, want_logprobs=True)
    assert_parity(s, cuda_device)


@pytest.mark.parametrize("top_k,top_p", [(1, 1.0), (5, 1.0), (0, 0.5), (0, 1e-4), (0, 0.999999), (4095, 0.9),
                                         (4096, 0.9), (10000, 0.9), (300, 0.97), (0, 1.0)])
def test_topk_topp_grid(cuda_device, top_k, top_p):
    s = W.penalty_sweep(seed=31, rows=128).with_(top_k=top_k, top_p=top_p, want_scores=True, want_logprobs=True)
    assert_parity(s, cuda_device)


def test_force_radix_paths(cuda_device):
    for s in (W.penalty_sweep(seed=41, rows=128), W.batched_decode(seed=42, pairs=64),
              W.penalty_sweep(seed=43, rows=64, vocab=16384, history=128)):
        s = s.with_(flags=s.flags | N.FLAG_FORCE_RADIX, want_scores=True, want_logprobs=True)
        ref, got = assert_parity(s, cuda_device)
        assert (got["out_status"] & N.ROW_SLOW_PATH).any()


def test_wide_nucleus_dense_path(cuda_device):
    # fp32, low temperature spread: thousands of survivors -> dense top-p and draw
    rng = np.random.default_rng(5)
    x = rng.normal(0, 0.3, size=(200, 4096)).astype(np.float32)
    s = W.StepInputs(logits=x, dtype="f32", num_rows=200, select_mode=N.SELECT_SAMPLE, top_p=0.99,
                     uniforms=rng.random(200, dtype=np.float32), want_scores=True, want_logprobs=True)
    assert_parity(s, cuda_device)
    assert_parity(s.with_(top_p=1.0), cuda_device)


# ---------------------------------------------------------------- edge cases
@pytest.mark.parametrize("vocab", [1, 2, 7, 33, 1000, 4099, 5000])
@pytest.mark.parametrize("dtype", ["f32", "bf16", "f16"])
def test_ragged_vocab_and_dtypes(cuda_device, vocab, dtype):
    rng = np.random.default_rng(vocab)
    rows = 9
    x = rng.normal(0, 2, size=(2 * rows, vocab)).astype(np.float32)
    logits = {"f32": x, "bf16": W.bf16_bits(x), "f16": x.astype(np.float16)}[dtype]
    ids = rng.integers(0, vocab, size=(rows, 17)).astype(np.int64)
    s = W.StepInputs(logits=logits, dtype=dtype, num_rows=rows, cfg_scale=1.3, input_ids=ids,
                     repetition_penalty=1.2, frequency_penalty=0.1, presence_penalty=0.05,
                     mono_mode=N.MONO_SCAN, ts_start=0, ts_end=max(1, vocab // 2), sos_ids=(vocab - 1,),
                     temperature=0.8, select_mode=N.SELECT_SAMPLE, top_k=min(5, vocab), top_p=0.9,
                     uniforms=rng.random(rows, dtype=np.float32), want_scores=True, want_logprobs=True)
    assert_parity(s, cuda_device)


def test_masked_nan_inf_rows(cuda_device):
    rng = np.random.default_rng(7)
    x = rng.normal(0, 1, size=(6, 256)).astype(np.float32)
    x[0, :] = -np.inf            # all masked
    x[1, 17] = np.nan            # NaN
    x[2, 3] = np.inf             # +inf
    x[3, :] = -np.inf
    x[3, 200] = 0.5              # single survivor
    x[4, 10:20] = np.nan
    for mode in (N.SELECT_SAMPLE, N.SELECT_ARGMAX, N.SELECT_NONE):
        s = W.StepInputs(logits=x, dtype="f32", num_rows=6, select_mode=mode, top_p=0.9, pad_id=3,
                         uniforms=rng.random(6, dtype=np.float32), want_scores=True, want_logprobs=True)
        ref, got = assert_parity(s, cuda_device)
        if mode == N.SELECT_ARGMAX:
            assert got["out_ids"][0] == 0 and got["out_ids"][1] == 17 and got["out_ids"][2] == 3
        assert got["out_status"][0] & N.ROW_ALL_MASKED
        assert got["out_status"][1] & N.ROW_NONFINITE


def test_ties_everywhere(cuda_device):
    rng = np.random.default_rng(8)
    x = rng.integers(-3, 4, size=(64, 4096)).astype(np.float32)
    for tk, tp, mode in [(0, 0.5, N.TOPP_HF), (7, 1.0, N.TOPP_HF), (50, 0.3, N.TOPP_SAMPLE_FN), (0, 0.01, N.TOPP_HF)]:
        s = W.StepInputs(logits=x, dtype="f32", num_rows=64, select_mode=N.SELECT_SAMPLE, top_k=tk, top_p=tp,
                         top_p_mode=mode, uniforms=rng.random(64, dtype=np.float32), want_scores=True)
        assert_parity(s, cuda_device)
        assert_parity(s.with_(flags=N.FLAG_FORCE_RADIX), cuda_device)


def test_uniform_extremes_and_bad_ids(cuda_device):
    s = W.penalty_sweep(seed=51, rows=8)
    ids = s.input_ids.copy()
    ids[0, 5] = 4096
    ids[1, 0] = -3
    u = np.array([0.0, np.nextafter(np.float32(1), np.float32(0)), -0.5, 1.0, np.nan, 0.5, 0.25, 1e-30],
                 dtype=np.float32)
    ref, got = assert_parity(s.with_(input_ids=ids, uniforms=u), cuda_device)
    assert got["out_status"][0] & N.ROW_BAD_ID and got["out_status"][1] & N.ROW_BAD_ID
    assert got["out_status"][2] & N.ROW_BAD_UNIFORM and got["out_status"][4] & N.ROW_BAD_UNIFORM


def test_empty_history_and_conditional_temperature(cuda_device):
    rng = np.random.default_rng(9)
    x = rng.normal(0, 2, size=(4, 512)).astype(np.float32)
    conds = [(0.5, 1, G.bits_for([100, 101], 512)), (2.0, 3, G.bits_for([7], 512))]
    for L in (0, 1, 2, 3, 9):
        ids = rng.integers(0, 512, size=(4, L)).astype(np.int64)
        if L >= 3:
            ids[0, -1] = 100
            ids[1, -3] = 7
        s = W.StepInputs(logits=x, dtype="f32", num_rows=4, input_ids=ids, temp_mode=N.TEMP_ROW_CONDITIONAL,
                         temperature=1.1, cond=conds, mono_mode=N.MONO_SCAN, ts_start=0, ts_end=256, sos_ids=(1,),
                         flags=N.FLAG_GRAMMAR_PREV_FROM_IDS, grammar_class_of=(np.arange(512) % 4).astype(np.uint8),
                         grammar_allow=np.array([0b0011, 0b0110, 0b1100, 0b1001], dtype=np.uint32),
                         repetition_penalty=1.3, select_mode=N.SELECT_SAMPLE, top_p=0.8,
                         uniforms=rng.random(4, dtype=np.float32), want_scores=True, want_logprobs=True)
        assert_parity(s, cuda_device)


def test_finished_rows_and_eos(cuda_device):
    s = W.batched_decode(seed=61, pairs=32)
    unf = np.ones(32, dtype=np.uint8)
    unf[::3] = 0
    s = s.with_(unfinished=unf, pad_id=7, eos_ids=(5, 9), eos_ranges=((0, 1000),),
                flags=N.FLAG_MONO_UPDATE_FROM_SAMPLE | N.FLAG_GRAMMAR_UPDATE_FROM_SAMPLE)
    ref, got = assert_parity(s, cuda_device)
    assert (got["out_ids"][::3] == 7).all()


# ---------------------------------------------------------------- multi-step state
def test_state_carried_over_steps(cuda_device):
    import torch

    base = forced(W.batched_decode(seed=71, pairs=48).with_(
        flags=N.FLAG_MONO_UPDATE_FROM_SAMPLE | N.FLAG_GRAMMAR_UPDATE_FROM_SAMPLE, sos_ids=(4094, 3000)))
    rng = np.random.default_rng(72)
    host = base
    dev = None
    for step in range(12):
        x = rng.normal(0, 1.5, size=(96, 4096)).astype(np.float32)
        u = rng.random(48, dtype=np.float32)
        host = host.with_(logits=W.bf16_bits(x), uniforms=u)
        ref = oracle.run(host)
        dev = DeviceStep(host, cuda_device)
        dev.launch()
        torch.cuda.synchronize()
        got = dev.results()
        assert not oracle.compare(ref, got), step
        host = host.with_(mono_state=ref["mono_state"], prev_token=ref["prev_token"])


def test_scan_equals_incremental_state(cuda_device):
    import torch

    rng = np.random.default_rng(81)
    B, V = 16, 256
    ids = rng.integers(0, 40, size=(B, 30)).astype(np.int64)
    x = rng.normal(0, 1, size=(B, V)).astype(np.float32)
    state = None
    for L in range(1, 31):
        scan = W.StepInputs(logits=x, dtype="f32", num_rows=B, input_ids=np.ascontiguousarray(ids[:, :L]),
                            mono_mode=N.MONO_SCAN, ts_start=10, ts_end=30, sos_ids=(1, 2),
                            select_mode=N.SELECT_NONE, want_scores=True)
        ref = oracle.run(scan)
        if state is None:
            inc = scan.with_(mono_state=np.full(B, -1, np.int32))
        else:
            inc = scan.with_(mono_mode=N.MONO_STATE, flags=N.FLAG_MONO_UPDATE_FROM_IDS, mono_state=state)
        dev = DeviceStep(forced(inc), cuda_device)
        dev.launch()
        torch.cuda.synchronize()
        got = dev.results()
        assert np.array_equal(got["out_scores"].view(np.uint32), ref["out_scores"].view(np.uint32)), L
        state = got["mono_state"]


# ---------------------------------------------------------------- reference fixtures on the GPU
@pytest.mark.parametrize("name", G.CHAIN_CASES)
def test_reference_fixture_processed_scores(cuda_device, name):
    import torch

    c = G.case(name)
    dev = DeviceStep(forced(G.chain_step(name)), cuda_device)
    dev.launch()
    torch.cuda.synchronize()
    got = dev.results()["out_scores"]
    assert np.array_equal(got.view(np.uint32), c["processed"].view(np.uint32))
    m = c["meta"]
    s = G.chain_step(name, top_k=m["top_k"], top_p=m["top_p"])
    assert_parity(s, cuda_device)


# ---------------------------------------------------------------- graph capture
def test_cuda_graph_capture_replay(cuda_device):
    import torch

    s = forced(W.penalty_sweep(seed=91, rows=256))
    dev = DeviceStep(s, cuda_device)
    stream = torch.cuda.Stream(cuda_device)
    dev.launch(stream)  # warm (sets kernel attributes outside capture)
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=stream):
        dev.launch(torch.cuda.current_stream())
    dev.tensors["out_ids"].fill_(-1)
    g.replay()
    torch.cuda.synchronize()
    ref = oracle.run(s)
    assert np.array_equal(dev.results()["out_ids"], ref["out_ids"])


@pytest.mark.parametrize("dtype", ["bf16", "f32"])
def test_grammar_class_byte_path(cuda_device, dtype):
    # the kernel masks from class bytes when no per-class vocabulary bitmap is given
    s = W.batched_decode(seed=101, pairs=48, dtype=dtype).with_(grammar_bits=False, want_scores=True)
    assert_parity(s, cuda_device)
    s = W.sharded_decode(seed=102, pairs=64, dtype=dtype).with_(grammar_bits=False, want_scores=True)
    assert_parity(s, cuda_device)


def test_column_temperature_ranges_split_chunks(cuda_device):
    # range edges inside 8-id chunks and overlapping ranges (first match wins)
    rng = np.random.default_rng(111)
    x = rng.normal(0, 2, size=(64, 4096)).astype(np.float32)
    s = W.StepInputs(logits=W.bf16_bits(x), dtype="bf16", num_rows=64, temp_mode=N.TEMP_COLUMN_RANGES,
                     temperature=1.3, col_ranges=[(3, 2003, 0.9), (1000, 1005, 0.5), (4090, 4096, 2.0)],
                     select_mode=N.SELECT_SAMPLE, top_p=0.9, uniforms=rng.random(64, dtype=np.float32),
                     want_scores=True, want_logprobs=True)
    assert_parity(s, cuda_device)


# ---------------------------------------------------------------- penalty paths of the row-per-warp kernel
@pytest.mark.parametrize("ids_dtype", [np.int64, np.int32])
def test_long_history_penalty_window(cuda_device, ids_dtype):
    # histories longer than the 512 ids a warp keeps in registers, penalty windows
    # that start inside the history, repeated ids, int32 and int64 ids
    rng = np.random.default_rng(121)
    rows, V = 320, 4096
    x = W.bf16_bits(rng.normal(0, 2, size=(rows, V)).astype(np.float32))
    for L, start in ((1500, 0), (1500, 700), (700, 650), (513, 0)):
        ids = rng.integers(0, V, size=(rows, L)).astype(ids_dtype)
        ids[:, -40:] = rng.integers(0, 64, size=(rows, 40))
        s = W.StepInputs(logits=x, dtype="bf16", num_rows=rows, input_ids=ids, penalty_start=start,
                         repetition_penalty=1.2, frequency_penalty=0.3, presence_penalty=0.05,
                         select_mode=N.SELECT_SAMPLE, top_k=40, top_p=0.9,
                         uniforms=rng.random(rows, dtype=np.float32), want_scores=True)
        assert_parity(s, cuda_device)


@pytest.mark.parametrize("rp", [1.2, 0.5, 2.0 ** 31, 2.0 ** -31])
def test_penalty_rare_operands(cuda_device, rp):
    # signed zeros and huge scores at penalised ids (the divide leaves the fast
    # path) and repetition penalties on both sides of the fast divide's range
    rng = np.random.default_rng(131)
    rows, V = 320, 4096
    xf = rng.normal(0, 2, size=(rows, V)).astype(np.float32)
    ids = rng.integers(0, V, size=(rows, 256)).astype(np.int64)
    r = np.arange(rows)[:, None]
    xf[r, ids[:, :6]] = 0.0
    xf[r, ids[:, 6:9]] = -0.0
    xf[r, ids[:, 9:11]] = 3.0e30
    s = W.StepInputs(logits=W.bf16_bits(xf), dtype="bf16", num_rows=rows, input_ids=ids, repetition_penalty=rp,
                     frequency_penalty=0.1, presence_penalty=0.2, select_mode=N.SELECT_SAMPLE, top_k=50, top_p=0.95,
                     uniforms=rng.random(rows, dtype=np.float32), want_scores=True, want_logprobs=True)
    assert_parity(s, cuda_device)


@pytest.mark.parametrize("temp", ["scalar", "conditional", "columns"])
def test_penalties_then_temperature(cuda_device, temp):
    # penalties come before temperature: a temperature pass follows the penalty update
    rng = np.random.default_rng(141)
    rows, V = 320, 4096
    x = W.bf16_bits(rng.normal(0, 2, size=(2 * rows, V)).astype(np.float32))
    ids = rng.integers(0, V, size=(rows, 300)).astype(np.int64)
    kw = dict(temperature=0.7)
    if temp == "conditional":
        ids[: rows // 2, -1] = 5
        kw = dict(temp_mode=N.TEMP_ROW_CONDITIONAL, temperature=1.0, cond=[(0.6, 1, G.bits_for([5, 6], V))])
    elif temp == "columns":
        kw = dict(temp_mode=N.TEMP_COLUMN_RANGES, temperature=1.0, col_ranges=[(0, 2003, 0.9), (2003, 3001, 1.7)])
    s = W.StepInputs(logits=x, dtype="bf16", num_rows=rows, cfg_scale=1.5, input_ids=ids, repetition_penalty=1.1,
                     frequency_penalty=0.2, presence_penalty=0.1, select_mode=N.SELECT_SAMPLE, top_k=50, top_p=0.95,
                     uniforms=rng.random(rows, dtype=np.float32), want_scores=True, **kw)
    assert_parity(s, cuda_device)


@pytest.mark.parametrize("ids_dtype", [np.int64, np.int32])
def test_repeated_ids_count_wrap(cuda_device, ids_dtype):
    # one id repeated 255, 256, 300 and 511 times inside a 512-id window, next to
    # its neighbour ids: the row-per-warp kernel's 8-bit counts wrap from the
    # 256th repeat on and the row is counted again exactly
    rng = np.random.default_rng(151)
    rows, V, L = 320, 4096, 512
    x = W.bf16_bits(rng.normal(0, 2, size=(rows, V)).astype(np.float32))
    for start in (0, 100):
        ids = rng.integers(0, V, size=(rows, L)).astype(ids_dtype)
        for r in range(rows):
            reps = (255, 256, 300, 511)[r % 4]
            h = int(rng.integers(1, V - 1))
            pos = rng.permutation(L)
            ids[r, pos[:reps]] = h
            if reps < L:
                ids[r, pos[reps:reps + 1]] = h + 1
            if reps + 1 < L:
                ids[r, pos[reps + 1:reps + 2]] = h - 1
        s = W.StepInputs(logits=x, dtype="bf16", num_rows=rows, input_ids=ids, penalty_start=start,
                         repetition_penalty=1.2, frequency_penalty=0.01, presence_penalty=0.05,
                         select_mode=N.SELECT_SAMPLE, top_k=40, top_p=0.9,
                         uniforms=rng.random(rows, dtype=np.float32), want_scores=True)
        assert_parity(s, cuda_device)


# ---------------------------------------------------------------- bounded waits
def test_row_warp_copy_timeout_marks_every_remaining_row(cuda_device):
    """The row-per-warp kernel's bounded wait for a staged row: with the test hook
    the first wait of every CTA gives up at once; that row and every later row of
    the CTA get pad_id and MTR_ROW_COPY_TIMEOUT (no row keeps an earlier token),
    the CTA drains its copy, and the next launch is unaffected."""
    import torch

    if _kernel["name"] != "warp":
        pytest.skip("row-per-warp kernel only")
    s = W.penalty_sweep(seed=161, rows=4096).with_(pad_id=11)
    dev = DeviceStep(s.with_(flags=N.FLAG_KERNEL_ROW_WARP | N.FLAG_TEST_COPY_TIMEOUT), cuda_device)
    dev.launch()
    torch.cuda.synchronize(cuda_device)
    got = dev.results()
    assert (got["out_status"] & N.ROW_COPY_TIMEOUT).all()
    assert (got["out_ids"] == 11).all()
    assert_parity(s, cuda_device)  # the same rows again, without the hook


# ---------------------------------------------------------------- lookback bias
@pytest.mark.parametrize("name", G.LOOKBACK_CASES)
def test_lookback_fixture_steps(cuda_device, name):
    # the reference fixtures' consecutive calls: kernel == oracle bit for bit
    # (scores and lb_state), the kernel's state carried to the next call
    c = G.case(name)
    B = c["input_ids"].shape[0]
    state = np.full(B, np.nan, dtype=np.float32)
    for t in range(c["meta"]["steps"]):
        ref, got = assert_parity(G.lookback_step(name, t, state), cuda_device)
        assert G.lookback_close(got["out_scores"], G.lookback_reference(name, t), 16) == [], t
        if "lb_state" in got:
            state = got["lb_state"]


@pytest.mark.parametrize("vocab,pairs,dtype", [(4096, 64, "bf16"), (4096, 512, "f32"), (32768, 4, "bf16"),
                                               (131072, 2, "f16")])
def test_lookback_sampling_steps(cuda_device, vocab, pairs, dtype):
    # CFG + monotonic + temperature + lookback + top-k + top-p + draw over four
    # steps; clusters for the large vocabularies
    state = None
    for step in range(4):
        s = W.lookback_decode(seed=vocab + pairs, pairs=pairs, vocab=vocab, dtype=dtype, step=step, lb_state=state)
        s = s.with_(want_scores=step % 2 == 0, want_logprobs=step % 2 == 1)
        ref, got = assert_parity(s, cuda_device)
        state = got["lb_state"]
        assert np.isfinite(state).mean() > 0.9


def test_lookback_edges(cuda_device):
    # empty range (lb_start == lb_end), p = 1 (NaN at lb_start), p = 0, a NaN row,
    # an all -inf row, an empty history, and the mask form
    s = W.lookback_decode(seed=3, pairs=8, vocab=1000, dtype="f32")
    x = s.logits.copy()
    x[4] = np.nan
    x[12] = -np.inf
    x[5] = -np.inf
    state = np.array([1.0, 0.0, 0.5, np.nan, 0.3, 0.3, 0.99999994, 1e-30], dtype=np.float32)
    s = s.with_(logits=x, lb_state=state, want_scores=True, want_logprobs=True)
    assert_parity(s, cuda_device)
    assert_parity(s.with_(lb_end=s.lb_start), cuda_device)
    assert_parity(s.with_(input_ids=s.input_ids[:, :0]), cuda_device)
    assert_parity(s.with_(lookback_mode=N.LOOKBACK_MASK), cuda_device)
    assert_parity(s.with_(lookback_mode=N.LOOKBACK_MASK, lb_end=1000, lb_start=990), cuda_device)


# ---------------------------------------------------------------- token append and stop counters
@pytest.mark.parametrize("workload", ["batched", "penalty"])
def test_append_and_stop_counts(cuda_device, workload):
    # pad-on-finished, EOS (ids and a range), id-buffer column from a host value
    # and from a device value, cumulative stop counters -- on every kernel
    if workload == "batched":
        s = W.batched_decode(seed=63, pairs=48)
        B = 48
    else:
        s = W.penalty_sweep(seed=64, rows=1024).with_(top_p=0.9)
        B = 1024
    rng = np.random.default_rng(65)
    unf = (rng.random(B) < 0.8).astype(np.uint8)
    buf = np.full((B, 40), -1, dtype=np.int64)
    counts = np.array([3, 5], dtype=np.uint32)  # cumulative: earlier steps' counts stay
    s = s.with_(unfinished=unf, pad_id=7, eos_ids=(5, 9), eos_ranges=((0, 2048),), id_buffer=buf, cur_len=17,
                stop_counts=counts)
    ref, got = assert_parity(s, cuda_device)
    assert (got["id_buffer"][:, 17] == got["out_ids"]).all()
    assert ref["stop_counts"][1] > 5  # some rows finished in this step
    ref, got = assert_parity(s.with_(cur_len_dev=np.array([39], dtype=np.int32)), cuda_device)
    assert (got["id_buffer"][:, 39] == got["out_ids"]).all() and (got["id_buffer"][:, 17] == -1).all()
    ref, got = assert_parity(s.with_(cur_len_dev=np.array([40], dtype=np.int32)), cuda_device)
    assert (got["out_status"] & N.ROW_APPEND_SKIPPED).all() and (got["id_buffer"] == -1).all()


@pytest.mark.parametrize("mode", [N.SELECT_SAMPLE, N.SELECT_NONE])
def test_dense_mass_path_branches(cuda_device, mode):
    # rows without a top-k list: Gaussian rows (the crossing bin lists < 64 candidates),
    # a narrow score band (hundreds per 1/16-logit bin: the 256-sub-bin split) and
    # exact ties (no split separates them: the radix path) -- on every kernel
    rng = np.random.default_rng(71)
    V, B = 4096, 96
    x = rng.normal(0.0, 2.2, size=(B, V)).astype(np.float32)
    x[1::3] = rng.uniform(0.0, 0.5, size=(len(x[1::3]), V)).astype(np.float32)
    x[2::3] = 0.0
    x[2::3, :10] = 1.0
    s = W.StepInputs(logits=W.bf16_bits(x), dtype="bf16", num_rows=B, temperature=0.9, top_p=0.9, select_mode=mode,
                     uniforms=rng.random(B, dtype=np.float32), want_scores=True, want_logprobs=True)
    ref, got = assert_parity(s, cuda_device)
    if _kernel["name"] == "warp":
        slow = (got["out_status"] & N.ROW_SLOW_PATH) != 0
        assert not slow[0::3].any() and not slow[1::3].any() and slow[2::3].all()


@pytest.mark.parametrize("top_k,top_p,mode,scores", [(50, 0.9, N.TOPP_HF, False), (100, 0.95, N.TOPP_SAMPLE_FN, True),
                                                     (100, 1.0, N.TOPP_HF, False), (64, 0.5, N.TOPP_HF, True)])
def test_quantized_scores_long_candidate_lists(cuda_device, top_k, top_p, mode, scores):
    # scores on a 1/4-logit grid: the tie group at the k-th score makes the
    # candidate list 65 .. 128 long in most rows (the row-per-warp kernel's
    # 128-key sort) and longer in some (its fine-bin list path)
    rng = np.random.default_rng(81 + top_k)
    B, V, L = 256, 4096, 256
    x = (np.round(rng.normal(0.0, 2.0, size=(B, V)) * 4.0) / 4.0).astype(np.float32)
    s = W.StepInputs(logits=W.bf16_bits(x), dtype="bf16", num_rows=B, select_mode=N.SELECT_SAMPLE, top_k=top_k,
                     top_p=top_p, top_p_mode=mode, uniforms=rng.random(B, dtype=np.float32), want_scores=scores,
                     input_ids=rng.integers(0, V, size=(B, L)).astype(np.int64), repetition_penalty=1.25,
                     presence_penalty=0.25)
    assert_parity(s, cuda_device)

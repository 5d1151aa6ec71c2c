"""The C-ABI library loads on a CPU-only host, exports every symbol the header
declares and rejects invalid arguments before any CUDA call."""

import ctypes
import re
from pathlib import Path

import numpy as np
import pytest

from mapperatorinator_b200 import _native as N
from mapperatorinator_b200 import build as B

HEADER = Path(__file__).resolve().parents[1] / "include" / "mtr_sampler.h"


def header_functions():
    text = HEADER.read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"^\s*[A-Za-z_][\w\s\*]*?\b(mtr_\w+)\s*\(", text, flags=re.M)))


@pytest.fixture(scope="module")
def lib():
    B.build()
    return N.load()


def test_header_symbols_exported(lib):
    names = header_functions()
    assert names, "no declarations parsed"
    assert set(names) == set(N.EXPORTS), (names, sorted(N.EXPORTS))
    for n in names:
        assert hasattr(lib, n), n


def test_struct_layout(lib):
    assert lib.mtr_abi_version() == N.ABI_VERSION
    assert lib.mtr_args_size() == ctypes.sizeof(N.MtrSamplerArgs)


def test_args_init_defaults(lib):
    a = N.new_args()
    assert a.abi_version == N.ABI_VERSION and a.struct_size == ctypes.sizeof(a)
    assert a.temperature == 1.0 and a.top_p == 1.0 and a.repetition_penalty == 1.0
    assert a.select_mode == N.SELECT_NONE and a.mono_mode == N.MONO_OFF


def _valid_args():
    a = N.new_args()
    a.logits = 0x10000
    a.logits_row_stride = 4096
    a.logits_dtype = N.DTYPE_BF16
    a.num_rows = 4
    a.vocab = 4096
    a.select_mode = N.SELECT_SAMPLE
    a.uniforms = 0x20000
    a.out_ids = 0x30000
    return a


def test_validate_accepts_valid(lib):
    assert N.validate(_valid_args()) == N.OK


@pytest.mark.parametrize(
    "field,value,code",
    [
        ("vocab", 0, N.ERR_BAD_SHAPE),
        ("vocab", N.MAX_VOCAB + 1, N.ERR_BAD_SHAPE),
        ("num_rows", -1, N.ERR_BAD_SHAPE),
        ("logits", 0, N.ERR_NULL_ARG),
        ("logits", 0x10001, N.ERR_ALIGNMENT),
        ("logits_row_stride", 100, N.ERR_BAD_SHAPE),
        ("logits_dtype", 9, N.ERR_BAD_PARAM),
        ("top_p", 0.0, N.ERR_BAD_PARAM),
        ("top_p", 1.5, N.ERR_BAD_PARAM),
        ("top_k", -1, N.ERR_BAD_PARAM),
        ("temperature", 0.0, N.ERR_BAD_PARAM),
        ("temperature", float("nan"), N.ERR_BAD_PARAM),
        ("repetition_penalty", 0.0, N.ERR_BAD_PARAM),
        ("frequency_penalty", float("inf"), N.ERR_BAD_PARAM),
        ("uniforms", 0, N.ERR_NULL_ARG),
        ("out_ids", 0, N.ERR_NULL_ARG),
        ("select_mode", 7, N.ERR_BAD_PARAM),
        ("top_p_mode", 5, N.ERR_BAD_PARAM),
        ("mono_mode", N.MONO_STATE, N.ERR_NULL_ARG),
        ("ts_end", 5000, N.ERR_BAD_SHAPE),
        ("flags", 1 << 20, N.ERR_BAD_PARAM),
        ("abi_version", 99, N.ERR_ABI),
        ("ids_len", N.MAX_IDS_LEN + 1, N.ERR_BAD_SHAPE),
        ("n_sos", 17, N.ERR_BAD_PARAM),
        ("n_eos", 17, N.ERR_BAD_PARAM),
        ("cfg_scale", float("nan"), N.ERR_BAD_PARAM),
    ],
)
def test_validate_rejects(lib, field, value, code):
    a = _valid_args()
    if field == "cfg_scale":
        a.cfg_enabled = 1
    setattr(a, field, value)
    assert N.validate(a) == code
    # the launcher validates first, so no CUDA call is made for bad input
    assert lib.mtr_sampler_launch(ctypes.byref(a), None) == code


def test_penalties_need_history(lib):
    a = _valid_args()
    a.repetition_penalty = 1.1
    a.ids_len = 16
    assert N.validate(a) == N.ERR_NULL_ARG


def test_grammar_requirements(lib):
    a = _valid_args()
    a.grammar_class_of = 0x40000
    assert N.validate(a) == N.ERR_NULL_ARG
    a.grammar_allow = 0x50000
    a.grammar_n_classes = 40
    assert N.validate(a) == N.ERR_BAD_PARAM
    a.grammar_n_classes = 16
    assert N.validate(a) == N.ERR_NULL_ARG  # prev_token missing
    a.flags = N.FLAG_GRAMMAR_PREV_FROM_IDS
    assert N.validate(a) == N.OK


def test_zero_rows_is_a_noop(lib):
    a = _valid_args()
    a.num_rows = 0
    assert lib.mtr_sampler_launch(ctypes.byref(a), None) == N.OK


@pytest.mark.parametrize("vocab,rows,cs", [(1, 10, 1), (4096, 10, 1), (4096, 1000, 1), (4097, 10, 2), (8192, 10, 2),
                                           (16384, 10, 4), (65536, 10, 8), (131072, 10, 8)])
def test_query_geometry(lib, vocab, rows, cs):
    # few rows of a small vocabulary get one 512-thread CTA each (latency)
    info = N.query(vocab, rows, True)
    assert info.cluster_size == cs
    assert info.threads * info.elems_per_thread * info.cluster_size >= vocab
    assert info.grid == rows * cs
    assert info.candidate_cap == 256
    assert info.dyn_smem_bytes == info.threads * info.elems_per_thread * 10


@pytest.mark.parametrize("rows,vocab,top_k,select,flags,kernel", [
    (4096, 4096, 50, N.SELECT_SAMPLE, 0, N.KERNEL_ROW_WARP),      # many rows, short top-k list
    (64, 4096, 50, N.SELECT_SAMPLE, 0, N.KERNEL_ROW_CTA),         # few rows: latency geometry
    (444, 4096, 50, N.SELECT_SAMPLE, 0, N.KERNEL_ROW_CTA),        # one round of CTAs (3 per SM x 148)
    (445, 4096, 50, N.SELECT_SAMPLE, 0, N.KERNEL_ROW_WARP),       # past one round: row per warp
    (256, 65536, 50, N.SELECT_SAMPLE, 0, N.KERNEL_STREAM),        # large vocabulary: 16 warps per row
    (256, 16384, 50, N.SELECT_NONE, 0, N.KERNEL_STREAM),          # processor output with top-k
    (4096, 8192, 50, N.SELECT_SAMPLE, 0, N.KERNEL_STREAM),
    (4096, 4096, 0, N.SELECT_ARGMAX, 0, N.KERNEL_ROW_WARP),
    (4096, 4096, 100, N.SELECT_SAMPLE, 0, N.KERNEL_ROW_WARP),     # top-k past the stream kernel's 64
    (4096, 16384, 100, N.SELECT_SAMPLE, 0, N.KERNEL_ROW_CTA),     # large vocabulary, long top-k list
    (4096, 4096, 0, N.SELECT_SAMPLE, 0, N.KERNEL_ROW_CTA),        # top-p over the whole row
    (4096, 4096, 500, N.SELECT_SAMPLE, 0, N.KERNEL_ROW_CTA),      # long top-k list
    (4096, 131072, 50, N.SELECT_SAMPLE, 0, N.KERNEL_ROW_CTA),     # vocabulary above 65536
    (4096, 4096, 50, N.SELECT_SAMPLE, N.FLAG_KERNEL_ROW_CTA, N.KERNEL_ROW_CTA),
    (4096, 4096, 50, N.SELECT_SAMPLE, N.FLAG_KERNEL_ROW_WARP, N.KERNEL_ROW_WARP),
    (8, 4096, 0, N.SELECT_SAMPLE, N.FLAG_KERNEL_ROW_WARP, N.KERNEL_ROW_WARP),
    (8, 4096, 5, N.SELECT_SAMPLE, N.FLAG_KERNEL_STREAM, N.KERNEL_STREAM),
])
def test_query_args_kernel_choice(lib, rows, vocab, top_k, select, flags, kernel):
    a = _valid_args()
    a.num_rows, a.vocab, a.logits_row_stride = rows, vocab, vocab
    a.top_k, a.select_mode, a.flags = top_k, select, flags
    info = N.query_args(a)
    assert info.kernel == kernel
    if kernel == N.KERNEL_ROW_WARP:
        assert (info.threads, info.cluster_size) == (32, 1)
        assert min(rows, 148) <= info.grid <= rows  # persistent: at most one warp per row
        assert info.threads * info.elems_per_thread >= vocab
        assert info.dyn_smem_bytes <= 48 * 1024
        if vocab == 4096:  # ten one-warp CTAs per SM: 228 KB, per CTA 1 KB reserved + 16 B static, 128 B units
            assert (info.dyn_smem_bytes + 16 + 127) // 128 * 128 * 10 + 10 * 1024 <= 228 * 1024
    elif kernel == N.KERNEL_STREAM:
        # row groups of G warps (G * 32 threads * 16 chunks * 8 ids >= V), persistent grid
        assert info.threads in (128, 256, 512) and info.cluster_size == 1
        assert info.candidate_cap == 256
        groups_per_cta = max(1, 128 // info.threads)
        g_threads = info.threads // groups_per_cta
        assert g_threads * info.elems_per_thread >= vocab
        assert info.grid * groups_per_cta <= rows + groups_per_cta
        if vocab == 65536:
            # sixteen warps per row, two CTAs per SM within 228 KB
            assert info.threads == 512
            assert 2 * (info.dyn_smem_bytes + 1024) <= 228 * 1024
    else:
        assert info.grid == rows * info.cluster_size


def test_kernel_flags_validated(lib):
    a = _valid_args()
    a.flags = N.FLAG_KERNEL_ROW_CTA | N.FLAG_KERNEL_ROW_WARP
    assert N.validate(a) == N.ERR_BAD_PARAM
    a.flags = N.FLAG_KERNEL_ROW_WARP | N.FLAG_KERNEL_STREAM
    assert N.validate(a) == N.ERR_BAD_PARAM
    a.flags = N.FLAG_KERNEL_ROW_WARP
    a.vocab = a.logits_row_stride = 4097
    assert N.validate(a) == N.ERR_UNSUPPORTED
    a.vocab = a.logits_row_stride = 4096
    assert N.validate(a) == N.OK
    # the streaming kernel: top-k in [1, 64], sampling or processor output, V % 8 == 0
    a.flags = N.FLAG_KERNEL_STREAM
    a.top_k = 50
    assert N.validate(a) == N.OK
    for field, value in (("top_k", 0), ("top_k", 65), ("select_mode", N.SELECT_ARGMAX), ("vocab", 4100),
                         ("temp_mode", N.TEMP_COLUMN_RANGES)):
        b = _valid_args()
        b.flags, b.top_k = N.FLAG_KERNEL_STREAM, 50
        setattr(b, field, value)
        if field == "vocab":
            b.logits_row_stride = value
        assert N.validate(b) == N.ERR_UNSUPPORTED, field


def test_status_strings(lib):
    assert N.status_string(N.OK) == "MTR_OK"
    assert N.status_string(N.ERR_ABI) == "MTR_ERR_ABI"
    with pytest.raises(ValueError):
        N.check(N.ERR_BAD_PARAM)


def _lookback_args():
    a = _valid_args()
    a.lookback_mode = N.LOOKBACK_RENORM
    a.lb_start, a.lb_end = 100, 600
    a.n_lb_eos = 2
    a.lb_eos_ids[0], a.lb_eos_ids[1] = 2, 3
    a.lb_state = 0x60000
    a.lb_timed_bits = 0x70000
    a.input_ids, a.ids_len, a.ids_row_stride, a.ids_dtype = 0x80000, 4, 4, N.IDS_I64
    return a


def test_lookback_validation_and_kernel(lib):
    a = _lookback_args()
    assert N.validate(a) == N.OK
    # the lookback bias is served by the row-per-CTA kernel only
    a.num_rows, a.top_k = 4096, 50
    assert N.query_args(a).kernel == N.KERNEL_ROW_CTA
    a.vocab = a.logits_row_stride = 65536
    assert N.query_args(a).kernel == N.KERNEL_ROW_CTA
    for flag in (N.FLAG_KERNEL_ROW_WARP, N.FLAG_KERNEL_STREAM):
        b = _lookback_args()
        b.flags = flag
        b.top_k = 50
        assert N.validate(b) == N.ERR_UNSUPPORTED
    b = _lookback_args()
    b.lookback_mode = N.LOOKBACK_MASK
    b.flags = N.FLAG_KERNEL_ROW_WARP
    assert N.validate(b) == N.ERR_UNSUPPORTED
    cases = [("lookback_mode", 3, N.ERR_BAD_PARAM), ("lb_start", -1, N.ERR_BAD_SHAPE),
             ("lb_end", 50, N.ERR_BAD_SHAPE), ("lb_end", 5000, N.ERR_BAD_SHAPE), ("n_lb_eos", 9, N.ERR_BAD_PARAM),
             ("lb_state", 0, N.ERR_NULL_ARG), ("lb_state", 0x60002, N.ERR_ALIGNMENT),
             ("lb_timed_bits", 0, N.ERR_NULL_ARG), ("input_ids", 0, N.ERR_NULL_ARG)]
    for field, value, code in cases:
        b = _lookback_args()
        setattr(b, field, value)
        assert N.validate(b) == code, field
    b = _lookback_args()
    b.lb_eos_ids[1] = 4096
    assert N.validate(b) == N.ERR_BAD_PARAM
    b = _lookback_args()
    b.lb_start = b.lb_end = 4096  # the renormalising form writes lb_start: it must be an id
    assert N.validate(b) == N.ERR_BAD_SHAPE
    b.lookback_mode = N.LOOKBACK_MASK  # an empty mask range at the end is fine
    assert N.validate(b) == N.OK
    b = _lookback_args()
    b.ids_len = b.ids_row_stride = 0
    b.input_ids = 0
    b.lb_timed_bits = 0  # no history: no last token to look up
    assert N.validate(b) == N.OK


def test_append_and_stop_validation(lib):
    a = _valid_args()
    a.id_buffer, a.id_buffer_row_stride, a.cur_len = 0x90000, 64, 10
    a.stop_counts = 0xA0000
    assert N.validate(a) == N.OK
    for field, value, code in (("cur_len", 64, N.ERR_BAD_SHAPE), ("cur_len", -1, N.ERR_BAD_SHAPE),
                               ("id_buffer_row_stride", 0, N.ERR_BAD_SHAPE), ("id_buffer", 0x90004, N.ERR_ALIGNMENT),
                               ("stop_counts", 0xA0002, N.ERR_ALIGNMENT), ("cur_len_dev", 0xB0002, N.ERR_ALIGNMENT),
                               ("select_mode", N.SELECT_NONE, N.ERR_BAD_PARAM)):
        b = _valid_args()
        b.id_buffer, b.id_buffer_row_stride, b.cur_len = 0x90000, 64, 10
        b.stop_counts = 0xA0000
        setattr(b, field, value)
        assert N.validate(b) == code, (field, value)
    b = _valid_args()
    b.id_buffer, b.id_buffer_row_stride, b.cur_len, b.cur_len_dev = 0x90000, 64, 1000, 0xB0000
    assert N.validate(b) == N.OK  # a device column is checked by the kernel (MTR_ROW_APPEND_SKIPPED)


def _lm_args():
    a = N.new_lmhead_args()
    a.hidden, a.hidden_row_stride = 0x100000, 768
    a.weight, a.weight_row_stride = 0x200000, 768
    a.logits, a.logits_row_stride = 0x300000, 4096
    a.rows, a.d_model, a.vocab = 256, 768, 4096
    return a


def test_lmhead_validation(lib):
    assert N.lmhead_validate(_lm_args()) == N.OK  # also: the ctypes struct has the C size
    for field, value, code in (("d_model", 100, N.ERR_BAD_SHAPE), ("d_model", 0, N.ERR_BAD_SHAPE),
                               ("vocab", 4100, N.ERR_BAD_SHAPE), ("vocab", N.MAX_VOCAB + 8, N.ERR_BAD_SHAPE),
                               ("rows", -1, N.ERR_BAD_SHAPE), ("tile_n", 32, N.ERR_BAD_PARAM),
                               ("hidden", 0, N.ERR_NULL_ARG), ("weight", 0x200008, N.ERR_ALIGNMENT),
                               ("logits_row_stride", 4095, N.ERR_BAD_SHAPE),
                               ("hidden_row_stride", 772, N.ERR_ALIGNMENT), ("struct_size", 8, N.ERR_ABI)):
        b = _lm_args()
        setattr(b, field, value)
        assert N.lmhead_validate(b) == code, field
        # the launchers validate first: no CUDA call for bad input
        assert lib.mtr_lmhead_launch(ctypes.byref(b), None) == code, field
    b = _lm_args()
    b.rows = 0
    assert lib.mtr_lmhead_launch(ctypes.byref(b), None) == N.OK


def test_lmhead_sample_pairing_checked(lib):
    lm = _lm_args()
    a = _valid_args()
    a.logits, a.logits_row_stride, a.vocab, a.num_rows = lm.logits, 4096, 4096, 128
    a.cfg_enabled, a.cfg_scale = 1, 1.5
    # the sampler must read the projection's own buffer, as bf16, inside its rows
    for field, value in (("logits", 0x400000), ("logits_dtype", N.DTYPE_F32), ("num_rows", 129)):
        b = N.MtrSamplerArgs()
        ctypes.pointer(b)[0] = a
        setattr(b, field, value)
        if field == "logits_dtype":
            b.logits_row_stride = 4096
        rc = lib.mtr_lmhead_sample_launch(ctypes.byref(lm), ctypes.byref(b), None)
        assert rc in (N.ERR_BAD_PARAM, N.ERR_BAD_SHAPE), field

"""ctypes binding of ``include/mtr_sampler.h``.

The product path is this library and nothing else: if it cannot be loaded,
every operation raises :class:`NativeLibraryError` (there is no Python or CPU
fallback).  ``MtrSamplerArgs`` mirrors the C struct field for field; the
library reports ``sizeof(MtrSamplerArgs)`` so a layout drift is caught at load
time.
"""

from __future__ import annotations

import ctypes
import threading
from ctypes import c_float, c_int32, c_int64, c_uint32, c_void_p
from pathlib import Path

from . import build as _build

ABI_VERSION = 2
MAX_VOCAB = 131072
MAX_IDS_LEN = 65535
MAX_SOS_IDS = 16
MAX_COND_TEMPS = 4
MAX_COL_TEMP_RANGES = 8
MAX_GRAMMAR_CLASSES = 32
MAX_EOS_IDS = 16
MAX_EOS_RANGES = 2
MAX_LB_EOS = 8

# MtrStatus
OK = 0
ERR_NULL_ARG = 1
ERR_BAD_SHAPE = 2
ERR_BAD_PARAM = 3
ERR_UNSUPPORTED = 4
ERR_ALIGNMENT = 5
ERR_CUDA = 6
ERR_ABI = 7

# per-row status bits
ROW_NONFINITE = 1 << 0
ROW_ALL_MASKED = 1 << 1
ROW_BAD_ID = 1 << 2
ROW_BAD_UNIFORM = 1 << 3
ROW_SLOW_PATH = 1 << 4
ROW_TIE_AT_CUT = 1 << 5
ROW_COPY_TIMEOUT = 1 << 6
ROW_APPEND_SKIPPED = 1 << 7

DTYPE_F32, DTYPE_BF16, DTYPE_F16 = 0, 1, 2
IDS_I64, IDS_I32 = 0, 1
MONO_OFF, MONO_STATE, MONO_SCAN = 0, 1, 2
TEMP_SCALAR, TEMP_ROW_CONDITIONAL, TEMP_COLUMN_RANGES = 0, 1, 2
TOPP_HF, TOPP_SAMPLE_FN = 0, 1
SELECT_NONE, SELECT_ARGMAX, SELECT_SAMPLE = 0, 1, 2
LOOKBACK_OFF, LOOKBACK_MASK, LOOKBACK_RENORM = 0, 1, 2

FLAG_MONO_UPDATE_FROM_IDS = 1 << 0
FLAG_MONO_UPDATE_FROM_SAMPLE = 1 << 1
FLAG_GRAMMAR_PREV_FROM_IDS = 1 << 2
FLAG_GRAMMAR_UPDATE_FROM_SAMPLE = 1 << 3
FLAG_FORCE_RADIX = 1 << 4
FLAG_KERNEL_ROW_CTA = 1 << 5
FLAG_KERNEL_ROW_WARP = 1 << 6
FLAG_KERNEL_STREAM = 1 << 7
FLAG_TEST_COPY_TIMEOUT = 1 << 8


class MtrSamplerArgs(ctypes.Structure):
    _fields_ = [
        ("abi_version", c_uint32),
        ("struct_size", c_uint32),
        ("logits", c_void_p),
        ("logits_row_stride", c_int64),
        ("cfg_second_offset", c_int64),
        ("logits_dtype", c_int32),
        ("num_rows", c_int32),
        ("vocab", c_int32),
        ("cfg_enabled", c_int32),
        ("cfg_scale", c_float),
        ("flags", c_uint32),
        ("input_ids", c_void_p),
        ("ids_row_stride", c_int64),
        ("ids_dtype", c_int32),
        ("ids_len", c_int32),
        ("penalty_start", c_int32),
        ("mono_mode", c_int32),
        ("ts_start", c_int32),
        ("ts_end", c_int32),
        ("n_sos", c_int32),
        ("sos_ids", c_int32 * MAX_SOS_IDS),
        ("mono_state", c_void_p),
        ("timeshift_bias", c_float),
        ("grammar_class_of", c_void_p),
        ("grammar_allow", c_void_p),
        ("grammar_vocab_bits", c_void_p),
        ("grammar_n_classes", c_int32),
        ("prev_token", c_void_p),
        ("repetition_penalty", c_float),
        ("frequency_penalty", c_float),
        ("presence_penalty", c_float),
        ("temp_mode", c_int32),
        ("temperature", c_float),
        ("n_cond", c_int32),
        ("cond_temperature", c_float * MAX_COND_TEMPS),
        ("cond_offset", c_int32 * MAX_COND_TEMPS),
        ("cond_token_bits", c_void_p * MAX_COND_TEMPS),
        ("n_col_ranges", c_int32),
        ("col_start", c_int32 * MAX_COL_TEMP_RANGES),
        ("col_end", c_int32 * MAX_COL_TEMP_RANGES),
        ("col_temperature", c_float * MAX_COL_TEMP_RANGES),
        ("select_mode", c_int32),
        ("top_k", c_int32),
        ("top_p", c_float),
        ("top_p_mode", c_int32),
        ("uniforms", c_void_p),
        ("out_ids", c_void_p),
        ("out_scores", c_void_p),
        ("out_scores_row_stride", c_int64),
        ("out_logprobs", c_void_p),
        ("out_logprobs_row_stride", c_int64),
        ("out_status", c_void_p),
        ("unfinished", c_void_p),
        ("pad_id", c_int64),
        ("n_eos", c_int32),
        ("eos_ids", c_int32 * MAX_EOS_IDS),
        ("n_eos_ranges", c_int32),
        ("eos_range_start", c_int32 * MAX_EOS_RANGES),
        ("eos_range_end", c_int32 * MAX_EOS_RANGES),
        ("lookback_mode", c_int32),
        ("lb_start", c_int32),
        ("lb_end", c_int32),
        ("n_lb_eos", c_int32),
        ("lb_eos_ids", c_int32 * MAX_LB_EOS),
        ("lb_timed_bits", c_void_p),
        ("lb_state", c_void_p),
        ("id_buffer", c_void_p),
        ("id_buffer_row_stride", c_int64),
        ("cur_len_dev", c_void_p),
        ("cur_len", c_int32),
        ("reserved1", c_int32),
        ("stop_counts", c_void_p),
    ]


class MtrLaunchInfo(ctypes.Structure):
    _fields_ = [
        ("threads", c_int32),
        ("elems_per_thread", c_int32),
        ("cluster_size", c_int32),
        ("grid", c_int32),
        ("dyn_smem_bytes", c_int32),
        ("max_vocab", c_int32),
        ("max_ids_len", c_int32),
        ("candidate_cap", c_int32),
        ("kernel", c_int32),
    ]


KERNEL_ROW_CTA = 0
KERNEL_ROW_WARP = 1
KERNEL_STREAM = 2


class MtrLmHeadArgs(ctypes.Structure):
    """include/mtr_sampler.h MtrLmHeadArgs: the tensor-core output projection."""

    _fields_ = [
        ("abi_version", c_uint32),
        ("struct_size", c_uint32),
        ("hidden", c_void_p),
        ("hidden_row_stride", c_int64),
        ("weight", c_void_p),
        ("weight_row_stride", c_int64),
        ("logits", c_void_p),
        ("logits_row_stride", c_int64),
        ("rows", c_int32),
        ("d_model", c_int32),
        ("vocab", c_int32),
        ("tile_n", c_int32),
        ("error_word", c_void_p),
    ]


# Every symbol include/mtr_sampler.h declares: (name, restype, argtypes).
EXPORTS = {
    "mtr_abi_version": (ctypes.c_int, []),
    "mtr_args_size": (ctypes.c_size_t, []),
    "mtr_args_init": (ctypes.c_int, [ctypes.POINTER(MtrSamplerArgs)]),
    "mtr_sampler_validate": (ctypes.c_int, [ctypes.POINTER(MtrSamplerArgs)]),
    "mtr_sampler_query": (ctypes.c_int, [c_int32, c_int32, c_int32, ctypes.POINTER(MtrLaunchInfo)]),
    "mtr_sampler_query_args": (ctypes.c_int, [ctypes.POINTER(MtrSamplerArgs), ctypes.POINTER(MtrLaunchInfo)]),
    "mtr_sampler_launch": (ctypes.c_int, [ctypes.POINTER(MtrSamplerArgs), c_void_p]),
    "mtr_status_string": (ctypes.c_char_p, [ctypes.c_int]),
    "mtr_last_cuda_error": (ctypes.c_int, []),
    "mtr_lmhead_validate": (ctypes.c_int, [ctypes.POINTER(MtrLmHeadArgs)]),
    "mtr_lmhead_launch": (ctypes.c_int, [ctypes.POINTER(MtrLmHeadArgs), c_void_p]),
    "mtr_lmhead_sample_launch": (ctypes.c_int, [ctypes.POINTER(MtrLmHeadArgs), ctypes.POINTER(MtrSamplerArgs),
                                                c_void_p]),
}


class NativeLibraryError(RuntimeError):
    """The CUDA library is missing, stale or incompatible."""


class SamplerError(RuntimeError):
    """A library call returned an error code."""

    def __init__(self, code: int, message: str):
        super().__init__(message)
        self.code = code


_lock = threading.Lock()
_lib = None


def library_path() -> Path:
    return _build.LIB_PATH


def load(path: str | Path | None = None) -> ctypes.CDLL:
    """Load (once) and check the native library."""
    global _lib
    with _lock:
        if _lib is not None and path is None:
            return _lib
        p = Path(path) if path is not None else _build.LIB_PATH
        if not p.exists():
            raise NativeLibraryError(
                f"native sampler library not found at {p}; build it with "
                "`python -m mapperatorinator_b200.build` (needs nvcc)"
            )
        try:
            lib = ctypes.CDLL(str(p))
        except OSError as exc:  # pragma: no cover - depends on the host
            raise NativeLibraryError(f"cannot load {p}: {exc}") from exc
        for name, (restype, argtypes) in EXPORTS.items():
            fn = getattr(lib, name, None)
            if fn is None:
                raise NativeLibraryError(f"{p} does not export {name}")
            fn.restype = restype
            fn.argtypes = argtypes
        if lib.mtr_abi_version() != ABI_VERSION:
            raise NativeLibraryError(f"ABI version {lib.mtr_abi_version()} != {ABI_VERSION}")
        if lib.mtr_args_size() != ctypes.sizeof(MtrSamplerArgs):
            raise NativeLibraryError(
                f"MtrSamplerArgs size mismatch: library {lib.mtr_args_size()} vs "
                f"binding {ctypes.sizeof(MtrSamplerArgs)}"
            )
        if path is None:
            _lib = lib
        return lib


def new_args() -> MtrSamplerArgs:
    args = MtrSamplerArgs()
    rc = load().mtr_args_init(ctypes.byref(args))
    check(rc, "mtr_args_init")
    return args


def status_string(code: int) -> str:
    return load().mtr_status_string(code).decode()


def check(rc: int, what: str = "mtr_sampler_launch") -> None:
    if rc != OK:
        lib = load()
        msg = f"{what} failed: {lib.mtr_status_string(rc).decode()}"
        if rc == ERR_CUDA:
            msg += f" (cudaError {lib.mtr_last_cuda_error()})"
        exc_type = ValueError if rc in (ERR_NULL_ARG, ERR_BAD_SHAPE, ERR_BAD_PARAM, ERR_ALIGNMENT) else SamplerError
        if exc_type is ValueError:
            raise ValueError(msg)
        raise SamplerError(rc, msg)


def validate(args: MtrSamplerArgs) -> int:
    return load().mtr_sampler_validate(ctypes.byref(args))


def launch(args: MtrSamplerArgs, stream: int | None) -> None:
    """Enqueue one fused step on ``stream`` (a cudaStream_t handle as int)."""
    rc = load().mtr_sampler_launch(ctypes.byref(args), c_void_p(stream or 0))
    check(rc)


def query(vocab: int, num_rows: int, with_penalties: bool = False) -> MtrLaunchInfo:
    info = MtrLaunchInfo()
    check(load().mtr_sampler_query(vocab, num_rows, int(with_penalties), ctypes.byref(info)), "mtr_sampler_query")
    return info


def query_args(args: MtrSamplerArgs) -> MtrLaunchInfo:
    """Kernel and geometry the launcher picks for these exact arguments."""
    info = MtrLaunchInfo()
    check(load().mtr_sampler_query_args(ctypes.byref(args), ctypes.byref(info)), "mtr_sampler_query_args")
    return info


def new_lmhead_args() -> MtrLmHeadArgs:
    a = MtrLmHeadArgs()
    ctypes.memset(ctypes.byref(a), 0, ctypes.sizeof(a))
    a.abi_version = ABI_VERSION
    a.struct_size = ctypes.sizeof(a)
    return a


def lmhead_validate(args: MtrLmHeadArgs) -> int:
    return load().mtr_lmhead_validate(ctypes.byref(args))


def lmhead_launch(args: MtrLmHeadArgs, stream: int | None) -> None:
    check(load().mtr_lmhead_launch(ctypes.byref(args), c_void_p(stream or 0)), "mtr_lmhead_launch")


def lmhead_sample_launch(lm: MtrLmHeadArgs, args: MtrSamplerArgs, stream: int | None) -> None:
    check(load().mtr_lmhead_sample_launch(ctypes.byref(lm), ctypes.byref(args), c_void_p(stream or 0)),
          "mtr_lmhead_sample_launch")

"""Python entry to the CPU oracle (``oracle/mtr_oracle.c``).

TEST INFRASTRUCTURE ONLY: used by tests/, ``__graft_entry__.smoke()`` and the
CPU baseline leg of bench.py as the checker.  Nothing in the product package
imports this module.
"""

from __future__ import annotations

import ctypes
import subprocess
from pathlib import Path

import numpy as np

from mapperatorinator_b200 import _native as N
from tests.harness.stepargs import STATE_KEYS, fill_args, host_arrays
from tests.harness.workloads import StepInputs

ORACLE_DIR = Path(__file__).resolve().parent
LIB = ORACLE_DIR / "_build" / "libmtr_oracle.so"
_lib = None


def build(force: bool = False) -> Path:
    src = ORACLE_DIR / "mtr_oracle.c"
    hdr = ORACLE_DIR.parent / "include" / "mtr_sampler.h"
    if force or _stale():
        subprocess.run(["make", "-s", "-C", str(ORACLE_DIR), "-B" if force else "_build/libmtr_oracle.so"],
                       check=True)
    return LIB


def _stale() -> bool:
    src = ORACLE_DIR / "mtr_oracle.c"
    hdr = ORACLE_DIR.parent / "include" / "mtr_sampler.h"
    return not LIB.exists() or LIB.stat().st_mtime < max(src.stat().st_mtime, hdr.stat().st_mtime)


def load() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        if _stale():
            build()
        lib = ctypes.CDLL(str(LIB))
        lib.mtr_oracle_args_size.restype = ctypes.c_size_t
        if lib.mtr_oracle_args_size() != ctypes.sizeof(N.MtrSamplerArgs):
            raise RuntimeError(f"oracle library {LIB} was built for another MtrSamplerArgs layout; rebuild it")
        lib.mtr_oracle_run.restype = ctypes.c_int
        lib.mtr_oracle_run.argtypes = [ctypes.POINTER(N.MtrSamplerArgs)]
        lib.mtr_oracle_expfx.restype = ctypes.c_uint32
        lib.mtr_oracle_expfx.argtypes = [ctypes.c_float]
        lib.mtr_oracle_markstein_div.restype = ctypes.c_float
        lib.mtr_oracle_markstein_div.argtypes = [ctypes.c_float, ctypes.c_float]
        lib.mtr_oracle_log_d.restype = ctypes.c_double
        lib.mtr_oracle_log_d.argtypes = [ctypes.c_double]
        _lib = lib
    return _lib


def expfx(d: float) -> int:
    return int(load().mtr_oracle_expfx(ctypes.c_float(d)))


def log_d(x: float) -> float:
    return float(load().mtr_oracle_log_d(ctypes.c_double(x)))


def markstein_div(x: float, t: float) -> float:
    return float(load().mtr_oracle_markstein_div(ctypes.c_float(x), ctypes.c_float(t)))


def _init_args() -> N.MtrSamplerArgs:
    a = N.MtrSamplerArgs()
    ctypes.memset(ctypes.byref(a), 0, ctypes.sizeof(a))
    a.abi_version = N.ABI_VERSION
    a.struct_size = ctypes.sizeof(a)
    a.cfg_scale = 1.0
    a.repetition_penalty = 1.0
    a.temperature = 1.0
    a.top_p = 1.0
    return a


def run(s: StepInputs) -> dict:
    """Run the oracle on host copies of ``s``; returns outputs and final state."""
    arrays = host_arrays(s)
    args = fill_args(_init_args(), s, lambda k: arrays[k].ctypes.data if k in arrays else 0)
    load().mtr_oracle_run(ctypes.byref(args))
    return {k: arrays[k] for k in STATE_KEYS if k in arrays}


def compare(ref: dict, got: dict, *, lp_rtol: float = 1e-5, lp_atol: float = 1e-6) -> list[str]:
    """Differences between two result dicts (empty list = parity).

    Token ids, row status, states and processed scores must be bit-exact;
    log-probabilities agree within lp_rtol * |ref| + lp_atol (NaN == NaN).
    """
    errs = []
    ref, got = dict(ref), dict(got)
    if "out_status" in ref:
        # MTR_ROW_SLOW_PATH only says which exact selection path the kernel took
        info = np.uint32(N.ROW_SLOW_PATH)
        ref["out_status"] = ref["out_status"] & ~info
        got["out_status"] = got["out_status"] & ~info
    for k in ("out_ids", "out_status", "mono_state", "prev_token", "unfinished", "stop_counts"):
        if k in ref:
            if not np.array_equal(ref[k], got[k]):
                bad = np.nonzero(ref[k] != got[k])[0]
                errs.append(f"{k}: {len(bad)} rows differ, first {bad[:5].tolist()} "
                            f"ref {ref[k][bad[:5]].tolist()} got {got[k][bad[:5]].tolist()}")
    if "id_buffer" in ref and not np.array_equal(ref["id_buffer"], got["id_buffer"]):
        bad = np.argwhere(ref["id_buffer"] != got["id_buffer"])
        errs.append(f"id_buffer: {len(bad)} entries differ, first {bad[:5].tolist()}")
    if "lb_state" in ref:
        r, g = ref["lb_state"], got["lb_state"]
        same = (r.view(np.uint32) == g.view(np.uint32)) | (np.isnan(r) & np.isnan(g))
        if not same.all():
            bad = np.nonzero(~same)[0]
            errs.append(f"lb_state: {len(bad)} rows differ, first {bad[:5].tolist()} "
                        f"ref {r[bad[:5]].tolist()} got {g[bad[:5]].tolist()}")
    if "out_scores" in ref:
        r, g = ref["out_scores"], got["out_scores"]
        same = (r.view(np.uint32) == g.view(np.uint32)) | (np.isnan(r) & np.isnan(g))
        if not same.all():
            rows, cols = np.nonzero(~same)
            errs.append(f"out_scores: {len(rows)} elements differ, first (row, col) "
                        f"{list(zip(rows[:5].tolist(), cols[:5].tolist()))} ref {r[rows[:5], cols[:5]].tolist()} "
                        f"got {g[rows[:5], cols[:5]].tolist()}")
    if "out_logprobs" in ref:
        r, g = ref["out_logprobs"], got["out_logprobs"]
        both_nan = np.isnan(r) & np.isnan(g)
        same_inf = np.isinf(r) & (r == g)
        with np.errstate(invalid="ignore"):
            close = np.abs(r.astype(np.float64) - g.astype(np.float64)) <= lp_rtol * np.abs(r) + lp_atol
        ok = both_nan | same_inf | close
        if not ok.all():
            rows, cols = np.nonzero(~ok)
            errs.append(f"out_logprobs: {len(rows)} elements out of tolerance, first "
                        f"{list(zip(rows[:5].tolist(), cols[:5].tolist()))}")
    return errs

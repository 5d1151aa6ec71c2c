"""CPU checks of the decision arithmetic shared by the kernel and the oracle."""

import ctypes

import numpy as np
import pytest

from oracle import oracle


def test_expfx_accuracy():
    lib = oracle.load()
    d = np.concatenate([np.linspace(-21.4, 0.0, 20001), -np.logspace(-8, 1.3, 2000)]).astype(np.float32)
    got = np.array([lib.mtr_oracle_expfx(ctypes.c_float(v)) for v in d], dtype=np.float64)
    exact = np.exp(d.astype(np.float64)) * 2.0**31
    # fp32 evaluation (a few units of 2^-24 relative) plus truncation to an
    # integer number of 2^-31 units
    err = np.abs(got - exact)
    assert (err <= 4e-7 * exact + 1.0).all(), (err - 4e-7 * exact).max()
    assert oracle.expfx(0.0) == 2**31
    assert oracle.expfx(-40.0) == 0 and oracle.expfx(float("-inf")) == 0


def test_expfx_monotone_on_grid():
    d = np.linspace(-22, 0, 50001).astype(np.float32)
    q = np.array([oracle.expfx(float(v)) for v in d], dtype=np.int64)
    assert (np.diff(q) >= -2).all()  # non-monotone wiggles stay within truncation noise


@pytest.mark.parametrize("t", [0.9, 1.1, 0.7, 1.3, 0.85, 2.5, 0.123, 7.77, 0.99999994, 1.9999999, 1.4999999,
                               3.0, 1.0 / 3.0, 0.5000001])
def test_markstein_division_matches_ieee(t):
    lib = oracle.load()
    fn = lib.mtr_oracle_markstein_mismatches
    fn.restype = ctypes.c_uint64
    fn.argtypes = [ctypes.c_float, ctypes.c_int, ctypes.c_int, ctypes.c_uint32]
    # every 7th significand of the binades [2^-20, 2^20): ~48M checks per value
    assert fn(ctypes.c_float(t), -20, 20, 7) == 0
    # range limits the kernel relies on (|x| in [2^-60, 2^60))
    assert fn(ctypes.c_float(t), -60, -56, 101) == 0
    assert fn(ctypes.c_float(t), 56, 60, 101) == 0


def test_markstein_random_temperatures():
    lib = oracle.load()
    fn = lib.mtr_oracle_markstein_mismatches
    fn.restype = ctypes.c_uint64
    fn.argtypes = [ctypes.c_float, ctypes.c_int, ctypes.c_int, ctypes.c_uint32]
    rng = np.random.default_rng(3)
    for t in rng.uniform(0.05, 20.0, size=24).astype(np.float32):
        assert fn(ctypes.c_float(float(t)), -8, 8, 997) == 0, t

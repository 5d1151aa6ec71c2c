"""Load the reference fixtures and turn each chain case into StepInputs."""

from __future__ import annotations

import json
from functools import lru_cache
from pathlib import Path

import numpy as np

from mapperatorinator_b200 import _native as N
from tests.harness.workloads import StepInputs, bf16_bits

GOLDEN = Path(__file__).resolve().parent / "golden" / "reference_chain.npz"
CHAIN_CASES = ("chain_cfg_mono_temp", "chain_condtemp", "chain_condtemp_b1", "chain_bias_cfg2", "chain_c0_shape",
               "chain_c1_bf16")


@lru_cache(maxsize=1)
def fixtures():
    z = np.load(GOLDEN)
    data = {k: z[k] for k in z.files}
    meta = json.loads(bytes(data.pop("meta.json")).decode())
    return data, meta


def case(name: str) -> dict:
    data, meta = fixtures()
    out = {k.split(".", 1)[1]: v for k, v in data.items() if k.startswith(name + ".")}
    out["meta"] = meta.get(name, {})
    return out


def bits_for(ids, vocab):
    words = np.zeros((vocab + 31) // 32, dtype=np.uint32)
    for t in ids:
        words[t >> 5] |= np.uint32(1 << (t & 31))
    return words


def conditionals(meta: dict, vocab: int):
    """The reference's conditional temperature list (logit_processors.py:61-66)."""
    t, tt, mt, kt = meta["temps"]
    tt = t if tt is None else tt
    mt = t if mt is None else mt
    kt = t if kt is None else kt
    ex = meta.get("extra", {})
    conds = []
    beat = [ex[k][0] for k in ("BEAT", "MEASURE") if k in ex]
    if "TIMING_POINT" in ex:
        beat.append(ex["TIMING_POINT"][0])
    mania = [ex[k][0] for k in ("CIRCLE", "HOLD_NOTE", "HOLD_NOTE_END")] if "HOLD_NOTE_END" in ex else []
    taiko = list(range(*ex["SCROLL_SPEED"])) if "SCROLL_SPEED" in ex else []
    if tt != t and beat:
        conds.append((tt, 1, bits_for(beat, vocab)))
    if mt != t and mania:
        conds.append((mt, 3, bits_for(mania, vocab)))
    if kt != t and taiko:
        conds.append((kt, 1, bits_for(taiko, vocab)))
    return conds


def chain_step(name: str, *, select_mode=N.SELECT_NONE, top_k=0, top_p=1.0, top_p_mode=N.TOPP_HF) -> StepInputs:
    c = case(name)
    m = c["meta"]
    V, B = m["V"], m["B"]
    x = c["logits"].astype(np.float32)
    dtype = m.get("dtype", "f32")
    logits = bf16_bits(x) if dtype == "bf16" else x
    temps = m["temps"]
    if m["types_first"]:
        temp_mode, conds = N.TEMP_ROW_CONDITIONAL, conditionals(m, V)
    else:
        temp_mode, conds = N.TEMP_SCALAR, []
    return StepInputs(
        logits=logits, dtype=dtype, num_rows=B, cfg_scale=m["cfg"], input_ids=c["input_ids"].astype(np.int64),
        mono_mode=N.MONO_SCAN, ts_start=m["ts"][0], ts_end=m["ts"][1], sos_ids=tuple(m["sos"]),
        timeshift_bias=m["bias"], temp_mode=temp_mode, temperature=temps[0], cond=conds,
        select_mode=select_mode, top_k=top_k, top_p=top_p, top_p_mode=top_p_mode,
        uniforms=np.zeros(B, dtype=np.float32), want_scores=True,
    )


def explain_keep_mismatch(scores: np.ndarray, ref_keep: np.ndarray, got_keep: np.ndarray, top_p: float,
                          status: int | None = None, margin: float = 1e-5) -> bool:
    """True when a keep-set difference in one row is a tie at the cut or a
    cumulative mass within `margin` of top_p (float64 reference mass).

    A tie at the cut: every differing token has the score of the smallest
    kept score (the group the two sides split at different ids).  When the
    kernel's ``status`` is given it must also carry MTR_ROW_TIE_AT_CUT for the
    tie to excuse the difference; the flag alone excuses nothing."""
    diff_ids = np.nonzero(ref_keep != got_keep)[0]
    cut = min(scores[ref_keep].min(), scores[got_keep].min())
    tie = bool((scores[diff_ids] == cut).all())
    if tie and (status is None or status & N.ROW_TIE_AT_CUT):
        return True
    fin = np.isfinite(scores)
    x = scores[fin].astype(np.float64)
    ids = np.nonzero(fin)[0]
    p = np.exp(x - x.max())
    p /= p.sum()
    order = np.lexsort((ids, -x))
    above = np.concatenate([[0.0], np.cumsum(p[order])[:-1]])
    diff = np.nonzero(ref_keep != got_keep)[0]
    pos = {int(t): i for i, t in enumerate(ids[order])}
    return all(abs(above[pos[int(t)]] - top_p) < margin for t in diff if int(t) in pos)


LOOKBACK_CASES = ("lookback_renorm", "lookback_mask", "lookback_chain")


def lookback_tokenizer(meta: dict):
    """A duck-typed tokenizer with the event layout a lookback fixture was made with."""
    import enum
    from types import SimpleNamespace

    et = enum.Enum("EventType", ["TIME_SHIFT"] + list(meta["extra"]))
    ts0, ts1 = meta["ts"]
    return SimpleNamespace(
        sos_id=1, context_sos={}, eos_id=meta["eos"][0], context_eos={i: e for i, e in enumerate(meta["eos"][1:])},
        event_start={et.TIME_SHIFT: ts0, **{et[k]: v[0] for k, v in meta["extra"].items()}},
        event_end={et.TIME_SHIFT: ts1, **{et[k]: v[1] for k, v in meta["extra"].items()}},
        event_range={et.TIME_SHIFT: SimpleNamespace(min_value=meta["ts_min"],
                                                    max_value=meta["ts_min"] + ts1 - ts0 - 1)},
        vocab_size_out=meta["vocab"])


def lookback_step(name: str, t: int, lb_state: np.ndarray, **kw) -> StepInputs:
    """Step t of a lookback fixture (processor output only), carrying lb_state."""
    from mapperatorinator_b200.logit_processors import lookback_spec

    c = case(name)
    m = c["meta"]
    V = m["vocab"]
    spec = lookback_spec(m["lookback_time"], lookback_tokenizer(m), m["types_first"])
    ids = np.ascontiguousarray(c["input_ids"][:, : m["prefix"] + t + 1].astype(np.int64))
    B = ids.shape[0]
    base = dict(dtype="f32", num_rows=B, input_ids=ids, select_mode=N.SELECT_NONE, want_scores=True,
                uniforms=np.zeros(B, dtype=np.float32), lookback_mode=spec["mode"], lb_start=spec["start"],
                lb_end=spec["end"], lb_eos_ids=spec["eos_ids"], lb_timed_bits=bits_for(spec["timed"], V),
                lb_state=lb_state)
    if name == "lookback_chain":
        base.update(logits=c["logits"][t], cfg_scale=m["cfg"], mono_mode=N.MONO_SCAN, ts_start=m["ts"][0],
                    ts_end=m["ts"][1], sos_ids=tuple(m["sos"]), timeshift_bias=m["bias"],
                    temp_mode=N.TEMP_ROW_CONDITIONAL, temperature=m["temps"][0], cond=conditionals(m, V))
    else:
        base.update(logits=c["scores"][t])
    base.update(kw)
    return StepInputs(**base)


def lookback_reference(name: str, t: int) -> np.ndarray:
    c = case(name)
    return c["out"][t] if "out" in c else c["processed"][t]


def lookback_close(got: np.ndarray, ref: np.ndarray, lb_start: int, atol: float = 1e-5, rtol: float = 1e-6,
                   patol: float = 1e-6) -> list:
    """Elements where the fixed-point / double lookback transform and the
    reference's float32 softmax-and-log disagree: -inf must match exactly,
    finite log-probabilities within atol + rtol |ref|.  The lb_start column is
    log((s - 1) p / (1 - p)), a difference of nearly equal float32 numbers in
    the reference (absolute error ~1e-7 in probability), so it is compared as a
    probability: |e^got - e^ref| <= patol."""
    got = got.astype(np.float64)
    ref = ref.astype(np.float64)
    cols = np.ones(ref.shape[1], dtype=bool)
    cols[lb_start] = False
    g, r = got[:, cols], ref[:, cols]
    bad = np.zeros(ref.shape, dtype=bool)
    with np.errstate(invalid="ignore"):
        b = (np.isneginf(r) != np.isneginf(g)) | (np.isfinite(r) & ~(np.abs(g - r) <= atol + rtol * np.abs(r)))
        bad[:, cols] = b
        bad[:, lb_start] = ~(np.abs(np.exp(got[:, lb_start]) - np.exp(ref[:, lb_start])) <= patol)
    return np.argwhere(bad).tolist()

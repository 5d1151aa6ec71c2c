"""Seeded synthetic decode-step workloads.

No checkpoint, song or dataset is involved: the sampler consumes a logits
matrix and per-row decode state, and these generators build those with the
shapes and value distributions of the five sampler workloads this project is
measured on (vocabulary split 0-1999 time shift / 2000-3599 position /
3600-4095 type and special for V = 4096):

* ``cfg_pair_fp32``   B=1 with CFG (2 rows), V=4096 fp32 ~ N(0, 1.5^2) + 8 spike
  ids at +8; CFG 1.5, monotonic mask, T=0.9 on time-shift ids, top_p 0.9.
* ``batched_decode``  64 CFG pairs (128 rows), V=4096 bf16, as above plus an
  event-grammar mask (16 random classes, random 16x16 transition table).
* ``penalty_sweep``   1024 rows, V=4096 bf16 ~ N(0, 2^2), 512-id history,
  repetition 1.1 / frequency 0.2 / presence 0.1, top_k 50 then top_p 0.95.
* ``sharded_decode``  4096 CFG pairs (8192 rows), V=4096 bf16 ~ N(0, 2^2),
  penalty chain + monotonic + grammar.

Everything is produced with numpy's PCG64 from an explicit seed, so the CPU
oracle and the GPU see the same bytes.
"""

from __future__ import annotations

from dataclasses import dataclass, field, replace

import numpy as np

TS_END_4096 = 2000       # time-shift ids [0, 2000)
POS_END_4096 = 3600      # position ids [2000, 3600)
SOS_IDS_4096 = (4094,)   # a structural start id inside the special range


def bf16_bits(x: np.ndarray) -> np.ndarray:
    """Round float32 to bfloat16 (nearest even); returns the uint16 bit patterns."""
    u = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32)
    nan = (u & 0x7FFFFFFF) > 0x7F800000
    r = ((u >> 16) & 1) + 0x7FFF
    out = ((u + r) >> 16).astype(np.uint16)
    out[nan] = ((u[nan] >> 16) | 0x40).astype(np.uint16)
    return out


def bf16_to_f32(bits: np.ndarray) -> np.ndarray:
    return (bits.astype(np.uint32) << 16).view(np.float32)


@dataclass
class StepInputs:
    """One decode step of the fused chain (host arrays; CPU-oracle layout)."""

    logits: np.ndarray                 # [R, V]; float32, float16 or uint16 (bf16 bits)
    dtype: str                         # "f32" | "bf16" | "f16"
    num_rows: int                      # B output rows
    cfg_scale: float = 1.0             # CFG active when > 1 (rows i and B + i)
    input_ids: np.ndarray | None = None  # [B, L] int64 / int32
    # monotonic
    mono_mode: int = 0
    ts_start: int = 0
    ts_end: int = 0
    sos_ids: tuple = ()
    mono_state: np.ndarray | None = None  # [B] int32
    timeshift_bias: float = 0.0
    flags: int = 0
    # grammar
    grammar_class_of: np.ndarray | None = None  # [V] uint8
    grammar_allow: np.ndarray | None = None     # [C] uint32
    prev_token: np.ndarray | None = None        # [B] int32
    grammar_bits: bool = True                   # pass the per-class vocabulary bitmaps
    # penalties
    repetition_penalty: float = 1.0
    frequency_penalty: float = 0.0
    presence_penalty: float = 0.0
    penalty_start: int = 0
    # temperature
    temp_mode: int = 0
    temperature: float = 1.0
    cond: list = field(default_factory=list)        # [(T, offset, bits[uint32])]
    col_ranges: list = field(default_factory=list)  # [(start, end, T)]
    # selection
    select_mode: int = 2
    top_k: int = 0
    top_p: float = 1.0
    top_p_mode: int = 0
    uniforms: np.ndarray | None = None  # [B] float32
    # outputs / finishing
    want_scores: bool = False
    want_logprobs: bool = False
    unfinished: np.ndarray | None = None  # [B] uint8
    pad_id: int = 0
    eos_ids: tuple = ()
    eos_ranges: tuple = ()
    # lookback bias (0 off, 1 mask, 2 renormalise)
    lookback_mode: int = 0
    lb_start: int = 0
    lb_end: int = 0
    lb_eos_ids: tuple = ()
    lb_timed_bits: np.ndarray | None = None  # [ceil(V/32)] uint32
    lb_state: np.ndarray | None = None       # [B] float32, NaN = no previous step
    # token append and stop counters
    id_buffer: np.ndarray | None = None      # [B, S] int64
    cur_len: int = 0
    cur_len_dev: np.ndarray | None = None    # [1] int32 (device-side column index)
    stop_counts: np.ndarray | None = None    # [2] uint32

    @property
    def vocab(self) -> int:
        return int(self.logits.shape[1])

    def with_(self, **kw) -> "StepInputs":
        return replace(self, **kw)


def _spiky_rows(rng, rows, vocab, sigma, spikes=8):
    x = rng.normal(0.0, sigma, size=(rows, vocab)).astype(np.float32)
    ids = rng.choice(vocab, size=spikes, replace=False)
    x[:, ids] = 8.0
    return x


def grammar_tables(rng, vocab, n_classes=16, p_allow=0.5):
    class_of = rng.integers(0, n_classes, size=vocab).astype(np.uint8)
    table = rng.random((n_classes, n_classes)) < p_allow
    for c in range(n_classes):  # keep every row non-empty
        if not table[c].any():
            table[c, rng.integers(0, n_classes)] = True
    allow = np.zeros(n_classes, dtype=np.uint32)
    for c in range(n_classes):
        for d in range(n_classes):
            if table[c, d]:
                allow[c] |= np.uint32(1 << d)
    return class_of, allow


def cfg_pair_fp32(seed: int = 0, vocab: int = 4096) -> StepInputs:
    rng = np.random.default_rng(seed)
    logits = _spiky_rows(rng, 2, vocab, 1.5)
    return StepInputs(
        logits=logits, dtype="f32", num_rows=1, cfg_scale=1.5,
        mono_mode=1, ts_start=0, ts_end=min(TS_END_4096, vocab), sos_ids=SOS_IDS_4096,
        mono_state=np.array([rng.integers(0, min(TS_END_4096, vocab))], dtype=np.int32),
        temp_mode=2, temperature=1.0, col_ranges=[(0, min(TS_END_4096, vocab), 0.9)],
        select_mode=2, top_p=0.9, top_p_mode=0,
        uniforms=rng.random(1, dtype=np.float32),
    )


def batched_decode(seed: int = 1, pairs: int = 64, vocab: int = 4096, dtype: str = "bf16") -> StepInputs:
    rng = np.random.default_rng(seed)
    x = _spiky_rows(rng, 2 * pairs, vocab, 1.5)
    logits = bf16_bits(x) if dtype == "bf16" else x
    class_of, allow = grammar_tables(rng, vocab)
    ts_end = min(TS_END_4096, vocab)
    return StepInputs(
        logits=logits, dtype=dtype, num_rows=pairs, cfg_scale=1.5,
        mono_mode=1, ts_start=0, ts_end=ts_end, sos_ids=SOS_IDS_4096,
        mono_state=rng.integers(0, ts_end, size=pairs).astype(np.int32),
        grammar_class_of=class_of, grammar_allow=allow,
        prev_token=rng.integers(0, vocab, size=pairs).astype(np.int32),
        temp_mode=2, temperature=1.0, col_ranges=[(0, ts_end, 0.9)],
        select_mode=2, top_p=0.9, top_p_mode=0,
        uniforms=rng.random(pairs, dtype=np.float32),
    )


def penalty_sweep(seed: int = 2, rows: int = 1024, vocab: int = 4096, history: int = 512,
                  dtype: str = "bf16") -> StepInputs:
    rng = np.random.default_rng(seed)
    x = rng.normal(0.0, 2.0, size=(rows, vocab)).astype(np.float32)
    logits = bf16_bits(x) if dtype == "bf16" else x
    ids = rng.integers(0, vocab, size=(rows, history)).astype(np.int64)
    return StepInputs(
        logits=logits, dtype=dtype, num_rows=rows, input_ids=ids,
        repetition_penalty=1.1, frequency_penalty=0.2, presence_penalty=0.1,
        select_mode=2, top_k=50, top_p=0.95, top_p_mode=0,
        uniforms=rng.random(rows, dtype=np.float32),
    )


def sharded_decode(seed: int = 4, pairs: int = 4096, vocab: int = 4096, history: int = 512,
                   dtype: str = "bf16") -> StepInputs:
    rng = np.random.default_rng(seed)
    x = rng.normal(0.0, 2.0, size=(2 * pairs, vocab)).astype(np.float32)
    logits = bf16_bits(x) if dtype == "bf16" else x
    class_of, allow = grammar_tables(rng, vocab)
    ts_end = min(TS_END_4096, vocab)
    return StepInputs(
        logits=logits, dtype=dtype, num_rows=pairs, cfg_scale=1.5,
        input_ids=rng.integers(0, vocab, size=(pairs, history)).astype(np.int64),
        mono_mode=1, ts_start=0, ts_end=ts_end, sos_ids=SOS_IDS_4096,
        mono_state=rng.integers(0, ts_end, size=pairs).astype(np.int32),
        grammar_class_of=class_of, grammar_allow=allow,
        prev_token=rng.integers(0, vocab, size=pairs).astype(np.int32),
        repetition_penalty=1.1, frequency_penalty=0.2, presence_penalty=0.1,
        select_mode=2, top_k=50, top_p=0.95, top_p_mode=0,
        uniforms=rng.random(pairs, dtype=np.float32),
    )


WORKLOADS = {
    "cfg_pair_fp32": cfg_pair_fp32,
    "batched_decode": batched_decode,
    "penalty_sweep": penalty_sweep,
    "sharded_decode": sharded_decode,
}


def lookback_decode(seed: int = 7, pairs: int = 64, vocab: int = 4096, dtype: str = "bf16", step: int = 0,
                    lb_state: np.ndarray | None = None) -> StepInputs:
    """A sampling step with the lookback bias renormalising (types_first=True):
    CFG pairs, monotonic state, lookback range [100, 600), EOS ids (2, 7, 9)
    boosted per row, timed-event ids = a seeded 1/8 of the vocabulary, last
    input id timed on about half the rows.  `step` reseeds the scores and last
    ids; `lb_state` carries the previous step's EOS probabilities (default: a
    mix of NaN and values in [0, 0.9])."""
    rng = np.random.default_rng(seed)
    timed = np.sort(rng.choice(vocab, size=max(vocab // 8, 1), replace=False))
    untimed = np.setdiff1d(np.arange(vocab), timed)
    bits = np.zeros((vocab + 31) // 32, dtype=np.uint32)
    np.bitwise_or.at(bits, timed >> 5, (np.uint32(1) << (timed & 31).astype(np.uint32)))
    if lb_state is None:
        lb_state = rng.uniform(0.0, 0.9, size=pairs).astype(np.float32)
        lb_state[rng.random(pairs) < 0.2] = np.nan
    rs = np.random.default_rng(seed * 1000 + step + 1)
    x = _spiky_rows(rs, 2 * pairs, vocab, 1.5)
    x[:, [2, 7, 9]] += rs.uniform(-2.0, 5.0, size=(2 * pairs, 1)).astype(np.float32)
    ids = rs.integers(0, vocab, size=(pairs, 6)).astype(np.int64)
    pick = rs.random(pairs) < 0.5
    ids[:, -1] = np.where(pick, rs.choice(timed, size=pairs), rs.choice(untimed, size=pairs))
    lb_end = min(600, vocab)
    ts_end = min(TS_END_4096, vocab)
    return StepInputs(
        logits=bf16_bits(x) if dtype == "bf16" else x.astype(np.float16) if dtype == "f16" else x, dtype=dtype,
        num_rows=pairs, cfg_scale=1.5, input_ids=ids,
        mono_mode=1, ts_start=0, ts_end=ts_end, sos_ids=SOS_IDS_4096,
        mono_state=rs.integers(0, 64, size=pairs).astype(np.int32), temperature=0.9,
        select_mode=2, top_k=40, top_p=0.9, top_p_mode=0, uniforms=rs.random(pairs, dtype=np.float32),
        lookback_mode=2, lb_start=min(100, vocab - 1), lb_end=lb_end, lb_eos_ids=(2, 7, 9), lb_timed_bits=bits,
        lb_state=lb_state)

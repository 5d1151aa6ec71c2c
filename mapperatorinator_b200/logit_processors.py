"""Drop-in logits processors backed by the fused sm_100a kernel.

Mirrors osuT5/osuT5/inference/logit_processors.py: the same class names,
constructor arguments, ``__call__(input_ids, scores) -> scores`` signature and
error behaviour, so a ``LogitsProcessorList`` built here slots into the
reference's generate loops (server.model_generate, the optimized single
engine, the fast decoder loop).  Every processor runs on CUDA through the C ABI
library; there is no CPU path (CPU tensors raise ``ValueError``).

``build_logits_processor_list`` returns a list holding ONE
:class:`FusedLogitsProcessor` that performs the whole chain -- CFG ->
monotonic time-shift mask -> timeshift bias -> temperature (scalar or
per-row conditional) -> lookback bias and, optionally, the top-k / top-p warpers that
``generate()`` would append -- in a single kernel launch with no host
synchronisation.  The individual classes run the same kernel with only their
own stage enabled.
"""

from __future__ import annotations

import ctypes
from typing import Iterable

import torch

from . import _native as N
from .sampling import set_input_ids, set_logits, token_bitmap

try:  # the base class is only a marker; any object with __call__ works in HF lists
    from transformers import LogitsProcessor as _LogitsProcessorBase
except Exception:  # pragma: no cover - transformers is optional
    class _LogitsProcessorBase:  # type: ignore[no-redef]
        pass


MILISECONDS_PER_STEP = 10


# ---------------------------------------------------------------- tokenizer helpers
def _event_key(table: dict, name: str):
    """Find the EventType member called `name` among a tokenizer's keys, so both
    the reference's EventType and any other enum with the same names work."""
    for k in table:
        if getattr(k, "name", k) == name:
            return k
    return None


def _event_start(tokenizer, name: str):
    k = _event_key(tokenizer.event_start, name)
    return None if k is None else tokenizer.event_start[k]


def _event_end(tokenizer, name: str):
    k = _event_key(tokenizer.event_end, name)
    return None if k is None else tokenizer.event_end[k]


def _time_shift_range(tokenizer) -> tuple[int, int]:
    start, end = _event_start(tokenizer, "TIME_SHIFT"), _event_end(tokenizer, "TIME_SHIFT")
    if start is None or end is None:
        raise KeyError("tokenizer has no TIME_SHIFT event range")
    return int(start), int(end)


def get_beat_type_tokens(tokenizer) -> tuple[int, ...]:
    """logit_processors.py:12-19"""
    beat = [_event_start(tokenizer, "BEAT"), _event_start(tokenizer, "MEASURE")]
    if _event_key(tokenizer.event_start, "TIMING_POINT") is not None:
        beat.append(_event_start(tokenizer, "TIMING_POINT"))
    return tuple(beat)


def get_mania_type_tokens(tokenizer) -> tuple[int, ...]:
    """logit_processors.py:22-27"""
    if _event_key(tokenizer.event_start, "HOLD_NOTE_END") is None:
        return ()
    return (_event_start(tokenizer, "CIRCLE"), _event_start(tokenizer, "HOLD_NOTE"),
            _event_start(tokenizer, "HOLD_NOTE_END"))


def get_scroll_speed_tokens(tokenizer) -> tuple[int, ...]:
    """logit_processors.py:30-32"""
    if _event_key(tokenizer.event_start, "SCROLL_SPEED") is None:
        return ()
    return tuple(range(_event_start(tokenizer, "SCROLL_SPEED"), _event_end(tokenizer, "SCROLL_SPEED")))


def _sos_ids(tokenizer) -> tuple[int, ...]:
    return (int(tokenizer.sos_id),) + tuple(int(v) for v in getattr(tokenizer, "context_sos", {}).values())


# Event types whose tokens carry a time (osuT5/osuT5/dataset/data_utils.py:60-78);
# the lookback bias acts after one of them.  Names, so any EventType enum with
# these member names works.
TIMED_EVENT_NAMES = ("CIRCLE", "SPINNER", "SPINNER_END", "SLIDER_HEAD", "LAST_ANCHOR", "SLIDER_END", "BEAT",
                     "MEASURE", "TIMING_POINT", "KIAI", "HOLD_NOTE", "HOLD_NOTE_END", "DRUMROLL", "DRUMROLL_END",
                     "DENDEN", "DENDEN_END", "SCROLL_SPEED_CHANGE")


def _encode_time_shift(tokenizer, value: int) -> int:
    """tokenizer.encode(Event(TIME_SHIFT, value)) (tokenizer.py:276-290): the
    range's first id + value - min_value, ValueError outside [min, max]."""
    start = _event_start(tokenizer, "TIME_SHIFT")
    if start is None:
        raise ValueError("unknown event type: TIME_SHIFT")
    er_table = getattr(tokenizer, "event_range", None)
    lo, hi = 0, None
    if er_table:
        k = _event_key(er_table, "TIME_SHIFT")
        if k is not None:
            lo, hi = int(er_table[k].min_value), int(er_table[k].max_value)
    else:
        hi = _event_end(tokenizer, "TIME_SHIFT") - start - 1
    if value < lo or (hi is not None and value > hi):
        raise ValueError(f"event value {value} is not within range [{lo}, {hi}] for event type TIME_SHIFT")
    return int(start) + value - lo


def lookback_spec(lookback_max_time: float, tokenizer, types_first: bool) -> dict:
    """The constants LookbackBiasLogitsWarper derives from the tokenizer
    (logit_processors.py:127-141): the lookback time-shift ids [start, end),
    the EOS ids (eos + every context eos) and the timed-event ids."""
    start = int(_event_start(tokenizer, "TIME_SHIFT"))
    end = _encode_time_shift(tokenizer, int(lookback_max_time / MILISECONDS_PER_STEP))
    eos = (int(tokenizer.eos_id),) + tuple(int(v) for v in getattr(tokenizer, "context_eos", {}).values())
    if len(eos) > N.MAX_LB_EOS:
        raise ValueError(f"at most {N.MAX_LB_EOS} eos / context-eos ids")
    timed = []
    for name in TIMED_EVENT_NAMES:
        k = _event_key(tokenizer.event_start, name)
        if k is not None:
            timed.extend(range(int(tokenizer.event_start[k]), int(tokenizer.event_end[k])))
    return {"mode": N.LOOKBACK_RENORM if types_first else N.LOOKBACK_MASK, "start": start, "end": end,
            "eos_ids": eos, "timed": tuple(timed)}


def _bitmap(tokens: Iterable[int], vocab: int, device) -> torch.Tensor:
    return token_bitmap(tokens, vocab, device)


# ---------------------------------------------------------------- the fused processor
class FusedLogitsProcessor(_LogitsProcessorBase):
    """The whole processor chain of ``build_logits_processor_list`` in one launch.

    ``__call__(input_ids [B, L], scores [R, V]) -> [B, V] float32`` with R = 2B
    when ``cfg_scale > 1`` (first half = conditional rows, as HF's
    ClassifierFreeGuidanceLogitsProcessor).  ``scores`` may be float32,
    bfloat16 or float16.  With CFG a new tensor is returned; without CFG and
    with float32 scores the result is written in place and ``scores`` itself
    is returned (the reference's monotonic processor also mutates in place).
    """

    def __init__(self, *, vocab_size: int | None = None, cfg_scale: float = 1.0,
                 time_shift_range: tuple[int, int] | None = None, sos_ids: tuple[int, ...] = (),
                 stateful_monotonic: bool = False, timeshift_bias: float = 0.0, temperature: float = 1.0,
                 conditionals: list[tuple[float, tuple[int, ...], int]] = (), top_k: int = 0, top_p: float = 1.0,
                 top_p_mode: str = "hf", grammar=None, repetition_penalty: float = 1.0,
                 frequency_penalty: float = 0.0, presence_penalty: float = 0.0, lookback: dict | None = None,
                 inplace: bool = True):
        if cfg_scale <= 1.0 and cfg_scale != 1.0:
            cfg_scale = 1.0
        if not (temperature > 0):
            raise ValueError(f"`temperature` (={temperature}) has to be a strictly positive float")
        if not (0.0 < top_p <= 1.0):
            raise ValueError(f"`top_p` has to be a float > 0 and <= 1, but is {top_p}")
        if top_k < 0:
            raise ValueError(f"`top_k` has to be a non-negative integer, but is {top_k}")
        if len(sos_ids) > N.MAX_SOS_IDS or len(conditionals) > N.MAX_COND_TEMPS:
            raise ValueError("too many sos ids or conditional temperatures")
        self.vocab_size = vocab_size
        self.cfg_scale = float(cfg_scale)
        self.time_shift_range = time_shift_range
        self.sos_ids = tuple(int(s) for s in sos_ids)
        self.stateful_monotonic = stateful_monotonic
        self.timeshift_bias = float(timeshift_bias)
        self.temperature = float(temperature)
        self.conditionals = [(float(t), tuple(int(x) for x in toks), int(off)) for t, toks, off in conditionals]
        self.top_k = int(top_k)
        self.top_p = float(top_p)
        self.top_p_mode = {"hf": N.TOPP_HF, "sample_fn": N.TOPP_SAMPLE_FN}[top_p_mode]
        self.grammar = grammar
        self.repetition_penalty = float(repetition_penalty)
        self.frequency_penalty = float(frequency_penalty)
        self.presence_penalty = float(presence_penalty)
        self.lookback = lookback
        self.inplace = inplace
        self._bits: dict = {}
        self._state: dict = {}
        self._state_len: dict = {}
        self._lb_state: dict = {}

    # per-device constant tables
    def _cond_bits(self, vocab: int, device):
        key = (vocab, device)
        if key not in self._bits:
            self._bits[key] = [_bitmap(toks, vocab, device) for _t, toks, _o in self.conditionals]
        return self._bits[key]

    def _timed_bits(self, vocab: int, device):
        key = ("timed", vocab, device)
        if key not in self._bits:
            self._bits[key] = _bitmap(self.lookback["timed"], vocab, device)
        return self._bits[key]

    def reset(self) -> None:
        """Forget the per-row state: the stateful monotonic state (the next call
        re-scans input_ids) and the lookback bias's previous EOS probability."""
        self._state.clear()
        self._state_len.clear()
        self._lb_state.clear()

    def __call__(self, input_ids: torch.LongTensor, scores: torch.FloatTensor) -> torch.FloatTensor:
        if not scores.is_cuda:
            raise ValueError("FusedLogitsProcessor runs on CUDA tensors only")
        if scores.dim() != 2:
            raise ValueError("scores must be [batch, vocab]")
        cfg = self.cfg_scale > 1.0
        B = input_ids.shape[0]
        if cfg and scores.shape[0] != 2 * B:
            raise ValueError(
                f"Logits should have twice the batch size of the input ids, the first half of batches corresponding to "
                f"the conditional inputs, and the second half of batches corresponding to the unconditional inputs. Got "
                f"batch size {scores.shape[0]} for the logits and {B} for the input ids.")
        if not cfg and scores.shape[0] != B:
            raise ValueError(f"scores has {scores.shape[0]} rows for {B} input rows")
        V = scores.shape[1]
        if self.vocab_size is not None and V != self.vocab_size:
            raise ValueError(f"vocabulary {V} != {self.vocab_size}")
        dev = scores.device
        if scores.stride(1) != 1:
            scores = scores.contiguous()
        input_ids = input_ids.to(dev)
        if input_ids.dim() != 2:
            raise ValueError("input_ids must be [batch, length]")
        if input_ids.shape[1] and input_ids.stride(1) != 1:
            input_ids = input_ids.contiguous()

        a = N.new_args()
        set_logits(a, scores)
        a.num_rows = B
        a.cfg_enabled = int(cfg)
        a.cfg_scale = self.cfg_scale
        a.cfg_second_offset = B
        set_input_ids(a, input_ids)
        L = input_ids.shape[1]
        if self.time_shift_range is not None:
            a.ts_start, a.ts_end = self.time_shift_range
            a.n_sos = len(self.sos_ids)
            for i, s in enumerate(self.sos_ids):
                a.sos_ids[i] = s
            if self.stateful_monotonic:
                key = (dev, B)
                st = self._state.get(key)
                if st is None:
                    st = torch.full((B,), -1, dtype=torch.int32, device=dev)
                    self._state[key] = st
                prev_len = self._state_len.get(key)
                a.mono_state = st.data_ptr()
                if prev_len is not None and L == prev_len + 1:
                    a.mono_mode = N.MONO_STATE
                    a.flags |= N.FLAG_MONO_UPDATE_FROM_IDS
                else:
                    a.mono_mode = N.MONO_SCAN
                self._state_len[key] = L
            else:
                a.mono_mode = N.MONO_SCAN
        a.timeshift_bias = self.timeshift_bias
        a.temperature = self.temperature
        keep = []
        if self.conditionals:
            a.temp_mode = N.TEMP_ROW_CONDITIONAL
            bits = self._cond_bits(V, dev)
            a.n_cond = len(self.conditionals)
            for i, ((t, _toks, off), b) in enumerate(zip(self.conditionals, bits)):
                a.cond_temperature[i] = t
                a.cond_offset[i] = off
                a.cond_token_bits[i] = b.data_ptr()
        if self.grammar is not None:
            a.grammar_class_of = self.grammar.class_of.data_ptr()
            a.grammar_allow = self.grammar.allow.data_ptr()
            a.grammar_vocab_bits = self.grammar.bits().data_ptr()
            a.grammar_n_classes = self.grammar.allow.numel()
            a.flags |= N.FLAG_GRAMMAR_PREV_FROM_IDS
        a.repetition_penalty = self.repetition_penalty
        a.frequency_penalty = self.frequency_penalty
        a.presence_penalty = self.presence_penalty
        if self.lookback is not None:
            lb = self.lookback
            a.lookback_mode = lb["mode"]
            a.lb_start, a.lb_end = lb["start"], lb["end"]
            if lb["mode"] == N.LOOKBACK_RENORM:
                a.n_lb_eos = len(lb["eos_ids"])
                for i, t in enumerate(lb["eos_ids"]):
                    a.lb_eos_ids[i] = t
                a.lb_timed_bits = self._timed_bits(V, dev).data_ptr()
                key = (dev, B)
                st = self._lb_state.get(key)
                if st is None:  # the reference's last_scores is None: no bias on the first call
                    st = torch.full((B,), float("nan"), dtype=torch.float32, device=dev)
                    self._lb_state[key] = st
                a.lb_state = st.data_ptr()
        a.select_mode = N.SELECT_NONE
        a.top_k = self.top_k if self.top_k < V else 0
        a.top_p = self.top_p
        a.top_p_mode = self.top_p_mode
        if self.inplace and not cfg and scores.dtype == torch.float32:
            out = scores
        else:
            out = torch.empty((B, V), dtype=torch.float32, device=dev)
        a.out_scores = out.data_ptr()
        a.out_scores_row_stride = out.stride(0)
        N.launch(a, torch.cuda.current_stream(dev).cuda_stream)
        del keep
        return out


# ---------------------------------------------------------------- single-stage processors
class TimeshiftBias(FusedLogitsProcessor):
    """logit_processors.py:35-43: scores[:, time range] += bias (new tensor)."""

    def __init__(self, timeshift_bias: float, time_start: int, time_end: int):
        super().__init__(timeshift_bias=timeshift_bias, time_shift_range=None, inplace=False)
        self.time_range = slice(time_start, time_end)
        self._range = (int(time_start), int(time_end))

    def __call__(self, input_ids, scores):
        if not scores.is_cuda:
            raise ValueError("TimeshiftBias runs on CUDA tensors only")
        a = N.new_args()
        set_logits(a, scores.contiguous())
        a.num_rows = scores.shape[0]
        a.ts_start, a.ts_end = self._range
        a.timeshift_bias = self.timeshift_bias
        out = torch.empty(scores.shape, dtype=torch.float32, device=scores.device)
        a.out_scores = out.data_ptr()
        a.out_scores_row_stride = out.stride(0)
        N.launch(a, torch.cuda.current_stream(scores.device).cuda_stream)
        return out


class ConditionalTemperatureLogitsWarper(FusedLogitsProcessor):
    """logit_processors.py:46-119: per-row temperature, first matching conditional."""

    def __init__(self, temperature: float, timing_temperature: float, mania_column_temperature: float,
                 taiko_hit_temperature: float, types_first: bool, beat_type_tokens: tuple[int, ...],
                 mania_type_tokens: tuple[int, ...], scroll_speed_tokens: tuple[int, ...]):
        conditionals = []
        if timing_temperature != temperature and len(beat_type_tokens) > 0:
            conditionals.append((timing_temperature, beat_type_tokens, 1))
        if mania_column_temperature != temperature and len(mania_type_tokens) > 0:
            conditionals.append((mania_column_temperature, mania_type_tokens, 3))
        if taiko_hit_temperature != temperature and len(scroll_speed_tokens) > 0:
            conditionals.append((taiko_hit_temperature, scroll_speed_tokens, 1))
        if not types_first:
            print("WARNING: Conditional temperature is not supported for types_first=False. Ignoring.")
            conditionals = []
        super().__init__(temperature=temperature, conditionals=conditionals, inplace=False)
        self.max_offset = max([o for _, _, o in self.conditionals], default=0)


class MonotonicTimeShiftLogitsProcessor(FusedLogitsProcessor):
    """logit_processors.py:173-237: full-scan monotonic time-shift mask, in place
    on float32 scores (returns the same tensor)."""

    def __init__(self, tokenizer, *, stateful_batch1: bool = False):
        if stateful_batch1:
            raise ValueError(
                "stateful_batch1 moved to optimized single inference; use "
                "osuT5.osuT5.inference.optimized.single.logits."
            )
        self.tokenizer = tokenizer
        self.time_shift_start, self.time_shift_end = _time_shift_range(tokenizer)
        self.stateful_batch1 = False
        super().__init__(time_shift_range=(self.time_shift_start, self.time_shift_end), sos_ids=_sos_ids(tokenizer))


class StatefulMonotonicTimeShiftLogitsProcessor(FusedLogitsProcessor):
    """optimized/single/logits.py:13-113: O(1)-per-step state kept on the device
    for every row (not only batch 1); re-derived by a full scan whenever the
    sequence does not grow by exactly one token."""

    def __init__(self, tokenizer, *, stateful_batch1: bool = True):
        self.tokenizer = tokenizer
        self.time_shift_start, self.time_shift_end = _time_shift_range(tokenizer)
        self.stateful_batch1 = stateful_batch1
        super().__init__(time_shift_range=(self.time_shift_start, self.time_shift_end), sos_ids=_sos_ids(tokenizer),
                         stateful_monotonic=stateful_batch1)


class LookbackBiasLogitsWarper(FusedLogitsProcessor):
    """logit_processors.py:122-170.  types_first=False: the lookback time
    shifts [event_start[TIME_SHIFT], encode(TIME_SHIFT, lookback_max_time / 10))
    are masked to -inf.  types_first=True: after a timed-event token the
    probability of the lookback range is moved to EOS (the range's first id
    carries the extra EOS mass, the rest of it is -inf), using the previous
    call's EOS probability, which the kernel keeps per row on the device.
    Returns a new tensor; ``scores`` is not modified."""

    def __init__(self, lookback_max_time: float, tokenizer, types_first: bool, device=None):
        spec = lookback_spec(lookback_max_time, tokenizer, types_first)
        self.types_first = types_first
        self.lookback_start = spec["start"]
        self.lookback_end = spec["end"]
        self.eos_ids = spec["eos_ids"]
        self.timed_tokens = spec["timed"]
        super().__init__(lookback=spec, inplace=False)


# ---------------------------------------------------------------- list builders
class FusedLogitsProcessorList(list):
    """A LogitsProcessorList-compatible list (``__call__(input_ids, scores)``)."""

    def __call__(self, input_ids, scores, **kwargs):
        for p in self:
            scores = p(input_ids, scores)
        return scores


def _list_type():
    try:
        from transformers import LogitsProcessorList

        return LogitsProcessorList
    except Exception:  # pragma: no cover
        return FusedLogitsProcessorList


def build_logits_processor_list(tokenizer, *, cfg_scale: float = 1.0, timeshift_bias: float = 0.0,
                                types_first: bool = False, temperature: float = 1.0,
                                timing_temperature: float | None = None,
                                mania_column_temperature: float | None = None,
                                taiko_hit_temperature: float | None = None, lookback_time: float = 0.0, device=None,
                                monotonic_processor_factory=MonotonicTimeShiftLogitsProcessor, top_k: int = 0,
                                top_p: float = 1.0, top_p_mode: str = "hf"):
    """logit_processors.py:240-307 as one fused processor.

    ``top_k`` / ``top_p`` optionally absorb the warpers that ``generate()``
    appends (pass ``top_k=0, top_p=1.0`` to generate() then).  The monotonic
    policy follows ``monotonic_processor_factory``: the stateful factory keeps
    per-row state on the device, the default re-scans input_ids each step.
    """
    if not isinstance(temperature, float) and not isinstance(temperature, int):
        raise ValueError(f"`temperature` (={temperature}) has to be a strictly positive float")
    timing_temperature = temperature if timing_temperature is None else timing_temperature
    mania_column_temperature = temperature if mania_column_temperature is None else mania_column_temperature
    taiko_hit_temperature = temperature if taiko_hit_temperature is None else taiko_hit_temperature
    conditionals = []
    if types_first:
        beat, mania, taiko = (get_beat_type_tokens(tokenizer), get_mania_type_tokens(tokenizer),
                              get_scroll_speed_tokens(tokenizer))
        if timing_temperature != temperature and beat:
            conditionals.append((timing_temperature, beat, 1))
        if mania_column_temperature != temperature and mania:
            conditionals.append((mania_column_temperature, mania, 3))
        if taiko_hit_temperature != temperature and taiko:
            conditionals.append((taiko_hit_temperature, taiko, 1))
    stateful = monotonic_processor_factory is StatefulMonotonicTimeShiftLogitsProcessor
    proc = FusedLogitsProcessor(
        cfg_scale=cfg_scale, time_shift_range=_time_shift_range(tokenizer), sos_ids=_sos_ids(tokenizer),
        stateful_monotonic=stateful, timeshift_bias=timeshift_bias, temperature=float(temperature),
        conditionals=conditionals, top_k=top_k, top_p=top_p, top_p_mode=top_p_mode,
        lookback=lookback_spec(lookback_time, tokenizer, types_first) if lookback_time > 0 else None)
    lst = _list_type()()
    lst.append(proc)
    return lst


def build_single_logits_processor_list(tokenizer, *, cfg_scale: float = 1.0, timeshift_bias: float = 0.0,
                                       types_first: bool = False, temperature: float = 1.0,
                                       timing_temperature: float | None = None,
                                       mania_column_temperature: float | None = None,
                                       taiko_hit_temperature: float | None = None, lookback_time: float = 0.0,
                                       device=None, stateful_monotonic: bool = True, top_k: int = 0,
                                       top_p: float = 1.0):
    """optimized/single/logits.py:116-147 as one fused processor."""
    factory = StatefulMonotonicTimeShiftLogitsProcessor if stateful_monotonic else MonotonicTimeShiftLogitsProcessor
    return build_logits_processor_list(
        tokenizer, cfg_scale=cfg_scale, timeshift_bias=timeshift_bias, types_first=types_first,
        temperature=temperature, timing_temperature=timing_temperature,
        mania_column_temperature=mania_column_temperature, taiko_hit_temperature=taiko_hit_temperature,
        lookback_time=lookback_time, device=device, monotonic_processor_factory=factory, top_k=top_k, top_p=top_p)

"""Sampler entry points: ``_sample`` and the stateful fused decode step.

``_sample`` keeps the signature and semantics of the fast decode loop's
sampler (osuT5/osuT5/inference/compiled_decode.py:1135-1158): greedy argmax,
or temperature -> top-k -> top-p (descending-cumsum, shifted-by-one rule) ->
draw, returning ``LongTensor[B, 1]``.  The draw is an inverse CDF in token-id
order from caller-supplied uniforms (``uniforms=``), or from ``torch.rand``
with ``generator=`` when none are given.

:class:`FusedSampler` is the whole per-step tail of the decode loops
(decode_loop.py:289-316, HF generation/utils.py:2762-2800) in one kernel:
processor chain, draw, pad-on-finished, EOS tracking and the monotonic /
grammar state updates, all on the device with no host synchronisation, so a
step can be captured in a CUDA graph next to the decoder replay.
"""

from __future__ import annotations

import ctypes
from dataclasses import dataclass
from typing import Sequence

import torch

from . import _native as N

_TORCH_DTYPES = {torch.float32: N.DTYPE_F32, torch.bfloat16: N.DTYPE_BF16, torch.float16: N.DTYPE_F16}


def dtype_code(t: torch.Tensor) -> int:
    try:
        return _TORCH_DTYPES[t.dtype]
    except KeyError:
        raise TypeError(f"logits dtype {t.dtype} is not supported (float32, bfloat16, float16)") from None


def _require_cuda(t: torch.Tensor, what: str) -> None:
    if not t.is_cuda:
        raise ValueError(f"{what} must be a CUDA tensor (the sampler has no CPU path)")


def _ids_code(t: torch.Tensor) -> int:
    if t.dtype == torch.int64:
        return N.IDS_I64
    if t.dtype == torch.int32:
        return N.IDS_I32
    raise TypeError(f"input_ids dtype {t.dtype} is not supported (int64, int32)")


def set_logits(args: N.MtrSamplerArgs, logits: torch.Tensor) -> None:
    if logits.dim() != 2 or logits.stride(1) != 1:
        raise ValueError("logits must be a 2-D tensor with unit stride along the vocabulary")
    args.logits = logits.data_ptr()
    args.logits_row_stride = logits.stride(0)
    args.logits_dtype = dtype_code(logits)
    args.vocab = logits.shape[1]


def set_input_ids(args: N.MtrSamplerArgs, input_ids: torch.Tensor | None) -> None:
    if input_ids is None:
        args.input_ids = None
        args.ids_len = 0
        args.ids_row_stride = 0
        return
    if input_ids.dim() != 2 or (input_ids.shape[1] > 0 and input_ids.stride(1) != 1):
        raise ValueError("input_ids must be [B, L] with unit stride along L")
    _require_cuda(input_ids, "input_ids")
    args.input_ids = input_ids.data_ptr() if input_ids.numel() else None
    args.ids_dtype = _ids_code(input_ids)
    args.ids_len = input_ids.shape[1]
    args.ids_row_stride = input_ids.stride(0) if input_ids.shape[1] else 0


def token_bitmap(tokens, vocab: int, device) -> torch.Tensor:
    """int32 [ceil(vocab / 32)] membership bitmap: bit t & 31 of word t >> 5."""
    words = torch.zeros((vocab + 31) // 32, dtype=torch.int64)
    for t in tokens:
        t = int(t)
        if 0 <= t < vocab:
            words[t >> 5] |= 1 << (t & 31)
    words = torch.where(words >= 2**31, words - 2**32, words)
    return words.to(torch.int32).to(device)


def _lmhead_args(hidden: torch.Tensor, weight: torch.Tensor, out: torch.Tensor, tile_n: int) -> N.MtrLmHeadArgs:
    for t, what in ((hidden, "hidden"), (weight, "weight"), (out, "logits")):
        _require_cuda(t, what)
        if t.dtype != torch.bfloat16 or t.dim() != 2 or t.stride(1) != 1:
            raise ValueError(f"{what} must be a 2-D bfloat16 CUDA tensor with unit column stride")
    if hidden.shape[1] != weight.shape[1]:
        raise ValueError(f"hidden d_model {hidden.shape[1]} != weight d_model {weight.shape[1]}")
    if out.shape[0] != hidden.shape[0] or out.shape[1] != weight.shape[0]:
        raise ValueError("logits must be [hidden rows, vocab]")
    a = N.new_lmhead_args()
    a.hidden, a.hidden_row_stride = hidden.data_ptr(), hidden.stride(0)
    a.weight, a.weight_row_stride = weight.data_ptr(), weight.stride(0)
    a.logits, a.logits_row_stride = out.data_ptr(), out.stride(0)
    a.rows, a.d_model, a.vocab = hidden.shape[0], hidden.shape[1], weight.shape[0]
    a.tile_n = int(tile_n)
    return a


def lm_head_logits(hidden: torch.Tensor, weight: torch.Tensor, out: torch.Tensor | None = None, *,
                   tile_n: int = 0) -> torch.Tensor:
    """``proj_out(hidden)`` (modeling_varwhisper.py:1583, an nn.Linear without
    bias in bf16) on the tcgen05 tensor cores: bf16 ``[R, V]`` logits with fp32
    accumulation.  ``hidden`` is ``[R, d]``, ``weight`` the Linear's ``[V, d]``."""
    if out is None:
        out = torch.empty((hidden.shape[0], weight.shape[0]), dtype=torch.bfloat16, device=hidden.device)
    a = _lmhead_args(hidden, weight, out, tile_n)
    N.lmhead_launch(a, torch.cuda.current_stream(hidden.device).cuda_stream)
    return out


def _uniforms(n: int, device, uniforms, generator) -> torch.Tensor:
    if uniforms is None:
        return torch.rand(n, device=device, generator=generator, dtype=torch.float32)
    if uniforms.dtype != torch.float32 or uniforms.numel() != n:
        raise ValueError(f"uniforms must be float32 with {n} elements")
    _require_cuda(uniforms, "uniforms")
    return uniforms.reshape(n).contiguous()


def _sample(logits: torch.Tensor, do_sample: bool, top_p: float, top_k: int, temperature: float, *,
            uniforms: torch.Tensor | None = None, generator: torch.Generator | None = None) -> torch.Tensor:
    """Fused replacement of compiled_decode._sample; returns LongTensor[B, 1]."""
    _require_cuda(logits, "logits")
    B, V = logits.shape
    args = N.new_args()
    set_logits(args, logits)
    args.num_rows = B
    out = torch.empty(B, dtype=torch.int64, device=logits.device)
    args.out_ids = out.data_ptr()
    if not do_sample:
        args.select_mode = N.SELECT_ARGMAX
    else:
        if not temperature > 0:
            raise ValueError("temperature must be > 0")
        args.select_mode = N.SELECT_SAMPLE
        args.temperature = float(temperature)
        if top_k > 0:
            args.top_k = int(min(top_k, V))
        if 0 < top_p < 1.0:
            args.top_p = float(top_p)
        args.top_p_mode = N.TOPP_SAMPLE_FN
        u = _uniforms(B, logits.device, uniforms, generator)
        args.uniforms = u.data_ptr()
    N.launch(args, torch.cuda.current_stream(logits.device).cuda_stream)
    return out.view(B, 1)


def sample_next_tokens(scores: torch.Tensor, do_sample: bool, *, uniforms: torch.Tensor | None = None,
                       generator: torch.Generator | None = None) -> torch.Tensor:
    """softmax + multinomial (or argmax) of already-processed scores, as the
    decode loops do after the processor list (decode_loop.py:296-301); [B]."""
    return _sample(scores, do_sample, 1.0, 0, 1.0, uniforms=uniforms, generator=generator).view(-1)


@dataclass
class GrammarTable:
    """Event-grammar mask: ``allow[c]`` has bit ``d`` set when a token of class
    ``d`` may follow a token of class ``c``; ``class_of[v]`` is the class of id v."""

    class_of: torch.Tensor  # [V] uint8
    allow: torch.Tensor     # [C] int32 (bit patterns)
    vocab_bits: torch.Tensor | None = None  # [C, ceil(V/32)] int32, built on first use

    def bits(self) -> torch.Tensor:
        """Per-class vocabulary bitmaps (bit v of row c = allow[c] >> class_of[v] & 1),
        which let the kernel mask 8 ids per lookup."""
        if self.vocab_bits is None:
            dev = self.class_of.device
            V, C = self.class_of.numel(), self.allow.numel()
            cls = self.class_of.to(torch.int64)
            allow = self.allow.to(torch.int64) & 0xFFFFFFFF
            ok = cls < C
            allowed = ((allow.view(C, 1) >> cls.clamp(max=31).view(1, V)) & 1).bool() & ok.view(1, V)
            words = (V + 31) // 32
            padded = torch.zeros((C, words * 32), dtype=torch.int64, device=dev)
            padded[:, :V] = allowed.to(torch.int64)
            w = (padded.view(C, words, 32) << torch.arange(32, device=dev, dtype=torch.int64)).sum(-1)
            w = torch.where(w >= 2**31, w - 2**32, w)
            self.vocab_bits = w.to(torch.int32).contiguous()
        return self.vocab_bits

    @classmethod
    def from_bool_table(cls, class_of, table, device) -> "GrammarTable":
        table = torch.as_tensor(table, dtype=torch.bool)
        c = table.shape[0]
        if table.shape != (c, c) or c > N.MAX_GRAMMAR_CLASSES:
            raise ValueError("transition table must be square with at most 32 classes")
        weights = (1 << torch.arange(c, dtype=torch.int64))
        allow = (table.to(torch.int64) * weights).sum(1)
        allow = torch.where(allow >= 2**31, allow - 2**32, allow).to(torch.int32)
        return cls(torch.as_tensor(class_of, dtype=torch.uint8).to(device), allow.to(device))


# Row status bits (include/mtr_sampler.h MTR_ROW_*): which ones mean the row's
# token is not a draw from its scores.
ROW_STATUS_NAMES = {N.ROW_NONFINITE: "nonfinite", N.ROW_ALL_MASKED: "all_masked", N.ROW_BAD_ID: "bad_id",
                    N.ROW_BAD_UNIFORM: "bad_uniform", N.ROW_SLOW_PATH: "slow_path",
                    N.ROW_TIE_AT_CUT: "tie_at_cut", N.ROW_COPY_TIMEOUT: "copy_timeout",
                    N.ROW_APPEND_SKIPPED: "append_skipped"}
PADDED_ROW_BITS = N.ROW_NONFINITE | N.ROW_ALL_MASKED | N.ROW_COPY_TIMEOUT


def row_status_report(status, ids=None, pad_id: int | None = None) -> dict:
    """Reads the per-row status words of a step: ``{name: [rows]}`` for every bit
    that is set, plus ``"padded"`` — the rows whose token is ``pad_id`` because
    the row could not be sampled (non-finite or fully masked scores, or a staged
    copy that never landed: that row and every later row of its CTA).  ``status``
    is a uint32 / int32 tensor or array of one word per row; with ``ids`` and
    ``pad_id`` the report also checks that those rows carry ``pad_id``."""
    import numpy as np

    st = np.asarray(status.cpu() if hasattr(status, "cpu") else status).astype(np.int64) & 0xFFFFFFFF
    rep = {name: np.nonzero(st & bit)[0].tolist() for bit, name in ROW_STATUS_NAMES.items() if (st & bit).any()}
    padded = np.nonzero(st & PADDED_ROW_BITS)[0]
    rep["padded"] = padded.tolist()
    if ids is not None and pad_id is not None:
        got = np.asarray(ids.cpu() if hasattr(ids, "cpu") else ids)
        bad = [int(r) for r in padded if int(got[r]) != int(pad_id)]
        if bad:
            raise ValueError(f"rows {bad[:8]} are marked unsampleable but do not carry pad_id {pad_id}")
    return rep


class FusedSampler:
    """Stateful fused decode step for a fixed batch of ``num_rows`` rows.

    Chain order: CFG -> monotonic time-shift mask -> timeshift bias -> grammar
    mask -> repetition / frequency / presence penalties -> temperature ->
    lookback bias -> top-k -> top-p -> draw.  Device state per row: last
    time-shift value (monotonic mask), previous token (grammar), unfinished
    flag, previous EOS probability (lookback bias).
    """

    def __init__(self, *, vocab_size: int, num_rows: int, device, cfg_scale: float = 1.0,
                 time_shift_range: tuple[int, int] | None = None, sos_ids: Sequence[int] = (),
                 timeshift_bias: float = 0.0, grammar: GrammarTable | None = None,
                 repetition_penalty: float = 1.0, frequency_penalty: float = 0.0, presence_penalty: float = 0.0,
                 penalty_start: int = 0, temperature: float = 1.0,
                 conditional_temperatures: Sequence[tuple[float, int, torch.Tensor]] = (),
                 column_temperatures: Sequence[tuple[int, int, float]] = (),
                 top_k: int = 0, top_p: float = 1.0, top_p_mode: str = "hf", do_sample: bool = True,
                 eos_token_ids: Sequence[int] = (), eos_ranges: Sequence[tuple[int, int]] = (),
                 pad_token_id: int = 0, track_finished: bool = False,
                 return_scores: bool = False, return_logprobs: bool = False, lookback: dict | None = None):
        self.device = torch.device(device)
        self.vocab_size = int(vocab_size)
        self.num_rows = int(num_rows)
        B, V = self.num_rows, self.vocab_size
        a = N.new_args()
        a.num_rows = B
        a.vocab = V
        a.cfg_enabled = int(cfg_scale > 1.0)
        a.cfg_scale = float(cfg_scale)
        a.cfg_second_offset = B
        self.mono_state = torch.full((B,), -1, dtype=torch.int32, device=self.device)
        if time_shift_range is not None:
            a.ts_start, a.ts_end = map(int, time_shift_range)
            a.mono_mode = N.MONO_STATE
            a.mono_state = self.mono_state.data_ptr()
            if len(sos_ids) > N.MAX_SOS_IDS:
                raise ValueError("at most 16 sos ids")
            a.n_sos = len(sos_ids)
            for i, t in enumerate(sos_ids):
                a.sos_ids[i] = int(t)
            a.flags |= N.FLAG_MONO_UPDATE_FROM_SAMPLE
        a.timeshift_bias = float(timeshift_bias)
        self.prev_token = torch.full((B,), -1, dtype=torch.int32, device=self.device)
        self.grammar = grammar
        if grammar is not None:
            a.grammar_class_of = grammar.class_of.data_ptr()
            a.grammar_allow = grammar.allow.data_ptr()
            a.grammar_vocab_bits = grammar.bits().data_ptr()
            a.grammar_n_classes = grammar.allow.numel()
            a.prev_token = self.prev_token.data_ptr()
            a.flags |= N.FLAG_GRAMMAR_UPDATE_FROM_SAMPLE
        a.repetition_penalty = float(repetition_penalty)
        a.frequency_penalty = float(frequency_penalty)
        a.presence_penalty = float(presence_penalty)
        a.penalty_start = int(penalty_start)
        a.temperature = float(temperature)
        self._keep = []
        if conditional_temperatures:
            a.temp_mode = N.TEMP_ROW_CONDITIONAL
            a.n_cond = len(conditional_temperatures)
            for i, (t, off, bits) in enumerate(conditional_temperatures):
                a.cond_temperature[i] = float(t)
                a.cond_offset[i] = int(off)
                bits = bits.to(self.device, torch.int32).contiguous()
                self._keep.append(bits)
                a.cond_token_bits[i] = bits.data_ptr()
        elif column_temperatures:
            a.temp_mode = N.TEMP_COLUMN_RANGES
            a.n_col_ranges = len(column_temperatures)
            for i, (s, e, t) in enumerate(column_temperatures):
                a.col_start[i], a.col_end[i], a.col_temperature[i] = int(s), int(e), float(t)
        a.select_mode = N.SELECT_SAMPLE if do_sample else N.SELECT_ARGMAX
        a.top_k = int(top_k)
        a.top_p = float(top_p)
        a.top_p_mode = {"hf": N.TOPP_HF, "sample_fn": N.TOPP_SAMPLE_FN}[top_p_mode]
        self.out_ids = torch.zeros(B, dtype=torch.int64, device=self.device)
        self.status = torch.zeros(B, dtype=torch.int32, device=self.device)
        a.out_ids = self.out_ids.data_ptr()
        a.out_status = self.status.data_ptr()
        self.scores = self.logprobs = None
        if return_scores:
            self.scores = torch.empty((B, V), dtype=torch.float32, device=self.device)
            a.out_scores = self.scores.data_ptr()
            a.out_scores_row_stride = V
        if return_logprobs:
            self.logprobs = torch.empty((B, V), dtype=torch.float32, device=self.device)
            a.out_logprobs = self.logprobs.data_ptr()
            a.out_logprobs_row_stride = V
        self.unfinished = torch.ones(B, dtype=torch.uint8, device=self.device)
        if track_finished:
            a.unfinished = self.unfinished.data_ptr()
        # cumulative since reset(): [0] live rows that emitted an EOS id, [1] rows finished
        self.stop_counts = torch.zeros(2, dtype=torch.int32, device=self.device)
        a.pad_id = int(pad_token_id)
        if len(eos_token_ids) > N.MAX_EOS_IDS or len(eos_ranges) > N.MAX_EOS_RANGES:
            raise ValueError("too many eos ids / ranges")
        a.n_eos = len(eos_token_ids)
        for i, t in enumerate(eos_token_ids):
            a.eos_ids[i] = int(t)
        a.n_eos_ranges = len(eos_ranges)
        for i, (s, e) in enumerate(eos_ranges):
            a.eos_range_start[i], a.eos_range_end[i] = int(s), int(e)
        # lookback bias (logit_processors.lookback_spec): previous EOS probability per row
        self.lb_state = torch.full((B,), float("nan"), dtype=torch.float32, device=self.device)
        self._keep_lb = None
        if lookback is not None:
            a.lookback_mode = int(lookback["mode"])
            a.lb_start, a.lb_end = int(lookback["start"]), int(lookback["end"])
            if a.lookback_mode == N.LOOKBACK_RENORM:
                eos = tuple(lookback["eos_ids"])
                if len(eos) > N.MAX_LB_EOS:
                    raise ValueError(f"at most {N.MAX_LB_EOS} lookback eos ids")
                a.n_lb_eos = len(eos)
                for i, t in enumerate(eos):
                    a.lb_eos_ids[i] = int(t)
                words = token_bitmap(lookback["timed"], V, self.device)
                self._keep_lb = words
                a.lb_timed_bits = words.data_ptr()
                a.lb_state = self.lb_state.data_ptr()
        self._base = a
        self._scan_next = time_shift_range is not None
        self._prev_from_ids_next = grammar is not None

    def reset(self) -> None:
        """Forget per-row state; the next step re-derives it from input_ids."""
        self.mono_state.fill_(-1)
        self.prev_token.fill_(-1)
        self.unfinished.fill_(1)
        self.stop_counts.zero_()
        self.lb_state.fill_(float("nan"))
        self._scan_next = self._base.mono_mode != N.MONO_OFF
        self._prev_from_ids_next = self.grammar is not None

    def _args(self, logits: torch.Tensor, input_ids, uniforms, id_buffer=None, cur_len=None) -> N.MtrSamplerArgs:
        a = N.MtrSamplerArgs()
        ctypes.pointer(a)[0] = self._base
        set_logits(a, logits)
        if a.vocab != self.vocab_size:
            raise ValueError(f"logits vocabulary {a.vocab} != {self.vocab_size}")
        rows = logits.shape[0]
        if rows != (2 * self.num_rows if a.cfg_enabled else self.num_rows):
            raise ValueError(f"expected {2 * self.num_rows if a.cfg_enabled else self.num_rows} logits rows, got {rows}")
        set_input_ids(a, input_ids)
        if a.lookback_mode == N.LOOKBACK_RENORM and input_ids is None:
            raise ValueError("the lookback bias reads the last input id: pass input_ids every step")
        if input_ids is not None and input_ids.shape[0] != self.num_rows:
            raise ValueError("input_ids must have one row per output row")
        if self._scan_next and input_ids is not None:
            a.mono_mode = N.MONO_SCAN
        if self._prev_from_ids_next and input_ids is not None and input_ids.shape[1] > 0:
            a.flags |= N.FLAG_GRAMMAR_PREV_FROM_IDS
        if a.select_mode == N.SELECT_SAMPLE:
            a.uniforms = uniforms.data_ptr()
        if a.select_mode != N.SELECT_NONE:
            a.stop_counts = self.stop_counts.data_ptr()
        if id_buffer is not None:
            _require_cuda(id_buffer, "id_buffer")
            if id_buffer.dtype != torch.int64 or id_buffer.dim() != 2 or id_buffer.shape[0] != self.num_rows \
                    or id_buffer.stride(1) != 1:
                raise ValueError("id_buffer must be an int64 [num_rows, S] tensor with unit column stride")
            a.id_buffer = id_buffer.data_ptr()
            a.id_buffer_row_stride = id_buffer.stride(0)
            if isinstance(cur_len, torch.Tensor):
                _require_cuda(cur_len, "cur_len")
                if cur_len.dtype != torch.int32 or cur_len.numel() != 1:
                    raise ValueError("a device cur_len must be a one-element int32 tensor")
                a.cur_len_dev = cur_len.data_ptr()
            else:
                if cur_len is None or not 0 <= int(cur_len) < id_buffer.shape[1]:
                    raise ValueError(f"cur_len {cur_len} outside the id buffer's {id_buffer.shape[1]} columns")
                a.cur_len = int(cur_len)
        return a

    def launch_info(self, logits: torch.Tensor, input_ids: torch.Tensor | None = None,
                    uniforms: torch.Tensor | None = None) -> N.MtrLaunchInfo:
        """Kernel and geometry the next ``step`` with these tensors would launch
        (``info.kernel``: 0 row-per-CTA, 1 row-per-warp)."""
        if self._base.select_mode == N.SELECT_SAMPLE and uniforms is None:
            uniforms = torch.zeros(self.num_rows, dtype=torch.float32, device=logits.device)
        return N.query_args(self._args(logits, input_ids, uniforms))

    def step(self, logits: torch.Tensor, input_ids: torch.Tensor | None = None,
             uniforms: torch.Tensor | None = None, generator: torch.Generator | None = None, *,
             id_buffer: torch.Tensor | None = None, cur_len=None) -> torch.Tensor:
        """Process one decoder step's logits ([B, V], or [2B, V] with CFG) and
        return the next tokens ``LongTensor[B]`` (a view of an internal buffer
        that the next step overwrites).

        With ``id_buffer`` (int64 [B, S]) the emitted tokens are also written to
        column ``cur_len`` -- an int, or a one-element int32 CUDA tensor that a
        captured graph advances between replays (compiled_decode.py:1072's
        ``id_buffer[:, cur_len] = next_token``).  ``stop_counts`` then tells the
        loop when to stop without a per-step host sync."""
        _require_cuda(logits, "logits")
        if self._base.select_mode == N.SELECT_SAMPLE:
            uniforms = _uniforms(self.num_rows, logits.device, uniforms, generator)
        a = self._args(logits, input_ids, uniforms, id_buffer, cur_len)
        N.launch(a, torch.cuda.current_stream(logits.device).cuda_stream)
        if input_ids is not None:
            self._scan_next = False
            self._prev_from_ids_next = False
        self._last_uniforms = uniforms  # keep alive until the kernel has consumed them
        return self.out_ids

    def step_hidden(self, hidden: torch.Tensor, weight: torch.Tensor, input_ids: torch.Tensor | None = None,
                    uniforms: torch.Tensor | None = None, generator: torch.Generator | None = None, *,
                    id_buffer: torch.Tensor | None = None, cur_len=None, tile_n: int = 0) -> torch.Tensor:
        """The decoder's last hidden states to the next tokens: the tensor-core
        output projection (``lm_head_logits``) writes bf16 logits that this
        step's fused kernel reads, launched as its programmatic dependent.
        ``hidden`` has the logits' rows ([2B, d] with CFG).  The logits stay
        readable in ``self.lm_logits`` until the next call."""
        _require_cuda(hidden, "hidden")
        rows = hidden.shape[0]
        if rows != (2 * self.num_rows if self._base.cfg_enabled else self.num_rows):
            raise ValueError(f"hidden has {rows} rows")
        if weight.shape[0] != self.vocab_size:
            raise ValueError(f"weight vocabulary {weight.shape[0]} != {self.vocab_size}")
        buf = getattr(self, "lm_logits", None)
        if buf is None or buf.shape != (rows, self.vocab_size) or buf.device != hidden.device:
            buf = torch.empty((rows, self.vocab_size), dtype=torch.bfloat16, device=hidden.device)
            self.lm_logits = buf
        lm = _lmhead_args(hidden, weight, buf, tile_n)
        if self._base.select_mode == N.SELECT_SAMPLE:
            uniforms = _uniforms(self.num_rows, hidden.device, uniforms, generator)
        a = self._args(buf, input_ids, uniforms, id_buffer, cur_len)
        N.lmhead_sample_launch(lm, a, torch.cuda.current_stream(hidden.device).cuda_stream)
        if input_ids is not None:
            self._scan_next = False
            self._prev_from_ids_next = False
        self._last_uniforms = uniforms
        return self.out_ids

    def any_eos(self) -> bool:
        """A live row has emitted an EOS id since reset() (compiled_decode.py:1078's
        stop test; one host sync)."""
        return bool(self.stop_counts[0].item() > 0)

    def all_finished(self) -> bool:
        """Every row has finished (the HF loop's stop test; needs track_finished; one host sync)."""
        return bool(self.stop_counts[1].item() >= self.num_rows)

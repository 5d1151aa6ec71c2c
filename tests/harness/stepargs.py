"""Marshal one decode step into ``MtrSamplerArgs``.

``fill_args`` is memory-agnostic: ``addr`` maps each named array of a
:class:`~mapperatorinator_b200.workloads.StepInputs` (or an output buffer) to
an address.  :class:`DeviceStep` uses it with CUDA tensors for the library;
the CPU oracle uses it with numpy arrays, so both sides read the same
parameters from the same struct.
"""

from __future__ import annotations

from typing import Callable

import numpy as np

from mapperatorinator_b200 import _native as N
from .workloads import StepInputs

_DTYPE_CODES = {"f32": N.DTYPE_F32, "bf16": N.DTYPE_BF16, "f16": N.DTYPE_F16}


def fill_args(args: N.MtrSamplerArgs, s: StepInputs, addr: Callable[[str], int],
              *, with_outputs: bool = True) -> N.MtrSamplerArgs:
    """Populate ``args`` (already initialised) from ``s``; ``addr(name)`` gives
    the address of array ``name`` (0 when absent)."""
    B, V = s.num_rows, s.vocab
    args.logits = addr("logits")
    args.logits_row_stride = V
    args.logits_dtype = _DTYPE_CODES[s.dtype]
    args.num_rows = B
    args.vocab = V
    args.cfg_enabled = int(s.cfg_scale > 1.0)
    args.cfg_scale = float(s.cfg_scale)
    args.cfg_second_offset = B
    args.flags = int(s.flags)
    if s.input_ids is not None:
        args.input_ids = addr("input_ids")
        args.ids_row_stride = int(s.input_ids.shape[1])
        args.ids_len = int(s.input_ids.shape[1])
        args.ids_dtype = N.IDS_I32 if s.input_ids.dtype == np.int32 else N.IDS_I64
    args.penalty_start = int(s.penalty_start)
    args.mono_mode = int(s.mono_mode)
    args.ts_start = int(s.ts_start)
    args.ts_end = int(s.ts_end)
    if len(s.sos_ids) > N.MAX_SOS_IDS:
        raise ValueError("too many sos ids")
    args.n_sos = len(s.sos_ids)
    for i, t in enumerate(s.sos_ids):
        args.sos_ids[i] = int(t)
    args.mono_state = addr("mono_state")
    args.timeshift_bias = float(s.timeshift_bias)
    if s.grammar_class_of is not None:
        args.grammar_class_of = addr("grammar_class_of")
        args.grammar_allow = addr("grammar_allow")
        args.grammar_vocab_bits = addr("grammar_vocab_bits")
        args.grammar_n_classes = int(len(s.grammar_allow))
    args.prev_token = addr("prev_token")
    args.repetition_penalty = float(s.repetition_penalty)
    args.frequency_penalty = float(s.frequency_penalty)
    args.presence_penalty = float(s.presence_penalty)
    args.temp_mode = int(s.temp_mode)
    args.temperature = float(s.temperature)
    args.n_cond = len(s.cond)
    for i, (t, off, _bits) in enumerate(s.cond):
        args.cond_temperature[i] = float(t)
        args.cond_offset[i] = int(off)
        args.cond_token_bits[i] = addr(f"cond_bits{i}")
    args.n_col_ranges = len(s.col_ranges)
    for i, (a, b, t) in enumerate(s.col_ranges):
        args.col_start[i] = int(a)
        args.col_end[i] = int(b)
        args.col_temperature[i] = float(t)
    args.select_mode = int(s.select_mode)
    args.top_k = int(s.top_k)
    args.top_p = float(s.top_p)
    args.top_p_mode = int(s.top_p_mode)
    args.uniforms = addr("uniforms")
    if with_outputs:
        args.out_ids = addr("out_ids")
        args.out_status = addr("out_status")
        if s.want_scores:
            args.out_scores = addr("out_scores")
            args.out_scores_row_stride = V
        if s.want_logprobs:
            args.out_logprobs = addr("out_logprobs")
            args.out_logprobs_row_stride = V
    args.unfinished = addr("unfinished")
    args.pad_id = int(s.pad_id)
    args.n_eos = len(s.eos_ids)
    for i, t in enumerate(s.eos_ids):
        args.eos_ids[i] = int(t)
    args.n_eos_ranges = len(s.eos_ranges)
    for i, (a, b) in enumerate(s.eos_ranges):
        args.eos_range_start[i] = int(a)
        args.eos_range_end[i] = int(b)
    args.lookback_mode = int(s.lookback_mode)
    args.lb_start = int(s.lb_start)
    args.lb_end = int(s.lb_end)
    if len(s.lb_eos_ids) > N.MAX_LB_EOS:
        raise ValueError("too many lookback eos ids")
    args.n_lb_eos = len(s.lb_eos_ids)
    for i, t in enumerate(s.lb_eos_ids):
        args.lb_eos_ids[i] = int(t)
    args.lb_timed_bits = addr("lb_timed_bits")
    args.lb_state = addr("lb_state")
    if s.id_buffer is not None:
        args.id_buffer = addr("id_buffer")
        args.id_buffer_row_stride = int(s.id_buffer.shape[1])
    args.cur_len = int(s.cur_len)
    args.cur_len_dev = addr("cur_len_dev")
    args.stop_counts = addr("stop_counts")
    return args


def grammar_vocab_bits(class_of: np.ndarray, allow: np.ndarray) -> np.ndarray:
    """[C, ceil(V/32)] uint32: bit v of row c = (allow[c] >> class_of[v]) & 1."""
    class_of = np.asarray(class_of, dtype=np.int64)
    allow = np.asarray(allow, dtype=np.uint64)
    V, C = len(class_of), len(allow)
    ok = class_of < C
    allowed = np.zeros((C, V), dtype=bool)
    for c in range(C):
        allowed[c] = ok & (((allow[c] >> np.minimum(class_of, 63).astype(np.uint64)) & np.uint64(1)) == 1)
    words = (V + 31) // 32
    padded = np.zeros((C, words * 32), dtype=bool)
    padded[:, :V] = allowed
    weights = (np.uint64(1) << np.arange(32, dtype=np.uint64))
    return (padded.reshape(C, words, 32).astype(np.uint64) * weights).sum(-1).astype(np.uint32)


def host_arrays(s: StepInputs) -> dict:
    """Named host arrays of a step (inputs, mutable state and outputs)."""
    B, V = s.num_rows, s.vocab
    arr = {"logits": np.ascontiguousarray(s.logits)}
    if s.input_ids is not None:
        arr["input_ids"] = np.ascontiguousarray(s.input_ids)
    if s.mono_state is not None:
        arr["mono_state"] = np.array(s.mono_state, dtype=np.int32, copy=True)
    if s.grammar_class_of is not None:
        arr["grammar_class_of"] = np.ascontiguousarray(s.grammar_class_of, dtype=np.uint8)
        arr["grammar_allow"] = np.ascontiguousarray(s.grammar_allow, dtype=np.uint32)
        if s.grammar_bits:
            arr["grammar_vocab_bits"] = grammar_vocab_bits(s.grammar_class_of, s.grammar_allow)
    if s.prev_token is not None:
        arr["prev_token"] = np.array(s.prev_token, dtype=np.int32, copy=True)
    for i, (_t, _off, bits) in enumerate(s.cond):
        arr[f"cond_bits{i}"] = np.ascontiguousarray(bits, dtype=np.uint32)
    if s.uniforms is not None:
        arr["uniforms"] = np.ascontiguousarray(s.uniforms, dtype=np.float32)
    if s.unfinished is not None:
        arr["unfinished"] = np.array(s.unfinished, dtype=np.uint8, copy=True)
    if s.lb_timed_bits is not None:
        arr["lb_timed_bits"] = np.ascontiguousarray(s.lb_timed_bits, dtype=np.uint32)
    if s.lb_state is not None:
        arr["lb_state"] = np.array(s.lb_state, dtype=np.float32, copy=True)
    if s.id_buffer is not None:
        arr["id_buffer"] = np.array(s.id_buffer, dtype=np.int64, copy=True)
    if s.cur_len_dev is not None:
        arr["cur_len_dev"] = np.array(s.cur_len_dev, dtype=np.int32, copy=True).reshape(1)
    if s.stop_counts is not None:
        arr["stop_counts"] = np.array(s.stop_counts, dtype=np.uint32, copy=True).reshape(2)
    arr["out_ids"] = np.full(B, -7, dtype=np.int64)
    arr["out_status"] = np.full(B, 0xFFFFFFFF, dtype=np.uint32)
    if s.want_scores:
        arr["out_scores"] = np.full((B, V), np.float32(123.0), dtype=np.float32)
    if s.want_logprobs:
        arr["out_logprobs"] = np.full((B, V), np.float32(123.0), dtype=np.float32)
    return arr


STATE_KEYS = ("out_ids", "out_status", "out_scores", "out_logprobs", "mono_state", "prev_token", "unfinished",
              "lb_state", "id_buffer", "stop_counts")


class DeviceStep:
    """A step whose arrays live on a CUDA device, ready to launch."""

    def __init__(self, s: StepInputs, device="cuda"):
        import torch

        self.step = s
        self.device = torch.device(device)
        self.tensors = {}
        for name, a in host_arrays(s).items():
            t = torch.from_numpy(np.ascontiguousarray(a))
            if a.dtype == np.uint32:
                t = torch.from_numpy(a.view(np.int32))
            elif a.dtype == np.uint16:
                t = torch.from_numpy(a.view(np.int16))
            self.tensors[name] = t.to(self.device)
        self.args = N.new_args()
        fill_args(self.args, s, self._addr)

    def _addr(self, name: str) -> int:
        t = self.tensors.get(name)
        return 0 if t is None else int(t.data_ptr())

    def launch(self, stream=None) -> None:
        import torch

        if stream is None:
            stream = torch.cuda.current_stream(self.device)
        N.launch(self.args, int(stream.cuda_stream))

    def results(self) -> dict:
        out = {}
        for k in STATE_KEYS:
            t = self.tensors.get(k)
            if t is None:
                continue
            a = t.cpu().numpy()
            if k in ("out_status", "stop_counts"):
                a = a.view(np.uint32)
            out[k] = a
        return out

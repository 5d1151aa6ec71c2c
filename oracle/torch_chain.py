"""PyTorch CPU restatement of the reference decode-step chain.

TEST INFRASTRUCTURE / CPU BASELINE ONLY (tests/, bench.py's reference arm and
CPU-baseline leg).  It performs the same torch operations, in the same order,
as the reference processors it restates, so it runs at the reference's CPU
speed and reproduces its processed scores bit for bit:

  ClassifierFreeGuidanceLogitsProcessor  transformers generation/logits_process.py:2160-2174
  MonotonicTimeShiftLogitsProcessor      osuT5/osuT5/inference/logit_processors.py:190-229
  TimeshiftBias                          logit_processors.py:35-43
  RepetitionPenaltyLogitsProcessor       transformers generation/logits_process.py:407-413
  TemperatureLogitsWarper                transformers generation/logits_process.py:297-301
  ConditionalTemperatureLogitsWarper     logit_processors.py:82-117 (batched form)
  TopKLogitsWarper / TopPLogitsWarper    transformers generation/logits_process.py:581-588 / 521-535
  softmax + torch.multinomial            osuT5/osuT5/inference/optimized/single/decode_loop.py:296-301

The event-grammar mask and the frequency / presence penalties have no
reference implementation; they are written with the same style of torch ops.
"""

from __future__ import annotations

from dataclasses import dataclass, field

import torch


@dataclass
class ChainParams:
    cfg_scale: float = 1.0
    ts_range: tuple | None = None
    sos_ids: tuple = ()
    timeshift_bias: float = 0.0
    grammar_class_of: torch.Tensor | None = None   # [V] long
    grammar_table: torch.Tensor | None = None      # [C, C] bool
    repetition_penalty: float = 1.0
    frequency_penalty: float = 0.0
    presence_penalty: float = 0.0
    temperature: float = 1.0
    column_temperatures: list = field(default_factory=list)  # [(start, end, T)]
    top_k: int = 0
    top_p: float = 1.0


def cfg(scores: torch.Tensor, scale: float) -> torch.Tensor:
    b = scores.shape[0] // 2
    cond, uncond = scores.split(b, dim=0)
    return uncond + (cond - uncond) * scale


def monotonic_full_scan(input_ids, scores, ts_start, ts_end, sos_ids):
    batch_size, seq_len = input_ids.shape
    is_ts = (input_ids >= ts_start) & (input_ids < ts_end)
    is_sos = (input_ids.unsqueeze(-1) == torch.tensor(sos_ids, dtype=input_ids.dtype)).any(dim=-1)
    idx = torch.arange(seq_len).expand(batch_size, -1)
    last_ts = torch.max(torch.where(is_ts, idx, -1), dim=1).values
    last_sos = torch.max(torch.where(is_sos, idx, -1), dim=1).values
    last_val = torch.where(last_ts != -1, input_ids[torch.arange(batch_size), last_ts] - ts_start, 0)
    apply = (last_ts != -1) & (last_ts > last_sos)
    ts_vocab = torch.arange(ts_start, ts_end)
    invalid = ts_vocab.unsqueeze(0) < (ts_start + last_val).unsqueeze(1)
    mask = torch.full_like(scores, False, dtype=torch.bool)
    mask[:, ts_start:ts_end] = invalid
    scores[apply] = scores[apply].masked_fill(mask[apply], -torch.inf)
    return scores


def grammar_mask(scores, prev, class_of, table):
    allowed = table[class_of[prev]][:, class_of]  # [B, V]
    return scores.masked_fill(~allowed, -torch.inf)


def repetition(scores, input_ids, penalty):
    score = torch.gather(scores, 1, input_ids)
    score = torch.where(score < 0, score * penalty, score / penalty)
    return scores.scatter(1, input_ids, score)


def frequency_presence(scores, input_ids, freq, pres):
    counts = torch.zeros_like(scores).scatter_add_(1, input_ids, torch.ones_like(input_ids, dtype=scores.dtype))
    if freq:
        scores = scores - freq * counts
    if pres:
        scores = scores - pres * (counts > 0).to(scores.dtype)
    return scores


def top_k(scores, k):
    k = min(k, scores.size(-1))
    remove = scores < torch.topk(scores, k)[0][..., -1, None]
    return scores.masked_fill(remove, -float("inf"))


def top_p(scores, p):
    sorted_logits, sorted_idx = torch.sort(scores, descending=False)
    cum = sorted_logits.softmax(dim=-1).cumsum(dim=-1)
    remove_sorted = cum <= (1 - p)
    remove_sorted[..., -1:] = 0
    remove = remove_sorted.scatter(1, sorted_idx, remove_sorted)
    return scores.masked_fill(remove, -float("inf"))


def processed_scores(logits: torch.Tensor, input_ids: torch.Tensor | None, prm: ChainParams,
                     prev_tokens: torch.Tensor | None = None) -> torch.Tensor:
    """Everything before the draw, as float32 [B, V] (CPU tensors)."""
    scores = logits.to(torch.float32, copy=True)
    if prm.cfg_scale > 1.0:
        scores = cfg(scores, prm.cfg_scale)
    if prm.ts_range is not None and input_ids is not None:
        scores = monotonic_full_scan(input_ids, scores, prm.ts_range[0], prm.ts_range[1], prm.sos_ids)
    if prm.timeshift_bias != 0 and prm.ts_range is not None:
        scores = scores.clone()
        scores[:, prm.ts_range[0]:prm.ts_range[1]] += prm.timeshift_bias
    if prm.grammar_table is not None and prev_tokens is not None:
        scores = grammar_mask(scores, prev_tokens, prm.grammar_class_of, prm.grammar_table)
    if prm.repetition_penalty != 1.0 and input_ids is not None:
        scores = repetition(scores, input_ids, prm.repetition_penalty)
    if (prm.frequency_penalty or prm.presence_penalty) and input_ids is not None:
        scores = frequency_presence(scores, input_ids, prm.frequency_penalty, prm.presence_penalty)
    if prm.column_temperatures:
        temps = torch.full((scores.shape[1],), prm.temperature, dtype=scores.dtype)
        for s, e, t in reversed(prm.column_temperatures):
            temps[s:e] = t
        scores = scores / temps
    elif prm.temperature != 1.0:
        scores = scores / prm.temperature
    if prm.top_k:
        scores = top_k(scores, prm.top_k)
    if prm.top_p < 1.0:
        scores = top_p(scores, prm.top_p)
    return scores


def sample_step(logits, input_ids, prm: ChainParams, prev_tokens=None, generator=None) -> torch.Tensor:
    scores = processed_scores(logits, input_ids, prm, prev_tokens)
    probs = torch.nn.functional.softmax(scores, dim=-1)
    return torch.multinomial(probs, num_samples=1, generator=generator).squeeze(1)

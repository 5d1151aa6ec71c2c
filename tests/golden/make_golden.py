"""Generate the golden fixtures that pin the CPU oracle to the reference.

Run where the Mapperatorinator sources are available -- MTR_REFERENCE_DIR,
or the copy that baseline/install_reference.sh places in baseline/_ref --
with the transformers package installed:

    MTR_REFERENCE_DIR=<reference checkout> python tests/golden/make_golden.py

It imports the reference's own processor modules by path -- the package
``__init__`` files pull in dependencies that are not needed here, so the
package roots are stubbed, as the reference's own tests do
(tests/test_logit_processors.py:11-29) -- together with the installed HF
warpers, runs them on seeded inputs and writes ``reference_chain.npz`` next
to this script.  ``_sample`` (osuT5/osuT5/inference/compiled_decode.py:1135)
is executed from the reference source with ``torch.multinomial`` observed, so
its keep set is recorded without changing its code.

The fixtures hold inputs and reference outputs only; the test suite never
reads the reference checkout.
"""

from __future__ import annotations

import json
import os
import sys
from pathlib import Path

import numpy as np
import torch

ROOT = Path(__file__).resolve().parents[2]
OUT = Path(__file__).resolve().parent / "reference_chain.npz"
sys.path.insert(0, str(ROOT))
from oracle.reference_loader import load_reference as _load_reference  # noqa: E402
from oracle.reference_loader import make_tokenizer  # noqa: E402


def reference_dir() -> Path:
    """MTR_REFERENCE_DIR, else the copy placed by baseline/install_reference.sh."""
    env = os.environ.get("MTR_REFERENCE_DIR")
    ref = Path(env) if env else ROOT / "baseline" / "_ref"
    if not (ref / "osuT5").exists():
        raise SystemExit(f"reference sources not found at {ref}: set MTR_REFERENCE_DIR or run "
                         "baseline/install_reference.sh")
    return ref


def load_reference():
    return _load_reference(reference_dir())



class _TorchObserver:
    """Forwards to torch; records the probabilities handed to multinomial."""

    def __init__(self):
        self.probs = None

    def __getattr__(self, name):
        return getattr(torch, name)

    def multinomial(self, probs, num_samples):
        self.probs = probs.clone()
        return torch.multinomial(probs, num_samples)


def run_sample(fn_module, logits, do_sample, top_p, top_k, temperature):
    obs = _TorchObserver()
    ns = {"torch": obs, "F": torch.nn.functional}
    exec(compile(fn_module, "compiled_decode._sample", "exec"), ns)
    out = ns["_sample"](logits.clone(), do_sample, top_p, top_k, temperature)
    return out, obs.probs


def hf_warpers(scores, top_k, top_p):
    from transformers import TopKLogitsWarper, TopPLogitsWarper

    if top_k:
        scores = TopKLogitsWarper(top_k=top_k, min_tokens_to_keep=1)(None, scores)
    if top_p < 1.0:
        scores = TopPLogitsWarper(top_p=top_p, min_tokens_to_keep=1)(None, scores)
    return scores


def main() -> None:
    ev, lp, sl, sample_mod = load_reference()
    g = torch.Generator().manual_seed(20240611)
    fixtures: dict[str, np.ndarray] = {}
    meta: dict[str, dict] = {}

    def put(name, **arrays):
        for k, v in arrays.items():
            fixtures[f"{name}.{k}"] = np.asarray(v)

    # ---- the reference's own test vectors (tests/test_logit_processors.py) ----
    tok64 = make_tokenizer(ev, ts=(10, 20), sos=1)
    mono = lp.MonotonicTimeShiftLogitsProcessor(tok64)
    ids = torch.tensor([[1, 12, 5, 15, 3]])
    sc = torch.arange(64, dtype=torch.float32).reshape(1, 64) / 10
    put("ref_mono_vector", input_ids=ids.numpy(), scores=sc.numpy(), out=mono(ids.clone(), sc.clone()).numpy())
    meta["ref_mono_vector"] = {"ts": [10, 20], "sos": [1]}

    ct = lp.ConditionalTemperatureLogitsWarper(1.0, 2.0, 4.0, 8.0, True, (10, 11), (20,), (30,))
    ids = torch.tensor([[0, 0, 10], [20, 0, 0], [0, 0, 30], [20, 0, 10], [0, 0, 0]])
    sc = torch.full((5, 4), 8.0)
    put("ref_condtemp_batch", input_ids=ids.numpy(), scores=sc.numpy(), out=ct(ids, sc).numpy())
    meta["ref_condtemp_batch"] = {"temps": [1.0, 2.0, 4.0, 8.0], "beat": [10, 11], "mania": [20], "taiko": [30]}

    # stateful monotonic over growing prefixes and random trials
    seq = torch.tensor([[1, 12, 5, 11, 7, 15, 3, 1, 14, 9]])
    st = sl.MonotonicTimeShiftLogitsProcessor(tok64)
    outs = []
    for n in range(1, seq.shape[1] + 1):
        s0 = torch.arange(64, dtype=torch.float32).reshape(1, 64) / 10
        outs.append(st(seq[:, :n].clone(), s0.clone()).numpy()[0])
    put("ref_stateful_prefixes", input_ids=seq.numpy(), out=np.stack(outs))
    for bsz in (1, 2, 5):
        gen = torch.Generator().manual_seed(34567 + bsz)
        trial_ids, trial_scores, trial_out, lens = [], [], [], []
        for _ in range(32):
            L = int(torch.randint(1, 48, (), generator=gen).item())
            ii = torch.randint(0, 30, (bsz, L), generator=gen)
            ss = torch.randn((bsz, 64), generator=gen)
            trial_ids.append(np.pad(ii.numpy(), ((0, 0), (0, 48 - L)), constant_values=-1))
            trial_scores.append(ss.numpy())
            trial_out.append(mono(ii.clone(), ss.clone()).numpy())
            lens.append(L)
        put(f"ref_random_b{bsz}", input_ids=np.stack(trial_ids), scores=np.stack(trial_scores),
            out=np.stack(trial_out), lens=np.array(lens))

    # ---- full chains: build_logits_processor_list + HF warpers / _sample ----
    def chain_case(name, *, B, V, L, cfg, ts, sos, ctx_sos, types_first, temps, bias, top_k, top_p,
                   dtype="f32", extra=None, spikes=0, sigma=1.5, history_fn=None):
        tok = make_tokenizer(ev, ts=ts, sos=sos, context_sos=ctx_sos, extra=extra)
        R = 2 * B if cfg > 1.0 else B
        x = torch.randn((R, V), generator=g) * sigma
        if spikes:
            sid = torch.randperm(V, generator=g)[:spikes]
            x[:, sid] = 8.0
        if dtype == "bf16":
            x = x.to(torch.bfloat16).to(torch.float32)
        ids = history_fn(B, L) if history_fn else torch.randint(0, V, (B, L), generator=g)
        procs = lp.build_logits_processor_list(
            tok, cfg_scale=cfg, timeshift_bias=bias, types_first=types_first, temperature=temps[0],
            timing_temperature=temps[1], mania_column_temperature=temps[2], taiko_hit_temperature=temps[3])
        processed = procs(ids.clone(), x.clone())
        final = hf_warpers(processed.clone(), top_k, top_p)
        _, probs = run_sample(sample_mod, processed.clone(), True, top_p, top_k, 1.0)
        greedy, _ = run_sample(sample_mod, processed.clone(), False, top_p, top_k, 1.0)
        put(name, logits=x.numpy(), input_ids=ids.numpy(), processed=processed.numpy(), final_hf=final.numpy(),
            sample_fn_probs=probs.numpy(), greedy=greedy.numpy())
        meta[name] = {"B": B, "V": V, "cfg": cfg, "ts": list(ts), "sos": [sos] + list((ctx_sos or {}).values()),
                      "types_first": types_first, "temps": list(temps), "bias": bias, "top_k": top_k,
                      "top_p": top_p, "dtype": dtype,
                      "extra": {k: list(v) for k, v in (extra or {}).items()}}

    def ts_heavy_history(B, L, V=256, ts=(16, 116), sos=(1, 3)):
        h = torch.randint(120, V, (B, L), generator=g)
        for b in range(B):
            k = int(torch.randint(0, 4, (), generator=g))
            pos = torch.randperm(L, generator=g)[:6]
            h[b, pos] = torch.randint(ts[0], ts[1], (6,), generator=g)
            if k == 0:
                h[b, -1] = sos[0]
            if k == 1:
                h[b, int(pos.max()) - 1 if int(pos.max()) > 0 else 0] = sos[1]
        return h

    ctx = {ev.ContextType.TIMING: 3}
    chain_case("chain_cfg_mono_temp", B=4, V=256, L=24, cfg=1.5, ts=(16, 116), sos=1, ctx_sos=ctx, types_first=False,
               temps=(0.9, None, None, None), bias=0.0, top_k=0, top_p=0.9, history_fn=ts_heavy_history)
    extra = {"BEAT": (130, 131), "MEASURE": (131, 132), "TIMING_POINT": (132, 133), "CIRCLE": (140, 141),
             "HOLD_NOTE": (141, 142), "HOLD_NOTE_END": (142, 143), "SCROLL_SPEED": (150, 170)}

    def cond_history(B, L):
        h = torch.randint(0, 256, (B, L), generator=g)
        picks = [130, 131, 132, 140, 141, 142, 155, 169, 7, 200]
        for b in range(B):
            h[b, -1] = picks[b % len(picks)]
            h[b, -3] = picks[(3 * b + 1) % len(picks)]
        return h

    chain_case("chain_condtemp", B=10, V=256, L=12, cfg=1.0, ts=(16, 116), sos=1, ctx_sos=None, types_first=True,
               temps=(1.0, 0.7, 1.3, 1.1), bias=0.0, top_k=10, top_p=0.8, extra=extra, history_fn=cond_history)
    chain_case("chain_condtemp_b1", B=1, V=256, L=12, cfg=1.0, ts=(16, 116), sos=1, ctx_sos=None, types_first=True,
               temps=(1.0, 0.7, 1.3, 1.1), bias=0.0, top_k=0, top_p=0.95, extra=extra,
               history_fn=lambda B, L: torch.tensor([[5] * (L - 1) + [131]]))
    chain_case("chain_bias_cfg2", B=3, V=256, L=16, cfg=2.0, ts=(16, 116), sos=1, ctx_sos=None, types_first=False,
               temps=(1.2, None, None, None), bias=0.5, top_k=5, top_p=1.0, history_fn=ts_heavy_history)
    chain_case("chain_c0_shape", B=1, V=4096, L=32, cfg=1.5, ts=(0, 2000), sos=4094, ctx_sos=None,
               types_first=False, temps=(0.9, None, None, None), bias=0.0, top_k=0, top_p=0.9, spikes=8)
    chain_case("chain_c1_bf16", B=2, V=4096, L=32, cfg=1.5, ts=(0, 2000), sos=4094, ctx_sos=None,
               types_first=False, temps=(0.9, None, None, None), bias=0.0, top_k=0, top_p=0.9, spikes=8,
               dtype="bf16")

    # ---- HF repetition penalty + top-k + top-p (third-party processors the chain appends) ----
    from transformers import RepetitionPenaltyLogitsProcessor

    B, V, L = 4, 512, 64
    x = (torch.randn((B, V), generator=g) * 2.0).to(torch.bfloat16).to(torch.float32)
    ids = torch.randint(0, V, (B, L), generator=g)
    rep = RepetitionPenaltyLogitsProcessor(1.1)(ids, x.clone())
    put("hf_repetition", logits=x.numpy(), input_ids=ids.numpy(), processed=rep.numpy(),
        final_hf=hf_warpers(rep.clone(), 50, 0.95).numpy())
    meta["hf_repetition"] = {"penalty": 1.1, "top_k": 50, "top_p": 0.95}

    # ---- the reference's decode loop on scripted one-hot logits: pad-on-finished and
    # wait-for-all-rows (the scenario of tests/test_optimized_single_decode_loop_migration.py:297-324,
    # greedy, EOS 2, pad 0, V = 8), plus seeded random schedules ----
    import importlib
    from types import SimpleNamespace

    from transformers import StoppingCriteriaList

    dl = importlib.import_module("osuT5.osuT5.inference.optimized.single.decode_loop")

    class Scripted:
        """A decoder whose step t puts logit +1000 on schedule[t][row], -1000 elsewhere."""

        def __init__(self, schedule, vocab):
            self.schedule = schedule
            self.vocab = vocab
            self.t = 0
            self.config = SimpleNamespace(is_encoder_decoder=False, _attn_implementation="sdpa")

        def _get_initial_cache_position(self, cur_len, device, model_kwargs):
            return model_kwargs

        def _valid_auto_compile_criteria(self, model_kwargs, generation_config):
            return False

        def _has_unfinished_sequences(self, finished, synced_gpus, device):
            return not bool(finished)

        def prepare_inputs_for_generation(self, input_ids, **model_kwargs):
            return {"input_ids": input_ids[:, -1:], "decoder_attention_mask": model_kwargs["decoder_attention_mask"]}

        def __call__(self, **kwargs):
            tokens = torch.tensor(self.schedule[self.t])
            self.t += 1
            logits = torch.full((len(tokens), 1, self.vocab), -1000.0)
            logits[torch.arange(len(tokens)), 0, tokens] = 1000.0
            return SimpleNamespace(logits=logits)

        def _update_model_kwargs_for_generation(self, outputs, model_kwargs, is_encoder_decoder):
            mask = model_kwargs["decoder_attention_mask"]
            model_kwargs["decoder_attention_mask"] = torch.cat((mask, torch.ones((mask.shape[0], 1), dtype=mask.dtype)), 1)
            return model_kwargs

    class RowEos:
        eos_token_id = 2

        def __call__(self, input_ids, scores):
            return input_ids[:, -1].eq(self.eos_token_id)

    def decode_case(name, schedule, prompt):
        steps = len(schedule)
        cfg = SimpleNamespace(return_dict_in_generate=False, output_attentions=False, output_hidden_states=False,
                              output_scores=False, output_logits=False, prefill_chunk_size=None,
                              _pad_token_tensor=torch.tensor(0), max_length=prompt.shape[1] + steps + 1,
                              do_sample=False)
        out = dl.active_prefix_decode_generate(Scripted(schedule, 8), prompt, logits_processor=lambda i, s: s,
                                               stopping_criteria=StoppingCriteriaList([RowEos()]),
                                               generation_config=cfg, decoder_attention_mask=prompt.ne(0))
        gen = out[:, prompt.shape[1]:]
        put(name, schedule=np.array(schedule, dtype=np.int64), generated=gen.numpy())
        meta[name] = {"eos": 2, "pad": 0, "vocab": 8}

    decode_case("ref_decode_pad", [(2, 5, 5), (7, 2, 5), (7, 7, 2)], torch.tensor(((0, 9), (8, 9), (0, 9))))
    rs = np.random.default_rng(4242)
    sched = rs.integers(3, 8, size=(7, 6))
    for r in range(6):  # every row ends: an EOS at a random step, the last step for the rest
        sched[rs.integers(0, 7) if r < 5 else 6, r] = 2
    sched[6, :] = 2
    decode_case("ref_decode_pad_random", [tuple(int(v) for v in row) for row in sched],
                torch.randint(1, 8, (6, 3), generator=g))

    # ---- lookback bias over consecutive calls (LookbackBiasLogitsWarper keeps the
    # previous call's scores): seeded scores with EOS ids boosted per row, some
    # masked ids, and a last input token that is a timed event on about half the
    # rows.  TIME_SHIFT's values start at -20 (tokenizer.py:54 uses -512), so the
    # lookback range is [16, 16 + 20 + 30).  Also the full chain with lookback. ----
    gl = torch.Generator().manual_seed(777)
    lb_extra = {"CIRCLE": (140, 141), "BEAT": (130, 131), "MEASURE": (131, 132), "TIMING_POINT": (132, 133),
                "SLIDER_HEAD": (143, 150), "HOLD_NOTE": (141, 142), "HOLD_NOTE_END": (142, 143),
                "SCROLL_SPEED": (150, 170)}
    lb_tok = make_tokenizer(ev, ts=(16, 116), sos=1, extra=lb_extra,
                            context_eos={ev.ContextType.TIMING: 4, ev.ContextType.KIAI: 5}, ts_min=-20, vocab=256)
    lb_meta = {"ts": [16, 116], "ts_min": -20, "lookback_time": 300.0, "eos": [2, 4, 5],
               "extra": {k: list(v) for k, v in lb_extra.items()}, "vocab": 256}

    def lb_history(B, T):
        ids = torch.randint(0, 256, (B, 4 + T), generator=gl)
        timed = torch.tensor([140, 130, 131, 145, 149, 141])
        untimed = torch.tensor([20, 60, 200, 3, 115, 170])
        pick = torch.rand((B, T), generator=gl) < 0.5
        ti = timed[torch.randint(0, len(timed), (B, T), generator=gl)]
        ui = untimed[torch.randint(0, len(untimed), (B, T), generator=gl)]
        ids[:, 4:] = torch.where(pick, ti, ui)
        return ids

    def lb_scores(R):
        x = torch.randn((R, 256), generator=gl) * 1.5
        x[:, [2, 4, 5]] += torch.rand((R, 1), generator=gl) * 6.0 - 2.0
        x[: R // 2, 20:28] = -float("inf")
        return x

    for name, types_first in (("lookback_renorm", True), ("lookback_mask", False)):
        B, T = 6, 6
        ids = lb_history(B, T)
        w = lp.LookbackBiasLogitsWarper(300.0, lb_tok, types_first, "cpu")
        xs, outs = [], []
        for t in range(T):
            x = lb_scores(B)
            outs.append(w(ids[:, : 4 + t + 1].clone(), x.clone()).numpy())
            xs.append(x.numpy())
        put(name, input_ids=ids.numpy(), scores=np.stack(xs), out=np.stack(outs))
        meta[name] = dict(lb_meta, types_first=types_first, steps=T, prefix=4)

    B, T = 4, 5
    ids = lb_history(B, T)
    procs = lp.build_logits_processor_list(lb_tok, cfg_scale=1.5, timeshift_bias=0.25, types_first=True,
                                           temperature=0.9, timing_temperature=0.8, lookback_time=300.0)
    xs, outs = [], []
    for t in range(T):
        x = lb_scores(2 * B)
        outs.append(procs(ids[:, : 4 + t + 1].clone(), x.clone()).numpy())
        xs.append(x.numpy())
    put("lookback_chain", input_ids=ids.numpy(), logits=np.stack(xs), processed=np.stack(outs))
    meta["lookback_chain"] = dict(lb_meta, types_first=True, steps=T, prefix=4, cfg=1.5, bias=0.25,
                                  temps=[0.9, 0.8, 0.9, 0.9], sos=[1])

    fixtures["meta.json"] = np.frombuffer(json.dumps(meta).encode(), dtype=np.uint8)
    np.savez_compressed(OUT, **fixtures)
    print(f"wrote {OUT} ({OUT.stat().st_size} bytes, {len(fixtures)} arrays)")


if __name__ == "__main__":
    main()

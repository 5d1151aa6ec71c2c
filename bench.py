#!/usr/bin/env python
"""Decode-sampling step benchmark (one JSON line on rank 0).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
    torchrun --nproc-per-node N bench.py --gpus N ...      (N > 1)

Workload ("sharded_decode"): 4096 CFG pairs (8192 logits rows) x V=4096 bf16
per step, 512-id int64 history per pair; chain = CFG 1.5 -> monotonic
time-shift mask -> event-grammar mask -> repetition 1.1 / frequency 0.2 /
presence 0.1 -> top_k 50 -> top_p 0.95 -> draw.  Rows are split evenly over
the N GPUs (no collective on the path; "strong" scaling).  A step is one
fused launch over this GPU's shard.  Inputs rotate over a pool of buffers
larger than 3x L2 so every step reads its logits from HBM.

Reported: device-timed sampled tokens/s (max over ranks), end-to-end tokens/s
through FusedSampler with host copies, HBM roofline of the kernel, the CPU
baseline (PyTorch restatement of the reference chain on the host cores), the
µs per step of the 64-pair batched decode, and SM clocks sampled during the
timed region.
"""

from __future__ import annotations

import argparse
import json
import math
import os
import sys
import threading
import time
from pathlib import Path

import numpy as np
import torch

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

PAIRS = 4096
VOCAB = 4096
HISTORY = 512
TS_END = 2000
SOS_ID = 4094
N_CLASSES = 16
METRIC = "sampled tokens/sec (device-timed)"
WORKLOAD = ("sharded_decode: 4096 CFG pairs (8192 rows) x V=4096 bf16 logits, 512-id int64 history; "
            "CFG 1.5 -> monotonic -> grammar(16 classes) -> repetition 1.1 / frequency 0.2 / presence 0.1 -> "
            "top_k 50 -> top_p 0.95 -> inverse-CDF draw")
L2_BYTES = 126 * 1024 * 1024


def parse_args():
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=4096)
    p.add_argument("--warmup", type=int, default=32)
    p.add_argument("--impl", choices=["ours", "reference"], default="ours")
    p.add_argument("--e2e-steps", type=int, default=48)
    p.add_argument("--b64-steps", type=int, default=2048)
    p.add_argument("--cpu-seconds", type=float, default=12.0)
    p.add_argument("--profile", type=int, default=0,
                   help="only run this many eager launches of one workload (for ncu), print nothing")
    p.add_argument("--profile-workload", choices=["sharded", "b64", "lmhead", "v65536", "topp1024"], default="sharded")
    p.add_argument("--lm-steps", type=int, default=1024, help="steps per timed variant of the lm_head leg (0: skip)")
    p.add_argument("--sweep-steps", type=int, default=512, help="steps per sweep workload (0: skip)")
    p.add_argument("--rows-curve", action="store_true",
                   help="instead of the headline line: one line per pair count of the sharded step (16 .. 4096 "
                        "CFG pairs, default kernel choice): how the step time follows the rows per GPU")
    p.add_argument("--sweep", action="store_true",
                   help="instead of the headline line: one line per vocabulary-sweep workload (rows x V bf16, "
                        "penalties + top_k 50 + top_p 0.95), device-timed, with its HBM roofline")
    return p.parse_args()


# ---------------------------------------------------------------- distributed plumbing
class Dist:
    def __init__(self):
        self.world = int(os.environ.get("WORLD_SIZE", "1"))
        self.rank = int(os.environ.get("RANK", "0"))
        self.local = int(os.environ.get("LOCAL_RANK", "0"))
        self.pg = None
        if self.world > 1:
            import datetime

            import torch.distributed as dist

            backend = "nccl" if torch.cuda.is_available() else "gloo"
            if backend == "nccl":
                torch.cuda.set_device(self.local)
            dist.init_process_group(backend, timeout=datetime.timedelta(seconds=120))
            self.pg = dist

    def barrier(self):
        if self.pg:
            if torch.cuda.is_available():
                self.pg.barrier(device_ids=[self.local])
            else:
                self.pg.barrier()

    def max(self, v: float) -> float:
        if not self.pg:
            return v
        dev = torch.device("cuda", self.local) if torch.cuda.is_available() else torch.device("cpu")
        t = torch.tensor([v], dtype=torch.float64, device=dev)
        self.pg.all_reduce(t, op=self.pg.ReduceOp.MAX)
        return float(t.item())

    def close(self):
        if self.pg:
            self.pg.destroy_process_group()


# ---------------------------------------------------------------- clocks (NVML, read only)
_REASONS = {0x1: "gpu_idle", 0x2: "applications_clocks_setting", 0x4: "sw_power_cap", 0x8: "hw_slowdown",
            0x10: "sync_boost", 0x20: "sw_thermal_slowdown", 0x40: "hw_thermal_slowdown",
            0x80: "hw_power_brake_slowdown", 0x100: "display_clock_setting"}


class ClockSampler:
    def __init__(self, device_index: int, interval: float = 0.005):
        self.samples, self.reasons, self.max_mhz = [], 0, None
        self._stop = threading.Event()
        self._thread = None
        try:
            import pynvml

            pynvml.nvmlInit()
            props = torch.cuda.get_device_properties(device_index)
            uuid = str(getattr(props, "uuid", ""))
            h = None
            if uuid:
                for cand in (uuid if uuid.startswith("GPU-") else "GPU-" + uuid, uuid):
                    try:
                        h = pynvml.nvmlDeviceGetHandleByUUID(cand.encode() if isinstance(cand, str) else cand)
                        break
                    except Exception:
                        h = None
            if h is None:
                h = pynvml.nvmlDeviceGetHandleByIndex(device_index)
            self.nvml, self.h = pynvml, h
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(h, pynvml.NVML_CLOCK_SM)
        except Exception as exc:  # pragma: no cover - depends on the box
            self.nvml, self.h, self.error = None, None, str(exc)
        self.interval = interval

    def _run(self):
        get_reasons = getattr(self.nvml, "nvmlDeviceGetCurrentClocksEventReasons", None) or \
            getattr(self.nvml, "nvmlDeviceGetCurrentClocksThrottleReasons")
        while not self._stop.is_set():
            try:
                self.samples.append(self.nvml.nvmlDeviceGetClockInfo(self.h, self.nvml.NVML_CLOCK_SM))
                self.reasons |= int(get_reasons(self.h))
            except Exception:
                pass
            time.sleep(self.interval)

    def __enter__(self):
        if self.nvml:
            self._thread = threading.Thread(target=self._run, daemon=True)
            self._thread.start()
        return self

    def __exit__(self, *exc):
        self._stop.set()
        if self._thread:
            self._thread.join()

    def summary(self):
        if not self.nvml:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "note": getattr(self, "error", "no NVML")}
        names = [n for bit, n in _REASONS.items() if self.reasons & bit and n != "gpu_idle"]
        return {"sm_mhz": float(np.median(self.samples)) if self.samples else None, "sm_max_mhz": self.max_mhz,
                "reasons": names, "samples": len(self.samples)}


# ---------------------------------------------------------------- inputs
def measured_peak():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        try:
            return float(json.loads(p.read_text())["hbm_gbs"]), "measured"
        except Exception:
            pass
    return 6650.0, "fallback"


def make_tables(gen, device):
    class_of = torch.randint(0, N_CLASSES, (VOCAB,), generator=gen, device=device).to(torch.uint8)
    table = torch.rand((N_CLASSES, N_CLASSES), generator=gen, device=device) < 0.5
    table[:, 0] = True
    return class_of, table


def sharded_sampler(device, pairs, gen):
    from mapperatorinator_b200.sampling import FusedSampler, GrammarTable

    class_of, table = make_tables(gen, device)
    grammar = GrammarTable.from_bool_table(class_of, table.cpu(), device)
    s = FusedSampler(vocab_size=VOCAB, num_rows=pairs, device=device, cfg_scale=1.5, time_shift_range=(0, TS_END),
                     sos_ids=(SOS_ID,), grammar=grammar, repetition_penalty=1.1, frequency_penalty=0.2,
                     presence_penalty=0.1, top_k=50, top_p=0.95)
    s.mono_state.copy_(torch.randint(0, TS_END, (pairs,), generator=gen, device=device).to(torch.int32))
    s.prev_token.copy_(torch.randint(0, VOCAB, (pairs,), generator=gen, device=device).to(torch.int32))
    s._scan_next = False
    s._prev_from_ids_next = False
    return s


def algorithmic_bytes(pairs: int) -> int:
    rows = 2 * pairs
    per_row_state = 4 + 4 + 4 + 4 + 4 + 8 + 4  # mono r/w, prev r/w, uniform, out id, status
    return rows * VOCAB * 2 + pairs * HISTORY * 8 + pairs * per_row_state + VOCAB + N_CLASSES * 4


def time_graph(fn_step, steps, stream, dist):
    """Capture `steps` calls of fn_step(i) in one CUDA graph; return (ms, graph)."""
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=stream):
        for i in range(steps):
            fn_step(i)
    torch.cuda.synchronize()
    dist.barrier()
    torch.cuda.synchronize()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(stream):
        start.record(stream)
        g.replay()
        end.record(stream)
    torch.cuda.synchronize()
    dist.barrier()
    return start.elapsed_time(end), g


# ---------------------------------------------------------------- our arm
def run_ours(args, dist: Dist):
    from mapperatorinator_b200 import _native
    from mapperatorinator_b200.parallel import shard_range

    _native.load()  # fail loudly without the native library
    device = torch.device("cuda", dist.local)
    torch.cuda.set_device(device)
    if args.profile and args.profile_workload == "b64":
        run_b64(args, device, torch.cuda.Stream(device), dist, profile=args.profile)
        return
    if args.profile and args.profile_workload == "lmhead":
        run_lmhead(args, device, torch.cuda.Stream(device), dist, profile=args.profile)
        return
    if args.profile and args.profile_workload in ("v65536", "topp1024"):
        rows, vocab, chain = (256, 65536, "penalties") if args.profile_workload == "v65536" else (1024, 4096, "topp")
        run_sweep_case(args, device, torch.cuda.Stream(device), dist, rows, vocab, chain, profile=args.profile)
        return
    start, end = shard_range(PAIRS, dist.world, dist.rank)
    pairs = end - start
    gen = torch.Generator(device).manual_seed(1234 + dist.rank)
    sampler = sharded_sampler(device, pairs, gen)
    history = torch.randint(0, VOCAB, (pairs, HISTORY), generator=gen, device=device)
    buf_bytes = 2 * pairs * VOCAB * 2
    nbuf = max(6, math.ceil(3 * L2_BYTES / buf_bytes))
    pool = [(torch.randn((2 * pairs, VOCAB), generator=gen, device=device) * 2.0).to(torch.bfloat16)
            for _ in range(nbuf)]
    upool = torch.rand((nbuf, pairs), generator=gen, device=device)
    stream = torch.cuda.Stream(device)

    def step(i):
        sampler.step(pool[i % nbuf], history, uniforms=upool[i % nbuf])

    with torch.cuda.stream(stream):
        for i in range(args.warmup):
            step(i)
    torch.cuda.synchronize()
    if args.profile:
        with torch.cuda.stream(stream):
            for i in range(args.profile):
                step(i)
        torch.cuda.synchronize()
        return
    info = sampler.launch_info(pool[0], history, upool[0])
    kernel_name = KERNEL_NAMES[info.kernel]
    with ClockSampler(device.index) as clocks:
        ms, graph = time_graph(step, args.steps, stream, dist)
    ms = dist.max(ms)
    del graph
    tokens = PAIRS * args.steps
    value = tokens / (ms / 1e3)
    per_launch_s = ms / 1e3 / args.steps
    bytes_launch = algorithmic_bytes(pairs)
    peak, peak_kind = measured_peak()
    achieved = bytes_launch / per_launch_s / 1e9

    # ---- end to end through FusedSampler with host buffers
    e2e_steps = max(1, min(args.e2e_steps, args.steps))
    host_logits = pool[0].cpu().pin_memory()
    host_u = upool[0].cpu().pin_memory()
    host_out = torch.empty(pairs, dtype=torch.int64).pin_memory()
    dev_logits = torch.empty_like(pool[0])
    dev_u = torch.empty_like(upool[0])
    torch.cuda.synchronize()
    dist.barrier()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(stream):
        ev0.record(stream)
        for _ in range(e2e_steps):
            dev_logits.copy_(host_logits, non_blocking=True)
            dev_u.copy_(host_u, non_blocking=True)
            ids = sampler.step(dev_logits, history, uniforms=dev_u)
            host_out.copy_(ids, non_blocking=True)
            stream.synchronize()
        ev1.record(stream)
    torch.cuda.synchronize()
    e2e_ms = dist.max(ev0.elapsed_time(ev1))
    dist.barrier()

    # ---- µs per step of the 64-pair batched decode (latency, per GPU)
    b64 = run_b64(args, device, stream, dist)
    # ---- the lm_head variant and the sweep (per GPU, same on every rank)
    lmhead = run_lmhead(args, device, stream, dist) if args.lm_steps > 0 else None
    sweep = run_sweep_lines(args, device, stream, dist) if args.sweep_steps > 0 else None

    cpu = None
    if dist.world == 1 and dist.rank == 0:
        cpu = cpu_baseline(args.cpu_seconds)

    if dist.rank == 0:
        line = {
            "metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": dist.world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms / args.steps, "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None, "dtype": "f32", "input_dtype": "bf16",
            "data": "synthetic: seeded N(0, 2^2) bf16 logits, uniform 512-id histories, random grammar table",
            "config": {"workload": WORKLOAD, "global_batch": PAIRS, "rows_per_gpu": 2 * pairs, "vocab": VOCAB,
                       "parallelism": f"row-sharded x{dist.world}, no collective",
                       "l2": f"logits rotate over {nbuf} buffers ({nbuf * buf_bytes / 2**20:.0f} MiB per GPU, "
                             f"> 3x L2)", "graph": f"{args.steps} launches captured in one CUDA graph"},
            "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                         "frac": achieved / peak, "peak_kind": peak_kind, "traffic": None,
                         "traffic_note": "DRAM bytes per launch come from an ncu capture (profiles/), not from this run",
                         "algorithmic_bytes_per_launch": bytes_launch, "kernel": kernel_name,
                         "grid": info.grid, "threads": info.threads,
                         "avg_launch_us": per_launch_s * 1e6},
            "cpu_baseline": cpu,
            "e2e": {"value": PAIRS * e2e_steps / (e2e_ms / 1e3), "unit": "tokens/s",
                    "h2d_bytes_per_step": 2 * PAIRS * VOCAB * 2 + PAIRS * 4, "d2h_bytes_per_step": PAIRS * 8,
                    "steps": e2e_steps, "api": "FusedSampler.step, pinned host buffers, sync per step"},
            "gpu_launches": args.steps,
            "clocks": clocks.summary(),
            "decode_step_b64": b64,
            "lmhead_fused": lmhead,
            "sweep": sweep,
        }
        print(json.dumps(line), flush=True)


def run_b64(args, device, stream, dist, profile=0):
    """64 CFG pairs x V=4096 bf16, CFG + monotonic + grammar + T 0.9 on time shifts + top_p 0.9."""
    from mapperatorinator_b200.sampling import FusedSampler, GrammarTable

    pairs = 64
    gen = torch.Generator(device).manual_seed(77 + dist.rank)
    class_of, table = make_tables(gen, device)
    s = FusedSampler(vocab_size=VOCAB, num_rows=pairs, device=device, cfg_scale=1.5, time_shift_range=(0, TS_END),
                     sos_ids=(SOS_ID,), grammar=GrammarTable.from_bool_table(class_of, table.cpu(), device),
                     column_temperatures=[(0, TS_END, 0.9)], top_p=0.9)
    s.mono_state.copy_(torch.randint(0, TS_END, (pairs,), generator=gen, device=device).to(torch.int32))
    s.prev_token.copy_(torch.randint(0, VOCAB, (pairs,), generator=gen, device=device).to(torch.int32))
    s._scan_next = s._prev_from_ids_next = False
    nbuf = math.ceil(3 * L2_BYTES / (2 * pairs * VOCAB * 2))
    x = torch.randn((nbuf, 2 * pairs, VOCAB), generator=gen, device=device) * 1.5
    spikes = torch.randperm(VOCAB, generator=gen, device=device)[:8]
    x[:, :, spikes] = 8.0
    pool = x.to(torch.bfloat16)
    del x
    u = torch.rand((nbuf, pairs), generator=gen, device=device)
    steps = args.b64_steps

    def step(i):
        s.step(pool[i % nbuf], uniforms=u[i % nbuf])

    with torch.cuda.stream(stream):
        for i in range(16 + profile):
            step(i)
    torch.cuda.synchronize()
    if profile:
        return None
    ms, g = time_graph(step, steps, stream, dist)
    del g
    return {"us_per_step": ms * 1e3 / steps, "steps": steps, "pairs": pairs,
            "workload": "batched_decode: 64 CFG pairs x V=4096 bf16, CFG 1.5 + monotonic + grammar + "
                        "T=0.9 on time shifts + top_p 0.9, graph-replayed, inputs rotating over > 3x L2"}


def run_lmhead(args, device, stream, dist, profile=0):
    """The lm_head variant: 256 hidden rows (128 CFG pairs) x d=768 bf16 ~ N(0, 1), proj_out weight
    V=4096 x 768 bf16 ~ N(0, 0.02^2), then the batched-decode chain (CFG 1.5, monotonic, grammar,
    T=0.9 on time shifts, top_p 0.9, draw).  Times, each over one captured graph of `steps` steps
    with hidden states and weights rotating over > 3x L2: the tcgen05 projection alone, the
    projection -> sampler pair (programmatic dependent launch), torch's bf16 matmul (cuBLAS, the
    reference's nn.Linear) alone and followed by the same sampler, and the sampler alone."""
    from mapperatorinator_b200.sampling import FusedSampler, GrammarTable, lm_head_logits

    pairs, d = 128, 768
    gen = torch.Generator(device).manual_seed(99 + dist.rank)
    class_of, table = make_tables(gen, device)
    s = FusedSampler(vocab_size=VOCAB, num_rows=pairs, device=device, cfg_scale=1.5, time_shift_range=(0, TS_END),
                     sos_ids=(SOS_ID,), grammar=GrammarTable.from_bool_table(class_of, table.cpu(), device),
                     column_temperatures=[(0, TS_END, 0.9)], top_p=0.9)
    s.mono_state.copy_(torch.randint(0, TS_END, (pairs,), generator=gen, device=device).to(torch.int32))
    s.prev_token.copy_(torch.randint(0, VOCAB, (pairs,), generator=gen, device=device).to(torch.int32))
    s._scan_next = s._prev_from_ids_next = False
    step_bytes = VOCAB * d * 2 + 2 * pairs * d * 2
    nbuf = math.ceil(3 * L2_BYTES / step_bytes)
    W = (torch.randn((nbuf, VOCAB, d), generator=gen, device=device) * 0.02).to(torch.bfloat16)
    H = torch.randn((nbuf, 2 * pairs, d), generator=gen, device=device).to(torch.bfloat16)
    U = torch.rand((nbuf, pairs), generator=gen, device=device)
    logits = torch.empty((2 * pairs, VOCAB), dtype=torch.bfloat16, device=device)
    variants = {
        "fused": lambda i: s.step_hidden(H[i % nbuf], W[i % nbuf], uniforms=U[i % nbuf]),
        "projection": lambda i: lm_head_logits(H[i % nbuf], W[i % nbuf], out=logits),
        "cublas_then_sampler": lambda i: (torch.matmul(H[i % nbuf], W[i % nbuf].T, out=logits),
                                          s.step(logits, uniforms=U[i % nbuf])),
        "cublas": lambda i: torch.matmul(H[i % nbuf], W[i % nbuf].T, out=logits),
        "sampler": lambda i: s.step(logits, uniforms=U[i % nbuf]),
    }
    with torch.cuda.stream(stream):
        for fn in variants.values():
            for i in range(8):
                fn(i)
    torch.cuda.synchronize()
    if profile:
        with torch.cuda.stream(stream):
            for i in range(profile):
                variants["fused"](i)
        torch.cuda.synchronize()
        return None
    steps = args.lm_steps
    us = {}
    for name, fn in variants.items():
        ms, g = time_graph(fn, steps, stream, dist)
        us[name] = dist.max(ms) * 1e3 / steps
        del g
    flops = 2.0 * 2 * pairs * VOCAB * d
    tflops = flops / (us["projection"] * 1e-6) / 1e12
    try:
        peak = float(json.loads((ROOT / "MEASURED_PEAKS.json").read_text())["bf16_tflops"])
        peak_kind = "measured (burst)"
    except Exception:
        peak, peak_kind = 1590.0, "fallback"
    return {"workload": "lmhead: 256 hidden rows (128 CFG pairs) x d=768 bf16 -> V=4096 bf16 logits (tcgen05) "
                        "-> CFG 1.5 + monotonic + grammar + T=0.9 on time shifts + top_p 0.9 + draw",
            "us_per_step": us["fused"], "tokens_per_s": pairs / (us["fused"] * 1e-6),
            "us": {k: round(v, 3) for k, v in us.items()},
            "projection_roofline": {"bound": "tensor", "achieved": tflops, "peak": peak, "unit": "TFLOP/s",
                                    "frac": tflops / peak, "peak_kind": peak_kind, "flops_per_launch": flops,
                                    "kernel": "mtr::lm::lmhead_gemm_kernel"},
            "speedup_vs_cublas_then_sampler": us["cublas_then_sampler"] / us["fused"],
            "steps": steps, "l2": f"hidden + weights rotate over {nbuf} sets ({nbuf * step_bytes / 2**20:.0f} MiB)"}


def run_sweep_lines(args, device, stream, dist):
    """The throughput sweep (rows x V bf16 N(0, 2^2), 512-id history, repetition 1.1 / frequency 0.2 /
    presence 0.1, top_k 50, top_p 0.95, draw) and the reference's production preset (temperature
    0.9, top_p 0.9, no top_k) at 1024 x 4096: one dict per workload, device-timed."""
    out = []
    cases = [(rows, vocab, "penalties") for rows, vocab in SWEEP] + [(1024, 4096, "topp")]
    for rows, vocab, chain in cases:
        out.append(run_sweep_case(args, device, stream, dist, rows, vocab, chain))
        torch.cuda.empty_cache()
    return out


def run_sweep_case(args, device, stream, dist, rows, vocab, chain, profile=0):
    """One sweep workload: `chain` "penalties" = repetition 1.1 / frequency 0.2 / presence 0.1 + top_k 50 +
    top_p 0.95 over a 512-id history; "topp" = temperature 0.9 + top_p 0.9 (the reference's production
    preset).  Logits rotate over > 3x L2.  With `profile`, only runs that many eager launches."""
    from mapperatorinator_b200.sampling import FusedSampler

    peak, peak_kind = measured_peak()
    gen = torch.Generator(device).manual_seed(4321 + rows + vocab)
    if chain == "topp":
        s = FusedSampler(vocab_size=vocab, num_rows=rows, device=device, temperature=0.9, top_p=0.9)
        hist = None
    else:
        s = FusedSampler(vocab_size=vocab, num_rows=rows, device=device, repetition_penalty=1.1,
                         frequency_penalty=0.2, presence_penalty=0.1, top_k=50, top_p=0.95)
        hist = torch.randint(0, vocab, (rows, HISTORY), generator=gen, device=device)
    buf_bytes = rows * vocab * 2
    nbuf = max(4, math.ceil(3 * L2_BYTES / buf_bytes))
    pool = [(torch.randn((rows, vocab), generator=gen, device=device) * 2.0).to(torch.bfloat16) for _ in range(nbuf)]
    upool = torch.rand((nbuf, rows), generator=gen, device=device)

    def step(i):
        s.step(pool[i % nbuf], hist, uniforms=upool[i % nbuf])

    with torch.cuda.stream(stream):
        for i in range(max(3, args.warmup) + profile):
            step(i)
    torch.cuda.synchronize()
    if profile:
        return None
    info = s.launch_info(pool[0], hist, upool[0])
    steps = args.sweep_steps
    ms, graph = time_graph(step, steps, stream, dist)
    ms = dist.max(ms)
    del graph
    us = ms * 1e3 / steps
    nbytes = rows * vocab * 2 + (rows * HISTORY * 8 if hist is not None else 0) + rows * (4 + 8 + 4)
    gbs = nbytes / (us * 1e-6) / 1e9
    return {"rows": rows, "vocab": vocab,
            "chain": "penalties_topk50_topp0.95" if chain == "penalties" else "T0.9_topp0.9",
            "us_per_step": round(us, 3), "tokens_per_s": rows / (us * 1e-6), "algorithmic_bytes_per_launch": nbytes,
            "achieved_gbs": round(gbs, 1), "frac": round(gbs / peak, 4), "peak_kind": peak_kind,
            "kernel": KERNEL_NAMES[info.kernel], "grid": info.grid, "threads": info.threads,
            "cluster": info.cluster_size, "l2": f"logits rotate over {nbuf} buffers"}


KERNEL_NAMES = {0: "mtr::sampler_kernel", 1: "mtr::row_warp_kernel", 2: "mtr::stream_kernel"}


# ---------------------------------------------------------------- CPU side
REF_DIR = ROOT / "baseline" / "_ref"


def _cpu_chain(pairs, seed=5):
    """The sharded_decode chain on the host, returned as (step function, kind).

    kind "reference": the reference's own processors, path-loaded from the
    unmodified copy in baseline/_ref (baseline/install_reference.sh) --
    build_logits_processor_list (HF ClassifierFreeGuidance + the reference's
    MonotonicTimeShift) and HF's RepetitionPenalty / TopK / TopP, then softmax +
    torch.multinomial as the reference's decode loop does.  The event-grammar
    mask and the frequency / presence penalties have no reference
    implementation and come from oracle/torch_chain.py.  kind "port": the whole
    chain from oracle/torch_chain.py (when baseline/_ref is absent)."""
    from oracle import torch_chain as TC

    g = torch.Generator().manual_seed(seed)
    class_of = torch.randint(0, N_CLASSES, (VOCAB,), generator=g)
    table = torch.rand((N_CLASSES, N_CLASSES), generator=g) < 0.5
    table[:, 0] = True
    logits = (torch.randn((2 * pairs, VOCAB), generator=g) * 2.0).to(torch.bfloat16)
    ids = torch.randint(0, VOCAB, (pairs, HISTORY), generator=g)
    ids[:, -2] = torch.randint(0, TS_END, (pairs,), generator=g)  # a late time shift: the monotonic mask is active
    prev = torch.randint(0, VOCAB, (pairs,), generator=g)
    try:
        from oracle.reference_loader import load_reference, make_tokenizer
        from transformers import RepetitionPenaltyLogitsProcessor, TopKLogitsWarper, TopPLogitsWarper

        ev, lp, _sl, _ = load_reference(REF_DIR)
    except (FileNotFoundError, ImportError):
        prm = TC.ChainParams(cfg_scale=1.5, ts_range=(0, TS_END), sos_ids=(SOS_ID,), grammar_class_of=class_of,
                             grammar_table=table, repetition_penalty=1.1, frequency_penalty=0.2,
                             presence_penalty=0.1, top_k=50, top_p=0.95)
        return (lambda: TC.sample_step(logits, ids, prm, prev_tokens=prev, generator=g)), "port"
    tok = make_tokenizer(ev, ts=(0, TS_END), sos=SOS_ID)
    procs = lp.build_logits_processor_list(tok, cfg_scale=1.5, types_first=False, temperature=1.0)
    rep, topk, topp = RepetitionPenaltyLogitsProcessor(1.1), TopKLogitsWarper(50), TopPLogitsWarper(0.95)

    def step():
        scores = procs(ids, logits.to(torch.float32))
        scores = TC.grammar_mask(scores, prev, class_of, table)
        scores = rep(ids, scores)
        scores = TC.frequency_presence(scores, ids, 0.2, 0.1)
        scores = topp(ids, topk(ids, scores))
        return torch.multinomial(torch.nn.functional.softmax(scores, dim=-1), 1, generator=g).squeeze(1)

    return step, "reference"


def cpu_baseline(seconds: float, pairs: int = 64):
    """The reference chain on the host cores (bounded sample of the workload)."""
    torch.set_num_threads(os.cpu_count() or 1)
    step, kind = _cpu_chain(pairs)
    step()
    n, t0 = 0, time.perf_counter()
    while time.perf_counter() - t0 < seconds and n < 500:
        step()
        n += 1
    dt = (time.perf_counter() - t0) / n
    return {"value": pairs / dt, "unit": "tokens/s", "cores": torch.get_num_threads(), "kind": kind,
            "sample": f"{pairs} CFG pairs of the sharded_decode chain per step, {n} steps, "
                      f"torch {torch.__version__} CPU, {dt * 1e3:.1f} ms/step"}


def run_reference(args, dist: Dist):
    if dist.rank != 0:
        return
    torch.set_num_threads(os.cpu_count() or 1)
    step, kind = _cpu_chain(64)
    t = time.perf_counter()
    step()
    t64 = time.perf_counter() - t
    budget = 120.0
    pairs = int(max(1, min(64, math.floor(64 * budget / max(1e-9, args.steps * t64)))))
    step, kind = _cpu_chain(pairs)
    for _ in range(args.warmup):
        step()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        step()
    dt = time.perf_counter() - t0
    value = pairs * args.steps / dt
    cores = torch.get_num_threads()
    what = ("the reference's own processors (build_logits_processor_list, HF repetition / top-k / top-p) + "
            "grammar and frequency / presence from oracle/torch_chain.py" if kind == "reference" else
            "PyTorch CPU restatement of the reference chain (oracle/torch_chain.py)")
    sample = f"{pairs} CFG pairs of the sharded_decode chain per step ({what}), softmax + multinomial, {args.steps} steps"
    line = {"metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": dist.world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": dt * 1e3 / args.steps, "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "f32", "impl": "reference",
            "data": "synthetic: seeded N(0, 2^2) bf16 logits, uniform 512-id histories",
            "config": {"workload": WORKLOAD, "global_batch": PAIRS, "sample_pairs_per_step": pairs},
            "cpu_baseline": {"value": value, "unit": "tokens/s", "cores": cores, "kind": kind, "sample": sample},
            "e2e": {"value": value, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


# ---------------------------------------------------------------- step time against rows per GPU
CURVE_PAIRS = (16, 64, 256, 512, 1024, 2048, 4096)


def run_rows_curve(args, dist):
    """`--rows-curve`: the sharded step (same chain as the headline) at each pair count of CURVE_PAIRS on
    one GPU, graph-timed, logits rotating over > 3x L2.  Below one round of resident rows the step time
    is the latency of one row, which is what bounds strong scaling across GPUs."""
    from mapperatorinator_b200 import _native

    _native.load()  # fail loudly without the native library
    device = torch.device("cuda", dist.local)
    torch.cuda.set_device(device)
    stream = torch.cuda.Stream(device)
    steps = max(64, min(args.steps, 1024))
    peak, peak_kind = measured_peak()
    for pairs in CURVE_PAIRS:
        gen = torch.Generator(device).manual_seed(4321 + pairs)
        sampler = sharded_sampler(device, pairs, gen)
        history = torch.randint(0, VOCAB, (pairs, HISTORY), generator=gen, device=device)
        nbuf = max(4, math.ceil(3 * L2_BYTES / (2 * pairs * VOCAB * 2)))
        pool = [(torch.randn((2 * pairs, VOCAB), generator=gen, device=device) * 2.0).to(torch.bfloat16)
                for _ in range(nbuf)]
        upool = torch.rand((nbuf, pairs), generator=gen, device=device)

        def step(i):
            sampler.step(pool[i % nbuf], history, uniforms=upool[i % nbuf])

        with torch.cuda.stream(stream):
            for i in range(max(3, args.warmup)):
                step(i)
        torch.cuda.synchronize()
        info = sampler.launch_info(pool[0], history, upool[0])
        ms, graph = time_graph(step, steps, stream, dist)
        ms = dist.max(ms)
        del graph
        us = ms * 1e3 / steps
        gbs = algorithmic_bytes(pairs) / (us * 1e-6) / 1e9
        if dist.rank == 0:
            print(json.dumps({"workload": "rows_curve", "pairs": pairs, "us_per_step": round(us, 3),
                              "tokens_per_s": pairs / (us * 1e-6), "achieved_gbs": round(gbs, 1),
                              "frac": round(gbs / peak, 4), "peak_kind": peak_kind,
                              "kernel": KERNEL_NAMES[info.kernel], "grid": info.grid, "threads": info.threads,
                              "steps": steps}), flush=True)
        del pool, upool, sampler, history
        torch.cuda.empty_cache()


# ---------------------------------------------------------------- vocabulary sweep
SWEEP = ((256, 4096), (256, 16384), (256, 65536), (1024, 4096))


def run_sweep(args, dist):
    """`--sweep`: one JSON line per sweep workload instead of the headline line."""
    from mapperatorinator_b200 import _native

    _native.load()  # fail loudly without the native library
    device = torch.device("cuda", dist.local)
    torch.cuda.set_device(device)
    stream = torch.cuda.Stream(device)
    args.sweep_steps = max(64, min(args.steps, 2048))
    for line in run_sweep_lines(args, device, stream, dist):
        if dist.rank == 0:
            print(json.dumps(dict(line, workload="vocab_sweep")), flush=True)


def main():
    args = parse_args()
    dist = Dist()
    try:
        if args.sweep:
            run_sweep(args, dist)
        elif args.rows_curve:
            run_rows_curve(args, dist)
        elif args.impl == "reference":
            run_reference(args, dist)
        else:
            run_ours(args, dist)
    finally:
        dist.close()


if __name__ == "__main__":
    main()

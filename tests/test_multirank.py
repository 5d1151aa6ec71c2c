"""Multi-rank host logic on CPU (gloo, world_size 2): row sharding is a
partition, per-rank results reassemble to the full-batch result, and the
timing reduction takes the max over ranks.  The oracle stands in for each
rank's device step, as the checker."""

import os
import socket

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

from mapperatorinator_b200 import parallel
from tests.harness import workloads as W


def test_shard_range_partitions():
    for total in (0, 1, 7, 64, 4096, 4097):
        for world in (1, 2, 3, 8):
            spans = [parallel.shard_range(total, world, r) for r in range(world)]
            assert spans[0][0] == 0 and spans[-1][1] == total
            assert all(a[1] == b[0] for a, b in zip(spans, spans[1:]))
            sizes = [e - s for s, e in spans]
            assert max(sizes) - min(sizes) <= 1
    with pytest.raises(ValueError):
        parallel.shard_range(10, 2, 2)


def test_local_cfg_rows_keeps_pairs():
    x = torch.arange(2 * 6 * 4, dtype=torch.float32).view(12, 4)
    loc = parallel.local_cfg_rows(x, 6, 2, 5)
    assert torch.equal(loc[:3], x[2:5]) and torch.equal(loc[3:], x[8:11])


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, out):
    import torch.distributed as dist

    from oracle import oracle

    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world)
    try:
        full = W.sharded_decode(seed=9, pairs=40, history=64)
        s, e = parallel.shard_range(full.num_rows, world, rank)
        n = e - s
        logits = np.concatenate([full.logits[s:e], full.logits[full.num_rows + s:full.num_rows + e]])
        shard = full.with_(logits=logits, num_rows=n, input_ids=full.input_ids[s:e],
                           mono_state=full.mono_state[s:e], prev_token=full.prev_token[s:e],
                           uniforms=full.uniforms[s:e])
        ids = oracle.run(shard)["out_ids"]
        gathered = [torch.zeros(parallel.shard_range(full.num_rows, world, r)[1]
                                - parallel.shard_range(full.num_rows, world, r)[0], dtype=torch.int64)
                    for r in range(world)]
        dist.all_gather(gathered, torch.from_numpy(ids))
        t = parallel.max_over_ranks(1.0 + rank)
        if rank == 0:
            out.put((torch.cat(gathered).numpy(), t))
        dist.barrier()
    finally:
        dist.destroy_process_group()


def test_two_rank_sharding_matches_full_batch():
    from oracle import oracle

    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    # spawned ranks import torch afresh, which takes minutes on a busy host
    try:
        ids, tmax = q.get(timeout=600)
    finally:
        for p in procs:
            p.join(timeout=120)
            if p.exitcode is None:
                p.kill()
    for p in procs:
        assert p.exitcode == 0
    full = W.sharded_decode(seed=9, pairs=40, history=64)
    assert np.array_equal(ids, oracle.run(full)["out_ids"])
    assert tmax == 2.0


def test_max_over_ranks_without_group():
    assert parallel.max_over_ranks(3.5) == 3.5

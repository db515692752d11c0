"""The multi-GPU path's host logic on CPU ranks (gloo, world size 2): the
workload's sequences are partitioned across the ranks the way bench.py does
it (contiguous shares, the first ranks taking one more when the count does
not divide), each rank runs its share with no collective on the data path,
and the max-over-ranks timing and a gather of token streams are the only
collectives. The gathered streams, in sequence order, must equal a
single-process run of the whole workload."""

import os
import socket

import numpy as np
import pytest


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


TOTAL = 5  # sequences in the workload: 3 on rank 0, 2 on rank 1


def _worker(rank, world, port, archive, steps, results):
    import sys

    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    sys.path.insert(0, root)
    sys.path.insert(0, os.path.join(root, "needle-rs_b200"))
    import torch
    import torch.distributed as dist

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    import bench
    from oracle import oracle as orc

    m = orc.Model(archive)
    first, S = bench.shard(TOTAL, world, rank)
    prompts, masks = bench.make_inputs(first, S, steps, m.out_rows)
    b = orc.Batch(m, S, threads=1)
    b.prefill(prompts)
    import time

    t0 = time.perf_counter()
    toks = np.stack([b.step(masks[k]) for k in range(steps)], 1)
    t = torch.tensor([time.perf_counter() - t0], dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    gathered = [None] * world
    dist.all_gather_object(gathered, (first, toks.tolist(), float(t.item())))
    if rank == 0:
        results.put(gathered)
    dist.barrier()
    dist.destroy_process_group()


def test_two_ranks_shard_sequences(small_archive):
    import torch.multiprocessing as mp

    import bench
    from oracle import oracle as orc

    steps, world = 3, 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, small_archive, steps, q)) for r in range(world)]
    for p in procs:
        p.start()
    gathered = q.get(timeout=300)
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    m = orc.Model(small_archive)
    times = {g[2] for g in gathered}
    assert len(times) == 1, "every rank sees the same max-over-ranks time"
    assert [bench.shard(TOTAL, world, r) for r in range(world)] == [(0, 3), (3, 2)]
    streams = [row for _, toks, _ in sorted(gathered) for row in toks]
    assert len(streams) == TOTAL, "the shares cover every sequence once"
    prompts, masks = bench.make_inputs(0, TOTAL, steps, m.out_rows)
    one = orc.Batch(m, TOTAL, threads=1)
    one.prefill(prompts)
    want = np.stack([one.step(masks[k]) for k in range(steps)], 1)
    assert streams == want.tolist(), "a partitioned run equals the single-process run"
    # a share's inputs are the same rows of the whole workload's
    p1, m1 = bench.make_inputs(3, 2, steps, m.out_rows)
    assert np.array_equal(p1, prompts[3:]) and np.array_equal(m1, masks[:, 3:])

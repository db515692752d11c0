"""The multi-GPU path's host logic on CPU ranks (gloo, world size 2): each
rank builds its own shard of sequences the way bench.py does, runs it with
no collective on the data path, and the max-over-ranks timing and a gather
of token streams are the only collectives. The gathered streams must equal
single-process runs of the same sequences."""

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
    S = 2
    prompts, masks = bench.make_inputs(rank, S, steps, m.out_rows)
    b = orc.Batch(m, S, threads=1)
    b.prefill(prompts)
    import time

    t0 = time.perf_counter()
    toks = np.stack([b.step(masks[k]) for k in range(steps)], 1)
    t = torch.tensor([time.perf_counter() - t0], dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    gathered = [None] * world
    dist.all_gather_object(gathered, (rank, toks.tolist(), float(t.item())))
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
    seen = set()
    for rank, toks, _ in gathered:
        prompts, masks = bench.make_inputs(rank, 2, steps, m.out_rows)
        for s in range(2):
            want = m.generate(prompts[s].astype(np.uint32), steps, masks=masks[:, s])
            assert toks[s] == [int(v) for v in want]
            seen.add(tuple(prompts[s][:8]))
    assert len(seen) == 4, "ranks hold distinct sequences"

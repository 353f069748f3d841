"""The multi-process path on CPU: two `gloo` ranks each run their own shard
(with the oracle standing in for the GPU kernels), exchange nothing but the
timing reduction bench.py uses, and the gathered result equals the
single-process one."""
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank),
                      WORLD_SIZE=str(world))
    try:
        import bench
        from oracle import oracle
        from rocm_flashinfer_contest_b200 import inputs, partition
        dist.init_process_group("gloo", rank=rank, world_size=world)
        args = inputs.decode_inputs(7, 4, 8, seed=9)
        shard = partition.plan_decode(7, 4, 8, world)[rank]
        out = oracle.decode(*partition.apply_decode(args, shard), threads=1)
        gathered = [None] * world
        dist.all_gather_object(gathered, (shard, out))   # test-only: check the shards
        t = bench.max_over_ranks(float(rank + 1), world, torch.device("cpu"))
        if rank == 0:
            shards = [g[0] for g in gathered]
            o, s = partition.gather_decode(shards, [g[1] for g in gathered], 7, 8)
            ro, rs = oracle.decode(*args, threads=1)
            q.put(("ok", bool(torch.equal(o, ro) and torch.equal(s, rs)), t))
        dist.destroy_process_group()
    except Exception as e:  # report instead of hanging the parent
        q.put(("error", repr(e), None))


def test_two_gloo_ranks_reproduce_single_process():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    try:
        status, equal, tmax = q.get(timeout=180)
    finally:
        for p in procs:
            p.join(timeout=60)
            if p.is_alive():
                p.terminate()
    assert status == "ok", equal
    assert equal
    assert tmax == 2.0  # the max over ranks of (rank + 1)

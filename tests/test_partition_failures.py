"""Host-side failure handling of the sharded path (partition.run_shards), on
CPU with three processes sharing a TCPStore: rank 1's work raises, rank 2's
work sleeps past the deadline.  Rank 0 must report both (kind "raised" and
"timeout"), re-run their shards itself, and the gathered result must equal
the single-process one (the oracle stands in for the GPU kernels).  Nothing
waits on a GPU: a failed rank is seen on the host, as in the reference's
harness, which records a raising solution as a failed workload
(tools/local_verify.py:114-117)."""
import datetime
import socket
import time

import torch
import torch.multiprocessing as mp


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, q, sleep_s):
    try:
        import torch.distributed as dist
        from oracle import oracle
        from rocm_flashinfer_contest_b200 import inputs, partition
        store = dist.TCPStore("127.0.0.1", port, world, rank == 0, timeout=datetime.timedelta(seconds=60))
        args = inputs.decode_inputs(9, 4, 8, seed=21)
        shards = partition.plan_decode(9, 4, 8, world)

        def work(shard):
            if rank == 1 and shard.rank == 1:
                raise RuntimeError("injected failure on rank 1")
            if rank == 2 and shard.rank == 2:
                time.sleep(sleep_s)
            return oracle.decode(*partition.apply_decode(args, shard), threads=1)

        res = partition.run_shards(work, shards, rank, world, store, timeout_s=2.0)
        if rank == 0:
            results, failures = res
            o, s = partition.gather_decode(shards, results, 9, 8)
            ro, rs = oracle.decode(*args, threads=1)
            q.put(("ok", [(f.rank, f.kind) for f in failures], bool(torch.equal(o, ro) and torch.equal(s, rs))))
            store.set("done", "1")
        else:
            store.wait(["done"], datetime.timedelta(seconds=60))  # keep the store's server alive until then
    except Exception as e:  # report instead of hanging the parent
        q.put(("error", repr(e), False))


def test_failed_and_late_ranks_are_reported_and_rerun():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 3, port, q, 6.0)) for r in range(3)]
    for p in procs:
        p.start()
    try:
        status, failures, equal = q.get(timeout=180)
    finally:
        for p in procs:
            p.join(timeout=60)
            if p.is_alive():
                p.terminate()
    assert status == "ok", failures
    assert failures == [(1, "raised"), (2, "timeout")]
    assert equal

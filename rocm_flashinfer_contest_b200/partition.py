"""Shards GDN decode / prefill work across the GPUs of one node, with no collective.

Every (sequence, v-head) recurrence is independent; v-head h needs only q/k
head h // (HV/H), its own A_log/dt_bias/a/b and its own state.  So a shard
is a set of sequences times a group of v-heads aligned to HV/H, and no data
moves between GPUs: each rank is handed its inputs, runs the same kernels on
its own device, and keeps its outputs.  The reference has no multi-GPU path
(everything runs on cuda:0, tools/local_verify.py:60); this module is the
B200 build's partitioner for the 1/2/4/8-GPU decode configuration.

* ``plan_decode(B, H, HV, world)`` splits the batch into contiguous slices;
  when there are fewer sequences than ranks it also splits the v-heads into
  groups of whole q/k heads.
* ``plan_prefill(seqlens, H, HV, world)`` bins sequences by token count
  (longest first onto the least-loaded rank); with fewer sequences than ranks
  it splits v-head groups instead.

``apply_decode`` / ``apply_prefill`` cut a rank's inputs out of the full
argument list; ``gather_*`` reassembles full outputs (used by tests only: in a
real deployment the outputs stay where they were computed); an empty shard's
result may be None.
"""
from __future__ import annotations

from dataclasses import dataclass

import torch


@dataclass(frozen=True)
class Shard:
    rank: int
    seqs: tuple          # sequence (batch) indices owned by this rank, ascending
    heads: tuple         # (h0, h1): half-open v-head range, a multiple of HV/H wide

    @property
    def empty(self) -> bool:
        return len(self.seqs) == 0 or self.heads[0] == self.heads[1]


def _head_groups(H: int, HV: int, parts: int):
    """Split the H q/k heads (and their HV/H v-heads each) into `parts`
    contiguous groups as evenly as possible; returns v-head ranges."""
    rep = HV // H
    out = []
    for p in range(parts):
        lo, hi = (H * p) // parts, (H * (p + 1)) // parts
        out.append((lo * rep, hi * rep))
    return out


def plan_decode(B: int, H: int, HV: int, world: int):
    if world < 1:
        raise ValueError("world must be >= 1")
    if HV % H:
        raise ValueError("HV must be a multiple of H")
    if B >= world or B == 0:
        shards = []
        for r in range(world):
            lo, hi = (B * r) // world, (B * (r + 1)) // world
            shards.append(Shard(r, tuple(range(lo, hi)), (0, HV)))
        return shards
    # fewer sequences than ranks: ranks share a sequence, split by head group
    per_seq = world // B
    shards = []
    r = 0
    for s in range(B):
        n = per_seq + (1 if s < world % B else 0)
        for hg in _head_groups(H, HV, min(n, H)) + [(HV, HV)] * max(0, n - H):
            shards.append(Shard(r, (s,), hg))
            r += 1
    return shards


def plan_prefill(seqlens, H: int, HV: int, world: int):
    if world < 1:
        raise ValueError("world must be >= 1")
    if HV % H:
        raise ValueError("HV must be a multiple of H")
    N = len(seqlens)
    if N >= world:
        load = [0] * world
        owned = [[] for _ in range(world)]
        for i in sorted(range(N), key=lambda i: (-seqlens[i], i)):
            r = min(range(world), key=lambda r: (load[r], r))
            owned[r].append(i)
            load[r] += max(1, seqlens[i])
        return [Shard(r, tuple(sorted(owned[r])), (0, HV)) for r in range(world)]
    groups = _head_groups(H, HV, min(world, H)) + [(HV, HV)] * max(0, world - H)
    # with fewer sequences than ranks every rank takes all sequences, one head group
    return [Shard(r, tuple(range(N)), groups[r]) for r in range(world)]


def apply_decode(args, shard: Shard):
    """Rank-local decode arguments (q, k, v, state, A_log, a, dt_bias, b, scale)."""
    q, k, v, state, A_log, a, dt_bias, b, scale = args
    H, HV = q.shape[2], v.shape[2]
    rep = HV // H
    h0, h1 = shard.heads
    idx = torch.tensor(shard.seqs, dtype=torch.long, device=q.device)
    sel = lambda t: t.index_select(0, idx)  # noqa: E731
    return [sel(q)[:, :, h0 // rep:h1 // rep].contiguous(),
            sel(k)[:, :, h0 // rep:h1 // rep].contiguous(),
            sel(v)[:, :, h0:h1].contiguous(),
            None if state is None else sel(state)[:, h0:h1].contiguous(),
            A_log[h0:h1].contiguous(), sel(a)[:, :, h0:h1].contiguous(),
            dt_bias[h0:h1].contiguous(), sel(b)[:, :, h0:h1].contiguous(), scale]


def apply_prefill(args, shard: Shard):
    """Rank-local prefill arguments; tokens of the owned sequences are packed
    in order and cu_seqlens is rebuilt for them."""
    q, k, v, state, A_log, a, dt_bias, b, cu, scale = args
    H, HV = q.shape[1], v.shape[1]
    rep = HV // H
    h0, h1 = shard.heads
    cu_l = [int(x) for x in cu.tolist()]
    toks = [t for s in shard.seqs for t in range(cu_l[s], cu_l[s + 1])]
    tidx = torch.tensor(toks, dtype=torch.long, device=q.device)
    sidx = torch.tensor(shard.seqs, dtype=torch.long, device=q.device)
    lens = [cu_l[s + 1] - cu_l[s] for s in shard.seqs]
    new_cu = torch.zeros(len(lens) + 1, dtype=cu.dtype)
    if lens:
        new_cu[1:] = torch.cumsum(torch.tensor(lens, dtype=torch.int64), 0).to(cu.dtype)
    tsel = lambda t: t.index_select(0, tidx)  # noqa: E731
    return [tsel(q)[:, h0 // rep:h1 // rep].contiguous(), tsel(k)[:, h0 // rep:h1 // rep].contiguous(),
            tsel(v)[:, h0:h1].contiguous(),
            None if state is None else state.index_select(0, sidx)[:, h0:h1].contiguous(),
            A_log[h0:h1].contiguous(), tsel(a)[:, h0:h1].contiguous(), dt_bias[h0:h1].contiguous(),
            tsel(b)[:, h0:h1].contiguous(), new_cu.to(cu.device), scale]


def gather_decode(shards, outs, B: int, HV: int, V: int = 128, K: int = 128):
    """Reassemble (output [B,1,HV,V], new_state [B,HV,V,K]) from per-rank results."""
    o = torch.zeros((B, 1, HV, V), dtype=torch.bfloat16)
    s = torch.zeros((B, HV, V, K), dtype=torch.float32)
    for sh, res in zip(shards, outs):
        if sh.empty:
            continue
        so, ss = res
        h0, h1 = sh.heads
        idx = torch.tensor(sh.seqs, dtype=torch.long)
        o[idx, :, h0:h1] = so.cpu()
        s[idx, h0:h1] = ss.cpu()
    return o, s


def gather_prefill(shards, outs, cu, HV: int, V: int = 128, K: int = 128):
    cu_l = [int(x) for x in cu.tolist()]
    N, T = len(cu_l) - 1, cu_l[-1]
    o = torch.zeros((T, HV, V), dtype=torch.bfloat16)
    s = torch.zeros((N, HV, V, K), dtype=torch.float32)
    for sh, res in zip(shards, outs):
        if sh.empty:
            continue
        so, ss = res
        h0, h1 = sh.heads
        pos = 0
        for j, seq in enumerate(sh.seqs):
            n = cu_l[seq + 1] - cu_l[seq]
            o[cu_l[seq]:cu_l[seq + 1], h0:h1] = so[pos:pos + n].cpu()
            s[seq, h0:h1] = ss[j].cpu()
            pos += n
    return o, s


# ---------------------------------------------------------------------------
# host-side failure handling: per-rank deadline, re-run of failed shards

@dataclass(frozen=True)
class ShardFailure:
    rank: int
    kind: str       # "raised" (the rank's work raised) or "timeout" (no result by the deadline)
    detail: str


def run_shards(work, shards, rank: int, world: int, store, timeout_s: float, poll_s: float = 0.02,
               prefix: str = "gdn_shards"):
    """Runs ``work(shard)`` for this rank's shard and reports through ``store``
    (a torch.distributed Store shared by the ranks, e.g. the process group's
    TCPStore; no collective is used, so a rank that hangs or dies cannot
    block the others).

    Every rank publishes its result (pickled) or the error it raised.  Rank 0
    waits until ``timeout_s`` after it has finished its own shard for the
    others, then re-runs every shard whose rank raised or missed the deadline
    itself (a surviving rank, which here holds the full inputs), and returns
    ``(results, failures)``: the per-shard results in rank order and a list of
    ShardFailure.  Other ranks return None once they have published.  Work
    inside a rank stays between kernel launches: a failure is detected on the
    host, never by stalling a GPU kernel."""
    import pickle
    import time

    key = lambda r, what: f"{prefix}/{r}/{what}"  # noqa: E731
    try:
        mine = work(shards[rank])
        store.set(key(rank, "ok"), pickle.dumps(mine))
    except Exception as e:  # noqa: BLE001 - any failure of the work is reported, not raised
        mine = None
        store.set(key(rank, "err"), repr(e)[:500])
        if rank != 0:
            return None
    if rank != 0:
        return None
    results = [None] * world
    failures = []
    pending = set(range(1, world))
    if mine is None:
        failures.append(ShardFailure(0, "raised", store.get(key(0, "err")).decode()))
    else:
        results[0] = mine
    deadline = time.monotonic() + timeout_s
    while pending and time.monotonic() < deadline:
        for r in sorted(pending):
            if store.check([key(r, "ok")]):
                results[r] = pickle.loads(store.get(key(r, "ok")))
                pending.discard(r)
            elif store.check([key(r, "err")]):
                failures.append(ShardFailure(r, "raised", store.get(key(r, "err")).decode()))
                pending.discard(r)
        if pending:
            time.sleep(poll_s)
    for r in sorted(pending):
        failures.append(ShardFailure(r, "timeout", f"no result within {timeout_s:.1f} s"))
    for f in failures:  # re-run each failed shard here, on a surviving rank
        results[f.rank] = work(shards[f.rank])
    return results, sorted(failures, key=lambda f: f.rank)

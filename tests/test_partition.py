"""Sequence x v-head partitioner (no collective): every (sequence, v-head)
recurrence lands on exactly one rank, head groups stay aligned to whole q/k
heads, and running the oracle per shard then gathering reproduces the
single-device result."""
import pytest
import torch

from oracle import oracle
from rocm_flashinfer_contest_b200 import inputs, partition


def _cover(shards, n_seqs, HV):
    seen = torch.zeros(n_seqs, HV, dtype=torch.int32)
    for sh in shards:
        for s in sh.seqs:
            seen[s, sh.heads[0]:sh.heads[1]] += 1
    return seen


@pytest.mark.parametrize("B,H,HV,world", [(64, 16, 32, 1), (64, 16, 32, 2), (1024, 16, 32, 8),
                                           (5, 4, 8, 4), (1, 16, 32, 8), (2, 4, 8, 8), (3, 2, 4, 8)])
def test_plan_decode_covers_each_recurrence_once(B, H, HV, world):
    shards = partition.plan_decode(B, H, HV, world)
    assert len(shards) == world
    assert bool((_cover(shards, B, HV) == 1).all())
    rep = HV // H
    for sh in shards:
        assert sh.heads[0] % rep == 0 and sh.heads[1] % rep == 0
    if B >= world:
        sizes = [len(s.seqs) for s in shards]
        assert max(sizes) - min(sizes) <= 1


@pytest.mark.parametrize("lens,world", [([100, 5, 300, 7, 0, 64], 2), ([8192], 8), ([10] * 16, 4),
                                        ([1, 1024, 3, 500, 77], 8)])
def test_plan_prefill_covers_and_balances(lens, world):
    H, HV = 16, 32
    shards = partition.plan_prefill(lens, H, HV, world)
    assert bool((_cover(shards, len(lens), HV) == 1).all())
    if len(lens) >= world:
        loads = [sum(max(1, lens[s]) for s in sh.seqs) for sh in shards]
        assert max(loads) <= sum(max(1, x) for x in lens) / world + max(lens)


def test_decode_shards_reassemble_the_full_result():
    args = inputs.decode_inputs(6, 2, 4, seed=5)
    full_o, full_s = oracle.decode(*args)
    for world in (2, 4, 8):
        shards = partition.plan_decode(6, 2, 4, world)
        outs = [oracle.decode(*partition.apply_decode(args, sh)) if not sh.empty else None for sh in shards]
        o, s = partition.gather_decode(shards, outs, 6, 4)
        assert torch.equal(o, full_o) and torch.equal(s, full_s)


def test_prefill_shards_reassemble_the_full_result():
    args = inputs.prefill_inputs([40, 0, 13, 70], 2, 4, seed=6)
    full_o, full_s = oracle.prefill(*args)
    for world in (2, 3, 8):
        shards = partition.plan_prefill([40, 0, 13, 70], 2, 4, world)
        outs = [oracle.prefill(*partition.apply_prefill(args, sh)) if not sh.empty else None for sh in shards]
        o, s = partition.gather_prefill(shards, outs, args[8], 4)
        assert torch.equal(o, full_o) and torch.equal(s, full_s)

"""Seeded synthetic inputs for the GDN decode / prefill workloads.

The contest's trace dataset (flashinfer-ai/mlsys26-contest) is not available
offline, so these stand in for it with the shapes and value distributions the
benchmark configurations name: q, k ~ N(0, 1) then L2-normalised per head and
cast to bf16; v, a, b ~ N(0, 1) bf16; A_log ~ U[0, ln 16] fp32;
dt_bias ~ U[-1, 1] fp32; state ~ N(0, 0.1^2) fp32 in k-last layout;
scale = 1/sqrt(128).  Default heads: H = 16 q/k heads, HV = 32 v-heads,
head_size 128 (the contest definitions use H = 4, HV = 8).
"""
from __future__ import annotations

import math

import torch

D = 128


def _gen(seed: int, device) -> torch.Generator:
    g = torch.Generator(device=device)
    g.manual_seed(seed)
    return g


def _normal(shape, g, device, std=1.0):
    return torch.randn(shape, generator=g, device=device, dtype=torch.float32) * std


def _uniform(shape, lo, hi, g, device):
    return torch.rand(shape, generator=g, device=device, dtype=torch.float32) * (hi - lo) + lo


def _l2norm_bf16(x):
    return (x / x.norm(dim=-1, keepdim=True).clamp_min(1e-6)).to(torch.bfloat16)


def decode_inputs(B: int, H: int = 16, HV: int = 32, K: int = D, V: int = D, seed: int = 0,
                  device="cpu", with_state: bool = True, state_std: float = 0.1):
    """Arguments of gdn_decode.run, in order:
    (q, k, v, state, A_log, a, dt_bias, b, scale)."""
    g = _gen(seed, device)
    q = _l2norm_bf16(_normal((B, 1, H, K), g, device))
    k = _l2norm_bf16(_normal((B, 1, H, K), g, device))
    v = _normal((B, 1, HV, V), g, device).to(torch.bfloat16)
    A_log = _uniform((HV,), 0.0, math.log(16.0), g, device)
    a = _normal((B, 1, HV), g, device).to(torch.bfloat16)
    dt_bias = _uniform((HV,), -1.0, 1.0, g, device)
    b = _normal((B, 1, HV), g, device).to(torch.bfloat16)
    state = _normal((B, HV, V, K), g, device, state_std) if with_state else None
    return [q, k, v, state, A_log, a, dt_bias, b, 1.0 / math.sqrt(K)]


def decode_inputs_for(seq_ids, H: int = 16, HV: int = 32, K: int = D, V: int = D, seed: int = 0,
                      device="cpu", state_std: float = 0.1):
    """Decode arguments for the sequences `seq_ids` of one large batch in which
    sequence i is drawn from its own generator (seed, i): any subset, e.g. a
    rank's shard, is materialised alone and equals the same rows of the whole
    batch.  A_log and dt_bias come from the generator `seed`."""
    g = _gen(seed, device)
    A_log = _uniform((HV,), 0.0, math.log(16.0), g, device)
    dt_bias = _uniform((HV,), -1.0, 1.0, g, device)
    rows = []
    for i in seq_ids:
        gi = _gen(seed * 1_000_003 + 7 * int(i) + 1, device)
        rows.append((_l2norm_bf16(_normal((1, 1, H, K), gi, device)),
                     _l2norm_bf16(_normal((1, 1, H, K), gi, device)),
                     _normal((1, 1, HV, V), gi, device).to(torch.bfloat16),
                     _normal((1, HV, V, K), gi, device, state_std),
                     _normal((1, 1, HV), gi, device).to(torch.bfloat16),
                     _normal((1, 1, HV), gi, device).to(torch.bfloat16)))
    cat = [torch.cat([r[j] for r in rows]) if rows else None for j in range(6)]
    q, k, v, state, a, b = cat
    return [q, k, v, state, A_log, a, dt_bias, b, 1.0 / math.sqrt(K)]


def seqlens_split(total: int, num_seqs: int, seed: int):
    """`num_seqs` positive lengths summing to `total` (seeded uniform cut
    points): stands in for a contest workload of which only the total length
    and the sequence count are published."""
    if num_seqs <= 0 or total < num_seqs:
        raise ValueError("need total >= num_seqs > 0")
    g = _gen(seed + 104729, "cpu")
    cuts = sorted(torch.randperm(total - 1, generator=g)[:num_seqs - 1].add(1).tolist())
    bounds = [0] + cuts + [total]
    return [bounds[i + 1] - bounds[i] for i in range(num_seqs)]


def seqlens_uniform(num_seqs: int, lo: int, hi: int, seed: int, max_total: int | None = None):
    """Sequence lengths drawn uniformly from [lo, hi] (seeded); if max_total is
    given, lengths are scaled down so the total stays within it."""
    g = _gen(seed + 7919, "cpu")
    lens = torch.randint(lo, hi + 1, (num_seqs,), generator=g).tolist()
    if max_total is not None and sum(lens) > max_total:
        f = max_total / sum(lens)
        lens = [max(lo, int(x * f)) for x in lens]
        while sum(lens) > max_total:
            i = max(range(len(lens)), key=lambda j: lens[j])
            lens[i] -= 1
    return lens


def prefill_inputs(seqlens, H: int = 16, HV: int = 32, K: int = D, V: int = D, seed: int = 0,
                   device="cpu", with_state: bool = True, state_std: float = 0.1,
                   cu_dtype=torch.int32):
    """Arguments of gdn_prefill.run, in order:
    (q, k, v, state, A_log, a, dt_bias, b, cu_seqlens, scale)."""
    g = _gen(seed, device)
    T, N = int(sum(seqlens)), len(seqlens)
    q = _l2norm_bf16(_normal((T, H, K), g, device))
    k = _l2norm_bf16(_normal((T, H, K), g, device))
    v = _normal((T, HV, V), g, device).to(torch.bfloat16)
    A_log = _uniform((HV,), 0.0, math.log(16.0), g, device)
    a = _normal((T, HV), g, device).to(torch.bfloat16)
    dt_bias = _uniform((HV,), -1.0, 1.0, g, device)
    b = _normal((T, HV), g, device).to(torch.bfloat16)
    state = _normal((N, HV, V, K), g, device, state_std) if with_state else None
    cu = torch.zeros(N + 1, dtype=torch.int64)
    cu[1:] = torch.cumsum(torch.tensor(seqlens, dtype=torch.int64), 0)
    cu = cu.to(cu_dtype).to(device)
    return [q, k, v, state, A_log, a, dt_bias, b, cu, 1.0 / math.sqrt(K)]


def to_device(args, device):
    return [x.to(device) if isinstance(x, torch.Tensor) else x for x in args]


def to_cpu(args):
    return [x.cpu() if isinstance(x, torch.Tensor) else x for x in args]


def mtp_inputs(B: int, T: int, pool_size: int, H: int = 16, HV: int = 32, K: int = D, V: int = D,
               seed: int = 0, device="cpu", state_std: float = 0.1, indices=None,
               idx_dtype=torch.int32, intermediate: bool = False):
    """Arguments of gdn_mtp.run, in order: (q, k, v, initial_state,
    initial_state_indices, A_log, a, dt_bias, b, scale, intermediate_states_buffer).
    Indices default to a seeded permutation of distinct pool slots."""
    g = _gen(seed, device)
    q = _l2norm_bf16(_normal((B, T, H, K), g, device))
    k = _l2norm_bf16(_normal((B, T, H, K), g, device))
    v = _normal((B, T, HV, V), g, device).to(torch.bfloat16)
    A_log = _uniform((HV,), 0.0, math.log(16.0), g, device)
    a = _normal((B, T, HV), g, device).to(torch.bfloat16)
    dt_bias = _uniform((HV,), -1.0, 1.0, g, device)
    b = _normal((B, T, HV), g, device).to(torch.bfloat16)
    pool = _normal((pool_size, HV, V, K), g, device, state_std)
    if indices is None:
        perm = torch.randperm(pool_size, generator=_gen(seed + 1, "cpu"))[:B]
        indices = perm
    idx = torch.as_tensor(indices, dtype=torch.int64).to(idx_dtype).to(device)
    inter = torch.zeros((pool_size, T, HV, V, K), device=device) if intermediate else None
    return [q, k, v, pool, idx, A_log, a, dt_bias, b, 1.0 / math.sqrt(K), inter]

"""Parity of the sm_100a varlen prefill (through the C ABI) with the CPU oracle.

Cases: the benchmark configurations (one 8192-token sequence with a zero
state; 16 sequences of seeded lengths in [1, 1024] with non-zero states), the
contest shape, zero-length sequences, lengths around the 64-token chunk
(1, 63, 64, 65, 127, 129), int32 / int64 cu_seqlens, H == HV, many short
sequences, tokens outside every sequence, in-place update and non-mutation,
state checkpoints, and in-kernel q/k L2 normalisation on raw q/k.
"""
import pytest
import torch

from oracle import oracle
from parity import assert_output_close, assert_state_close
from rocm_flashinfer_contest_b200 import gdn_prefill, inputs

pytestmark = pytest.mark.gpu


@pytest.fixture(params=["chunk2", "chunk3", "chunk4", "recurrent"])
def path(request, monkeypatch):
    """Runs a test through the chunked tensor-core kernels (threshold 0) with
    one chain kernel forced (split-path chain2, transposed chain3, scan over
    per-chunk transitions chain4), or the token-serial kernel (threshold
    above any T used here)."""
    if request.param == "recurrent":
        monkeypatch.setenv("GDN_PREFILL_CHUNK_MIN", "1000000000")
    else:
        monkeypatch.setenv("GDN_PREFILL_CHUNK_MIN", "0")
        monkeypatch.setenv("GDN_PREFILL_CHAIN", request.param[-1])
    return request.param


def _check(args, dev, head_subset=None):
    dargs = inputs.to_device(args, dev)
    o, s = gdn_prefill.run(*dargs)
    torch.cuda.synchronize()
    o, s = o.cpu(), s.cpu()
    cpu = inputs.to_cpu(args)
    if head_subset is not None:
        # v-heads are independent: check the v-heads of q/k head `j` only
        j = head_subset
        q, k, v, st, A_log, a, dt_bias, b, cu, scale = cpu
        H, HV = q.shape[1], v.shape[1]
        rep = HV // H
        hs = slice(j * rep, (j + 1) * rep)
        cpu = [q[:, j:j + 1], k[:, j:j + 1], v[:, hs], None if st is None else st[:, hs],
               A_log[hs], a[:, hs], dt_bias[hs], b[:, hs], cu, scale]
        o, s = o[:, hs], s[:, hs]
    ro, rs = oracle.prefill(*cpu)
    rep_o = assert_output_close(o, ro)
    rep = assert_state_close(s, rs)
    print("parity", rep_o, rep)
    return rep


@pytest.mark.parametrize("lens,H,HV,with_state,cu_dtype", [
    ([64], 4, 8, True, torch.int32),
    ([1], 16, 32, True, torch.int64),
    ([63, 65, 64, 1, 127, 129], 4, 8, True, torch.int32),
    ([5, 0, 17, 0, 1], 4, 8, True, torch.int64),   # zero-length sequences
    ([0], 2, 4, True, torch.int32),                 # only an empty sequence
    ([300, 20], 16, 32, False, torch.int32),        # zero initial state
    ([100, 37], 8, 8, True, torch.int64),           # H == HV
    ([1] * 48, 4, 8, True, torch.int32),            # many one-token sequences
    ([6], 4, 8, True, torch.int32),
    ([139 // 3, 139 // 3, 139 - 2 * (139 // 3)], 4, 8, True, torch.int32),
])
def test_prefill_matches_oracle(cuda_device, path, lens, H, HV, with_state, cu_dtype):
    args = inputs.prefill_inputs(lens, H, HV, seed=sum(lens) + len(lens), with_state=with_state,
                                 cu_dtype=cu_dtype)
    _check(args, cuda_device)


def test_prefill_config3_varlen_16(cuda_device, path):
    """Benchmark config 3: 16 sequences, lengths U[1, 1024], total <= 8192,
    non-zero initial states."""
    lens = inputs.seqlens_uniform(16, 1, 1024, seed=0, max_total=8192)
    args = inputs.prefill_inputs(lens, seed=3)
    _check(args, cuda_device)


def test_prefill_config2_8k(cuda_device, path):
    """Benchmark config 2: one 8192-token sequence, zero initial state, all
    16 q/k heads (32 v-heads) checked against the oracle."""
    args = inputs.prefill_inputs([8192], seed=2, with_state=False)
    _check(args, cuda_device)


@pytest.mark.parametrize("j", [0, 11])
def test_prefill_config2_8k_head_subset(cuda_device, path, j):
    """The oracle restricted to the v-heads of q/k head j (its inputs sliced)
    agrees with the same heads of the full GPU run: heads are independent."""
    args = inputs.prefill_inputs([8192], seed=2, with_state=False)
    _check(args, cuda_device, head_subset=j)


def test_prefill_uncovered_tokens_are_zero(cuda_device, path):
    args = inputs.prefill_inputs([10, 20], 4, 8, seed=21, device=cuda_device)
    cu = args[8]
    # sequences cover tokens [3, 25) of 30; the rest belong to no sequence
    args[8] = torch.tensor([3, 13, 25], dtype=cu.dtype, device=cuda_device)
    o = torch.full((30, 8, 128), 5.0, device=cuda_device).to(torch.bfloat16)
    s = torch.empty((2, 8, 128, 128), device=cuda_device)
    gdn_prefill.run_into(*args, output=o, new_state=s)
    torch.cuda.synchronize()
    assert bool((o[:3] == 0).all()) and bool((o[25:] == 0).all())
    ro, rs = oracle.prefill(*inputs.to_cpu(args))
    assert_output_close(o.cpu(), ro)
    assert_state_close(s.cpu(), rs)


def test_prefill_in_place_and_no_mutation(cuda_device, path):
    args = inputs.prefill_inputs([70, 5, 130], 4, 8, seed=22, device=cuda_device)
    snap = [x.clone() if isinstance(x, torch.Tensor) else x for x in args]
    o1, s1 = gdn_prefill.run(*args)
    torch.cuda.synchronize()
    for x, y in zip(args, snap):
        if isinstance(x, torch.Tensor):
            assert torch.equal(x, y)
    st = args[3].clone()
    o2 = torch.empty_like(o1)
    gdn_prefill.run_into(*args[:3], st, *args[4:], output=o2, new_state=st)
    torch.cuda.synchronize()
    assert torch.equal(o1, o2) and torch.equal(s1, st)


def test_prefill_no_sequences(cuda_device, path):
    args = inputs.prefill_inputs([], 4, 8, device=cuda_device)
    o, s = gdn_prefill.run(*args)
    assert o.shape == (0, 8, 128) and s.shape == (0, 8, 128, 128)


def test_prefill_device_status_clean(cuda_device):
    """No bounded wait in the tensor-core kernel ran out during the suite."""
    from rocm_flashinfer_contest_b200 import _lib
    torch.cuda.synchronize()
    assert _lib.lib().gdn_device_status(1) == 0


def test_prefill_strong_decay_and_saturated_gates(cuda_device, path):
    """Very strong decay (A_log = ln 16 with large a) and saturated beta: every
    in-chunk factor e^{gamma_i - gamma_j} underflows towards 0 without overflow."""
    args = inputs.prefill_inputs([200, 70], 4, 8, seed=31)
    T = 270
    pat_a = torch.tensor([25.0, -30.0, 19.5, 0.0, -5.0, 40.0, 8.0, 3.0])
    pat_b = torch.tensor([30.0, -30.0, 8.0, -8.0, 0.0, 1.0, -1.0, 15.0])
    args[4] = torch.full((8,), 2.77)
    args[5] = pat_a.repeat(T).view(T, 8).to(torch.bfloat16)
    args[7] = pat_b.repeat(T).view(T, 8).to(torch.bfloat16)
    _check(args, cuda_device)


# ---- state checkpoints (flashinfer's chunk_gated_delta_rule checkpoint arguments) ----

@pytest.mark.parametrize("lens,H,HV,every", [
    ([130, 0, 200, 64], 4, 8, 64),        # tails, an empty sequence, an exact multiple
    ([300, 127, 128], 4, 8, 128),         # a sequence shorter than `every`
    ([1000, 513], 16, 32, 192),           # benchmark heads, every = 3 chunks
    ([640], 4, 8, 64),                    # last checkpoint == final state
])
def test_prefill_checkpoints(cuda_device, path, lens, H, HV, every):
    args = inputs.prefill_inputs(lens, H, HV, seed=sum(lens) + every, with_state=True,
                                 cu_dtype=torch.int64)
    dargs = inputs.to_device(args, cuda_device)
    starts = gdn_prefill.checkpoint_cu_starts_for(dargs[8], every)
    total = int(starts[-1])
    ck = torch.full((total, HV, 128, 128), 7.0, device=cuda_device)
    o, s = gdn_prefill.run(*dargs, state_checkpoints=ck, checkpoint_cu_starts=starts,
                           checkpoint_every_n_tokens=every)
    torch.cuda.synchronize()
    ro, rs, rck = oracle.prefill(*inputs.to_cpu(args), checkpoint_every_n_tokens=every)
    assert total == rck.shape[0] == sum(L // every for L in lens)
    assert_output_close(o.cpu(), ro)
    assert_state_close(s.cpu(), rs)
    assert_state_close(ck.cpu(), rck, what="checkpoints")
    # a sequence whose length is a multiple of `every` ends on its final state
    st = starts.tolist()
    for n, L in enumerate(lens):
        if L and L % every == 0:
            assert torch.equal(ck[st[n + 1] - 1], s[n])


def test_prefill_checkpoint_arguments(cuda_device):
    args = inputs.to_device(inputs.prefill_inputs([128], 4, 8, seed=5), cuda_device)
    starts = gdn_prefill.checkpoint_cu_starts_for(args[8], 64)
    ck = torch.zeros((2, 8, 128, 128), device=cuda_device)
    with pytest.raises(ValueError):
        gdn_prefill.run(*args, state_checkpoints=ck, checkpoint_cu_starts=starts, checkpoint_every_n_tokens=96)
    with pytest.raises(ValueError):
        gdn_prefill.run(*args, state_checkpoints=ck, checkpoint_every_n_tokens=64)
    with pytest.raises(ValueError):
        gdn_prefill.run(*args, state_checkpoints=ck, checkpoint_cu_starts=starts)


# ---- in-kernel q/k L2 normalisation (use_qk_l2norm_in_kernel) ----

def _raw_qk(args, seed):
    """Replace the (unit-norm) q and k by raw bf16 vectors of norm ~34."""
    g = torch.Generator().manual_seed(seed)
    for i in (0, 1):
        args[i] = (torch.randn(args[i].shape, generator=g) * 3.0).to(torch.bfloat16)
    return args


@pytest.mark.parametrize("lens,H,HV,with_state", [
    ([200, 0, 64, 129], 4, 8, True),     # chunk tails, an empty sequence, cross-chunk Gram tiles
    ([1, 63, 65], 16, 32, True),          # benchmark heads, lengths around one chunk
    ([300], 2, 2, False),                 # H == HV, zero initial state
])
def test_prefill_qk_l2norm_matches_oracle(cuda_device, path, lens, H, HV, with_state):
    args = _raw_qk(inputs.prefill_inputs(lens, H, HV, seed=400 + sum(lens), with_state=with_state,
                                         cu_dtype=torch.int64), 500 + sum(lens))
    o, s = gdn_prefill.run(*inputs.to_device(args, cuda_device), use_qk_l2norm_in_kernel=True)
    torch.cuda.synchronize()
    ro, rs = oracle.prefill(*inputs.to_cpu(args), qk_l2norm=True)
    print("parity", assert_output_close(o.cpu(), ro), assert_state_close(s.cpu(), rs))


def test_prefill_qk_l2norm_on_unit_vectors_is_the_plain_run(cuda_device, path):
    """Inputs that are already unit vectors: the flag changes (almost) nothing."""
    args = inputs.to_device(inputs.prefill_inputs([190, 70], 4, 8, seed=41), cuda_device)
    o0, s0 = gdn_prefill.run(*args)
    o1, s1 = gdn_prefill.run(*args, use_qk_l2norm_in_kernel=True)
    torch.cuda.synchronize()
    assert_output_close(o1.cpu(), o0.cpu())
    assert_state_close(s1.cpu(), s0.cpu())


def test_prefill_qk_l2norm_with_checkpoints(cuda_device, path):
    lens, every = [260, 64, 0, 131], 64
    args = _raw_qk(inputs.prefill_inputs(lens, 4, 8, seed=43, with_state=True, cu_dtype=torch.int64), 44)
    dargs = inputs.to_device(args, cuda_device)
    starts = gdn_prefill.checkpoint_cu_starts_for(dargs[8], every)
    ck = torch.full((int(starts[-1]), 8, 128, 128), 7.0, device=cuda_device)
    o, s = gdn_prefill.run(*dargs, state_checkpoints=ck, checkpoint_cu_starts=starts,
                           checkpoint_every_n_tokens=every, use_qk_l2norm_in_kernel=True)
    torch.cuda.synchronize()
    ro, rs, rck = oracle.prefill(*inputs.to_cpu(args), checkpoint_every_n_tokens=every, qk_l2norm=True)
    assert_output_close(o.cpu(), ro)
    assert_state_close(s.cpu(), rs)
    assert_state_close(ck.cpu(), rck, what="checkpoints")

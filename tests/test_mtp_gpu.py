"""Parity of the sm_100a pool-indexed multi-token decode kernel (gdn_mtp_fwd,
through the C ABI) with the CPU oracle and the golden fixtures.

Cases: the golden K = 128 fixture; the contest shape and the benchmark heads
at T = 1..8; int32 and int64 indices; padding entries (-1 and pool_size);
intermediate-state buffers with cache_steps > T and fewer slots than the
pool; untouched pool slots; the in-place / no-update / L2-norm modes of the
flashinfer-style API; T = 1 against the single-token decode kernel.
"""
import os

import numpy as np
import pytest
import torch

from oracle import oracle
from parity import assert_output_close, assert_state_close, bf16_from_u16
from rocm_flashinfer_contest_b200 import gdn_decode, gdn_mtp, inputs

pytestmark = pytest.mark.gpu

GOLD = os.path.join(os.path.dirname(__file__), "golden", "gdn_golden.npz")
FIELDS = ("q", "k", "v", "initial_state", "initial_state_indices", "A_log", "a", "dt_bias", "b")


def _oracle(args, buf=None, l2=False):
    cpu = inputs.to_cpu(args[:10])
    rb = None if buf is None else torch.zeros(buf.shape)
    ro, rs = oracle.mtp(*cpu, rb, qk_l2norm=l2)
    return ro, rs, rb


def test_mtp_matches_golden(cuda_device):
    z = np.load(GOLD)
    name = "mtp_k128"
    args = []
    for f in FIELDS:
        a = z[f"{name}/{f}"]
        args.append(bf16_from_u16(a) if f in ("q", "k", "v", "a", "b") else torch.from_numpy(np.array(a)))
    dargs = inputs.to_device(args, cuda_device)
    o, s = gdn_mtp.run(*dargs, float(z[f"{name}/scale"]))
    torch.cuda.synchronize()
    assert_output_close(o.cpu(), bf16_from_u16(z[f"{name}/out"]))
    assert_state_close(s.cpu(), torch.from_numpy(z[f"{name}/new_state"]))


@pytest.mark.parametrize("B,T,pool,H,HV,idx_dtype,inter,seed", [
    (8, 4, 16, 4, 8, torch.int32, True, 0),      # contest heads, spec-decode T = 4
    (8, 2, 8, 4, 8, torch.int64, False, 1),
    (64, 4, 128, 16, 32, torch.int32, True, 2),  # benchmark heads, B = 64
    (3, 1, 5, 16, 32, torch.int64, True, 3),     # T = 1: pool-indexed decode
    (5, 8, 9, 1, 4, torch.int32, False, 4),      # GVA 4, long draft
    (40, 3, 40, 16, 32, torch.int64, False, 5),  # above the small-grid threshold
    (24, 6, 30, 16, 32, torch.int32, True, 6),   # two chunks of the chunk form, the second padded
    (6, 5, 6, 4, 8, torch.int64, True, 7),       # a chunk of four and one of a single token
])
def test_mtp_matches_oracle(cuda_device, B, T, pool, H, HV, idx_dtype, inter, seed):
    args = inputs.mtp_inputs(B, T, pool, H, HV, seed=seed, idx_dtype=idx_dtype, intermediate=inter)
    dargs = inputs.to_device(args, cuda_device)
    pool_before = dargs[3].clone()
    o, s = gdn_mtp.run(*dargs[:10], intermediate_states_buffer=dargs[10])
    torch.cuda.synchronize()
    assert torch.equal(dargs[3], pool_before)  # the definition does not modify its inputs
    ro, rs, rb = _oracle(args, args[10])
    assert o.shape == (B, T, HV, 128) and o.dtype == torch.bfloat16
    assert_output_close(o.cpu(), ro)
    assert_state_close(s.cpu(), rs)
    used = set(args[4].tolist())
    for slot in range(pool):
        if slot not in used:
            assert torch.equal(s[slot].cpu(), args[3][slot])
    if inter:
        for slot in used:
            assert_state_close(dargs[10][slot].cpu(), rb[slot], what=f"intermediate[{slot}]")


def test_mtp_padding(cuda_device):
    B, T, pool = 6, 3, 8
    idx = [3, -1, 0, 8, 5, -7]  # -1, pool_size and another negative are padding
    args = inputs.mtp_inputs(B, T, pool, 4, 8, seed=20, indices=idx, idx_dtype=torch.int64,
                             intermediate=True)
    dargs = inputs.to_device(args, cuda_device)
    dargs[10].fill_(7.0)
    out = torch.full((B, T, 8, 128), 3.0, dtype=torch.bfloat16, device=cuda_device)
    fs = torch.empty_like(dargs[3])
    gdn_mtp.run_into(*dargs[:10], out, fs, intermediate_states_buffer=dargs[10])
    torch.cuda.synchronize()
    ro, rs, _ = _oracle(args)
    assert_output_close(out.cpu(), ro)
    for b in (1, 3, 5):
        assert not out[b].float().any()
    assert_state_close(fs.cpu(), rs)
    for slot in (1, 2, 4, 6, 7):  # not named: pool copied, buffer untouched
        assert torch.equal(fs[slot].cpu(), args[3][slot])
        assert bool((dargs[10][slot] == 7.0).all())


def test_mtp_intermediate_layout(cuda_device):
    """cache_steps > T and a buffer with fewer slots than the pool."""
    B, T, pool = 4, 3, 6
    idx = [5, 1, 3, 0]
    args = inputs.mtp_inputs(B, T, pool, 4, 8, seed=21, indices=idx)
    dargs = inputs.to_device(args, cuda_device)
    buf = torch.full((4, T + 2, 8, 128, 128), -1.0, device=cuda_device)  # slots 0..3 only
    o, s = gdn_mtp.run(*dargs[:10], intermediate_states_buffer=buf)
    torch.cuda.synchronize()
    ro, rs, _ = _oracle(args)
    assert_output_close(o.cpu(), ro)
    assert_state_close(s.cpu(), rs)
    ref_buf = torch.zeros((pool, T + 2, 8, 128, 128))
    oracle.mtp(*inputs.to_cpu(args[:10]), ref_buf)
    for slot in (0, 1, 3):
        assert_state_close(buf[slot, :T].cpu(), ref_buf[slot, :T])
        assert bool((buf[slot, T:] == -1.0).all())
    assert bool((buf[2] == -1.0).all())
    # the last snapshot is the final state
    assert torch.equal(buf[1, T - 1], s[1])


@pytest.mark.parametrize("B,T,pool,H,HV", [(6, 4, 10, 4, 8), (6, 2, 6, 4, 8), (40, 5, 40, 16, 32)])
def test_mtp_flashinfer_api_modes(cuda_device, B, T, pool, H, HV):
    args = inputs.mtp_inputs(B, T, pool, H, HV, seed=30)
    # raw (unnormalised) q, k for use_qk_l2norm
    g = torch.Generator().manual_seed(31)
    args[0] = (torch.randn(args[0].shape, generator=g) * 2.5).to(torch.bfloat16)
    args[1] = (torch.randn(args[1].shape, generator=g) * 2.5).to(torch.bfloat16)
    dargs = inputs.to_device(args, cuda_device)
    ro, rs, _ = _oracle(args, l2=True)

    pool_dev = dargs[3].clone()
    o, ret = gdn_mtp.gated_delta_rule_mtp(*dargs[:3], pool_dev, *dargs[4:10],
                                          disable_state_update=True, use_qk_l2norm=True)
    torch.cuda.synchronize()
    assert ret is pool_dev and torch.equal(pool_dev, dargs[3])
    assert_output_close(o.cpu(), ro)

    out = torch.empty((B, T, HV, 128), dtype=torch.bfloat16, device=cuda_device)
    o2, ret = gdn_mtp.gated_delta_rule_mtp(*dargs[:3], pool_dev, *dargs[4:9], scale=None, output=out,
                                           disable_state_update=False, use_qk_l2norm=True)
    torch.cuda.synchronize()
    assert o2 is out and ret is pool_dev
    assert_output_close(out.cpu(), ro)
    assert_state_close(pool_dev.cpu(), rs)


def test_mtp_t1_equals_decode(cuda_device):
    """T = 1 with the identity slot map is the single-token decode step: same
    formula and summation order, so the results agree to rounding."""
    B, H, HV = 16, 16, 32
    d = inputs.to_device(inputs.decode_inputs(B, H, HV, seed=40), cuda_device)
    o_dec, s_dec = gdn_decode.run(*d)
    idx = torch.arange(B, dtype=torch.int32, device=cuda_device)
    o_mtp, s_mtp = gdn_mtp.run(*d[:3], d[3], idx, *d[4:8], d[8])
    torch.cuda.synchronize()
    assert float((o_dec.float() - o_mtp.float()).abs().max()) <= 2 ** -7 * float(o_dec.float().abs().max())
    assert torch.allclose(s_dec, s_mtp, rtol=1e-6, atol=1e-7)


def test_mtp_empty_and_bad_args(cuda_device):
    args = inputs.to_device(inputs.mtp_inputs(0, 2, 4, 4, 8, seed=50), cuda_device)
    o, s = gdn_mtp.run(*args[:10])
    torch.cuda.synchronize()
    assert o.shape == (0, 2, 8, 128)
    assert torch.equal(s, args[3])  # the new pool is a copy
    args = inputs.to_device(inputs.mtp_inputs(2, 2, 4, 4, 8, seed=51), cuda_device)
    with pytest.raises(ValueError):
        gdn_mtp.run(*args[:4], args[4].float(), *args[5:10])
    with pytest.raises(ValueError):
        gdn_mtp.run(*args[:10], intermediate_states_buffer=torch.zeros((4, 1, 8, 128, 128),
                                                                       device=cuda_device))


# ---- bf16 state, output slots and flashinfer's decode API ----

def _bf16_tol(sol, ref):
    """bf16 state: within one bf16 rounding step of the oracle's bf16 value."""
    s, r = sol.float().cpu(), ref.float()
    d = (s - r).abs()
    assert sol.dtype == torch.bfloat16
    assert bool((d <= 1e-7 + 2 ** -7 * r.abs()).all()), float(d.max())
    assert float((d == 0).float().mean()) >= 0.97


@pytest.mark.parametrize("B,T,pool,H,HV,seed", [
    (64, 1, 96, 16, 32, 60),   # bf16-state decode at the benchmark heads
    (8, 4, 12, 4, 8, 61),      # bf16-state MTP, contest heads
    (5, 2, 5, 1, 4, 62),       # GVA 4, small grid
    (32, 4, 40, 16, 32, 63),   # 64-row CTAs (large grid), chunk of four
    (32, 2, 32, 16, 32, 64),   # 64-row CTAs, chunk of two
    (20, 7, 24, 16, 32, 65),   # 32-row CTAs, two chunks
])
def test_mtp_bf16_state_matches_oracle(cuda_device, B, T, pool, H, HV, seed):
    args = inputs.mtp_inputs(B, T, pool, H, HV, seed=seed)
    args[3] = args[3].to(torch.bfloat16)
    dargs = inputs.to_device(args, cuda_device)
    o, s = gdn_mtp.run(*dargs[:10])
    torch.cuda.synchronize()
    ro, rs = oracle.mtp(*inputs.to_cpu(args[:10]))
    assert s.dtype == torch.bfloat16 and rs.dtype == torch.bfloat16
    assert_output_close(o.cpu(), ro)
    _bf16_tol(s, rs)


def test_mtp_golden_bf16_state(cuda_device):
    z = np.load(GOLD)
    name = "mtp_bf16state_t1"
    args = []
    for f in FIELDS:
        a = z[f"{name}/{f}"]
        bf = f in ("q", "k", "v", "a", "b", "initial_state")
        args.append(bf16_from_u16(a) if bf else torch.from_numpy(np.array(a)))
    o, s = gdn_mtp.run(*inputs.to_device(args, cuda_device), float(z[f"{name}/scale"]))
    torch.cuda.synchronize()
    assert_output_close(o.cpu(), bf16_from_u16(z[f"{name}/out"]))
    _bf16_tol(s, bf16_from_u16(z[f"{name}/new_state"]))


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("form", ["", "stream", "chunk"])
def test_mtp_output_state_indices(cuda_device, monkeypatch, dtype, form):
    if form:
        monkeypatch.setenv("GDN_MTP_FORM", form)
    B, T, pool = 4, 2, 10
    idx = [1, 3, -1, 6]
    oidx = [7, 2, 5, 11]          # entry 3 writes out of range: no state write
    args = inputs.mtp_inputs(B, T, pool, 4, 8, seed=63, indices=idx, idx_dtype=torch.int64)
    args[3] = args[3].to(dtype)
    dargs = inputs.to_device(args, cuda_device)
    out_idx = torch.tensor(oidx, dtype=torch.int32, device=cuda_device)
    pool_dev = dargs[3].clone()
    out = torch.empty((B, T, 8, 128), dtype=torch.bfloat16, device=cuda_device)
    gdn_mtp.run_into(*dargs[:3], pool_dev, *dargs[4:10], out, pool_dev, output_state_indices=out_idx)
    torch.cuda.synchronize()
    ro, rs = oracle.mtp(*inputs.to_cpu(args[:10]), output_state_indices=out_idx.cpu())
    assert_output_close(out.cpu(), ro)
    if dtype == torch.bfloat16:
        _bf16_tol(pool_dev, rs)
    else:
        assert_state_close(pool_dev.cpu(), rs)
    for slot in (0, 1, 3, 4, 6, 8, 9):   # read-only or untouched slots keep their value
        assert torch.equal(pool_dev[slot].cpu(), args[3][slot])


@pytest.mark.parametrize("dtype,T", [(torch.float32, 1), (torch.bfloat16, 1), (torch.bfloat16, 3)])
def test_decode_pretranspose_api(cuda_device, dtype, T):
    B, H, HV = 6, 4, 8
    args = inputs.mtp_inputs(B, T, B, H, HV, seed=64, indices=list(range(B)))
    g = torch.Generator().manual_seed(65)
    args[0] = (torch.randn(args[0].shape, generator=g) * 2.0).to(torch.bfloat16)
    args[1] = (torch.randn(args[1].shape, generator=g) * 2.0).to(torch.bfloat16)
    args[3] = args[3].to(dtype)
    ro, rs = oracle.mtp(*inputs.to_cpu(args[:10]), qk_l2norm=True)
    d = inputs.to_device(args, cuda_device)
    state = d[3].clone()
    o, ret = gdn_decode.gated_delta_rule_decode_pretranspose(
        d[0], d[1], d[2], state, d[5], d[6], d[7], d[8])        # scale=None, use_qk_l2norm=True
    torch.cuda.synchronize()
    assert ret is state and o.shape == (B, T, HV, 128)
    assert_output_close(o.cpu(), ro)
    if dtype == torch.bfloat16:
        _bf16_tol(state, rs)
    else:
        assert_state_close(state.cpu(), rs)


def test_decode_pretranspose_pool_mode(cuda_device):
    B, pool, H, HV = 5, 9, 16, 32
    idx = [4, -1, 0, 7, 2]
    args = inputs.mtp_inputs(B, 1, pool, H, HV, seed=66, indices=idx, idx_dtype=torch.int64)
    args[3] = args[3].to(torch.bfloat16)
    d = inputs.to_device(args, cuda_device)
    pool_dev = d[3].clone()
    out = torch.empty((B, 1, HV, 128), dtype=torch.bfloat16, device=cuda_device)
    o, ret = gdn_decode.gated_delta_rule_decode_pretranspose(
        d[0], d[1], d[2], None, d[5], d[6], d[7], d[8], scale=0.0, output=out, use_qk_l2norm=False,
        initial_state=pool_dev, initial_state_indices=d[4])
    torch.cuda.synchronize()
    assert o is out and ret is pool_dev
    ro, rs = oracle.mtp(*inputs.to_cpu(args[:10]))
    assert_output_close(out.cpu(), ro)
    assert not out[1].float().any()
    _bf16_tol(pool_dev, rs)


@pytest.mark.parametrize("T,steps,rows_entries", [(4, 4, 6), (3, 5, 4), (2, 2, 3), (1, 1, 6)])
@pytest.mark.parametrize("form", ["", "stream"])
def test_mtp_serving_api_snapshots_by_entry(cuda_device, monkeypatch, T, steps, rows_entries, form):
    """gated_delta_rule_mtp puts snapshots where flashinfer's kernel does: batch
    entry i, token t at row i * T + t of the buffer seen as [slots * steps]
    rows (buffer[i, t] when steps == T); padding entries and entries whose T
    rows do not fit write nothing."""
    if form:
        monkeypatch.setenv("GDN_MTP_FORM", form)
    B, pool, H, HV = 6, 10, 4, 8
    idx = [7, -1, 2, 9, 0, 4]
    args = inputs.mtp_inputs(B, T, pool, H, HV, seed=60 + T, indices=idx)
    slots = max(1, rows_entries * T // steps)
    buf = torch.full((slots, steps, HV, 128, 128), -3.0)
    _, _ = oracle.mtp(*args[:10], intermediate_states_buffer=buf, snapshots_by_entry=True)
    ro, rs = oracle.mtp(*args[:10])
    dargs = inputs.to_device(args, cuda_device)
    dbuf = torch.full((slots, steps, HV, 128, 128), -3.0, device=cuda_device)
    pool_dev = dargs[3].clone()
    o, _ = gdn_mtp.gated_delta_rule_mtp(*dargs[:3], pool_dev, *dargs[4:10], intermediate_states_buffer=dbuf,
                                        disable_state_update=False, use_qk_l2norm=False)
    torch.cuda.synchronize()
    assert_output_close(o.cpu(), ro)
    assert_state_close(pool_dev.cpu(), rs)
    got, want = dbuf.cpu().view(-1, HV, 128, 128), buf.view(-1, HV, 128, 128)
    untouched = want == -3.0
    assert torch.equal(untouched, got == -3.0)   # the same rows written
    assert_state_close(got[~untouched.all(-1).all(-1).all(-1)], want[~untouched.all(-1).all(-1).all(-1)],
                       what="snapshots")


# ---- every T > 1 kernel form, whatever the default routing picks ----

@pytest.mark.parametrize("form", ["stream", "staged", "chunk"])
@pytest.mark.parametrize("dtype,B,T,inter,l2,seed", [
    (torch.float32, 40, 2, False, False, 70),   # benchmark heads, above the small-grid threshold
    (torch.float32, 40, 4, True, False, 71),    # snapshots
    (torch.float32, 40, 6, False, True, 72),    # two chunks / stages, L2 norm
    (torch.bfloat16, 40, 3, False, False, 73),
    (torch.bfloat16, 40, 8, False, True, 74),
])
def test_mtp_forms_match_oracle(cuda_device, monkeypatch, form, dtype, B, T, inter, l2, seed):
    monkeypatch.setenv("GDN_MTP_FORM", form)
    pool = B + 3
    idx = list(range(1, B)) + [-1]  # the last entry is padding
    args = inputs.mtp_inputs(B, T, pool, 16, 32, seed=seed, indices=idx, intermediate=inter and dtype == torch.float32,
                             idx_dtype=torch.int64 if seed % 2 else torch.int32)  # both index widths
    if l2:
        g = torch.Generator().manual_seed(seed + 100)
        args[0] = (torch.randn(args[0].shape, generator=g) * 2.0).to(torch.bfloat16)
        args[1] = (torch.randn(args[1].shape, generator=g) * 2.0).to(torch.bfloat16)
    args[3] = args[3].to(dtype)
    dargs = inputs.to_device(args, cuda_device)
    pool_dev = dargs[3].clone()
    out = torch.empty((B, T, 32, 128), dtype=torch.bfloat16, device=cuda_device)
    gdn_mtp.run_into(*dargs[:3], pool_dev, *dargs[4:10], out, pool_dev,
                     intermediate_states_buffer=dargs[10], qk_l2norm=l2)
    torch.cuda.synchronize()
    rb = None if args[10] is None else torch.zeros(args[10].shape)
    ro, rs = oracle.mtp(*inputs.to_cpu(args[:10]), rb, qk_l2norm=l2)
    assert_output_close(out.cpu(), ro)
    assert bool((out[-1] == 0).all())  # padding entry: zero output
    if dtype == torch.float32:
        assert_state_close(pool_dev.cpu(), rs)
    else:
        _bf16_tol(pool_dev, rs)
    assert torch.equal(pool_dev[0].cpu(), args[3][0])  # a slot no entry reads is untouched
    if rb is not None:
        for slot in range(1, B):
            assert_state_close(dargs[10][slot].cpu(), rb[slot], what=f"intermediate[{slot}]")

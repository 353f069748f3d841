"""Parity of the sm_100a decode kernel (through the C ABI) with the CPU oracle.

Cases cover the benchmark configurations (B = 1, 64 and 1024 with H = 16,
HV = 32), the contest shape (H = 4, HV = 8), H == HV, a zero initial state,
scale given as a tensor / 0, saturated gates, in-place update, non-mutation
of inputs, guard regions around the outputs, a side stream and CUDA-graph
replay.
"""
import math

import pytest
import torch

from oracle import oracle
from parity import assert_output_close, assert_state_close
from rocm_flashinfer_contest_b200 import gdn_decode, inputs

pytestmark = pytest.mark.gpu


def _run_both(args, dev):
    dargs = inputs.to_device(args, dev)
    o, s = gdn_decode.run(*dargs)
    torch.cuda.synchronize()
    ro, rs = oracle.decode(*inputs.to_cpu(args))
    return o.cpu(), s.cpu(), ro, rs


@pytest.mark.parametrize("B,H,HV,with_state,seed", [
    (1, 16, 32, True, 0),      # benchmark config 0
    (64, 16, 32, True, 1),     # benchmark config 1
    (1, 4, 8, True, 2),        # contest shape qk4_v8
    (48, 4, 8, True, 3),
    (5, 1, 1, True, 4),        # H == HV == 1
    (3, 2, 8, True, 5),        # GVA ratio 4
    (7, 16, 32, False, 6),     # zero initial state
    (2, 8, 8, True, 7),        # H == HV
    (9, 16, 32, True, 8),      # B*HV below the small-batch threshold
])
def test_decode_matches_oracle(cuda_device, B, H, HV, with_state, seed):
    args = inputs.decode_inputs(B, H, HV, seed=seed, with_state=with_state)
    o, s, ro, rs = _run_both(args, cuda_device)
    assert o.shape == (B, 1, HV, 128) and o.dtype == torch.bfloat16
    assert s.shape == (B, HV, 128, 128) and s.dtype == torch.float32
    assert_output_close(o, ro)
    assert_state_close(s, rs)


@pytest.mark.parametrize("scale", [0.0, 0.5, "tensor"])
def test_decode_scale_forms(cuda_device, scale):
    args = inputs.decode_inputs(4, 4, 8, seed=11)
    args[8] = torch.tensor(0.3, device=cuda_device) if scale == "tensor" else scale
    o, s = gdn_decode.run(*inputs.to_device(args, cuda_device))
    cpu = inputs.to_cpu(args)
    ro, rs = oracle.decode(*cpu)
    assert_output_close(o.cpu(), ro)
    assert_state_close(s.cpu(), rs)


def test_decode_saturated_gates(cuda_device):
    args = inputs.decode_inputs(4, 4, 8, seed=12)
    pat_a = torch.tensor([25.0, -30.0, 19.5, 0.0, -5.0, 40.0, 21.0, -21.0])
    pat_b = torch.tensor([30.0, -30.0, 8.0, -8.0, 0.0, 1.0, -1.0, 15.0])
    args[5] = pat_a.repeat(4).view(4, 1, 8).to(torch.bfloat16)
    args[7] = pat_b.repeat(4).view(4, 1, 8).to(torch.bfloat16)
    o, s, ro, rs = _run_both(args, cuda_device)
    assert_output_close(o, ro)
    assert_state_close(s, rs)


def test_decode_large_batch_sampled(cuda_device):
    """Benchmark config 4 (B = 1024) on one GPU; batch entries are independent,
    so a seeded sample of them is checked against the oracle."""
    B = 1024
    args = inputs.decode_inputs(B, seed=13, device=cuda_device)
    o, s = gdn_decode.run(*args)
    torch.cuda.synchronize()
    pick = torch.randperm(B, generator=torch.Generator().manual_seed(0))[:24].tolist()
    sub = [x[pick] if isinstance(x, torch.Tensor) and x.dim() > 1 else x for x in args]
    ro, rs = oracle.decode(*inputs.to_cpu(sub))
    assert_output_close(o[pick].cpu(), ro)
    assert_state_close(s[pick].cpu(), rs)


def test_decode_in_place_equals_out_of_place(cuda_device):
    args = inputs.decode_inputs(16, seed=14, device=cuda_device)
    o1, s1 = gdn_decode.run(*args)
    st = args[3].clone()
    o2 = torch.empty_like(o1)
    gdn_decode.run_into(*args[:3], st, *args[4:], output=o2, new_state=st)
    torch.cuda.synchronize()
    assert torch.equal(o1, o2)
    assert torch.equal(s1, st)


def test_decode_does_not_mutate_inputs(cuda_device):
    args = inputs.decode_inputs(8, seed=15, device=cuda_device)
    snap = [x.clone() if isinstance(x, torch.Tensor) else x for x in args]
    gdn_decode.run(*args)
    torch.cuda.synchronize()
    for x, y in zip(args, snap):
        if isinstance(x, torch.Tensor):
            assert torch.equal(x, y)


def test_decode_guard_regions_untouched(cuda_device):
    B, HV = 3, 8
    args = inputs.decode_inputs(B, 4, HV, seed=16, device=cuda_device)
    pad = 4096
    n_o, n_s = B * HV * 128, B * HV * 128 * 128
    ob = torch.full((n_o + 2 * pad,), 7.0, device=cuda_device).to(torch.bfloat16)
    sb = torch.full((n_s + 2 * pad,), -3.0, device=cuda_device)
    o = ob[pad:pad + n_o].view(B, 1, HV, 128)
    s = sb[pad:pad + n_s].view(B, HV, 128, 128)
    gdn_decode.run_into(*args, output=o, new_state=s)
    torch.cuda.synchronize()
    assert bool((ob[:pad] == 7.0).all()) and bool((ob[-pad:] == 7.0).all())
    assert bool((sb[:pad] == -3.0).all()) and bool((sb[-pad:] == -3.0).all())
    ro, rs = oracle.decode(*inputs.to_cpu(args))
    assert_output_close(o.cpu(), ro)
    assert_state_close(s.cpu(), rs)


def test_decode_on_side_stream_and_graph(cuda_device):
    args = inputs.decode_inputs(32, seed=17, device=cuda_device)
    ref_o, ref_s = gdn_decode.run(*args)
    side = torch.cuda.Stream()
    out = torch.empty_like(ref_o)
    ns = torch.empty_like(ref_s)
    with torch.cuda.stream(side):
        gdn_decode.run_into(*args, output=out, new_state=ns)
    side.synchronize()
    assert torch.equal(out, ref_o) and torch.equal(ns, ref_s)
    out.zero_()
    ns.zero_()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        gdn_decode.run_into(*args, output=out, new_state=ns)
    g.replay()
    torch.cuda.synchronize()
    assert torch.equal(out, ref_o) and torch.equal(ns, ref_s)


def test_decode_empty_batch(cuda_device):
    args = inputs.decode_inputs(0, 4, 8, device=cuda_device)
    o, s = gdn_decode.run(*args)
    assert o.shape == (0, 1, 8, 128) and s.shape == (0, 8, 128, 128)


def test_decode_rejects_unsupported_head_size(cuda_device):
    args = inputs.decode_inputs(2, 1, 2, K=64, V=64, device=cuda_device)
    with pytest.raises(RuntimeError, match="unsupported"):
        gdn_decode.run(*args)


def test_decode_default_scale_value(cuda_device):
    args = inputs.decode_inputs(2, 1, 2, seed=18, device=cuda_device)
    args[8] = 0.0
    o0, _ = gdn_decode.run(*args)
    args[8] = 1 / math.sqrt(128)
    o1, _ = gdn_decode.run(*args)
    assert torch.equal(o0, o1)


@pytest.mark.parametrize("B,with_state,chunks", [(64, True, 8), (64, True, 0), (13, True, 4), (13, True, 3),
                                                  (5, False, 8), (1, True, 0), (3, True, 1)])
def test_decode_host_buffers_match_device_run(cuda_device, B, with_state, chunks):
    """run_host_into (pinned host tensors, chunked copies both ways) gives
    exactly the device run's results and leaves its inputs untouched."""
    args = inputs.decode_inputs(B, 16, 32, seed=70 + B, with_state=with_state)
    host = [x.pin_memory() if isinstance(x, torch.Tensor) else x for x in args]
    before = [x.clone() if isinstance(x, torch.Tensor) else x for x in host]
    out = torch.empty((B, 1, 32, 128), dtype=torch.bfloat16).pin_memory()
    ns = torch.full((B, 32, 128, 128), float("nan")).pin_memory()
    gdn_decode.run_host_into(*host, out, ns, device=cuda_device, chunks=chunks)
    torch.cuda.current_stream(cuda_device).synchronize()
    ro, rs = gdn_decode.run(*inputs.to_device(args, cuda_device))
    torch.cuda.synchronize()
    assert torch.equal(out, ro.cpu())
    assert torch.equal(ns, rs.cpu())
    for x, y in zip(host, before):
        if isinstance(x, torch.Tensor):
            assert torch.equal(x, y)


def test_decode_host_buffers_reject_unpinned(cuda_device):
    args = inputs.decode_inputs(2, 4, 8, seed=80)
    out = torch.empty((2, 1, 8, 128), dtype=torch.bfloat16).pin_memory()
    ns = torch.empty((2, 8, 128, 128)).pin_memory()
    with pytest.raises(ValueError):
        gdn_decode.run_host_into(*args, out, ns, device=cuda_device)


def test_decode_host_buffers_in_place_and_back_to_back(cuda_device):
    """Two calls queued without a synchronisation between them (the second
    reuses the first one's workspace memory) and a host state advanced in
    place give the device runs' results."""
    B = 24
    a1 = inputs.decode_inputs(B, 16, 32, seed=91)
    a2 = inputs.decode_inputs(B, 16, 32, seed=92)
    h1 = [x.pin_memory() if isinstance(x, torch.Tensor) else x for x in a1]
    h2 = [x.pin_memory() if isinstance(x, torch.Tensor) else x for x in a2]
    o1 = torch.empty((B, 1, 32, 128), dtype=torch.bfloat16).pin_memory()
    o2 = torch.empty_like(o1).pin_memory()
    s2 = h2[3]                                   # advanced in place
    scratch = torch.empty_like(h1[3]).pin_memory()   # kept alive until the synchronisation
    gdn_decode.run_host_into(*h1, o1, scratch, device=cuda_device, chunks=5)
    ns1 = torch.empty_like(h1[3]).pin_memory()
    gdn_decode.run_host_into(*h1, o1, ns1, device=cuda_device, chunks=2)
    gdn_decode.run_host_into(*h2, o2, s2, device=cuda_device, chunks=7)
    torch.cuda.current_stream(cuda_device).synchronize()
    r1o, r1s = gdn_decode.run(*inputs.to_device(a1, cuda_device))
    r2o, r2s = gdn_decode.run(*inputs.to_device(a2, cuda_device))
    torch.cuda.synchronize()
    assert torch.equal(o1, r1o.cpu()) and torch.equal(ns1, r1s.cpu())
    assert torch.equal(o2, r2o.cpu()) and torch.equal(s2, r2s.cpu())

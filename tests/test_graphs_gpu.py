"""CUDA-graph capture of the serving steps.

A serving loop captures its decode / speculative-verification step once and
replays it with new inputs copied into static buffers; every entry point on
that path enqueues on the current stream, allocates through torch's caching
allocator (the graph's private pool during capture) and never synchronises,
so a replay must give exactly the eager results.
"""
import pytest
import torch

from rocm_flashinfer_contest_b200 import gdn_decode, gdn_mtp, gdn_prefill, inputs

pytestmark = pytest.mark.gpu


def _fill(dst, src):
    for d, s in zip(dst, src):
        if isinstance(d, torch.Tensor):
            d.copy_(s)


@pytest.mark.parametrize("snapshots", [True, False])  # the staged loop / the streaming kernel
def test_mtp_serving_step_replays(cuda_device, snapshots):
    """gated_delta_rule_mtp with the pool updated in place (and per-token
    snapshots), captured once and replayed on two new batches."""
    B, T, pool, H, HV = 16, 4, 24, 16, 32
    static = inputs.mtp_inputs(B, T, pool, H, HV, seed=70, device=cuda_device, indices=list(range(3, 3 + B)))
    buf = torch.zeros((B, T, HV, 128, 128), device=cuda_device) if snapshots else None
    out = torch.empty((B, T, HV, 128), dtype=torch.bfloat16, device=cuda_device)

    def step():
        gdn_mtp.gated_delta_rule_mtp(*static[:3], static[3], *static[4:9], scale=None, output=out,
                                     intermediate_states_buffer=buf, disable_state_update=False,
                                     use_qk_l2norm=True)

    step()  # eager warm-up outside the capture
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        step()
    for seed in (71, 72):
        new = inputs.mtp_inputs(B, T, pool, H, HV, seed=seed, device=cuda_device,
                                indices=list(reversed(range(5, 5 + B))))
        _fill(static, new)
        # the eager reference on copies of the same inputs
        ref_pool = new[3].clone()
        ref_buf = torch.zeros_like(buf) if snapshots else None
        ref_o, _ = gdn_mtp.gated_delta_rule_mtp(*new[:3], ref_pool, *new[4:9], scale=None,
                                                intermediate_states_buffer=ref_buf,
                                                disable_state_update=False, use_qk_l2norm=True)
        g.replay()
        torch.cuda.synchronize()
        assert torch.equal(out, ref_o)
        assert torch.equal(static[3], ref_pool)
        if snapshots:
            assert torch.equal(buf, ref_buf)


def test_mtp_stream_first_call_inside_capture(cuda_device):
    """The streaming kernel's one-time set-up (function attributes, occupancy)
    also works when its first call of an instantiation is being captured: a
    bf16 pool at T = 2, no snapshots, captured without an eager warm-up."""
    B, T, pool, H, HV = 24, 2, 30, 16, 32
    static = inputs.mtp_inputs(B, T, pool, H, HV, seed=75, device=cuda_device, indices=list(range(B)))
    static[3] = static[3].to(torch.bfloat16)
    out = torch.empty((B, T, HV, 128), dtype=torch.bfloat16, device=cuda_device)
    start = static[3].clone()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        gdn_mtp.run_into(*static[:3], static[3], *static[4:10], out, static[3])
    static[3].copy_(start)
    g.replay()
    torch.cuda.synchronize()
    ref_pool = start.clone()
    ref_o = torch.empty_like(out)
    gdn_mtp.run_into(*static[:3], ref_pool, *static[4:10], ref_o, ref_pool)
    torch.cuda.synchronize()
    assert torch.equal(out, ref_o)
    assert torch.equal(static[3], ref_pool)


def test_bf16_pool_decode_replays(cuda_device):
    """gated_delta_rule_decode_pretranspose on a bf16 state pool."""
    B, pool, H, HV = 32, 40, 16, 32
    static = inputs.mtp_inputs(B, 1, pool, H, HV, seed=80, device=cuda_device, indices=list(range(B)))
    static[3] = static[3].to(torch.bfloat16)
    out = torch.empty((B, 1, HV, 128), dtype=torch.bfloat16, device=cuda_device)

    def step():
        gdn_decode.gated_delta_rule_decode_pretranspose(
            *static[:3], None, static[5], static[6], static[7], static[8], scale=None, output=out,
            use_qk_l2norm=False, initial_state=static[3], initial_state_indices=static[4])

    step()
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        step()
    new = inputs.mtp_inputs(B, 1, pool, H, HV, seed=81, device=cuda_device, indices=list(range(8, 8 + B)))
    new[3] = new[3].to(torch.bfloat16)
    _fill(static, new)
    ref_pool = new[3].clone()
    ref_o, _ = gdn_decode.gated_delta_rule_decode_pretranspose(
        *new[:3], None, new[5], new[6], new[7], new[8], scale=None, use_qk_l2norm=False,
        initial_state=ref_pool, initial_state_indices=new[4])
    g.replay()
    torch.cuda.synchronize()
    assert torch.equal(out, ref_o)
    assert torch.equal(static[3], ref_pool)


def test_chunked_prefill_replays(cuda_device):
    """The chunked prefill (workspace from the graph's pool) replayed on new data."""
    lens = [300, 212]
    static = inputs.prefill_inputs(lens, seed=90, device=cuda_device)
    T, N = sum(lens), len(lens)
    out = torch.empty((T, 32, 128), dtype=torch.bfloat16, device=cuda_device)
    ns = torch.empty((N, 32, 128, 128), device=cuda_device)

    def step():
        gdn_prefill.run_into(*static, out, ns)

    step()
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        step()
    new = inputs.prefill_inputs(lens, seed=91, device=cuda_device)
    _fill(static, new)
    ref_o, ref_s = gdn_prefill.run(*new)
    g.replay()
    torch.cuda.synchronize()
    assert torch.equal(out, ref_o)
    assert torch.equal(ns, ref_s)

"""The host-buffer prefill (gdn_prefill_fwd_host through
gdn_prefill.run_host_into): pinned host tensors in and out, token segments
pipelined over three streams, every sequence's state carried on the device
across segment boundaries.  Results must match gdn_prefill.run on device
copies to the parity bar (a segment boundary inside a sequence that does not
start on a multiple of 64 tokens moves a chunk boundary)."""
import pytest
import torch

from parity import assert_output_close, assert_state_close
from rocm_flashinfer_contest_b200 import gdn_prefill, inputs

pytestmark = pytest.mark.gpu


def _pin(args):
    return [x.pin_memory() if isinstance(x, torch.Tensor) else x for x in args]


def _host_run(args, seg, dev, in_place=False):
    host = _pin(args)
    q, k, v, st, A_log, a, dt_bias, b, cu, scale = host
    T, N, HV = q.shape[0], cu.numel() - 1, v.shape[1]
    out = torch.full((T, HV, 128), 5.0, dtype=torch.bfloat16).pin_memory()
    ns = st if (in_place and st is not None) else torch.full((N, HV, 128, 128), 5.0).pin_memory()
    gdn_prefill.run_host_into(q, k, v, st, A_log, a, dt_bias, b, cu, scale, out, ns, device=dev,
                              segment_tokens=seg)
    return out, ns, host


def _check(args, seg, dev):
    ro, rs = gdn_prefill.run(*inputs.to_device(args, dev))
    o, s, host = _host_run(args, seg, dev)
    torch.cuda.synchronize()
    assert_output_close(o, ro.cpu())
    assert_state_close(s, rs.cpu())
    for x, y in zip(host, args):   # inputs untouched
        if isinstance(x, torch.Tensor):
            assert torch.equal(x, y)


@pytest.mark.parametrize("seg", [0, 1024, 4096, 8192])
def test_host_prefill_config2(cuda_device, seg):
    _check(inputs.prefill_inputs([8192], seed=2, with_state=False), seg, cuda_device)


@pytest.mark.parametrize("seg", [0, 512, 64])
def test_host_prefill_config3_varlen(cuda_device, seg):
    lens = inputs.seqlens_uniform(16, 1, 1024, seed=0, max_total=8192)
    _check(inputs.prefill_inputs(lens, seed=3), seg, cuda_device)


@pytest.mark.parametrize("lens,seg,cu_dtype", [
    ([128, 0, 0, 200, 0], 128, torch.int32),     # empty sequences on a segment boundary and at the end
    ([5, 0, 17, 1], 64, torch.int64),            # token-serial kernel, many segments
    ([0], 64, torch.int32),                      # only an empty sequence
    ([300, 7, 129], 192, torch.int64),
])
def test_host_prefill_edges(cuda_device, lens, seg, cu_dtype):
    _check(inputs.prefill_inputs(lens, 4, 8, seed=sum(lens) + seg, cu_dtype=cu_dtype), seg, cuda_device)


@pytest.mark.parametrize("lens", [
    [1000],            # segments 512 + 256 + 232: the last one ends mid-chunk
    [2500],            # 2048 + 256 + 196
    [700, 1300, 333],  # sequences cut by the shrinking tail segments
])
def test_host_prefill_tail_segments(cuda_device, lens):
    """Default segments: the last 2048 tokens (or fewer) are halved down to
    256-token pieces, so sequence boundaries and segment cuts fall at
    uneven places; the results still equal the device-buffer call."""
    _check(inputs.prefill_inputs(lens, seed=sum(lens)), 0, cuda_device)


def test_host_prefill_tokens_outside_sequences(cuda_device):
    args = inputs.prefill_inputs([100, 50], 4, 8, seed=9)
    T = args[0].shape[0]
    pad = 37
    # 37 tokens before the first sequence and 37 after the last: zero output there
    big = [torch.cat([torch.zeros_like(x[:pad]), x, torch.zeros_like(x[:pad])]) if i in (0, 1, 2, 5, 7) else x
           for i, x in enumerate(args)]
    big[8] = args[8] + pad
    _check(big, 64, cuda_device)
    o, _, _ = _host_run(big, 64, cuda_device)
    torch.cuda.synchronize()
    assert bool((o[:pad] == 0).all()) and bool((o[pad + T:] == 0).all())


def test_host_prefill_no_sequences(cuda_device):
    args = inputs.prefill_inputs([40], 4, 8, seed=11)
    args[8] = torch.zeros(1, dtype=torch.int32)
    args[3] = None
    host = _pin(args)
    out = torch.full((40, 8, 128), 5.0, dtype=torch.bfloat16).pin_memory()
    ns = torch.empty((0, 8, 128, 128)).pin_memory()
    gdn_prefill.run_host_into(*host, out, ns, device=cuda_device, segment_tokens=64)
    torch.cuda.synchronize()
    assert bool((out == 0).all())


def test_host_prefill_back_to_back_and_in_place(cuda_device):
    """Two calls queued without a synchronisation (the second reuses the first's
    workspace memory), the second advancing its host state in place."""
    a1 = inputs.prefill_inputs([700, 333], 16, 32, seed=21)
    a2 = inputs.prefill_inputs([500, 64, 1], 16, 32, seed=22)
    r1 = gdn_prefill.run(*inputs.to_device(a1, cuda_device))
    r2 = gdn_prefill.run(*inputs.to_device(a2, cuda_device))
    o1, s1, _ = _host_run(a1, 256, cuda_device)
    o2, s2, h2 = _host_run(a2, 128, cuda_device, in_place=True)
    torch.cuda.synchronize()
    assert s2 is h2[3]
    assert_output_close(o1, r1[0].cpu()); assert_state_close(s1, r1[1].cpu())
    assert_output_close(o2, r2[0].cpu()); assert_state_close(s2, r2[1].cpu())


def test_host_prefill_rejects_unpinned(cuda_device):
    args = inputs.prefill_inputs([64], 4, 8, seed=12)
    out = torch.empty((64, 8, 128), dtype=torch.bfloat16).pin_memory()
    ns = torch.empty((1, 8, 128, 128)).pin_memory()
    with pytest.raises(ValueError):
        gdn_prefill.run_host_into(*args, out, ns, device=cuda_device)

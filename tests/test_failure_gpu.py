"""Failure detection on the GPU without a fault: a bounded wait that runs out.

Every wait of the tensor-core kernels on an mbarrier has a clock budget; on
expiry the kernel records the timeout in a status word, frees its tensor
memory and returns, so the context stays usable.  The self-test kernel has a
mode in which nothing ever arrives on the mbarrier it waits for (no MMA is
issued, nothing is left in flight): with a budget of 200,000 cycles (~0.1 ms)
the wait must run out, the call must report GDN_ERR_DEVICE, and afterwards
the same process must still run the tensor cores and a chunked prefill
correctly.  The reference records a raising solution as a failed workload
(tools/local_verify.py:114-117); here the error is a status the host reads.
"""
import pytest
import torch

from oracle import oracle
from parity import assert_output_close, assert_state_close
from rocm_flashinfer_contest_b200 import _lib, gdn_prefill, inputs

pytestmark = pytest.mark.gpu

NO_ARRIVE = 2


def _selftest(dev, mode, wait_cycles, seed=5):
    g = torch.Generator(device=dev).manual_seed(seed)
    A = torch.randn(128, 64, device=dev, generator=g)
    B = torch.randn(64, 64, device=dev, generator=g)
    D = torch.full((128, 64), float("nan"), device=dev)
    st = _lib.lib().gdn_umma_selftest_ex(A.data_ptr(), B.data_ptr(), D.data_ptr(), 64, 64, 0, 0, 0,
                                         mode, wait_cycles, torch.cuda.current_stream(dev).cuda_stream)
    return st, A, B, D


def test_bounded_wait_runs_out_and_the_gpu_keeps_working(cuda_device, monkeypatch):
    st, _, _, D = _selftest(cuda_device, NO_ARRIVE, 200_000)
    assert st == _lib.GDN_ERR_DEVICE, _lib.strerror(st)
    assert bool(torch.isnan(D).all())          # the kernel gave up before writing any result
    # the context is intact: the same kernel, waited on normally, computes its product
    st, A, B, D = _selftest(cuda_device, 0, 0)
    assert st == _lib.GDN_OK, _lib.strerror(st)
    ref = A.half().float() @ B.half().float().T
    assert (D - ref).abs().max().item() <= 1e-4 * ref.abs().max().item() + 1e-5
    # and a chunked prefill (tensor cores, bounded waits of its own) still matches the oracle
    monkeypatch.setenv("GDN_PREFILL_CHUNK_MIN", "0")
    host = inputs.prefill_inputs([200, 70], 4, 8, seed=77)
    o, s = gdn_prefill.run(*inputs.to_device(host, cuda_device))
    torch.cuda.synchronize()
    ro, rs = oracle.prefill(*host)
    assert_output_close(o.cpu(), ro, "prefill output after a timed-out wait")
    assert_state_close(s.cpu(), rs, "prefill state after a timed-out wait")
    assert _lib.lib().gdn_device_status(0) == 0   # the prefill's own waits all completed

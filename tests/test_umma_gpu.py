"""Tensor-core layer check: tcgen05.mma with the shared-memory operand layouts
of csrc/umma.cuh (K-major / MN-major, 128-byte swizzle, f16 / bf16) must
reproduce a plain matmul of the same rounded operands."""
import pytest
import torch

from rocm_flashinfer_contest_b200 import _lib

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("a_mn,b_mn", [(0, 0), (0, 1), (1, 1), (1, 0)])
@pytest.mark.parametrize("fmt", [0, 1])
@pytest.mark.parametrize("N,K", [(64, 128), (64, 64), (128, 16), (16, 128), (32, 64), (128, 128)])
def test_umma_layouts(cuda_device, a_mn, b_mn, fmt, N, K):
    if b_mn and N % 64 and N != 32:
        pytest.skip("MN-major B: whole 64-wide blocks, or one 32-wide block (64-byte swizzle)")
    g = torch.Generator(device=cuda_device).manual_seed(N * 1000 + K * 10 + fmt)
    A = torch.randn(128, K, device=cuda_device, generator=g)
    B = torch.randn(N, K, device=cuda_device, generator=g)
    D = torch.full((128, N), float("nan"), device=cuda_device)
    st = _lib.lib().gdn_umma_selftest(A.data_ptr(), B.data_ptr(), D.data_ptr(), N, K, a_mn, b_mn,
                                      fmt, torch.cuda.current_stream().cuda_stream)
    _lib.check("gdn_umma_selftest", st)
    dt = torch.bfloat16 if fmt else torch.float16
    ref = A.to(dt).float() @ B.to(dt).float().T
    err = (D - ref).abs().max().item()
    assert err <= 1e-4 * ref.abs().max().item() + 1e-5, err


@pytest.mark.parametrize("b_mn", [0, 1])
@pytest.mark.parametrize("fmt", [0, 1])
@pytest.mark.parametrize("N,K", [(128, 128), (128, 64), (64, 64), (32, 64), (64, 128), (16, 16)])
def test_umma_a_in_tensor_memory(cuda_device, b_mn, fmt, N, K):
    """The TMEM-A form of tcgen05.mma: A staged in tensor memory (row m in
    lane m, two 16-bit elements per 32-bit column), B in shared memory."""
    if b_mn and N % 64 and N != 32:
        pytest.skip("MN-major B: whole 64-wide blocks, or one 32-wide block (64-byte swizzle)")
    g = torch.Generator(device=cuda_device).manual_seed(N * 1000 + K * 10 + fmt + 7)
    A = torch.randn(128, K, device=cuda_device, generator=g)
    B = torch.randn(N, K, device=cuda_device, generator=g)
    D = torch.full((128, N), float("nan"), device=cuda_device)
    st = _lib.lib().gdn_umma_selftest_ex(A.data_ptr(), B.data_ptr(), D.data_ptr(), N, K, 0, b_mn, fmt,
                                         1, 0, torch.cuda.current_stream().cuda_stream)
    _lib.check("gdn_umma_selftest_ex", st)
    dt = torch.bfloat16 if fmt else torch.float16
    ref = A.to(dt).float() @ B.to(dt).float().T
    err = (D - ref).abs().max().item()
    assert err <= 1e-4 * ref.abs().max().item() + 1e-5, err

"""gdn_prefill_fwd_noalloc: the prefill entry point for callers that cannot
allocate device memory (a host binding the C ABI directly, with no caching
allocator to take a workspace from, or a runtime that forbids allocation
after start-up).  It takes its workspace from a fixed 16 MiB scratch array
inside the library instead of from the caller.

This file is collected last, so a run that stops at the first failure has run
every other test before it.  The checks go through the C ABI: two calls in a
row, on different inputs, must return exactly what gdn_prefill_fwd (the
entry point with a caller-provided workspace) returns for the same inputs --
the same kernels run on the same data, so the bits agree -- and both must
match the CPU oracle within the parity tolerances used everywhere else; a
problem that needs more than the 16 MiB must be refused before anything is
launched.
"""
import pytest
import torch

from oracle import oracle
from parity import assert_output_close, assert_state_close
from rocm_flashinfer_contest_b200 import _lib, inputs

pytestmark = pytest.mark.gpu


def _noalloc(args, output, new_state, dev):
    q, k, v, state, A_log, a, dt_bias, b, cu, scale = args
    T, H, K = q.shape
    HV, V = v.shape[1], v.shape[2]
    return _lib.lib().gdn_prefill_fwd_noalloc(
        q.data_ptr(), k.data_ptr(), v.data_ptr(), 0 if state is None else state.data_ptr(),
        A_log.data_ptr(), a.data_ptr(), dt_bias.data_ptr(), b.data_ptr(), cu.data_ptr(),
        1 if cu.dtype == torch.int64 else 0, cu.numel() - 1, T, float(scale), H, HV, K, V,
        output.data_ptr(), new_state.data_ptr(), torch.cuda.current_stream(dev).cuda_stream)


def _with_workspace(args, output, new_state, dev):
    q, k, v, state, A_log, a, dt_bias, b, cu, scale = args
    T, H, K = q.shape
    HV, V = v.shape[1], v.shape[2]
    N = cu.numel() - 1
    nbytes = _lib.lib().gdn_prefill_workspace_bytes(N, T, H, HV)
    ws = torch.empty(max(nbytes, 16), dtype=torch.uint8, device=dev)
    st = _lib.lib().gdn_prefill_fwd(
        q.data_ptr(), k.data_ptr(), v.data_ptr(), 0 if state is None else state.data_ptr(),
        A_log.data_ptr(), a.data_ptr(), dt_bias.data_ptr(), b.data_ptr(), cu.data_ptr(),
        1 if cu.dtype == torch.int64 else 0, N, T, float(scale), H, HV, K, V,
        output.data_ptr(), new_state.data_ptr(), ws.data_ptr(), nbytes,
        torch.cuda.current_stream(dev).cuda_stream)
    torch.cuda.synchronize()
    return st


def test_noalloc_matches_workspace_entry_point(cuda_device, monkeypatch):
    # the chunked kernels are the ones that use scratch: run them for every size
    monkeypatch.setenv("GDN_PREFILL_CHUNK_MIN", "0")
    for call, lens in enumerate(([150, 37, 0, 64], [300, 5, 129])):
        host = inputs.prefill_inputs(lens, 4, 8, seed=40 + call)
        args = inputs.to_device(host, cuda_device)
        N, T, HV = len(lens), sum(lens), 8
        ref_o = torch.full((T, HV, 128), float("nan"), dtype=torch.bfloat16, device=cuda_device)
        ref_s = torch.full((N, HV, 128, 128), float("nan"), device=cuda_device)
        _lib.check("gdn_prefill_fwd", _with_workspace(args, ref_o, ref_s, cuda_device))
        out = torch.full_like(ref_o, float("nan"))
        new_state = torch.full_like(ref_s, float("nan"))
        _lib.check("gdn_prefill_fwd_noalloc", _noalloc(args, out, new_state, cuda_device))
        torch.cuda.synchronize()
        # same kernels, same inputs: the same bits as the workspace entry point
        assert torch.equal(out.view(torch.int16), ref_o.view(torch.int16)), f"call {call}: output differs"
        assert torch.equal(new_state.view(torch.int32), ref_s.view(torch.int32)), f"call {call}: state differs"
        # and the reference semantics, through the CPU oracle
        o_cpu, s_cpu = oracle.prefill(*host)
        assert_output_close(out.cpu(), o_cpu, what=f"call {call} output vs oracle")
        assert_state_close(new_state.cpu(), s_cpu, what=f"call {call} new_state vs oracle")


def test_noalloc_refuses_problems_beyond_its_scratch(cuda_device, monkeypatch):
    monkeypatch.setenv("GDN_PREFILL_CHUNK_MIN", "0")
    T, HV = 4096, 32  # (4096 / 64 + 1) slots of 32 * 17,424 + 16 * 49,152 bytes > 16 MiB
    assert _lib.lib().gdn_prefill_workspace_bytes(1, T, 16, HV) > 16 << 20
    st = _lib.lib().gdn_prefill_fwd_noalloc(16, 16, 16, 0, 16, 16, 16, 16, 16, 1, 1, T, 0.0, 16, HV,
                                            128, 128, 16, 16, None)
    assert st == _lib.GDN_ERR_TOO_LARGE
    assert "16 MiB" in _lib.strerror(st)

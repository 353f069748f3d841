"""Size-independent properties at the benchmark sizes, where the CPU oracle
would take minutes: both sides of every comparison run on the GPU through
the public entry points, held to the parity bar of tests/parity.py.

* resume: prefilling tokens [0, T) in one call equals prefilling [0, t) and
  then [t, T) from the first call's final state (chunk-aligned and unaligned
  split points) — the recurrence is a left fold over tokens;
* the chunked tensor-core kernels (with each chain kernel) and the
  token-serial kernel agree on the whole config-2 sequence (8192 tokens, all
  32 v-heads) and on config 3;
* a prefill of one-token sequences equals one decode step, and a
  multi-token (MTP) call over T tokens equals T single-token decode steps.
"""
import pytest
import torch

from parity import assert_output_close, assert_state_close
from rocm_flashinfer_contest_b200 import gdn_decode, gdn_mtp, gdn_prefill, inputs

pytestmark = pytest.mark.gpu


def _run_range(args, t0, t1, state, dev):
    """gdn_prefill.run over tokens [t0, t1) of a one-sequence input, starting from `state`."""
    q, k, v, _, A_log, a, dt_bias, b, cu, scale = args
    cu1 = torch.tensor([0, t1 - t0], dtype=cu.dtype, device=dev)
    return gdn_prefill.run(q[t0:t1], k[t0:t1], v[t0:t1], state, A_log, a[t0:t1], dt_bias, b[t0:t1], cu1, scale)


@pytest.mark.parametrize("split", [4096, 4000, 64, 8191])
def test_prefill_resume_equals_one_call(cuda_device, split):
    args = inputs.prefill_inputs([8192], seed=2, with_state=False, device=cuda_device)
    o, s = gdn_prefill.run(*args)
    o1, s1 = _run_range(args, 0, split, None, cuda_device)
    o2, s2 = _run_range(args, split, 8192, s1, cuda_device)
    torch.cuda.synchronize()
    assert_output_close(torch.cat([o1, o2]).cpu(), o.cpu())
    assert_state_close(s2.cpu(), s.cpu())


def test_prefill_resume_past_32_bit_offsets(cuda_device):
    """One sequence of 525,288 tokens: the output holds more than 2^31
    elements (4.3 GB), the workspace more than 2^32 bytes and the prep grid
    262,656 CTAs, so every offset must be 64-bit.  The last 4096 tokens of
    the one call equal a resume of them from the state after the first
    T - 4096 (an unaligned split, so the chunk boundaries differ)."""
    T, tail = 524288 + 1000, 4096
    args = inputs.prefill_inputs([T], seed=5, with_state=False, device=cuda_device)
    o, s = gdn_prefill.run(*args)
    o_tail = o[T - tail:].cpu()
    del o
    torch.cuda.empty_cache()
    _, s1 = _run_range(args, 0, T - tail, None, cuda_device)
    torch.cuda.empty_cache()
    o2, s2 = _run_range(args, T - tail, T, s1, cuda_device)
    torch.cuda.synchronize()
    assert_output_close(o2.cpu(), o_tail)
    assert_state_close(s2.cpu(), s.cpu())


@pytest.mark.parametrize("chain", ["2", "3", "4"])
def test_prefill_chunked_and_token_serial_agree_full_size(cuda_device, monkeypatch, chain):
    args = inputs.prefill_inputs([8192], seed=2, with_state=False, device=cuda_device)
    monkeypatch.setenv("GDN_PREFILL_CHAIN", chain)
    monkeypatch.setenv("GDN_PREFILL_CHUNK_MIN", "0")
    oc, sc = gdn_prefill.run(*args)
    monkeypatch.setenv("GDN_PREFILL_CHUNK_MIN", "1000000000")
    orr, sr = gdn_prefill.run(*args)
    torch.cuda.synchronize()
    assert_output_close(oc.cpu(), orr.cpu())
    assert_state_close(sc.cpu(), sr.cpu())


@pytest.mark.parametrize("chain", ["2", "3", "4"])
def test_prefill_varlen_chunked_and_token_serial_agree(cuda_device, monkeypatch, chain):
    """Config 3 (16 sequences, lengths U[1, 1024], non-zero states)."""
    lens = inputs.seqlens_uniform(16, 1, 1024, seed=0, max_total=8192)
    args = inputs.prefill_inputs(lens, seed=3, device=cuda_device)
    monkeypatch.setenv("GDN_PREFILL_CHAIN", chain)
    monkeypatch.setenv("GDN_PREFILL_CHUNK_MIN", "0")
    oc, sc = gdn_prefill.run(*args)
    monkeypatch.setenv("GDN_PREFILL_CHUNK_MIN", "1000000000")
    orr, sr = gdn_prefill.run(*args)
    torch.cuda.synchronize()
    assert_output_close(oc.cpu(), orr.cpu())
    assert_state_close(sc.cpu(), sr.cpu())


@pytest.mark.parametrize("path", ["chunk2", "chunk3", "chunk4", "recurrent"])
def test_one_token_prefills_equal_a_decode_step(cuda_device, monkeypatch, path):
    B = 64
    monkeypatch.setenv("GDN_PREFILL_CHUNK_MIN", "1000000000" if path == "recurrent" else "0")
    if path != "recurrent":
        monkeypatch.setenv("GDN_PREFILL_CHAIN", path[-1])
    q, k, v, st, A_log, a, dt_bias, b, scale = inputs.decode_inputs(B, seed=31, device=cuda_device)
    cu = torch.arange(B + 1, dtype=torch.int32, device=cuda_device)
    po, ps = gdn_prefill.run(q[:, 0], k[:, 0], v[:, 0], st, A_log, a[:, 0], dt_bias, b[:, 0], cu, scale)
    do, ds = gdn_decode.run(q, k, v, st, A_log, a, dt_bias, b, scale)
    torch.cuda.synchronize()
    assert_output_close(po.cpu(), do[:, 0].cpu())
    assert_state_close(ps.cpu(), ds.cpu())


@pytest.mark.parametrize("T", [2, 3, 4, 5, 8])
def test_mtp_equals_stepwise_decode(cuda_device, T):
    B, pool = 64, 64
    q, k, v, pool_state, idx, A_log, a, dt_bias, b, scale, _ = inputs.mtp_inputs(
        B, T, pool, seed=40 + T, device=cuda_device, indices=list(range(B)))
    out, final = gdn_mtp.run(q, k, v, pool_state, idx, A_log, a, dt_bias, b, scale)
    s = pool_state.clone()
    outs = []
    for t in range(T):
        o, s = gdn_decode.run(q[:, t:t + 1], k[:, t:t + 1], v[:, t:t + 1], s, A_log, a[:, t:t + 1], dt_bias,
                              b[:, t:t + 1], scale)
        outs.append(o)
    torch.cuda.synchronize()
    assert_output_close(out.cpu(), torch.cat(outs, dim=1).cpu())
    assert_state_close(final.cpu(), s.cpu())

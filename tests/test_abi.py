"""The C ABI library loads without a GPU, exports every function that
include/gdn_b200.h declares, and rejects bad arguments with status codes
before anything is launched (no CUDA call is made on these paths)."""
import ctypes
import os
import re
import subprocess

import pytest

from rocm_flashinfer_contest_b200 import _lib

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER_DIR = os.path.join(ROOT, "include")


def _declared():
    names = set()
    for fn in os.listdir(HEADER_DIR):
        if fn.endswith(".h"):
            src = open(os.path.join(HEADER_DIR, fn)).read()
            src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
            names |= set(re.findall(r"\b(gdn_\w+)\s*\(", src))
    return names


def test_header_declares_the_abi():
    assert {"gdn_decode_fwd", "gdn_prefill_fwd", "gdn_mtp_fwd", "gdn_abi_version",
            "gdn_strerror"} <= _declared()


def test_library_exports_every_declared_symbol():
    lib = _lib.lib()
    for name in _declared():
        assert hasattr(lib, name), name
    out = subprocess.run(["nm", "-D", "--defined-only", _lib.LIB_PATH], capture_output=True,
                         text=True, check=True).stdout
    exported = set(re.findall(r"\bT (gdn_\w+)", out))
    assert _declared() <= exported


def test_python_signatures_cover_the_header():
    assert _declared() == set(_lib.SIGNATURES)


def test_version_and_strerror():
    lib = _lib.lib()
    assert lib.gdn_abi_version() == 4
    for code in (0, 1, 2, 3, 4):
        assert lib.gdn_strerror(code)
    assert b"unknown" in lib.gdn_strerror(99)


def _decode(**over):
    d = dict(q=16, k=16, v=16, state=16, A_log=16, a=16, dt_bias=16, b=16, scale=0.0,
             B=1, H=1, HV=2, K=128, V=128, out=16, new_state=16, stream=None)
    d.update(over)
    return _lib.lib().gdn_decode_fwd(*d.values())


def _prefill(**over):
    d = dict(q=16, k=16, v=16, state=16, A_log=16, a=16, dt_bias=16, b=16, cu=16, cu64=1,
             N=1, T=4, scale=0.0, H=1, HV=2, K=128, V=128, out=16, new_state=16, ws=None, ws_bytes=0,
             stream=None)
    d.update(over)
    return _lib.lib().gdn_prefill_fwd(*d.values())


@pytest.mark.parametrize("over,code", [
    (dict(K=64), _lib.GDN_ERR_UNSUPPORTED),
    (dict(V=96), _lib.GDN_ERR_UNSUPPORTED),
    (dict(H=3, HV=4), _lib.GDN_ERR_UNSUPPORTED),
    (dict(H=0), _lib.GDN_ERR_INVALID),
    (dict(B=-1), _lib.GDN_ERR_INVALID),
    (dict(q=None), _lib.GDN_ERR_INVALID),
    (dict(new_state=None), _lib.GDN_ERR_INVALID),
    (dict(state=24), _lib.GDN_ERR_ALIGN),
    (dict(q=18), _lib.GDN_ERR_ALIGN),
    (dict(B=0), _lib.GDN_OK),  # nothing to do: returns before any launch
])
def test_decode_rejects_bad_arguments(over, code):
    assert _decode(**over) == code


def _decode_host(**over):
    B, H, HV = over.get("B", 2), over.get("H", 1), over.get("HV", 2)
    need = _lib.lib().gdn_decode_host_workspace_bytes(max(B, 1), H, HV)
    d = dict(q=16, k=16, v=16, state=16, A_log=16, a=16, dt_bias=16, b=16, scale=0.0,
             B=B, H=H, HV=HV, K=128, V=128, out=16, new_state=16, ws=4096, ws_bytes=need,
             chunks=0, stream=None)
    d.update(over)
    return _lib.lib().gdn_decode_fwd_host(*d.values())


@pytest.mark.parametrize("over,code", [
    (dict(K=64), _lib.GDN_ERR_UNSUPPORTED),
    (dict(H=3, HV=8), _lib.GDN_ERR_UNSUPPORTED),
    (dict(B=-1), _lib.GDN_ERR_INVALID),
    (dict(chunks=-1), _lib.GDN_ERR_INVALID),
    (dict(out=None), _lib.GDN_ERR_INVALID),
    (dict(ws=None), _lib.GDN_ERR_INVALID),
    (dict(ws_bytes=1024), _lib.GDN_ERR_INVALID),           # smaller than the workspace needs
    (dict(ws=4096 + 128), _lib.GDN_ERR_ALIGN),             # workspace must be 256-byte aligned
    (dict(B=0), _lib.GDN_OK),                              # nothing to do: no CUDA call
])
def test_decode_host_rejects_bad_arguments(over, code):
    assert _decode_host(**over) == code


def test_decode_host_workspace_bytes():
    f = _lib.lib().gdn_decode_host_workspace_bytes
    up = lambda x: (x + 255) // 256 * 256  # noqa: E731
    B, H, HV = 64, 16, 32
    want = (up(B * HV * 128 * 128 * 4) + 2 * up(B * H * 128 * 2) + 2 * up(B * HV * 128 * 2)
            + 2 * up(B * HV * 2) + 2 * up(HV * 4))
    assert f(B, H, HV) == want
    assert f(0, H, HV) == 0 and f(B, 0, HV) == 0


@pytest.mark.parametrize("over,code", [
    (dict(K=64), _lib.GDN_ERR_UNSUPPORTED),
    (dict(H=5, HV=8), _lib.GDN_ERR_UNSUPPORTED),
    (dict(N=-1), _lib.GDN_ERR_INVALID),
    (dict(T=-2), _lib.GDN_ERR_INVALID),
    (dict(cu64=2), _lib.GDN_ERR_INVALID),
    (dict(cu=None), _lib.GDN_ERR_INVALID),
    (dict(new_state=None), _lib.GDN_ERR_INVALID),
    (dict(cu=20, cu64=1), _lib.GDN_ERR_ALIGN),
    (dict(new_state=40), _lib.GDN_ERR_ALIGN),
    (dict(N=0, T=0), _lib.GDN_OK),
    (dict(T=4096, N=2), _lib.GDN_ERR_INVALID),            # chunk path without a workspace
    (dict(T=4096, N=2, ws=40, ws_bytes=1 << 30), _lib.GDN_ERR_ALIGN),
    (dict(q=24), _lib.GDN_ERR_ALIGN),                     # prefill needs 16-byte aligned q/k/v/out
])
def test_prefill_rejects_bad_arguments(over, code):
    assert _prefill(**over) == code


def _prefill_noalloc(**over):
    d = dict(q=16, k=16, v=16, state=16, A_log=16, a=16, dt_bias=16, b=16, cu=16, cu64=1,
             N=1, T=4096, scale=0.0, H=16, HV=32, K=128, V=128, out=16, new_state=16, stream=None)
    d.update(over)
    return _lib.lib().gdn_prefill_fwd_noalloc(*d.values())


@pytest.mark.parametrize("over,code", [
    # argument errors come before the scratch-size check (these sizes are too large)
    (dict(K=64), _lib.GDN_ERR_UNSUPPORTED),
    (dict(V=96), _lib.GDN_ERR_UNSUPPORTED),
    (dict(H=5, HV=32), _lib.GDN_ERR_UNSUPPORTED),
    (dict(N=-1), _lib.GDN_ERR_INVALID),
    (dict(H=0), _lib.GDN_ERR_INVALID),
    (dict(cu64=2), _lib.GDN_ERR_INVALID),
    (dict(cu=None), _lib.GDN_ERR_INVALID),
    (dict(q=None), _lib.GDN_ERR_INVALID),
    (dict(new_state=None), _lib.GDN_ERR_INVALID),
    (dict(q=24), _lib.GDN_ERR_ALIGN),
    (dict(cu=20, cu64=1), _lib.GDN_ERR_ALIGN),
    (dict(), _lib.GDN_ERR_TOO_LARGE),                     # 65 slots x (32 x 17,424 + 16 x 49,152) B
    (dict(N=0, T=0), _lib.GDN_OK),                       # nothing to do: no CUDA call
])
def test_prefill_noalloc_rejects_bad_arguments(over, code):
    assert _prefill_noalloc(**over) == code


def _mtp(**over):
    d = dict(q=16, k=16, v=16, pool_in=4096, pool_out=4096, bf16=0, idx=16, out_idx=None, idx64=0,
             A_log=16, a=16, dt_bias=16, b=16, scale=0.0, B=2, T=3, H=1, HV=2, K=128, V=128, pool=4,
             l2=0, out=16, inter=None, inter_slots=0, steps=0, stream=None)  # l2 = the flags word
    d.update(over)
    return _lib.lib().gdn_mtp_fwd(*d.values())


@pytest.mark.parametrize("over,code", [
    (dict(K=64), _lib.GDN_ERR_UNSUPPORTED),
    (dict(H=3, HV=4), _lib.GDN_ERR_UNSUPPORTED),
    (dict(B=-1), _lib.GDN_ERR_INVALID),
    (dict(T=-1), _lib.GDN_ERR_INVALID),
    (dict(pool=-1), _lib.GDN_ERR_INVALID),
    (dict(idx64=2), _lib.GDN_ERR_INVALID),
    (dict(l2=4), _lib.GDN_ERR_INVALID),                                 # unknown flag bit
    (dict(l2=-1), _lib.GDN_ERR_INVALID),
    (dict(l2=3, B=0), _lib.GDN_OK),                                     # l2norm | snapshots by entry
    (dict(idx=None), _lib.GDN_ERR_INVALID),
    (dict(out=None), _lib.GDN_ERR_INVALID),
    (dict(inter=4096, inter_slots=4, steps=2), _lib.GDN_ERR_INVALID),   # cache_steps < T
    (dict(pool_out=4096 + 1024), _lib.GDN_ERR_INVALID),                 # partial overlap
    (dict(idx=20, idx64=1), _lib.GDN_ERR_ALIGN),
    (dict(q=18), _lib.GDN_ERR_ALIGN),
    (dict(inter=4104, inter_slots=4, steps=3), _lib.GDN_ERR_ALIGN),
    (dict(bf16=2), _lib.GDN_ERR_INVALID),
    (dict(bf16=1, inter=4096, inter_slots=4, steps=3), _lib.GDN_ERR_INVALID),  # snapshots need fp32
    (dict(out_idx=18), _lib.GDN_ERR_ALIGN),
    (dict(pool_out=4096 + 512, bf16=1), _lib.GDN_ERR_INVALID),       # bf16 pool: 256 KiB, overlaps
    (dict(B=0), _lib.GDN_OK),                       # in place, nothing to do: no CUDA call
    (dict(T=0, pool_out=None), _lib.GDN_OK),
])
def test_mtp_rejects_bad_arguments(over, code):
    assert _mtp(**over) == code


def _prefill_ckpt(**over):
    d = dict(q=16, k=16, v=16, state=16, A_log=16, a=16, dt_bias=16, b=16, cu=16, cu64=1,
             N=1, T=4, scale=0.0, H=1, HV=2, K=128, V=128, out=16, new_state=16,
             ckpt=16, ckpt_cu=16, total=1, every=64, ws=None, ws_bytes=0, stream=None)
    d.update(over)
    return _lib.lib().gdn_prefill_fwd_checkpointed(*d.values())


@pytest.mark.parametrize("over,code", [
    (dict(ckpt=None), _lib.GDN_ERR_INVALID),
    (dict(every=0), _lib.GDN_ERR_INVALID),
    (dict(every=96), _lib.GDN_ERR_INVALID),     # not a multiple of the chunk size
    (dict(ckpt_cu=None), _lib.GDN_ERR_INVALID),
    (dict(total=-1), _lib.GDN_ERR_INVALID),
    (dict(ckpt=24), _lib.GDN_ERR_ALIGN),
    (dict(ckpt_cu=20), _lib.GDN_ERR_ALIGN),
    (dict(K=64), _lib.GDN_ERR_UNSUPPORTED),
    (dict(N=0, T=0), _lib.GDN_OK),
])
def test_prefill_checkpointed_rejects_bad_arguments(over, code):
    assert _prefill_ckpt(**over) == code


def _prefill_ex(**over):
    d = dict(q=16, k=16, v=16, state=16, A_log=16, a=16, dt_bias=16, b=16, cu=16, cu64=1,
             N=1, T=4, scale=0.0, H=1, HV=2, K=128, V=128, out=16, new_state=16,
             ckpt=None, ckpt_cu=None, total=0, every=0, flags=0, ws=None, ws_bytes=0, stream=None)
    d.update(over)
    return _lib.lib().gdn_prefill_fwd_ex(*d.values())


@pytest.mark.parametrize("over,code", [
    (dict(flags=2), _lib.GDN_ERR_INVALID),                 # unknown flag bit
    (dict(flags=-1), _lib.GDN_ERR_INVALID),
    (dict(every=64), _lib.GDN_ERR_INVALID),                # every > 0 without checkpoints
    (dict(ckpt=16, ckpt_cu=16, total=1), _lib.GDN_ERR_INVALID),  # checkpoints with every == 0
    (dict(ckpt=16, ckpt_cu=16, total=1, every=96), _lib.GDN_ERR_INVALID),
    (dict(ckpt=24, ckpt_cu=16, total=1, every=64), _lib.GDN_ERR_ALIGN),
    (dict(flags=1, K=64), _lib.GDN_ERR_UNSUPPORTED),
    (dict(flags=1, N=0, T=0), _lib.GDN_OK),
    (dict(flags=1, N=0, T=0, ckpt=16, ckpt_cu=16, total=0, every=64), _lib.GDN_OK),
])
def test_prefill_ex_rejects_bad_arguments(over, code):
    assert _prefill_ex(**over) == code


def _prefill_host(cu, **over):
    import numpy as np
    cu_arr = np.asarray(cu, dtype=np.int64)
    N, T = len(cu) - 1, over.pop("T", 8)
    need = _lib.lib().gdn_prefill_host_workspace_bytes(N, T, 1, 2, 0)
    d = dict(q=16, k=16, v=16, state=16, A_log=16, a=16, dt_bias=16, b=16, cu=cu_arr.ctypes.data, cu64=1,
             N=N, T=T, scale=0.0, H=1, HV=2, K=128, V=128, out=16, new_state=16, ws=4096, ws_bytes=need,
             seg=0, stream=None)
    d.update(over)
    return _lib.lib().gdn_prefill_fwd_host(*d.values())


@pytest.mark.parametrize("cu,over,code", [
    ([0, 5, 3], {}, _lib.GDN_ERR_INVALID),                 # cu_seqlens decreasing (read on the host)
    ([0, 9], {}, _lib.GDN_ERR_INVALID),                    # cu_seqlens[N] > T
    ([-1, 4], {}, _lib.GDN_ERR_INVALID),
    ([0, 8], dict(ws_bytes=1024), _lib.GDN_ERR_INVALID),   # workspace too small
    ([0, 8], dict(ws=4096 + 64), _lib.GDN_ERR_ALIGN),
    ([0, 8], dict(seg=-1), _lib.GDN_ERR_INVALID),
    ([0, 8], dict(cu64=2), _lib.GDN_ERR_INVALID),
    ([0, 8], dict(K=64), _lib.GDN_ERR_UNSUPPORTED),
    ([0, 8], dict(out=None), _lib.GDN_ERR_INVALID),
    ([0], dict(T=0), _lib.GDN_OK),                          # nothing to do: no CUDA call
])
def test_prefill_host_rejects_bad_arguments(cu, over, code):
    assert _prefill_host(cu, **over) == code


def test_prefill_host_workspace_bytes():
    f = _lib.lib().gdn_prefill_host_workspace_bytes
    assert f(0, 0, 16, 32, 0) == 0 and f(-1, 8, 16, 32, 0) == 0 and f(1, 8, 16, 32, -1) == 0
    # one sequence of 8192 tokens in 2048-token segments: its state, two segments of
    # q, k, v, a, b and output, and one segment's chunk workspace
    seg_io = 2048 * (2 * 16 * 128 * 2 + 2 * 32 * 128 * 2 + 2 * 32 * 2)
    assert f(1, 8192, 16, 32, 0) >= 32 * 128 * 128 * 4 + 2 * seg_io
    assert f(1, 8192, 16, 32, 0) == f(1, 8192, 16, 32, 2048)
    assert f(1, 8192, 16, 32, 1024) < f(1, 8192, 16, 32, 2048)
    assert f(4, 100, 16, 32, 0) > 0 and f(0, 100, 16, 32, 0) > 0   # T < 2048: one 128-token segment


def test_prefill_workspace_size(monkeypatch):
    """The workspace covers both layouts of the chunked path: per 64-token
    slot, the split/transposed chains' [T;P'] records and [K;Q] + G tiles,
    and the scan chain's 73,984-byte transition records per v-head plus a
    4-byte ready flag each (the flags rounded up to 256 bytes)."""
    ws = _lib.lib().gdn_prefill_workspace_bytes

    def want(N, T, H, HV):
        slots = T // 64 + N
        split = slots * (HV * 17424 + H * (32768 + 16384))
        scan = slots * HV * 73984 + (slots * HV * 4 + 255) // 256 * 256
        return max(split, scan)

    monkeypatch.setenv("GDN_PREFILL_CHUNK_MIN", "128")
    assert ws(1, 8192, 16, 32) == want(1, 8192, 16, 32)
    assert ws(16, 5000, 4, 8) == want(16, 5000, 4, 8)
    assert ws(3, 100, 4, 8) == 0          # below the threshold: token-serial kernel, no workspace
    assert ws(0, 0, 4, 8) == 0
    monkeypatch.setenv("GDN_PREFILL_CHUNK_MIN", "0")
    assert ws(3, 100, 4, 8) == want(3, 100, 4, 8)
    assert ws(2, 640, 16, 16) == want(2, 640, 16, 16)
    assert ws(2, 640, 4, 32) == want(2, 640, 4, 32) == 12 * 32 * 73984 + 1536  # the scan layout


def test_error_is_raised_as_exception():
    with pytest.raises(_lib.GDNError) as ei:
        _lib.check("gdn_decode_fwd", _decode(K=64))
    assert ei.value.status == _lib.GDN_ERR_UNSUPPORTED


@pytest.mark.parametrize("mode,wait,a_mn,code", [
    (4, 0, 0, _lib.GDN_ERR_INVALID),        # unknown mode bit
    (2, -1, 0, _lib.GDN_ERR_INVALID),       # negative wait budget
    (1, 0, 1, _lib.GDN_ERR_UNSUPPORTED),    # a TMEM-resident A is K-major
])
def test_selftest_ex_rejects_bad_arguments(mode, wait, a_mn, code):
    assert _lib.lib().gdn_umma_selftest_ex(16, 16, 16, 64, 64, a_mn, 0, 0, mode, wait, None) == code

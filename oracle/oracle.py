"""ctypes front end of the CPU oracle in gdn_oracle.c (test infrastructure only).

Takes and returns torch CPU tensors in the contest layouts and dtypes, so a test
can hand the same seeded inputs to the oracle and to the CUDA path:

* ``decode(q, k, v, state, A_log, a, dt_bias, b, scale)`` mirrors the contest
  definition ``gdn_decode_*_k_last`` (flashinfer-python 0.6.11.post2,
  flashinfer/trace/templates/gdn.py:27-94) and the reference solution's
  ``run`` signature (solutions/gdn_decode/main.py:117).
* ``prefill(q, k, v, state, A_log, a, dt_bias, b, cu_seqlens, scale)`` mirrors
  ``gdn_prefill_*_k_last`` (gdn.py:189-273; solutions/gdn_prefill/main.py:31).
* ``mtp(q, k, v, initial_state, initial_state_indices, A_log, a, dt_bias, b,
  scale, intermediate_states_buffer=None)`` mirrors the multi-token decode
  definition ``gdn_mtp`` (gdn.py:378-465), with out-of-range indices as
  padding.

All return ``(output bf16, new_state fp32)``; ``prefill`` with
``checkpoint_every_n_tokens > 0`` adds the state checkpoints.  ``threads``
<= 0 uses every core.
"""
from __future__ import annotations

import ctypes
import math
import os
import subprocess

import torch

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "libgdn_oracle.so")
_lib = None

_f32p = ctypes.POINTER(ctypes.c_float)
_u16p = ctypes.POINTER(ctypes.c_uint16)
_i64p = ctypes.POINTER(ctypes.c_int64)


def build() -> str:
    """Compile gdn_oracle.c (make; a no-op when the library is current)."""
    subprocess.run(["make", "-s", "-C", _HERE], check=True)
    return _LIB_PATH


def _load():
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(_LIB_PATH):
        build()
    lib = ctypes.CDLL(_LIB_PATH)
    lib.gdn_oracle_decode.restype = ctypes.c_int
    lib.gdn_oracle_decode.argtypes = [
        _f32p, _f32p, _f32p, _f32p, _f32p, _f32p, _f32p, _f32p, ctypes.c_float,
        ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int,
        _u16p, _f32p, _f32p, ctypes.c_int,
    ]
    lib.gdn_oracle_prefill.restype = ctypes.c_int
    lib.gdn_oracle_prefill.argtypes = [
        _f32p, _f32p, _f32p, _f32p, _f32p, _f32p, _f32p, _f32p, _i64p,
        ctypes.c_int, ctypes.c_int, ctypes.c_float,
        ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int,
        _u16p, _f32p, _f32p, _i64p, ctypes.c_int, ctypes.c_int, ctypes.c_int,
    ]
    lib.gdn_oracle_mtp.restype = ctypes.c_int
    lib.gdn_oracle_mtp.argtypes = [
        _f32p, _f32p, _f32p, _f32p, _f32p, _i64p, _i64p, _f32p, _f32p, _f32p, _f32p, ctypes.c_float,
        ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int,
        ctypes.c_int, ctypes.c_int, ctypes.c_int, _u16p, _f32p, ctypes.c_int, ctypes.c_longlong,
        ctypes.c_int, ctypes.c_int,
    ]
    _lib = lib
    return lib


def _f32(t):
    """Contiguous fp32 CPU copy (bf16 widens exactly)."""
    return t.detach().to("cpu", torch.float32).contiguous()


def _ptr(t, ty):
    return ctypes.cast(t.data_ptr(), ty) if t is not None else None


def _scale(scale, K):
    if isinstance(scale, torch.Tensor):
        scale = float(scale.item())
    scale = 0.0 if scale is None else float(scale)
    return 1.0 / math.sqrt(K) if scale == 0.0 else scale


def decode(q, k, v, state, A_log, a, dt_bias, b, scale, threads: int = 0, return_f32=False):
    lib = _load()
    B, _, H, K = q.shape
    HV, V = v.shape[2], v.shape[3]
    qf, kf, vf = _f32(q), _f32(k), _f32(v)
    sf = _f32(state) if state is not None else None
    Af, af, dtf, bf = _f32(A_log), _f32(a), _f32(dt_bias), _f32(b)
    out = torch.empty((B, 1, HV, V), dtype=torch.int16)
    out32 = torch.empty((B, 1, HV, V), dtype=torch.float32)
    new_state = torch.empty((B, HV, V, K), dtype=torch.float32)
    rc = lib.gdn_oracle_decode(
        _ptr(qf, _f32p), _ptr(kf, _f32p), _ptr(vf, _f32p), _ptr(sf, _f32p),
        _ptr(Af, _f32p), _ptr(af, _f32p), _ptr(dtf, _f32p), _ptr(bf, _f32p),
        _scale(scale, K), B, H, HV, K, V,
        _ptr(out, _u16p), _ptr(out32, _f32p), _ptr(new_state, _f32p), int(threads))
    if rc != 0:
        raise ValueError(f"gdn_oracle_decode rejected its arguments (rc={rc})")
    o = out.view(torch.bfloat16)
    return (o, new_state, out32) if return_f32 else (o, new_state)


def checkpoint_cu_starts(cu_seqlens, every: int) -> torch.Tensor:
    """[N + 1] int64 cumulative checkpoint counts: sequence n gets len_n // every."""
    cu = cu_seqlens.detach().to("cpu", torch.int64)
    out = torch.zeros(cu.numel(), dtype=torch.int64)
    out[1:] = torch.cumsum((cu[1:] - cu[:-1]).clamp_min(0) // every, 0)
    return out


def prefill(q, k, v, state, A_log, a, dt_bias, b, cu_seqlens, scale, threads: int = 0,
            checkpoint_every_n_tokens: int = 0, qk_l2norm: bool = False):
    """Returns (output, new_state), plus the checkpoints [total, HV, V, K] when
    checkpoint_every_n_tokens > 0.  qk_l2norm normalises every q and k head
    vector as x / sqrt(sum(x^2) + 1e-6) first (AITER's / FLA's
    use_qk_l2norm_in_kernel, fla/modules/l2norm.py:42)."""
    lib = _load()
    T, H, K = q.shape
    HV, V = v.shape[1], v.shape[2]
    cu = cu_seqlens.detach().to("cpu", torch.int64).contiguous()
    N = cu.numel() - 1
    qf, kf, vf = _f32(q), _f32(k), _f32(v)
    sf = _f32(state) if state is not None else None
    Af, af, dtf, bf = _f32(A_log), _f32(a), _f32(dt_bias), _f32(b)
    out = torch.empty((T, HV, V), dtype=torch.int16)
    new_state = torch.empty((N, HV, V, K), dtype=torch.float32)
    every = int(checkpoint_every_n_tokens)
    ckpt = ckpt_cu = None
    if every > 0:
        ckpt_cu = checkpoint_cu_starts(cu, every)
        ckpt = torch.zeros((int(ckpt_cu[-1]), HV, V, K), dtype=torch.float32)
    rc = lib.gdn_oracle_prefill(
        _ptr(qf, _f32p), _ptr(kf, _f32p), _ptr(vf, _f32p), _ptr(sf, _f32p),
        _ptr(Af, _f32p), _ptr(af, _f32p), _ptr(dtf, _f32p), _ptr(bf, _f32p), _ptr(cu, _i64p),
        N, T, _scale(scale, K), H, HV, K, V,
        _ptr(out, _u16p), _ptr(new_state, _f32p), _ptr(ckpt, _f32p), _ptr(ckpt_cu, _i64p), every,
        int(bool(qk_l2norm)), int(threads))
    if rc != 0:
        raise ValueError(f"gdn_oracle_prefill rejected its arguments (rc={rc})")
    if every > 0:
        return out.view(torch.bfloat16), new_state, ckpt
    return out.view(torch.bfloat16), new_state


def mtp(q, k, v, initial_state, initial_state_indices, A_log, a, dt_bias, b, scale,
        intermediate_states_buffer=None, qk_l2norm: bool = False, output_state_indices=None,
        threads: int = 0, snapshots_by_entry: bool = False):
    """Returns (output [B,T,HV,V] bf16, final_state [pool,HV,V,K]) and fills
    intermediate_states_buffer ([slots,cache_steps>=T,HV,V,K] fp32) in place
    when given: the state after token t of the entry reading slot s goes to
    buffer[s, t], or with snapshots_by_entry to row i * T + t of the buffer
    seen as [slots * cache_steps] rows for batch entry i; an entry whose rows
    do not fit is skipped.  A bf16 initial_state selects the bf16-state form
    and gives a bf16 final_state."""
    lib = _load()
    B, T, H, K = q.shape
    HV, V = v.shape[2], v.shape[3]
    pool = initial_state.shape[0]
    qf, kf, vf = _f32(q), _f32(k), _f32(v)
    pin = _f32(initial_state)
    idx = initial_state_indices.detach().to("cpu", torch.int64).contiguous()
    oidx = None
    if output_state_indices is not None:
        oidx = output_state_indices.detach().to("cpu", torch.int64).contiguous()
    bf16_state = initial_state.dtype == torch.bfloat16
    Af, af, dtf, bf = _f32(A_log), _f32(a), _f32(dt_bias), _f32(b)
    out = torch.empty((B, T, HV, V), dtype=torch.int16)
    pout = torch.empty_like(pin)
    inter, steps, rows = None, T, 0
    if intermediate_states_buffer is not None:
        inter = _f32(intermediate_states_buffer).clone()
        steps = inter.shape[1]
        rows = inter.shape[0] * steps
    rc = lib.gdn_oracle_mtp(
        _ptr(qf, _f32p), _ptr(kf, _f32p), _ptr(vf, _f32p), _ptr(pin, _f32p), _ptr(pout, _f32p),
        _ptr(idx, _i64p), _ptr(oidx, _i64p), _ptr(Af, _f32p), _ptr(af, _f32p), _ptr(dtf, _f32p),
        _ptr(bf, _f32p), _scale(scale, K), B, T, H, HV, K, V, pool, int(bf16_state),
        int(bool(qk_l2norm)), _ptr(out, _u16p), _ptr(inter, _f32p), steps, rows,
        int(bool(snapshots_by_entry)), int(threads))
    if rc != 0:
        raise ValueError(f"gdn_oracle_mtp rejected its arguments (rc={rc})")
    if inter is not None:
        intermediate_states_buffer.copy_(inter)
    if bf16_state:
        pout = pout.to(torch.bfloat16)  # exact: every stored value is bf16-rounded
    return out.view(torch.bfloat16), pout

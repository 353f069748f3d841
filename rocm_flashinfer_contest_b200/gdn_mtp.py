"""Pool-indexed multi-token GDN decode (speculative verification) on B200.

Two entry points over the one CUDA kernel (``gdn_mtp_fwd`` in gdn_b200.h):

``run(q, k, v, initial_state, initial_state_indices, A_log, a, dt_bias, b,
scale, intermediate_states_buffer=None) -> (output, final_state)``
    The contest's MTP definition (flashinfer-python 0.6.11.post2,
    flashinfer/trace/templates/gdn.py:378-465): ``final_state`` is a new pool,
    a copy of ``initial_state`` with the named slots advanced; inputs are not
    modified; ``intermediate_states_buffer`` is filled in place.

``gated_delta_rule_mtp(q, k, v, initial_state, initial_state_indices, A_log,
a, dt_bias, b, scale=None, output=None, intermediate_states_buffer=None,
disable_state_update=None, use_qk_l2norm=True) -> (output, initial_state)``
    flashinfer's serving API (flashinfer/gdn_decode.py:557-745): the pool is
    updated in place unless ``disable_state_update``; q and k are
    L2-normalised in the kernel when ``use_qk_l2norm``.  As there,
    ``disable_state_update=None`` means True with a one-time warning, and the
    snapshots go where flashinfer's kernel puts them: batch entry i's state
    after token t to row i * T + t of the buffer seen as
    [slots * cache_steps] rows (gdn_kernels/gdn_decode_mtp.py:645; that is
    buffer[i, t] when cache_steps == T), where ``run`` follows the contest
    definition's buffer[slot, t].

Shapes: q, k [B, T, H, 128] bf16; v [B, T, HV, 128] bf16; a, b [B, T, HV]
bf16; A_log, dt_bias [HV] fp32; initial_state [pool, HV, 128, 128] fp32 or
bf16 (k-last; bf16 = the bf16-state form: advanced in fp32, rounded once when
stored); initial_state_indices [B] int32/int64; intermediate_states_buffer
[>= max slot + 1, >= T, HV, 128, 128] fp32 (fp32 pools only); output
[B, T, HV, 128] bf16.

An index outside [0, pool) is padding (flashinfer's -1): zero output, no state
touched.  The other indices must be distinct.
"""
from __future__ import annotations

import warnings

import torch

from . import _common as C
from ._lib import check, lib

_warned_default = False


def _validate(q, k, v, initial_state, initial_state_indices, A_log, a, dt_bias, b, buf):
    dev = C.cuda_device_of(q)
    bf, f32 = torch.bfloat16, torch.float32
    q = C.require(q, "q", bf, dev)
    k = C.require(k, "k", bf, dev)
    v = C.require(v, "v", bf, dev)
    a = C.require(a, "a", bf, dev)
    b = C.require(b, "b", bf, dev)
    A_log = C.require(A_log, "A_log", f32, dev)
    dt_bias = C.require(dt_bias, "dt_bias", f32, dev)
    if q.dim() != 4:
        raise ValueError(f"q must be [B, T, H, K], got {tuple(q.shape)}")
    B, T, H, K = q.shape
    if tuple(k.shape) != (B, T, H, K):
        raise ValueError(f"k must be {(B, T, H, K)}, got {tuple(k.shape)}")
    if v.dim() != 4 or tuple(v.shape[:2]) != (B, T):
        raise ValueError(f"v must be [B, T, HV, V], got {tuple(v.shape)}")
    HV, V = v.shape[2], v.shape[3]
    for name, t, shp in (("a", a, (B, T, HV)), ("b", b, (B, T, HV)),
                         ("A_log", A_log, (HV,)), ("dt_bias", dt_bias, (HV,))):
        if tuple(t.shape) != shp:
            raise ValueError(f"{name} must be {shp}, got {tuple(t.shape)}")
    if not isinstance(initial_state, torch.Tensor) or initial_state.dtype not in (f32, bf) \
            or initial_state.device != dev:
        raise TypeError("initial_state must be an fp32 or bf16 tensor on the inputs' device")
    if initial_state.dim() != 4 or tuple(initial_state.shape[1:]) != (HV, V, K):
        raise ValueError(f"initial_state must be [pool, {HV}, {V}, {K}], got {tuple(initial_state.shape)}")
    idx = initial_state_indices
    if not isinstance(idx, torch.Tensor) or idx.dtype not in (torch.int32, torch.int64) \
            or idx.device != dev or tuple(idx.shape) != (B,):
        raise ValueError(f"initial_state_indices must be an int32/int64 [{B}] tensor on {dev}")
    idx = idx.contiguous()
    steps = slots = 0
    if buf is not None and initial_state.dtype != f32:
        raise ValueError("intermediate_states_buffer needs an fp32 state pool")
    if buf is not None:
        if not isinstance(buf, torch.Tensor) or buf.dtype != f32 or buf.device != dev \
                or not buf.is_contiguous():
            raise ValueError("intermediate_states_buffer must be a contiguous fp32 tensor on the inputs' device")
        if buf.dim() != 5 or tuple(buf.shape[2:]) != (HV, V, K) or buf.shape[1] < T:
            raise ValueError(f"intermediate_states_buffer must be [slots, >= {T}, {HV}, {V}, {K}], "
                             f"got {tuple(buf.shape)}")
        slots, steps = buf.shape[0], buf.shape[1]
    return dev, (q, k, v, idx, A_log, a, dt_bias, b), (B, T, H, HV, K, V), (slots, steps)


def _out_indices(out_idx, idx, B, dev):
    if out_idx is None:
        return None
    if not isinstance(out_idx, torch.Tensor) or out_idx.device != dev or tuple(out_idx.shape) != (B,) \
            or out_idx.dtype not in (torch.int32, torch.int64):
        raise ValueError(f"output_state_indices must be an int32/int64 [{B}] tensor on {dev}")
    return out_idx.to(idx.dtype).contiguous()


GDN_MTP_QK_L2NORM = 1           # gdn_mtp_fwd flags (include/gdn_b200.h)
GDN_MTP_SNAPSHOTS_BY_ENTRY = 2


def _launch(dev, tensors, dims, pool_in, pool_out, scale, output, buf, slots, steps, l2norm,
            out_idx=None, snapshots_by_entry=False):
    q, k, v, idx, A_log, a, dt_bias, b = tensors
    B, T, H, HV, K, V = dims
    flags = (GDN_MTP_QK_L2NORM if l2norm else 0) | (GDN_MTP_SNAPSHOTS_BY_ENTRY if snapshots_by_entry else 0)
    st = lib().gdn_mtp_fwd(
        C.ptr(q), C.ptr(k), C.ptr(v), C.ptr(pool_in), C.ptr(pool_out),
        int(pool_in.dtype == torch.bfloat16), C.ptr(idx), C.ptr(out_idx),
        int(idx.dtype == torch.int64), C.ptr(A_log), C.ptr(a), C.ptr(dt_bias), C.ptr(b),
        C.normalize_scale(scale, K), B, T, H, HV, K, V, pool_in.shape[0], flags,
        C.ptr(output), C.ptr(buf), slots, steps, C.stream_handle(dev))
    check("gdn_mtp_fwd", st)


def _check_output(output, B, T, HV, V, dev):
    if output.dtype != torch.bfloat16 or tuple(output.shape) != (B, T, HV, V) \
            or not output.is_contiguous() or output.device != dev:
        raise ValueError(f"output must be a contiguous bf16 {(B, T, HV, V)} tensor on {dev}")


def run_into(q, k, v, initial_state, initial_state_indices, A_log, a, dt_bias, b, scale,
             output, final_state, intermediate_states_buffer=None, qk_l2norm: bool = False,
             output_state_indices=None):
    """Destination-passing form: writes ``output`` and ``final_state``
    (``final_state`` may be ``initial_state`` for an in-place update, or None
    to leave every state as it is); ``output_state_indices`` redirects each
    entry's final state to another slot."""
    dev, tensors, dims, (slots, steps) = _validate(
        q, k, v, initial_state, initial_state_indices, A_log, a, dt_bias, b, intermediate_states_buffer)
    B, T, H, HV, K, V = dims
    _check_output(output, B, T, HV, V, dev)
    if not initial_state.is_contiguous():
        raise ValueError("initial_state must be contiguous")
    if final_state is not None and (final_state.dtype != initial_state.dtype or final_state.device != dev
                                    or tuple(final_state.shape) != tuple(initial_state.shape)
                                    or not final_state.is_contiguous()):
        raise ValueError("final_state must be a contiguous tensor shaped and typed like initial_state")
    oidx = _out_indices(output_state_indices, tensors[3], B, dev)
    _launch(dev, tensors, dims, initial_state, final_state, scale, output,
            intermediate_states_buffer, slots, steps, qk_l2norm, oidx)
    return output, final_state


def run(q, k, v, initial_state, initial_state_indices, A_log, a, dt_bias, b, scale,
        intermediate_states_buffer=None):
    """Contest MTP definition; see the module docstring."""
    dev, tensors, dims, (slots, steps) = _validate(
        q, k, v, initial_state, initial_state_indices, A_log, a, dt_bias, b, intermediate_states_buffer)
    B, T, H, HV, K, V = dims
    pool_in = initial_state.contiguous()
    output = torch.empty((B, T, HV, V), dtype=torch.bfloat16, device=dev)
    final_state = torch.empty_like(pool_in)
    _launch(dev, tensors, dims, pool_in, final_state, scale, output, intermediate_states_buffer, slots, steps,
            False)
    return output, final_state


def gated_delta_rule_mtp(q, k, v, initial_state, initial_state_indices, A_log, a, dt_bias, b,
                         scale=None, output=None, intermediate_states_buffer=None,
                         disable_state_update=None, use_qk_l2norm: bool = True):
    """flashinfer's ``gated_delta_rule_mtp``; see the module docstring."""
    global _warned_default
    if disable_state_update is None:
        if not _warned_default:
            warnings.warn("gated_delta_rule_mtp(): 'disable_state_update' defaults to True; "
                          "pass it explicitly", stacklevel=2)
            _warned_default = True
        disable_state_update = True
    dev, tensors, dims, (slots, steps) = _validate(
        q, k, v, initial_state, initial_state_indices, A_log, a, dt_bias, b, intermediate_states_buffer)
    B, T, H, HV, K, V = dims
    target = None
    if output is None or output.dtype != torch.bfloat16 or not output.is_contiguous():
        target = output
        output = torch.empty((B, T, HV, V), dtype=torch.bfloat16, device=dev)
    _check_output(output, B, T, HV, V, dev)
    pool = initial_state if initial_state.is_contiguous() else initial_state.contiguous()
    _launch(dev, tensors, dims, pool, None if disable_state_update else pool, scale, output,
            intermediate_states_buffer, slots, steps, use_qk_l2norm, snapshots_by_entry=True)
    if not disable_state_update and pool is not initial_state:
        initial_state.copy_(pool)
    if target is not None:
        target.copy_(output)
        output = target
    return output, initial_state

"""``run`` for the contest definition ``gdn_prefill_*_k_last`` on B200.

Same signature, argument order, dtypes and return tuple as the reference
solution (solutions/gdn_prefill/main.py:31-84) and the contest definition
(flashinfer/trace/templates/gdn.py:276-373):

    run(q, k, v, state, A_log, a, dt_bias, b, cu_seqlens, scale)
        -> (output, new_state)

    q, k     [T, H, 128] bf16          v     [T, HV, 128] bf16
    state    [N, HV, 128, 128] fp32 (k-last) or None
    A_log    [HV] fp32    a, b [T, HV] bf16    dt_bias [HV] fp32
    cu_seqlens [N + 1] int32 or int64 (read on the device only)
    output   [T, HV, 128] bf16         new_state [N, HV, 128, 128] fp32

A zero-length sequence gets an all-zero final state (gdn.py:234-235).

State checkpoints (keyword-only, the names and rules of flashinfer's
chunk_gated_delta_rule, flashinfer/gdn_prefill.py:113-115,161-214):
``state_checkpoints`` [total, HV, 128, 128] fp32, ``checkpoint_cu_starts``
[N + 1] int64 (sequence n owns ``len_n // every`` slots, see
``checkpoint_cu_starts_for``) and ``checkpoint_every_n_tokens`` (a positive
multiple of 64, 0 = off): the state after tokens every, 2*every, ... of each
sequence is written to its slots.
``use_qk_l2norm_in_kernel=True`` (keyword-only, the option of the AITER
kernels the reference calls, solutions/gdn_prefill/main.py:72,79) normalises
every q and k head vector in the kernel as x * rsqrt(sum(x^2) + 1e-6).
``run_host_into(...)`` is the same prefill for tensors in pinned host memory
(``gdn_prefill_fwd_host``): token segments are copied up, prefilled and
copied back on overlapping streams.
Inputs are never modified; ``run_into`` is the destination-passing form and
accepts ``new_state is state``.  The chunked kernels' workspace
(gdn_prefill_workspace_bytes) comes from torch's caching allocator, so a
call makes no cudaMalloc in steady state.
"""
from __future__ import annotations

import torch

from . import _common as C
from ._lib import check, lib

GDN_PREFILL_QK_L2NORM = 1  # gdn_prefill_fwd_ex flag (include/gdn_b200.h)

def _validate(q, k, v, state, A_log, a, dt_bias, b, cu_seqlens):
    dev = C.cuda_device_of(q)
    bf, f32 = torch.bfloat16, torch.float32
    q = C.require(q, "q", bf, dev)
    k = C.require(k, "k", bf, dev)
    v = C.require(v, "v", bf, dev)
    a = C.require(a, "a", bf, dev)
    b = C.require(b, "b", bf, dev)
    A_log = C.require(A_log, "A_log", f32, dev)
    dt_bias = C.require(dt_bias, "dt_bias", f32, dev)
    if not isinstance(cu_seqlens, torch.Tensor) or cu_seqlens.dtype not in (torch.int32, torch.int64):
        raise TypeError("cu_seqlens must be an int32 or int64 tensor")
    if cu_seqlens.device != dev:
        raise ValueError(f"cu_seqlens is on {cu_seqlens.device}, expected {dev}")
    cu_seqlens = cu_seqlens.contiguous()
    if q.dim() != 3:
        raise ValueError(f"q must be [T, H, K], got {tuple(q.shape)}")
    T, H, K = q.shape
    if tuple(k.shape) != (T, H, K):
        raise ValueError(f"k must be {(T, H, K)}, got {tuple(k.shape)}")
    if v.dim() != 3 or v.shape[0] != T:
        raise ValueError(f"v must be [T, HV, V], got {tuple(v.shape)}")
    HV, V = v.shape[1], v.shape[2]
    if cu_seqlens.dim() != 1 or cu_seqlens.numel() < 1:
        raise ValueError("cu_seqlens must be a 1-d tensor of N + 1 offsets")
    N = cu_seqlens.numel() - 1
    for name, t, shp in (("a", a, (T, HV)), ("b", b, (T, HV)),
                         ("A_log", A_log, (HV,)), ("dt_bias", dt_bias, (HV,))):
        if tuple(t.shape) != shp:
            raise ValueError(f"{name} must be {shp}, got {tuple(t.shape)}")
    if state is not None:
        state = C.require(state, "state", f32, dev)
        if tuple(state.shape) != (N, HV, V, K):
            raise ValueError(f"state must be {(N, HV, V, K)}, got {tuple(state.shape)}")
    return dev, (q, k, v, state, A_log, a, dt_bias, b, cu_seqlens), (T, N, H, HV, K, V)


def checkpoint_cu_starts_for(cu_seqlens: torch.Tensor, every: int) -> torch.Tensor:
    """``checkpoint_cu_starts`` for ``cu_seqlens``: [N + 1] int64 on the same
    device, sequence n getting ``len_n // every`` slots."""
    cu = cu_seqlens.to(torch.int64)
    out = torch.zeros_like(cu)
    out[1:] = torch.cumsum((cu[1:] - cu[:-1]).clamp_min(0) // every, 0)
    return out


def _validate_checkpoints(state_checkpoints, checkpoint_cu_starts, every, N, HV, K, dev):
    every = int(every)
    if every < 0:
        raise ValueError(f"checkpoint_every_n_tokens must be non-negative, got {every}")
    if every == 0:
        if state_checkpoints is not None or checkpoint_cu_starts is not None:
            raise ValueError("state_checkpoints and checkpoint_cu_starts must be None "
                             "when checkpoint_every_n_tokens == 0")
        return None
    if every % 64 != 0:
        raise ValueError(f"checkpoint_every_n_tokens must be a multiple of the chunk size (64), got {every}")
    if state_checkpoints is None or checkpoint_cu_starts is None:
        raise ValueError("state_checkpoints and checkpoint_cu_starts must both be provided "
                         "when checkpoint_every_n_tokens > 0")
    if state_checkpoints.dtype != torch.float32 or state_checkpoints.device != dev \
            or state_checkpoints.dim() != 4 or tuple(state_checkpoints.shape[1:]) != (HV, K, K) \
            or not state_checkpoints.is_contiguous():
        raise ValueError(f"state_checkpoints must be a contiguous fp32 [*, {HV}, {K}, {K}] tensor on {dev}")
    if checkpoint_cu_starts.dtype != torch.int64 or checkpoint_cu_starts.device != dev \
            or tuple(checkpoint_cu_starts.shape) != (N + 1,):
        raise ValueError(f"checkpoint_cu_starts must be an int64 [{N + 1}] tensor on {dev}")
    return state_checkpoints, checkpoint_cu_starts.contiguous(), every


def run_into(q, k, v, state, A_log, a, dt_bias, b, cu_seqlens, scale, output, new_state, *,
             state_checkpoints=None, checkpoint_cu_starts=None, checkpoint_every_n_tokens: int = 0,
             use_qk_l2norm_in_kernel: bool = False):
    """Destination-passing prefill into ``output`` [T,HV,V] bf16 and
    ``new_state`` [N,HV,V,K] fp32 (``new_state`` may be ``state``)."""
    return _run_checked(*_validate(q, k, v, state, A_log, a, dt_bias, b, cu_seqlens), scale, output, new_state,
                        state_checkpoints, checkpoint_cu_starts, checkpoint_every_n_tokens,
                        use_qk_l2norm_in_kernel)


def _run_checked(dev, args, dims, scale, output, new_state, state_checkpoints, checkpoint_cu_starts,
                 checkpoint_every_n_tokens, use_qk_l2norm_in_kernel):
    T, N, H, HV, K, V = dims
    ck = _validate_checkpoints(state_checkpoints, checkpoint_cu_starts, checkpoint_every_n_tokens,
                               N, HV, K, dev)
    q, k, v, state, A_log, a, dt_bias, b, cu = args
    if output.dtype != torch.bfloat16 or tuple(output.shape) != (T, HV, V) \
            or not output.is_contiguous() or output.device != dev:
        raise ValueError("output must be a contiguous bf16 [T, HV, V] tensor on the inputs' device")
    if new_state.dtype != torch.float32 or tuple(new_state.shape) != (N, HV, V, K) \
            or not new_state.is_contiguous() or new_state.device != dev:
        raise ValueError("new_state must be a contiguous fp32 [N, HV, V, K] tensor on the inputs' device")
    scale = C.normalize_scale(scale, K)
    ws_bytes = lib().gdn_prefill_workspace_bytes(N, T, H, HV)
    ws = torch.empty(ws_bytes, dtype=torch.uint8, device=dev) if ws_bytes else None
    if ck is None and not use_qk_l2norm_in_kernel:
        st = lib().gdn_prefill_fwd(
            C.ptr(q), C.ptr(k), C.ptr(v), C.ptr(state), C.ptr(A_log), C.ptr(a), C.ptr(dt_bias),
            C.ptr(b), C.ptr(cu), 1 if cu.dtype == torch.int64 else 0, N, T, scale, H, HV, K, V,
            C.ptr(output), C.ptr(new_state), C.ptr(ws), ws_bytes, C.stream_handle(dev))
        check("gdn_prefill_fwd", st)
    else:
        ckpt, ckpt_cu, every = ck if ck is not None else (None, None, 0)
        st = lib().gdn_prefill_fwd_ex(
            C.ptr(q), C.ptr(k), C.ptr(v), C.ptr(state), C.ptr(A_log), C.ptr(a), C.ptr(dt_bias),
            C.ptr(b), C.ptr(cu), 1 if cu.dtype == torch.int64 else 0, N, T, scale, H, HV, K, V,
            C.ptr(output), C.ptr(new_state), C.ptr(ckpt), C.ptr(ckpt_cu),
            0 if ckpt is None else ckpt.shape[0], every, GDN_PREFILL_QK_L2NORM if use_qk_l2norm_in_kernel else 0,
            C.ptr(ws), ws_bytes, C.stream_handle(dev))
        check("gdn_prefill_fwd_ex", st)
    return output, new_state


def run(q, k, v, state, A_log, a, dt_bias, b, cu_seqlens, scale, *,
        state_checkpoints=None, checkpoint_cu_starts=None, checkpoint_every_n_tokens: int = 0,
        use_qk_l2norm_in_kernel: bool = False):
    """Contest entry point; see the module docstring."""
    dev, args, dims = _validate(q, k, v, state, A_log, a, dt_bias, b, cu_seqlens)
    T, N, H, HV, K, V = dims
    output = torch.empty((T, HV, V), dtype=torch.bfloat16, device=dev)
    new_state = torch.empty((N, HV, V, K), dtype=torch.float32, device=dev)
    return _run_checked(dev, args, dims, scale, output, new_state, state_checkpoints, checkpoint_cu_starts,
                        checkpoint_every_n_tokens, use_qk_l2norm_in_kernel)


def run_host_into(q, k, v, state, A_log, a, dt_bias, b, cu_seqlens, scale, output, new_state, *,
                  device=None, segment_tokens: int = 0):
    """Prefill with every tensor in pinned host memory (``gdn_prefill_fwd_host``):
    writes ``output`` [T,HV,V] bf16 and ``new_state`` [N,HV,V,K] fp32 (host,
    pinned) and returns them.  ``cu_seqlens`` is a host int32/int64 tensor.
    The work is queued on ``device`` (default: the current CUDA device) on its
    current stream, which continues after the last copy back, so a
    synchronisation of that stream (or an event recorded on it) marks the
    results as ready.  Tokens go up, through the kernels and back in segments
    of ``segment_tokens`` (0: 2048; the last ones halved down to 256) on
    overlapping streams; the results equal
    ``run`` on device copies to rounding.  The inputs must stay unmodified and
    alive until then, as with any non-blocking copy."""
    dev = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
    host = {"q": q, "k": k, "v": v, "a": a, "b": b, "A_log": A_log, "dt_bias": dt_bias,
            "cu_seqlens": cu_seqlens, "output": output, "new_state": new_state}
    if state is not None:
        host["state"] = state
    for name, t in host.items():
        if not isinstance(t, torch.Tensor) or t.device.type != "cpu" or not t.is_contiguous() \
                or (t.numel() > 0 and not t.is_pinned()):
            raise ValueError(f"{name} must be a contiguous pinned host tensor")
    if q.dim() != 3:
        raise ValueError(f"q must be [T, H, K], got {tuple(q.shape)}")
    T, H, K = q.shape
    if v.dim() != 3:
        raise ValueError(f"v must be [T, HV, V], got {tuple(v.shape)}")
    HV, V = v.shape[1], v.shape[2]
    if cu_seqlens.dim() != 1 or cu_seqlens.dtype not in (torch.int32, torch.int64):
        raise ValueError("cu_seqlens must be a 1-D int32 or int64 tensor")
    N = cu_seqlens.numel() - 1
    bf, f32 = torch.bfloat16, torch.float32
    spec = {"q": (bf, (T, H, K)), "k": (bf, (T, H, K)), "v": (bf, (T, HV, V)), "a": (bf, (T, HV)),
            "b": (bf, (T, HV)), "A_log": (f32, (HV,)), "dt_bias": (f32, (HV,)), "output": (bf, (T, HV, V)),
            "new_state": (f32, (N, HV, V, K)), "state": (f32, (N, HV, V, K))}
    for name, t in host.items():
        if name in spec and (t.dtype != spec[name][0] or tuple(t.shape) != spec[name][1]):
            raise ValueError(f"{name} must be {spec[name][0]} {spec[name][1]}, got {t.dtype} {tuple(t.shape)}")
    L = lib()
    nbytes = L.gdn_prefill_host_workspace_bytes(N, T, H, HV, int(segment_tokens))
    if nbytes == 0:
        return output, new_state
    with torch.cuda.device(dev):
        # allocated on the stream the call joins at its end: freeing it when this
        # function returns is ordered after the last copy back
        ws = torch.empty(nbytes, dtype=torch.uint8, device=dev)
        st = L.gdn_prefill_fwd_host(
            q.data_ptr(), k.data_ptr(), v.data_ptr(), None if state is None else state.data_ptr(),
            A_log.data_ptr(), a.data_ptr(), dt_bias.data_ptr(), b.data_ptr(), cu_seqlens.data_ptr(),
            int(cu_seqlens.dtype == torch.int64), N, T, C.normalize_scale(scale, K), H, HV, K, V,
            output.data_ptr(), new_state.data_ptr(), ws.data_ptr(), ws.numel(), int(segment_tokens),
            C.stream_handle(dev))
    check("gdn_prefill_fwd_host", st)
    return output, new_state

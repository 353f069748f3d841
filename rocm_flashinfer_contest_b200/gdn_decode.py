"""``run`` for the contest definition ``gdn_decode_*_k_last`` on B200.

Same signature, argument order, dtypes and return tuple as the reference
solution (solutions/gdn_decode/main.py:117-135) and the contest definition
(flashinfer/trace/templates/gdn.py:97-184):

    run(q, k, v, state, A_log, a, dt_bias, b, scale) -> (output, new_state)

    q, k     [B, 1, H, 128]   bf16        v        [B, 1, HV, 128] bf16
    state    [B, HV, 128, 128] fp32 (k-last [B, HV, V, K]) or None
    A_log    [HV] fp32        a, b [B, 1, HV] bf16      dt_bias [HV] fp32
    scale    float or 0-d tensor; 0 / None -> 1/sqrt(128)
    output   [B, 1, HV, 128]  bf16        new_state [B, HV, 128, 128] fp32

Inputs are never modified: ``new_state`` is a fresh tensor, as in the
reference (main.py:104).

``run_host_into(q, k, v, state, A_log, a, dt_bias, b, scale, output, new_state)``
is the same decode for a caller whose states live in (pinned) host memory,
e.g. a serving loop that offloads recurrent states between steps: the batch
is cut into chunks, chunk i + 1 is copied up while chunk i's results are
copied back (PCIe moves data both ways at once), and each chunk runs the same
kernel, so the results are identical to ``run`` on device copies.

``gated_delta_rule_decode_pretranspose(...)`` is flashinfer's serving decode
API (flashinfer/gdn_decode.py:118-330): state fp32 or bf16 ([B, HV, V, K],
updated in place) or a slot pool (``initial_state`` + ``initial_state_indices``,
optional ``output_state_indices``, ``-1`` padding), T >= 1 tokens per entry,
in-kernel q/k L2-norm by default.  It runs the pool kernel of gdn_mtp.  ``run_into`` is the destination-passing form; it
accepts ``new_state is state`` for an in-place update with identical traffic.
One kernel launch on the current stream of the inputs' device; no host sync
unless ``scale`` is a device tensor (the reference reads it with ``.item()``).
"""
from __future__ import annotations

import torch

from . import _common as C
from ._lib import check, lib


def _validate(q, k, v, state, A_log, a, dt_bias, b):
    dev = C.cuda_device_of(q)
    bf, f32 = torch.bfloat16, torch.float32
    q = C.require(q, "q", bf, dev)
    k = C.require(k, "k", bf, dev)
    v = C.require(v, "v", bf, dev)
    a = C.require(a, "a", bf, dev)
    b = C.require(b, "b", bf, dev)
    A_log = C.require(A_log, "A_log", f32, dev)
    dt_bias = C.require(dt_bias, "dt_bias", f32, dev)
    if q.dim() != 4 or q.shape[1] != 1:
        raise ValueError(f"q must be [B, 1, H, K], got {tuple(q.shape)}")
    B, _, H, K = q.shape
    if tuple(k.shape) != (B, 1, H, K):
        raise ValueError(f"k must be {(B, 1, H, K)}, got {tuple(k.shape)}")
    if v.dim() != 4 or v.shape[0] != B or v.shape[1] != 1:
        raise ValueError(f"v must be [B, 1, HV, V], got {tuple(v.shape)}")
    HV, V = v.shape[2], v.shape[3]
    for name, t, shp in (("a", a, (B, 1, HV)), ("b", b, (B, 1, HV)),
                         ("A_log", A_log, (HV,)), ("dt_bias", dt_bias, (HV,))):
        if tuple(t.shape) != shp:
            raise ValueError(f"{name} must be {shp}, got {tuple(t.shape)}")
    if state is not None:
        state = C.require(state, "state", f32, dev)
        if tuple(state.shape) != (B, HV, V, K):
            raise ValueError(f"state must be {(B, HV, V, K)}, got {tuple(state.shape)}")
    return dev, (q, k, v, state, A_log, a, dt_bias, b), (B, H, HV, K, V)


def run_into(q, k, v, state, A_log, a, dt_bias, b, scale, output, new_state):
    """Destination-passing decode: writes ``output`` [B,1,HV,V] bf16 and
    ``new_state`` [B,HV,V,K] fp32 (``new_state`` may be ``state``)."""
    return _run_checked(*_validate(q, k, v, state, A_log, a, dt_bias, b), scale, output, new_state)


def _run_checked(dev, tensors, dims, scale, output, new_state):
    q, k, v, state, A_log, a, dt_bias, b = tensors
    B, H, HV, K, V = dims
    if output.dtype != torch.bfloat16 or tuple(output.shape) != (B, 1, HV, V) \
            or not output.is_contiguous() or output.device != dev:
        raise ValueError("output must be a contiguous bf16 [B, 1, HV, V] tensor on the inputs' device")
    if new_state.dtype != torch.float32 or tuple(new_state.shape) != (B, HV, V, K) \
            or not new_state.is_contiguous() or new_state.device != dev:
        raise ValueError("new_state must be a contiguous fp32 [B, HV, V, K] tensor on the inputs' device")
    scale = C.normalize_scale(scale, K)
    st = lib().gdn_decode_fwd(
        C.ptr(q), C.ptr(k), C.ptr(v), C.ptr(state), C.ptr(A_log), C.ptr(a), C.ptr(dt_bias),
        C.ptr(b), scale, B, H, HV, K, V, C.ptr(output), C.ptr(new_state), C.stream_handle(dev))
    check("gdn_decode_fwd", st)
    return output, new_state


def run(q, k, v, state, A_log, a, dt_bias, b, scale):
    """Contest entry point; see the module docstring."""
    dev, tensors, (B, H, HV, K, V) = _validate(q, k, v, state, A_log, a, dt_bias, b)
    output = torch.empty((B, 1, HV, V), dtype=torch.bfloat16, device=dev)
    new_state = torch.empty((B, HV, V, K), dtype=torch.float32, device=dev)
    return _run_checked(dev, tensors, (B, H, HV, K, V), scale, output, new_state)


def gated_delta_rule_decode_pretranspose(q, k, v, state, A_log, a, dt_bias, b, scale=None,
                                         output=None, use_qk_l2norm: bool = True,
                                         initial_state=None, initial_state_indices=None,
                                         output_state_indices=None):
    """flashinfer's ``gated_delta_rule_decode_pretranspose``: returns
    ``(output [B, T, HV, V], state or initial_state)``, the state updated in
    place.  Padding entries (index outside the pool) get a zero output and
    leave every slot untouched, for fp32 and bf16 states alike."""
    from . import gdn_mtp

    use_pool = initial_state is not None
    if use_pool != (initial_state_indices is not None):
        raise ValueError("initial_state and initial_state_indices must be provided together")
    if output_state_indices is not None and not use_pool:
        raise ValueError("output_state_indices can only be used with initial_state (pool mode)")
    dev = C.cuda_device_of(q)
    if q.dim() != 4:
        raise ValueError(f"q must be [B, T, H, K], got {tuple(q.shape)}")
    B, T = q.shape[0], q.shape[1]
    if use_pool:
        pool, idx = initial_state, initial_state_indices
    else:
        if state is None:
            raise ValueError("either state or initial_state must be provided")
        pool, idx = state, torch.arange(B, dtype=torch.int32, device=dev)
    if not pool.is_contiguous():
        raise ValueError("the state must be contiguous (k-last [.., HV, V, K])")
    HV, V = v.shape[2], v.shape[3]
    target = output
    out = output if (output is not None and output.dtype == torch.bfloat16 and output.is_contiguous()
                     and tuple(output.shape) == (B, T, HV, V)) else None
    if out is None:
        out = torch.empty((B, T, HV, V), dtype=torch.bfloat16, device=dev)
    gdn_mtp.run_into(q, k, v, pool, idx, A_log, a, dt_bias, b, scale, out, pool,
                     qk_l2norm=use_qk_l2norm, output_state_indices=output_state_indices)
    if target is not None and target is not out:
        target.copy_(out.view(target.shape))
        out = target
    return out, (initial_state if use_pool else state)


def run_host_into(q, k, v, state, A_log, a, dt_bias, b, scale, output, new_state, *, device=None,
                  chunks: int = 0):
    """Decode with every tensor in pinned host memory (``gdn_decode_fwd_host``):
    writes ``output`` [B,1,HV,V] bf16 and ``new_state`` [B,HV,V,K] fp32 (host,
    pinned; ``new_state`` may be ``state``) and returns them.  The work is
    queued on ``device`` (default: the current CUDA device) on its current
    stream, which continues after the last copy back, so
    ``torch.cuda.current_stream().synchronize()`` (or an event recorded on
    it) marks the results as ready.  ``chunks`` batch slices pipeline the two
    copy directions (0: about 16 MiB of state each).  The inputs must stay
    unmodified and alive until then, as with any non-blocking copy."""
    dev = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
    host = {"q": q, "k": k, "v": v, "a": a, "b": b, "A_log": A_log, "dt_bias": dt_bias,
            "output": output, "new_state": new_state}
    if state is not None:
        host["state"] = state
    for name, t in host.items():
        if not isinstance(t, torch.Tensor) or t.device.type != "cpu" or not t.is_pinned() or not t.is_contiguous():
            raise ValueError(f"{name} must be a contiguous pinned host tensor")
    if q.dim() != 4 or q.shape[1] != 1:
        raise ValueError(f"q must be [B, 1, H, K], got {tuple(q.shape)}")
    B, _, H, K = q.shape
    if v.dim() != 4:
        raise ValueError(f"v must be [B, 1, HV, V], got {tuple(v.shape)}")
    HV, V = v.shape[2], v.shape[3]
    bf, f32 = torch.bfloat16, torch.float32
    spec = {"q": (bf, (B, 1, H, K)), "k": (bf, (B, 1, H, K)), "v": (bf, (B, 1, HV, V)),
            "a": (bf, (B, 1, HV)), "b": (bf, (B, 1, HV)), "A_log": (f32, (HV,)), "dt_bias": (f32, (HV,)),
            "output": (bf, (B, 1, HV, V)), "new_state": (f32, (B, HV, V, K)), "state": (f32, (B, HV, V, K))}
    for name, t in host.items():
        dt, shp = spec[name]
        if t.dtype != dt or tuple(t.shape) != shp:
            raise ValueError(f"{name} must be {dt} {shp}, got {t.dtype} {tuple(t.shape)}")
    if B == 0:
        return output, new_state
    L = lib()
    # allocated on the stream the call joins at its end, so freeing it when
    # this function returns is ordered after the last copy back
    with torch.cuda.device(dev):
        ws = torch.empty(L.gdn_decode_host_workspace_bytes(B, H, HV), dtype=torch.uint8, device=dev)
        rc = L.gdn_decode_fwd_host(
            q.data_ptr(), k.data_ptr(), v.data_ptr(), None if state is None else state.data_ptr(),
            A_log.data_ptr(), a.data_ptr(), dt_bias.data_ptr(), b.data_ptr(), C.normalize_scale(scale, K),
            B, H, HV, K, V, output.data_ptr(), new_state.data_ptr(), ws.data_ptr(), ws.numel(), int(chunks),
            C.stream_handle(dev))
    check("gdn_decode_fwd_host", rc)
    return output, new_state

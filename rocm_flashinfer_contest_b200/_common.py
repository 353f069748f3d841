"""Argument handling shared by the decode and prefill ``run`` shims."""
from __future__ import annotations

import math

import torch


def normalize_scale(scale, K: int) -> float:
    """The reference's scale rule (solutions/gdn_decode/main.py:118-123,
    solutions/gdn_prefill/main.py:32-37): a tensor is read with ``.item()``,
    ``None`` or 0 means 1/sqrt(K)."""
    if isinstance(scale, torch.Tensor):
        scale = float(scale.item())
    elif scale is None:
        scale = 0.0
    else:
        scale = float(scale)
    if scale == 0.0:
        scale = 1.0 / math.sqrt(K)
    return scale


def require(t: torch.Tensor, name: str, dtype: torch.dtype, device: torch.device) -> torch.Tensor:
    if not isinstance(t, torch.Tensor):
        raise TypeError(f"{name} must be a torch.Tensor, got {type(t).__name__}")
    if t.dtype != dtype:
        raise TypeError(f"{name} must be {dtype}, got {t.dtype}")
    if t.device != device:
        raise ValueError(f"{name} is on {t.device}, expected {device}")
    return t if t.is_contiguous() else t.contiguous()


def cuda_device_of(q: torch.Tensor) -> torch.device:
    if not isinstance(q, torch.Tensor) or q.device.type != "cuda":
        raise RuntimeError(
            "the GDN kernels run on CUDA devices only (sm_100a); got "
            f"{getattr(q, 'device', type(q).__name__)} — there is no CPU path")
    return q.device


_raw_stream = getattr(torch._C, "_cuda_getCurrentRawStream", None)


def stream_handle(device: torch.device) -> int:
    """The device's current CUDA stream as a raw handle (torch's internal
    accessor, ~0.1 us, when it exists; the public one builds a Stream object
    on every call, ~2 us)."""
    if _raw_stream is not None:
        return _raw_stream(device.index if device.index is not None else torch.cuda.current_device())
    return torch.cuda.current_stream(device).cuda_stream


def ptr(t) -> int:
    return 0 if t is None else t.data_ptr()

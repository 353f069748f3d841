"""Tolerances and comparison helpers shared by the parity tests.

The parity bar (the contest's, tools/run_benchmarks.py:138-141 of the
reference, tightened for the state):
  * bf16 outputs: |s - r| <= 1e-2 + 1e-2 * |r| for every element
    (allclose with atol = rtol = 1e-2, matched ratio 1.0);
  * fp32 final state: |s - r| <= 1e-3 * |r| + 1e-3 * max|r| for every element,
    and the normwise relative error ||s - r|| / ||r|| is reported.
"""
from __future__ import annotations

import numpy as np
import torch

OUT_ATOL = 1e-2
OUT_RTOL = 1e-2
STATE_RTOL = 1e-3
STATE_MAXREL = 1e-3


def _f32(x):
    if isinstance(x, np.ndarray):
        x = torch.from_numpy(x)
    return x.detach().to("cpu", torch.float32)


def output_report(sol, ref, atol=OUT_ATOL, rtol=OUT_RTOL):
    s, r = _f32(sol), _f32(ref)
    assert s.shape == r.shape, (s.shape, r.shape)
    err = (s - r).abs()
    bound = atol + rtol * r.abs()
    bad = int((err > bound).sum())
    return {"max_abs": float(err.max()) if err.numel() else 0.0,
            "bad": bad, "n": err.numel(), "nonfinite": int((~torch.isfinite(s)).sum())}


def state_report(sol, ref, rtol=STATE_RTOL, maxrel=STATE_MAXREL):
    s, r = _f32(sol), _f32(ref)
    assert s.shape == r.shape, (s.shape, r.shape)
    err = (s - r).abs()
    rmax = float(r.abs().max()) if r.numel() else 0.0
    bound = rtol * r.abs() + maxrel * rmax
    bad = int((err > bound).sum())
    rn = float(r.norm())
    return {"max_abs": float(err.max()) if err.numel() else 0.0,
            "normwise": float((s - r).norm()) / rn if rn > 0 else float((s - r).norm()),
            "bad": bad, "n": err.numel(), "nonfinite": int((~torch.isfinite(s)).sum())}


def assert_output_close(sol, ref, what="output", **kw):
    rep = output_report(sol, ref, **kw)
    assert rep["nonfinite"] == 0 and rep["bad"] == 0, f"{what}: {rep}"
    return rep


def assert_state_close(sol, ref, what="new_state", **kw):
    rep = state_report(sol, ref, **kw)
    assert rep["nonfinite"] == 0 and rep["bad"] == 0, f"{what}: {rep}"
    return rep


def bf16_from_u16(a: np.ndarray) -> torch.Tensor:
    return torch.from_numpy(a.astype(np.uint16).view(np.int16)).view(torch.bfloat16)

"""Generates the golden fixtures that pin the CPU oracle (oracle/gdn_oracle.c).

The fixtures are inputs and outputs of the contest's own pure-torch reference
for the GDN definitions, ``_gdn_decode_reference`` and
``_gdn_prefill_reference`` (third-party package flashinfer-python
0.6.11.post2, flashinfer/trace/templates/gdn.py:27-94 and :189-273), run on
the CPU on small seeded inputs.  That reference is the oracle the reference
repository is scored against (its tools/local_verify.py:94,108 builds and runs
it through flashinfer-bench).  The reference repository's own solutions
import AITER at module level (solutions/gdn_decode/main.py:32-35,
solutions/gdn_prefill/main.py:21-24), which is not installed here, so they
cannot be run.

Run once where flashinfer is importable:
    python tests/golden/make_golden.py
It writes tests/golden/gdn_golden.npz (bf16 tensors stored as uint16 bits).
The tests only read the .npz; they never import flashinfer.
"""
from __future__ import annotations

import math
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))

from rocm_flashinfer_contest_b200.inputs import decode_inputs, mtp_inputs, prefill_inputs  # noqa: E402

# (name, B, H, HV, K, with_state, scale, seed, gate_override)
DECODE_CASES = [
    ("dec_small", 3, 2, 4, 16, True, 0.0, 1, None),
    ("dec_nostate", 2, 1, 2, 32, False, 0.5, 2, None),
    ("dec_k128", 1, 1, 2, 128, True, 1.0 / math.sqrt(128), 3, None),
    ("dec_gva4_extreme", 2, 1, 4, 16, True, 0.25, 4, "extreme"),
    ("dec_contest_b2", 2, 4, 8, 32, True, 0.0, 5, None),
]
# (name, seqlens, H, HV, K, with_state, scale, seed, cu dtype)
PREFILL_CASES = [
    ("pre_varlen_empty", [5, 0, 17, 1], 2, 4, 16, True, 0.0, 11, torch.int64),
    ("pre_nostate", [70], 1, 2, 32, False, 0.3, 12, torch.int32),
    ("pre_k128", [40, 90], 1, 2, 128, True, 0.0, 13, torch.int32),
    ("pre_gva4_extreme", [9, 3], 1, 4, 16, True, 1.0, 14, torch.int64),
]

# (name, seqlens, H, HV, K, seed): raw (unnormalised) q/k, normalised the way
# AITER's / FLA's use_qk_l2norm_in_kernel does (x / sqrt(sum(x^2) + 1e-6),
# fla/modules/l2norm.py:42) before the template runs; the fixture keeps the
# raw q/k and a qk_l2norm flag
PREFILL_L2_CASES = [
    ("pre_l2norm", [45, 0, 70], 2, 4, 32, 17),
    ("pre_l2norm_k128", [33, 64], 1, 2, 128, 18),
]

# (name, seqlens, checkpoint_every_n_tokens, seed); H = 1, HV = 2, K = V = 16
CKPT_CASES = [
    ("ckpt_every64", [130, 0, 200, 64], 64, 15),
    ("ckpt_every128", [300, 127, 128], 128, 16),
]

# (name, B, T, pool, H, HV, K, scale, seed, intermediate buffer, qk_l2norm, bf16 state)
# qk_l2norm cases feed raw (unnormalised) q/k and normalise them the way
# flashinfer's gated_delta_rule_mtp kernel does (x * rsqrt(sum(x^2) + 1e-6),
# flashinfer/gdn_kernels/gdn_decode_mtp.py:359-360) before the template runs.
# bf16-state cases (flashinfer/gdn_decode.py:206-260) hold the pool in bf16:
# the template runs on the widened pool and its final state is rounded to
# bf16 (nearest even), the state being fp32 in between.
MTP_CASES = [
    ("mtp_small", 3, 4, 5, 2, 4, 16, 0.0, 21, True, False, False),
    ("mtp_k128", 2, 3, 3, 1, 2, 128, 0.0, 22, False, False, False),
    ("mtp_gva4", 2, 2, 4, 1, 4, 32, 0.4, 23, True, False, False),
    ("mtp_l2norm", 2, 3, 3, 1, 2, 32, 0.0, 24, True, True, False),
    ("mtp_bf16state_t1", 3, 1, 4, 1, 2, 128, 0.0, 25, False, False, True),
    ("mtp_bf16state_t3", 2, 3, 5, 2, 4, 32, 0.0, 26, False, False, True),
]


def _extreme_gates(args, a_idx, b_idx):
    """Push a and b into the saturating ranges: softplus threshold (x > 20),
    sigmoid near 0 and 1, and a decay g near 1 (very negative a)."""
    a = args[a_idx].float()
    b = args[b_idx].float()
    flat_a = a.view(-1)
    flat_b = b.view(-1)
    pattern_a = torch.tensor([25.0, -30.0, 19.5, 0.0, -5.0, 40.0])
    pattern_b = torch.tensor([30.0, -30.0, 8.0, -8.0, 0.0, 1.0])
    for i in range(flat_a.numel()):
        flat_a[i] = pattern_a[i % len(pattern_a)]
        flat_b[i] = pattern_b[i % len(pattern_b)]
    args[a_idx] = a.to(torch.bfloat16)
    args[b_idx] = b.to(torch.bfloat16)


def _np(t):
    if t is None:
        return None
    if t.dtype == torch.bfloat16:
        return t.contiguous().view(torch.int16).numpy().view(np.uint16)
    return t.contiguous().numpy()


def main():
    from flashinfer.trace.templates.gdn import _gdn_decode_reference, _gdn_prefill_reference

    out = {}
    for name, B, H, HV, K, with_state, scale, seed, gate in DECODE_CASES:
        args = decode_inputs(B, H, HV, K, K, seed=seed, with_state=with_state)
        args[8] = scale
        if gate == "extreme":
            _extreme_gates(args, 5, 7)
        o, s = _gdn_decode_reference(*args)
        keys = ["q", "k", "v", "state", "A_log", "a", "dt_bias", "b"]
        for kname, t in zip(keys, args[:8]):
            if t is not None:
                out[f"{name}/{kname}"] = _np(t)
        out[f"{name}/scale"] = np.float32(scale)
        out[f"{name}/out"] = _np(o)
        out[f"{name}/new_state"] = _np(s)
    for name, lens, H, HV, K, with_state, scale, seed, cu_dtype in PREFILL_CASES:
        args = prefill_inputs(lens, H, HV, K, K, seed=seed, with_state=with_state, cu_dtype=cu_dtype)
        args[9] = scale
        if name.endswith("extreme"):
            _extreme_gates(args, 5, 7)
        o, s = _gdn_prefill_reference(*args)
        keys = ["q", "k", "v", "state", "A_log", "a", "dt_bias", "b", "cu_seqlens"]
        for kname, t in zip(keys, args[:9]):
            if t is not None:
                out[f"{name}/{kname}"] = _np(t)
        out[f"{name}/scale"] = np.float32(scale)
        out[f"{name}/out"] = _np(o)
        out[f"{name}/new_state"] = _np(s)
    for name, lens, H, HV, K, seed in PREFILL_L2_CASES:
        args = prefill_inputs(lens, H, HV, K, K, seed=seed, with_state=True, cu_dtype=torch.int64)
        args[9] = 0.0
        run_args = list(args[:10])
        g = torch.Generator().manual_seed(seed + 100)
        for i in (0, 1):
            raw = (torch.randn(args[i].shape, generator=g) * 3.0).to(torch.bfloat16)
            args[i] = raw
            xf = raw.float()
            run_args[i] = xf / torch.sqrt((xf * xf).sum(-1, keepdim=True) + 1e-6)
        o, s = _gdn_prefill_reference(*run_args)
        keys = ["q", "k", "v", "state", "A_log", "a", "dt_bias", "b", "cu_seqlens"]
        for kname, t in zip(keys, args[:9]):
            out[f"{name}/{kname}"] = _np(t)
        out[f"{name}/qk_l2norm"] = np.int32(1)
        out[f"{name}/scale"] = np.float32(0.0)
        out[f"{name}/out"] = _np(o)
        out[f"{name}/new_state"] = _np(s)
    # state checkpoints (flashinfer's chunk_gated_delta_rule, gdn_prefill.py:161-174):
    # checkpoint i of sequence n is the template's final state over the
    # sequence's first (i + 1) * every tokens
    for name, lens, every, seed in CKPT_CASES:
        args = prefill_inputs(lens, 1, 2, 16, 16, seed=seed, with_state=True, cu_dtype=torch.int64)
        args[9] = 0.0
        keys = ["q", "k", "v", "state", "A_log", "a", "dt_bias", "b", "cu_seqlens"]
        for kname, t in zip(keys, args[:9]):
            out[f"{name}/{kname}"] = _np(t)
        o, s = _gdn_prefill_reference(*args)
        out[f"{name}/scale"] = np.float32(0.0)
        out[f"{name}/out"] = _np(o)
        out[f"{name}/new_state"] = _np(s)
        cu = args[8].tolist()
        ck, starts = [], [0]
        for n in range(len(lens)):
            t0 = cu[n]
            for i in range(lens[n] // every):
                t1 = t0 + (i + 1) * every
                sub = [args[0][t0:t1], args[1][t0:t1], args[2][t0:t1], args[3][n:n + 1], args[4],
                       args[5][t0:t1], args[6], args[7][t0:t1],
                       torch.tensor([0, t1 - t0], dtype=torch.int64), 0.0]
                ck.append(_gdn_prefill_reference(*sub)[1][0])
            starts.append(len(ck))
        out[f"{name}/checkpoints"] = _np(torch.stack(ck))
        out[f"{name}/checkpoint_cu_starts"] = np.array(starts, dtype=np.int64)
        out[f"{name}/every"] = np.int32(every)
    from flashinfer.trace.templates.gdn import _gdn_mtp_reference
    for name, B, T, pool, H, HV, K, scale, seed, inter, l2, bf16_state in MTP_CASES:
        args = mtp_inputs(B, T, pool, H, HV, K, K, seed=seed, intermediate=inter)
        args[9] = scale
        if bf16_state:
            args[3] = args[3].to(torch.bfloat16)
        run_args = list(args[:10])
        if bf16_state:
            run_args[3] = args[3].float()
        if l2:
            g = torch.Generator().manual_seed(seed + 100)
            for i in (0, 1):
                raw = (torch.randn(args[i].shape, generator=g) * 3.0).to(torch.bfloat16)
                args[i] = raw
                xf = raw.float()
                run_args[i] = xf * torch.rsqrt((xf * xf).sum(-1, keepdim=True) + 1e-6)
        keys = ["q", "k", "v", "initial_state", "initial_state_indices", "A_log", "a", "dt_bias", "b"]
        for kname, t in zip(keys, args[:9]):
            out[f"{name}/{kname}"] = _np(t)
        out[f"{name}/qk_l2norm"] = np.int32(l2)
        buf = args[10]
        o, s = _gdn_mtp_reference(*run_args, intermediate_states_buffer=buf)
        out[f"{name}/scale"] = np.float32(scale)
        out[f"{name}/out"] = _np(o)
        out[f"{name}/new_state"] = _np(s.to(torch.bfloat16) if bf16_state else s)
        if buf is not None:
            out[f"{name}/intermediate"] = _np(buf)
    path = os.path.join(HERE, "gdn_golden.npz")
    np.savez_compressed(path, **out)
    print(f"wrote {path}: {len(out)} arrays, {os.path.getsize(path)} bytes")


if __name__ == "__main__":
    main()

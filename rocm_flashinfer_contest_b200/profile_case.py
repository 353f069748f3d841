"""Runs one GDN workload a few times so a profiler can wrap it.

The B200 counterpart of the reference's tools/profile_kernel.py:30-94 (which
drives one solution's run() on one workload under rocprofv3): inputs are
built once, outside the profiled loop, then the kernel is launched
``--warmup`` + ``--iters`` times.  Use with ncu, e.g.

    ncu --set full --clock-control none -k regex:gdn_decode -s 2 -c 1 \\
        python -m rocm_flashinfer_contest_b200.profile_case decode --B 64
"""
from __future__ import annotations

import argparse

import torch

from . import gdn_decode, gdn_mtp, gdn_prefill, inputs


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("op", choices=["decode", "prefill", "mtp"])
    ap.add_argument("--B", type=int, default=64)
    ap.add_argument("--T", type=int, default=8192)
    ap.add_argument("--seqs", type=int, default=1)
    ap.add_argument("--H", type=int, default=16)
    ap.add_argument("--HV", type=int, default=32)
    ap.add_argument("--warmup", type=int, default=2)
    ap.add_argument("--iters", type=int, default=1)
    ap.add_argument("--no-state", action="store_true")
    ap.add_argument("--steps", type=int, default=4, help="mtp: tokens per batch entry")
    ap.add_argument("--no-snapshots", action="store_true", help="mtp: no intermediate states")
    ap.add_argument("--bf16-state", action="store_true", help="mtp: bf16 state pool (no snapshots)")
    a = ap.parse_args(argv)
    dev = torch.device("cuda:0")
    if a.op == "decode":
        args = inputs.decode_inputs(a.B, a.H, a.HV, seed=0, device=dev, with_state=not a.no_state)
        out = torch.empty((a.B, 1, a.HV, 128), dtype=torch.bfloat16, device=dev)
        ns = args[3] if args[3] is not None else torch.empty((a.B, a.HV, 128, 128), device=dev)
        fn = lambda: gdn_decode.run_into(*args, output=out, new_state=ns)  # noqa: E731
    elif a.op == "mtp":
        args = inputs.mtp_inputs(a.B, a.steps, 2 * a.B, a.H, a.HV, seed=0, device=dev,
                                 intermediate=not (a.no_snapshots or a.bf16_state))
        if a.bf16_state:
            args[3] = args[3].to(torch.bfloat16)
        out = torch.empty((a.B, a.steps, a.HV, 128), dtype=torch.bfloat16, device=dev)
        fn = lambda: gdn_mtp.run_into(*args[:10], out, args[3],  # noqa: E731
                                      intermediate_states_buffer=args[10])
    else:
        lens = [a.T // a.seqs] * a.seqs
        lens[-1] += a.T - sum(lens)
        args = inputs.prefill_inputs(lens, a.H, a.HV, seed=0, device=dev, with_state=not a.no_state)
        out = torch.empty((a.T, a.HV, 128), dtype=torch.bfloat16, device=dev)
        ns = torch.empty((a.seqs, a.HV, 128, 128), device=dev)
        fn = lambda: gdn_prefill.run_into(*args, output=out, new_state=ns)  # noqa: E731
    torch.cuda.synchronize()
    for _ in range(a.warmup + a.iters):
        fn()
    torch.cuda.synchronize()
    print(f"profile_case {a.op}: {a.warmup} + {a.iters} launches done")


if __name__ == "__main__":
    main()

"""Benchmark of the B200 GDN kernels; prints ONE JSON line (rank 0).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Headline metric: GDN decode at B = 64 (H = 16, HV = 32,
K = V = 128, state read and written in place), reported as state GB/s with
us/step beside it; the prefill tokens/s at one 8192-token sequence (zero
initial state) and the pool-indexed multi-token decode (B = 64, T = 4 draft
tokens, per-token state snapshots, in-place pool) ride along in the same line
under "prefill" and "mtp".

* ``value``: whole-job state GB/s, device-timed with CUDA events around each
  step's kernel, inputs resident in HBM, L2 flushed (a 256 MiB write) before
  every timed step.  Multi-GPU: one process per GPU (torchrun), each rank runs
  its own B = 64 shard of a 64*N batch (weak scaling, no data-path
  collective); the time is the max over ranks.
* ``e2e``: the same metric through the public ``gdn_decode.run`` with every
  input copied from pinned host memory and both outputs copied back inside
  the timed region.
* ``roofline``: the decode kernel's algorithmic bytes per launch over its
  event-timed duration, against the measured HBM copy bandwidth.
* ``cpu_baseline``: the C oracle (oracle/gdn_oracle.c, all host cores) on the
  same workload, rank 0 at N = 1 only.
* ``--impl reference``: the reference's algorithm on the host cores (the C
  oracle port; the reference's own solutions are Triton/AITER code for
  MI300X and cannot run here), same metric and config.
"""
from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import time

import torch

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

D = 128
H, HV = 16, 32
DECODE_B = 64
DECODE_B_STRONG = 1024  # config 4: one B = 1024 batch split across the ranks
PREFILL_T = 8192
FLUSH_BYTES = 256 << 20

METRIC = "gdn_decode state GB/s at B=64 (H=16, HV=32, d=128)"
UNIT = "GB/s"


def decode_state_bytes(B):
    return 2 * B * HV * D * D * 4


def decode_alg_bytes(B):
    """Algorithmic HBM bytes of one decode launch: state in + out (fp32),
    q and k (bf16), v in and o out (bf16), a and b (bf16), A_log and dt_bias."""
    return (decode_state_bytes(B) + 2 * B * H * D * 2 + 2 * B * HV * D * 2 + 2 * B * HV * 2
            + 2 * HV * 4)


MTP_B, MTP_T = 64, 4


def mtp_alg_bytes(B, T, snapshots=True):
    """Algorithmic HBM bytes of one MTP launch (fp32 pool): each pool row read
    once and written once, with snapshots one more write per token, plus q, k
    (bf16), v in and o out (bf16), a and b (bf16) for every token."""
    head = D * D * 4
    return (B * HV * head * (2 + (T if snapshots else 0))
            + T * (2 * B * H * D * 2 + 2 * B * HV * D * 2 + 2 * B * HV * 2) + B * 4 + 2 * HV * 4)


def prefill_alg_flops(T):
    """Chunk-form algorithmic FLOPs (C = 64, d = 128): per chunk-head
    5 * 2C^2d + 3 * 2Cd^2 = 11,534,336, i.e. 180,224 per token-head."""
    return T * HV * 180224


def load_peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            d = json.load(f)
        return {"hbm_gbs": d["hbm_gbs"], "bf16_tflops": d["bf16_tflops"], "src": "measured"}
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "src": "fallback"}


def profile_traffic(name):
    """DRAM bytes per launch from a committed ncu summary (a line
    'traffic_bytes_per_launch: N'), or None when no capture exists yet."""
    p = os.path.join(ROOT, "profiles", name)
    if not os.path.exists(p):
        return None
    with open(p) as f:
        for line in f:
            if line.startswith("traffic_bytes_per_launch:"):
                return int(float(line.split(":", 1)[1].strip()))
    return None


# ---------------------------------------------------------------------------
# distributed plumbing (barrier and max-over-ranks of timings only)

def dist_setup():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import datetime
        import torch.distributed as dist
        backend = "nccl" if torch.cuda.is_available() else "gloo"
        if backend == "nccl":
            torch.cuda.set_device(local)
        dist.init_process_group(backend, timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local) if backend == "nccl" else None)
    return rank, world, local


def barrier(world):
    if world > 1:
        import torch.distributed as dist
        dist.barrier()


def max_over_ranks(x: float, world: int, device) -> float:
    if world == 1:
        return x
    import torch.distributed as dist
    t = torch.tensor([x], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


# ---------------------------------------------------------------------------
# clocks: nvidia-smi sampler around the measured window

class ClockSampler:
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device: torch.device):
        try:  # address the GPU by UUID: indices differ under CUDA_VISIBLE_DEVICES
            self.gpu = "GPU-" + str(torch.cuda.get_device_properties(device).uuid)
        except Exception:
            self.gpu = str(device.index or 0)
        self.proc = None
        self.path = os.path.join("/tmp", f"gdn_clocks_{os.getpid()}.csv")

    def __enter__(self):
        try:
            self.fh = open(self.path, "w")
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "50"],
                stdout=self.fh, stderr=subprocess.DEVNULL)
        except (OSError, FileNotFoundError):
            self.proc = None
        return self

    def __exit__(self, *exc):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
            self.fh.close()

    def summary(self):
        if self.proc is None or not os.path.exists(self.path):
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        sm, smax, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        with open(self.path) as f:
            for line in f:
                parts = [p.strip() for p in line.split(",")]
                if len(parts) < 9:
                    continue
                try:
                    sm.append(float(parts[1]))
                    smax.append(float(parts[2]))
                except ValueError:
                    continue
                for n, v in zip(names, parts[5:9]):
                    if v.lower() == "active":
                        reasons.add(n)
        os.unlink(self.path)
        return {"sm_mhz": statistics.median(sm) if sm else None,
                "sm_max_mhz": max(smax) if smax else None,
                "reasons": sorted(reasons), "samples": len(sm),
                "window": "warm-up soak + timed steps"}


# ---------------------------------------------------------------------------
# our arm

def timed_steps(fn, steps, flush, stream, clean=None):
    """Run `steps` steps; before each, flush L2 (outside the events).  Returns
    per-step device milliseconds from CUDA events recorded on `stream`.
    With `clean` (a second buffer larger than L2) the write flush is followed
    by a read of it, which writes the flush's dirty lines back before the
    timed region and leaves L2 holding clean, unrelated data."""
    evs = []
    torch.cuda.nvtx.range_push("timed")  # ncu --nvtx-include timed/ selects these launches
    with torch.cuda.stream(stream):
        for _ in range(steps):
            flush.add_(1)  # 256 MiB read-modify-write evicts L2 (126 MB)
            if clean is not None:
                clean.sum()
            s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            s.record(stream)
            fn()
            e.record(stream)
            evs.append((s, e))
    torch.cuda.nvtx.range_pop()
    torch.cuda.synchronize()
    return [s.elapsed_time(e) for s, e in evs]


def _stats(ms):
    """This rank's per-step device times: mean, median, min and max (ms)."""
    return {"mean": round(statistics.mean(ms), 5), "median": round(statistics.median(ms), 5),
            "min": round(min(ms), 5), "max": round(max(ms), 5), "n": len(ms)}


# ---------------------------------------------------------------------------
# GPU bars: the best library kernels for the same work, on the same GPU, timed
# in alternation with ours (flush, ours, flush, bar, ...), as the reference
# pairs candidate and baseline runs (tools/run_benchmarks.py:293-305,334-347).

def _paired(fns, steps, flush, stream):
    """Per-step device ms of each function in `fns`, the functions alternating
    within every step, each launch preceded by the L2 flush."""
    evs = [[] for _ in fns]
    with torch.cuda.stream(stream):
        for _ in range(steps):
            for i, fn in enumerate(fns):
                flush.add_(1)
                s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                s.record(stream)
                fn()
                e.record(stream)
                evs[i].append((s, e))
    torch.cuda.synchronize()
    return [[s.elapsed_time(e) for s, e in ev] for ev in evs]


def _bar_entry(name, ours_ms, bar_ms, **extra):
    o, b = statistics.median(ours_ms), statistics.median(bar_ms)
    return {"bar": name, "bar_us": round(b * 1e3, 2), "ours_us": round(o * 1e3, 2),
            "speedup": round(b / o, 3), "steps": len(ours_ms),
            "timing": "paired: flush, ours, flush, bar per step; medians of CUDA-event times", **extra}


def _why(e):
    return f"{type(e).__name__}: {str(e).splitlines()[0] if str(e) else ''}"[:240]


def bar_decode(dev, flush, stream, steps):
    """flashinfer's CuTe-DSL decode (gated_delta_rule_decode_pretranspose,
    fp32 k-last state, in place) against gdn_decode at B = 64."""
    try:
        from flashinfer.gdn_decode import gated_delta_rule_decode_pretranspose as fi_decode
    except Exception as e:  # noqa: BLE001 - any import failure makes the bar unavailable
        return {"unavailable": "flashinfer decode import failed: " + _why(e)}
    from rocm_flashinfer_contest_b200 import gdn_decode, inputs
    q, k, v, state, A_log, a, dt_bias, b, scale = inputs.decode_inputs(DECODE_B, H, HV, seed=7000,
                                                                        device=dev)
    s_ours, s_bar = state.clone(), state.clone()
    o_ours = torch.empty((DECODE_B, 1, HV, D), dtype=torch.bfloat16, device=dev)
    o_bar = torch.empty_like(o_ours)

    def ours():
        gdn_decode.run_into(q, k, v, s_ours, A_log, a, dt_bias, b, scale, output=o_ours, new_state=s_ours)

    def bar():
        fi_decode(q, k, v, s_bar, A_log, a, dt_bias, b, scale=scale, output=o_bar, use_qk_l2norm=False)

    try:
        ours()
        bar()  # first call compiles the CuTe DSL kernel
        torch.cuda.synchronize()
        diff = {"max_abs_diff_output": float((o_ours.float() - o_bar.float()).abs().max()),
                "max_abs_diff_state": float((s_ours - s_bar).abs().max())}
        for _ in range(3):
            ours()
            bar()
        torch.cuda.synchronize()
        t_ours, t_bar = _paired([ours, bar], steps, flush, stream)
    except Exception as e:  # noqa: BLE001
        return {"unavailable": "flashinfer decode failed on this GPU: " + _why(e)}
    return _bar_entry("flashinfer 0.6.11 gated_delta_rule_decode_pretranspose (CuTe DSL, fp32 state, "
                      "use_qk_l2norm=False), B=64", t_ours, t_bar, first_step=diff)


def bar_mtp(dev, flush, stream, steps):
    """flashinfer's CuTe-DSL gated_delta_rule_mtp (B = 64, T = 4, fp32 pool of
    128 slots updated in place, per-token snapshots by batch entry) against
    this library's mirror of the same call."""
    try:
        from flashinfer.gdn_decode import gated_delta_rule_mtp as fi_mtp
    except Exception as e:  # noqa: BLE001
        return {"unavailable": "flashinfer MTP import failed: " + _why(e)}
    from rocm_flashinfer_contest_b200 import gdn_mtp, inputs
    q, k, v, pool, idx, A_log, a, dt_bias, b, scale, _ = inputs.mtp_inputs(
        MTP_B, MTP_T, 2 * MTP_B, H, HV, seed=7100, device=dev)
    p_ours, p_bar = pool.clone(), pool.clone()
    snap_ours = torch.zeros((MTP_B, MTP_T, HV, D, D), device=dev)
    snap_bar = torch.zeros_like(snap_ours)
    o_ours = torch.empty((MTP_B, MTP_T, HV, D), dtype=torch.bfloat16, device=dev)
    o_bar = torch.empty_like(o_ours)

    def ours():
        gdn_mtp.gated_delta_rule_mtp(q, k, v, p_ours, idx, A_log, a, dt_bias, b, scale, output=o_ours,
                                     intermediate_states_buffer=snap_ours, disable_state_update=False,
                                     use_qk_l2norm=False)

    def bar():
        fi_mtp(q, k, v, p_bar, idx, A_log, a, dt_bias, b, scale=scale, output=o_bar,
               intermediate_states_buffer=snap_bar, disable_state_update=False, use_qk_l2norm=False)

    try:
        ours()
        bar()
        torch.cuda.synchronize()
        diff = {"max_abs_diff_output": float((o_ours.float() - o_bar.float()).abs().max()),
                "max_abs_diff_snapshots": float((snap_ours - snap_bar).abs().max())}
        for _ in range(3):
            ours()
            bar()
        torch.cuda.synchronize()
        t_ours, t_bar = _paired([ours, bar], steps, flush, stream)
    except Exception as e:  # noqa: BLE001
        return {"unavailable": "flashinfer MTP failed on this GPU: " + _why(e)}
    return _bar_entry("flashinfer 0.6.11 gated_delta_rule_mtp (CuTe DSL, fp32 pool, snapshots by entry), "
                      f"B={MTP_B}, T={MTP_T}", t_ours, t_bar, first_step=diff)


def bar_prefill(dev, flush, stream, steps):
    """Chunked GDN prefill libraries at T = 8192 (one sequence, zero state,
    final state returned): FLA's Triton chunk_gated_delta_rule and flashinfer's
    Blackwell CuTe-DSL kernel, each against gdn_prefill.  Their gates (log
    decay and beta, fp32 per token and v-head) are computed before the timed
    region, which gdn_prefill computes inside its kernels."""
    from rocm_flashinfer_contest_b200 import gdn_prefill, inputs
    q, k, v, _, A_log, a, dt_bias, b, cu, scale = inputs.prefill_inputs([PREFILL_T], H, HV, seed=7200,
                                                                        device=dev, with_state=False)
    x = a.float() + dt_bias
    log_g = -torch.exp(A_log) * torch.where(x > 20.0, x, torch.log1p(torch.exp(x)))
    beta = torch.sigmoid(b.float())
    o_ours = torch.empty((PREFILL_T, HV, D), dtype=torch.bfloat16, device=dev)
    s_ours = torch.empty((1, HV, D, D), device=dev)

    def ours():
        gdn_prefill.run_into(q, k, v, None, A_log, a, dt_bias, b, cu, scale, output=o_ours, new_state=s_ours)

    out = {}
    try:
        from fla.ops.gated_delta_rule import chunk_gated_delta_rule as fla_chunk
        cu64 = cu.to(torch.int64)
        fq, fk, fv = q.unsqueeze(0), k.unsqueeze(0), v.unsqueeze(0)
        fg, fb = log_g.unsqueeze(0), beta.unsqueeze(0)
        res = {}

        def fla():
            res["o"], res["s"] = fla_chunk(fq, fk, fv, fg, fb, scale=scale, initial_state=None,
                                           output_final_state=True, cu_seqlens=cu64,
                                           transpose_state_layout=True)

        ours()
        fla()  # first call compiles / autotunes the Triton kernels
        torch.cuda.synchronize()
        diff = {"max_abs_diff_output": float((o_ours.float() - res["o"][0].float()).abs().max()),
                "max_abs_diff_state": float((s_ours - res["s"].reshape(s_ours.shape)).abs().max())}
        for _ in range(3):
            ours()
            fla()
        torch.cuda.synchronize()
        t_ours, t_bar = _paired([ours, fla], steps, flush, stream)
        out["fla"] = _bar_entry("fla 0.5.1 chunk_gated_delta_rule (Triton), T=8192, gates precomputed",
                                t_ours, t_bar, first_step=diff)
    except Exception as e:  # noqa: BLE001
        out["fla"] = {"unavailable": "fla chunk_gated_delta_rule failed on this GPU: " + _why(e)}
    try:
        from flashinfer.gdn_kernels import _has_blackwell_prefill, chunk_gated_delta_rule_sm100
        if not _has_blackwell_prefill or chunk_gated_delta_rule_sm100 is None:
            raise RuntimeError("flashinfer.gdn_kernels reports no Blackwell prefill kernel")
        o_fi = torch.empty_like(o_ours)
        s_fi = torch.empty_like(s_ours)
        alpha = torch.exp(log_g)
        cu32 = cu.to(torch.int32)

        def fi():
            chunk_gated_delta_rule_sm100(q, k, v, alpha, beta, o_fi, cu32, None, s_fi, scale)

        fi()
        torch.cuda.synchronize()
        diff = {"max_abs_diff_output": float((o_ours.float() - o_fi.float()).abs().max()),
                "max_abs_diff_state": float((s_ours - s_fi).abs().max())}
        for _ in range(3):
            ours()
            fi()
        torch.cuda.synchronize()
        t_ours, t_bar = _paired([ours, fi], steps, flush, stream)
        out["flashinfer"] = _bar_entry("flashinfer 0.6.11 chunk_gated_delta_rule_sm100 (Blackwell CuTe DSL, "
                                       "called directly), T=8192, gates precomputed", t_ours, t_bar,
                                       first_step=diff)
    except Exception as e:  # noqa: BLE001
        out["flashinfer"] = {"unavailable": "flashinfer Blackwell prefill: " + _why(e) +
                             " (its public chunk_gated_delta_rule selects it only for CUDA >= 13; torch here "
                             "is cu128)"}
    return out


def _sample_seqs(seqs, n=2):
    """Up to `n` sequence indices spread over `seqs` (first, last, ...)."""
    if not seqs:
        return []
    if len(seqs) <= n:
        return list(seqs)
    return [seqs[(len(seqs) - 1) * i // (n - 1)] for i in range(n)]


def decode_shard_parity(kargs, shard, dev):
    """One out-of-place decode step of this rank's shard, with the sampled
    sequences checked against the CPU oracle (outside every timed region)."""
    sys.path.insert(0, os.path.join(ROOT, "tests"))
    from oracle import oracle
    from parity import output_report, state_report
    from rocm_flashinfer_contest_b200 import gdn_decode
    o, s = gdn_decode.run(*kargs)
    torch.cuda.synchronize()
    pos = [shard.seqs.index(i) for i in _sample_seqs(list(shard.seqs))]
    sel = torch.tensor(pos, dtype=torch.long, device=dev)
    sub = [x.index_select(0, sel).cpu() if isinstance(x, torch.Tensor) and x.dim() >= 2 else
           (x.cpu() if isinstance(x, torch.Tensor) else x) for x in kargs]
    ro, rs = oracle.decode(*sub)
    ro_ = output_report(o.index_select(0, sel).cpu(), ro)
    rs_ = state_report(s.index_select(0, sel).cpu(), rs)
    return {"checked": len(pos), "bad": ro_["bad"] + rs_["bad"] + ro_["nonfinite"] + rs_["nonfinite"],
            "out_max_abs": ro_["max_abs"], "state_normwise": rs_["normwise"]}


def _gather_floats(vals, world, dev):
    """Every rank's list of floats (same length), in rank order."""
    if world == 1:
        return [list(vals)]
    import torch.distributed as dist
    t = torch.zeros((world, len(vals)), dtype=torch.float64, device=dev)
    t[int(os.environ.get("RANK", "0"))] = torch.tensor(vals, dtype=torch.float64)
    dist.all_reduce(t)
    return t.cpu().tolist()


# contest workloads with published MI300X latencies (H = 4, HV = 8; the
# reference's results/amd_mi300.md:35-40); lengths of the multi-sequence
# prefills are seeded stand-ins with the published totals and counts
CONTEST_H, CONTEST_HV = 4, 8
CONTEST_DECODE = [(1, 0.038), (16, 0.033), (64, 0.030)]
CONTEST_PREFILL = [(6, 1, 0.168), (139, 3, 0.174), (8192, 39, 0.528)]


def contest_workloads(dev, flush, stream, steps):
    """Latency of the contest `run` calls (outputs allocated per call, as the
    harness times them) on the published workloads, median of CUDA-event
    times with L2 flushed before each call."""
    from rocm_flashinfer_contest_b200 import gdn_decode, gdn_prefill, inputs
    rows, launches = [], 0
    for B, mi300 in CONTEST_DECODE:
        args = inputs.decode_inputs(B, CONTEST_H, CONTEST_HV, seed=8000 + B, device=dev)
        fn = lambda args=args: gdn_decode.run(*args)  # noqa: E731
        for _ in range(3):
            fn()
        ms = timed_steps(fn, steps, flush, stream)
        launches += steps
        rows.append({"kernel": "gdn_decode", "workload": {"batch_size": B},
                     "ms": round(statistics.median(ms), 5), "ms_min": round(min(ms), 5),
                     "mi300x_ms": mi300, "speedup_vs_mi300x": round(mi300 / statistics.median(ms), 2)})
    for T, N, mi300 in CONTEST_PREFILL:
        lens = inputs.seqlens_split(T, N, seed=8100 + T)
        args = inputs.prefill_inputs(lens, CONTEST_H, CONTEST_HV, seed=8200 + T, device=dev)
        fn = lambda args=args: gdn_prefill.run(*args)  # noqa: E731
        for _ in range(3):
            fn()
        ms = timed_steps(fn, steps, flush, stream)
        launches += steps * (2 if T >= 128 else 1)  # chunked: prep + chain; token-serial: one kernel
        rows.append({"kernel": "gdn_prefill", "workload": {"total_seq_len": T, "num_seqs": N},
                     "ms": round(statistics.median(ms), 5), "ms_min": round(min(ms), 5),
                     "mi300x_ms": mi300, "speedup_vs_mi300x": round(mi300 / statistics.median(ms), 2)})
    return {"rows": rows, "H": CONTEST_H, "HV": CONTEST_HV,
            "note": "contest definitions gdn_*_qk4_v8_d128_k_last; MI300X figures from the reference's "
                    "results/amd_mi300.md:35-40 (other hardware, context only)"}, launches


def bench_ours(args, rank, world, local):
    from rocm_flashinfer_contest_b200 import gdn_decode, gdn_mtp, gdn_prefill, inputs, partition

    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    stream = torch.cuda.current_stream(dev)
    peaks = load_peaks()
    flush = torch.zeros(FLUSH_BYTES // 4, dtype=torch.float32, device=dev)

    # ---- decode: this rank's shard of a 64*N batch (weak scaling) ----
    Bglob = DECODE_B * world
    shard = partition.plan_decode(Bglob, H, HV, world)[rank]
    Bloc = len(shard.seqs)
    dargs = inputs.decode_inputs(Bloc, H, HV, seed=1000 + rank, device=dev)
    out = torch.empty((Bloc, 1, HV, D), dtype=torch.bfloat16, device=dev)
    state = dargs[3]

    def dec_step():
        gdn_decode.run_into(*dargs[:3], state, *dargs[4:], output=out, new_state=state)

    for _ in range(max(3, args.warmup)):
        dec_step()
    torch.cuda.synchronize()

    # ---- config 4 inputs: this rank's shard of ONE B = 1024 batch (strong
    # scaling), sequence i drawn from its own generator so the shard equals the
    # same rows of the whole batch; sampled rows checked against the oracle ----
    s1k = partition.plan_decode(DECODE_B_STRONG, H, HV, world)[rank]
    kargs = inputs.decode_inputs_for(s1k.seqs, H, HV, seed=5000, device=dev)
    parity = decode_shard_parity(kargs, s1k, dev)
    b1k = len(s1k.seqs)
    kout = torch.empty((b1k, 1, HV, D), dtype=torch.bfloat16, device=dev)

    # ---- config 3: 16 varlen sequences with initial states, split by
    # token-balanced bins across the ranks (plan_prefill) ----
    c3_lens = inputs.seqlens_uniform(16, 1, 1024, seed=0, max_total=8192)
    c3_shard = partition.plan_prefill(c3_lens, H, HV, world)[rank]
    c3_args = inputs.to_device(partition.apply_prefill(
        inputs.prefill_inputs(c3_lens, H, HV, seed=2500), c3_shard), dev)
    c3_tokens = sum(c3_lens[i] for i in c3_shard.seqs)
    c3_out = torch.empty((max(c3_tokens, 1), HV, D), dtype=torch.bfloat16, device=dev)[:c3_tokens]
    c3_state = torch.empty((len(c3_shard.seqs), HV, D, D), dtype=torch.float32, device=dev)

    with ClockSampler(dev) as clk:
        # soak so the clock sampler sees the GPU under this load
        t_end = time.time() + 1.5
        while time.time() < t_end:
            for _ in range(50):
                dec_step()
            torch.cuda.synchronize()
        barrier(world)
        torch.cuda.synchronize()
        dec_ms = timed_steps(dec_step, args.steps, flush, stream)
        # the same launches after a clean L2 (write flush, then a read of a second buffer)
        clean = torch.zeros(FLUSH_BYTES // 4, dtype=torch.float32, device=dev)
        dec_clean_ms = timed_steps(dec_step, args.steps, flush, stream, clean=clean)
        del clean
        torch.cuda.synchronize()
        barrier(world)

        # ---- decode: this rank's shard of one B = 1024 batch (strong scaling) ----
        def b1k_step():
            gdn_decode.run_into(*kargs[:3], kargs[3], *kargs[4:], output=kout, new_state=kargs[3])

        for _ in range(3):
            b1k_step()
        torch.cuda.synchronize()
        barrier(world)
        b1k_ms = timed_steps(b1k_step, args.steps, flush, stream)
        del kargs, kout
        torch.cuda.synchronize()
        barrier(world)

        # ---- prefill: one 8192-token sequence per rank, zero initial state ----
        pargs = inputs.prefill_inputs([PREFILL_T], H, HV, seed=2000 + rank, device=dev,
                                      with_state=False)
        pout = torch.empty((PREFILL_T, HV, D), dtype=torch.bfloat16, device=dev)
        pstate = torch.empty((1, HV, D, D), dtype=torch.float32, device=dev)

        def pre_step():
            gdn_prefill.run_into(*pargs, output=pout, new_state=pstate)

        for _ in range(max(3, args.warmup)):
            pre_step()
        torch.cuda.synchronize()
        barrier(world)
        pre_ms = timed_steps(pre_step, args.steps, flush, stream)
        barrier(world)

        # ---- prefill config 3: this rank's bin of the 16 varlen sequences ----
        def c3_step():
            if c3_shard.seqs:
                gdn_prefill.run_into(*c3_args, output=c3_out, new_state=c3_state)

        for _ in range(3):
            c3_step()
        torch.cuda.synchronize()
        barrier(world)
        c3_ms = timed_steps(c3_step, args.steps, flush, stream)
        barrier(world)

        # ---- mtp: B = 64 entries x 4 tokens over a 128-slot pool, in place ----
        margs = inputs.mtp_inputs(MTP_B, MTP_T, 2 * MTP_B, H, HV, seed=3000 + rank, device=dev,
                                  intermediate=True)
        mout = torch.empty((MTP_B, MTP_T, HV, D), dtype=torch.bfloat16, device=dev)
        mpool = margs[3]

        def mtp_step():
            gdn_mtp.run_into(*margs[:10], mout, mpool, intermediate_states_buffer=margs[10])

        for _ in range(max(3, args.warmup)):
            mtp_step()
        torch.cuda.synchronize()
        barrier(world)
        mtp_ms = timed_steps(mtp_step, args.steps, flush, stream)
        barrier(world)
        # the same batch without snapshots (serving without rollback, or
        # flashinfer's disable_state_update=False without a cache): no longer
        # HBM-bound at T = 4 by the snapshot writes
        def mtp_ns_step():
            gdn_mtp.run_into(*margs[:10], mout, mpool)

        for _ in range(max(3, args.warmup)):
            mtp_ns_step()
        torch.cuda.synchronize()
        barrier(world)
        mtp_ns_ms = timed_steps(mtp_ns_step, args.steps, flush, stream)
        barrier(world)

        # ---- bf16-state decode: B = 64, state pool in bf16, in place ----
        bargs = inputs.mtp_inputs(DECODE_B, 1, DECODE_B, H, HV, seed=4000 + rank, device=dev,
                                  indices=list(range(DECODE_B)))
        bpool = bargs[3].to(torch.bfloat16)
        bout = torch.empty((DECODE_B, 1, HV, D), dtype=torch.bfloat16, device=dev)

        def bf16_step():
            gdn_mtp.run_into(*bargs[:3], bpool, *bargs[4:10], bout, bpool)

        for _ in range(max(3, args.warmup)):
            bf16_step()
        torch.cuda.synchronize()
        barrier(world)
        bf16_ms = timed_steps(bf16_step, args.steps, flush, stream)
        barrier(world)
        # the same launches after a clean L2 (as for the headline decode): at
        # 128 MB per step the flush's dirty lines, written back inside the
        # timed kernel, are a large share of the plain-flush time
        clean = torch.zeros(FLUSH_BYTES // 4, dtype=torch.float32, device=dev)
        bf16_clean_ms = timed_steps(bf16_step, args.steps, flush, stream, clean=clean)
        del clean
        torch.cuda.synchronize()
        barrier(world)
    clocks = clk.summary()
    mtp_step_ms = max_over_ranks(statistics.mean(mtp_ms), world, dev)
    mtp_ns_step_ms = max_over_ranks(statistics.mean(mtp_ns_ms), world, dev)
    bf16_step_ms = max_over_ranks(statistics.mean(bf16_ms), world, dev)

    dec_step_ms = max_over_ranks(statistics.mean(dec_ms), world, dev)
    b1k_step_ms = max_over_ranks(statistics.mean(b1k_ms), world, dev)
    pre_step_ms = max_over_ranks(statistics.mean(pre_ms), world, dev)
    c3_per_rank = _gather_floats([statistics.mean(c3_ms), float(c3_tokens)], world, dev)
    par_all = _gather_floats([parity["checked"], parity["bad"], parity["out_max_abs"],
                              parity["state_normwise"]], world, dev)

    # ---- e2e through the public run() with host buffers ----
    host_in = [x.cpu().pin_memory() if isinstance(x, torch.Tensor) else x for x in dargs]
    h2d = sum(x.numel() * x.element_size() for x in host_in if isinstance(x, torch.Tensor))
    host_o = torch.empty((Bloc, 1, HV, D), dtype=torch.bfloat16).pin_memory()
    host_s = torch.empty((Bloc, HV, D, D), dtype=torch.float32).pin_memory()
    d2h = host_o.numel() * 2 + host_s.numel() * 4

    # gdn_decode_fwd_host's default slicing: ~16 MiB of state per slice, <= 16
    host_slices = min(16, max(1, host_s.numel() * 4 // (16 << 20)), Bloc)

    def e2e_step():
        # the host-buffer entry point (gdn_decode_fwd_host): batch slices
        # copied up and back concurrently
        gdn_decode.run_host_into(*host_in, host_o, host_s, device=dev)

    for _ in range(3):
        e2e_step()
    torch.cuda.synchronize()
    barrier(world)
    e2e_steps = max(3, min(args.steps, 20))
    pe2e_steps = max(3, min(args.steps, 10))
    e2e_ms = timed_steps(e2e_step, e2e_steps, flush, stream)
    e2e_step_ms = max_over_ranks(statistics.mean(e2e_ms), world, dev)

    # prefill e2e
    phost = [x.cpu().pin_memory() if isinstance(x, torch.Tensor) else x for x in pargs[:3]] + \
        [None] + [x.cpu().pin_memory() for x in pargs[4:9]] + [pargs[9]]
    p_h2d = sum(x.numel() * x.element_size() for x in phost if isinstance(x, torch.Tensor))
    p_ho = torch.empty((PREFILL_T, HV, D), dtype=torch.bfloat16).pin_memory()
    p_hs = torch.empty((1, HV, D, D), dtype=torch.float32).pin_memory()
    p_d2h = p_ho.numel() * 2 + p_hs.numel() * 4

    # gdn_prefill_fwd_host's launches per call: the int32 cu_seqlens widened
    # once, then a cu kernel, the prep and the chain per segment (segments of
    # 2048 tokens, the last 2048 halved down to 256: the library's
    # segment_starts schedule)
    n_seg, s0 = 0, 0
    while PREFILL_T - s0 > 2048:
        n_seg, s0 = n_seg + 1, s0 + 2048
    while PREFILL_T - s0 > 256:
        n_seg, s0 = n_seg + 1, s0 + ((PREFILL_T - s0) // 2 + 63) // 64 * 64
    n_seg += 1 if PREFILL_T > s0 else 0
    host_pre_launches = (0 if phost[8].dtype == torch.int64 else 1) + 3 * n_seg

    def pre_e2e_step():
        # the host-buffer entry point (gdn_prefill_fwd_host): token segments
        # copied up, prefilled and copied back on overlapping streams
        gdn_prefill.run_host_into(*phost, p_ho, p_hs, device=dev)

    for _ in range(2):
        pre_e2e_step()
    torch.cuda.synchronize()
    barrier(world)
    pe2e_ms = timed_steps(pre_e2e_step, pe2e_steps, flush, stream)
    pe2e_step_ms = max_over_ranks(statistics.mean(pe2e_ms), world, dev)

    if rank != 0:
        return None

    # one GPU: the library bars (paired with ours) and the contest workloads
    bars, contest, contest_launches = None, None, 0
    if world == 1 and not args.no_bars:
        bar_steps = max(5, min(args.steps, 20))
        bars = {"decode": bar_decode(dev, flush, stream, bar_steps),
                "mtp": bar_mtp(dev, flush, stream, bar_steps),
                "prefill": bar_prefill(dev, flush, stream, bar_steps)}
        contest, contest_launches = contest_workloads(dev, flush, stream, bar_steps)
        # each paired bar step launches one of our decode / MTP kernels or one prefill (prep + chain)
        for key, per in (("decode", 1), ("mtp", 1)):
            if "steps" in bars[key]:
                contest_launches += per * bars[key]["steps"]
        for sub in bars["prefill"].values():
            if "steps" in sub:
                contest_launches += 2 * sub["steps"]

    state_bytes = decode_state_bytes(DECODE_B) * world
    value = state_bytes / (dec_step_ms * 1e-3) / 1e9
    alg = decode_alg_bytes(DECODE_B)
    achieved = alg / (statistics.mean(dec_ms) * 1e-3) / 1e9
    pre_flops = prefill_alg_flops(PREFILL_T)
    bf16_alg = decode_alg_bytes(DECODE_B) - decode_state_bytes(DECODE_B) // 2 + DECODE_B * 4
    pre_achieved = pre_flops / (statistics.mean(pre_ms) * 1e-3) / 1e12
    # one kernel per decode / MTP call, two per chunked prefill call (prep +
    # chain), one per batch slice of the host-buffer decode, and per
    # host-buffer prefill step a cu_seqlens widening plus (cu, prep, chain)
    # per segment; the paired bars and contest workloads (one GPU) add
    # theirs; counted over every timed region
    launch_regions = {"decode": args.steps, "decode_clean_l2": args.steps,
                      "decode_b1024": args.steps, "prefill": 2 * args.steps,
                      "prefill_config3": 2 * args.steps if c3_shard.seqs else 0,
                      "mtp": args.steps, "mtp_no_snapshots": args.steps,
                      "decode_bf16_state": 2 * args.steps,
                      "decode_e2e": e2e_steps * host_slices,
                      "prefill_e2e": pe2e_steps * host_pre_launches,
                      "bars_and_contest_workloads": contest_launches}
    c3_times = [r[0] for r in c3_per_rank]
    c3_toks = [r[1] for r in c3_per_rank]
    c3_max = max(c3_times)
    line = {
        "metric": METRIC,
        "value": round(value, 2),
        "unit": UNIT,
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": round(dec_step_ms, 5),
        "step_ms_stats": _stats(dec_ms),
        "clean_l2": {"us_per_step": round(statistics.mean(dec_clean_ms) * 1e3, 2),
                     "achieved_gbs": round(alg / (statistics.mean(dec_clean_ms) * 1e-3) / 1e9, 1),
                     "frac": round(alg / (statistics.mean(dec_clean_ms) * 1e-3) / 1e9 / peaks["hbm_gbs"], 4),
                     "note": "same launches, L2 written then read clean before each step: the timed kernel "
                             "no longer writes back the flush's dirty lines"},
        "us_per_step": round(dec_step_ms * 1e3, 2),
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "f32 state / bf16 io",
        "data": "synthetic (seeded; contest dataset not available offline)",
        "config": {"workload": "gdn_decode B=64 per GPU, in-place state (BASELINE configs[1])",
                   "B_per_gpu": DECODE_B, "B_total": DECODE_B * world, "H": H, "HV": HV,
                   "head_size": D, "l2": "flushed (256 MiB write) before every timed step",
                   "parallelism": f"sequence shards x{world}, no collective"},
        "roofline": {"bound": "hbm", "achieved": round(achieved, 1),
                     "peak": peaks["hbm_gbs"], "unit": "GB/s",
                     "frac": round(achieved / peaks["hbm_gbs"], 4),
                     "traffic": profile_traffic("gdn_decode_B64_ncu.txt"),
                     "alg_bytes_per_launch": alg, "peak_src": peaks["src"]},
        "e2e": {"value": round(state_bytes / (e2e_step_ms * 1e-3) / 1e9, 3), "unit": UNIT,
                "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                "path": "gdn_decode.run_host_into -> C-ABI gdn_decode_fwd_host: pinned host inputs -> "
                        "device -> pinned host outputs, batch slices of ~16 MiB of state with the two "
                        "copy directions overlapped"},
        "gpu_launches": sum(launch_regions.values()),
        "gpu_launches_by_region": launch_regions,
        "clocks": clocks,
        "decode_b1024": {
            "metric": f"gdn_decode state GB/s, one B={DECODE_B_STRONG} batch split across the ranks",
            "value": round(decode_state_bytes(DECODE_B_STRONG) / (b1k_step_ms * 1e-3) / 1e9, 1), "unit": UNIT,
            "us_per_step": round(b1k_step_ms * 1e3, 2), "step_ms_stats": _stats(b1k_ms),
            "B_per_gpu": len(partition.plan_decode(DECODE_B_STRONG, H, HV, world)[0].seqs),
            "scaling": "strong",
            "shard_parity": {
                "what": "each rank: one out-of-place step of its shard of the B=1024 batch, sampled "
                        "sequences checked against the CPU oracle (bf16 output atol=rtol=1e-2, state "
                        "1e-3 rel + 1e-3 of max), outside the timed region",
                "ranks": world, "checked_seqs": int(sum(r[0] for r in par_all)),
                "bad_elements": int(sum(r[1] for r in par_all)),
                "pass": all(r[1] == 0 for r in par_all),
                "out_max_abs": max(r[2] for r in par_all),
                "state_normwise_max": max(r[3] for r in par_all)},
        },
        "prefill": {
            "metric": "gdn_prefill tokens/s at T=8192 (1 sequence, zero state)",
            "value": round(PREFILL_T * world / (pre_step_ms * 1e-3), 1), "unit": "tokens/s",
            "ms_per_step": round(pre_step_ms, 4),
            "step_ms_stats": _stats(pre_ms),
            "roofline": {"bound": "tensor", "achieved": round(pre_achieved, 3),
                         "peak": peaks["bf16_tflops"], "unit": "TFLOP/s",
                         "frac": round(pre_achieved / peaks["bf16_tflops"], 5),
                         "traffic": profile_traffic("gdn_prefill_scan_T8192_ncu.txt"),
                         "alg_flops_per_launch": pre_flops, "peak_src": peaks["src"]},
            "e2e": {"value": round(PREFILL_T * world / (pe2e_step_ms * 1e-3), 1), "unit": "tokens/s",
                    "h2d_bytes_per_step": p_h2d, "d2h_bytes_per_step": p_d2h,
                    "path": "gdn_prefill.run_host_into -> C-ABI gdn_prefill_fwd_host: pinned host inputs, "
                            "2048-token segments (the last 2048 tokens as 1024 + 512 + 256 + 256) uploaded / prefilled / downloaded on overlapping streams"},
        },
        "prefill_config3": {
            "metric": "gdn_prefill tokens/s, 16 varlen sequences (BASELINE configs[3]) split across the "
                      "ranks by token-balanced bins (partition.plan_prefill)",
            "value": round(sum(c3_lens) / (c3_max * 1e-3), 1), "unit": "tokens/s",
            "ms_per_step": round(c3_max, 4), "total_tokens": sum(c3_lens),
            "per_rank_ms": [round(t, 4) for t in c3_times],
            "per_rank_tokens": [int(t) for t in c3_toks],
            "balance_tokens": round(sum(c3_toks) / (world * max(c3_toks)), 4) if max(c3_toks) else None,
            "balance_time": round(statistics.mean(c3_times) / c3_max, 4) if c3_max else None,
            "scaling": "strong",
        },
        "mtp": {
            "metric": f"gdn_mtp GB/s at B={MTP_B}, T={MTP_T} (pool 128 slots, snapshots, in place)",
            "value": round(mtp_alg_bytes(MTP_B, MTP_T) * world / (mtp_step_ms * 1e-3) / 1e9, 2),
            "unit": "GB/s", "ms_per_step": round(mtp_step_ms, 5), "step_ms_stats": _stats(mtp_ms),
            "roofline": {"bound": "hbm",
                         "achieved": round(mtp_alg_bytes(MTP_B, MTP_T) / (statistics.mean(mtp_ms) * 1e-3) / 1e9, 1),
                         "peak": peaks["hbm_gbs"], "unit": "GB/s",
                         "frac": round(mtp_alg_bytes(MTP_B, MTP_T) / (statistics.mean(mtp_ms) * 1e-3) / 1e9
                                       / peaks["hbm_gbs"], 4),
                         "traffic": profile_traffic("gdn_mtp_B64_T4_ncu.txt"),
                         "alg_bytes_per_launch": mtp_alg_bytes(MTP_B, MTP_T), "peak_src": peaks["src"]},
        },
        "mtp_no_snapshots": {
            "metric": f"gdn_mtp GB/s at B={MTP_B}, T={MTP_T} (pool 128 slots, no snapshots, in place)",
            "value": round(mtp_alg_bytes(MTP_B, MTP_T, False) * world / (mtp_ns_step_ms * 1e-3) / 1e9, 2),
            "unit": "GB/s", "ms_per_step": round(mtp_ns_step_ms, 5), "step_ms_stats": _stats(mtp_ns_ms),
            "kernel": "gdn_mtp_stream_kernel (persistent, bulk-copy ring)",
            "roofline": {"bound": "hbm",
                         "achieved": round(mtp_alg_bytes(MTP_B, MTP_T, False)
                                           / (statistics.mean(mtp_ns_ms) * 1e-3) / 1e9, 1),
                         "peak": peaks["hbm_gbs"], "unit": "GB/s",
                         "frac": round(mtp_alg_bytes(MTP_B, MTP_T, False) / (statistics.mean(mtp_ns_ms) * 1e-3)
                                       / 1e9 / peaks["hbm_gbs"], 4),
                         "alg_bytes_per_launch": mtp_alg_bytes(MTP_B, MTP_T, False), "peak_src": peaks["src"]},
        },
        "decode_bf16_state": {
            "metric": "gdn decode with a bf16 state pool, B=64 (H=16, HV=32), in place: us/step",
            "value": round(bf16_step_ms * 1e3, 2), "unit": "us/step", "higher_is_better": False,
            "state_gbs": round(decode_state_bytes(DECODE_B) / 2 * world / (bf16_step_ms * 1e-3) / 1e9, 1),
            "roofline": {"bound": "hbm",
                         "achieved": round(bf16_alg / (statistics.mean(bf16_ms) * 1e-3) / 1e9, 1),
                         "peak": peaks["hbm_gbs"], "unit": "GB/s",
                         "frac": round(bf16_alg / (statistics.mean(bf16_ms) * 1e-3) / 1e9 / peaks["hbm_gbs"], 4),
                         "alg_bytes_per_launch": bf16_alg, "peak_src": peaks["src"]},
            "clean_l2": {"us_per_step": round(statistics.mean(bf16_clean_ms) * 1e3, 2),
                         "achieved_gbs": round(bf16_alg / (statistics.mean(bf16_clean_ms) * 1e-3) / 1e9, 1),
                         "frac": round(bf16_alg / (statistics.mean(bf16_clean_ms) * 1e-3) / 1e9 / peaks["hbm_gbs"], 4),
                         "note": "same launches, L2 written then read clean before each step"},
        },
    }
    if bars is not None:
        line["bar"] = bars
        line["contest_workloads"] = contest
    if world == 1 and not args.no_cpu_baseline:
        line["cpu_baseline"] = cpu_baseline(seconds=args.cpu_seconds)
        line["prefill"]["cpu_baseline"] = cpu_prefill_baseline()
        line["cpu_baseline_template"] = cpu_template_baseline()
    return line


# ---------------------------------------------------------------------------
# CPU: the reference algorithm on the host cores (C oracle port)

def _cpu_decode_rate(seconds, steps=None, warmup=0, B=DECODE_B):
    from oracle import oracle
    from rocm_flashinfer_contest_b200 import inputs
    args = inputs.decode_inputs(B, H, HV, seed=1000)
    cores = os.cpu_count() or 1
    for _ in range(warmup):
        oracle.decode(*args, threads=cores)
    times = []
    t_stop = time.perf_counter() + seconds
    while True:
        t0 = time.perf_counter()
        oracle.decode(*args, threads=cores)
        times.append(time.perf_counter() - t0)
        if steps is not None and len(times) >= steps:
            break
        if steps is None and time.perf_counter() > t_stop and len(times) >= 3:
            break
    return times, cores


def cpu_baseline(seconds=10.0):
    times, cores = _cpu_decode_rate(seconds)
    t = statistics.median(times)
    return {"value": round(decode_state_bytes(DECODE_B) / t / 1e9, 3), "unit": UNIT, "cores": cores,
            "kind": "port",
            "sample": f"full gdn_decode B=64 steps on the CPU oracle (oracle/gdn_oracle.c, "
                      f"{cores} OpenMP threads), median of {len(times)} runs, {t * 1e3:.1f} ms each"}


def cpu_prefill_baseline(tokens=PREFILL_T):
    """Prefill tokens/s of the C oracle on the whole 8192-token workload (one
    sequence, all 32 v-heads, zero initial state), all host cores."""
    from oracle import oracle
    from rocm_flashinfer_contest_b200 import inputs
    args = inputs.prefill_inputs([tokens], H, HV, seed=2000, with_state=False)
    cores = os.cpu_count() or 1
    times = []
    for _ in range(3):
        t0 = time.perf_counter()
        oracle.prefill(*args, threads=cores)
        times.append(time.perf_counter() - t0)
    t = statistics.median(times)
    return {"value": round(tokens / t, 1), "unit": "tokens/s", "cores": cores, "kind": "port",
            "sample": f"the whole T={tokens} sequence, all {HV} v-heads, C oracle port, {cores} OpenMP "
                      f"threads, median of 3 ({t * 1e3:.0f} ms each)"}


def cpu_template_baseline():
    """The contest's own pure-torch reference (flashinfer-python's
    _gdn_decode_reference, flashinfer/trace/templates/gdn.py:27-94) on the
    host cores for one decode step at B = 64: the definition's reference
    implementation, timed once (it is ~70x slower than the C port)."""
    try:
        from flashinfer.trace.templates import gdn as tmpl
        ref = tmpl._gdn_decode_reference
    except Exception as e:  # noqa: BLE001
        return {"unavailable": "flashinfer's torch template could not be imported: " + _why(e)}
    from rocm_flashinfer_contest_b200 import inputs
    cores = os.cpu_count() or 1
    torch.set_num_threads(cores)
    args = inputs.decode_inputs(DECODE_B, H, HV, seed=1000)
    q, k, v, state, A_log, a, dt_bias, b, scale = args
    try:
        t0 = time.perf_counter()
        ref(q, k, v, state, A_log, a, dt_bias, b, scale)
        t = time.perf_counter() - t0
    except Exception as e:  # noqa: BLE001
        return {"unavailable": "flashinfer's torch template failed on the CPU: " + _why(e)}
    return {"value": round(decode_state_bytes(DECODE_B) / t / 1e9, 4), "unit": UNIT, "cores": cores,
            "kind": "reference",
            "sample": f"one gdn_decode B=64 step of flashinfer 0.6.11's _gdn_decode_reference (the contest "
                      f"definition's torch reference) on the CPU, torch.set_num_threads({cores}), "
                      f"{t * 1e3:.0f} ms"}


def bench_reference(args, rank, world):
    if rank != 0:
        return None
    B = DECODE_B * world  # the same whole-job batch as our arm at this world size
    times, cores = _cpu_decode_rate(0.0, steps=args.steps, warmup=args.warmup, B=B)
    t = statistics.mean(times)
    value = decode_state_bytes(B) / t / 1e9
    return {
        "impl": "reference",
        "metric": METRIC, "value": round(value, 3), "unit": UNIT, "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(t * 1e3, 3),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "f32 state / bf16 io",
        "data": "synthetic (seeded; contest dataset not available offline)",
        "config": {"workload": "gdn_decode B=64 per GPU, in-place state (BASELINE configs[1])",
                   "B_per_gpu": DECODE_B, "B_total": B, "H": H, "HV": HV, "head_size": D,
                   "l2": "flushed (256 MiB write) before every timed step",
                   "parallelism": f"sequence shards x{world}, no collective"},
        "e2e": {"value": round(value, 3), "unit": UNIT, "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
        "cpu_baseline": {"value": round(value, 3), "unit": UNIT, "cores": cores, "kind": "port",
                         "sample": f"{len(times)} full gdn_decode B={B} steps, C oracle port of the "
                                   f"contest reference, {cores} OpenMP threads"},
        "note": "the reference's own GDN solutions are Triton/AITER kernels for MI300X (ROCm); "
                "its algorithm is timed on the host cores through the C oracle port",
    }


def _json_channel():
    """The JSON line is the only thing this program writes to stdout: a
    duplicate of the original stdout carries it, and file descriptor 1 is
    pointed at stderr so that library banners (NCCL prints its version at
    communicator creation) cannot reach stdout."""
    sys.stdout.flush()
    out = os.fdopen(os.dup(1), "w")
    os.dup2(2, 1)
    return out


def main():
    json_out = _json_channel()
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--cpu-seconds", type=float, default=10.0)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-bars", action="store_true",
                    help="skip the paired library bars and the contest workloads (one GPU)")
    args = ap.parse_args()
    if args.warmup < 3:
        ap.error("--warmup must be >= 3")
    if args.impl == "reference":
        # the reference arm is host-only: rank 0 runs it, other ranks exit at once
        rank = int(os.environ.get("RANK", "0"))
        world = int(os.environ.get("WORLD_SIZE", "1"))
        line = bench_reference(args, rank, world)
        if line is not None:
            print(json.dumps(line), file=json_out, flush=True)
        return
    rank, world, local = dist_setup()
    if world != args.gpus and world > 1:
        print(f"warning: --gpus {args.gpus} but WORLD_SIZE {world}", file=sys.stderr)
    try:
        line = bench_ours(args, rank, world, local)
        if rank == 0 and line is not None:
            print(json.dumps(line), file=json_out, flush=True)
    finally:
        if world > 1:
            import torch.distributed as dist
            dist.destroy_process_group()


if __name__ == "__main__":
    main()

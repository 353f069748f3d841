"""Harness-style verification sweep through the packed solutions.

Mirrors the reference's correctness loop (tools/local_verify.py:89-136,
tools/run_benchmarks.py:188-199): pack both solutions, load main.py from the
source text in solution.json as the harness's PythonBuilder does, build the
inputs of each contest workload bucket (definitions gdn_*_qk4_v8_d128_k_last:
H = 4, HV = 8; decode batch 1..64, prefill total length 6..8192 with 1..39
sequences, docs/ROADMAP.md:41-42), call ``run`` positionally on clones,
compare every output with the CPU oracle at the contest's atol = rtol = 1e-2
with a matched ratio of 1.0, and check that the inputs were not modified
(the harness times on shared inputs and flags mutation).  The fp32 state is
also held to this build's tighter bound (1e-3 relative + 1e-3 of max).
"""
import importlib.util
import json

import pytest
import torch

from oracle import oracle
from parity import assert_state_close, output_report
from rocm_flashinfer_contest_b200 import inputs
from rocm_flashinfer_contest_b200.solution import pack

pytestmark = pytest.mark.gpu

H, HV = 4, 8
DECODE_BUCKETS = [1, 4, 8, 16, 32, 48, 64]
PREFILL_BUCKETS = [(6, 1), (139, 3), (1024, 8), (8192, 39)]


@pytest.fixture(scope="module")
def solutions(tmp_path_factory):
    d = tmp_path_factory.mktemp("solutions")
    runs = {}
    for path, (definition, name, _) in zip(pack.pack(str(d)), pack.SOLUTIONS):
        sol = json.load(open(path))
        assert sol["spec"]["entry_point"] == "main.py::run"
        main = d / f"{name}_main.py"
        main.write_text(sol["sources"][0]["content"])
        spec = importlib.util.spec_from_file_location(f"{name}_main", main)
        mod = importlib.util.module_from_spec(spec)
        spec.loader.exec_module(mod)
        runs[definition.split("_qk")[0]] = mod.run
    return runs


def _clone(args):
    return [x.clone() if isinstance(x, torch.Tensor) else x for x in args]


def _contest_close(sol, ref, what):
    rep = output_report(sol, ref, atol=1e-2, rtol=1e-2)
    assert rep["nonfinite"] == 0 and rep["bad"] == 0, f"{what}: matched ratio below 1.0: {rep}"


def _check(run, host, dev, shapes):
    shared = inputs.to_device(host, dev)
    pristine = _clone(shared)
    o, s = run(*_clone(shared))                   # correctness on clones
    o2, s2 = run(*shared)                         # timing path: shared inputs
    torch.cuda.synchronize()
    for i, (x, y) in enumerate(zip(shared, pristine)):
        if isinstance(x, torch.Tensor):
            assert torch.equal(x, y), f"input {i} was modified"
    assert torch.equal(o, o2) and torch.equal(s, s2)
    assert (tuple(o.shape), o.dtype, tuple(s.shape), s.dtype) == shapes
    return o.cpu(), s.cpu()


@pytest.mark.parametrize("B", DECODE_BUCKETS)
def test_decode_bucket(solutions, cuda_device, B):
    host = inputs.decode_inputs(B, H, HV, seed=600 + B)
    o, s = _check(solutions["gdn_decode"], host, cuda_device,
                  ((B, 1, HV, 128), torch.bfloat16, (B, HV, 128, 128), torch.float32))
    ro, rs = oracle.decode(*host)
    _contest_close(o, ro, f"decode B={B} output")
    _contest_close(s, rs, f"decode B={B} new_state")
    assert_state_close(s, rs, f"decode B={B} new_state")


@pytest.mark.parametrize("cu_dtype", [torch.int32, torch.int64])
@pytest.mark.parametrize("T,N", PREFILL_BUCKETS)
def test_prefill_bucket(solutions, cuda_device, T, N, cu_dtype):
    lens = inputs.seqlens_split(T, N, seed=700 + T)
    host = inputs.prefill_inputs(lens, H, HV, seed=800 + T, cu_dtype=cu_dtype)
    o, s = _check(solutions["gdn_prefill"], host, cuda_device,
                  ((T, HV, 128), torch.bfloat16, (N, HV, 128, 128), torch.float32))
    ro, rs = oracle.prefill(*host)
    _contest_close(o, ro, f"prefill T={T} N={N} output")
    _contest_close(s, rs, f"prefill T={T} N={N} new_state")
    assert_state_close(s, rs, f"prefill T={T} N={N} new_state")

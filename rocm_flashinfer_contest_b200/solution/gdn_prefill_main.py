"""B200 (sm_100a) solution for gdn_prefill_*_k_last.

Entry point main.py::run with the definition's positional inputs
(q, k, v, state, A_log, a, dt_bias, b, cu_seqlens, scale) -> (output, new_state);
the kernels live in the rocm_flashinfer_contest_b200 package (libgdn_b200.so).
"""
from rocm_flashinfer_contest_b200.gdn_prefill import run  # noqa: F401

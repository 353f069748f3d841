"""B200 (sm_100a) gated-delta-rule kernels behind the contest's GDN ``run`` API.

* ``gdn_decode.run(q, k, v, state, A_log, a, dt_bias, b, scale)``
* ``gdn_prefill.run(q, k, v, state, A_log, a, dt_bias, b, cu_seqlens, scale)``
* ``gdn_mtp.run(q, k, v, initial_state, initial_state_indices, A_log, a, dt_bias,
  b, scale, intermediate_states_buffer=None)`` and flashinfer's
  ``gdn_mtp.gated_delta_rule_mtp(...)`` (pool-indexed multi-token decode)

Both call hand-written CUDA kernels through the C ABI in ``include/gdn_b200.h``
(``libgdn_b200.so``, built by ``python -m rocm_flashinfer_contest_b200.build``).
"""
from . import gdn_decode, gdn_mtp, gdn_prefill  # noqa: F401
from ._lib import GDNError, LIB_PATH  # noqa: F401

__all__ = ["gdn_decode", "gdn_mtp", "gdn_prefill", "GDNError", "LIB_PATH"]

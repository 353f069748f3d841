"""Host-side logic of the run() shims and the input generator (no GPU)."""
import math

import pytest
import torch

from rocm_flashinfer_contest_b200 import _common as C
from rocm_flashinfer_contest_b200 import gdn_decode, gdn_prefill, inputs


@pytest.mark.parametrize("scale,expect", [
    (0.0, 1 / math.sqrt(128)), (None, 1 / math.sqrt(128)), (0.5, 0.5),
    (torch.tensor(0.25), 0.25), (torch.tensor(0.0), 1 / math.sqrt(128)), (2, 2.0),
])
def test_scale_rule(scale, expect):
    assert C.normalize_scale(scale, 128) == pytest.approx(expect)


def test_cpu_tensors_fail_loudly():
    args = inputs.decode_inputs(1, 1, 2)
    with pytest.raises(RuntimeError, match="CUDA"):
        gdn_decode.run(*args)
    pargs = inputs.prefill_inputs([3, 2], 1, 2)
    with pytest.raises(RuntimeError, match="CUDA"):
        gdn_prefill.run(*pargs)


def test_decode_input_shapes_and_distributions():
    q, k, v, state, A_log, a, dt_bias, b, scale = inputs.decode_inputs(4, seed=0)
    assert q.shape == (4, 1, 16, 128) and q.dtype == torch.bfloat16
    assert v.shape == (4, 1, 32, 128) and state.shape == (4, 32, 128, 128)
    assert a.shape == b.shape == (4, 1, 32) and A_log.shape == dt_bias.shape == (32,)
    norms = q.float().norm(dim=-1)
    assert torch.allclose(norms, torch.ones_like(norms), atol=1e-2)
    assert 0.0 <= float(A_log.min()) and float(A_log.max()) <= math.log(16)
    assert -1.0 <= float(dt_bias.min()) and float(dt_bias.max()) <= 1.0
    assert abs(float(state.std()) - 0.1) < 0.01
    assert scale == pytest.approx(1 / math.sqrt(128))
    again = inputs.decode_inputs(4, seed=0)
    assert torch.equal(again[0], q) and torch.equal(again[3], state)


def test_prefill_inputs_and_seqlens():
    lens = inputs.seqlens_uniform(16, 1, 1024, seed=0, max_total=8192)
    assert len(lens) == 16 and sum(lens) <= 8192 and min(lens) >= 1 and max(lens) <= 1024
    args = inputs.prefill_inputs([5, 0, 7], H=2, HV=4, cu_dtype=torch.int64)
    q, k, v, state, A_log, a, dt_bias, b, cu, scale = args
    assert q.shape == (12, 2, 128) and v.shape == (12, 4, 128) and state.shape == (3, 4, 128, 128)
    assert cu.tolist() == [0, 5, 5, 12] and cu.dtype == torch.int64


def test_shape_validation_messages():
    # validation order: device first, so a CPU tensor fails with the CUDA message
    args = inputs.decode_inputs(1, 1, 2)
    args[0] = args[0][..., :64]
    with pytest.raises(RuntimeError):
        gdn_decode.run(*args)

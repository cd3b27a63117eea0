"""Failure detection on the GPU without a GPU fault: a sweep kernel's stage wait is made to run
out (its iteration limit set to 0 through pq_set_wait_limit), so the kernel records
ERR_MBAR_TIMEOUT, waits with its fixed limit for the bulk copies it has already issued, and
returns.  The host reads the status, the cost pass raises instead of returning partial numbers,
and the context stays usable: the next sweep with the default limit is exact again."""
import numpy as np
import pytest
import torch

from oracle import pq_oracle as O
from prismaquant_b200 import _lib
from prismaquant_b200 import export_native_compressed as enc
from prismaquant_b200 import format_registry as fr
from tests._helpers import to_cuda_bf16

pytestmark = pytest.mark.gpu

ERR_MBAR_TIMEOUT = 1


def _plan():
    bits = O.synthetic_weight_bits((512, 4096), seed=11, outlier_frac=0.001)
    specs = [fr.get_format(f) for f in ("NVFP4", "MXFP8", "FP8_E4M3", "BF16")]
    return bits, enc.SweepExportPlan({"model.layers.0.mlp.down_proj": to_cuda_bf16(bits)}, specs)


def test_stage_wait_timeout_is_reported_and_context_survives():
    assert _lib.device_error() == 0
    bits, plan = _plan()
    _lib.set_wait_limit(0)
    try:
        plan.run()
        torch.cuda.synchronize()
    finally:
        _lib.set_wait_limit(None)
    assert _lib.device_error() == ERR_MBAR_TIMEOUT   # read and cleared
    assert _lib.device_error() == 0
    # the same plan, default limit: exact again, no error
    plan.run()
    costs = plan.costs()["model.layers.0.mlp.down_proj"]
    for f in ("NVFP4", "MXFP8", "FP8_E4M3"):
        assert costs[f] == pytest.approx(O.cost_mse(bits, f), rel=1e-5)
    want = O.nvfp4_pack(O.bf16_bits_to_f32(bits))
    assert np.array_equal(plan.outputs[0][0].cpu().numpy(), want[0])


def test_cost_pass_raises_on_timeout():
    _, plan = _plan()
    _lib.set_wait_limit(0)
    try:
        plan.run()
        with pytest.raises(RuntimeError, match="bounded wait gave up"):
            plan.costs()
    finally:
        _lib.set_wait_limit(None)
    assert _lib.device_error() == 0

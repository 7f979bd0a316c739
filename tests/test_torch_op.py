"""The registered torch operator ``torch.ops.strassen_b200.strassen_matmul`` (no GPU needed).

Its fake implementation must give the shapes and dtypes the reference derives
(strassen_pallas.py:1132-1141) so the operator can sit inside traced torch code;
the CUDA implementation is checked against the direct call in
test_gpu_torch_op.py.
"""

from __future__ import annotations

import pytest
import torch
from torch._subclasses.fake_tensor import FakeTensorMode

import strassen_tpu_b200  # noqa: F401  (registers the operator)

BF = torch.bfloat16
OP = torch.ops.strassen_b200.strassen_matmul


def test_schema_keeps_the_reference_argument_names():
    names = [arg.name for arg in OP.default._schema.arguments]
    for name in ("a", "b", "bm", "bn", "bk", "epilogue", "residual", "bias", "rope_cos", "rope_sin",
                 "rope_scale", "rope_head_dim", "rope_eps", "norm_scale", "norm_eps", "output_dtype",
                 "interleave_products", "block_permutation", "formula_variant", "classical_panels",
                 "panel_schedule", "product_aware_swiglu", "product_aware_residual"):
        assert name in names, name
    assert OP.default._schema.returns[0].type.kind() == "TensorType"


@pytest.mark.parametrize("kw, shape, dtype", [
    (dict(), (512, 1024), BF),
    (dict(output_dtype=torch.float32), (512, 1024), torch.float32),
    (dict(epilogue="swiglu"), (512, 512), BF),
    (dict(epilogue="geglu"), (512, 512), BF),
    (dict(epilogue="residual_add"), (512, 1024), BF),
])
def test_fake_shapes(kw, shape, dtype):
    with FakeTensorMode():
        a = torch.empty(512, 256, dtype=BF)
        b = torch.empty(256, 1024, dtype=BF)
        out = OP(a, b, 256, 512, 256, **kw)
    assert tuple(out.shape) == shape and out.dtype == dtype


def test_fake_rejects_mismatched_inner_dimensions():
    with FakeTensorMode():
        with pytest.raises(ValueError, match="matching inner dimensions"):
            OP(torch.empty(512, 256, dtype=BF), torch.empty(512, 256, dtype=BF), 256, 256, 256)


def test_real_call_on_cpu_tensors_fails_loudly():
    # No CPU fallback: the operator's only implementation is the CUDA library.
    with pytest.raises(ValueError, match="runs on a CUDA device"):
        OP(torch.zeros(256, 256, dtype=BF), torch.zeros(256, 256, dtype=BF), 256, 256, 256)

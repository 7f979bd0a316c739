"""``torch.ops.strassen_b200.strassen_matmul`` on a B200: the registered operator
gives exactly what the direct call gives, passes torch's operator checks, and
runs inside a compiled torch function (the torch counterpart of the reference
calling ``strassen_matmul`` under ``jax.jit``, strassen_pallas.py:882-911)."""

from __future__ import annotations

import pytest
import torch

pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(not torch.cuda.is_available(), reason="needs a CUDA device")]


def _inputs(m=512, k=512, n=1024, seed=3):
    g = torch.Generator(device="cuda").manual_seed(seed)
    a = torch.randn(m, k, device="cuda", generator=g).to(torch.bfloat16)
    b = torch.randn(k, n, device="cuda", generator=g).to(torch.bfloat16)
    return a, b


@pytest.mark.parametrize("kw", [dict(), dict(output_dtype=torch.float32), dict(epilogue="swiglu"),
                                dict(formula_variant="dual", block_permutation=3)])
def test_op_equals_direct_call(kw):
    import strassen_tpu_b200 as sb
    a, b = _inputs()
    op = torch.ops.strassen_b200.strassen_matmul(a, b, 256, 512, 256, **kw)
    direct = sb.strassen_matmul(a, b, bm=256, bn=512, bk=256, **kw)
    assert torch.equal(op, direct)


def test_opcheck():
    a, b = _inputs()
    torch.library.opcheck(torch.ops.strassen_b200.strassen_matmul.default, (a, b, 256, 512, 256))


def test_inside_a_compiled_function():
    import strassen_tpu_b200 as sb
    a, b = _inputs()
    residual = torch.randn(512, 1024, device="cuda").to(torch.bfloat16)

    def block(x, w, r):
        y = torch.ops.strassen_b200.strassen_matmul(x, w, 256, 512, 256, epilogue="residual_add", residual=r)
        return y.float().square().mean()

    compiled = torch.compile(block, fullgraph=True)
    want = sb.strassen_matmul(a, b, bm=256, bn=512, bk=256, epilogue="residual_add", residual=residual)
    torch.testing.assert_close(compiled(a, b, residual), want.float().square().mean(), rtol=1e-5, atol=0)

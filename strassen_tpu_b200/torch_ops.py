"""``strassen_matmul`` as a registered torch operator: ``torch.ops.strassen_b200.strassen_matmul``.

The reference's operator is a JAX function that XLA traces into a larger
program (strassen_pallas.py:882-911: functional, fresh output buffer, every
shape rule checked on the host at trace time).  The torch counterpart of that
contract is a ``torch.library`` custom operator: it has a schema, a fake
(meta) implementation that gives the output's shape and dtype without running
anything, and a CUDA implementation that calls :func:`strassen_matmul`.  That
lets callers put the operator inside code that torch traces (``torch.compile``,
``torch.export``, CUDA-graph capture through torch's own tools) the way the
reference's callers put ``strassen_matmul`` inside ``jax.jit``.

Arguments keep the reference's names and meaning; the arguments that only steer
the TPU compiler (``dot_precision``, ``allow_input_fusion``,
``vmem_limit_bytes``) and ``interpret`` are left out because they do not change
the result.  ``output_dtype`` is a torch dtype (or None = the input dtype).
The operator is inference-only, like the reference's kernel (no autograd
formula).
"""

from __future__ import annotations

from typing import Optional

import torch

from . import strassen as _sp

_FUSED_HALF = ("swiglu", "geglu")


@torch.library.custom_op("strassen_b200::strassen_matmul", mutates_args=())
def strassen_matmul_op(
    a: torch.Tensor,
    b: torch.Tensor,
    bm: int,
    bn: int,
    bk: int,
    epilogue: Optional[str] = None,
    residual: Optional[torch.Tensor] = None,
    bias: Optional[torch.Tensor] = None,
    rope_cos: Optional[torch.Tensor] = None,
    rope_sin: Optional[torch.Tensor] = None,
    rope_scale: Optional[torch.Tensor] = None,
    rope_head_dim: int = 128,
    rope_eps: float = 1e-6,
    norm_scale: Optional[torch.Tensor] = None,
    norm_eps: float = 1e-6,
    output_dtype: Optional[torch.dtype] = None,
    interleave_products: bool = False,
    block_permutation: int = 0,
    formula_variant: str = "classical",
    classical_panels: Optional[list[int]] = None,
    panel_schedule: Optional[torch.Tensor] = None,
    product_aware_swiglu: bool = False,
    product_aware_residual: bool = False,
    narrow_bn: bool = False,
) -> torch.Tensor:
    """``strassen_matmul(a, b, bm=, bn=, bk=, ...)`` (strassen_pallas.py:882-1221)."""
    return _sp.strassen_matmul(
        a, b, bm=bm, bn=bn, bk=bk, epilogue=epilogue, residual=residual, bias=bias,
        rope_cos=rope_cos, rope_sin=rope_sin, rope_scale=rope_scale, rope_head_dim=rope_head_dim,
        rope_eps=rope_eps, norm_scale=norm_scale, norm_eps=norm_eps, output_dtype=output_dtype,
        interleave_products=interleave_products, block_permutation=block_permutation,
        formula_variant=formula_variant, classical_panels=tuple(classical_panels or ()),
        panel_schedule=panel_schedule, product_aware_swiglu=product_aware_swiglu,
        product_aware_residual=product_aware_residual, narrow_bn=narrow_bn)


@strassen_matmul_op.register_fake
def _strassen_matmul_fake(a, b, bm, bn, bk, epilogue=None, residual=None, bias=None, rope_cos=None,
                          rope_sin=None, rope_scale=None, rope_head_dim=128, rope_eps=1e-6,
                          norm_scale=None, norm_eps=1e-6, output_dtype=None, interleave_products=False,
                          block_permutation=0, formula_variant="classical", classical_panels=None,
                          panel_schedule=None, product_aware_swiglu=False, product_aware_residual=False,
                          narrow_bn=False):
    # Output shape and dtype as strassen_pallas.py:1132-1141 derives them: fused
    # epilogues write a bf16 tile; swiglu/geglu halve the columns.
    if a.dim() != 2 or b.dim() != 2 or a.shape[1] != b.shape[0]:
        raise ValueError("strassen_matmul expects two rank-2 matrices with matching inner dimensions")
    m, n = a.shape[0], b.shape[1]
    if epilogue in _FUSED_HALF:
        n = n // 2
    dtype = a.dtype if output_dtype is None or epilogue is not None else output_dtype
    return a.new_empty((m, n), dtype=dtype)

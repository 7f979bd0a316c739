"""B200-native (sm_100a) tile-local Strassen GEMM with fused Qwen3 epilogues.

Drop-in for the reference operator API ``strassen_pallas`` (sarsid/strassen-tpu):
``strassen_matmul``, ``native_matmul``, ``tuned_matmul``, ``check_tiling`` and the
weight/table layout helpers.  The kernels live in ``csrc/`` behind the C ABI declared in
``include/strassen_b200.h``.
"""

from .layouts import (
    rope_layout_tables,
    rope_layout_to_heads,
    rope_scale_layout,
    rope_weight_layout,
    swiglu_weight_layout,
)
from .strassen import (
    TUNED_BK,
    TUNED_BM,
    TUNED_BN,
    check_tiling,
    classical_matmul,
    native_matmul,
    pair_matmul,
    planes_matmul,
    quad_matmul,
    rms_norm,
    StrassenBOperands,
    strassen_b_operands,
    strassen_matmul,
    strassen_matmul_lhs_transposed,
    strassen_matmul_streamed,
    workspace_bytes,
)
from .torch_ops import strassen_matmul_op  # registers torch.ops.strassen_b200.strassen_matmul

__all__ = [
    "TUNED_BM", "TUNED_BN", "TUNED_BK",
    "check_tiling", "classical_matmul", "native_matmul", "rms_norm", "strassen_matmul",
    "pair_matmul", "planes_matmul", "quad_matmul", "StrassenBOperands", "strassen_b_operands", "strassen_matmul_lhs_transposed", "strassen_matmul_streamed", "tuned_matmul",
    "workspace_bytes", "strassen_matmul_op",
    "rope_layout_tables", "rope_layout_to_heads", "rope_scale_layout", "rope_weight_layout",
    "swiglu_weight_layout",
]


def __getattr__(name):
    # tuned_matmul lives in .tuning, imported on first use so that
    # `python -m strassen_tpu_b200.tuning` does not import the module twice.
    if name == "tuned_matmul":
        from .tuning import tuned_matmul
        return tuned_matmul
    raise AttributeError(f"module {__name__!r} has no attribute {name!r}")

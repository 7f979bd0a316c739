"""Host-side contract of ``strassen_matmul`` (no GPU needed).

Validation mirrors the reference's ValueError/TypeError conditions and messages
(strassen_pallas.py:927-1057, check_tiling :127-140), raised before any launch.
CPU tensors are used: every case here fails validation first.
"""

from __future__ import annotations

import pytest
import torch

import strassen_tpu_b200 as sb

BF = torch.bfloat16


def mats(m=256, k=256, n=256, dtype=BF):
    return torch.zeros(m, k, dtype=dtype), torch.zeros(k, n, dtype=dtype)


def call(a=None, b=None, **kw):
    if a is None:
        a, b = mats()
    kw.setdefault("bm", 256)
    kw.setdefault("bn", 256)
    kw.setdefault("bk", 256)
    return sb.strassen_matmul(a, b, **kw)


@pytest.mark.parametrize("kw, match", [
    (dict(a=torch.zeros(2, 2, 2, dtype=BF), b=torch.zeros(2, 2, dtype=BF)), "two rank-2 matrices"),
    (dict(a=torch.zeros(256, 512, dtype=BF), b=torch.zeros(256, 256, dtype=BF)), "inner dimensions disagree: 512 vs 256"),
    (dict(a=torch.zeros(256, 256, dtype=BF), b=torch.zeros(256, 256, dtype=torch.float32)), "input dtypes disagree"),
    (dict(a=torch.zeros(256, 256, dtype=torch.float16), b=torch.zeros(256, 256, dtype=torch.float16)), "BF16 or FP32"),
    (dict(block_permutation=8), "block_permutation"),
    (dict(formula_variant="winograd"), "formula_variant"),
    (dict(epilogue="relu"), "unknown epilogue 'relu'"),
    (dict(epilogue="swiglu", output_dtype=torch.float32), "fused epilogues write a BF16 output tile"),
    (dict(epilogue="residual_add"), "residual_add epilogue requires residual="),
    (dict(epilogue="bias_add"), "bias_add epilogue requires bias="),
    (dict(residual=torch.zeros(256, 256, dtype=BF)), "residual= is only used"),
    (dict(bias=torch.zeros(256, dtype=BF)), "bias= is only used"),
    (dict(epilogue="norm_residual_add"), "norm_residual_add requires residual= and norm_scale="),
    (dict(epilogue="qk_norm_rope"), "qk_norm_rope epilogue requires rope_cos="),
    (dict(rope_cos=torch.zeros(256, 128, dtype=BF)), "rope_\\* are only used"),
    (dict(product_aware_swiglu=True), "product_aware_swiglu is only valid"),
    (dict(product_aware_residual=True), "product_aware_residual is only valid"),
    (dict(allow_input_fusion=(True,)), "one boolean per operand: expected 2, got 1"),
    (dict(classical_panels=(0,), panel_schedule=[0]), "either classical_panels"),
    (dict(classical_panels=(5,)), "outside 0..0"),
    (dict(bm=48), "M=256 is not divisible by 48"),
    (dict(bn=128, a=torch.zeros(256, 256, dtype=BF), b=torch.zeros(256, 256, dtype=BF)), "bn=128 must be a multiple of 256"),
    (dict(bm=8, a=torch.zeros(16, 256, dtype=BF), b=torch.zeros(256, 256, dtype=BF)), "bm=8 must be a multiple of 16"),
    (dict(output_dtype="float16"), "output_dtype must be BF16 or FP32"),
])
def test_reference_value_errors(kw, match):
    with pytest.raises(ValueError, match=match):
        call(**kw)


def test_allow_input_fusion_type_error():
    with pytest.raises(TypeError, match="entries must be bool"):
        call(allow_input_fusion=(1, 0))


def test_norm_residual_requires_full_row_tile():
    a, b = mats(256, 256, 512)
    with pytest.raises(ValueError, match="bn=256 must equal n=512"):
        call(a, b, epilogue="norm_residual_add", residual=torch.zeros(256, 512, dtype=BF),
             norm_scale=torch.ones(512, dtype=BF))


def test_qk_norm_rope_shape_contract():
    a, b = mats(256, 256, 512)
    with pytest.raises(ValueError, match="bn a multiple of 2\\*head_dim=768"):
        call(a, b, bn=512, epilogue="qk_norm_rope", rope_head_dim=384, rope_cos=torch.zeros(256, 256),
             rope_sin=torch.zeros(256, 256), rope_scale=torch.zeros(512))
    with pytest.raises(ValueError, match="rope tables must be \\(256, 256\\)"):
        call(a, b, bn=512, epilogue="qk_norm_rope", rope_cos=torch.zeros(256, 128),
             rope_sin=torch.zeros(256, 128), rope_scale=torch.zeros(512))
    with pytest.raises(ValueError, match="rope_scale must be laid out to \\(512,\\)"):
        call(a, b, bn=512, epilogue="qk_norm_rope", rope_cos=torch.zeros(256, 256),
             rope_sin=torch.zeros(256, 256), rope_scale=torch.zeros(128))


def test_no_cpu_path():
    # A valid call on CPU tensors must refuse, not silently compute on the host.
    with pytest.raises(ValueError, match="no CPU fallback"):
        call()
    with pytest.raises(NotImplementedError, match="no CPU path"):
        call(interpret=True)


def test_unbuilt_reference_options_refuse_loudly():
    with pytest.raises(NotImplementedError, match="FP32 inputs"):
        call(*mats(dtype=torch.float32))
    with pytest.raises(NotImplementedError, match="quadrant-basis"):
        call(formula_variant="powers", panel_schedule=[1])


def test_research_options_reach_the_device_check():
    # dual / block_permutation / exact panels are built: on CPU tensors they
    # fail only at the device check, after validation.
    for kw in (dict(formula_variant="dual"), dict(block_permutation=3), dict(classical_panels=(0,)),
               dict(panel_schedule=[1]), dict(formula_variant="powers")):
        with pytest.raises(ValueError, match="no CPU fallback"):
            call(**kw)


def test_product_aware_schedule_contract():
    a, b = mats(256, 512, 512)
    with pytest.raises(ValueError, match="product-aware SwiGLU requires unpermuted classical"):
        call(a, b, bn=512, epilogue="swiglu", product_aware_swiglu=True, classical_panels=(1,))
    with pytest.raises(ValueError, match="product-aware SwiGLU requires unpermuted classical"):
        call(a, b, bn=512, epilogue="swiglu", product_aware_swiglu=True, block_permutation=1)
    with pytest.raises(ValueError, match="product-aware residual requires"):
        call(a, b, epilogue="residual_add", residual=torch.zeros(256, 512, dtype=BF),
             product_aware_residual=True, formula_variant="dual")
    with pytest.raises(ValueError, match="panel_schedule must have shape \\(2,\\)"):
        call(a, b, panel_schedule=[1, 0, 1])


def test_check_tiling_message():
    with pytest.raises(ValueError) as err:
        sb.check_tiling(8, 128, 100)
    msg = str(err.value)
    assert msg.startswith("tile breaks TPU v5e alignment:")
    assert "bm=8 must be a multiple of 16" in msg
    assert "bn=128 must be a multiple of 256" in msg
    assert "bk=100 must be a multiple of 256" in msg
    sb.check_tiling(16, 256, 256)


def test_streamed_validates_before_touching_the_device():
    a = torch.zeros(2048, 512, dtype=torch.bfloat16)
    b = torch.zeros(512, 1024, dtype=torch.bfloat16)
    with pytest.raises(ValueError, match="residual= is not streamed"):
        sb.strassen_matmul_streamed(a, b, bm=1024, bn=1024, bk=512, epilogue="residual_add", residual=a)
    with pytest.raises(ValueError, match="row_chunk=1536"):
        sb.strassen_matmul_streamed(a, b, bm=1024, bn=1024, bk=512, row_chunk=1536)
    with pytest.raises(ValueError, match="inner dimensions disagree"):
        sb.strassen_matmul_streamed(a, b.t(), bm=1024, bn=1024, bk=512)
    with pytest.raises(ValueError, match="is not divisible by"):
        sb.strassen_matmul_streamed(a[:1536], b, bm=1024, bn=1024, bk=512)


# --- the two-CTA kernel's host API (pair_matmul, strassen_b_operands) ---------

@pytest.mark.parametrize("kw, match", [
    (dict(a=torch.zeros(2, 2, 2, dtype=BF)), "two rank-2 matrices"),
    (dict(a=torch.zeros(256, 512, dtype=BF)), "inner dimensions disagree: 512 vs 256"),
    (dict(a=torch.zeros(256, 256, dtype=torch.float32)), "inputs must be BF16"),
    (dict(bm=48), "M=256 is not divisible by 48"),
    (dict(bn=128), "bn=128 must be a multiple of 256"),
    (dict(), "runs on a CUDA device"),  # valid arguments, but CPU tensors: no CPU fallback
])
def test_pair_matmul_value_errors(kw, match):
    a = kw.pop("a", torch.zeros(256, 256, dtype=BF))
    b = torch.zeros(256, 256, dtype=BF)
    kw.setdefault("bm", 256)
    kw.setdefault("bn", 256)
    kw.setdefault("bk", 256)
    with pytest.raises(ValueError, match=match):
        sb.pair_matmul(a, b, **kw)


def test_pair_matmul_checks_the_operand_planes():
    a = torch.zeros(256, 512, dtype=BF)
    ops = lambda t, bn=256, bk=256: sb.StrassenBOperands(t, bn, bk)
    with pytest.raises(ValueError, match="StrassenBOperands returned by strassen_b_operands"):
        sb.pair_matmul(a, None, b_operands=torch.zeros(7, 256, 128, dtype=BF), bm=256, bn=256, bk=256)
    with pytest.raises(ValueError, match=r"\[7, K/2, N/2\] bf16 planes"):
        sb.pair_matmul(a, None, b_operands=ops(torch.zeros(6, 256, 128, dtype=BF)), bm=256, bn=256, bk=256)
    with pytest.raises(ValueError, match="describe a 512x256 B, b is"):
        sb.pair_matmul(a, torch.zeros(512, 512, dtype=BF), b_operands=ops(torch.zeros(7, 256, 128, dtype=BF)),
                       bm=256, bn=256, bk=256)
    # Planes formed for another tile are refused: their layout would silently give a wrong product.
    with pytest.raises(ValueError, match="formed for bn=256, bk=512; this call uses bn=256, bk=256"):
        sb.pair_matmul(a, None, b_operands=ops(torch.zeros(7, 256, 128, dtype=BF), 256, 512),
                       bm=256, bn=256, bk=256)
    # Planes of a 512x256 B: shapes agree, so only the device check is left.
    with pytest.raises(ValueError, match="runs on a CUDA device"):
        sb.pair_matmul(a, None, b_operands=ops(torch.zeros(7, 256, 128, dtype=BF)), bm=256, bn=256, bk=256)


def test_strassen_b_operands_refuses_host_tensors_and_other_dtypes():
    with pytest.raises(ValueError, match="rank-2 BF16"):
        sb.strassen_b_operands(torch.zeros(512, 512, dtype=torch.float32), bn=256, bk=256)
    with pytest.raises(ValueError, match="CUDA device"):
        sb.strassen_b_operands(torch.zeros(512, 512, dtype=BF), bn=256, bk=256)


# --- narrow_bn (B200 extension: bn a multiple of 128) -------------------------

def test_narrow_bn_admits_128_wide_tiles():
    # Valid arguments reach the device check; without narrow_bn the reference's rule stands.
    with pytest.raises(ValueError, match="runs on a CUDA device"):
        call(bn=128, narrow_bn=True)
    with pytest.raises(ValueError, match="bn=128 must be a multiple of 256"):
        call(bn=128)
    with pytest.raises(ValueError, match="narrow_bn: bn=64 must be a multiple of 128"):
        call(bn=64, narrow_bn=True)


def test_narrow_bn_qk_norm_rope_needs_whole_half_heads():
    rope = dict(epilogue="qk_norm_rope", rope_cos=torch.zeros(256, 64, dtype=BF),
                rope_sin=torch.zeros(256, 64, dtype=BF), rope_scale=torch.zeros(128, dtype=BF))
    with pytest.raises(ValueError, match="runs on a CUDA device"):
        call(bn=128, narrow_bn=True, rope_head_dim=128, **rope)
    with pytest.raises(ValueError, match="narrow_bn needs bn a multiple of head_dim=256"):
        call(bn=128, narrow_bn=True, rope_head_dim=256, **rope)
    with pytest.raises(ValueError, match="needs bn a multiple of 2\\*head_dim=512"):
        call(bn=256, rope_head_dim=256, **rope)


# --- planes_matmul (the seven-product-GEMM path) --------------------------------

@pytest.mark.parametrize("kw, match", [
    (dict(a=torch.zeros(2, 2, 2, dtype=BF)), "two rank-2 matrices"),
    (dict(a=torch.zeros(512, 256, dtype=BF), b=torch.zeros(512, 512, dtype=BF)), "inner dimensions disagree"),
    (dict(a=torch.zeros(512, 256, dtype=torch.float32)), "inputs must be BF16"),
    (dict(a=torch.zeros(256, 256, dtype=BF)), "M % 512 == 0"),
    (dict(b=torch.zeros(256, 256, dtype=BF)), "N % 512 == 0"),
    (dict(bn=128), "bn=128 must be a multiple of 256"),
    (dict(), "runs on a CUDA device"),  # valid arguments, CPU tensors: no CPU fallback
])
def test_planes_matmul_value_errors(kw, match):
    a = kw.pop("a", torch.zeros(512, 256, dtype=BF))
    b = kw.pop("b", torch.zeros(256, 512, dtype=BF))
    kw.setdefault("bm", 256)
    kw.setdefault("bn", 256)
    kw.setdefault("bk", 256)
    with pytest.raises(ValueError, match=match):
        sb.planes_matmul(a, b, **kw)


# --- rms_norm (the row kernel the decoder's norms run on) -----------------------

@pytest.mark.parametrize("x, scale, match", [
    (torch.zeros(4, 256), torch.ones(256), "expects a bf16 input"),
    (torch.zeros(4, 256, dtype=BF), torch.ones(128), "scale must hold 256 values"),
    (torch.zeros(4, 256, dtype=BF), torch.ones(256), "no CPU fallback"),
])
def test_rms_norm_value_errors(x, scale, match):
    with pytest.raises(ValueError, match=match):
        sb.rms_norm(x, scale)

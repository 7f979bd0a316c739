"""Parity of the two-CTA Strassen kernel (``sb_strassen_gemm_pair`` and
``sb_strassen_gemm_pair_planes``, needs a B200).

The kernel computes the same products as ``sb_strassen_gemm`` (the reference's
strassen_pallas.py:156-880 without an epilogue) with the seven products split
over a cluster of two CTAs.  "raw" forms the B operand sums in the kernel;
"planes" reads them from ``strassen_b_operands``.  Bar: the parity rule of
test_gpu_parity.assert_parity against the reference's own golden vectors,
bit-exact integer and constant known answers, bit-exact agreement between the
two B modes, and agreement with the one-CTA kernel to fp32 rounding (the two
kernels recombine the products in a different fp32 order).
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from conftest import golden_output
from golden_inputs import make_inputs
from oracle import strassen_ref as ref
from test_gpu_parity import GOLDEN_CASES, assert_parity, dev_bf16, fp64_yardstick, host

pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(not torch.cuda.is_available(), reason="needs a CUDA device")]

# Golden cases without an epilogue or research option (interleave_products only
# reorders the reference's fp32 accumulation; it is accepted and ignored here).
PLAIN = [c for c in GOLDEN_CASES if c in {
    "config1_1024_plain", "int_16x256x256", "int_32x768x512", "int_512x1024x512_f32",
    "interleaved_512x512x512", "normal_1024x512x256_bm64", "normal_16x256x256_seed23",
    "normal_256x512x768_f32", "normal_512x512x512_tile512", "sentinel_256x512x256"}]


MODES = ["raw", "planes"]


def pair(a, b, mode, **kw):
    """pair_matmul on device tensors, with B raw or as its operand planes."""
    import strassen_tpu_b200 as sb
    if mode == "planes":
        planes = sb.strassen_b_operands(b, bn=kw["bn"], bk=kw["bk"])
        return sb.pair_matmul(a, None, b_operands=planes, **kw)
    return sb.pair_matmul(a, b, **kw)


@pytest.mark.parametrize("mode", MODES)
@pytest.mark.parametrize("case", PLAIN)
def test_pair_golden_case(golden, case, mode):
    manifest, arrays = golden
    p = manifest[case]
    a, b, extra = make_inputs(p)
    assert not extra
    od = p["kwargs"].get("output_dtype")
    out = pair(dev_bf16(a), dev_bf16(b), mode, bm=p["bm"], bn=p["bn"], bk=p["bk"],
               output_dtype=torch.float32 if od == "float32" else None)
    torch.cuda.synchronize()
    got = host(out)
    assert list(got.shape) == p["shape"]
    stride = p["row_stride"]
    want = golden_output(p, arrays[case])
    got = got[::stride]
    if p["inputs"]["kind"] in ("int", "const"):
        np.testing.assert_array_equal(got, want)
        return
    assert_parity(got, want, fp64_yardstick(p, a, b, extra, slice(None, None, stride)),
                  rounding_step=p["output"] == "bf16_bits")


@pytest.mark.parametrize("shape, tile", [
    ((16, 256, 256), (16, 256, 256)),       # 8 valid product rows of a 128-row tile
    ((48, 512, 512), (16, 256, 256)),       # partial product-row tile, two K panels
    ((384, 768, 1024), (128, 512, 256)),    # 64-row blocks, two column tiles per block
    ((2048, 1024, 768), (1024, 256, 512)),  # large blocks, several row tiles per block
])
@pytest.mark.parametrize("mode", MODES)
def test_pair_exact_integer_products(shape, tile, mode):
    m, k, n = shape
    a = ref.integers_bf16((m, k), -2, 2, 11)
    b = ref.integers_bf16((k, n), -2, 2, 12)
    got = host(pair(dev_bf16(a), dev_bf16(b), mode, bm=tile[0], bn=tile[1], bk=tile[2],
                    output_dtype=torch.float32))
    np.testing.assert_array_equal(got, a @ b)


@pytest.mark.parametrize("m, n, k", [(1024, 1536, 2048), (4096, 4096, 4096)])
def test_pair_matches_one_cta_kernel(m, n, k):
    import strassen_tpu_b200 as sb
    g = torch.Generator(device="cuda").manual_seed(7)
    a = torch.randn(m, k, device="cuda", generator=g).to(torch.bfloat16)
    b = torch.randn(k, n, device="cuda", generator=g).to(torch.bfloat16)
    tile = dict(bm=1024 if m % 1024 == 0 else 256, bn=512, bk=512)
    # An empty workspace keeps a plain product on the one-CTA kernel.
    one = sb.strassen_matmul(a, b, output_dtype=torch.float32, **tile,
                             workspace=torch.empty(0, dtype=torch.uint8, device="cuda"))
    two = sb.pair_matmul(a, b, output_dtype=torch.float32, **tile)
    # Same products and operand sums; the fp32 order of the final four-term sums
    # (and the tensor core's accumulation order at N=128 vs N=64) may differ.
    rms = one.pow(2).mean().sqrt().item()
    assert (two - one).abs().max().item() <= 1e-4 * rms
    bf = sb.pair_matmul(a, b, **tile)
    assert torch.equal(bf, two.to(torch.bfloat16))
    # The planes carry exactly the operand values the in-kernel sums form.
    planes = sb.strassen_b_operands(b, bn=tile["bn"], bk=tile["bk"])
    assert torch.equal(sb.pair_matmul(a, None, b_operands=planes, output_dtype=torch.float32, **tile), two)
    from strassen_tpu_b200 import _native
    assert _native.device_status() == 0


def test_pair_accumulators_reset_between_calls():
    import strassen_tpu_b200 as sb
    a = dev_bf16(ref.normal_bf16((512, 512), 1))
    b = dev_bf16(ref.normal_bf16((512, 512), 2))
    first = sb.pair_matmul(a, b, bm=256, bn=256, bk=256, output_dtype=torch.float32)
    second = sb.pair_matmul(-a, b, bm=256, bn=256, bk=256, output_dtype=torch.float32)
    torch.testing.assert_close(second, -first, rtol=0, atol=0)


def test_pair_validation_matches_the_reference_messages():
    import strassen_tpu_b200 as sb
    a = torch.zeros(256, 256, dtype=torch.bfloat16, device="cuda")
    with pytest.raises(ValueError, match="not divisible"):
        sb.pair_matmul(a, a, bm=256, bn=512, bk=256)
    with pytest.raises(ValueError, match="multiple of 256"):
        sb.pair_matmul(a, a, bm=256, bn=128, bk=256)


def test_b_operand_planes_are_the_reference_pre_adds():
    """Plane i at (kappa, u) is operand i of block (kappa // (bk/2), u // (bn/2)),
    each sum rounded once to bf16 (strassen_pallas.py:324-379)."""
    import strassen_tpu_b200 as sb
    k, n, bn, bk = 1024, 1536, 512, 512
    b = ref.normal_bf16((k, n), 31)
    got = sb.strassen_b_operands(dev_bf16(b), bn=bn, bk=bk).planes.float().cpu().numpy()
    hbn, hbk = bn // 2, bk // 2
    blocks = b.reshape(k // bk, 2, hbk, n // bn, 2, hbn)  # [P, qk, k', J, qc, c']
    q = lambda qk, qc: blocks[:, qk, :, :, qc, :].reshape(k // 2, n // 2)
    b0, b1, b2, b3 = q(0, 0), q(0, 1), q(1, 0), q(1, 1)
    r = ref.bf16_round
    want = np.stack([r(b1 - b3), b3, r(b2 + b3), r(b0 + b3), b0, r(b2 - b0), r(b0 + b1)])
    np.testing.assert_array_equal(got, want)


def test_b_operand_planes_validation():
    import strassen_tpu_b200 as sb
    b = torch.zeros(512, 512, dtype=torch.bfloat16, device="cuda")
    with pytest.raises(ValueError, match="divisible"):
        sb.strassen_b_operands(b, bn=1024, bk=256)
    planes = sb.strassen_b_operands(b, bn=256, bk=256)
    a = torch.zeros(256, 256, dtype=torch.bfloat16, device="cuda")
    with pytest.raises(ValueError, match="inner dimensions"):
        sb.pair_matmul(a, None, b_operands=planes, bm=256, bn=256, bk=256)

"""Parity of the four-CTA Strassen kernel (``sb_strassen_gemm_quad``, needs a B200).

The kernel computes the same products as ``sb_strassen_gemm`` (the reference's
strassen_pallas.py:156-880 without an epilogue) on clusters of two CTA pairs
(tcgen05 ``cta_group::2``), from A operands and B operand planes that the call
forms first.  Bar: the parity rule of test_gpu_parity.assert_parity against the
reference's own golden vectors (the cases its shape rules admit: M % 512,
bn % 256, bk % 256), bit-exact integer known answers, and agreement with the
one-CTA kernel to fp32 rounding (the recombination's fp32 order differs).
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from conftest import golden_output
from golden_inputs import make_inputs
from oracle import strassen_ref as ref
from test_gpu_pair import PLAIN
from test_gpu_parity import assert_parity, dev_bf16, fp64_yardstick, host

pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(not torch.cuda.is_available(), reason="needs a CUDA device")]


def _admitted(case):
    import json
    from conftest import GOLDEN
    p = json.loads((GOLDEN / "golden_cases.json").read_text())["cases"][case]
    m = p["shape"][0]
    return m % 512 == 0 and p["bn"] % 256 == 0 and p["bk"] % 256 == 0


QUAD_CASES = [c for c in PLAIN if _admitted(c)]


@pytest.mark.parametrize("case", QUAD_CASES)
def test_quad_golden_case(golden, case):
    import strassen_tpu_b200 as sb
    manifest, arrays = golden
    p = manifest[case]
    a, b, extra = make_inputs(p)
    assert not extra
    od = p["kwargs"].get("output_dtype")
    out = sb.quad_matmul(dev_bf16(a), dev_bf16(b), bm=p["bm"], bn=p["bn"], bk=p["bk"],
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
    ((512, 256, 256), (64, 256, 256)),      # 32-row blocks: a 256-row tile spans eight blocks
    ((1024, 768, 512), (256, 256, 256)),    # three K panels, two column tiles
    ((2048, 1024, 768), (1024, 256, 512)),  # large blocks, several row tiles per block
])
def test_quad_exact_integer_products(shape, tile):
    import strassen_tpu_b200 as sb
    m, k, n = shape
    a = ref.integers_bf16((m, k), -2, 2, 11)
    b = ref.integers_bf16((k, n), -2, 2, 12)
    got = host(sb.quad_matmul(dev_bf16(a), dev_bf16(b), bm=tile[0], bn=tile[1], bk=tile[2],
                              output_dtype=torch.float32))
    np.testing.assert_array_equal(got, a @ b)


@pytest.mark.parametrize("m, n, k", [(1024, 1536, 2048), (4096, 4096, 4096)])
def test_quad_matches_one_cta_kernel(m, n, k):
    import strassen_tpu_b200 as sb
    from strassen_tpu_b200 import _native
    g = torch.Generator(device="cuda").manual_seed(7)
    a = torch.randn(m, k, device="cuda", generator=g).to(torch.bfloat16)
    b = torch.randn(k, n, device="cuda", generator=g).to(torch.bfloat16)
    tile = dict(bm=1024 if m % 1024 == 0 else 256, bn=512, bk=512)
    # An empty workspace keeps a plain product on the one-CTA kernel.
    one = sb.strassen_matmul(a, b, output_dtype=torch.float32, **tile,
                             workspace=torch.empty(0, dtype=torch.uint8, device="cuda"))
    four = sb.quad_matmul(a, b, output_dtype=torch.float32, **tile)
    rms = one.pow(2).mean().sqrt().item()
    assert (four - one).abs().max().item() <= 1e-4 * rms
    bf = sb.quad_matmul(a, b, **tile)
    assert torch.equal(bf, four.to(torch.bfloat16))
    assert _native.device_status() == 0


def test_quad_raster_does_not_change_the_result():
    import strassen_tpu_b200 as sb
    a = dev_bf16(ref.normal_bf16((2048, 1024), 5))
    b = dev_bf16(ref.normal_bf16((1024, 2048), 6))
    outs = [sb.quad_matmul(a, b, bm=512, bn=512, bk=512, raster=r) for r in (0, 1, 3, 16)]
    for o in outs[1:]:
        assert torch.equal(o, outs[0])


def test_quad_accumulators_reset_between_calls():
    import strassen_tpu_b200 as sb
    a = dev_bf16(ref.normal_bf16((512, 512), 1))
    b = dev_bf16(ref.normal_bf16((512, 512), 2))
    first = sb.quad_matmul(a, b, bm=256, bn=256, bk=256, output_dtype=torch.float32)
    second = sb.quad_matmul(-a, b, bm=256, bn=256, bk=256, output_dtype=torch.float32)
    torch.testing.assert_close(second, -first, rtol=0, atol=0)


def test_quad_validation():
    import strassen_tpu_b200 as sb
    from strassen_tpu_b200 import _native
    a = torch.zeros(256, 256, dtype=torch.bfloat16, device="cuda")
    with pytest.raises(ValueError, match="M % 512"):
        sb.quad_matmul(a, a, bm=256, bn=256, bk=256)
    a = torch.zeros(512, 256, dtype=torch.bfloat16, device="cuda")
    b = torch.zeros(256, 256, dtype=torch.bfloat16, device="cuda")
    with pytest.raises(ValueError, match="workspace"):
        sb.quad_matmul(a, b, bm=256, bn=256, bk=256, workspace=torch.empty(16, dtype=torch.uint8, device="cuda"))
    assert _native.device_status() == 0

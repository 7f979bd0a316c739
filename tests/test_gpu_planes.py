"""Parity of the seven-product-GEMM path (``sb_strassen_gemm_planes``, needs a B200).

The path computes the same seven products as ``sb_strassen_gemm`` (the
reference's strassen_pallas.py:156-880 without an epilogue) from operand planes
formed by two passes, each product a full-width GEMM on CTA pairs, and
recombines them in the one-CTA kernel's fp32 order.  Bar: the parity rule of
test_gpu_parity.assert_parity against the reference's own golden vectors (the
cases its shape rules admit: M % 512, N % 512, K % 128), bit-exact integer
known answers, and agreement with the one-CTA kernel.
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
    m, n = p["shape"]
    return m % 512 == 0 and n % 512 == 0


PLANES_CASES = [c for c in PLAIN if _admitted(c)]


@pytest.mark.parametrize("case", PLANES_CASES)
def test_planes_golden_case(golden, case):
    import strassen_tpu_b200 as sb
    manifest, arrays = golden
    p = manifest[case]
    a, b, extra = make_inputs(p)
    assert not extra
    if a.shape[1] % 128:
        pytest.skip("K not a multiple of 128")
    od = p["kwargs"].get("output_dtype")
    out = sb.planes_matmul(dev_bf16(a), dev_bf16(b), bm=p["bm"], bn=p["bn"], bk=p["bk"],
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
    ((512, 256, 512), (64, 256, 256)),       # one product tile, 32-row blocks
    ((1024, 768, 1024), (256, 512, 256)),    # several K steps, two column tiles
    ((2048, 1024, 1536), (1024, 512, 512)),  # large blocks
])
def test_planes_exact_integer_products(shape, tile):
    import strassen_tpu_b200 as sb
    m, k, n = shape
    a = ref.integers_bf16((m, k), -2, 2, 21)
    b = ref.integers_bf16((k, n), -2, 2, 22)
    got = host(sb.planes_matmul(dev_bf16(a), dev_bf16(b), bm=tile[0], bn=tile[1], bk=tile[2],
                                output_dtype=torch.float32))
    np.testing.assert_array_equal(got, a @ b)


@pytest.mark.parametrize("m, n, k", [(1024, 1536, 2048), (4096, 4096, 4096)])
def test_planes_matches_one_cta_kernel(m, n, k):
    import strassen_tpu_b200 as sb
    from strassen_tpu_b200 import _native
    g = torch.Generator(device="cuda").manual_seed(9)
    a = torch.randn(m, k, device="cuda", generator=g).to(torch.bfloat16)
    b = torch.randn(k, n, device="cuda", generator=g).to(torch.bfloat16)
    tile = dict(bm=1024 if m % 1024 == 0 else 256, bn=512, bk=512)
    # An empty workspace keeps a plain product on the one-CTA kernel.
    one = sb.strassen_matmul(a, b, output_dtype=torch.float32, **tile,
                             workspace=torch.empty(0, dtype=torch.uint8, device="cuda"))
    seven = sb.planes_matmul(a, b, output_dtype=torch.float32, **tile)
    rms = one.pow(2).mean().sqrt().item()
    assert (seven - one).abs().max().item() <= 1e-4 * rms
    bf = sb.planes_matmul(a, b, **tile)
    assert torch.equal(bf, seven.to(torch.bfloat16))
    assert _native.device_status() == 0


def test_planes_raster_and_reuse():
    import strassen_tpu_b200 as sb
    a = dev_bf16(ref.normal_bf16((2048, 1024), 5))
    b = dev_bf16(ref.normal_bf16((1024, 2048), 6))
    outs = [sb.planes_matmul(a, b, bm=512, bn=512, bk=512, raster=r) for r in (0, 1, 3)]
    for o in outs[1:]:
        assert torch.equal(o, outs[0])
    neg = sb.planes_matmul(-a, b, bm=512, bn=512, bk=512)
    assert torch.equal(neg, -outs[0])


def test_planes_validation():
    import strassen_tpu_b200 as sb
    from strassen_tpu_b200 import _native
    a = torch.zeros(256, 256, dtype=torch.bfloat16, device="cuda")
    with pytest.raises(ValueError, match="M % 512"):
        sb.planes_matmul(a, a, bm=256, bn=256, bk=256)
    a = torch.zeros(512, 256, dtype=torch.bfloat16, device="cuda")
    b = torch.zeros(256, 512, dtype=torch.bfloat16, device="cuda")
    with pytest.raises(ValueError, match="workspace"):
        sb.planes_matmul(a, b, bm=256, bn=256, bk=256, workspace=torch.empty(16, dtype=torch.uint8, device="cuda"))
    with pytest.raises(ValueError, match="out must be"):
        sb.planes_matmul(a, b, bm=256, bn=256, bk=256, out=torch.empty(512, 256, dtype=torch.bfloat16, device="cuda"))
    with pytest.raises(ValueError, match="workspace must be a contiguous"):
        sb.planes_matmul(a, b, bm=256, bn=256, bk=256, workspace=torch.empty(16, dtype=torch.uint8))
    # strassen_matmul refuses a workspace the kernels could not write.
    for bad in (torch.empty(16, dtype=torch.uint8), torch.empty(32, dtype=torch.uint8, device="cuda")[::2]):
        with pytest.raises(ValueError, match="workspace must be a contiguous tensor"):
            sb.strassen_matmul(a, b, bm=256, bn=256, bk=256, workspace=bad)
    assert _native.device_status() == 0


@pytest.mark.parametrize("epilogue", ["residual_add", "bias_add", "swiglu", "geglu", "qk_norm_rope",
                                      "norm_residual_add"])
def test_planes_epilogues_match_one_cta_kernel(epilogue):
    """A product on the planes path (large enough, workspace given) applies the
    fused epilogue to the same recombined fp32 values as the one-CTA kernel."""
    import strassen_tpu_b200 as sb
    m, k, n = 8192, 4096, 4096
    g = torch.Generator(device="cuda").manual_seed(11)
    a = torch.randn(m, k, device="cuda", generator=g).to(torch.bfloat16)
    b = (torch.randn(k, n, device="cuda", generator=g) * 0.05).to(torch.bfloat16)
    kw = dict(bm=1024, bn=1024, bk=512, epilogue=epilogue)
    if epilogue == "norm_residual_add":
        # The norm spans the row (bn == n): single pass over the products on
        # the planes path, GEMM + fp32 rows + row pass on the one-CTA kernel.
        kw["bn"] = n
        kw["residual"] = torch.randn(m, n, device="cuda", generator=g).to(torch.bfloat16)
        kw["norm_scale"] = (1 + 0.1 * torch.randn(n, device="cuda", generator=g)).to(torch.bfloat16)
    elif epilogue == "residual_add":
        kw["residual"] = torch.randn(m, n, device="cuda", generator=g).to(torch.bfloat16)
    elif epilogue == "bias_add":
        kw["bias"] = torch.randn(n, device="cuda", generator=g).to(torch.bfloat16)
    elif epilogue == "qk_norm_rope":
        cos = torch.rand(m, 512, device="cuda", generator=g).to(torch.bfloat16)
        sin = torch.rand(m, 512, device="cuda", generator=g).to(torch.bfloat16)  # [M, bn/2]
        scale = (1 + 0.1 * torch.randn(1024, device="cuda", generator=g)).to(torch.bfloat16)
        kw.update(rope_cos=cos, rope_sin=sin, rope_scale=scale, rope_head_dim=128)
    assert sb.workspace_bytes(m, n, k, epilogue) > 0  # the planes path is the default here
    seven = sb.strassen_matmul(a, b, **kw)
    # A workspace below the planes path's keeps the one-CTA kernel (for
    # norm_residual_add: exactly its fp32 rows).
    small = m * n * 4 if epilogue == "norm_residual_add" else 0
    one = sb.strassen_matmul(a, b, **kw, workspace=torch.empty(small, dtype=torch.uint8, device="cuda"))
    torch.cuda.synchronize()
    assert seven.shape == one.shape
    assert_parity(host(seven), host(one), rounding_step=True)


def _capture_and_replay(fn):
    g = torch.cuda.CUDAGraph()
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        with torch.cuda.graph(g):
            out = fn()
    torch.cuda.current_stream().wait_stream(s)
    g.replay()
    torch.cuda.synchronize()
    return out, g


def test_planes_path_in_a_cuda_graph():
    """The two-half schedule (a fork onto the library's side stream and a join)
    captures into a CUDA graph; a host thread that has never run the planes path
    captures the halves in sequence instead.  Both replay the eager result."""
    import threading
    import strassen_tpu_b200 as sb
    m, k, n = 8192, 4096, 4096
    g = torch.Generator(device="cuda").manual_seed(12)
    a = torch.randn(m, k, device="cuda", generator=g).to(torch.bfloat16)
    b = torch.randn(k, n, device="cuda", generator=g).to(torch.bfloat16)
    tile = dict(bm=1024, bn=1024, bk=512)
    want = sb.strassen_matmul(a, b, **tile)
    ws = torch.empty(sb.workspace_bytes(m, n, k), dtype=torch.uint8, device="cuda")
    out, graph = _capture_and_replay(lambda: sb.strassen_matmul(a, b, workspace=ws, **tile))
    assert torch.equal(out, want)
    del graph
    result = {}

    def fresh_thread():
        torch.cuda.set_device(a.device)
        o, gr = _capture_and_replay(lambda: sb.strassen_matmul(a, b, workspace=ws, **tile))
        result["equal"] = torch.equal(o, want)
        del gr

    t = threading.Thread(target=fresh_thread)
    t.start()
    t.join()
    assert result.get("equal") is True

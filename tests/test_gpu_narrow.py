"""Parity of 128-wide tiles (``strassen_matmul(narrow_bn=True)``, needs a B200).

``narrow_bn`` is a B200 extension: the reference's TPU lane rule asks
bn % 256 == 0 (strassen_pallas.py:127-140), which leaves a 128-wide column
shard (one kv head per rank in a tensor-parallel Qwen3 at TP=8) without a
Strassen tile.  The product layout is the reference's tile-local Strassen
(strassen_pallas.py:156-880) at bn = 128, so the oracle run at bn = 128 is the
yardstick: bit-exact integer products, the parity rule of
test_gpu_parity.assert_parity for normal inputs (plain and qk_norm_rope, whose
rule becomes bn % head_dim == 0: each half tile holds one half-head).
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import strassen_ref as ref
from test_gpu_parity import assert_parity, dev_bf16, host

pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(not torch.cuda.is_available(), reason="needs a CUDA device")]


@pytest.mark.parametrize("m, k, n, bm, bk", [
    (512, 512, 128, 256, 256),
    (1024, 1536, 384, 1024, 512),   # three narrow column tiles, three K panels
    (4096, 4096, 128, 1024, 512),   # a Qwen3-8B k/v shard at TP=8, 4096 tokens
])
def test_narrow_plain_matches_oracle(m, k, n, bm, bk):
    import strassen_tpu_b200 as sb
    from strassen_tpu_b200 import _native
    a = ref.normal_bf16((m, k), 31)
    b = ref.normal_bf16((k, n), 32)
    ad, bd = dev_bf16(a), dev_bf16(b)
    got32 = host(sb.strassen_matmul(ad, bd, bm=bm, bn=128, bk=bk, output_dtype=torch.float32, narrow_bn=True))
    got = host(sb.strassen_matmul(ad, bd, bm=bm, bn=128, bk=bk, narrow_bn=True))
    assert _native.device_status() == 0
    want32 = ref.strassen_matmul_ref(a, b, bm=bm, bn=128, bk=bk, output_dtype="float32")
    exact = ref.classical_f64(a, b)
    assert_parity(got32, want32, exact)
    assert_parity(got, ref.bf16_round(want32), exact, rounding_step=True)


def test_narrow_exact_integer_products():
    import strassen_tpu_b200 as sb
    a = ref.integers_bf16((1024, 1024), -2, 2, 41)
    b = ref.integers_bf16((1024, 640), -2, 2, 42)
    got = host(sb.strassen_matmul(dev_bf16(a), dev_bf16(b), bm=512, bn=128, bk=512,
                                  output_dtype=torch.float32, narrow_bn=True))
    np.testing.assert_array_equal(got, a @ b)


@pytest.mark.parametrize("heads", [1, 3])
def test_narrow_qk_norm_rope_matches_oracle(heads):
    import strassen_tpu_b200 as sb
    m, k, hd, bn = 1024, 1024, 128, 128
    a = ref.normal_bf16((m, k), 51)
    w = ref.normal_bf16((k, heads * hd), 52) * np.float32(0.05)
    w = ref.bf16_round(w)
    cos, sin = ref.rope_values(m, hd)
    scale = ref.bf16_round(1.0 + 0.1 * ref.normal_bf16((hd,), 53))
    # One head per 128-wide tile: the rope column layout is the identity here.
    assert np.array_equal(ref.rope_weight_layout(w, bn, hd), w)
    c_l, s_l = ref.rope_layout_tables(cos, sin, bn // 2, hd)
    sc_l = ref.rope_scale_layout(scale, bn, hd)
    kw = dict(epilogue="qk_norm_rope", rope_head_dim=hd)
    got = host(sb.strassen_matmul(dev_bf16(a), dev_bf16(w), bm=512, bn=bn, bk=512, narrow_bn=True,
                                  rope_cos=dev_bf16(c_l), rope_sin=dev_bf16(s_l), rope_scale=dev_bf16(sc_l), **kw))
    want = ref.strassen_matmul_ref(a, w, bm=512, bn=bn, bk=512, rope_cos=c_l, rope_sin=s_l,
                                   rope_scale=sc_l, **kw)
    exact = ref.epilogue_f64(ref.classical_f64(a, w), bm=512, bn=bn, rope_cos=c_l, rope_sin=s_l,
                             rope_scale=sc_l, **kw)
    assert_parity(got, want, exact, rounding_step=True)
    # The same heads through the torch decoder math (RMSNorm per head, rotate-half RoPE).
    from strassen_tpu_b200.qwen3 import apply_rope_torch, rms_norm_torch
    x = torch.from_numpy(ref.classical_f64(a, w).astype(np.float32)).view(m, heads, hd)
    t = apply_rope_torch(rms_norm_torch(x, torch.from_numpy(scale), 1e-6),
                         torch.from_numpy(cos), torch.from_numpy(sin)).float().reshape(m, heads * hd).numpy()
    rms = np.sqrt(np.mean(t.astype(np.float64) ** 2))
    assert np.abs(got - t).max() <= 0.1 * rms

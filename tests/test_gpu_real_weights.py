"""Parity on real Qwen3-0.6B weights (needs a B200).

The weights are the fixture's slices of the reference's pinned layer-0 tensors
(tests/golden/real_weights.*: down_proj^T [1024, 256], q_proj^T heads 0-1
[1024, 256]); the activations are seeded N(0, 1) bf16.  The same parity rule as
the synthetic cases (test_gpu_parity.assert_parity) against the oracle, for the
plain GEMM, the residual_add epilogue of the down projection
(strassen_pallas.py:778-792) and the fused qk_norm_rope of the q projection
(:793-835, with the reference's rope layouts :1315-1378).
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import strassen_ref as ref
from test_gpu_parity import assert_parity, dev_bf16, host
from test_real_weights import load_real_weights

pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(not torch.cuda.is_available(), reason="needs a CUDA device")]

TILE = dict(bm=256, bn=256, bk=256)


def test_down_projection_plain_and_residual():
    import strassen_tpu_b200 as sb
    w, _ = load_real_weights()
    wd = w["down_t"]
    x = ref.normal_bf16((1024, wd.shape[0]), 71)
    res = ref.normal_bf16((1024, wd.shape[1]), 72)
    exact = ref.classical_f64(x, wd)
    got32 = host(sb.strassen_matmul(dev_bf16(x), dev_bf16(wd), output_dtype=torch.float32, **TILE))
    want32 = ref.strassen_matmul_ref(x, wd, output_dtype="float32", **TILE)
    assert_parity(got32, want32, exact)
    got = host(sb.strassen_matmul(dev_bf16(x), dev_bf16(wd), epilogue="residual_add",
                                  residual=dev_bf16(res), **TILE))
    want = ref.strassen_matmul_ref(x, wd, epilogue="residual_add", residual=res, **TILE)
    assert_parity(got, want, exact + res, rounding_step=True)


def test_q_projection_qk_norm_rope():
    import strassen_tpu_b200 as sb
    w, _ = load_real_weights()
    hd = 128
    wq = ref.rope_weight_layout(w["q_t"], 256, hd)
    m = 1024
    x = ref.normal_bf16((m, wq.shape[0]), 73)
    cos, sin = ref.rope_values(m, hd)
    scale = ref.bf16_round(1.0 + 0.02 * ref.normal_bf16((hd,), 74))
    c_l, s_l = ref.rope_layout_tables(cos, sin, 128, hd)
    sc_l = ref.rope_scale_layout(scale, 256, hd)
    kw = dict(epilogue="qk_norm_rope", rope_head_dim=hd, **TILE)
    got = host(sb.strassen_matmul(dev_bf16(x), dev_bf16(wq), rope_cos=dev_bf16(c_l), rope_sin=dev_bf16(s_l),
                                  rope_scale=dev_bf16(sc_l), **kw))
    want = ref.strassen_matmul_ref(x, wq, rope_cos=c_l, rope_sin=s_l, rope_scale=sc_l, **kw)
    exact = ref.epilogue_f64(ref.classical_f64(x, wq), epilogue="qk_norm_rope", bm=256, bn=256,
                             rope_cos=c_l, rope_sin=s_l, rope_scale=sc_l, rope_head_dim=hd)
    assert np.isfinite(got).all()
    assert_parity(got, want, exact, rounding_step=True)

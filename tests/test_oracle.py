"""The CPU oracle, pinned against the reference (no GPU needed).

* Golden vectors: outputs of the reference's own kernel and wrapper
  (strassen_pallas.py) executed on CPU, see tests/golden/make_golden.py.
* Known-answer tests of the reference's test-suite:
  Strassen_MM_Focus/tests/test_kernels_v001.py:59-96 (exact integer products,
  bounded non-zero rounding error) and
  experiments/qwen3/benchmark_cubic_control.py:454-499 (constant sentinel).
"""

from __future__ import annotations

import numpy as np
import pytest

from conftest import golden_output
from golden_inputs import make_inputs
from oracle import strassen_ref as ref


def _run_oracle(p):
    a, b, extra = make_inputs(p)
    return ref.strassen_matmul_ref(a, b, bm=p["bm"], bn=p["bn"], bk=p["bk"], **p["kwargs"], **extra)


def test_golden_manifest_is_complete(golden):
    manifest, arrays = golden
    assert len(manifest) >= 30
    for name in manifest:
        assert name in arrays


def _case_names():
    import json
    from conftest import GOLDEN
    return sorted(json.loads((GOLDEN / "golden_cases.json").read_text())["cases"])


@pytest.mark.parametrize("case", _case_names())
def test_oracle_matches_reference_bit_for_bit(golden, case):
    manifest, arrays = golden
    p = manifest[case]
    got = _run_oracle(p)
    assert list(got.shape) == p["shape"]
    want = golden_output(p, arrays[case])
    np.testing.assert_array_equal(got[::p["row_stride"]], want)


@pytest.mark.parametrize("shape", [(16, 256, 256), (32, 512, 768), (48, 768, 512)])
@pytest.mark.parametrize("interleave", [False, True])
def test_exact_integer_products(shape, interleave):
    # Integers in [-2, 2]: bf16 pre-adds and fp32 products are exact, so a
    # Strassen result must equal a @ b exactly (test_kernels_v001.py:59-80).
    m, k, n = shape
    a = ref.integers_bf16((m, k), -2, 2, 187)
    b = ref.integers_bf16((k, n), -2, 2, 188)
    got = ref.strassen_matmul_ref(a, b, bm=16, bn=256, bk=256, interleave_products=interleave,
                                  output_dtype="float32")
    np.testing.assert_array_equal(got, a @ b)


def test_bounded_nonzero_rounding_error():
    # test_kernels_v001.py:82-96: relative L2 vs fp64 is > 0 and < 0.02.
    rng = np.random.default_rng(23)
    a = ref.bf16_round(rng.normal(size=(16, 256)).astype(np.float32))
    b = ref.bf16_round(rng.normal(size=(256, 256)).astype(np.float32))
    want = ref.classical_f64(a, b)
    got = ref.strassen_matmul_ref(a, b, bm=16, bn=256, bk=256, output_dtype="float32")
    rel = np.linalg.norm(got - want) / np.linalg.norm(want)
    assert 0.0 < rel < 0.02


def test_constant_sentinel():
    # benchmark_cubic_control.py:454-499: A = 0.5, B = -0.25 => C = -K/8 exactly.
    m, k, n = 256, 1024, 512
    a = np.full((m, k), 0.5, np.float32)
    b = np.full((k, n), -0.25, np.float32)
    got = ref.strassen_matmul_ref(a, b, bm=256, bn=256, bk=512)
    assert np.all(got == -k / 8)


def test_bf16_rounding_is_round_to_nearest_even():
    x = np.array([1.0, 1.00390625, 1.005859375, 1.0078125, -3.3, 65504.0, 1e-40], np.float32)
    got = ref.bf16_round(x)
    # 1 + 2^-8 is a tie between 1 and 1 + 2^-7 -> even (1.0); 1 + 1.5*2^-8 rounds up.
    assert got[1] == 1.0 and got[2] == 1.0078125 and got[3] == 1.0078125
    np.testing.assert_array_equal(ref.from_bf16_bits(ref.bf16_bits(got)), got)


def test_layout_helpers_match_reference(golden):
    _, arrays = golden
    import strassen_tpu_b200.layouts as lay
    w = np.arange(4 * 1024, dtype=np.float32).reshape(4, 1024)
    for mod in (lay, ref):
        np.testing.assert_array_equal(mod.swiglu_weight_layout(w, 256), arrays["layout_swiglu_bn256"])
        np.testing.assert_array_equal(mod.swiglu_weight_layout(w, 512), arrays["layout_swiglu_bn512"])
        np.testing.assert_array_equal(mod.rope_weight_layout(w, 256), arrays["layout_rope_weight_bn256"])
        np.testing.assert_array_equal(mod.rope_weight_layout(w, 512, head_dim=64),
                                      arrays["layout_rope_weight_bn512_hd64"])
        tab = np.arange(8 * 128, dtype=np.float32).reshape(8, 128)
        c, s = mod.rope_layout_tables(tab, -tab, 256)
        np.testing.assert_array_equal(c, arrays["layout_rope_cos_hw256"])
        np.testing.assert_array_equal(s, arrays["layout_rope_sin_hw256"])
        np.testing.assert_array_equal(mod.rope_scale_layout(np.arange(128, dtype=np.float32), 512),
                                      arrays["layout_rope_scale_bn512"])


def test_rope_layout_to_heads_inverts_rope_weight_layout():
    import strassen_tpu_b200.layouts as lay
    heads, hd, bn = 8, 128, 512
    flat = np.arange(3 * heads * hd, dtype=np.float32).reshape(3, heads * hd)
    laid = lay.rope_weight_layout(flat, bn)
    back = lay.rope_layout_to_heads(laid, heads, bn)
    np.testing.assert_array_equal(back.reshape(3, heads * hd), flat)


def test_fused_epilogues_match_unfused_math():
    # The fused swiglu/residual epilogues equal the unfused composition applied
    # to the fp32 Strassen accumulators (strassen_pallas.py:762-792).
    a = ref.normal_bf16((256, 512), 5)
    w = ref.normal_bf16((512, 1024), 6)
    pre = ref.strassen_matmul_ref(a, w, bm=256, bn=512, bk=256, output_dtype="float32")
    fused = ref.strassen_matmul_ref(a, w, bm=256, bn=512, bk=256, epilogue="swiglu")
    blocks = pre.reshape(256, 2, 2, 256)
    want = ref.bf16_round((ref.silu(blocks[:, :, 0]) * blocks[:, :, 1]).reshape(256, 512))
    np.testing.assert_array_equal(fused, want)
    res = ref.normal_bf16((256, 1024), 7)
    fused = ref.strassen_matmul_ref(a, w, bm=256, bn=512, bk=256, epilogue="residual_add", residual=res)
    np.testing.assert_array_equal(fused, ref.bf16_round(pre + res))


def test_strassen_error_is_within_twice_native(golden):
    # Statistical anchor (archive/initial-snapshot/evidence/strassen_v5e_multiseed_accuracy.jsonl):
    # Strassen bf16-out rel-L2 vs fp64 is a small multiple of the native error.
    manifest, arrays = golden
    p = manifest["config1_1024_plain"]
    a, b, _ = make_inputs(p)
    exact = ref.classical_f64(a, b)
    strassen = golden_output(p, arrays["config1_1024_plain"])
    native = ref.native_matmul_ref(a, b)
    s = ref.error_stats(strassen, exact[::4])
    nat = ref.error_stats(native, exact)
    assert s["l2_relative"] < 0.01
    assert s["rmse"] <= 4.0 * nat["rmse"]


def test_lhs_transposed_oracle_matches_reference(golden_lhs_t):
    manifest, arrays = golden_lhs_t
    assert len(manifest) >= 3
    for name, c in manifest.items():
        at = ref.normal_bf16((c["k"], c["m"]), c["seed"])
        b = ref.normal_bf16((c["k"], c["n"]), c["seed"] + 1)
        got = ref.strassen_lhs_transposed_ref(at, b, bm=c["bm"], bn=c["bn"], bk=c["bk"],
                                              output_dtype=c["output"] if c["output"] == "float32"
                                              else "bfloat16", **c["kwargs"])
        want = golden_output(c, arrays[name])
        np.testing.assert_array_equal(got[::c["row_stride"]], want, err_msg=name)


def test_row_sampling_reproduces_block_rows():
    """Output row I*bm + r' pairs only with row I*bm + bm/2 + r' (the A quadrant
    split), so running the oracle on just those A rows with bm = 2 * rows gives
    the same values: the basis of the full-size sweep parity tests."""
    m, k, n, bm, bn, bk = 1024, 512, 512, 512, 256, 256
    a = ref.normal_bf16((m, k), 71)
    b = ref.normal_bf16((k, n), 72)
    full = ref.strassen_matmul_ref(a, b, bm=bm, bn=bn, bk=bk, output_dtype="float32")
    rows = np.concatenate([np.arange(base, base + 16) for base in (0, bm // 2, 512, 512 + bm // 2)])
    sub = ref.strassen_matmul_ref(a[rows], b, bm=32, bn=bn, bk=bk, output_dtype="float32")
    np.testing.assert_allclose(sub, full[rows], rtol=1e-6, atol=1e-6)

"""Re-create a golden case's inputs from its recorded recipe (seeded, deterministic).

Mirrors ``tests/golden/make_golden.py::make_inputs`` without importing the
reference or ml_dtypes, so the GPU box (which has no reference checkout) can
rebuild the same inputs bit for bit.
"""

from __future__ import annotations

import numpy as np

from oracle import strassen_ref as ref


def make_inputs(p):
    m, k, n = p["m"], p["k"], p["n"]
    spec = p["inputs"]
    if spec["kind"] == "int":
        a = ref.integers_bf16((m, k), spec["lo"], spec["hi"], spec["seed"])
        b = ref.integers_bf16((k, n), spec["lo"], spec["hi"], spec["seed"] + 1000)
    elif spec["kind"] == "const":
        a = np.full((m, k), 0.5, np.float32)
        b = np.full((k, n), -0.25, np.float32)
    else:
        a = ref.normal_bf16((m, k), spec["seed"])
        b = ref.normal_bf16((k, n), spec["seed"] + 1)
    kw = dict(p["kwargs"])
    extra = {}
    epi = kw.get("epilogue")
    seed = spec["seed"]
    if epi in ("residual_add", "norm_residual_add"):
        extra["residual"] = ref.normal_bf16((m, n), seed + 2)
    if epi == "bias_add":
        extra["bias"] = ref.normal_bf16((n,), seed + 3)
    if epi == "norm_residual_add":
        extra["norm_scale"] = ref.bf16_round(1.0 + 0.02 * ref.normal_bf16((n,), seed + 4))
    if epi == "qk_norm_rope":
        hd = kw.get("rope_head_dim", 128)
        cos, sin = ref.rope_values(m, head_dim=hd)
        c, s = ref.rope_layout_tables(cos, sin, p["bn"] // 2, head_dim=hd)
        extra["rope_cos"], extra["rope_sin"] = c, s
        scale = ref.bf16_round(1.0 + 0.02 * ref.normal_bf16((hd,), seed + 5))
        extra["rope_scale"] = ref.rope_scale_layout(scale, p["bn"], head_dim=hd)
    return a, b, extra

"""CPU oracle for the tile-local one-level Strassen GEMM -- TEST INFRASTRUCTURE ONLY.

This module restates the reference's algorithm (sarsid/strassen-tpu,
``strassen_pallas.py``) in NumPy so the CUDA kernels can be checked against it.
It is imported only by ``tests/``, by ``__graft_entry__.smoke()`` and by the
``cpu_baseline`` / ``--impl reference`` legs of ``bench.py`` -- never by the
product package, which has no CPU path.

Parity status: pinned.  ``tests/golden/`` holds outputs produced by the
reference's own kernel body and operator wrapper (strassen_pallas.py:156-1221,
1315-1411), executed on CPU under a NumPy-backed stand-in for the JAX/Pallas
modules (``tests/golden/make_golden.py``); ``tests/test_oracle.py`` checks this
restatement against them, plus the reference tests' known-answer cases
(Strassen_MM_Focus/tests/test_kernels_v001.py:59-96, exact integer products
and bounded error; experiments/qwen3/benchmark_cubic_control.py:454-499, the
constant-input sentinel C = -K/8).

Number representation: bf16 arrays are carried as float32 arrays whose values
are exactly representable in bf16 (``bf16_round`` is IEEE round-to-nearest-even
on the upper 16 bits).  Arithmetic follows the reference on CPU: bf16 operand
sums rounded once to bf16 (strassen_pallas.py:287, 327-328), bf16 x bf16
products accumulated in fp32 (``jnp.dot(..., preferred_element_type=f32)``),
fp32 quadrant accumulators updated per K panel in the product order the
reference executes (strassen_pallas.py:519-573, 593-712), epilogues in fp32
(strassen_pallas.py:739-879), one RNE rounding on the bf16 store.
"""

from __future__ import annotations

import numpy as np

F32 = np.float32

# ----------------------------------------------------------------- bf16 helpers


def bf16_round(x) -> np.ndarray:
    """Round float32 values to the nearest bf16 (ties to even); returns float32."""
    x = np.ascontiguousarray(np.asarray(x, dtype=F32))
    u = x.view(np.uint32).astype(np.uint64)
    r = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16) << 16
    out = r.astype(np.uint32).view(F32).reshape(x.shape)
    nan = np.isnan(x)
    if nan.any():
        out = out.copy()
        out[nan] = np.float32(np.nan)
    return out


def bf16_bits(x) -> np.ndarray:
    """uint16 bit patterns of bf16-representable float32 values."""
    x = np.ascontiguousarray(bf16_round(x))
    return (x.view(np.uint32) >> 16).astype(np.uint16)


def from_bf16_bits(bits) -> np.ndarray:
    """float32 values of uint16 bf16 bit patterns."""
    b = np.asarray(bits, dtype=np.uint16).astype(np.uint32) << 16
    return b.view(F32)


# ------------------------------------------------------------ product schedule
# strassen_pallas.py:324-379.  Each product: (A terms, B terms, quadrant updates);
# a term is (quadrant index, sign); an update is (output quadrant, sign).
PRODUCTS = {
    1: (((0, 1), (3, 1)), ((0, 1), (3, 1)), ((0, 1), (3, 1))),
    2: (((2, 1), (3, 1)), ((0, 1),), ((2, 1), (3, -1))),
    3: (((0, 1),), ((1, 1), (3, -1)), ((1, 1), (3, 1))),
    4: (((3, 1),), ((2, 1), (0, -1)), ((0, 1), (2, 1))),
    5: (((0, 1), (1, 1)), ((3, 1),), ((0, -1), (1, 1))),
    6: (((2, 1), (0, -1)), ((0, 1), (1, 1)), ((3, 1),)),
    7: (((1, 1), (3, -1)), ((2, 1), (3, 1)), ((0, 1),)),
}
PLAIN_ORDER = (1, 2, 3, 4, 5, 6, 7)                   # strassen_pallas.py:566-573
INTERLEAVED_ORDER = (4, 6, 5, 2, 7, 3, 1)             # strassen_pallas.py:556-565
PRODUCT_AWARE_SWIGLU_FINAL = (4, 5, 7, 3, 1, 6, 2)    # strassen_pallas.py:621-635
PRODUCT_AWARE_RESIDUAL_FINAL = (4, 6, 5, 2, 7, 3, 1)  # strassen_pallas.py:671-682

# The dual rank-7 formula Q1..Q7 (strassen_pallas.py:466-517), same layout as PRODUCTS.
DUAL_PRODUCTS = {
    1: (((0, 1), (3, 1)), ((0, 1), (3, 1)), ((0, 1), (3, 1))),
    2: (((0, 1),), ((1, 1), (3, 1)), ((1, 1), (3, -1))),
    3: (((2, 1), (3, -1)), ((0, 1),), ((2, 1), (3, 1))),
    4: (((1, 1), (0, -1)), ((3, 1),), ((0, 1), (1, 1))),
    5: (((3, 1),), ((0, 1), (2, 1)), ((0, -1), (2, 1))),
    6: (((0, 1), (2, 1)), ((1, 1), (0, -1)), ((3, 1),)),
    7: (((1, 1), (3, 1)), ((2, 1), (3, -1)), ((0, 1),)),
}
DUAL_PLAIN_ORDER = (1, 2, 3, 4, 5, 6, 7)              # strassen_pallas.py:549-556
DUAL_INTERLEAVED_ORDER = (5, 6, 4, 3, 7, 2, 1)        # strassen_pallas.py:540-548
# Exact eight-product panel (strassen_pallas.py:575-586): (output quadrant, A quadrant, B quadrant).
EXACT_PANEL = ((0, 0, 0), (1, 0, 1), (2, 2, 0), (3, 2, 1), (0, 1, 2), (1, 1, 3), (2, 3, 2), (3, 3, 3))


def _operand(quads, terms):
    """bf16 operand for a product: one quadrant, or a sum rounded once to bf16."""
    (q0, s0), *rest = terms
    if not rest:
        return quads[q0]
    (q1, s1), = rest
    return bf16_round(quads[q0] + (quads[q1] if s1 > 0 else -quads[q1]))


def _split_a(a, bm, bk):
    m, k = a.shape
    hm, hk = bm // 2, bk // 2
    blocks = a.reshape(m // bm, 2, hm, k // bk, 2, hk).transpose(0, 3, 1, 4, 2, 5)
    # [I, P, qr, qk, hm, hk] -> quadrant q = 2*qr + qk (strassen_pallas.py:188-193)
    return [np.ascontiguousarray(blocks[:, :, q // 2, q % 2]) for q in range(4)]


def _split_b(b, bk, bn):
    k, n = b.shape
    hk, hn = bk // 2, bn // 2
    blocks = b.reshape(k // bk, 2, hk, n // bn, 2, hn).transpose(0, 3, 1, 4, 2, 5)
    # [P, J, qk, qc, hk, hn] -> quadrant q = 2*qk + qc (strassen_pallas.py:194-199)
    return [np.ascontiguousarray(blocks[:, :, q // 2, q % 2]) for q in range(4)]


def _permuted(index_row, index_col, swap_rows, swap_cols):
    """strassen_pallas.py:210-211: quadrant index after swapping block halves."""
    return 2 * (index_row ^ swap_rows) + (index_col ^ swap_cols)


# The power-of-two formula R1..R7 (strassen_pallas.py:381-464).  Every bf16
# operation rounds, in the reference's order; x*0.5 and x*0.25 are exact.
def _h(x):
    return bf16_round(x * F32(0.5))


def _q(x):
    return bf16_round(x * F32(0.25))


def _sub(x, y):
    return bf16_round(x - y)


def _add(x, y):
    return bf16_round(x + y)


POWERS_A = {
    1: lambda a: _sub(a[2], a[1]),
    2: lambda a: _add(_sub(a[0], _h(a[2])), _sub(_h(a[1]), _q(a[3]))),
    3: lambda a: _sub(a[2], _h(a[3])),
    4: lambda a: _sub(a[1], _h(a[3])),
    5: lambda a: _add(a[2], _h(a[3])),
    6: lambda a: _add(_sub(a[0], _h(a[1])), _sub(_h(a[2]), _q(a[3]))),
    7: lambda a: _add(a[1], _h(a[3])),
}
POWERS_B = {
    1: lambda b: _sub(b[0], b[3]),
    2: lambda b: _add(b[0], _h(b[1])),
    3: lambda b: _sub(_h(b[1]), b[3]),
    4: lambda b: _add(_sub(_h(b[0]), b[2]), _sub(_q(b[1]), _h(b[3]))),
    5: lambda b: _add(_h(b[1]), b[3]),
    6: lambda b: _sub(b[0], _h(b[1])),
    7: lambda b: _sub(_add(_h(b[0]), b[2]), _add(_q(b[1]), _h(b[3]))),
}
# Basis updates z0..z3 (not permuted; strassen_pallas.py:398-464).
POWERS_UPDATES = {1: ((3, 1),), 2: ((2, 1),), 3: ((0, 1), (3, -1)), 4: ((2, -1), (3, 1)),
                  5: ((0, 1),), 6: ((1, 1),), 7: ((1, 1), (3, 1))}
POWERS_PLAIN_ORDER = (1, 2, 3, 4, 5, 6, 7)            # strassen_pallas.py:530-537
POWERS_INTERLEAVED_ORDER = (3, 2, 6, 5, 4, 7, 1)      # strassen_pallas.py:520-528


def powers_decode(z):
    """Output quadrants from the sparse basis z0..z3 (strassen_pallas.py:744-761)."""
    z0, z1, z2, z3 = z
    c3 = z0
    c2 = z3 + z0 * F32(0.5)
    c0 = (z1 + z2) * F32(0.5) + z0 * F32(0.25)
    c1 = ((z2 - z1) + z3) + z0 * F32(0.5)
    return [c0.astype(F32), c1.astype(F32), c2.astype(F32), c3.astype(F32)]


def strassen_accumulators(a, b, bm, bn, bk, *, interleave_products=False,
                          final_order=None, formula_variant="classical", block_permutation=0,
                          exact_panels=()):
    """fp32 quadrant accumulators acc[q][I, J, r, c] after all K panels.

    a, b: float32 arrays of bf16 values.  Reproduces the reference's per-panel
    accumulation (strassen_pallas.py:234-266, 519-573): at every panel P the
    products run in order and each updates its one or two quadrant
    accumulators.  ``final_order`` overrides the order on the last panel (the
    product-aware schedules).  ``formula_variant`` "classical" or "dual";
    ``block_permutation`` swaps M/K/N block halves before the formula and maps
    the quadrants back (strassen_pallas.py:205-226); panels in ``exact_panels``
    run the exact eight-product update instead (strassen_pallas.py:575-586).
    """
    a = np.asarray(a, F32)
    b = np.asarray(b, F32)
    aq = _split_a(a, bm, bk)   # each [nI, nP, hm, hk]
    bq = _split_b(b, bk, bn)   # each [nP, nJ, hk, hn]
    swap_m, swap_k, swap_n = (block_permutation & 1), (block_permutation >> 1) & 1, (block_permutation >> 2) & 1
    aq = [aq[_permuted(r, c, swap_m, swap_k)] for r in range(2) for c in range(2)]
    bq = [bq[_permuted(r, c, swap_k, swap_n)] for r in range(2) for c in range(2)]
    out_index = [_permuted(r, c, swap_m, swap_n) for r in range(2) for c in range(2)]
    n_i, n_p = aq[0].shape[:2]
    n_j = bq[0].shape[1]
    hm, hn = bm // 2, bn // 2
    if formula_variant == "powers":
        if exact_panels:
            raise NotImplementedError("exact panels need a quadrant-basis formula")
        order = POWERS_INTERLEAVED_ORDER if interleave_products else POWERS_PLAIN_ORDER
        z = [np.zeros((n_i, n_j, hm, hn), F32) for _ in range(4)]
        for p in range(n_p):
            ap = [x[:, p] for x in aq]
            bp = [x[p] for x in bq]
            for idx in order:
                prod = np.matmul(POWERS_A[idx](ap)[:, None], POWERS_B[idx](bp)[None]).astype(F32)
                for q, sign in POWERS_UPDATES[idx]:
                    if sign > 0:
                        z[q] += prod
                    else:
                        z[q] -= prod
        decoded = powers_decode(z)
        acc = [None] * 4
        for q in range(4):
            acc[out_index[q]] = decoded[q]
        return acc
    if formula_variant == "classical":
        table, order = PRODUCTS, (INTERLEAVED_ORDER if interleave_products else PLAIN_ORDER)
    elif formula_variant == "dual":
        table, order = DUAL_PRODUCTS, (DUAL_INTERLEAVED_ORDER if interleave_products else DUAL_PLAIN_ORDER)
    else:
        raise NotImplementedError(formula_variant)
    exact = set(int(x) for x in exact_panels)
    acc = [np.zeros((n_i, n_j, hm, hn), F32) for _ in range(4)]
    for p in range(n_p):
        ap = [x[:, p] for x in aq]         # [nI, hm, hk]
        bp = [x[p] for x in bq]            # [nJ, hk, hn]
        if p in exact:
            for q, ia, ib in EXACT_PANEL:
                acc[out_index[q]] += np.matmul(ap[ia][:, None], bp[ib][None]).astype(F32)
            continue
        this_order = final_order if (final_order is not None and p == n_p - 1) else order
        for idx in this_order:
            a_terms, b_terms, updates = table[idx]
            sa = _operand(ap, a_terms)
            sb = _operand(bp, b_terms)
            prod = np.matmul(sa[:, None], sb[None]).astype(F32)  # [nI, nJ, hm, hn]
            for q, sign in updates:
                if sign > 0:
                    acc[out_index[q]] += prod
                else:
                    acc[out_index[q]] -= prod
    return acc


def _assemble(acc, m, n, bm, bn):
    """Place quadrant accumulators [I, J, r, c] back into an [m, n] array."""
    hm, hn = bm // 2, bn // 2
    n_i, n_j = m // bm, n // bn
    out = np.empty((n_i, 2, hm, n_j, 2, hn), F32)
    for q in range(4):
        out[:, q // 2, :, :, q % 2, :] = acc[q].transpose(0, 2, 1, 3)
    return out.reshape(m, n)


def _assemble_half(top, bottom, m, bm, hn, n_j):
    """Gated epilogue output [m, n/2]: rows :hm from `top`, hm: from `bottom`."""
    hm = bm // 2
    n_i = m // bm
    out = np.empty((n_i, 2, hm, n_j, hn), F32)
    out[:, 0] = top.transpose(0, 2, 1, 3)
    out[:, 1] = bottom.transpose(0, 2, 1, 3)
    return out.reshape(m, n_j * hn)


def silu(x):
    """jax.nn.silu in fp32: x * logistic(x)."""
    x = np.asarray(x, F32)
    with np.errstate(over="ignore"):
        return (x * (F32(1) / (F32(1) + np.exp(-x)))).astype(F32)


def gelu_tanh(x):
    """jax.nn.gelu(approximate=True) in fp32."""
    x = np.asarray(x, F32)
    c = F32(np.sqrt(2.0 / np.pi))
    cdf = F32(0.5) * (F32(1) + np.tanh(c * (x + F32(0.044715) * (x ** 3))))
    return (x * cdf).astype(F32)


def rsqrt(x):
    x = np.asarray(x, F32)
    return (F32(1) / np.sqrt(x)).astype(F32)


def strassen_matmul_ref(a, b, *, bm, bn, bk, interleave_products=False, epilogue=None,
                        residual=None, bias=None, rope_cos=None, rope_sin=None, rope_scale=None,
                        rope_head_dim=128, rope_eps=1e-6, norm_scale=None, norm_eps=1e-6,
                        output_dtype="bfloat16", product_aware_swiglu=False,
                        product_aware_residual=False, formula_variant="classical",
                        block_permutation=0, classical_panels=(), panel_schedule=None):
    """Restatement of strassen_pallas.strassen_matmul for bf16 inputs.

    Returns a float32 array; for a bf16 output its values are bf16-rounded.
    Shapes follow the reference: [m, n], or [m, n/2] for swiglu/geglu.
    """
    a = bf16_round(a)
    b = bf16_round(b)
    m, k = a.shape
    _, n = b.shape
    for name, dim, blk in (("M", m, bm), ("N", n, bn), ("K", k, bk)):
        if dim % blk:
            raise ValueError(f"{name}={dim} is not divisible by {blk}")
    final = None
    if product_aware_swiglu:
        final = PRODUCT_AWARE_SWIGLU_FINAL
    elif product_aware_residual:
        final = PRODUCT_AWARE_RESIDUAL_FINAL
    exact = tuple(classical_panels)
    if panel_schedule is not None:
        exact = tuple(i for i, v in enumerate(np.asarray(panel_schedule).reshape(-1)) if v != 0)
    acc = strassen_accumulators(a, b, bm, bn, bk, interleave_products=interleave_products,
                                final_order=final, formula_variant=formula_variant,
                                block_permutation=block_permutation, exact_panels=exact)
    hm, hn = bm // 2, bn // 2
    n_i, n_j = m // bm, n // bn
    if epilogue is None:
        out = _assemble(acc, m, n, bm, bn)
        return out if output_dtype in ("float32", np.float32) else bf16_round(out)
    if epilogue in ("swiglu", "geglu"):  # strassen_pallas.py:762-777
        act = silu if epilogue == "swiglu" else gelu_tanh
        top = act(acc[0]) * acc[1]
        bottom = act(acc[2]) * acc[3]
        return bf16_round(_assemble_half(top, bottom, m, bm, hn, n_j))
    if epilogue == "residual_add":  # strassen_pallas.py:778-792
        pre = _assemble(acc, m, n, bm, bn)
        return bf16_round(pre + np.asarray(residual, F32))
    if epilogue == "bias_add":  # strassen_pallas.py:867-874
        pre = _assemble(acc, m, n, bm, bn)
        return bf16_round(pre + np.asarray(bias, F32)[None, :])
    if epilogue == "qk_norm_rope":  # strassen_pallas.py:793-835
        scale = np.asarray(rope_scale, F32)
        scale_a, scale_b = scale[:hn], scale[hn:]
        cos = np.asarray(rope_cos, F32).reshape(n_i, 2, hm, hn)
        sin = np.asarray(rope_sin, F32).reshape(n_i, 2, hm, hn)
        seg_width = rope_head_dim // 2
        inv = F32(1.0 / rope_head_dim)
        eps = F32(rope_eps)
        # Segment sums through a 0/1 matrix padded to 128 lanes, per tile, as
        # the reference does (strassen_pallas.py:1180-1197, 817-823).
        cols = np.arange(hn)
        segment = np.zeros((hn, 128), F32)
        segment[cols, cols // seg_width] = 1.0
        segment_t = np.ascontiguousarray(segment.T)

        def rotate(first, second, c, s):
            sums = np.dot(first * first, segment).astype(F32) + np.dot(second * second, segment).astype(F32)
            recip = np.dot(rsqrt(sums * inv + eps), segment_t).astype(F32)
            na = first * recip * scale_a
            nb = second * recip * scale_b
            return na * c - nb * s, nb * c + na * s

        quads = [np.empty_like(acc[0]) for _ in range(4)]
        with np.errstate(divide="ignore", over="ignore", invalid="ignore"):
            for i in range(n_i):
                for j in range(n_j):
                    for half in range(2):
                        first, second = acc[2 * half][i, j], acc[2 * half + 1][i, j]
                        oa, ob = rotate(first, second, cos[i, half], sin[i, half])
                        quads[2 * half][i, j] = oa
                        quads[2 * half + 1][i, j] = ob
        return bf16_round(_assemble(quads, m, n, bm, bn))
    if epilogue == "norm_residual_add":  # strassen_pallas.py:836-866
        if bn != n:
            raise ValueError("norm_residual_add needs bn == n")
        pre = _assemble(acc, m, n, bm, bn)
        left, right = pre[:, :hn], pre[:, hn:]
        squares = (left * left).sum(1, keepdims=True, dtype=F32) + \
            (right * right).sum(1, keepdims=True, dtype=F32)
        recip = rsqrt(squares * F32(1.0 / n) + F32(norm_eps))
        scale = np.asarray(norm_scale, F32)
        res = np.asarray(residual, F32)
        out = np.concatenate([left * recip * scale[:hn] + res[:, :hn],
                              right * recip * scale[hn:] + res[:, hn:]], axis=1)
        return bf16_round(out)
    raise ValueError(f"unknown epilogue {epilogue!r}")


def strassen_lhs_transposed_ref(at, b, *, bm, bn, bk, interleave_products=False,
                                output_dtype="bfloat16"):
    """Restatement of strassen_matmul_lhs_transposed (strassen_pallas.py:1224-1312).

    ``at`` is stored (K, M); the reference transposes each (bk, bm) tile in VMEM
    before the ordinary kernel, which equals the tile-local Strassen product of
    at.T and b.
    """
    return strassen_matmul_ref(np.asarray(at).T, b, bm=bm, bn=bn, bk=bk,
                               interleave_products=interleave_products, output_dtype=output_dtype)


# ------------------------------------------------------------- classical arms


def classical_f64(a, b) -> np.ndarray:
    """Exact-ish classical product in float64 (the error yardstick)."""
    return np.asarray(a, np.float64) @ np.asarray(b, np.float64)


def native_matmul_ref(a, b) -> np.ndarray:
    """strassen_pallas.native_matmul (strassen_pallas.py:1414-1421): fp32 acc, bf16 out."""
    return bf16_round(np.asarray(a, F32) @ np.asarray(b, F32))


def epilogue_f64(pre, *, epilogue=None, residual=None, bias=None, rope_cos=None, rope_sin=None,
                 rope_scale=None, rope_head_dim=128, rope_eps=1e-6, norm_scale=None,
                 norm_eps=1e-6, bm=None, bn=None):
    """The same epilogue applied in float64 to a float64 product (error yardstick)."""
    pre = np.asarray(pre, np.float64)
    m, n = pre.shape
    if epilogue is None:
        return pre
    hn = bn // 2
    if epilogue in ("swiglu", "geglu"):
        blocks = pre.reshape(m, n // bn, 2, hn)
        gate, up = blocks[:, :, 0], blocks[:, :, 1]
        if epilogue == "swiglu":
            act = gate / (1.0 + np.exp(-gate))
        else:
            act = 0.5 * gate * (1.0 + np.tanh(np.sqrt(2 / np.pi) * (gate + 0.044715 * gate ** 3)))
        return (act * up).reshape(m, n // 2)
    if epilogue == "residual_add":
        return pre + np.asarray(residual, np.float64)
    if epilogue == "bias_add":
        return pre + np.asarray(bias, np.float64)[None]
    if epilogue == "qk_norm_rope":
        seg = rope_head_dim // 2
        blocks = pre.reshape(m, n // bn, 2, hn)
        first, second = blocks[:, :, 0], blocks[:, :, 1]
        ss = (first ** 2).reshape(m, n // bn, hn // seg, seg).sum(-1) + \
            (second ** 2).reshape(m, n // bn, hn // seg, seg).sum(-1)
        recip = np.repeat(1.0 / np.sqrt(ss / rope_head_dim + rope_eps), seg, axis=-1)
        scale = np.asarray(rope_scale, np.float64)
        na = first * recip * scale[:hn]
        nb = second * recip * scale[hn:]
        c = np.asarray(rope_cos, np.float64)[:, None]
        s = np.asarray(rope_sin, np.float64)[:, None]
        out = np.stack([na * c - nb * s, nb * c + na * s], axis=2)
        return out.reshape(m, n)
    if epilogue == "norm_residual_add":
        recip = 1.0 / np.sqrt((pre ** 2).mean(1, keepdims=True) + norm_eps)
        return pre * recip * np.asarray(norm_scale, np.float64)[None] + np.asarray(residual, np.float64)
    raise ValueError(epilogue)


# -------------------------------------------------- layouts (strassen_pallas.py)


def swiglu_weight_layout(gate_up, bn):
    """strassen_pallas.py:1381-1411."""
    two_i = gate_up.shape[1]
    inter, half = two_i // 2, bn // 2
    order = []
    for block in range(inter // half):
        s = block * half
        order.extend(range(s, s + half))
        order.extend(range(inter + s, inter + s + half))
    return np.asarray(gate_up)[:, order]


def rope_weight_layout(weight, bn, head_dim=128):
    """strassen_pallas.py:1315-1349."""
    n = weight.shape[1]
    hh, heads, half = head_dim // 2, n // head_dim, bn // 2
    a_cols = [h * head_dim + j for h in range(heads) for j in range(hh)]
    b_cols = [h * head_dim + hh + j for h in range(heads) for j in range(hh)]
    order = []
    for block in range((n // 2) // half):
        lo, hi = block * half, (block + 1) * half
        order.extend(a_cols[lo:hi])
        order.extend(b_cols[lo:hi])
    return np.asarray(weight)[:, order]


def rope_layout_tables(cos, sin, half_width, head_dim=128):
    """strassen_pallas.py:1352-1368."""
    hh = head_dim // 2
    reps = half_width // hh
    return np.tile(np.asarray(cos)[:, :hh], (1, reps)), np.tile(np.asarray(sin)[:, :hh], (1, reps))


def rope_scale_layout(scale, bn, head_dim=128):
    """strassen_pallas.py:1371-1378."""
    hh = head_dim // 2
    reps = (bn // 2) // hh
    scale = np.asarray(scale)
    return np.concatenate((np.tile(scale[:hh], reps), np.tile(scale[hh:], reps)))


def rope_values(positions, head_dim=128, theta=1e6):
    """bf16 cos/sin tables [positions, head_dim] (benchmark_qwen3_32b_layer.py:258-267)."""
    pos = np.arange(positions, dtype=F32)[:, None]
    inv = (F32(1.0) / (F32(theta) ** (np.arange(0, head_dim, 2, dtype=F32) / F32(head_dim)))).astype(F32)
    ang = np.concatenate([pos * inv[None]] * 2, axis=-1).astype(F32)
    return bf16_round(np.cos(ang)), bf16_round(np.sin(ang))


def rms_norm_ref(x, scale, eps=1e-6):
    """benchmark_qwen3_32b_layer.py:270-276: bf16(x * rsqrt(mean(x^2) + eps) * scale)."""
    x = np.asarray(x, F32)
    r = rsqrt((x * x).mean(-1, keepdims=True, dtype=F32) + F32(eps))
    return bf16_round(x * r * np.asarray(scale, F32))


# ------------------------------------------------------------ seeded inputs


def normal_bf16(shape, seed):
    """Seeded N(0,1) input rounded to bf16 (BASELINE's synthetic-input recipe)."""
    rng = np.random.default_rng(seed)
    return bf16_round(rng.standard_normal(shape).astype(F32))


def integers_bf16(shape, lo, hi, seed):
    """Seeded integers in [lo, hi] as bf16 (the reference KAT recipe)."""
    rng = np.random.default_rng(seed)
    return rng.integers(lo, hi + 1, size=shape).astype(F32)


def error_stats(got, ref) -> dict:
    """The reference's accuracy vocabulary (experiments/qwen3/benchmark_common.py:27-60)."""
    got = np.asarray(got, np.float64)
    ref = np.asarray(ref, np.float64)
    diff = got - ref
    ref_norm = np.linalg.norm(ref)
    ref_max = np.abs(ref).max() if ref.size else 0.0
    return {
        "max_abs": float(np.abs(diff).max()) if diff.size else 0.0,
        "rmse": float(np.sqrt(np.mean(diff ** 2))) if diff.size else 0.0,
        "rms_ref": float(np.sqrt(np.mean(ref ** 2))) if ref.size else 0.0,
        "maxnorm_relative": float(np.abs(diff).max() / ref_max) if ref_max else 0.0,
        "l2_relative": float(np.linalg.norm(diff) / ref_norm) if ref_norm else 0.0,
    }

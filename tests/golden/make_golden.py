"""Generate golden vectors from the reference's own Strassen path.

JAX is not installable in this container, so the reference module
``strassen_pallas`` (sarsid/strassen-tpu) is imported under a small NumPy-backed
stand-in for the parts of ``jax`` / ``jax.numpy`` / ``jax.experimental.pallas``
it touches.  ``pallas_call`` is interpreted the way Pallas' own interpret mode
runs a grid: programs in row-major grid order (K steps innermost), each given
views of its input blocks, a view of its output block (which persists across
the K steps of one output tile) and scratch buffers allocated once per call.
Every line of the kernel body, the product schedules, the epilogues, the
operand wiring and the layout helpers therefore comes from the reference
itself; only the array library underneath is NumPy + ml_dtypes (bf16 arithmetic
upcasts to fp32 and rounds to nearest-even, the same contract as XLA's CPU
backend; dots accumulate in fp32).

Usage (needs the reference checkout and ml_dtypes; run in the build container):

    python tests/golden/make_golden.py --reference <path of the reference checkout>

Writes ``tests/golden/golden_cases.json`` (case parameters and input recipes)
and ``tests/golden/golden_outputs.npz`` (reference outputs as bf16 bit patterns
or float32).  Inputs are regenerated from their seeds by ``oracle.strassen_ref``
helpers, so the fixtures stay small.
"""

from __future__ import annotations

import argparse
import enum
import functools
import json
import sys
import types
from pathlib import Path

import ml_dtypes
import numpy as np

HERE = Path(__file__).resolve().parent
REPO = HERE.parent.parent
sys.path.insert(0, str(REPO))
sys.path.insert(0, str(REPO / "tests"))
from oracle import strassen_ref as ref  # noqa: E402  (seeded input recipes only)

BF16 = np.dtype(ml_dtypes.bfloat16)


# --------------------------------------------------------------- the stand-in
class _AtIndexer:
    def __init__(self, arr):
        self._arr = arr

    def __getitem__(self, idx):
        arr = self._arr

        class _Setter:
            def set(self, value):
                out = np.array(arr, copy=True)
                out[idx] = value
                return out

        return _Setter()


class _Array(np.ndarray):
    """ndarray with the functional ``.at[...].set(...)`` update JAX code uses."""

    @property
    def at(self):
        return _AtIndexer(np.asarray(self))


def _dtype(d):
    if d is None:
        return None
    return np.dtype(d)


def _asarray(x, dtype=None):
    return np.asarray(x).astype(_dtype(dtype)) if dtype is not None else np.asarray(x)


def _zeros(shape, dtype=np.float32):
    return np.zeros(shape, _dtype(dtype)).view(_Array)


def _dot(x, y, preferred_element_type=None, precision=None):
    out_t = _dtype(preferred_element_type) or np.result_type(x, y)
    return np.dot(np.asarray(x, np.float32), np.asarray(y, np.float32)).astype(out_t)


def _silu(x):
    x = np.asarray(x)
    one = np.asarray(1, x.dtype)
    with np.errstate(over="ignore"):
        return x * (one / (one + np.exp(-x)))


def _gelu(x, approximate=True):
    x = np.asarray(x)
    c = np.asarray(np.sqrt(2.0 / np.pi), x.dtype)
    cdf = np.asarray(0.5, x.dtype) * (np.asarray(1, x.dtype) + np.tanh(
        c * (x + np.asarray(0.044715, x.dtype) * (x ** 3))))
    return x * cdf


def _rsqrt(x):
    x = np.asarray(x)
    return np.asarray(1, x.dtype) / np.sqrt(x)


class _Precision(enum.Enum):
    DEFAULT = 0
    HIGH = 1
    HIGHEST = 2


class _ShapeDtypeStruct:
    def __init__(self, shape, dtype):
        self.shape = tuple(shape)
        self.dtype = _dtype(dtype)


class _BlockSpec:
    def __init__(self, block_shape, index_map):
        self.block_shape = tuple(block_shape)
        self.index_map = index_map


class _VMEM:
    def __init__(self, shape, dtype):
        self.shape = tuple(shape)
        self.dtype = _dtype(dtype)


class _CompilerParams:
    def __init__(self, **kwargs):
        self.kwargs = kwargs


class _PrefetchScalarGridSpec:
    def __init__(self, num_scalar_prefetch, grid, in_specs, out_specs, scratch_shapes=()):
        self.num_scalar_prefetch = num_scalar_prefetch
        self.grid = grid
        self.in_specs = in_specs
        self.out_specs = out_specs
        self.scratch_shapes = scratch_shapes


_GRID_STATE = {"ids": ()}


def _program_id(axis):
    return _GRID_STATE["ids"][axis]


def _when(cond):
    def deco(fn):
        if bool(cond):
            fn()
        return fn
    return deco


def _pallas_call(kernel, *, grid=None, grid_spec=None, in_specs=None, out_specs=None,
                 out_shape=None, scratch_shapes=(), compiler_params=None, interpret=False,
                 **_unused):
    n_prefetch = 0
    if grid_spec is not None:
        # Scalar-prefetch grid: the first operands are passed whole to the kernel
        # and appended to every index map's arguments.
        n_prefetch = grid_spec.num_scalar_prefetch
        grid, in_specs = grid_spec.grid, grid_spec.in_specs
        out_specs, scratch_shapes = grid_spec.out_specs, grid_spec.scratch_shapes

    def run(*operands):
        out = np.zeros(out_shape.shape, out_shape.dtype)
        scratch = [np.zeros(s.shape, s.dtype) for s in scratch_shapes]
        prefetch = [np.asarray(x) for x in operands[:n_prefetch]]
        tensors = operands[n_prefetch:]

        def block(array, spec, ids):
            idx = spec.index_map(*ids, *prefetch)
            return array[tuple(slice(i * s, (i + 1) * s) for i, s in zip(idx, spec.block_shape))]

        for ids in np.ndindex(*grid):
            _GRID_STATE["ids"] = ids
            in_refs = [block(np.asarray(x), spec, ids) for x, spec in zip(tensors, in_specs)]
            kernel(*prefetch, *in_refs, block(out, out_specs, ids), *scratch)
        return out

    return run


def install_stand_in():
    jax = types.ModuleType("jax")
    jax.__version__ = "0.0-numpy-stand-in"
    jnp = types.ModuleType("jax.numpy")
    for name in ("bfloat16",):
        setattr(jnp, name, ml_dtypes.bfloat16)
    jnp.float32 = np.float32
    jnp.int32 = np.int32
    jnp.asarray = _asarray
    jnp.dtype = np.dtype
    jnp.asarray = _asarray
    jnp.zeros = _zeros
    jnp.dot = _dot
    jnp.arange = np.arange
    jnp.tile = np.tile
    jnp.concatenate = np.concatenate
    jnp.sum = np.sum
    jnp.matmul = lambda a, b, precision=None, preferred_element_type=None: _dot(
        a, b, preferred_element_type=preferred_element_type)
    jnp.logical_and = np.logical_and
    jnp.logical_or = np.logical_or
    jnp.logical_not = np.logical_not
    jnp.swapaxes = np.swapaxes
    lax = types.ModuleType("jax.lax")
    lax.Precision = _Precision
    lax.rsqrt = _rsqrt
    nn = types.ModuleType("jax.nn")
    nn.silu = _silu
    nn.gelu = _gelu
    jax.numpy = jnp
    jax.lax = lax
    jax.nn = nn
    jax.ShapeDtypeStruct = _ShapeDtypeStruct
    jax.default_backend = lambda: "cpu"
    experimental = types.ModuleType("jax.experimental")
    pallas = types.ModuleType("jax.experimental.pallas")
    pallas.program_id = _program_id
    pallas.when = _when
    pallas.pallas_call = _pallas_call
    pallas.BlockSpec = _BlockSpec
    tpu = types.ModuleType("jax.experimental.pallas.tpu")
    tpu.VMEM = _VMEM
    tpu.CompilerParams = _CompilerParams
    tpu.PrefetchScalarGridSpec = _PrefetchScalarGridSpec
    pallas.tpu = tpu
    experimental.pallas = pallas
    jax.experimental = experimental
    sys.modules.update({
        "jax": jax, "jax.numpy": jnp, "jax.lax": lax, "jax.nn": nn,
        "jax.experimental": experimental, "jax.experimental.pallas": pallas,
        "jax.experimental.pallas.tpu": tpu,
    })


def import_reference(reference_root: Path):
    install_stand_in()
    sys.dont_write_bytecode = True  # the reference checkout is read-only
    sys.path.insert(0, str(reference_root))
    import strassen_pallas  # noqa: E402  (the reference module itself)
    return strassen_pallas


# ------------------------------------------------------------------- cases
def cases():
    """(name, parameters).  Input recipes are re-created by the tests from seeds."""
    out = []

    def gemm(name, m, k, n, tile, *, kind="normal", seed=0, lo=-2, hi=2, **kw):
        out.append((name, dict(m=m, k=k, n=n, bm=tile[0], bn=tile[1], bk=tile[2],
                               inputs=dict(kind=kind, seed=seed, lo=lo, hi=hi), kwargs=kw)))

    # 1024^3, tile 256x256x256, seed 20260902, bf16 out.
    gemm("config1_1024_plain", 1024, 1024, 1024, (256, 256, 256), seed=20260902)
    gemm("interleaved_512x512x512", 512, 512, 512, (256, 256, 256), seed=20260903,
         interleave_products=True)
    # Shapes in the reference KAT style: one tile, several K panels, multi-block rows.
    gemm("int_16x256x256", 16, 256, 256, (16, 256, 256), kind="int", seed=187)
    gemm("int_32x768x512", 32, 768, 512, (16, 256, 256), kind="int", seed=188)
    gemm("int_512x1024x512_f32", 512, 1024, 512, (512, 256, 512), kind="int", seed=189,
         output_dtype="float32")
    gemm("normal_16x256x256_seed23", 16, 256, 256, (16, 256, 256), seed=23)
    gemm("normal_256x512x768_f32", 256, 512, 768, (256, 256, 256), seed=31,
         output_dtype="float32")
    gemm("normal_512x512x512_tile512", 512, 512, 512, (512, 512, 512), seed=32)
    gemm("normal_1024x512x256_bm64", 1024, 512, 256, (64, 256, 256), seed=33)
    gemm("sentinel_256x512x256", 256, 512, 256, (256, 256, 256), kind="const")
    # Epilogues (strassen_pallas.py:739-879), sizes with several K panels.
    gemm("swiglu_512x512x1024", 512, 512, 1024, (256, 512, 256), seed=41, epilogue="swiglu")
    gemm("swiglu_product_aware", 512, 512, 1024, (256, 512, 256), seed=41, epilogue="swiglu",
         product_aware_swiglu=True, interleave_products=True)
    gemm("geglu_256x512x512", 256, 512, 512, (256, 256, 256), seed=42, epilogue="geglu")
    gemm("residual_512x768x512", 512, 768, 512, (256, 256, 256), seed=43, epilogue="residual_add")
    gemm("residual_product_aware", 512, 768, 512, (256, 256, 256), seed=43,
         epilogue="residual_add", product_aware_residual=True, interleave_products=True)
    gemm("bias_256x512x512", 256, 512, 512, (256, 256, 256), seed=44, epilogue="bias_add")
    gemm("qk_norm_rope_256x512x1024", 256, 512, 1024, (256, 512, 256), seed=45,
         epilogue="qk_norm_rope")
    gemm("qk_norm_rope_hd64", 256, 512, 512, (256, 256, 256), seed=46, epilogue="qk_norm_rope",
         rope_head_dim=64)
    gemm("norm_residual_256x512x512", 256, 512, 512, (256, 512, 256), seed=47,
         epilogue="norm_residual_add")
    # Research options: dual formula, block permutation, exact panels.
    gemm("dual_512", 512, 512, 512, (256, 256, 256), seed=51, formula_variant="dual")
    gemm("dual_interleaved_512", 512, 512, 512, (256, 256, 256), seed=52, formula_variant="dual",
         interleave_products=True)
    gemm("blockperm5_512", 512, 512, 512, (256, 256, 256), seed=53, block_permutation=5)
    gemm("blockperm7_dual_f32", 256, 512, 512, (256, 256, 256), seed=54, block_permutation=7,
         formula_variant="dual", output_dtype="float32")
    gemm("exact_panels_0_2", 512, 1024, 512, (256, 256, 256), seed=55, classical_panels=(0, 2))
    gemm("panel_schedule_1001", 512, 1024, 512, (256, 256, 256), seed=56,
         panel_schedule=[1, 0, 0, 1])
    gemm("panel_schedule_all", 256, 512, 256, (256, 256, 256), seed=57, panel_schedule=[1, 1])
    gemm("int_exact_dual_perm3", 64, 1024, 512, (32, 256, 256), kind="int", seed=58,
         classical_panels=(1,), formula_variant="dual", block_permutation=3,
         output_dtype="float32")
    gemm("swiglu_blockperm6", 512, 512, 1024, (256, 512, 256), seed=59, epilogue="swiglu",
         block_permutation=6)
    gemm("swiglu_product_aware_exact0", 512, 1024, 1024, (256, 512, 256), seed=60,
         epilogue="swiglu", product_aware_swiglu=True, interleave_products=True,
         classical_panels=(0,))
    gemm("residual_dual_exact1", 256, 1024, 512, (256, 256, 512), seed=61,
         epilogue="residual_add", formula_variant="dual", classical_panels=(1,))
    gemm("powers_512", 512, 512, 512, (256, 256, 256), seed=62, formula_variant="powers")
    gemm("powers_interleaved_f32", 256, 1024, 512, (256, 256, 256), seed=63,
         formula_variant="powers", interleave_products=True, output_dtype="float32")
    gemm("powers_blockperm3", 512, 512, 512, (256, 256, 256), seed=64, formula_variant="powers",
         block_permutation=3)
    gemm("int_powers_perm4", 64, 768, 512, (32, 256, 256), kind="int", seed=65,
         formula_variant="powers", block_permutation=4, output_dtype="float32")
    return out


def make_inputs(p):
    """Recreate a case's inputs (float32 arrays of bf16 values) from its recipe."""
    from golden_inputs import make_inputs as shared
    return shared(p)


def run_reference(sp, p):
    a, b, extra = make_inputs(p)
    kw = dict(p["kwargs"])
    out_dtype = kw.pop("output_dtype", None)
    args = {key: np.asarray(val).astype(BF16) for key, val in extra.items()}
    result = sp.strassen_matmul(
        np.asarray(a).astype(BF16), np.asarray(b).astype(BF16),
        bm=p["bm"], bn=p["bn"], bk=p["bk"], interpret=True,
        output_dtype=None if out_dtype is None else np.float32, **kw, **args)
    return np.asarray(result)


def main():
    parser = argparse.ArgumentParser()
    parser.add_argument("--reference", required=True, help="path of the reference checkout")
    parser.add_argument("--out", default=str(HERE))
    args = parser.parse_args()
    sp = import_reference(Path(args.reference))
    manifest, arrays, lhs_manifest = {}, {}, {}
    for name, p in cases():
        out = run_reference(sp, p)
        # Large outputs are stored row-subsampled (every ROW_STRIDE-th row).
        stride = 4 if out.shape[0] * out.shape[1] > 70_000 else 1
        p["row_stride"] = stride
        full_shape = list(out.shape)
        out = out[::stride]
        if out.dtype == BF16:
            arrays[name] = out.view(np.uint16)
            p["output"] = "bf16_bits"
        else:
            arrays[name] = out.astype(np.float32)
            p["output"] = "float32"
        p["shape"] = full_shape
        manifest[name] = p
        print(f"{name}: out {out.shape} {out.dtype}", flush=True)
    # strassen_matmul_lhs_transposed (strassen_pallas.py:1224-1312): a is stored (K, M).
    lt_cases = {
        "lhs_t_512x768x512": dict(m=512, k=768, n=512, tile=(256, 256, 256), seed=71, kw={}),
        "lhs_t_interleaved_f32": dict(m=256, k=512, n=512, tile=(256, 256, 256), seed=72,
                                      kw=dict(interleave_products=True), out="float32"),
        "lhs_t_bm128_1024": dict(m=1024, k=1024, n=512, tile=(128, 256, 512), seed=73, kw={}),
    }
    for name, c in lt_cases.items():
        at = ref.normal_bf16((c["k"], c["m"]), c["seed"])
        bt = ref.normal_bf16((c["k"], c["n"]), c["seed"] + 1)
        out = np.asarray(sp.strassen_matmul_lhs_transposed(
            np.asarray(at).astype(BF16), np.asarray(bt).astype(BF16), bm=c["tile"][0],
            bn=c["tile"][1], bk=c["tile"][2], interpret=True,
            output_dtype=np.float32 if c.get("out") == "float32" else None, **c["kw"]))
        full_shape = list(out.shape)
        stride = 4 if out.shape[0] * out.shape[1] > 70_000 else 1
        arrays["lhs_t/" + name] = (out.view(np.uint16) if out.dtype == BF16 else out.astype(np.float32))[::stride]
        lhs_manifest[name] = dict(m=c["m"], k=c["k"], n=c["n"], bm=c["tile"][0], bn=c["tile"][1],
                                  bk=c["tile"][2], seed=c["seed"], kwargs=c["kw"], shape=full_shape,
                                  row_stride=stride,
                                  output="float32" if out.dtype != BF16 else "bf16_bits")
        print(f"lhs_t/{name}: out {out.shape} {out.dtype}", flush=True)
    # Layout helpers (strassen_pallas.py:1315-1411) on index-valued inputs, so the
    # stored result is the column permutation itself.
    layouts = {}
    w = np.arange(4 * 1024, dtype=np.float32).reshape(4, 1024)
    arrays["layout_swiglu_bn256"] = np.asarray(sp.swiglu_weight_layout(w, 256))
    arrays["layout_swiglu_bn512"] = np.asarray(sp.swiglu_weight_layout(w, 512))
    arrays["layout_rope_weight_bn256"] = np.asarray(sp.rope_weight_layout(w, 256))
    arrays["layout_rope_weight_bn512_hd64"] = np.asarray(sp.rope_weight_layout(w, 512, head_dim=64))
    tab = np.arange(8 * 128, dtype=np.float32).reshape(8, 128)
    c, s_ = sp.rope_layout_tables(tab, -tab, 256)
    arrays["layout_rope_cos_hw256"] = np.asarray(c)
    arrays["layout_rope_sin_hw256"] = np.asarray(s_)
    arrays["layout_rope_scale_bn512"] = np.asarray(sp.rope_scale_layout(np.arange(128, dtype=np.float32), 512))
    layouts = sorted(k for k in arrays if k.startswith("layout_"))
    print("layouts:", layouts)
    out_dir = Path(args.out)
    (out_dir / "golden_cases.json").write_text(json.dumps(
        {"generator": "tests/golden/make_golden.py",
         "reference": "sarsid/strassen-tpu strassen_pallas.py (kernel + wrapper, CPU stand-in)",
         "cases": manifest, "lhs_transposed_cases": lhs_manifest}, indent=1, sort_keys=True))
    np.savez_compressed(out_dir / "golden_outputs.npz", **arrays)


if __name__ == "__main__":
    main()

"""The ``strassen_matmul`` operator API, backed by the sm_100a kernel.

Same entry points, argument names, argument meaning and error behaviour as the
reference module ``strassen_pallas`` (strassen_pallas.py:127-140, 882-1221,
1414-1421): validation raises ``ValueError``/``TypeError`` on the host with the
reference's messages before anything is launched.  Arguments that only steer
the TPU compiler (``dot_precision``, ``allow_input_fusion``,
``vmem_limit_bytes``, ``interleave_products``, ``product_aware_*``) are
accepted and validated but do not change the B200 arithmetic, which keeps the
seven products in separate fp32 TMEM accumulators over the whole K range and
recombines them once.  The research options (``formula_variant="dual"`` and
``"powers"``, ``block_permutation``, exact classical panels via
``classical_panels`` / ``panel_schedule``) run on the same kernel layout.
``bm``/``bn``/``bk`` keep their reference meaning: they define the Strassen
block whose quadrants are paired, so results follow the reference's pairing of
operands.

Tensors are ``torch.Tensor`` on a CUDA B200 device.  There is no CPU path:
``interpret=True`` and CPU tensors raise.
"""

from __future__ import annotations

from typing import NamedTuple

import ctypes

import torch

from . import _native
from ._native import SB_BF16, SB_F32, EPILOGUE_KINDS, FORMULAS, SbEpilogue, SbOptions

LANE = 128
SUBLANE = 8
# The reference's default deployment tile (strassen_pallas.py:20-25, "compact16").
TUNED_BM, TUNED_BN, TUNED_BK = 1024, 1024, 512

_EPILOGUES = ("swiglu", "geglu", "residual_add", "bias_add", "qk_norm_rope", "norm_residual_add")


def check_tiling(bm: int, bn: int, bk: int) -> None:
    """Validate tile alignment after the one-level split (strassen_pallas.py:127-140)."""
    requirements = (("bm", bm, 2 * SUBLANE), ("bn", bn, 2 * LANE), ("bk", bk, 2 * LANE))
    errors = [f"{name}={value} must be a multiple of {multiple}"
              for name, value, multiple in requirements if value % multiple]
    if errors:
        raise ValueError("tile breaks TPU v5e alignment:\n  " + "\n  ".join(errors))


def _dtype_name(dt) -> str:
    return str(dt).replace("torch.", "")


def _as_torch_dtype(dt):
    if dt is None:
        return None
    if isinstance(dt, torch.dtype):
        return dt
    name = str(getattr(dt, "name", dt)).lower()
    table = {"bfloat16": torch.bfloat16, "bf16": torch.bfloat16,
             "float32": torch.float32, "f32": torch.float32, "fp32": torch.float32}
    if name in table:
        return table[name]
    raise ValueError("output_dtype must be BF16 or FP32")


def _ld(t: torch.Tensor) -> int:
    return t.stride(0)


def _rowmajor(t: torch.Tensor) -> torch.Tensor:
    if t.dim() == 2 and t.stride(1) == 1 and t.stride(0) >= t.shape[1] and t.stride(0) % 8 == 0 \
            and t.data_ptr() % 16 == 0:
        return t
    return t.contiguous()


def _stream_handle(device: torch.device) -> ctypes.c_void_p:
    return ctypes.c_void_p(torch.cuda.current_stream(device).cuda_stream)


def _out_tensor(out, shape, dtype, device):
    """``out`` checked for what the kernels write (or allocated when None)."""
    if out is None:
        return torch.empty(shape, dtype=dtype, device=device)
    if tuple(out.shape) != tuple(shape) or out.dtype != dtype or out.device != device:
        raise ValueError(f"out must be a {tuple(shape)} {_dtype_name(dtype)} tensor on {device}")
    if out.stride(1) != 1 or (out.stride(0) * out.element_size()) % 16 or out.data_ptr() % 16:
        raise ValueError("out must be row-major with a 16-byte aligned row stride")
    return out


def _workspace_tensor(workspace, need: int, device):
    """A caller's uint8 workspace checked against ``need`` bytes (or allocated when None)."""
    if workspace is None:
        return torch.empty(need, dtype=torch.uint8, device=device)
    if (workspace.dtype != torch.uint8 or workspace.numel() < need or workspace.device != device
            or not workspace.is_contiguous()):
        raise ValueError(f"workspace must be a contiguous uint8 tensor of at least {need} bytes on {device}")
    return workspace


def strassen_matmul(
    a,
    b,
    *,
    bm=TUNED_BM,
    bn=TUNED_BN,
    bk=TUNED_BK,
    dot_precision=None,
    interleave_products=False,
    block_permutation=0,
    formula_variant="classical",
    classical_panels=(),
    panel_schedule=None,
    epilogue=None,
    residual=None,
    bias=None,
    rope_cos=None,
    rope_sin=None,
    rope_scale=None,
    rope_head_dim=128,
    rope_eps=1e-6,
    norm_scale=None,
    norm_eps=1e-6,
    output_dtype=None,
    allow_input_fusion=None,
    product_aware_swiglu=False,
    product_aware_residual=False,
    interpret=False,
    vmem_limit_bytes=None,
    out=None,
    workspace=None,
    narrow_bn=False,
):
    """Compute ``a @ b`` with one tile-local classical Strassen level on B200.

    Mirrors strassen_pallas.strassen_matmul (strassen_pallas.py:882-1221).
    Extra keyword arguments: ``out`` (a preallocated output tensor),
    ``workspace`` (a caller-owned uint8 CUDA buffer of at least
    :func:`workspace_bytes` bytes; allocated from torch's caching allocator
    when omitted -- for a large product without research options and with no
    epilogue, a residual_add / bias_add / swiglu / geglu / qk_norm_rope
    epilogue, or norm_residual_add at N <= 8192, that is the planes path's
    workspace, and a smaller buffer keeps the product on the one-CTA kernel,
    which needs none except M*N*4 bytes of fp32 rows for norm_residual_add;
    see :func:`planes_matmul`) and
    ``narrow_bn`` (B200 extension, no reference counterpart:
    bn may be any multiple of 128 instead of the reference's TPU lane rule of
    256, and qk_norm_rope then needs bn % rope_head_dim == 0 -- each half block
    holds whole half-heads; the tensor-parallel decoder uses it for one-head k/v
    shards).
    """
    # --- the reference's validation, in its order (strassen_pallas.py:927-1047)
    if a.ndim != 2 or b.ndim != 2:
        raise ValueError("strassen_matmul expects two rank-2 matrices")
    m, k = a.shape
    k2, n = b.shape
    if k != k2:
        raise ValueError(f"inner dimensions disagree: {k} vs {k2}")
    if a.dtype != b.dtype:
        raise ValueError(f"input dtypes disagree: {_dtype_name(a.dtype)} vs {_dtype_name(b.dtype)}")
    if a.dtype not in (torch.bfloat16, torch.float32):
        raise ValueError("inputs must be BF16 or FP32")
    if not isinstance(block_permutation, int) or not 0 <= block_permutation < 8:
        raise ValueError("block_permutation must be an integer from 0 through 7")
    if formula_variant not in ("classical", "dual", "powers"):
        raise ValueError("formula_variant must be 'classical', 'dual', or 'powers'")
    classical_panels = tuple(sorted({int(p) for p in classical_panels}))
    out_dt = _as_torch_dtype(output_dtype)
    if epilogue is not None:
        if epilogue not in _EPILOGUES:
            raise ValueError(
                f"unknown epilogue {epilogue!r}; choose 'swiglu' or 'residual_add' or 'bias_add'")
        if formula_variant == "powers":
            raise ValueError("fused epilogues require a quadrant-basis formula")
        if out_dt is not None and out_dt != torch.bfloat16:
            raise ValueError("fused epilogues write a BF16 output tile")
        if epilogue in ("swiglu", "geglu") and bn % 2:
            raise ValueError(f"{epilogue} epilogue needs an even bn, got {bn}")
        if epilogue == "residual_add" and residual is None:
            raise ValueError("residual_add epilogue requires residual=")
        if epilogue == "bias_add" and bias is None:
            raise ValueError("bias_add epilogue requires bias=")
    if residual is not None and epilogue not in ("residual_add", "norm_residual_add"):
        raise ValueError("residual= is only used by the residual_add and norm_residual_add epilogues")
    if bias is not None and epilogue != "bias_add":
        raise ValueError("bias= is only used by the bias_add epilogue")
    if epilogue == "norm_residual_add":
        if residual is None or norm_scale is None:
            raise ValueError("norm_residual_add requires residual= and norm_scale=")
        if bn != n:
            raise ValueError(
                "norm_residual_add normalises over the whole output row, so "
                f"the tile must span it: bn={bn} must equal n={n}")
        if tuple(residual.shape) != (m, n):
            raise ValueError(f"residual shape {tuple(residual.shape)} != output {(m, n)}")
        if tuple(norm_scale.shape) != (n,):
            raise ValueError(f"norm_scale shape {tuple(norm_scale.shape)} != output width {(n,)}")
    if epilogue == "qk_norm_rope":
        if rope_cos is None or rope_sin is None or rope_scale is None:
            raise ValueError(
                "qk_norm_rope epilogue requires rope_cos=, rope_sin= and "
                "rope_scale= (use rope_layout_tables and rope_scale_layout)")
        if narrow_bn and bn % rope_head_dim:
            raise ValueError(
                f"qk_norm_rope with narrow_bn needs bn a multiple of head_dim={rope_head_dim} so a "
                f"tile half holds whole half-heads, got bn={bn}")
        if not narrow_bn and bn % (2 * rope_head_dim):
            raise ValueError(
                f"qk_norm_rope needs bn a multiple of 2*head_dim={2 * rope_head_dim} so a "
                f"tile half holds whole heads, got bn={bn}")
        if tuple(rope_cos.shape) != (m, bn // 2) or tuple(rope_sin.shape) != (m, bn // 2):
            raise ValueError(
                f"rope tables must be {(m, bn // 2)}, got "
                f"{tuple(rope_cos.shape)} and {tuple(rope_sin.shape)}")
        if tuple(rope_scale.shape) != (bn,):
            raise ValueError(f"rope_scale must be laid out to {(bn,)}, got {tuple(rope_scale.shape)}")
    if rope_cos is not None and epilogue != "qk_norm_rope":
        raise ValueError("rope_* are only used by the qk_norm_rope epilogue")
    if product_aware_swiglu and epilogue not in ("swiglu", "geglu"):
        raise ValueError("product_aware_swiglu is only valid with epilogue='swiglu' or 'geglu'")
    if product_aware_residual and epilogue != "residual_add":
        raise ValueError("product_aware_residual is only valid with epilogue='residual_add'")
    if epilogue == "bias_add" and tuple(bias.shape) != (n,):
        raise ValueError(f"bias shape {tuple(bias.shape)} != output width {(n,)}")
    operand_count = 3 if epilogue in ("residual_add", "bias_add") else 2
    if epilogue == "norm_residual_add":
        operand_count = 4
    if epilogue == "qk_norm_rope":
        operand_count = 6
    if allow_input_fusion is not None:
        allow_input_fusion = tuple(allow_input_fusion)
        if len(allow_input_fusion) != operand_count:
            raise ValueError(
                "allow_input_fusion must contain one boolean per operand: "
                f"expected {operand_count}, got {len(allow_input_fusion)}")
        if not all(isinstance(value, bool) for value in allow_input_fusion):
            raise TypeError("allow_input_fusion entries must be bool")
    if panel_schedule is not None and classical_panels:
        raise ValueError("pass either classical_panels (static) or panel_schedule (prefetched), not both")
    if classical_panels:
        if formula_variant == "powers":
            raise ValueError("classical_panels requires a quadrant-basis formula")
        if classical_panels[0] < 0 or classical_panels[-1] >= k // bk:
            raise ValueError(f"classical_panels {classical_panels} outside 0..{k // bk - 1}")
    for name, dimension, block in (("M", m, bm), ("N", n, bn), ("K", k, bk)):
        if dimension % block:
            raise ValueError(f"{name}={dimension} is not divisible by {block}")
    if narrow_bn:
        if bn % 128:
            raise ValueError(f"narrow_bn: bn={bn} must be a multiple of 128")
        check_tiling(bm, 2 * LANE, bk)
    else:
        check_tiling(bm, bn, bk)
    out_dt = a.dtype if out_dt is None else out_dt
    if out_dt not in (torch.bfloat16, torch.float32):
        raise ValueError("output_dtype must be BF16 or FP32")
    if panel_schedule is not None and epilogue is not None:
        raise ValueError("panel_schedule does not support fused epilogues")
    if residual is not None and epilogue == "residual_add" and tuple(residual.shape) != (m, n):
        raise ValueError(f"residual shape {tuple(residual.shape)} != output shape {(m, n)}")

    nk = k // bk
    if panel_schedule is not None:
        schedule_shape = tuple(torch.as_tensor(panel_schedule).shape)
        if schedule_shape != (nk,):
            raise ValueError(f"panel_schedule must have shape ({nk},), got {schedule_shape}")
    # Checks the reference makes while tracing its kernel (strassen_pallas.py:282-312).
    if product_aware_swiglu and (
            out_dt == torch.float32 or formula_variant != "classical" or block_permutation != 0
            or (nk - 1) in classical_panels or panel_schedule is not None
            or epilogue not in ("swiglu", "geglu")):
        raise ValueError(
            "product-aware SwiGLU requires unpermuted classical Strassen "
            "with quadrant accumulators; exact panels are allowed except on "
            "the final K panel, whose product order the schedule owns")
    if product_aware_residual and (
            out_dt == torch.float32 or formula_variant != "classical" or block_permutation != 0
            or (nk - 1) in classical_panels or panel_schedule is not None
            or epilogue != "residual_add"):
        raise ValueError(
            "product-aware residual requires unpermuted classical Strassen "
            "with quadrant accumulators and the residual_add epilogue; exact "
            "panels are allowed except on the final K panel")

    # --- what the B200 build does not implement (yet): refuse loudly.
    if interpret:
        raise NotImplementedError(
            "interpret=True: the B200 build has no CPU path; the CPU restatement lives in "
            "oracle/ and is test infrastructure only")
    if a.dtype != torch.bfloat16:
        raise NotImplementedError("the B200 kernel computes bf16 inputs; FP32 inputs are not built")
    if formula_variant == "powers" and panel_schedule is not None:
        raise NotImplementedError("exact classical panels need a quadrant-basis formula")
    if not (a.is_cuda and b.is_cuda):
        raise ValueError("strassen_matmul runs on a CUDA device; got CPU tensors (no CPU fallback)")

    device = a.device
    if workspace is not None and (not isinstance(workspace, torch.Tensor) or workspace.device != device
                                  or not workspace.is_contiguous()):
        raise ValueError(f"workspace must be a contiguous tensor on {device} (the kernels write it)")
    a = _rowmajor(a)
    b = _rowmajor(b.to(device))
    gated = epilogue in ("swiglu", "geglu")
    out_shape = (m, n // 2) if gated else (m, n)
    if out is None:
        out = torch.empty(out_shape, dtype=out_dt, device=device)
    else:
        if tuple(out.shape) != out_shape or out.dtype != out_dt or out.device != device:
            raise ValueError(f"out must be a {out_shape} {_dtype_name(out_dt)} tensor on {device}")
        if out.stride(1) != 1 or out.stride(0) % 8 or out.data_ptr() % 16:
            raise ValueError("out must be row-major with a 16-byte aligned row stride")

    ep = SbEpilogue()
    ep.kind = EPILOGUE_KINDS[epilogue]
    keep_alive = []
    aux = [t for t in (bias, rope_cos, rope_sin, rope_scale, norm_scale) if t is not None]
    aux_dt = torch.float32 if any(t.dtype == torch.float32 for t in aux) else torch.bfloat16
    ep.aux_dtype = SB_F32 if aux_dt == torch.float32 else SB_BF16

    def prep_aux(t):
        t = t.to(device=device, dtype=aux_dt).contiguous()
        keep_alive.append(t)
        return t

    if residual is not None:
        r = residual.to(device)
        if r.dtype not in (torch.bfloat16, torch.float32):
            r = r.float()
        r = _rowmajor(r)
        keep_alive.append(r)
        ep.residual = r.data_ptr()
        ep.ld_residual = _ld(r)
        ep.residual_dtype = SB_F32 if r.dtype == torch.float32 else SB_BF16
    if bias is not None:
        ep.bias = prep_aux(bias).data_ptr()
    if rope_cos is not None:
        cos_t = prep_aux(rope_cos)
        ep.rope_cos = cos_t.data_ptr()
        ep.rope_sin = prep_aux(rope_sin).data_ptr()
        ep.ld_rope = cos_t.stride(0)
        ep.rope_scale = prep_aux(rope_scale).data_ptr()
    ep.rope_head_dim = int(rope_head_dim)
    ep.rope_eps = float(rope_eps)
    if norm_scale is not None:
        ep.norm_scale = prep_aux(norm_scale).data_ptr()
    ep.norm_eps = float(norm_eps)

    opts = SbOptions()
    opts.formula_variant = FORMULAS[formula_variant]
    opts.block_permutation = int(block_permutation)
    opts.narrow_bn = 1 if narrow_bn else 0
    if classical_panels or panel_schedule is not None:
        if panel_schedule is not None:
            sched = torch.as_tensor(panel_schedule).to(device=device, dtype=torch.int32).contiguous()
        else:
            sched = torch.zeros(nk, dtype=torch.int32)
            sched[list(classical_panels)] = 1
            sched = sched.to(device)
        keep_alive.append(sched)
        opts.panel_schedule = sched.data_ptr()

    lib = _native.load()
    ws_bytes = int(lib.sb_workspace_bytes(m, n, k, ep.kind))
    ws_ptr = None
    if ws_bytes:
        if workspace is None:
            workspace = torch.empty(ws_bytes, dtype=torch.uint8, device=device)
        have = workspace.numel() * workspace.element_size()
        if have < ws_bytes:
            if ep.kind == EPILOGUE_KINDS["norm_residual_add"]:
                # The one-CTA kernel's two-pass norm needs the fp32 rows.
                rows_bytes = m * n * 4
                if have < rows_bytes:
                    raise ValueError(f"workspace must hold {rows_bytes} bytes")
                ws_bytes, ws_ptr = have, workspace.data_ptr()
            else:
                # Without room for the planes path the product runs on the
                # one-CTA kernel, which needs no workspace.
                ws_bytes = 0
        else:
            ws_ptr = workspace.data_ptr()
    with torch.cuda.device(device):
        status = lib.sb_strassen_gemm_ex(
            _stream_handle(device), a.data_ptr(), b.data_ptr(), out.data_ptr(),
            m, n, k, _ld(a), _ld(b), _ld(out), bm, bn, bk,
            SB_F32 if out_dt == torch.float32 else SB_BF16, ctypes.byref(ep), ctypes.byref(opts),
            ws_ptr, ws_bytes)
    _native.check(status)
    return out


_SIDE_STREAMS: dict = {}


def _side_streams(device: torch.device):
    """The two copy streams of a device (host->device, device->host), created once."""
    key = device.index
    if key not in _SIDE_STREAMS:
        _SIDE_STREAMS[key] = (torch.cuda.Stream(device), torch.cuda.Stream(device))
    return _SIDE_STREAMS[key]


_UNSTREAMED = ("residual", "bias", "rope_cos", "rope_sin", "rope_scale", "norm_scale", "out", "workspace")


def strassen_matmul_streamed(a, b, *, bm=TUNED_BM, bn=TUNED_BN, bk=TUNED_BK, device=None, out=None,
                             row_chunk=None, **kwargs):
    """``strassen_matmul`` for host-resident operands, with the transfers overlapped.

    ``a`` [M, K] and ``b`` [K, N] are CPU tensors (pinned memory makes the copies
    asynchronous); the product lands in ``out``, a CPU tensor (pinned, allocated
    when omitted).  B is copied to ``device`` first, then A in chunks of
    ``row_chunk`` rows (a multiple of bm; default M/8 rounded to whole blocks) on
    a copy stream.  Each chunk's GEMM runs on the current stream as soon as its
    rows have landed, and its result rows return on a second copy stream while
    later chunks compute, so the transfer time, not the sum of transfers and
    compute, bounds the call.  Strassen block rows are independent: the result
    equals one ``strassen_matmul`` call bit for bit.

    The copies are asynchronous: ``out`` is complete once the current CUDA stream
    has reached the end of this call (``torch.cuda.current_stream().synchronize()``).
    Epilogues that read extra row-indexed operands (residual, rope tables,
    norm_scale, bias) are not streamed; call ``strassen_matmul`` with device
    tensors for those.  Other keyword arguments go to ``strassen_matmul``.
    """
    if a.dim() != 2 or b.dim() != 2:
        raise ValueError("strassen_matmul expects two rank-2 matrices")
    if a.is_cuda or b.is_cuda:
        raise ValueError("strassen_matmul_streamed takes host (CPU) tensors; use strassen_matmul on device tensors")
    for name in _UNSTREAMED:
        if kwargs.get(name) is not None:
            raise ValueError(f"{name}= is not streamed; call strassen_matmul with device tensors")
    m, k = a.shape
    k2, n = b.shape
    if k != k2:
        raise ValueError(f"inner dimensions disagree: {k} vs {k2}")
    if m % bm:
        raise ValueError(f"M={m} is not divisible by {bm}")
    blocks = m // bm
    if row_chunk is None:
        per = max(1, blocks // 8)
        while blocks % per:
            per -= 1
        row_chunk = per * bm
    if row_chunk <= 0 or row_chunk % bm or m % row_chunk:
        raise ValueError(f"row_chunk={row_chunk} must be a positive multiple of bm={bm} that divides M={m}")
    dev = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
    out_dt = _as_torch_dtype(kwargs.get("output_dtype")) or torch.bfloat16
    out_cols = n // 2 if kwargs.get("epilogue") in ("swiglu", "geglu") else n
    if out is None:
        out = torch.empty((m, out_cols), dtype=out_dt, pin_memory=True)
    elif out.is_cuda or tuple(out.shape) != (m, out_cols) or out.dtype != out_dt or not out.is_contiguous():
        raise ValueError(f"out must be a contiguous ({m}, {out_cols}) {_dtype_name(out_dt)} CPU tensor")

    h2d, d2h = _side_streams(dev)
    cur = torch.cuda.current_stream(dev)
    a_dev = torch.empty((m, k), dtype=a.dtype, device=dev)
    b_dev = torch.empty((k, n), dtype=b.dtype, device=dev)
    c_dev = torch.empty((m, out_cols), dtype=out_dt, device=dev)
    # The copy streams start after the work already queued on the current stream.
    h2d.wait_stream(cur)
    d2h.wait_stream(cur)
    chunks = [(i, i + row_chunk) for i in range(0, m, row_chunk)]
    landed = []
    with torch.cuda.stream(h2d):
        b_dev.copy_(b, non_blocking=True)
        for lo, hi in chunks:
            a_dev[lo:hi].copy_(a[lo:hi], non_blocking=True)
            ev = torch.cuda.Event()
            ev.record(h2d)
            landed.append(ev)  # also implies B has landed (same stream, earlier)
    for (lo, hi), ev in zip(chunks, landed):
        cur.wait_event(ev)
        strassen_matmul(a_dev[lo:hi], b_dev, bm=bm, bn=bn, bk=bk, out=c_dev[lo:hi], **kwargs)
        done = torch.cuda.Event()
        done.record(cur)
        d2h.wait_event(done)
        with torch.cuda.stream(d2h):
            out[lo:hi].copy_(c_dev[lo:hi], non_blocking=True)
    cur.wait_stream(d2h)
    # The device buffers were allocated on the current stream but are used on the
    # copy streams: keep the caching allocator from reusing them too early.
    a_dev.record_stream(h2d)
    b_dev.record_stream(h2d)
    c_dev.record_stream(d2h)
    return out


def strassen_matmul_lhs_transposed(
    a,
    b,
    *,
    bm=TUNED_BM,
    bn=TUNED_BN,
    bk=TUNED_BK,
    dot_precision=None,
    interleave_products=False,
    output_dtype=None,
    allow_input_fusion=None,
    interpret=False,
    vmem_limit_bytes=None,
    out=None,
):
    """Compute ``a.T @ b`` without materialising the transpose; ``a`` is (K, M).

    Mirrors strassen_pallas.strassen_matmul_lhs_transposed
    (strassen_pallas.py:1224-1312): the kernel loads M-major tiles of ``a`` with
    TMA and feeds them to the tensor cores as an MN-major operand.  B200
    restriction: ``bm`` must be a multiple of 128.
    """
    if a.ndim != 2 or b.ndim != 2:
        raise ValueError("strassen_matmul_lhs_transposed expects rank-2 inputs")
    k, m = a.shape
    k2, n = b.shape
    if k != k2:
        raise ValueError(f"contracting dimensions disagree: {k} vs {k2}")
    if a.dtype != b.dtype:
        raise ValueError(f"input dtypes disagree: {_dtype_name(a.dtype)} vs {_dtype_name(b.dtype)}")
    if a.dtype not in (torch.bfloat16, torch.float32):
        raise ValueError("inputs must be BF16 or FP32")
    for name, dimension, block in (("M", m, bm), ("N", n, bn), ("K", k, bk)):
        if dimension % block:
            raise ValueError(f"{name}={dimension} is not divisible by {block}")
    check_tiling(bm, bn, bk)
    if allow_input_fusion is not None:
        allow_input_fusion = tuple(allow_input_fusion)
        if len(allow_input_fusion) != 2:
            raise ValueError("allow_input_fusion must contain two booleans")
    out_dt = _as_torch_dtype(output_dtype) or a.dtype
    if out_dt not in (torch.bfloat16, torch.float32):
        raise ValueError("output_dtype must be BF16 or FP32")
    if interpret:
        raise NotImplementedError("interpret=True: the B200 build has no CPU path")
    if a.dtype != torch.bfloat16:
        raise NotImplementedError("the B200 kernel computes bf16 inputs; FP32 inputs are not built")
    if bm % 128:
        raise NotImplementedError(f"strassen_matmul_lhs_transposed on B200 needs bm a multiple of 128, got {bm}")
    if not (a.is_cuda and b.is_cuda):
        raise ValueError("strassen_matmul_lhs_transposed runs on a CUDA device; got CPU tensors (no CPU fallback)")
    device = a.device
    a, b = _rowmajor(a), _rowmajor(b.to(device))
    if out is None:
        out = torch.empty((m, n), dtype=out_dt, device=device)
    elif tuple(out.shape) != (m, n) or out.dtype != out_dt or out.device != device:
        raise ValueError(f"out must be a {(m, n)} {_dtype_name(out_dt)} tensor on {device}")
    elif out.stride(1) != 1 or out.stride(0) % 8 or out.data_ptr() % 16:
        raise ValueError("out must be row-major with a 16-byte aligned row stride")
    lib = _native.load()
    with torch.cuda.device(device):
        status = lib.sb_strassen_gemm_lhs_transposed(
            _stream_handle(device), a.data_ptr(), b.data_ptr(), out.data_ptr(), m, n, k,
            _ld(a), _ld(b), _ld(out), bm, bn, bk, SB_F32 if out_dt == torch.float32 else SB_BF16)
    _native.check(status)
    return out


def workspace_bytes(m: int, n: int, k: int, epilogue=None) -> int:
    """Scratch bytes :func:`strassen_matmul` needs (non-zero for norm_residual_add)."""
    return int(_native.load().sb_workspace_bytes(m, n, k, EPILOGUE_KINDS[epilogue]))


def classical_matmul(a, b, *, bm=TUNED_BM, bn=TUNED_BN, bk=TUNED_BK, output_dtype=None, out=None):
    """Matched-tile cubic control: the same sm_100a kernel skeleton with eight
    classical sub-block products and no operand sums.

    Mirrors the reference's blocked cubic Pallas control
    (experiments/qwen3/benchmark_cubic_control.py:57-237, variant="blocked").
    """
    if a.ndim != 2 or b.ndim != 2:
        raise ValueError("classical_matmul expects two rank-2 matrices")
    m, k = a.shape
    k2, n = b.shape
    if k != k2:
        raise ValueError(f"inner dimensions disagree: {k} vs {k2}")
    if a.dtype != torch.bfloat16 or b.dtype != torch.bfloat16:
        raise ValueError("inputs must be BF16")
    for name, dimension, block in (("M", m, bm), ("N", n, bn), ("K", k, bk)):
        if dimension % block:
            raise ValueError(f"{name}={dimension} is not divisible by {block}")
    check_tiling(bm, bn, bk)
    out_dt = _as_torch_dtype(output_dtype) or torch.bfloat16
    device = a.device
    a, b = _rowmajor(a), _rowmajor(b)
    if out is None:
        out = torch.empty((m, n), dtype=out_dt, device=device)
    lib = _native.load()
    with torch.cuda.device(device):
        status = lib.sb_classical_gemm(_stream_handle(device), a.data_ptr(), b.data_ptr(),
                                       out.data_ptr(), m, n, k, _ld(a), _ld(b), _ld(out),
                                       bm, bn, bk, SB_F32 if out_dt == torch.float32 else SB_BF16)
    _native.check(status)
    return out


class StrassenBOperands(NamedTuple):
    """B operand planes and the tile they were formed for.

    ``planes`` is ``[7, K/2, N/2]`` bf16; plane i at (kappa, u) belongs to block
    (kappa // (bk/2), u // (bn/2)), so the planes are only valid for a GEMM with
    the same ``bn`` and ``bk`` -- :func:`pair_matmul` checks this.
    """
    planes: torch.Tensor
    bn: int
    bk: int


def strassen_b_operands(b, *, bn=TUNED_BN, bk=TUNED_BK, out=None):
    """The seven B operands of every Strassen block of ``b`` for the tile (bn, bk).

    Returns a :class:`StrassenBOperands` whose ``planes`` are ``[7, K/2, N/2]``
    bf16 in the order P3 (b1-b3), P5 (b3), P7 (b2+b3), P1 (b0+b3), P2 (b0),
    P4 (b2-b0), P6 (b0+b1): the reference's B pre-adds
    (strassen_pallas.py:324-379), each rounded once to bf16.  Pass it to
    :func:`pair_matmul` as ``b_operands=``; the tile must match.  For a weight
    reused across calls this is an offline relayout, like
    :func:`swiglu_weight_layout`.  ``out``: a preallocated planes tensor.
    """
    if b.ndim != 2 or b.dtype != torch.bfloat16:
        raise ValueError("strassen_b_operands expects a rank-2 BF16 matrix")
    if b.device.type != "cuda":
        raise ValueError("strassen_b_operands runs on a CUDA device (no CPU fallback)")
    k, n = b.shape
    b = _rowmajor(b)
    shape = (7, k // 2, n // 2)
    if out is None:
        out = torch.empty(shape, dtype=torch.bfloat16, device=b.device)
    elif tuple(out.shape) != shape or out.dtype != torch.bfloat16 or not out.is_contiguous():
        raise ValueError(f"out must be a contiguous bf16 tensor of shape {shape}")
    lib = _native.load()
    with torch.cuda.device(b.device):
        status = lib.sb_strassen_b_operands(_stream_handle(b.device), b.data_ptr(), out.data_ptr(), k, n,
                                            _ld(b), bn, bk)
    _native.check(status)
    return StrassenBOperands(out, int(bn), int(bk))


def pair_matmul(a, b, *, bm=TUNED_BM, bn=TUNED_BN, bk=TUNED_BK, output_dtype=None, out=None,
                b_operands=None):
    """``strassen_matmul(a, b, bm=, bn=, bk=, output_dtype=)`` without an epilogue,
    on the two-CTA kernel (``sb_strassen_gemm_pair``): a cluster of two CTAs per
    128 x 128 product tile, 3.5 of the seven products each.  Same algorithm and
    operand pairing as strassen_pallas.py:156-880; the recombination's fp32
    order differs from :func:`strassen_matmul`.

    ``b_operands``: B's :class:`StrassenBOperands` from :func:`strassen_b_operands`,
    formed for the same bn, bk; then ``b`` may be None and the kernel forms no B
    sums (``sb_strassen_gemm_pair_planes``; bit-identical to the raw-B call).
    """
    if b_operands is not None:
        if not isinstance(b_operands, StrassenBOperands):
            raise ValueError("b_operands must be the StrassenBOperands returned by strassen_b_operands "
                             "(the planes' layout depends on the tile they were formed for)")
        if (b_operands.bn, b_operands.bk) != (bn, bk):
            raise ValueError(f"b_operands were formed for bn={b_operands.bn}, bk={b_operands.bk}; "
                             f"this call uses bn={bn}, bk={bk}")
        planes = b_operands.planes
        if planes.ndim != 3 or planes.shape[0] != 7 or planes.dtype != torch.bfloat16 \
                or not planes.is_contiguous():
            raise ValueError("b_operands must hold the contiguous [7, K/2, N/2] bf16 planes of strassen_b_operands")
        kb, nb = 2 * planes.shape[1], 2 * planes.shape[2]
        if b is not None and tuple(b.shape) != (kb, nb):
            raise ValueError(f"b_operands describe a {kb}x{nb} B, b is {tuple(b.shape)}")
    if a.ndim != 2 or (b is not None and b.ndim != 2):
        raise ValueError("pair_matmul expects two rank-2 matrices")
    m, k = a.shape
    k2, n = (kb, nb) if b_operands is not None else b.shape
    if k != k2:
        raise ValueError(f"inner dimensions disagree: {k} vs {k2}")
    if a.dtype != torch.bfloat16 or (b is not None and b.dtype != torch.bfloat16):
        raise ValueError("inputs must be BF16")
    for name, dimension, block in (("M", m, bm), ("N", n, bn), ("K", k, bk)):
        if dimension % block:
            raise ValueError(f"{name}={dimension} is not divisible by {block}")
    check_tiling(bm, bn, bk)
    if a.device.type != "cuda" or (b is not None and b.device.type != "cuda"):
        raise ValueError("pair_matmul runs on a CUDA device (no CPU fallback)")
    out_dt = _as_torch_dtype(output_dtype) or torch.bfloat16
    device = a.device
    a = _rowmajor(a)
    out = _out_tensor(out, (m, n), out_dt, device)
    lib = _native.load()
    od = SB_F32 if out_dt == torch.float32 else SB_BF16
    with torch.cuda.device(device):
        if b_operands is not None:
            status = lib.sb_strassen_gemm_pair_planes(_stream_handle(device), a.data_ptr(), planes.data_ptr(),
                                                      out.data_ptr(), m, n, k, _ld(a), _ld(out), bm, bn, bk, od)
        else:
            b = _rowmajor(b)
            status = lib.sb_strassen_gemm_pair(_stream_handle(device), a.data_ptr(), b.data_ptr(),
                                               out.data_ptr(), m, n, k, _ld(a), _ld(b), _ld(out), bm, bn, bk, od)
    _native.check(status)
    return out


def quad_matmul(a, b, *, bm=TUNED_BM, bn=TUNED_BN, bk=TUNED_BK, output_dtype=None, out=None, workspace=None,
                raster=0):
    """``strassen_matmul(a, b, bm=, bn=, bk=, output_dtype=)`` without an epilogue,
    on the four-CTA kernel (``sb_strassen_gemm_quad``): clusters of two CTA
    pairs on B200's paired tensor cores (tcgen05 ``cta_group::2``), one
    256 x 128 product tile per cluster, each pair 3.5 of the seven products.
    Same algorithm and operand pairing as strassen_pallas.py:156-880; the
    recombination's fp32 order differs from :func:`strassen_matmul`.

    The call forms A's operands and B's operand planes in a workspace (the
    ``sb_quad_workspace_bytes`` of the shape; allocated here unless
    ``workspace=`` passes a uint8 CUDA tensor at least that large) before the
    GEMM, all on the current stream.  Needs M % 512 == 0, bn % 256 == 0 and
    bk % 256 == 0.  ``raster``: product-row tiles per column sweep of the
    cluster tiles (0 = the kernel's default); the result does not depend on it.
    """
    if a.ndim != 2 or b.ndim != 2:
        raise ValueError("quad_matmul expects two rank-2 matrices")
    m, k = a.shape
    k2, n = b.shape
    if k != k2:
        raise ValueError(f"inner dimensions disagree: {k} vs {k2}")
    if a.dtype != torch.bfloat16 or b.dtype != torch.bfloat16:
        raise ValueError("inputs must be BF16")
    for name, dimension, block in (("M", m, bm), ("N", n, bn), ("K", k, bk)):
        if dimension % block:
            raise ValueError(f"{name}={dimension} is not divisible by {block}")
    check_tiling(bm, bn, bk)
    if m % 512 or bn % 256 or bk % 256:
        raise ValueError("the four-CTA kernel needs M % 512 == 0, bn % 256 == 0 and bk % 256 == 0")
    if a.device.type != "cuda" or b.device.type != "cuda":
        raise ValueError("quad_matmul runs on a CUDA device (no CPU fallback)")
    out_dt = _as_torch_dtype(output_dtype) or torch.bfloat16
    device = a.device
    a = _rowmajor(a)
    b = _rowmajor(b)
    out = _out_tensor(out, (m, n), out_dt, device)
    lib = _native.load()
    workspace = _workspace_tensor(workspace, int(lib.sb_quad_workspace_bytes(m, n, k)), device)
    od = SB_F32 if out_dt == torch.float32 else SB_BF16
    with torch.cuda.device(device):
        status = lib.sb_strassen_gemm_quad(_stream_handle(device), a.data_ptr(), b.data_ptr(), out.data_ptr(),
                                           m, n, k, _ld(a), _ld(b), _ld(out), bm, bn, bk, od,
                                           workspace.data_ptr(), workspace.numel(), int(raster))
    _native.check(status)
    return out


def planes_matmul(a, b, *, bm=TUNED_BM, bn=TUNED_BN, bk=TUNED_BK, output_dtype=None, out=None, workspace=None,
                  raster=0, stages=7, timing_events=None):
    """``strassen_matmul(a, b, bm=, bn=, bk=, output_dtype=)`` without an epilogue,
    as seven full-width product GEMMs (``sb_strassen_gemm_planes``): the A and
    B operand planes of every Strassen block (the reference's pre-adds,
    strassen_pallas.py:324-379, rounded once), the seven products on CTA pairs
    with 256 x 256 tiles into an fp32 workspace, and the recombination into C
    in the one-CTA kernel's fp32 order.

    ``workspace``: a uint8 CUDA tensor of at least ``sb_planes_workspace_bytes``
    of the shape (allocated here when omitted).  Needs M % 512 == 0,
    N % 512 == 0 and K % 128 == 0.  ``raster``: product-row tiles per column
    sweep (0 = the kernel's default); the result does not depend on it.
    ``stages``: bit 0 the operand passes, bit 1 the product GEMM, bit 2 the
    recombination (7 = all); separate calls with the same ``workspace`` and
    operands give the same result as one call (used to time the GEMM alone).
    The whole product runs in two halves of product rows on two streams so the
    passes and recombination of one half overlap the other's GEMM (joined back
    into the current stream before the call returns).  ``timing_events``: four
    ``torch.cuda.Event(enable_timing=True)`` the call records around its GEMM
    launches: 0/1 around the first half's, 2/3 around the second half's; when
    the GEMM runs as one launch (``stages=2``, fewer than two 256-row product
    tiles, or a first call inside a graph capture) 0/1 around it and 2/3 at its
    end.
    """
    if a.ndim != 2 or b.ndim != 2:
        raise ValueError("planes_matmul expects two rank-2 matrices")
    m, k = a.shape
    k2, n = b.shape
    if k != k2:
        raise ValueError(f"inner dimensions disagree: {k} vs {k2}")
    if a.dtype != torch.bfloat16 or b.dtype != torch.bfloat16:
        raise ValueError("inputs must be BF16")
    for name, dimension, block in (("M", m, bm), ("N", n, bn), ("K", k, bk)):
        if dimension % block:
            raise ValueError(f"{name}={dimension} is not divisible by {block}")
    check_tiling(bm, bn, bk)
    if m % 512 or n % 512 or k % 128:
        raise ValueError("the planes path needs M % 512 == 0, N % 512 == 0 and K % 128 == 0")
    if a.device.type != "cuda" or b.device.type != "cuda":
        raise ValueError("planes_matmul runs on a CUDA device (no CPU fallback)")
    out_dt = _as_torch_dtype(output_dtype) or torch.bfloat16
    device = a.device
    a = _rowmajor(a)
    b = _rowmajor(b)
    out = _out_tensor(out, (m, n), out_dt, device)
    lib = _native.load()
    workspace = _workspace_tensor(workspace, int(lib.sb_planes_workspace_bytes(m, n, k)), device)
    od = SB_F32 if out_dt == torch.float32 else SB_BF16
    events = None
    if timing_events is not None and len(timing_events) != 4:
        raise ValueError("timing_events must be four torch.cuda.Event(enable_timing=True)")
    with torch.cuda.device(device):
        if timing_events is not None:
            for e in timing_events:
                e.record()  # creates the CUDA event on this device; the call records it again
            events = (ctypes.c_void_p * 4)(*[e.cuda_event for e in timing_events])
        status = lib.sb_strassen_gemm_planes(_stream_handle(device), a.data_ptr(), b.data_ptr(), out.data_ptr(),
                                             m, n, k, _ld(a), _ld(b), _ld(out), bm, bn, bk, od,
                                             workspace.data_ptr(), workspace.numel(), int(raster), int(stages),
                                             events)
    _native.check(status)
    return out


def rms_norm(x, scale, eps: float = 1e-6, out=None):
    """bf16 RMSNorm with fp32 math on the sm_100a row kernel.

    Mirrors experiments/qwen3/benchmark_qwen3_32b_layer.py:270-276:
    ``bf16(x * rsqrt(mean(x^2, -1) + eps) * scale)``.  ``x`` is [..., n] bf16.
    """
    if x.dtype != torch.bfloat16:
        raise ValueError("rms_norm expects a bf16 input")
    n = x.shape[-1]
    if scale.numel() != n:
        raise ValueError(f"scale must hold {n} values (the row width), got {scale.numel()}")
    if not x.is_cuda:
        raise ValueError("rms_norm runs on a CUDA device (no CPU fallback)")
    x2 = x.reshape(-1, n).contiguous()
    w = scale.to(device=x.device).reshape(n)
    if w.dtype not in (torch.bfloat16, torch.float32):
        w = w.float()
    w = w.contiguous()
    if out is None:
        y = torch.empty_like(x2)
    else:
        if tuple(out.shape) != tuple(x.shape) or out.dtype != torch.bfloat16 or out.device != x.device \
                or not out.is_contiguous():
            raise ValueError(f"out must be a contiguous {tuple(x.shape)} bfloat16 tensor on {x.device}")
        y = out.view(-1, n)
    lib = _native.load()
    with torch.cuda.device(x.device):
        status = lib.sb_rms_norm(_stream_handle(x.device), x2.data_ptr(), w.data_ptr(), y.data_ptr(),
                                 x2.shape[0], n, SB_F32 if w.dtype == torch.float32 else SB_BF16,
                                 float(eps))
    _native.check(status)
    return y.reshape(x.shape)


def native_matmul(a, b):
    """Classical bf16 GEMM with fp32 accumulation (cuBLAS): the comparison arm.

    Mirrors strassen_pallas.native_matmul (strassen_pallas.py:1414-1421).
    """
    return torch.matmul(a, b).to(a.dtype)

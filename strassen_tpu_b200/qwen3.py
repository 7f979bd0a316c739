"""Qwen3 dense decoder prefill -- the caller of the Strassen operator, tensor-parallel.

Mirrors the reference's Qwen3 block composition
(experiments/qwen3/benchmark_qwen3_32b_layer.py:344-398,
benchmark_qwen3_32b_full_layer_product_inference.py:138-176): RMSNorm -> q/k
projections with the fused per-head RMSNorm + RoPE epilogue -> v -> causal
attention -> o projection + residual -> RMSNorm -> gate/up projection with the
fused SwiGLU epilogue -> down projection + residual.  Attention itself is not on
the hot path (torch SDPA, as the reference uses XLA's dot_product_attention).

Tensor parallelism over ``torch.distributed`` (NCCL on B200, gloo for CPU tests):
q/k/v/gate/up are split by output columns (whole heads / whole SwiGLU channel
pairs per rank), o/down by input rows; the o and down partial outputs are summed
with one all-reduce each.  Rank 0 fuses the residual into its o/down GEMM
epilogue, so the all-reduce adds it exactly once.

Backends: ``"strassen"`` runs every eligible site on the sm_100a kernels
(strassen_matmul with the reference's fused epilogues, rms_norm row kernel);
``"native"`` is the reference's XLA-classical arm (torch.matmul = cuBLAS on GPU,
unfused torch math) and is also what the CPU multi-process tests run.  A site
whose per-rank width no 256-multiple tile divides (k and v at TP=8: one
128-wide kv head, below the reference's bn = 2*head_dim) runs on 128-wide tiles
(strassen_matmul(narrow_bn=True), a B200 extension: one head per tile, so the
weight needs no relayout); a site that fits neither uses the native arm, the
same per-site choice the reference's harness makes.  ``native_sites`` moves
named sites to the native arm as well; :func:`measured_native_sites` chooses
them by timing every site of one layer of the shard on both arms (rank 0
times, every rank receives the choice), as the reference's harness picks
sites from its measurements.  Large Strassen sites run on the planes path
(``strassen_matmul`` takes the workspace it asks for from torch's caching
allocator); small-K shards stay on the one-CTA kernel.

Weights are random (N(0, 0.02); norm weights 1 + N(0, 0.02)) from per-tensor
seeds: every rank generates the same full tensor and keeps its shard.
"""

from __future__ import annotations

import math
from dataclasses import dataclass, field

import torch
import torch.nn.functional as F

from . import layouts
from . import strassen as sp


@dataclass(frozen=True)
class Qwen3Config:
    hidden: int
    layers: int
    heads: int
    kv_heads: int
    head_dim: int
    intermediate: int
    vocab: int = 151936
    rope_theta: float = 1e6
    rms_eps: float = 1e-6


# BASELINE.json configs 4 and 5, plus a small shape for tests.
QWEN3_8B = Qwen3Config(hidden=4096, layers=36, heads=32, kv_heads=8, head_dim=128, intermediate=12288)
QWEN3_32B = Qwen3Config(hidden=5120, layers=64, heads=64, kv_heads=8, head_dim=128, intermediate=25600)
QWEN3_TINY = Qwen3Config(hidden=512, layers=2, heads=8, kv_heads=4, head_dim=64, intermediate=1024,
                         vocab=1000)


@dataclass(frozen=True)
class StrassenTiles:
    """The reference's per-site (bm, bn, bk) choices; bn is capped per site so it
    divides the rank-local width."""

    bm: int = 1024
    bk: int = 512
    qk_bn: int = 1024
    up_bn: int = 1024
    bn: int = 1024


class TensorParallel:
    """Rank, world size and the one collective the decoder needs: the sum of the
    row-parallel projections' partial products plus the residual.

    ``collective="nccl"``: rank 0 adds the residual in its GEMM epilogue and an
    NCCL all-reduce sums the partials in place.  ``collective="p2p"``: the GEMMs
    write into a symmetric peer buffer and ``sb_p2p_reduce`` sums them with the
    residual over NVLink peer memory (:mod:`strassen_tpu_b200.p2p`); its
    buffers are sized by :meth:`ensure_buffers` before the first forward.
    """

    def __init__(self, group=None, collective: str = "nccl"):
        import torch.distributed as dist
        if collective not in ("nccl", "p2p"):
            raise ValueError(f"collective must be 'nccl' or 'p2p', got {collective!r}")
        self.dist = dist if dist.is_available() and dist.is_initialized() else None
        self.group = group
        self.rank = self.dist.get_rank(group) if self.dist else 0
        self.world = self.dist.get_world_size(group) if self.dist else 1
        self.collective = collective
        self.peer = None

    @property
    def peer_reduce(self) -> bool:
        """Whether the row-parallel sums run as sb_p2p_reduce (p2p, more than one rank)."""
        return self.collective == "p2p" and self.world > 1

    def ensure_buffers(self, rows: int, cols: int, device) -> None:
        """Size the p2p buffers for `rows` x `cols` partials (every rank calls it)."""
        if not self.peer_reduce:
            return
        if self.peer is None or self.peer.rows < rows or self.peer.cols != cols:
            from .p2p import PeerReduce
            if self.peer is not None:
                self.peer.close()
            self.peer = PeerReduce(rows, cols, device, group=self.group)

    def partial_out(self, row0: int, rows: int):
        """Where a row-parallel GEMM writes its partial for token rows row0:row0+rows
        (a peer-buffer view for p2p; None lets the GEMM allocate)."""
        if not self.peer_reduce:
            return None
        if self.peer is None:
            raise RuntimeError("collective='p2p' needs ensure_buffers(rows, hidden, device) before the "
                               "first row-parallel projection (Qwen3Prefill.forward calls it)")
        return self.peer.partial_rows(row0, row0 + rows)

    def all_reduce(self, x: torch.Tensor, residual: torch.Tensor | None = None) -> torch.Tensor:
        """Sum of x over the ranks (+ residual for p2p; nccl expects it fused on rank 0)."""
        if self.peer_reduce:
            return self.peer.reduce(x, residual)
        if self.world > 1:
            self.dist.all_reduce(x, group=self.group)
        return x

    def all_reduce_async(self, x: torch.Tensor, residual: torch.Tensor | None = None):
        """Start the sum; returns (result, handle) where handle.wait() orders the
        caller's stream after it (handle None on one rank)."""
        if self.peer_reduce:
            return self.peer.reduce(x, residual, async_op=True)
        if self.world > 1:
            return x, self.dist.all_reduce(x, group=self.group, async_op=True)
        return x, None

    def close(self) -> None:
        """Free the p2p buffers (every rank calls it, before the process group goes)."""
        if self.peer is not None:
            self.peer.close()
            self.peer = None


def _pick_bn(width: int, preferred: int, minimum: int) -> int | None:
    """Largest bn <= preferred that is a multiple of `minimum` and of 256 and divides width."""
    bn = preferred
    while bn >= max(minimum, 256):
        if width % bn == 0 and bn % 256 == 0 and bn % minimum == 0:
            return bn
        bn //= 2
    return None


def _narrow_bn(width: int, head_dim: int) -> int | None:
    """bn = 128 for a rank-local width that no 256-multiple tile divides (one
    128-wide head per rank: k and v of Qwen3-8B at TP=8), under
    strassen_matmul(narrow_bn=True); qk_norm_rope then needs head_dim | 128."""
    if width % 128 == 0 and 128 % head_dim == 0:
        return 128
    return None


def _randn(shape, seed, device, scale=0.02, offset=0.0):
    g = torch.Generator(device=device)
    g.manual_seed(seed)
    w = torch.randn(shape, generator=g, device=device, dtype=torch.float32)
    return (w * scale + offset).to(torch.bfloat16)


def rms_norm_torch(x, scale, eps):
    """benchmark_qwen3_32b_layer.py:270-276 in torch (fp32 math, bf16 out)."""
    x32 = x.float()
    return (x32 * torch.rsqrt((x32 * x32).mean(-1, keepdim=True) + eps) * scale.float()).to(torch.bfloat16)


def apply_rope_torch(x, cos, sin):
    """benchmark_qwen3_32b_layer.py:278-284: rotate-half RoPE in fp32. x [T, H, D], cos/sin [T, D]."""
    x32 = x.float()
    first, second = x32.chunk(2, dim=-1)
    rotated = torch.cat((-second, first), dim=-1)
    return (x32 * cos[:, None, :].float() + rotated * sin[:, None, :].float()).to(torch.bfloat16)


def rope_tables(positions: torch.Tensor, cfg: Qwen3Config):
    """bf16 cos/sin [len(positions), head_dim] (benchmark_qwen3_32b_layer.py:258-267)."""
    hd = cfg.head_dim
    inv = 1.0 / (cfg.rope_theta ** (torch.arange(0, hd, 2, dtype=torch.float32,
                                                  device=positions.device) / hd))
    ang = positions.float()[:, None] * inv[None, :]
    ang = torch.cat((ang, ang), dim=-1)
    return torch.cos(ang).to(torch.bfloat16), torch.sin(ang).to(torch.bfloat16)


@dataclass
class _Site:
    weight: torch.Tensor          # [K, N_rank] as the site's GEMM consumes it
    strassen: bool
    bn: int | None = None
    narrow: bool = False          # bn = 128 under strassen_matmul(narrow_bn=True)


@dataclass
class Qwen3Layer:
    cfg: Qwen3Config
    tp: TensorParallel
    backend: str
    tiles: StrassenTiles
    ln1: torch.Tensor = None
    ln2: torch.Tensor = None
    q_norm: torch.Tensor = None
    k_norm: torch.Tensor = None
    sites: dict = field(default_factory=dict)

    @property
    def heads_rank(self):
        return self.cfg.heads // self.tp.world

    @property
    def kv_rank(self):
        return self.cfg.kv_heads // self.tp.world

    @property
    def inter_rank(self):
        return self.cfg.intermediate // self.tp.world


def build_layer(cfg: Qwen3Config, index: int, tp: TensorParallel, device, backend="strassen",
                tiles: StrassenTiles = StrassenTiles(), seed: int = 20260910,
                native_sites=frozenset()) -> Qwen3Layer:
    """Random-init layer `index`, sharded for this rank and laid out for the fused epilogues.

    ``native_sites``: GEMM sites (q, k, v, o, up, down) that take the native arm
    even where a Strassen tile fits (see :func:`measured_native_sites`)."""
    if cfg.heads % tp.world or cfg.kv_heads % tp.world or cfg.intermediate % tp.world:
        raise ValueError(f"tensor parallel size {tp.world} does not divide heads/kv heads/intermediate")
    hd, r, w = cfg.head_dim, tp.rank, tp.world
    base = seed + 1000 * index
    layer = Qwen3Layer(cfg=cfg, tp=tp, backend=backend, tiles=tiles)
    layer.ln1 = _randn((cfg.hidden,), base + 1, device, offset=1.0)
    layer.ln2 = _randn((cfg.hidden,), base + 2, device, offset=1.0)
    layer.q_norm = _randn((hd,), base + 3, device, offset=1.0)
    layer.k_norm = _randn((hd,), base + 4, device, offset=1.0)
    hq, hkv, ir = cfg.heads // w, cfg.kv_heads // w, cfg.intermediate // w
    use = backend == "strassen"

    def cols(full, lo, hi):
        return full[:, lo:hi].contiguous()

    wq = cols(_randn((cfg.hidden, cfg.heads * hd), base + 10, device), r * hq * hd, (r + 1) * hq * hd)
    wk = cols(_randn((cfg.hidden, cfg.kv_heads * hd), base + 11, device), r * hkv * hd, (r + 1) * hkv * hd)
    wv = cols(_randn((cfg.hidden, cfg.kv_heads * hd), base + 12, device), r * hkv * hd, (r + 1) * hkv * hd)
    wo = _randn((cfg.heads * hd, cfg.hidden), base + 13, device)[r * hq * hd:(r + 1) * hq * hd].contiguous()
    wg = cols(_randn((cfg.hidden, cfg.intermediate), base + 14, device), r * ir, (r + 1) * ir)
    wu = cols(_randn((cfg.hidden, cfg.intermediate), base + 15, device), r * ir, (r + 1) * ir)
    wd = _randn((cfg.intermediate, cfg.hidden), base + 16, device)[r * ir:(r + 1) * ir].contiguous()

    for name, wt in (("q", wq), ("k", wk)):
        on = use and name not in native_sites
        bn = _pick_bn(wt.shape[1], tiles.qk_bn, 2 * hd) if on else None
        narrow = _narrow_bn(wt.shape[1], hd) if on and bn is None and hd == 128 else None
        if bn is not None:
            layer.sites[name] = _Site(layouts.rope_weight_layout(wt, bn, head_dim=hd), True, bn)
        elif narrow is not None:
            # 128-wide tiles hold one head each, already in the a|b half order
            # qk_norm_rope reads (first half-head, then its rotation partners).
            layer.sites[name] = _Site(wt, True, narrow, narrow=True)
        else:
            layer.sites[name] = _Site(wt, False)
    on = use and "v" not in native_sites
    bn = _pick_bn(wv.shape[1], tiles.bn, 256) if on else None
    if bn is None and on and _narrow_bn(wv.shape[1], 1) is not None:
        layer.sites["v"] = _Site(wv, True, 128, narrow=True)
    else:
        layer.sites["v"] = _Site(wv, bn is not None, bn)
    on = use and "o" not in native_sites
    bn = _pick_bn(cfg.hidden, tiles.bn, 256) if on and wo.shape[0] % tiles.bk == 0 else None
    layer.sites["o"] = _Site(wo, bn is not None, bn)
    gate_up = torch.cat([wg, wu], dim=1)
    bn = _pick_bn(2 * ir, tiles.up_bn, 256) if use and "up" not in native_sites else None
    if bn is not None and ir % (bn // 2) == 0:
        layer.sites["up"] = _Site(layouts.swiglu_weight_layout(gate_up, bn), True, bn)
    else:
        layer.sites["up"] = _Site(gate_up, False)
    on = use and "down" not in native_sites
    bn = _pick_bn(cfg.hidden, tiles.bn, 256) if on and ir % tiles.bk == 0 else None
    layer.sites["down"] = _Site(wd, bn is not None, bn)
    return layer


def _qk(layer: Qwen3Layer, name: str, h, heads, norm_w, cos, sin, cos_laid, sin_laid):
    cfg = layer.cfg
    site = layer.sites[name]
    t = h.shape[0]
    if site.strassen:
        bn = site.bn
        scale = layouts.rope_scale_layout(norm_w, bn, head_dim=cfg.head_dim)
        c, s = cos_laid[bn], sin_laid[bn]
        flat = sp.strassen_matmul(h, site.weight, bm=layer.tiles.bm, bn=bn, bk=layer.tiles.bk,
                                  epilogue="qk_norm_rope", rope_cos=c, rope_sin=s, rope_scale=scale,
                                  rope_head_dim=cfg.head_dim, rope_eps=cfg.rms_eps,
                                  narrow_bn=site.narrow)
        return layouts.rope_layout_to_heads(flat, heads, bn, head_dim=cfg.head_dim)
    x = sp.native_matmul(h, site.weight).view(t, heads, cfg.head_dim)
    x = rms_norm_torch(x, norm_w, cfg.rms_eps)
    return apply_rope_torch(x, cos, sin)


def _plain(layer: Qwen3Layer, name: str, h, residual=None, out=None):
    site = layer.sites[name]
    if site.strassen:
        kw = {}
        if residual is not None:
            kw = dict(epilogue="residual_add", residual=residual)
        return sp.strassen_matmul(h, site.weight, bm=layer.tiles.bm, bn=site.bn, bk=layer.tiles.bk,
                                  out=out, narrow_bn=site.narrow, **kw)
    res = sp.native_matmul(h, site.weight)
    if residual is not None:
        res = (res.float() + residual.float()).to(torch.bfloat16)
    if out is not None:
        out.copy_(res)
        return out
    return res


def _row_parallel(layer: Qwen3Layer, name: str, h, residual, row0: int):
    """A row-parallel projection: (this rank's partial, the residual the sum still
    needs).  nccl: rank 0 adds the residual in its epilogue; p2p: the partial
    lands in the peer buffer and the reduce adds the residual."""
    tp = layer.tp
    if getattr(tp, "peer_reduce", False):
        return _plain(layer, name, h, out=tp.partial_out(row0, h.shape[0])), residual
    return _plain(layer, name, h, residual=residual if tp.rank == 0 else None), None


def _attention_half(layer: Qwen3Layer, x: torch.Tensor, batch: int, seq: int, rope, row0: int = 0):
    """ln1 -> q/k/v (fused qk_norm_rope) -> causal attention -> o projection:
    this rank's partial sum of the new hidden state and the residual still to
    add (_row_parallel).  row0: x's first row in the forward's token batch."""
    cfg, tp = layer.cfg, layer.tp
    cos, sin, cos_laid, sin_laid = rope
    norm = sp.rms_norm if layer.backend == "strassen" else (lambda a, b, eps: rms_norm_torch(a, b, eps))
    h = norm(x, layer.ln1, cfg.rms_eps)
    hq, hkv, hd = layer.heads_rank, layer.kv_rank, cfg.head_dim
    q = _qk(layer, "q", h, hq, layer.q_norm, cos, sin, cos_laid, sin_laid)
    k = _qk(layer, "k", h, hkv, layer.k_norm, cos, sin, cos_laid, sin_laid)
    v = _plain(layer, "v", h).view(-1, hkv, hd)
    q4 = q.view(batch, seq, hq, hd).transpose(1, 2)
    k4 = k.view(batch, seq, hkv, hd).transpose(1, 2)
    v4 = v.view(batch, seq, hkv, hd).transpose(1, 2)
    # Grouped-query attention without materialising the repeated k/v heads (the
    # same result as repeat_interleave, bit for bit; 0.25 vs 0.59 ms at 8 x 2048
    # tokens, 32 q / 8 kv heads on a B200).
    attn = F.scaled_dot_product_attention(q4, k4, v4, is_causal=True, enable_gqa=hkv != hq)
    attn = attn.transpose(1, 2).reshape(batch * seq, hq * hd)
    return _row_parallel(layer, "o", attn, x, row0)


def _mlp_half(layer: Qwen3Layer, x1: torch.Tensor, row0: int = 0):
    """ln2 -> gate/up (fused SwiGLU) -> down projection: this rank's partial sum
    of the block output and the residual still to add (_row_parallel)."""
    cfg, tp = layer.cfg, layer.tp
    norm = sp.rms_norm if layer.backend == "strassen" else (lambda a, b, eps: rms_norm_torch(a, b, eps))
    h2 = norm(x1, layer.ln2, cfg.rms_eps)
    up = layer.sites["up"]
    if up.strassen:
        g = sp.strassen_matmul(h2, up.weight, bm=layer.tiles.bm, bn=up.bn, bk=layer.tiles.bk,
                               epilogue="swiglu", product_aware_swiglu=True, interleave_products=True)
    else:
        gu = sp.native_matmul(h2, up.weight).float()
        gate, upv = gu.chunk(2, dim=-1)
        g = (F.silu(gate) * upv).to(torch.bfloat16)
    return _row_parallel(layer, "down", g, x1, row0)


def layer_forward(layer: Qwen3Layer, x: torch.Tensor, batch: int, seq: int, rope) -> torch.Tensor:
    """One decoder block on x [batch*seq, hidden] (bf16); returns the new hidden state.

    The composition of benchmark_qwen3_32b_layer.py:344-398 with the row-parallel
    o and down projections each followed by one all-reduce."""
    tp = layer.tp
    x1 = tp.all_reduce(*_attention_half(layer, x, batch, seq, rope))
    return tp.all_reduce(*_mlp_half(layer, x1))


def _chunk_rope(rope, lo: int, hi: int):
    """Rows lo:hi of the per-token rope tables (the laid-out ones included)."""
    cos, sin, cos_laid, sin_laid = rope
    return (cos[lo:hi], sin[lo:hi], {k: v[lo:hi] for k, v in cos_laid.items()},
            {k: v[lo:hi] for k, v in sin_laid.items()})


def forward_blocks_chunked(blocks, x: torch.Tensor, batch: int, seq: int, rope, chunks: int) -> torch.Tensor:
    """All decoder blocks on x, software-pipelined over `chunks` groups of whole
    sequences so each chunk's all-reduces overlap the other chunks' compute.

    Per block and chunk the math is exactly layer_forward's (attention never
    crosses a sequence, every other op is per token); only the order changes:
    chunk i's o-projection all-reduce runs while chunk i+1 computes attention,
    and its down-projection all-reduce while the other chunks compute, up to the
    next block's use of chunk i.
    """
    if chunks <= 1 or batch % chunks:
        for blk in blocks:
            x = layer_forward(blk, x, batch, seq, rope)
        return x
    tp = blocks[0].tp
    per = batch // chunks
    rows = per * seq
    xs = [x[i * rows:(i + 1) * rows] for i in range(chunks)]
    ropes = [_chunk_rope(rope, i * rows, (i + 1) * rows) for i in range(chunks)]
    pending = [None] * chunks  # all-reduce in flight on xs[i]
    for blk in blocks:
        mids = []
        for i in range(chunks):
            if pending[i] is not None:
                pending[i].wait()
            part, res = _attention_half(blk, xs[i], per, seq, ropes[i], row0=i * rows)
            mids.append(tp.all_reduce_async(part, res))
        for i, (x1, work) in enumerate(mids):
            if work is not None:
                work.wait()
            part, res = _mlp_half(blk, x1, row0=i * rows)
            xs[i], pending[i] = tp.all_reduce_async(part, res)
    for work in pending:
        if work is not None:
            work.wait()
    return torch.cat(xs)


class Qwen3Prefill:
    """Embedding -> N decoder blocks -> final norm -> last-position logits.

    The LM head scores only the last position of each sequence (prefill serving
    semantics); the vocabulary projection is replicated on every rank.
    """

    def __init__(self, cfg: Qwen3Config, tp: TensorParallel, device, backend="strassen",
                 tiles: StrassenTiles = StrassenTiles(), layers: int | None = None, seed=20260910,
                 native_sites=frozenset()):
        self.cfg, self.tp, self.device, self.backend = cfg, tp, device, backend
        self.embed = _randn((cfg.vocab, cfg.hidden), seed, device)
        self.final_norm = _randn((cfg.hidden,), seed + 7, device, offset=1.0)
        self.lm_head = _randn((cfg.hidden, cfg.vocab), seed + 8, device)
        n = cfg.layers if layers is None else layers
        self.native_sites = frozenset(native_sites)
        self.blocks = [build_layer(cfg, i, tp, device, backend, tiles, seed, self.native_sites) for i in range(n)]

    def rope(self, batch: int, seq: int):
        pos = torch.arange(seq, device=self.device).repeat(batch)
        cos, sin = rope_tables(pos, self.cfg)
        cos_laid, sin_laid = {}, {}
        for blk in self.blocks[:1]:
            for site in ("q", "k"):
                s = blk.sites[site]
                if s.strassen and s.bn not in cos_laid:
                    c, si = layouts.rope_layout_tables(cos, sin, s.bn // 2, head_dim=self.cfg.head_dim)
                    cos_laid[s.bn], sin_laid[s.bn] = c.contiguous(), si.contiguous()
        return cos, sin, cos_laid, sin_laid

    def forward(self, tokens: torch.Tensor, rope=None, chunks: int = 1) -> torch.Tensor:
        """tokens [batch, seq] int64 -> logits [batch, vocab] of the last positions.

        chunks > 1 pipelines the blocks over groups of whole sequences so that
        the all-reduces overlap compute (forward_blocks_chunked); batch must be a
        multiple of chunks, else the blocks run unchunked."""
        batch, seq = tokens.shape
        rope = rope if rope is not None else self.rope(batch, seq)
        self.tp.ensure_buffers(batch * seq, self.cfg.hidden, self.device)
        x = self.embed[tokens.reshape(-1)]
        x = forward_blocks_chunked(self.blocks, x, batch, seq, rope, chunks)
        last = x.view(batch, seq, -1)[:, -1]
        last = rms_norm_torch(last, self.final_norm, self.cfg.rms_eps)
        return sp.native_matmul(last, self.lm_head)


class CapturedPrefill:
    """A CUDA-graph capture of ``Qwen3Prefill.forward`` for one token shape.

    Replaying the graph launches the whole prefill (every block, the kernels,
    torch ops and the NCCL all-reduces) without per-op host work, which bounds
    the chunk-pipelined forward at high TP.  Call with a tokens tensor of the
    captured shape: it is copied into the graph's input, the graph is replayed
    on the current stream, and the graph's logits tensor is returned (overwritten
    by the next call).  ``release()`` frees the graph; a graph holding NCCL
    calls must be released before the process group is destroyed.
    """

    def __init__(self, model: "Qwen3Prefill", tokens: torch.Tensor, rope=None, chunks: int = 1,
                 warmup: int = 2):
        self.model = model
        self.tokens = tokens.clone()
        batch, seq = tokens.shape
        self.rope = rope if rope is not None else model.rope(batch, seq)
        self.chunks = chunks
        side = torch.cuda.Stream(tokens.device)
        side.wait_stream(torch.cuda.current_stream(tokens.device))
        with torch.cuda.stream(side):
            for _ in range(warmup):
                model.forward(self.tokens, self.rope, chunks=chunks)
        torch.cuda.current_stream(tokens.device).wait_stream(side)
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph):
            self.logits = model.forward(self.tokens, self.rope, chunks=chunks)

    def __call__(self, tokens: torch.Tensor) -> torch.Tensor:
        if tokens.shape != self.tokens.shape:
            raise ValueError(f"captured for tokens {tuple(self.tokens.shape)}, got {tuple(tokens.shape)}")
        self.tokens.copy_(tokens, non_blocking=True)
        self.graph.replay()
        return self.logits

    def release(self) -> None:
        self.graph = None
        self.logits = None


def prefill_flops(cfg: Qwen3Config, batch: int, seq: int, layers: int | None = None) -> float:
    """GEMM + causal-attention FLOPs of one prefill (LM head on last positions only)."""
    n = cfg.layers if layers is None else layers
    t = batch * seq
    hd = cfg.head_dim
    gemm = 2 * t * cfg.hidden * (cfg.heads * hd + 2 * cfg.kv_heads * hd) \
        + 2 * t * cfg.heads * hd * cfg.hidden + 2 * t * cfg.hidden * 2 * cfg.intermediate \
        + 2 * t * cfg.intermediate * cfg.hidden
    attn = 2 * 2 * batch * cfg.heads * hd * seq * seq / 2
    return n * (gemm + attn) + 2 * batch * cfg.hidden * cfg.vocab


class _Shard:
    """Rank and world size of one tensor-parallel shard, without a process group."""

    def __init__(self, rank: int, world: int):
        self.rank, self.world = rank, world


def site_times(cfg: Qwen3Config, world: int, tokens: int, device, steps: int = 20, warmup: int = 3,
               seq: int = 2048) -> dict:
    """Device time (ms, CUDA events, mean of `steps` calls) of every op of one
    decoder layer of rank 0's shard at tensor-parallel size `world`, for both
    backends, on one GPU: the per-rank shapes of a TP=`world` prefill on `tokens`
    token rows (``tokens // seq`` whole sequences), without its collectives.

    Returns {op: {"strassen": ms, "native": ms, "strassen_site": bool, "bn": int|None}}
    for ln1, q, k, v, attention, o, ln2, up, down, where o and down include the
    residual add that rank 0 fuses.  Sites whose shard fits no Strassen tile run
    the native arm in both columns (strassen_site False)."""
    shard = _Shard(0, world)
    layers = {b: build_layer(cfg, 0, shard, device, backend=b) for b in ("strassen", "native")}
    model = Qwen3Prefill.__new__(Qwen3Prefill)
    model.cfg, model.device, model.blocks = cfg, device, [layers["strassen"]]
    batch = max(1, tokens // seq)
    rope = model.rope(batch, seq)
    cos, sin, cos_laid, sin_laid = rope
    g = torch.Generator(device=device).manual_seed(20260912)
    x = torch.randn(tokens, cfg.hidden, device=device, generator=g).to(torch.bfloat16)
    hq, hkv, hd, ir = cfg.heads // world, cfg.kv_heads // world, cfg.head_dim, cfg.intermediate // world
    attn_in = torch.randn(tokens, hq * hd, device=device, generator=g).to(torch.bfloat16)
    g_in = torch.randn(tokens, ir, device=device, generator=g).to(torch.bfloat16)
    qkv = [torch.randn(batch, n, seq, hd, device=device, generator=g).to(torch.bfloat16) for n in (hq, hkv, hkv)]

    def ops(layer):
        norm = sp.rms_norm if layer.backend == "strassen" else (lambda a, b, eps: rms_norm_torch(a, b, eps))

        def up():
            site = layer.sites["up"]
            if site.strassen:
                return sp.strassen_matmul(x, site.weight, bm=layer.tiles.bm, bn=site.bn, bk=layer.tiles.bk,
                                          epilogue="swiglu", product_aware_swiglu=True, interleave_products=True)
            gu = sp.native_matmul(x, site.weight).float()
            gate, upv = gu.chunk(2, dim=-1)
            return (F.silu(gate) * upv).to(torch.bfloat16)

        return {
            "ln1": lambda: norm(x, layer.ln1, cfg.rms_eps),
            "q": lambda: _qk(layer, "q", x, hq, layer.q_norm, cos, sin, cos_laid, sin_laid),
            "k": lambda: _qk(layer, "k", x, hkv, layer.k_norm, cos, sin, cos_laid, sin_laid),
            "v": lambda: _plain(layer, "v", x),
            "attention": lambda: F.scaled_dot_product_attention(*qkv, is_causal=True, enable_gqa=hkv != hq),
            "o": lambda: _plain(layer, "o", attn_in, residual=x),
            "ln2": lambda: norm(x, layer.ln2, cfg.rms_eps),
            "up": up,
            "down": lambda: _plain(layer, "down", g_in, residual=x),
        }

    def timed(fn):
        for _ in range(warmup):
            fn()
        torch.cuda.synchronize(device)
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        start.record()
        for _ in range(steps):
            fn()
        end.record()
        torch.cuda.synchronize(device)
        return start.elapsed_time(end) / steps

    out = {}
    s_ops, n_ops = ops(layers["strassen"]), ops(layers["native"])
    for name in s_ops:
        site = layers["strassen"].sites.get(name)
        out[name] = {"strassen": timed(s_ops[name]), "native": timed(n_ops[name]),
                     "strassen_site": bool(site.strassen) if site is not None else None,
                     "bn": site.bn if site is not None and site.strassen else None}
    return out


GEMM_SITES = ("q", "k", "v", "o", "up", "down")


def measured_native_sites(cfg: Qwen3Config, tp, tokens: int, device, seq: int = 2048, steps: int = 10,
                          warmup: int = 3) -> frozenset:
    """The GEMM sites whose native arm (cuBLAS + unfused torch epilogue) is faster
    than the Strassen site at this rank's shard shapes: the per-site choice the
    reference's harness makes from measurements (it runs Strassen only at the
    sites where it wins).  Rank 0 of ``tp``'s group times one layer with
    :func:`site_times` on ``tokens`` token rows and every rank takes its answer,
    so all ranks run the same kernels."""
    choice = None
    if tp.rank == 0:
        times = site_times(cfg, tp.world, tokens, device, steps=steps, warmup=warmup, seq=seq)
        choice = sorted(name for name in GEMM_SITES
                        if times[name]["strassen_site"] and times[name]["native"] < times[name]["strassen"])
    if tp.world > 1:
        box = [choice]
        src = tp.dist.get_global_rank(tp.group, 0) if tp.group is not None else 0
        tp.dist.broadcast_object_list(box, src=src, group=tp.group)
        choice = box[0]
    return frozenset(choice)

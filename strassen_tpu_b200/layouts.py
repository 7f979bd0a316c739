"""Offline weight / table relayouts that put epilogue partners in one tile.

These are the host-side helpers of the reference operator API
(strassen_pallas.py:1315-1411) plus the inverse relayout the Qwen3 harness
uses (experiments/qwen3/benchmark_qwen3_32b_layer.py:322-341).  They are pure
column permutations and work on ``torch.Tensor`` or ``numpy.ndarray`` inputs
(the result has the input's type).  The column orders are the reference's,
because the kernel's quadrant split -- quadrants 0/2 are the left half of each
``bn`` block, 1/3 the right half -- is what they are built to feed.
"""

from __future__ import annotations

import numpy as np

try:  # torch is optional: the helpers also serve numpy callers (tests, fixture scripts)
    import torch
except ImportError:  # pragma: no cover
    torch = None


def _is_torch(x) -> bool:
    return torch is not None and isinstance(x, torch.Tensor)


def _take_columns(x, order):
    if _is_torch(x):
        return x.index_select(-1, torch.as_tensor(order, dtype=torch.long, device=x.device))
    return np.asarray(x)[..., np.asarray(order, dtype=np.int64)]


def _tile(x, reps):
    if _is_torch(x):
        return x.repeat(*reps)
    return np.tile(x, reps)


def _concat(parts):
    if _is_torch(parts[0]):
        return torch.cat(parts)
    return np.concatenate(parts)


def _paired_halves(width: int, bn: int, partner_offset, source_of) -> list[int]:
    """Column order that puts, per ``bn`` block of the output, ``h = bn/2``
    consecutive "left" columns in the block's first half and their partners in
    its second half.

    Output column ``j`` lies in block ``j // bn`` at offset ``o = j % bn``; it
    takes the left list's entry ``i = (j // bn) * h + o % h``, and the partner
    of that entry when ``o >= h``.  ``source_of(i)`` maps list entries to
    source columns and ``partner_offset(i)`` gives the partner's distance.
    """
    j = np.arange(width, dtype=np.int64)
    h = bn // 2
    i = (j // bn) * h + (j % bn) % h
    return (source_of(i) + np.where((j % bn) >= h, partner_offset(i), 0)).tolist()


def rope_weight_order(n: int, bn: int, head_dim: int = 128) -> list[int]:
    """Column order of :func:`rope_weight_layout` (strassen_pallas.py:1315-1349).

    The left list holds every head's first ``head_dim/2`` channels in head
    order (entry ``i`` is channel ``i % (head_dim/2)`` of head
    ``i // (head_dim/2)``); each partner is the channel ``head_dim/2`` further
    on, its rotation pair.  Checks and messages follow the reference.
    """
    if n % head_dim:
        raise ValueError(f"width {n} is not a multiple of head_dim {head_dim}")
    if bn % (2 * head_dim):
        raise ValueError(
            f"bn={bn} must be a multiple of 2*head_dim={2 * head_dim} so each "
            "tile half holds whole heads")
    half_head = head_dim // 2
    if (n // 2) % (bn // 2):
        raise ValueError(f"half width {n // 2} is not divisible by bn//2={bn // 2}")
    return _paired_halves(n, bn, lambda i: half_head,
                          lambda i: (i // half_head) * head_dim + i % half_head)


def rope_weight_layout(weight, bn: int, head_dim: int = 128):
    """Reorder a q/k projection weight [K, heads*head_dim] for ``qk_norm_rope``.

    Per ``bn`` block the columns become ``a[0:h] b[0:h]`` with ``h = bn/2``,
    where ``a`` lists every head's first-half channels and ``b`` the matching
    rotation partners, so quadrants 0/2 of a tile hold ``a`` and 1/3 hold ``b``
    (strassen_pallas.py:1315-1349).
    """
    return _take_columns(weight, rope_weight_order(weight.shape[-1], bn, head_dim))


def rope_layout_tables(cos, sin, half_width: int, head_dim: int = 128):
    """Half-width RoPE tables [positions, half_width] (strassen_pallas.py:1352-1368)."""
    half_head = head_dim // 2
    if half_width % half_head:
        raise ValueError(f"half_width {half_width} is not a multiple of {half_head}")
    repeats = half_width // half_head
    return _tile(cos[:, :half_head], (1, repeats)), _tile(sin[:, :half_head], (1, repeats))


def rope_scale_layout(scale, bn: int, head_dim: int = 128):
    """Per-head RMSNorm scale [head_dim] laid out to [bn] (strassen_pallas.py:1371-1378)."""
    half_head = head_dim // 2
    repeats = (bn // 2) // half_head
    return _concat([_tile(scale[:half_head], (repeats,)), _tile(scale[half_head:], (repeats,))])


def swiglu_weight_order(two_i: int, bn: int) -> list[int]:
    """Column order of :func:`swiglu_weight_layout` (strassen_pallas.py:1381-1411).

    The left list is the gate columns ``0 .. I-1`` in order; each partner is
    the up column ``I`` further on.  Checks and messages follow the reference.
    """
    if two_i % 2:
        raise ValueError(f"combined gate/up width {two_i} is not even")
    intermediate = two_i // 2
    if intermediate % (bn // 2):
        raise ValueError(f"intermediate {intermediate} is not divisible by bn//2={bn // 2}")
    return _paired_halves(two_i, bn, lambda i: intermediate, lambda i: i)


def swiglu_weight_layout(gate_up, bn: int):
    """Reorder a combined ``[gate | up]`` weight [K, 2I] so SwiGLU fuses in-kernel.

    Per ``bn`` block the columns become ``gate[0:h] up[0:h]`` with ``h = bn/2``
    (strassen_pallas.py:1381-1411): quadrants 0/2 are gate, 1/3 are up.
    """
    return _take_columns(gate_up, swiglu_weight_order(gate_up.shape[-1], bn))


def rope_layout_to_heads(flat, heads: int, bn: int, head_dim: int = 128):
    """Regroup a ``qk_norm_rope`` output [tokens, heads*head_dim] to [tokens, heads, head_dim].

    Inverse of the rope column layout
    (experiments/qwen3/benchmark_qwen3_32b_layer.py:322-341): view each tile as
    (blocks, 2, heads_per_half, half_head) and swap the middle axes.
    """
    half_head = head_dim // 2
    heads_per_half = (bn // 2) // half_head
    blocks = (heads * head_dim) // bn
    tokens = flat.shape[0]
    x = flat.reshape(tokens, blocks, 2, heads_per_half, half_head)
    if _is_torch(x):
        x = x.permute(0, 1, 3, 2, 4)
    else:
        x = x.transpose(0, 1, 3, 2, 4)
    return x.reshape(tokens, heads, head_dim)

"""Tile classification of a packed verification mask (test infrastructure only).

The reference turns its dense float mask into a FlexAttention ``BlockMask``
with ``make_mask_mod`` (allowed <=> mask value > -0.1, D:148-153) and
``create_block_mask(..., BLOCK_SIZE=(128, 64))`` (D:94-106, H:1213-1221).
That torch routine evaluates the predicate over ``[Q, KV]``, pads both axes
up to whole tiles with *not allowed*, and classifies every 128x64 tile as
empty, partial or full.  ``kv_indices`` / ``full_kv_indices`` list, per
128-row query tile, the partial / full KV tiles in ascending order; only the
first ``kv_num_blocks`` / ``full_kv_num_blocks`` entries are meaningful.
"""
from __future__ import annotations

import numpy as np

Q_TILE = 128
KV_TILE = 64

EMPTY, PARTIAL, FULL = 0, 1, 2


def allowed_from_dense(mask) -> np.ndarray:
    """``make_mask_mod`` predicate (D:148-153): value > -0.1."""
    m = np.asarray(mask, dtype=np.float32)
    while m.ndim > 2:
        m = m[0]
    return m > -0.1


def tile_classes(allowed: np.ndarray, q_tile: int = Q_TILE,
                 kv_tile: int = KV_TILE) -> np.ndarray:
    """Per (query tile, KV tile) class: 0 empty, 1 partial, 2 full."""
    q, kv = allowed.shape
    nq = -(-q // q_tile)
    nk = -(-kv // kv_tile)
    pad = np.zeros((nq * q_tile, nk * kv_tile), dtype=bool)
    pad[:q, :kv] = allowed
    t = pad.reshape(nq, q_tile, nk, kv_tile)
    count = t.sum(axis=(1, 3))
    cls = np.where(count == 0, EMPTY,
                   np.where(count == q_tile * kv_tile, FULL, PARTIAL))
    return cls.astype(np.int32)


def block_mask_lists(allowed: np.ndarray):
    """``(kv_num_blocks, kv_indices, full_kv_num_blocks, full_kv_indices)``.

    Same meaning as the fields of torch's ``BlockMask`` built by
    ``create_block_mask`` at BLOCK_SIZE (128, 64); indices are returned as
    ragged Python lists (ascending), which is what the valid prefix of each
    torch row holds.
    """
    cls = tile_classes(allowed)
    partial = [list(np.nonzero(row == PARTIAL)[0]) for row in cls]
    full = [list(np.nonzero(row == FULL)[0]) for row in cls]
    return ([len(p) for p in partial], partial, [len(f) for f in full], full)


def executed_tiles(allowed: np.ndarray) -> int:
    """Number of 128x64 tiles FlexAttention runs (partial + full)."""
    return int((tile_classes(allowed) != EMPTY).sum())


def allowed_pairs(allowed: np.ndarray) -> int:
    return int(allowed.sum())

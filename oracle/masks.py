"""Packed verification masks (test infrastructure only).

Two views of the same mask:

* the reference's dense float mask ``[1, 1, Q, KV]`` (0 = allowed, -inf =
  masked), built at prefill by RD:232-245 and re-assembled every step by
  D:1634-1667 / D:1737-1748 (H:2186-2221 / H:2287-2301);
* the segment form the CUDA metadata kernel consumes: the packed query rows
  are split into segments; every row of a segment sees the segment's KV
  column set, plus an intra-segment pattern over the segment's own new
  columns (causal for speculative and prefill blocks, ancestor sets for tree
  blocks, ``[0, 0]`` only for normal blocks).

:func:`segments_to_allowed` expands the segment form; the functions named
after the reference restate its dense assembly so tests can check that the
two agree.
"""
from __future__ import annotations

import numpy as np
import torch

CAUSAL, TREE, SINGLE, NONE = 0, 1, 2, 3


def segments_to_allowed(q_len, kv_total, segments):
    """Dense bool ``[q_len, kv_total]`` from segment descriptors.

    Each segment is a dict with ``q_start``, ``q_len``, ``kind`` (CAUSAL /
    TREE / SINGLE / NONE), ``kv`` (bool ``[kv_total]`` visibility shared by
    all its rows) and, for TREE, ``parents`` (parent node index per real
    node; rows past ``len(parents)`` are padding).  The new columns of the
    step start at ``kv_total - q_len`` (D:1089 ``input_ids_in_attn_mask_start``).
    """
    base = kv_total - q_len
    out = np.zeros((q_len, kv_total), dtype=bool)
    for s in segments:
        qs, ql, kind = s["q_start"], s["q_len"], s["kind"]
        out[qs:qs + ql] |= np.asarray(s["kv"], dtype=bool)[None, :]
        c0 = base + qs
        if kind == CAUSAL:
            out[qs:qs + ql, c0:c0 + ql] |= np.tril(np.ones((ql, ql), bool))
        elif kind == SINGLE:
            out[qs, c0] = True
        elif kind == TREE:
            parents = s["parents"]
            for i in range(len(parents)):
                j = i
                while j >= 0:
                    out[qs + i, c0 + j] = True
                    j = parents[j]
    return out


def initial_packed_mask(block_lengths):
    """Prefill mask: block-diagonal causal over the packed input (RD:232-245)."""
    n = int(sum(block_lengths))
    pointer = np.cumsum(block_lengths) - 1
    causal = torch.ones((n, n), dtype=torch.bool)
    start = 0
    for p in pointer:
        end = int(p) + 1
        causal[start:end, start:end] = ~torch.tril(
            torch.ones((end - start, end - start), dtype=torch.bool))
        start = end
    mask = torch.zeros((1, 1, n, n), dtype=torch.float32)
    return mask.masked_fill(causal[None, None], float("-inf"))


def tree_block_mask(parents, padded_len):
    """Ancestor mask of a packed tree block (D:1488-1533)."""
    m = torch.zeros((padded_len, padded_len), dtype=torch.bool)
    for i in range(len(parents)):
        j = i
        while j >= 0:
            m[i, j] = True
            j = parents[j]
    return m


def normal_block_mask(length):
    """``_normal_causal_mask``: only [0, 0] allowed (D:1021-1025)."""
    m = torch.zeros((length, length), dtype=torch.bool)
    m[0, 0] = True
    return m


def spec_block_mask(length):
    """``_spec_tril_mask[:len, :len]`` (D:1027-1031, D:1442-1447)."""
    return torch.tril(torch.ones((length, length), dtype=torch.bool))


def assemble_next_mask(attention_mask, pointer, new_lengths, new_block_masks,
                       tight_pad_len=0, hunyuan=False):
    """Next-step dense mask, restating D:1634-1667 and D:1737-1748.

    ``attention_mask`` is the current mask *after* compaction
    (``index_select``) or dead-column ``masked_fill``; ``pointer`` holds,
    per block, the row of the current mask whose visibility the block's new
    rows inherit; ``new_lengths`` is each block's new row count (0 for
    finished blocks) and ``new_block_masks`` the intra-block bool masks
    (``None`` for finished blocks).  Trailing tight-pack rows inherit the
    last pointer in dots (D:1641-1644) and are fully masked in HunYuan
    (H:2290-2293).
    """
    pointer = torch.as_tensor(pointer, dtype=torch.long)
    lengths = torch.as_tensor(new_lengths, dtype=torch.long)
    idx = torch.repeat_interleave(pointer, lengths)
    q_real = int(lengths.sum())
    new_q = q_real + tight_pad_len
    if tight_pad_len:
        idx = torch.cat([idx, pointer[-1:].expand(tight_pad_len)])
    last = torch.full((1, 1, new_q, new_q), float("-inf"))
    blocks = [m for m in new_block_masks if m is not None]
    tril = torch.block_diag(*blocks) if blocks else torch.zeros((0, 0), dtype=torch.bool)
    last[0, 0, :tril.shape[0], :tril.shape[1]][tril] = 0
    inherited = attention_mask[:, :, idx, :].clone()
    if hunyuan and tight_pad_len:
        inherited[:, :, -tight_pad_len:, :] = float("-inf")
    return torch.cat([inherited, last], dim=-1)

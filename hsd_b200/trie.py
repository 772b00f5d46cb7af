"""Continuation trees of tree decoding, built on the device.

When KMP re-alignment does not find exactly one match, the reference
proposes a prefix tree (hsd/dots_ocr_pipeline/modeling_dots_ocr_hsd.py):
while ``kmp_search`` scans the draft it inserts, after every occurrence of
the match window's last token, the following ``max_tree_depth`` draft tokens
into a trie rooted at that token (D:573-586); the trie is then packed
breadth-first, capped at ``max_tree_len`` nodes, each node at position
``depth + base`` and seeing its ancestors (D:1488-1533).  Children keep the
order in which the scan first reached them, which fixes the BFS order and so
the packed layout.  ``hsd_continuation_trees`` builds the packed trees of
several blocks in one launch, with the attention-mask rows of every node.
"""
from __future__ import annotations

import ctypes as C
from dataclasses import dataclass

import torch

from . import _native as N


@dataclass
class Trees:
    """Packed trees of one launch (device tensors, row i = tree i)."""
    tokens: torch.Tensor    # int32 [n, cap]
    depths: torch.Tensor    # int32 [n, cap]
    parents: torch.Tensor   # int32 [n, cap], -1 for the root
    counts: torch.Tensor    # int32 [n]
    anc: torch.Tensor       # int64 [n, cap, ceil(cap / 64)]: node + ancestors bitset
    cap: int

    def host(self):
        """``[(tokens, depths, parents)]`` per tree, as Python lists."""
        cnt = self.counts.cpu().tolist()
        tok, dep, par = (t.cpu().tolist() for t in (self.tokens, self.depths, self.parents))
        return [(tok[i][:c], dep[i][:c], par[i][:c]) for i, c in enumerate(cnt)]


def continuation_trees(draft_pool, draft_off, draft_len, last_tokens, max_depth, cap,
                       status=None):
    """Build the packed continuation tree of every listed draft.

    draft_pool: int32 device tokens of all drafts; draft_off / draft_len /
    last_tokens: int32 device tensors, one entry per tree.  Asynchronous on
    the current stream; returns :class:`Trees`.
    """
    n = int(last_tokens.numel())
    dev = last_tokens.device
    aw = (int(cap) + 63) // 64
    out = Trees(torch.empty((n, cap), dtype=torch.int32, device=dev),
                torch.empty((n, cap), dtype=torch.int32, device=dev),
                torch.empty((n, cap), dtype=torch.int32, device=dev),
                torch.empty(n, dtype=torch.int32, device=dev),
                torch.empty((n, cap, aw), dtype=torch.int64, device=dev), int(cap))
    for t, name in ((draft_pool, "draft_pool"), (draft_off, "draft_off"),
                    (draft_len, "draft_len"), (last_tokens, "last_tokens")):
        if t.dtype != torch.int32 or t.device != dev or not t.is_contiguous():
            raise ValueError(f"continuation_trees: {name} must be contiguous int32 on {dev}")
    lib = N.load()
    N.check(lib.hsd_continuation_trees(
        N.ptr(draft_pool), N.ptr(draft_off), N.ptr(draft_len), N.ptr(last_tokens), n,
        int(max_depth), int(cap), N.ptr(out.tokens), N.ptr(out.depths), N.ptr(out.parents),
        N.ptr(out.counts), N.ptr(out.anc), N.ptr(status), N.stream_handle()),
        "hsd_continuation_trees")
    return out


def continuation_tree(draft, last_token, max_depth, cap, device="cuda"):
    """One tree from host lists: ``(tokens, depths, parents)`` (device build)."""
    d = torch.tensor(list(draft) or [0], dtype=torch.int32, device=device)
    z = torch.zeros(1, dtype=torch.int32, device=device)
    ln = torch.tensor([len(draft)], dtype=torch.int32, device=device)
    lt = torch.tensor([int(last_token)], dtype=torch.int32, device=device)
    return continuation_trees(d, z, ln, lt, max_depth, cap).host()[0]

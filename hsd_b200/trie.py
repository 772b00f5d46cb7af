"""Continuation tree of a block's draft for tree decoding (host side).

When KMP re-alignment does not find exactly one match, the reference
proposes a prefix tree (hsd/dots_ocr_pipeline/modeling_dots_ocr_hsd.py):
while ``kmp_search`` scans the draft it inserts, after every occurrence of
the match window's last token, the following ``max_tree_depth`` draft tokens
into a trie rooted at that token (D:573-586); the trie is then packed
breadth-first, capped at ``max_tree_len`` nodes, each node at position
``depth + base`` and seeing its ancestors (D:1488-1533).

Children keep the order in which the scan first reached them (the draft
order), which fixes the BFS order and so the packed layout.
"""
from __future__ import annotations

from collections import deque


def continuation_tree(draft, last_token, max_depth, cap):
    """``(tokens, depths, parents)`` of the BFS-packed continuation tree.

    Node 0 is the root (``last_token``, depth 0, parent -1); every other
    node's parent precedes it.  Only the root: no occurrence of
    ``last_token`` is followed by any token.
    """
    last_token = int(last_token)
    child_of = [{}]            # per node: token -> node, in insertion order
    tok, dep = [last_token], [0]
    n = len(draft)
    for i in range(n):
        if int(draft[i]) != last_token:
            continue
        node = 0
        for k in range(1, min(max_depth, n - 1 - i) + 1):
            t = int(draft[i + k])
            nxt = child_of[node].get(t)
            if nxt is None:
                nxt = len(tok)
                child_of[node][t] = nxt
                child_of.append({})
                tok.append(t)
                dep.append(k)
            node = nxt
    tokens, depths, parents = [], [], []
    order = deque([(0, -1)])
    while order and len(tokens) < cap:
        node, parent = order.popleft()
        here = len(tokens)
        tokens.append(tok[node])
        depths.append(dep[node])
        parents.append(parent)
        order.extend((c, here) for c in child_of[node].values())
    return tokens, depths, parents

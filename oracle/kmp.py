"""KMP re-alignment, restated from the reference (test infrastructure only).

Follows ``compute_lps`` (D:543-558), ``kmp_search`` (D:561-604) and
``find_all_matches_kmp`` (D:606-618) of
hsd/dots_ocr_pipeline/modeling_dots_ocr_hsd.py (byte-identical copies live at
H:366-441).  The trie node mirrors ``Node`` (D:511-521).
"""
from __future__ import annotations


class Node:
    """Continuation-trie node (D:511-521)."""

    __slots__ = ("value", "depth", "seg_id", "token_pos", "path",
                 "input_ids_index", "children")

    def __init__(self, value, seg_id, token_pos, path, depth=0):
        self.value = value
        self.depth = depth
        self.seg_id = seg_id
        self.token_pos = token_pos
        self.path = path
        self.input_ids_index = -1
        self.children = {}


def compute_lps(pattern):
    """KMP failure table (D:543-558)."""
    lps = [0] * len(pattern)
    length = 0
    i = 1
    while i < len(pattern):
        if pattern[i] == pattern[length]:
            length += 1
            lps[i] = length
            i += 1
        elif length != 0:
            length = lps[length - 1]
        else:
            lps[i] = 0
            i += 1
    return lps


def kmp_search(item_idx, text, pattern, lps, trie, depth):
    """All occurrences of ``pattern`` in ``text`` plus the continuation trie.

    D:561-604.  A match at ``start`` is kept only when
    ``start + len(pattern) <= len(text) - 1`` (D:595-597), i.e. at least one
    draft token follows it.  Independently of the pattern scan, every
    position ``i`` whose token equals ``pattern[-1]`` inserts
    ``text[i+1 : i+1+min(len(text)-i-1, depth)]`` into ``trie``
    (D:573-586); child dicts keep insertion order.
    """
    n = len(text)
    m = len(pattern)
    exact = []
    i = j = 0
    last = pattern[-1]
    while i < n:
        ti = text[i]
        if ti == last:
            node = trie
            remaining = min(n - i - 1, depth)
            k = 0
            while k < remaining:
                k += 1
                tok = text[i + k]
                child = node.children.get(tok)
                if child is None:
                    child = Node(tok, item_idx, i + k, node.path + (tok,), k)
                    node.children[tok] = child
                node = child
        if ti == pattern[j]:
            i += 1
            j += 1
            if j == m:
                start = i - j
                if start + m <= n - 1:
                    exact.append((item_idx, start, n))
                j = lps[j - 1]
        elif j != 0:
            j = lps[j - 1]
        else:
            i += 1
    return trie, exact


def find_all_matches_kmp(texts, pattern, lps, depth):
    """D:606-618: search every text; the trie root is ``pattern[-1]``."""
    trie = Node(pattern[-1], -1, -1, (-1, pattern[-1]), 0)
    matches = []
    for idx, text in enumerate(texts):
        trie, exact = kmp_search(idx, text, pattern, lps, trie, depth)
        matches.extend(exact)
    return trie, matches


def trie_bfs(root, cap):
    """BFS packing of a continuation trie (D:1488-1543).

    Returns ``(tokens, depths, parents)`` for at most ``cap`` nodes in BFS
    order.  ``parents[0] == -1``; every other node's parent precedes it.
    Nodes are numbered in visit order (their ``input_ids_index``).  The
    ancestor list of node ``i`` is ``i`` followed by its parent's list
    (D:1506-1514).
    """
    from collections import deque

    tokens, depths, parents = [], [], []
    index_of = {}
    queue = deque([(root, -1)])
    while queue and len(tokens) < cap:
        node, parent = queue.popleft()
        idx = len(tokens)
        index_of[id(node)] = idx
        tokens.append(node.value)
        depths.append(node.depth)
        parents.append(parent)
        for child in node.children.values():
            queue.append((child, idx))
    return tokens, depths, parents


def serialize_trie(root):
    """Nested-list form of a trie (token, [children...]) for fixtures."""
    return [root.value, [serialize_trie(c) for c in root.children.values()]]

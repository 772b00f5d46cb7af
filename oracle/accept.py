"""Per-block acceptance and re-alignment (test infrastructure only).

Restates the token-level parts of one iteration of the reference's
``batch_generate`` loop (hsd/dots_ocr_pipeline/modeling_dots_ocr_hsd.py):

* normal mode 1-token step (D:1107-1124)
* speculative acceptance (D:1126-1213): exact match, and below
  ``HSD_SPEC_THRESH`` < 1 the logit-ratio test from the first miss on
  (D:1147-1174)
* tree-walk acceptance (D:1215-1293), with the logit-ratio fallback among a
  node's children below ``HSD_TREE_THRESH`` < 1 in text mode (D:1228-1238,
  D:1256-1266)
* with ``variant="hunyuan"`` the HunYuan pipeline's rules
  (hsd/hunyuan_ocr_pipeline/modeling_hunyuan_vl_hsd.py, H:1653-1858): the
  speculative ratio on the last block only, outside formulas, accepted rows
  keeping the model's tokens, and the tree fallback at any threshold
* EOS and repetition stop (D:1299-1319)
* KMP re-alignment of non-page blocks (D:1321-1336, D:1417-1419)
* next block input: speculative slice, BFS tree, or normal (D:1421-1567)

The page block's text/select/bbox parser modes need the tokenizer and stay
on the host in both implementations; they are not restated here.
"""
from __future__ import annotations

import math
from dataclasses import dataclass, field

import numpy as np

from .kmp import compute_lps, find_all_matches_kmp, trie_bfs

NORMAL, SPEC, TREE, FINISHED = 0, 1, 2, 3


@dataclass
class BlockState:
    """Host bookkeeping of one packed block (D:979-992)."""

    mode: int = NORMAL
    gen: list = field(default_factory=list)      # generated_tokens[b]
    draft: list = field(default_factory=list)    # tokenized_draft[b]
    mws: int = 3                                 # match_window_sizes[b]
    matches_len: int = 0                         # matches_length[b]
    valid_count: int | None = None               # block_valid_counts[b]
    tree_tokens: list | None = None              # packed BFS tree (tree mode)
    tree_parents: list | None = None
    text_mode: bool = False                      # parser.text_mode (D:1229, D:1257)


@dataclass
class StepConfig:
    pad_token_id: int = 0
    eos_token_ids: tuple = (151643,)
    match_window_size: int = 3
    match_window_size_upper_bound: int = 10
    max_tree_depth: int = 15
    max_tree_len: int = 256
    min_input_length: int = 128
    max_spec_len: int = 0          # HSD_MAX_SPEC_LEN (D:61)
    tight_pack: bool = False       # HSD_TIGHT_PACK (D:52)
    enable_tree_decode: bool = False
    repeat_sentinel: int = 20993   # dots (D:1306); HunYuan uses 41153 (H:1873)
    spec_thresh: float = 1.0       # HSD_SPEC_THRESH (D:971); SPEC_THRESH (H:1471)
    tree_thresh: float = 1.0       # HSD_TREE_THRESH (D:970); fixed 1 in HunYuan (H:1470)
    variant: str = "dots"          # "dots" (D) or "hunyuan" (H)
    formula_tokens: tuple = (3, 1099)   # HunYuan '$' and '$$' (H:1685)
    spec_mode: str = "fmst"        # HunYuan SPEC_MODE (H:1668): "fmst", "topk", "adaptive"
    spec_topk: int = 3             # SPEC_TOPK (H:1714)
    spec_margin: float = 2.0       # SPEC_MARGIN (H:1720)


def bf16_f32(x):
    """float32 -> nearest bf16 (ties to even, the float -> bfloat16
    conversion torch applies to every bf16 result), returned as float32."""
    a = np.atleast_1d(np.asarray(x, dtype=np.float32)).copy()
    u = a.view(np.uint32)
    nan = np.isnan(a)
    r = (u + (((u >> 16) & 1) + np.uint32(0x7FFF))) & np.uint32(0xFFFF0000)
    out = np.where(nan, a, r.view(np.float32))
    return out if np.ndim(x) else out[0]


def logit_ratio(num, den):
    """``num / den`` of two bf16 logits as torch computes a bf16 quotient:
    the float32 quotient rounded to bf16 (D:1171, D:1233)."""
    with np.errstate(divide="ignore", invalid="ignore"):
        return bf16_f32(np.float32(num) / np.float32(den))


def ratio_passes(num, den, thresh):
    """``(num / den) >= thresh`` on bf16 tensors: torch compares in bf16,
    so the Python float threshold is rounded to bf16 first (0.9 -> 0.8984375)."""
    return bool(logit_ratio(num, den) >= bf16_f32(thresh))


def rank_and_second(row, ref_col, excl_col):
    """``(rank, second)`` of one row of bf16 logits (float32 array of bf16
    values) for HunYuan's ``topk`` / ``adaptive`` modes (H:1712-1736).

    ``rank``: the draft token ``ref_col``'s 0-based position when the row is
    sorted by descending logit, lower columns first among equal logits, so
    ``rank < k`` stands for ``ref in logits.topk(k).indices`` (torch leaves
    the order among equal values unspecified); ``second``: the largest logit
    outside column ``excl_col`` (the row's argmax), i.e. ``topk(2).values[1]``.
    """
    v = np.asarray(row, dtype=np.float32)
    thr = v[ref_col]
    if np.isnan(thr):       # a probe of a bad index ranks the token last
        rank = v.size - 1
    else:
        rank = int(np.count_nonzero(v > thr) + np.count_nonzero(v[:ref_col] == thr))
    second = np.float32(np.max(np.delete(v, excl_col))) if v.size > 1 else np.float32(-np.inf)
    return rank, second


def spec_mode_passes(cfg, pred, probe, thresh, rank=None, second=None):
    """A missed speculative row of HunYuan's last block passes (H:1710-1743):
    ``fmst``: the logit ratio; ``topk``: the draft token among the row's
    ``spec_topk`` best (``rank < k``); ``adaptive``: the ratio, or a bf16
    top-1 / top-2 margin below ``spec_margin`` with a positive draft logit
    (bf16 subtraction and a bf16 comparison, as torch does on the logits)."""
    pred = np.float32(pred)
    ratio = bool(pred > 0) and ratio_passes(probe, pred, thresh)
    if cfg.spec_mode == "fmst":
        return ratio
    if cfg.spec_mode == "topk":
        return int(rank) < int(cfg.spec_topk)
    if cfg.spec_mode == "adaptive":
        margin = bf16_f32(np.float32(pred) - np.float32(second))
        return ratio or (bool(margin < bf16_f32(np.float32(cfg.spec_margin)))
                         and bool(np.float32(probe) > 0))
    raise ValueError(f"spec_mode {cfg.spec_mode!r}")


def tree_ratio_fallback(node, tokens, parents, max_logit, probe_logit):
    """The ratios a tree walk's fallback compares when the target's token is
    not a child of ``node`` (D:1228-1238, D:1256-1266): ``logits[row, child
    token] / logits[row, decode]`` over the node's children in insertion
    (BFS) order, ``row`` being the node's packed row.  ``probe_logit[c]``
    (indexed from the block's first row) holds ``logits[row of c's parent,
    token c]``; ``max_logit``, the row's maximal logit, is ``logits[row,
    decode]``.  Returns ``(children, ratios)``, or None without children."""
    kids = [c for c in range(node + 1, len(tokens)) if parents[c] == node]
    if not kids:
        return None
    return kids, [logit_ratio(probe_logit[c], max_logit) for c in kids]


def _valid_length(st, input_list, bs, be, pad):
    if st.valid_count is not None:
        return st.valid_count
    return sum(1 for t in input_list[bs:be] if t != pad)


def _window_update(st, cfg, increment):
    if st.matches_len in (0, 1):
        st.mws = cfg.match_window_size
    else:
        st.mws += increment


def accept_block(st, bs, be, next_list, input_list, cfg, filt, kv_base,
                 allowed_row_fn, is_page_block, logits=None, is_last_block=False):
    """Acceptance for one block; mutates ``st`` and ``filt``.

    Returns ``(pointer, next_token, increment, finished_reason)`` where
    ``pointer`` is the absolute row (in the current packed query) of the
    block's last accepted token, ``finished_reason`` is 0 (running),
    1 (EOS) or 2 (repetition stop).  ``filt`` is the step's bool filter over
    KV columns; ``allowed_row_fn(row)`` gives the bool visibility of a query
    row (the mask row the EOS rule ORs in, D:1300-1302).  ``logits =
    (max_logit, probe_logit)``, per packed row, feeds the logit-ratio rules
    when a threshold is below 1: ``max_logit[r] = logits[r, next[r]]``; for a
    speculative row ``probe_logit[r] = logits[r, input[r + 1]]``, for tree
    node c of a block starting at bs ``probe_logit[bs + c] = logits[bs +
    parent(c), token(c)]``.
    """
    pad = cfg.pad_token_id
    mode = st.mode
    if mode == NORMAL:                                         # D:1107-1124
        valid = _valid_length(st, input_list, bs, be, pad)
        ptr = bs + valid - 1
        nxt = next_list[ptr]
        st.gen.append(nxt)
        inc = 1
        _window_update(st, cfg, 1)
    elif mode == SPEC:                                         # D:1126-1213
        valid = _valid_length(st, input_list, bs, be, pad)
        ptr = bs + valid - 1
        group = next_list[bs:be]
        ref = input_list[bs:be]
        blen = be - bs
        acc = [group[i] == ref[i + 1] for i in range(blen - 1)]
        hunyuan = cfg.variant == "hunyuan"
        thresh = cfg.spec_thresh if (not hunyuan or is_last_block) else 1.0   # H:1671
        if thresh < 1.0:                                       # D:1147-1174, H:1676-1744
            max_l, probe_l = logits[0], logits[1]
            rank_l, second_l = (logits[2], logits[3]) if len(logits) > 2 else (None, None)
            can = [True] * len(acc)
            if hunyuan:                                        # H:1681-1695
                in_formula = False
                for t in st.gen:
                    if t in cfg.formula_tokens:
                        in_formula = not in_formula
                for fi in range(blen):
                    dollar = ref[fi] in cfg.formula_tokens
                    if dollar:
                        in_formula = not in_formula
                    if fi < len(acc):
                        can[fi] = (not in_formula) and (not dollar)
            first_miss = next((i for i, ok in enumerate(acc) if not ok), len(acc))
            for i in range(first_miss, len(acc)):
                pred = np.float32(max_l[bs + i])
                if can[i] and hunyuan:
                    acc[i] = acc[i] or spec_mode_passes(
                        cfg, pred, probe_l[bs + i], thresh,
                        None if rank_l is None else rank_l[bs + i],
                        None if second_l is None else second_l[bs + i])
                elif can[i]:
                    acc[i] = acc[i] or (bool(pred > 0) and
                                        ratio_passes(probe_l[bs + i], pred, thresh))
        diff = len(acc)
        for i, ok in enumerate(acc):
            if not ok:
                diff = i
                break
        accepted = list(group[:diff + 1])
        if not hunyuan:                # HunYuan keeps the model's tokens (H:1750-1754)
            for i in range(diff):
                accepted[i] = ref[i + 1]
        st.gen.extend(accepted)
        inc = diff + 1
        nxt = group[diff]
        _window_update(st, cfg, diff + 1)
        if diff != blen - 1:
            ptr = bs + diff
            filt[kv_base + bs + diff + 1: kv_base + be] = True
    elif mode == TREE:                                         # D:1215-1293
        group = next_list[bs:be]
        tokens, parents = st.tree_tokens, st.tree_parents
        n_nodes = len(tokens)
        consumed = [False] * n_nodes

        def fallback(node, decode):                            # D:1228-1238
            # HunYuan runs the fallback at any threshold (H:1791, H:1821)
            if not ((cfg.variant == "hunyuan" or cfg.tree_thresh < 1.0) and st.text_mode):
                return decode
            if any(parents[c] == node and tokens[c] == decode for c in range(node + 1, n_nodes)):
                return decode
            max_l, probe_l = logits[0], logits[1]
            got = tree_ratio_fallback(node, tokens, parents, max_l[bs + node], probe_l[bs:])
            if got is None:
                return decode
            kids, ratios = got
            thr = bf16_f32(cfg.tree_thresh)
            if not any(r >= thr for r in ratios):
                return decode
            nans = [i for i, r in enumerate(ratios) if np.isnan(r)]
            best = nans[0] if nans else int(np.argmax(ratios))
            return tokens[kids[best]]

        decode = fallback(0, group[0])
        st.gen.append(decode)
        inc = 1
        filt[kv_base + bs] = True
        node = 0
        new_index = 0
        walked = 0
        while True:
            child = -1
            for c in range(node + 1, n_nodes):
                if parents[c] == node and tokens[c] == decode:
                    child = c
                    break
            if child < 0 or consumed[child]:
                break
            node = child
            new_index = child
            consumed[child] = True
            decode = fallback(node, group[new_index])          # D:1256-1266
            st.gen.append(decode)
            inc += 1
            walked += 1
            filt[kv_base + bs + new_index] = True
        ptr = bs + new_index
        seg = filt[kv_base + bs: kv_base + be]
        filt[kv_base + bs: kv_base + be] = ~seg
        nxt = group[new_index]
        _window_update(st, cfg, 1 + walked)
    else:
        return None, None, 0, 0

    if st.gen[-1] in cfg.eos_token_ids:                       # D:1299-1305
        filt |= allowed_row_fn(ptr)
        st.mode = FINISHED
        st.gen = st.gen[:-1]
        return ptr, nxt, inc, 1
    if not is_page_block:                                       # D:1306-1319
        tail = st.gen[-10:]
        reps = find_all_matches_kmp([st.gen], tail, compute_lps(tail), 1)[1]
        if len(reps) > 10 and cfg.repeat_sentinel not in st.gen:
            filt |= allowed_row_fn(ptr)
            st.gen = list(st.draft)
            st.mode = FINISHED
            return ptr, nxt, inc, 2
    return ptr, nxt, inc, 0


def realign_block(st, cfg):
    """KMP re-alignment of a region block (D:1321-1336, D:1417-1419).

    Returns ``(window, matches, trie)``.
    """
    w = min(cfg.match_window_size_upper_bound, st.mws)
    window = st.gen[-w:]
    trie, matches = find_all_matches_kmp([st.draft], window,
                                         compute_lps(window),
                                         cfg.max_tree_depth)
    st.matches_len = len(matches)
    return window, matches, trie


def next_block_input(st, cfg, window, matches, trie, next_token, pos_base):
    """Next input of a region block (D:1421-1567).

    Returns ``(input_ids, position_ids, intra_kind, new_len)`` and updates
    ``st.mode`` / ``st.valid_count`` / the packed tree.
    """
    pad = cfg.pad_token_id
    mil = cfg.min_input_length
    if len(matches) == 1:                                       # D:1421-1436
        _, start, end = matches[0]
        start += len(window) - 1
        ids = list(st.draft[start:end])
        if cfg.max_spec_len > 0 and len(ids) > cfg.max_spec_len:
            ids = ids[:cfg.max_spec_len]
        if not cfg.tight_pack:
            ids += [pad] * (math.ceil(len(ids) / mil) * mil - len(ids))
        pos = list(range(pos_base, pos_base + len(ids)))
        st.valid_count = len(ids) - (ids.count(pad) if not cfg.tight_pack else 0)
        st.mode = SPEC
        st.tree_tokens = st.tree_parents = None
        return ids, pos, "causal", len(ids)
    if cfg.enable_tree_decode and len(trie.children) > 0:       # D:1488-1543
        cap = (min(cfg.max_tree_len, cfg.max_spec_len) if cfg.max_spec_len > 0
               else cfg.max_tree_len)
        tokens, depths, parents = trie_bfs(trie, cap)
        ids = list(tokens)
        pos = [d + pos_base for d in depths]
        if not cfg.tight_pack:
            ids += [pad] * (math.ceil(len(ids) / mil) * mil - len(ids))
            pos += [0] * (len(ids) - len(pos))
        st.valid_count = len(tokens)
        st.mode = TREE
        st.tree_tokens, st.tree_parents = tokens, parents
        return ids, pos, "tree", len(ids)
    if cfg.tight_pack:                                           # D:1544-1565
        ids, pos = [next_token], [pos_base]
    else:
        ids = [next_token] + [pad] * (mil - 1)
        pos = [pos_base] + [0] * (mil - 1)
    st.valid_count = 1
    st.mode = NORMAL
    st.tree_tokens = st.tree_parents = None
    return ids, pos, "single", len(ids)


def kmp_match_summary(draft, window):
    """(count, first start) of the matches ``find_all_matches_kmp`` keeps."""
    _, matches = find_all_matches_kmp([draft], window, compute_lps(window), 1)
    if not matches:
        return 0, -1
    return len(matches), matches[0][1]


def as_int_array(x):
    return np.asarray(x, dtype=np.int64)

"""The page block of ``batch_generate`` restated on the CPU (test
infrastructure only).

Follows hsd/dots_ocr_pipeline/modeling_dots_ocr_hsd.py: the streaming JSON
watcher ``StreamingTextWatcher`` (D:261-317), the string helpers
``to_halfwidth_clean`` (D:155-173), ``clean_string_and_get_maps``
(D:178-218) and ``unescape_string_final`` (D:236-258), the select / bbox
candidate trees (D:648-744) and the last block's branch of the per-block
loop: parser feed, window, candidate selection (D:1337-1419) and next input
(D:1421-1567).  Tries are :class:`oracle.kmp.Node` trees built by the
restated ``find_all_matches_kmp``.
"""
from __future__ import annotations

import ast
import json
import math
import re
import unicodedata

from .kmp import compute_lps, find_all_matches_kmp, trie_bfs

BBOX_MARKER = '"bbox": ['          # D:277
TEXT_MARKER = '"text": "'          # D:278
CAT_MARKER = '"category": "'       # D:279
CLOSING_QUOTE = re.compile(r'(?<!\\)"')   # D:259


class StreamingTextWatcher:
    """D:261-317."""

    def __init__(self):
        self._buf = ""
        self.text_mode = False
        self.bbox_mode = False
        self.category_mode = False

    def feed(self, chunk: bytes):
        self._buf += chunk.decode("utf-8", errors="replace")
        s = self._buf
        bi = s.rfind(BBOX_MARKER)
        self.bbox_mode = (bi != -1) and (']' not in s[bi + len(BBOX_MARKER):])
        ti = s.rfind(TEXT_MARKER)
        if ti == -1:
            self.text_mode = False
        else:
            self.text_mode = CLOSING_QUOTE.search(s[ti + len(TEXT_MARKER):]) is None
        ci = s.rfind(CAT_MARKER)
        if ci == -1:
            self.category_mode = False
        else:
            self.category_mode = CLOSING_QUOTE.search(s[ci + len(CAT_MARKER):]) is None


def to_halfwidth_clean(s):
    """D:155-173."""
    if s is None:
        return s
    s = unicodedata.normalize('NFKC', s)
    s = s.replace('\n\n', '_SAVE_TAG_')
    s = s.replace('\n', '').replace('\r', '')
    s = s.replace('_SAVE_TAG_', '\n\n')
    s = s.replace('\\n\\n', '_SAVE_TAG_')
    s = s.replace('\\n', '').replace('\\r', '')
    s = s.replace('_SAVE_TAG_', '\\n\\n')
    s = s.replace("  ", "")
    return s


_KEEP = re.compile(r'[一-鿿぀-ヿa-zA-Z0-9]')


def clean_string_and_get_maps(input_string):
    """D:178-218 (the old-to-new map is not read by the loop)."""
    cleaned, new_to_old = [], []
    for old_idx, char in enumerate(input_string):
        if _KEEP.match(char):
            cleaned.append(char)
            new_to_old.append(old_idx)
    return {"cleaned_string": "".join(cleaned), "new_to_old_map": new_to_old}


def unescape_string_final(s):
    """D:236-258."""
    try:
        return ast.literal_eval('"' + s.replace('"', '\\"') + '"')
    except (ValueError, SyntaxError):
        return s


_CATEGORIES = ['Caption', 'Footnote', 'Formula', 'List-item', 'Page-footer', 'Page-header',
               'Picture', 'Section-header', 'Table', 'Text', 'Title']


def select_mode_tree(pre_tok):
    """D:648-671."""
    begin = pre_tok.encode("[")[0]
    all_draft = ['{"bbox": [', ' "text": "', ', {"bbox": [', '}]']
    all_draft += [f' "category": "{cat}' for cat in _CATEGORIES]
    for cat in _CATEGORIES:
        all_draft.append(f' "category": "{cat}", "text": "')
    tok = pre_tok(all_draft, add_special_tokens=False)['input_ids']
    tok = [[begin] + ids for ids in tok]
    tree, _ = find_all_matches_kmp(tok, [begin], compute_lps([begin]), 15)
    return tree


def bbox_mode_tree(pre_tok):
    """D:688-731."""
    begin = pre_tok.encode(" [")[0]
    all_draft = []
    for d in range(10):
        for d2 in range(10):
            all_draft.append(f"{d}{d2}")
        all_draft.append(f"{d}, ")
        all_draft.append(f"{d}]")
    for d in range(10):
        all_draft.append(f", {d}")
    tok = pre_tok(all_draft, add_special_tokens=False)['input_ids']
    tok = [[begin] + ids for ids in tok]
    tree, _ = find_all_matches_kmp(tok, [begin], compute_lps([begin]), 10)
    return tree


class OraclePage:
    """The last block's candidate selection and next input (D:1337-1567),
    with the loop-level state it reads: the parser, the cached select /
    bbox trees and the finished blocks' text cache (D:1354-1400)."""

    def __init__(self, tokenizer, norm_draft, cfg, pre_tokenizer=None):
        self.tok = tokenizer
        self.pre = pre_tokenizer or tokenizer
        self.norm_draft = list(norm_draft)
        self.cfg = cfg
        self.parser = StreamingTextWatcher()
        self.select_tree = None
        self.bbox_tree = None
        self.cache = {}

    def candidates(self, gen, increment, mws, generated, finished):
        """Returns ``(matches, tree, text_state)`` of the last block."""
        tok = self.tok
        new_chunk = tok.decode(gen[-increment:])
        self.parser.feed(new_chunk.encode('utf-8'))
        w = min(self.cfg.match_window_size_upper_bound, mws)
        window = gen[-w:]
        matches, tree, state = [], None, None
        if not (self.parser.bbox_mode or self.parser.text_mode):
            if self.select_tree is None:
                self.select_tree = select_mode_tree(self.pre)
            self.select_tree.value = gen[-1]
            tree = self.select_tree
        if self.parser.bbox_mode:
            if self.bbox_tree is None:
                self.bbox_tree = bbox_mode_tree(self.pre)
            self.bbox_tree.value = gen[-1]
            tree = self.bbox_tree
        if self.parser.text_mode:
            wtext = unescape_string_final(tok.decode(window))
            wclean = [c for c in clean_string_and_get_maps(wtext)['cleaned_string']]
            if len(generated) > 1:
                t_draft, t_tok, t_clean, t_map = [], [], [], []
                for bid in range(len(generated) - 1):
                    if bid in self.cache:
                        c = self.cache[bid]
                    else:
                        one = tok.batch_decode([generated[bid]], skip_special_tokens=True)[0]
                        one = one.replace("\n\n", "\n")
                        tt = tok.encode(json.dumps(one, ensure_ascii=False)[1:-1],
                                        add_special_tokens=False)
                        cl = clean_string_and_get_maps(one)
                        c = (one, tt, [ch for ch in cl['cleaned_string']], cl['new_to_old_map'])
                        if finished[bid]:
                            self.cache[bid] = c
                    t_draft.append(c[0])
                    t_tok.append(c[1])
                    t_clean.append(c[2])
                    t_map.append(c[3])
            else:
                one = self.norm_draft[0] if self.norm_draft else ""
                one = one.replace("\n\n", "\n")
                t_draft = [self.norm_draft[0]] if self.norm_draft else [""]
                t_tok = [tok.encode(json.dumps(one, ensure_ascii=False)[1:-1],
                                    add_special_tokens=False)]
                cl = clean_string_and_get_maps(one)
                t_clean = [[ch for ch in cl['cleaned_string']]]
                t_map = [cl['new_to_old_map']]
            if len(wclean) != 0:
                _, matches = find_all_matches_kmp(t_clean, wclean, compute_lps(wclean), 1)
            else:
                matches = []
            if len(matches) != 1:
                tree, _ = find_all_matches_kmp(t_tok, window, compute_lps(window),
                                               self.cfg.max_tree_depth)
            state = (wclean, t_draft, t_map)
        return matches, tree, state

    def next_input(self, gen, increment, mws, generated, finished, pos_base, next_token):
        """``(ids, pos, kind, valid, matches_len, parents)`` of the last block:
        kind "causal" (speculative), "tree" or "single" (normal, whose input
        is ``next_token_int``, D:1546-1565)."""
        cfg, tok = self.cfg, self.tok
        pad, mil = cfg.pad_token_id, cfg.min_input_length
        matches, tree, state = self.candidates(gen, increment, mws, generated, finished)
        if len(matches) == 1:                                     # D:1437-1467
            item_idx, start, _ = matches[0]
            wclean, t_draft, t_map = state
            start += len(wclean) - 1
            start = t_map[item_idx][start]
            one = t_draft[item_idx][start + 1:]
            one = json.dumps(one, ensure_ascii=False)[1:-1]
            might = tok.decode(gen[-1])
            if one.startswith(might):
                one = one[len(might):]
            ids = [gen[-1]] + tok.encode(one, add_special_tokens=False)
            if cfg.max_spec_len > 0 and len(ids) > cfg.max_spec_len:
                ids = ids[:cfg.max_spec_len]
            if not cfg.tight_pack:
                ids += [pad] * (math.ceil(len(ids) / mil) * mil - len(ids))
            valid = len(ids) - (ids.count(pad) if not cfg.tight_pack else 0)
            return ids, list(range(pos_base, pos_base + len(ids))), "causal", valid, 1, None
        if cfg.enable_tree_decode and tree is not None and len(tree.children) > 0:
            cap = (min(cfg.max_tree_len, cfg.max_spec_len) if cfg.max_spec_len > 0
                   else cfg.max_tree_len)
            tokens, depths, parents = trie_bfs(tree, cap)
            ids = list(tokens)
            pos = [d + pos_base for d in depths]
            if not cfg.tight_pack:
                ids += [pad] * (math.ceil(len(ids) / mil) * mil - len(ids))
                pos += [0] * (len(ids) - len(pos))
            return ids, pos, "tree", len(tokens), len(matches), (tokens, parents)
        nxt = next_token
        if cfg.tight_pack:
            return [nxt], [pos_base], "single", 1, len(matches), None
        return ([nxt] + [pad] * (mil - 1), [pos_base] + [0] * (mil - 1), "single", 1,
                len(matches), None)


class OracleHunyuanPage(OraclePage):
    """The HunYuan loop's last block (hsd/hunyuan_ocr_pipeline/
    modeling_hunyuan_vl_hsd.py H:1900-2025 and H:2046-2104): the text rule
    at every step without a parser, the other blocks' outputs prefixed with
    a blank line and not re-escaped, no speculative length cap, the tree cap
    ``max_tree_len``."""

    def next_input(self, gen, increment, mws, generated, finished, pos_base, next_token):
        cfg, tok = self.cfg, self.tok
        pad, mil = cfg.pad_token_id, cfg.min_input_length
        w = min(cfg.match_window_size_upper_bound, mws)
        window = gen[-w:]
        wtext = tok.decode(window)
        wclean = [c for c in clean_string_and_get_maps(wtext)['cleaned_string']]
        if len(generated) > 1:
            t_draft, t_tok, t_clean, t_map = [], [], [], []
            for bid in range(len(generated) - 1):
                if bid in self.cache:
                    c = self.cache[bid]
                else:
                    one = tok.batch_decode([generated[bid]], skip_special_tokens=True)[0]
                    one = one.replace("\n\n", "\n")
                    one = "\n\n" + one
                    cl = clean_string_and_get_maps(one)
                    c = (one, tok.encode(one, add_special_tokens=False),
                         [ch for ch in cl['cleaned_string']], cl['new_to_old_map'])
                    if finished[bid]:
                        self.cache[bid] = c
                t_draft.append(c[0])
                t_tok.append(c[1])
                t_clean.append(c[2])
                t_map.append(c[3])
        else:
            one = self.norm_draft[0] if self.norm_draft else ""
            one = one.replace("\n\n", "\n")
            one = "\n\n" + one
            t_draft = [self.norm_draft[0]] if self.norm_draft else [""]
            t_tok = [tok.encode(one, add_special_tokens=False)]
            cl = clean_string_and_get_maps(one)
            t_clean = [[ch for ch in cl['cleaned_string']]]
            t_map = [cl['new_to_old_map']]
        if len(wclean) != 0:
            _, matches = find_all_matches_kmp(t_clean, wclean, compute_lps(wclean), 1)
        else:
            matches = []
        tree = None
        if len(matches) != 1:
            tree, _ = find_all_matches_kmp(t_tok, window, compute_lps(window),
                                           cfg.max_tree_depth)
        if len(matches) == 1:
            item_idx, start, _ = matches[0]
            start += len(wclean) - 1
            start = t_map[item_idx][start]
            one = t_draft[item_idx][start + 1:]
            might = tok.decode(gen[-1])
            if one.startswith(might):
                one = one[len(might):]
            ids = [gen[-1]] + tok.encode(one, add_special_tokens=False)
            if not cfg.tight_pack:
                ids += [pad] * (math.ceil(len(ids) / mil) * mil - len(ids))
            valid = len(ids) - (ids.count(pad) if not cfg.tight_pack else 0)
            return ids, list(range(pos_base, pos_base + len(ids))), "causal", valid, 1, None
        if cfg.enable_tree_decode and len(tree.children) > 0:
            tokens, depths, parents = trie_bfs(tree, cfg.max_tree_len)
            ids = list(tokens)
            pos = [d + pos_base for d in depths]
            if not cfg.tight_pack:
                ids += [pad] * (math.ceil(len(ids) / mil) * mil - len(ids))
            pos += [0] * (len(ids) - len(pos))
            return ids, pos, "tree", len(tokens), len(matches), (tokens, parents)
        nxt = next_token
        if cfg.tight_pack:
            return [nxt], [pos_base], "single", 1, len(matches), None
        return ([nxt] + [pad] * (mil - 1), [pos_base] + [0] * (mil - 1), "single", 1,
                len(matches), None)

"""The page block of the verification loop (host side).

The reference packs the full page as the last block (RD:198-221).  Unlike a
region block, its next input does not come from KMP against its own draft:
a streaming parser follows the page output's layout JSON
(``StreamingTextWatcher``, hsd/dots_ocr_pipeline/modeling_dots_ocr_hsd.py
D:261-317) and, per step (D:1337-1419, D:1421-1567 for the last block):

* outside a bbox list and a text value ("select" mode) the candidate is a
  fixed tree of layout-JSON fragments (D:648-686);
* inside ``"bbox": [`` a fixed tree of digit / separator sequences
  (D:688-744);
* inside ``"text": "`` the generated window is matched, as cleaned
  characters, against the decoded outputs of the other blocks; exactly one
  match makes the rest of that output (re-escaped as JSON) the next
  speculative input, otherwise the candidate is the continuation trie of the
  window over the re-tokenized outputs.

Everything here needs the tokenizer and runs on the host while the device
finishes the step's acceptance, keep indices and compaction of the other
blocks (:mod:`hsd_b200.generate`).  Trees are packed breadth-first as the
reference's tree decoding does (D:1488-1543).
"""
from __future__ import annotations

import ast
import json
import math
import re
import unicodedata
from dataclasses import dataclass, field

# ---------------------------------------------------------------- parser
_BBOX = '"bbox": ['
_TEXT = '"text": "'
_CAT = '"category": "'
_UNESCAPED_QUOTE = re.compile(r'(?<!\\)"')


class LayoutParser:
    """Tracks whether the page output is inside a bbox list, a text value
    or a category value (D:261-317): the most recent opening marker counts,
    and a bbox list closes at the next ``]``, a text / category value at the
    next double quote not preceded by a backslash."""

    def __init__(self):
        self._buf = ""
        self.text_mode = False
        self.bbox_mode = False
        self.category_mode = False

    def feed(self, chunk: str):
        # the reference feeds the decoded chunk as UTF-8 bytes and decodes
        # them back with errors='replace': the identity on a str
        self._buf += chunk
        s = self._buf
        i = s.rfind(_BBOX)
        self.bbox_mode = i != -1 and "]" not in s[i + len(_BBOX):]
        i = s.rfind(_TEXT)
        self.text_mode = i != -1 and _UNESCAPED_QUOTE.search(s[i + len(_TEXT):]) is None
        i = s.rfind(_CAT)
        self.category_mode = i != -1 and _UNESCAPED_QUOTE.search(s[i + len(_CAT):]) is None


# ---------------------------------------------------------------- text
_KEEP = re.compile(r"[一-鿿぀-ヿa-zA-Z0-9]")


def halfwidth_clean(s):
    """NFKC normalisation, single newlines / carriage returns (real and
    backslash-escaped) dropped while double ones stay, double spaces
    removed (``to_halfwidth_clean``, D:155-173)."""
    if s is None:
        return s
    tag = "_SAVE_TAG_"     # the reference's placeholder (so inputs holding it map alike)
    s = unicodedata.normalize("NFKC", s)
    s = s.replace("\n\n", tag).replace("\n", "").replace("\r", "").replace(tag, "\n\n")
    s = s.replace("\\n\\n", tag).replace("\\n", "").replace("\\r", "").replace(tag, "\\n\\n")
    return s.replace("  ", "")


def cleaned_with_map(s):
    """The characters of ``s`` that are CJK ideographs, kana, ASCII letters or
    digits, and for each its index in ``s`` (``clean_string_and_get_maps``,
    D:178-218)."""
    chars, where = [], []
    for i, c in enumerate(s):
        if _KEEP.match(c):
            chars.append(c)
            where.append(i)
    return chars, where


def unescape_json_fragment(s):
    """Unescape a decoded window as a Python string literal with its double
    quotes escaped; the window itself when that fails
    (``unescape_string_final``, D:236-258)."""
    try:
        return ast.literal_eval('"' + s.replace('"', '\\"') + '"')
    except (ValueError, SyntaxError):
        return s


# ---------------------------------------------------------------- KMP / tries
def kmp_matches(texts, pattern):
    """Every occurrence ``(item, start, len(text))`` of ``pattern`` in each
    text that leaves at least one element after it (``start + len(pattern)
    <= len(text) - 1``), item-major, start ascending: the matches of
    ``find_all_matches_kmp`` (D:561-618), found here with the failure-table
    scan of Knuth-Morris-Pratt."""
    m = len(pattern)
    if m == 0:
        return []
    fail = [0] * m
    k = 0
    for i in range(1, m):
        while k and pattern[i] != pattern[k]:
            k = fail[k - 1]
        if pattern[i] == pattern[k]:
            k += 1
        fail[i] = k
    out = []
    for item, text in enumerate(texts):
        n = len(text)
        k = 0
        for i in range(n):
            while k and text[i] != pattern[k]:
                k = fail[k - 1]
            if text[i] == pattern[k]:
                k += 1
            if k == m:
                start = i - m + 1
                if start + m <= n - 1:
                    out.append((item, start, n))
                k = fail[k - 1]
    return out


class Trie:
    """Continuation trie: children in insertion order, node 0 the root."""

    def __init__(self, root_token):
        self.token = [int(root_token)]
        self.depth = [0]
        self.kids = [{}]

    def insert(self, seq):
        node = 0
        for d, t in enumerate(seq, 1):
            nxt = self.kids[node].get(t)
            if nxt is None:
                nxt = len(self.token)
                self.token.append(t)
                self.depth.append(d)
                self.kids.append({})
                self.kids[node][t] = nxt
            node = nxt

    def has_children(self):
        return bool(self.kids[0])

    def bfs(self, cap):
        """At most ``cap`` nodes in breadth-first order: ``(tokens, depths,
        parents)`` with ``parents[0] = -1`` (D:1488-1514)."""
        tokens, depths, parents = [], [], []
        queue, head = [(0, -1)], 0
        while head < len(queue) and len(tokens) < cap:
            node, parent = queue[head]
            head += 1
            idx = len(tokens)
            tokens.append(self.token[node])
            depths.append(self.depth[node])
            parents.append(parent)
            queue.extend((c, idx) for c in self.kids[node].values())
        return tokens, depths, parents


def continuation_trie(texts, last_token, depth):
    """The trie ``find_all_matches_kmp`` grows beside its matches (D:573-586):
    after every position of every text holding ``last_token``, the next
    ``min(depth, rest of the text)`` elements are inserted below the root."""
    trie = Trie(last_token)
    for text in texts:
        n = len(text)
        for i, t in enumerate(text):
            if t == last_token and i + 1 < n:
                trie.insert(text[i + 1:i + 1 + min(n - i - 1, depth)])
    return trie


# ---------------------------------------------------------------- candidates
_CATEGORIES = ["Caption", "Footnote", "Formula", "List-item", "Page-footer", "Page-header",
               "Picture", "Section-header", "Table", "Text", "Title"]


def _tokenize_all(pre_tokenizer, texts):
    return pre_tokenizer(texts, add_special_tokens=False)["input_ids"]


def select_candidate_trie(pre_tokenizer):
    """The select-mode candidates (D:648-671): after ``[`` the layout JSON's
    element and field openings, depth 15."""
    begin = pre_tokenizer.encode("[")[0]
    frags = ['{"bbox": [', ' "text": "', ', {"bbox": [', "}]"]
    frags += [f' "category": "{c}' for c in _CATEGORIES]
    frags += [f' "category": "{c}", "text": "' for c in _CATEGORIES]
    seqs = [[begin] + list(ids) for ids in _tokenize_all(pre_tokenizer, frags)]
    return continuation_trie(seqs, begin, 15)


def bbox_candidate_trie(pre_tokenizer):
    """The bbox-mode candidates (D:688-731): digit pairs, digit + separator
    and separator + digit sequences after `` [``, depth 10."""
    begin = pre_tokenizer.encode(" [")[0]
    frags = []
    for d in range(10):
        frags += [f"{d}{e}" for e in range(10)]
        frags += [f"{d}, ", f"{d}]"]
    frags += [f", {d}" for d in range(10)]
    seqs = [[begin] + list(ids) for ids in _tokenize_all(pre_tokenizer, frags)]
    return continuation_trie(seqs, begin, 10)


# ---------------------------------------------------------------- next input
@dataclass
class PageInput:
    """The page block's next input: ``kind`` is "spec", "tree" or "normal";
    ``ids`` / ``pos`` include padding; ``valid`` = real rows; ``parents`` /
    ``depths`` cover the real tree nodes; ``matches`` = the count the window
    rule of the next step reads (``matches_length``, D:1419)."""

    kind: str
    ids: list
    pos: list
    valid: int
    matches: int
    parents: list = field(default_factory=list)
    depths: list = field(default_factory=list)


class PageBlock:
    """Per-loop state of the page block: the parser, the candidate tries and
    the decoded outputs of finished blocks (D:1354-1400 caches them)."""

    def __init__(self, tokenizer, pre_tokenizer=None, *, max_tree_depth=15, tree_cap=256,
                 min_input_length=128, tight_pack=False, max_spec_len=0,
                 enable_tree_decode=False, match_window_size_upper_bound=10, norm_draft=None):
        self.tok = tokenizer
        self.pre = pre_tokenizer if pre_tokenizer is not None else tokenizer
        self.parser = LayoutParser()
        self.depth = int(max_tree_depth)
        self.cap = int(tree_cap)
        self.mil = int(min_input_length)
        self.tight = bool(tight_pack)
        self.max_spec = int(max_spec_len)
        self.tree_decode = bool(enable_tree_decode)
        self.mws_ub = int(match_window_size_upper_bound)
        self.norm_draft = list(norm_draft or [])
        self._select = self._bbox = None
        self._finished_text = {}
        self.mode = "select"

    # the reference builds each fixed trie once and only changes its root token
    def _select_trie(self):
        if self._select is None:
            self._select = select_candidate_trie(self.pre)
        return self._select

    def _bbox_trie(self):
        if self._bbox is None:
            self._bbox = bbox_candidate_trie(self.pre)
        return self._bbox

    def _others(self, outputs, finished):
        """Decoded, cleaned and re-tokenized outputs of the other blocks
        (D:1354-1400; one block: the page's own normalised draft)."""
        if len(outputs) == 0:
            one = self.norm_draft[0] if self.norm_draft else ""
            one = one.replace("\n\n", "\n")
            text = [self.norm_draft[0] if self.norm_draft else ""]
            toks = [self.tok.encode(json.dumps(one, ensure_ascii=False)[1:-1],
                                    add_special_tokens=False)]
            chars, where = cleaned_with_map(one)
            return text, toks, [chars], [where]
        text, toks, clean, where = [], [], [], []
        todo = [b for b in range(len(outputs)) if b not in self._finished_text]
        dec = (self.tok.batch_decode([outputs[b] for b in todo], skip_special_tokens=True)
               if todo else [])
        fresh = {}
        for b, d in zip(todo, dec):
            d = d.replace("\n\n", "\n")
            c, w = cleaned_with_map(d)
            entry = (d, self.tok.encode(json.dumps(d, ensure_ascii=False)[1:-1],
                                        add_special_tokens=False), c, w)
            fresh[b] = entry
            if finished[b]:
                self._finished_text[b] = entry
        for b in range(len(outputs)):
            d, t, c, w = self._finished_text.get(b) or fresh[b]
            text.append(d)
            toks.append(t)
            clean.append(c)
            where.append(w)
        return text, toks, clean, where

    def _pad(self, ids):
        if self.tight:
            return list(ids)
        n = len(ids)
        return list(ids) + [self.tok.pad_token_id] * (math.ceil(n / self.mil) * self.mil - n)

    def next_input(self, gen, increment, mws, pos_base, outputs, finished, next_token=None):
        """The page block's next input after a step that generated
        ``increment`` tokens (``gen``: all its tokens so far; ``mws``: its
        match window size after the step; ``outputs`` / ``finished``: the
        other blocks' generated tokens and whether they finished, or
        ``outputs`` a callable returning both, called only in text mode;
        ``next_token``: the step's next token of the block, the input of a
        normal step -- the target's own token at the last accepted node,
        which a tree fallback may have replaced in ``gen``, D:1288)."""
        self.parser.feed(self.tok.decode(gen[-increment:]) if increment else "")
        w = min(self.mws_ub, int(mws))
        window = list(gen[-w:])
        matches, trie = [], None
        self.mode = "select"
        if not (self.parser.bbox_mode or self.parser.text_mode):
            trie = self._select_trie()
        if self.parser.bbox_mode:
            self.mode = "bbox"
            trie = self._bbox_trie()
        if self.parser.text_mode:
            self.mode = "text"
            wtext = unescape_json_fragment(self.tok.decode(window))
            wclean = cleaned_with_map(wtext)[0]
            if callable(outputs):
                outputs, finished = outputs()
            text, toks, clean, where = self._others(outputs, finished)
            matches = kmp_matches(clean, wclean) if wclean else []
            trie = None if len(matches) == 1 else continuation_trie(toks, window[-1],
                                                                    self.depth)
        if len(matches) == 1:
            item, start, _ = matches[0]
            start = where[item][start + len(wclean) - 1]
            rest = json.dumps(text[item][start + 1:], ensure_ascii=False)[1:-1]
            overlap = self.tok.decode(gen[-1])
            if rest.startswith(overlap):
                rest = rest[len(overlap):]
            ids = [gen[-1]] + self.tok.encode(rest, add_special_tokens=False)
            if self.max_spec > 0 and len(ids) > self.max_spec:
                ids = ids[:self.max_spec]
            ids = self._pad(ids)
            # block_valid_counts (D:1483-1485): pad ids of the padded input are not counted
            valid = len(ids) if self.tight else len(ids) - ids.count(self.tok.pad_token_id)
            return PageInput("spec", ids, list(range(pos_base, pos_base + len(ids))), valid, 1)
        if self.tree_decode and trie is not None and trie.has_children():
            cap = min(self.cap, self.max_spec) if self.max_spec > 0 else self.cap
            tokens, depths, parents = trie.bfs(cap)
            tokens[0] = int(gen[-1])   # the root is the last generated token (D:675-684)
            n = len(tokens)
            ids = self._pad(tokens)
            pos = [d + pos_base for d in depths] + [0] * (len(ids) - n)
            return PageInput("tree", ids, pos, n, len(matches), parents, depths)
        nxt = gen[-1] if next_token is None else int(next_token)
        if self.tight:
            return PageInput("normal", [nxt], [pos_base], 1, len(matches))
        return PageInput("normal", [nxt] + [self.tok.pad_token_id] * (self.mil - 1),
                         [pos_base] + [0] * (self.mil - 1), 1, len(matches))


class HunyuanPageBlock(PageBlock):
    """The HunYuan pipeline's page block (hsd/hunyuan_ocr_pipeline/
    modeling_hunyuan_vl_hsd.py H:1900-2025): no layout parser -- every step
    matches the window's cleaned characters against the other blocks'
    decoded outputs, each prefixed with a blank line; a unique match makes
    the rest of that output (not re-escaped) the next speculative input, with
    no length cap; otherwise the continuation trie of the window over the
    re-tokenized outputs, capped at ``tree_cap`` nodes (H:2046-2104)."""

    def _others(self, outputs, finished):
        if len(outputs) == 0:
            one = self.norm_draft[0] if self.norm_draft else ""
            one = "\n\n" + one.replace("\n\n", "\n")
            chars, where = cleaned_with_map(one)
            return ([self.norm_draft[0] if self.norm_draft else ""],
                    [self.tok.encode(one, add_special_tokens=False)], [chars], [where])
        text, toks, clean, where = [], [], [], []
        todo = [b for b in range(len(outputs)) if b not in self._finished_text]
        dec = (self.tok.batch_decode([outputs[b] for b in todo], skip_special_tokens=True)
               if todo else [])
        fresh = {}
        for b, d in zip(todo, dec):
            d = "\n\n" + d.replace("\n\n", "\n")
            c, w = cleaned_with_map(d)
            entry = (d, self.tok.encode(d, add_special_tokens=False), c, w)
            fresh[b] = entry
            if finished[b]:
                self._finished_text[b] = entry
        for b in range(len(outputs)):
            d, t, c, w = self._finished_text.get(b) or fresh[b]
            text.append(d)
            toks.append(t)
            clean.append(c)
            where.append(w)
        return text, toks, clean, where

    def next_input(self, gen, increment, mws, pos_base, outputs, finished, next_token=None):
        w = min(self.mws_ub, int(mws))
        window = list(gen[-w:])
        self.mode = "text"
        wclean = cleaned_with_map(self.tok.decode(window))[0]
        if callable(outputs):
            outputs, finished = outputs()
        text, toks, clean, where = self._others(outputs, finished)
        matches = kmp_matches(clean, wclean) if wclean else []
        if len(matches) == 1:
            item, start, _ = matches[0]
            start = where[item][start + len(wclean) - 1]
            rest = text[item][start + 1:]
            overlap = self.tok.decode(gen[-1])
            if rest.startswith(overlap):
                rest = rest[len(overlap):]
            ids = self._pad([gen[-1]] + self.tok.encode(rest, add_special_tokens=False))
            valid = len(ids) if self.tight else len(ids) - ids.count(self.tok.pad_token_id)
            return PageInput("spec", ids, list(range(pos_base, pos_base + len(ids))), valid, 1)
        trie = continuation_trie(toks, window[-1], self.depth)
        if self.tree_decode and trie.has_children():
            tokens, depths, parents = trie.bfs(self.cap)
            n = len(tokens)
            ids = self._pad(tokens)
            pos = [d + pos_base for d in depths] + [0] * (len(ids) - n)
            return PageInput("tree", ids, pos, n, len(matches), parents, depths)
        nxt = gen[-1] if next_token is None else int(next_token)
        if self.tight:
            return PageInput("normal", [nxt], [pos_base], 1, len(matches))
        return PageInput("normal", [nxt] + [self.tok.pad_token_id] * (self.mil - 1),
                         [pos_base] + [0] * (self.mil - 1), 1, len(matches))

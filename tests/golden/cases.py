"""Seeded inputs shared by the fixture generator and the tests.

Every case is rebuilt from its seed, so the fixtures only hold the
reference's outputs (plus an input checksum that catches RNG drift).
"""
from __future__ import annotations

import json
import math
import random

import numpy as np
import torch

from oracle import masks as M


def kmp_cases():
    rng = random.Random(7)
    cases = []
    fixed = [
        ([], [5], 15),
        ([1, 2, 3], [1, 2, 3, 4], 15),
        ([1, 2, 3, 4], [3, 4], 15),            # match touching the tail: dropped
        ([1, 2, 3, 4, 5], [3, 4], 15),
        ([7, 7, 7, 7, 7, 7], [7, 7], 15),      # overlapping matches
        ([7, 7, 7, 7, 7, 7], [7], 3),
        ([1, 2, 1, 2, 1, 2, 1], [1, 2, 1], 2),
        ([4, 5, 6], [9], 15),
        ([9, 1, 9, 2, 9, 1, 9, 3], [9], 15),   # trie branching after the last token
    ]
    for text, pat, depth in fixed:
        cases.append(dict(texts=[text], pattern=pat, depth=depth))
    for _ in range(60):
        alpha = rng.choice([2, 3, 5, 50])
        n = rng.choice([0, 1, 5, 30, 200, 512])
        text = [rng.randrange(alpha) for _ in range(n)]
        m = rng.randint(1, 10)
        if text and rng.random() < 0.6:
            s = rng.randrange(len(text))
            pat = text[s:s + m] or [text[-1]]
        else:
            pat = [rng.randrange(alpha) for _ in range(m)]
        cases.append(dict(texts=[text], pattern=pat, depth=rng.choice([1, 15])))
    for _ in range(6):
        texts = [[rng.randrange(4) for _ in range(rng.randint(0, 40))]
                 for _ in range(rng.randint(2, 4))]
        cases.append(dict(texts=texts, pattern=[rng.randrange(4) for _ in range(3)],
                          depth=15))
    return cases


def cfg1_mask():
    """Config 1: 1024-token causal prefix + segments 64/96/128/200 (1512)."""
    segs = [64, 96, 128, 200]
    n = 1024 + sum(segs)
    allowed = np.zeros((n, n), dtype=bool)
    allowed[:1024, :1024] = np.tril(np.ones((1024, 1024), bool))
    s = 1024
    for L in segs:
        allowed[s:s + L, :1024] = True
        allowed[s:s + L, s:s + L] = np.tril(np.ones((L, L), bool))
        s += L
    return allowed


def _dense(allowed):
    m = torch.zeros((1, 1) + allowed.shape, dtype=torch.float32)
    return m.masked_fill(~torch.as_tensor(allowed)[None, None], float("-inf"))


def step_mask(seed=3, tight=False, hunyuan=False):
    """A second-step mask: inherited KV rows + spec / tree / normal blocks."""
    rng = random.Random(seed)
    lens = [rng.randint(20, 90) for _ in range(4)]
    mask = M.initial_packed_mask(lens)
    pointer = list(np.cumsum(lens) - 1)
    pointer = [p - rng.randint(0, 5) for p in pointer]
    spec = M.spec_block_mask(128)
    parents = [-1, 0, 0, 1, 1, 2, 3, 3, 5]
    tree = M.tree_block_mask(parents, 128 if not tight else len(parents))
    normal = M.normal_block_mask(128 if not tight else 1)
    blocks = [spec, tree, normal, M.spec_block_mask(37 if tight else 128)]
    new_lengths = [b.shape[0] for b in blocks]
    pad = 0
    if tight:
        tot = sum(new_lengths)
        pad = -(-tot // 128) * 128 - tot
    return M.assemble_next_mask(mask, pointer, new_lengths, blocks,
                                tight_pad_len=pad, hunyuan=hunyuan)


def blockmask_cases():
    cases = [("cfg1", _dense(cfg1_mask()))]
    small = np.zeros((200, 150), dtype=bool)
    small[:, :100] = True
    small[150:160, :] = False
    cases.append(("ragged_rows_masked", _dense(small)))
    cases.append(("step_padded", step_mask(3)))
    cases.append(("step_tight_dots", step_mask(4, tight=True)))
    cases.append(("step_tight_hunyuan", step_mask(5, tight=True, hunyuan=True)))
    return cases


def qkv(hq, hkv, q, kv, d=128, seed=0):
    torch.manual_seed(seed)
    s = 1.0 / math.sqrt(d)
    return (torch.randn(hq, q, d) * s, torch.randn(hkv, kv, d) * s,
            torch.randn(hkv, kv, d) * s)


def attention_cases():
    """(name, (q, k, v, dense_mask, scale, sample_rows))."""
    out = []
    allowed = cfg1_mask()
    q, k, v = qkv(12, 2, 1512, 1512, seed=0)
    rows = [0, 1, 127, 128, 1023, 1024, 1087, 1088, 1183, 1184, 1311, 1312,
            1400, 1511]
    out.append(("cfg1", (q, k, v, _dense(allowed), None, rows)))
    m = step_mask(3)
    qn, kvn = m.shape[-2], m.shape[-1]
    q, k, v = qkv(4, 2, qn, kvn, seed=1)
    out.append(("step_gqa4", (q, k, v, m, 0.05, [0, 5, 129, 200, 300, qn - 1])))
    small = np.zeros((200, 150), dtype=bool)
    small[:, :100] = True
    small[150:160, :] = False
    q, k, v = qkv(6, 1, 200, 150, seed=2)
    out.append(("masked_rows_mqa", (q, k, v, _dense(small), None,
                                    [0, 149, 150, 155, 160, 199])))
    return out


# ---------------------------------------------------------------- batch_generate
_WORDS = ("alpha beta gamma delta kappa omega sigma theta lambda zeta table figure "
          "value result model page line text data item score total mean rate").split()


def _sentence(rng, n_words):
    words = [str(rng.choice(_WORDS)) for _ in range(n_words)]
    if rng.random() < 0.5:
        words.insert(int(rng.integers(0, len(words))), str(int(rng.integers(10, 9999))))
    s = " ".join(words)
    return s[0].upper() + s[1:] + "."


def _perturb_chars(rng, text, p):
    out = []
    for c in text:
        u = rng.random()
        if u < p / 3:
            continue                                       # deletion
        out.append(chr(int(rng.integers(97, 123))) if u < 2 * p / 3 else c)
        if u > 1 - p / 3:
            out.append(chr(int(rng.integers(97, 123))))    # insertion
    return "".join(out)


def _page_json(texts, rng):
    cats = ["Text", "Title", "Caption", "Section-header"]
    items = []
    for i, t in enumerate(texts):
        x1, y1 = int(rng.integers(10, 500)), int(rng.integers(10, 900))
        box = [x1, y1, x1 + int(rng.integers(50, 900)), y1 + int(rng.integers(20, 90))]
        items.append('{"bbox": [%d, %d, %d, %d], "category": "%s", "text": %s}'
                     % (*box, cats[i % len(cats)], json.dumps(t)))
    return "[" + ", ".join(items) + "]"


def batch_generate_cases():
    """Seeded pages for the reference's ``batch_generate``: region blocks with
    a target text and a draft of it (clean, noisy, useless, or a periodic
    text that ends in the repetition stop), then the page block whose target
    is dots.ocr-style layout JSON quoting the region texts, so its parser
    passes through select, bbox and text modes.  Each case also names the
    loop switches (tree decoding, compaction period, tight packing, the
    speculative length cap)."""
    specs = [
        dict(name="plain_period3", seed=11, regions=3, tree=False, compact_period=3,
             tight_pack=False, max_spec_len=0, periodic=False),
        dict(name="tree_period1", seed=12, regions=4, tree=True, compact_period=1,
             tight_pack=False, max_spec_len=0, periodic=False),
        dict(name="tree_tight_period2_repeat", seed=13, regions=4, tree=True,
             compact_period=2, tight_pack=True, max_spec_len=0, periodic=True),
        dict(name="tree_tight_speccap", seed=14, regions=3, tree=True, compact_period=3,
             tight_pack=True, max_spec_len=24, periodic=False),
        dict(name="tight_never_compact", seed=15, regions=3, tree=False, compact_period=0,
             tight_pack=True, max_spec_len=0, periodic=False),
        # the logit-ratio rules below HSD_SPEC_THRESH / HSD_TREE_THRESH = 1
        # (D:1147-1174, D:1228-1266), on graded bf16 logits
        dict(name="ratio_spec", seed=16, regions=3, tree=False, compact_period=1,
             tight_pack=True, max_spec_len=0, periodic=False, spec_thresh=0.75),
        dict(name="ratio_spec_tree", seed=17, regions=3, tree=True, compact_period=2,
             tight_pack=False, max_spec_len=0, periodic=False, spec_thresh=0.8,
             tree_thresh=0.75),
    ]
    out = []
    for sp in specs:
        rng = np.random.default_rng(sp["seed"])
        texts, drafts, prompts = [], [], []
        for b in range(sp["regions"]):
            prompts.append("R%02d crop, read the text:" % b)
            if sp["periodic"] and b == 1:
                t = "xy" * 40
                d = t[:50]
            else:
                t = _sentence(rng, int(rng.integers(6, 12)))
                kind = b % 3
                d = (_perturb_chars(rng, t, 0.02) if kind == 0 else
                     _perturb_chars(rng, t, 0.12) if kind == 1 else
                     _sentence(rng, 5))
            texts.append(t)
            drafts.append(d)
        page = _page_json(texts, rng)
        prompts.append("PAGE%02d, give the layout as JSON:" % sp["seed"])
        texts.append(page)
        out.append(dict(name=sp["name"], prompts=prompts, texts=texts, drafts=drafts,
                        tree=sp["tree"], compact_period=sp["compact_period"],
                        tight_pack=sp["tight_pack"], max_spec_len=sp["max_spec_len"],
                        spec_thresh=sp.get("spec_thresh", 1.0),
                        tree_thresh=sp.get("tree_thresh", 1.0),
                        max_new_tokens=100000 if "spec_thresh" not in sp else 600))
    return out


def hunyuan_generate_cases():
    """Pages for the HunYuan loop: region blocks as in
    :func:`batch_generate_cases` and a page block whose target is the
    regions' texts as plain paragraphs (the HunYuan page output is text, not
    layout JSON); no reference run exists for these (its module needs a
    transformers model class absent here), the oracle's restatement is the
    check."""
    out = []
    for c in batch_generate_cases():
        texts = list(c["texts"][:-1])
        page = "\n\n".join(texts)
        out.append(dict(c, name="hunyuan_" + c["name"],
                        prompts=c["prompts"][:-1] + ["PAGE%s, read the page:" % c["name"][:2]],
                        texts=texts + [page]))
    return out

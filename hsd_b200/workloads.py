"""Seeded synthetic pages with the shapes of the verification workloads.

The reference measures on OmniDocBench pages with real dots.ocr / HunyuanOCR
weights and PP-StructureV3 drafts, none of which exist here; these seeded
synthetic pages stand in for them with the same shapes:

* ``stage1_regions`` -- Stage-1 region verification at dots.ocr scale
  (Qwen2-style decoder: 28 layers, 12 Q / 2 KV heads, head_dim 128).  Page
  prefix 2560 image-embedding + 64 prompt tokens; 32 region drafts packed as
  a depth-2 prefix tree (8 groups sharing a 16-token sub-prefix), draft
  lengths lognormal (median 60, sigma 0.6, cap 512), token ids uniform over a
  151936-token vocabulary.  Packing is tight (HSD_TIGHT_PACK semantics, total
  query padded to a multiple of 128 with fully masked rows).
* ``stage2_page`` -- one 3072-token causal page draft over a 4096-token prefix.
* ``hunyuan_regions`` -- 0.9B-class shapes: 24 layers, 16 Q / 8 KV heads,
  prefix 1600, 48 drafts (median 40, cap 384).
* ``multi_page`` -- pages as ``stage1_regions`` with region counts U[8, 64]
  and prefix lengths U[1024, 4096].

Each page also carries the per-block inputs of the acceptance step: the
block's draft, the tokens generated before this step, and a target argmax
stream that accepts a U(0.7, 1.0) fraction of every block (about 85%).
"""
from __future__ import annotations

import math
from dataclasses import dataclass, field

import numpy as np

VOCAB = 151936
EOS_ID = 151643  # Qwen2 <|endoftext|>; never drawn below (ids < VOCAB - 512)


@dataclass
class Segment:
    q_start: int
    q_len: int          # real tokens (no padding inside segments: tight packing)
    kind: int           # 0 causal
    sees: list          # [(lo, hi)) column ranges besides the intra pattern
    is_draft: bool
    draft: list = field(default_factory=list)   # tokenized draft of the block
    gen: list = field(default_factory=list)     # tokens generated before this step


@dataclass
class Page:
    name: str
    layers: int
    hq: int
    hkv: int
    head_dim: int
    prefix: int
    q_len: int          # padded packed query length
    q_real: int
    segments: list
    input_ids: np.ndarray
    next_ids: np.ndarray
    seed: int

    @property
    def kv_len(self):
        return self.prefix + self.q_len

    @property
    def verified_tokens(self):
        """Non-pad packed query tokens verified per step (all are draft tokens)."""
        return self.q_real


def _lognormal_lengths(rng, n, median, sigma, cap):
    x = np.exp(np.log(median) + sigma * rng.standard_normal(n))
    return np.clip(np.round(x), 1, cap).astype(int)


def _fill_block(rng, seg, ids, nxt, accept_frac):
    """Draft, generated prefix, packed input and target argmax of one block."""
    L = seg.q_len
    full = [int(t) for t in rng.integers(0, VOCAB - 512, L + 40)]
    p = 20
    seg.gen = full[:p]
    body = [full[p - 1]] + full[p:p + L - 1]
    seg.draft = full
    ids[seg.q_start:seg.q_start + L] = body
    acc = min(L - 1, int(math.floor(L * accept_frac)))
    row = [int(t) for t in rng.integers(0, VOCAB - 512, L)]
    for i in range(acc):
        row[i] = body[i + 1]
    if acc < L - 1 and row[acc] == body[acc + 1]:
        row[acc] = (row[acc] + 1) % (VOCAB - 512)
    nxt[seg.q_start:seg.q_start + L] = row


def _tree_page(name, rng, seed, layers, hq, hkv, prefix, groups, sub_prefix, drafts_per_group,
               median, sigma, cap):
    segs = []
    q = 0
    for g in range(groups):
        sp = Segment(q, sub_prefix, 0, [(0, prefix)], True)
        segs.append(sp)
        q += sub_prefix
        for L in _lognormal_lengths(rng, drafts_per_group, median, sigma, cap):
            # drafts see the page prefix and their group's sub-prefix (new columns)
            segs.append(Segment(q, int(L), 0, [(0, prefix), ("new", sp.q_start, sub_prefix)],
                                True))
            q += int(L)
    return _finish(name, rng, seed, layers, hq, hkv, prefix, segs, q)


def _finish(name, rng, seed, layers, hq, hkv, prefix, segs, q_real):
    q_len = -(-q_real // 128) * 128
    ids = np.zeros(q_len, dtype=np.int32)
    nxt = np.zeros(q_len, dtype=np.int32)
    for s in segs:
        _fill_block(rng, s, ids, nxt, float(rng.uniform(0.7, 1.0)))
    return Page(name, layers, hq, hkv, 128, prefix, q_len, q_real, segs, ids, nxt, seed)


def stage1_regions(seed=0, prefix=2624, groups=8, drafts_per_group=4):
    rng = np.random.default_rng(seed)
    return _tree_page("stage1_regions", rng, seed, 28, 12, 2, prefix, groups, 16,
                      drafts_per_group, 60, 0.6, 512)


def stage2_page(seed=0):
    rng = np.random.default_rng(seed)
    segs = [Segment(0, 3072, 0, [(0, 4096)], True)]
    return _finish("stage2_page", rng, seed, 28, 12, 2, 4096, segs, 3072)


def hunyuan_regions(seed=0):
    rng = np.random.default_rng(seed)
    segs = []
    q = 0
    for L in _lognormal_lengths(rng, 48, 40, 0.6, 384):
        segs.append(Segment(q, int(L), 0, [(0, 1600)], True))
        q += int(L)
    return _finish("hunyuan_regions", rng, seed, 24, 16, 8, 1600, segs, q)


def multi_page(index, base_seed=1000):
    rng = np.random.default_rng(base_seed + index)
    regions = int(rng.integers(8, 65))
    prefix = int(rng.integers(1024, 4097))
    groups = max(1, regions // 4)
    return _tree_page("multi_page", rng, base_seed + index, 28, 12, 2, prefix, groups, 16,
                      max(1, regions // groups), 60, 0.6, 512)


def segment_dicts(page):
    """Segment descriptors in the form ``hsd_b200.plan.PackedMask`` takes."""
    kv_len = page.kv_len
    base = kv_len - page.q_len
    out = []
    for s in page.segments:
        kv = np.zeros(kv_len, dtype=bool)
        for r in s.sees:
            if r[0] == "new":
                kv[base + r[1]:base + r[1] + r[2]] = True
            else:
                kv[r[0]:r[1]] = True
        out.append(dict(q_start=s.q_start, q_len=s.q_len, kind=s.kind, kv=kv))
    return out


WORKLOADS = {
    "stage1_regions": stage1_regions,
    "stage2_page": stage2_page,
    "hunyuan_regions": hunyuan_regions,
}

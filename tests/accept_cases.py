"""Seeded multi-block verification steps for the acceptance / KMP parity tests.

A scenario is one step of the packed loop: blocks in every mode, their
packed query rows, target argmax ids, drafts and generated prefixes, plus
the segment visibility each block's rows inherit.  ``run_oracle`` applies the
oracle restatement of the reference loop body to it.
"""
from __future__ import annotations

import copy

import numpy as np

from oracle import accept as OA
from oracle import kmp as OK
from oracle import masks as OM

PAD = 0
EOS = 99991
CAP = 2048


def make_scenario(seed, n_blocks=12, tight=False, vocab=None, last_mode=None):
    rng = np.random.default_rng(seed)
    vocab = vocab or int(rng.choice([4, 8, 30, 151936]))
    kv_old = int(rng.integers(100, 600))
    blocks, segs_q = [], []
    input_ids, next_ids = [], []
    q = 0
    for b in range(n_blocks):
        mode = int(rng.choice([OA.NORMAL, OA.SPEC, OA.SPEC, OA.TREE, OA.FINISHED]))
        if b in (0, 3):
            mode = OA.NORMAL  # 0: prefill-style block (causal rows); 3: repetition
        if b == n_blocks - 1 and last_mode is not None:
            mode = last_mode
        dlen = int(rng.integers(0, 300)) if rng.random() > 0.1 else 0
        draft = [int(x) for x in rng.integers(1, vocab, dlen)]
        if draft and rng.random() < 0.7:
            s = int(rng.integers(0, len(draft)))
            gen = draft[max(0, s - int(rng.integers(1, 30))):s + 1]
        else:
            gen = [int(x) for x in rng.integers(1, vocab, int(rng.integers(1, 40)))]
        if b == 3:  # repetition stop candidate
            gen = [5, 6] * 30
        st = dict(mode=mode, gen=gen, draft=draft, mws=int(rng.integers(1, 14)),
                  matches_len=int(rng.integers(0, 4)), valid=None, tree=None)
        ids = []
        kind, parents = OM.CAUSAL, None
        if mode == OA.FINISHED:
            blocks.append(dict(st, q_start=q, q_len=0, kind=OM.NONE))
            continue
        if mode == OA.NORMAL:
            if b == 0:
                L = int(rng.integers(20, 200))
                ids = [int(x) for x in rng.integers(1, vocab, L)]
                kind = OM.CAUSAL
                st["valid"] = L
                if not tight:
                    ids += [PAD] * ((-L) % 128)
            else:
                ids = [gen[-1]] + ([] if tight else [PAD] * 127)
                kind = OM.SINGLE
                st["valid"] = 1
            nxt = [int(x) for x in rng.integers(1, vocab, len(ids))]
            if b == 3:
                nxt[0] = 5  # continues the 5,6 loop -> repetition stop
        elif mode == OA.SPEC:
            L = int(rng.integers(1, 200))
            body = [gen[-1]] + [int(x) for x in rng.integers(1, vocab, L)]
            st["valid"] = len(body)
            ids = body + ([] if tight else [PAD] * ((-len(body)) % 128))
            agree = int(rng.integers(0, len(ids) + 1))
            nxt = [int(x) for x in rng.integers(1, vocab, len(ids))]
            for i in range(min(agree, len(ids) - 1)):
                nxt[i] = ids[i + 1]
            kind = OM.CAUSAL
        else:  # TREE
            src = draft or [int(x) for x in rng.integers(1, vocab, 50)]
            w = gen[-3:]
            trie, _ = OK.find_all_matches_kmp([src], w, OK.compute_lps(w), 15)
            if not trie.children:  # make sure there is something to walk
                trie.children[7] = OK.Node(7, 0, 0, trie.path + (7,), 1)
            toks, depths, parents = OK.trie_bfs(trie, 256)
            st["tree"] = (toks, parents)
            st["valid"] = len(toks)
            ids = list(toks) + ([] if tight else [PAD] * ((-len(toks)) % 128))
            nxt = [int(x) for x in rng.integers(1, vocab, len(ids))]
            # steer the target along a random root-to-leaf path
            node = 0
            while True:
                kids = [c for c in range(len(toks)) if parents[c] == node]
                if not kids or rng.random() < 0.15:
                    break
                c = int(rng.choice(kids))
                nxt[node] = toks[c]
                node = c
            kind = OM.TREE
        if b == 5 and mode != OA.TREE:
            nxt[0] = EOS  # EOS stop candidate
        blocks.append(dict(st, q_start=q, q_len=len(ids), kind=kind, parents=parents))
        input_ids += ids
        next_ids += nxt
        q += len(ids)
    q_len = q
    kv_len = kv_old + q_len
    segs = []
    for blk in blocks:
        kv = np.zeros(kv_len, bool)
        lo = int(rng.integers(0, kv_old))
        kv[lo:lo + int(rng.integers(1, kv_old))] = True
        kv[rng.integers(0, kv_old, 5)] = True
        blk["kv"] = kv
        if blk["q_len"]:
            d = dict(q_start=blk["q_start"], q_len=blk["q_len"], kind=blk["kind"], kv=kv)
            if blk["kind"] == OM.TREE:
                d["parents"] = blk["parents"]
            segs.append(d)
    return dict(blocks=blocks, input_ids=input_ids, next_ids=next_ids, q_len=q_len,
                kv_len=kv_len, kv_old=kv_old, segs=segs, eos=(EOS,), seed=seed)


def make_logits(sc, seed, thresh):
    """Per-row (max_logit, probe_logit) float32 arrays of bf16 values for the
    logit-ratio rules: maximal logits mostly positive (some zero or
    negative), probes at random ratios to them, a share of them placed at
    the bf16 threshold itself, where the rounding of the quotient decides."""
    rng = np.random.default_rng(10_000 + seed)
    q = sc["q_len"]
    max_l = rng.normal(6.0, 4.0, q).astype(np.float32)
    max_l[rng.random(q) < 0.05] = 0.0
    max_l = OA.bf16_f32(max_l)
    probe = OA.bf16_f32((max_l * rng.uniform(-0.2, 1.2, q)).astype(np.float32))
    at = rng.random(q) < 0.2
    probe[at] = OA.bf16_f32((max_l[at] * OA.bf16_f32(np.float32(thresh))).astype(np.float32))
    return max_l, probe


def run_oracle(sc, page_block=None, logits=None, spec_thresh=1.0, tree_thresh=1.0,
               text_mode=(), variant="dots", formula_tokens=(3, 1099), spec_mode="fmst",
               spec_topk=3, spec_margin=2.0):
    cfg = OA.StepConfig(pad_token_id=PAD, eos_token_ids=sc["eos"], spec_thresh=spec_thresh,
                        tree_thresh=tree_thresh, variant=variant, formula_tokens=formula_tokens,
                        spec_mode=spec_mode, spec_topk=spec_topk, spec_margin=spec_margin)
    allowed = OM.segments_to_allowed(sc["q_len"], sc["kv_len"], sc["segs"])
    filt = np.zeros(sc["kv_len"], bool)
    kv_base = sc["kv_len"] - sc["q_len"]
    out = []
    for i, blk in enumerate(sc["blocks"]):
        st = OA.BlockState(mode=blk["mode"], gen=list(blk["gen"]), draft=list(blk["draft"]),
                           mws=blk["mws"], matches_len=blk["matches_len"],
                           valid_count=blk["valid"])
        if blk["tree"]:
            st.tree_tokens, st.tree_parents = blk["tree"]
        st.text_mode = i in text_mode
        r = dict(finished=0, increment=0, pointer=-1, next_token=-1, match_count=0,
                 match_start=-1, slice_begin=-1, slice_end=-1)
        if blk["mode"] == OA.FINISHED:
            r["finished"] = 3
            out.append((r, st, None))
            continue
        bs, be = blk["q_start"], blk["q_start"] + blk["q_len"]
        ptr, nxt, inc, fin = OA.accept_block(
            st, bs, be, sc["next_ids"], sc["input_ids"], cfg, filt, kv_base,
            lambda row: allowed[row], is_page_block=(i == page_block), logits=logits,
            is_last_block=(i == len(sc["blocks"]) - 1))
        r.update(finished=fin, increment=inc, pointer=ptr, next_token=nxt)
        if not fin and i != page_block:
            window, matches, _ = OA.realign_block(st, cfg)
            r["match_count"] = len(matches)
            if matches:
                r["match_start"] = matches[0][1]
            if len(matches) == 1:
                r["slice_begin"] = matches[0][1] + len(window) - 1
                r["slice_end"] = matches[0][2]
        out.append((r, st, allowed[ptr].copy()))
    return out, filt

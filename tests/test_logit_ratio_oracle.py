"""Logit-ratio acceptance rules of the oracle, pinned against torch.

Below ``HSD_SPEC_THRESH`` / ``HSD_TREE_THRESH`` < 1 the reference accepts a
draft token or picks a tree child by a ratio of two bf16 logits computed
with torch on the logits tensor (D:1163-1174, D:1228-1238).  These tests
run those torch expressions on bf16 tensors and check that the oracle's
restatement (float32 quotient rounded to bf16, threshold rounded to bf16,
first maximal ratio with NaN counting as maximal) decides the same way.
"""
import numpy as np
import pytest
import torch

from oracle import accept as OA
from tests import accept_cases as AC


def _bf16_values(rng, n):
    """bf16 logits: mostly ordinary values, some zeros, negatives, ties."""
    x = rng.normal(0.0, 4.0, n).astype(np.float32)
    x[rng.random(n) < 0.05] = 0.0
    x[rng.random(n) < 0.05] = -0.0
    t = torch.from_numpy(x).to(torch.bfloat16)
    return t, t.float().numpy()


@pytest.mark.parametrize("thresh", [0.9, 0.5, 0.75, 0.99, 0.3, 1e-3])
def test_spec_ratio_matches_torch(thresh):
    rng = np.random.default_rng(int(thresh * 1000))
    ref_t, ref = _bf16_values(rng, 4096)
    pred_t, pred = _bf16_values(rng, 4096)
    # the reference's expression on bf16 tensors (D:1171)
    want = (((ref_t / pred_t) >= thresh) & (pred_t > 0)).numpy()
    got = np.array([bool(np.float32(p) > 0) and OA.ratio_passes(r, p, thresh)
                    for r, p in zip(ref, pred)])
    np.testing.assert_array_equal(got, want)
    # the quotient itself, bit for bit (NaN where torch has NaN)
    q = (ref_t / pred_t).float().numpy()
    mine = OA.logit_ratio(ref, pred)
    np.testing.assert_array_equal(np.isnan(mine), np.isnan(q))
    ok = ~np.isnan(q)
    np.testing.assert_array_equal(mine[ok].view(np.uint32), q[ok].view(np.uint32))


def test_threshold_is_compared_in_bf16():
    # 0.9 rounds to 0.8984375 in bf16: a ratio of exactly that value passes
    t = torch.tensor([0.8984375], dtype=torch.bfloat16)
    assert bool((t >= 0.9).item())
    assert OA.ratio_passes(np.float32(0.8984375), np.float32(1.0), 0.9)
    assert float(OA.bf16_f32(np.float32(0.9))) == 0.8984375


@pytest.mark.parametrize("seed", range(40))
def test_tree_fallback_choice_matches_torch(seed):
    rng = np.random.default_rng(seed)
    n_kids = int(rng.integers(1, 9))
    kid_t, kid = _bf16_values(rng, n_kids)
    if seed % 5 == 0:                      # ties among children
        kid_t[:] = kid_t[0]
        kid[:] = kid[0]
    den_t, den = _bf16_values(rng, 1)
    if seed % 7 == 0:                      # 0 / 0 gives a NaN ratio
        den_t[:] = 0.0
        den[:] = 0.0
        kid_t[0] = 0.0
        kid[0] = 0.0
    thresh = float(rng.choice([0.3, 0.5, 0.9]))
    # the reference's expressions (D:1231-1236), prob_ref a 0-d bf16 tensor
    ratio = kid_t / den_t[0]
    want_any = bool((ratio >= thresh).any())
    want_best = int(torch.argmax(ratio).item()) if want_any else None
    # oracle: a star tree, node 0 with children 1..n
    tokens = [0] + list(range(100, 100 + n_kids))
    parents = [-1] + [0] * n_kids
    probe = np.concatenate([[0.0], kid]).astype(np.float32)
    kids, ratios = OA.tree_ratio_fallback(0, tokens, parents, den[0], probe)
    assert kids == list(range(1, n_kids + 1))
    thr = OA.bf16_f32(thresh)
    got_any = any(r >= thr for r in ratios)
    assert got_any == want_any
    if want_any:
        nans = [i for i, r in enumerate(ratios) if np.isnan(r)]
        best = nans[0] if nans else int(np.argmax(ratios))
        assert best == want_best


def test_exact_thresholds_ignore_logits():
    """At the default thresholds (1.0) the logits are never read."""
    cfg = OA.StepConfig(pad_token_id=0, eos_token_ids=(2,))
    st = OA.BlockState(mode=OA.SPEC, gen=[5], draft=[5, 6, 7], valid_count=3)
    filt = np.zeros(16, bool)
    ptr, nxt, inc, fin = OA.accept_block(st, 0, 3, [6, 9, 4], [5, 6, 7], cfg, filt, 13,
                                         lambda r: np.zeros(16, bool), False, logits=None)
    assert (ptr, nxt, inc, fin) == (1, 9, 2, 0)
    assert st.gen == [5, 6, 9]


def test_spec_ratio_accepts_past_the_first_miss():
    """A miss whose ratio passes is accepted (the draft token is kept)."""
    cfg = OA.StepConfig(pad_token_id=0, eos_token_ids=(2,), spec_thresh=0.5)
    st = OA.BlockState(mode=OA.SPEC, gen=[5], draft=[], valid_count=4)
    filt = np.zeros(20, bool)
    next_ids = [6, 9, 8, 3]          # row 1 misses (9 != 7), row 2 misses (8 != 4)
    input_ids = [5, 6, 7, 4]
    max_l = np.array([3.0, 4.0, 4.0, 1.0], np.float32)
    probe = np.array([3.0, 2.0, 1.0, 0.0], np.float32)   # ratios 1, 0.5, 0.25
    ptr, nxt, inc, fin = OA.accept_block(st, 0, 4, next_ids, input_ids, cfg, filt, 16,
                                         lambda r: np.zeros(20, bool), False,
                                         logits=(max_l, probe))
    assert st.gen == [5, 6, 7, 8]    # row 1 accepted by ratio, row 2 rejected
    assert (ptr, nxt, inc) == (2, 8, 3)
    assert filt[16 + 3] and not filt[16 + 2]


def test_accept_logit_ratio_changes_decisions():
    """The ratio scenarios exercise both rules: some speculative rows and
    some tree children are accepted only through a ratio (checked on the
    oracle, so a regression to exact matching would not pass silently)."""
    spec_gain = tree_gain = 0
    for seed in range(16):
        sc = AC.make_scenario(seed, tight=bool(seed % 2))
        max_l, probe = AC.make_logits(sc, seed, 0.3)
        exact, _ = AC.run_oracle(sc)
        rng = np.random.default_rng(seed)
        text_mode = {i for i in range(len(sc["blocks"])) if rng.random() < 0.6}
        ratio, _ = AC.run_oracle(sc, logits=(max_l, probe), spec_thresh=0.3, tree_thresh=0.3,
                                 text_mode=text_mode)
        for blk, (re, _, _), (rr, _, _) in zip(sc["blocks"], exact, ratio):
            if rr["increment"] > re["increment"]:
                spec_gain += blk["mode"] == OA.SPEC
                tree_gain += blk["mode"] == OA.TREE
    assert spec_gain > 0 and tree_gain > 0, (spec_gain, tree_gain)


def _hy_cfg(**kw):
    return OA.StepConfig(pad_token_id=0, eos_token_ids=(2,), spec_thresh=0.5, variant="hunyuan",
                         formula_tokens=(3, 1099), **kw)


def _hy_spec(gen, input_ids, next_ids, max_l, probe, last=True):
    st = OA.BlockState(mode=OA.SPEC, gen=list(gen), draft=[], valid_count=len(input_ids))
    n = len(input_ids)
    filt = np.zeros(32 + n, bool)
    out = OA.accept_block(st, 0, n, next_ids, input_ids, _hy_cfg(), filt, 32,
                          lambda r: np.zeros(32 + n, bool), False,
                          logits=(np.asarray(max_l, np.float32), np.asarray(probe, np.float32)),
                          is_last_block=last)
    return st, out


def test_hunyuan_ratio_keeps_model_tokens_and_last_block_only():
    """H:1671, H:1750-1754: the ratio applies to the last block only and an
    accepted row keeps the model's token, not the draft's."""
    ids, nxt = [5, 6, 7, 8], [9, 10, 11, 12]        # every row misses
    max_l, probe = [4.0] * 4, [3.0, 3.0, 1.0, 0.0]  # ratios .75 .75 .25
    st, (ptr, tok, inc, _) = _hy_spec([4], ids, nxt, max_l, probe)
    assert st.gen == [4, 9, 10, 11] and (ptr, tok, inc) == (2, 11, 3)
    st, (ptr, tok, inc, _) = _hy_spec([4], ids, nxt, max_l, probe, last=False)
    assert st.gen == [4, 9] and (ptr, inc) == (0, 1)


def test_hunyuan_formula_rows_need_exact_match():
    """H:1681-1695: rows whose draft token is a delimiter, or that lie inside
    a formula opened by the generated tokens or the draft, use exact match
    only."""
    ratio_ok = ([4.0] * 6, [3.0] * 6)               # every ratio .75 passes
    nxt = [20, 21, 22, 23, 24, 25]                  # every row misses
    # no formula: all rows accepted by the ratio
    st, (_, _, inc, _) = _hy_spec([4], [5, 6, 7, 8, 9, 10], nxt, *ratio_ok)
    assert inc == 6
    # a '$' in the generated text opens a formula: row 0 is inside it
    st, (_, _, inc, _) = _hy_spec([4, 3, 6], [5, 6, 7, 8, 9, 10], nxt, *ratio_ok)
    assert inc == 1
    # the draft's row 2 closes it ('$$' also toggles): row 2 is a delimiter
    # (exact only), rows 0-1 inside; with exact matches on rows 0-2 the
    # ratio takes over from row 3
    ids = [5, 6, 1099, 8, 9, 10]
    nxt_exact = [6, 1099, 8, 23, 24, 25]
    st, (_, _, inc, _) = _hy_spec([4, 3], ids, nxt_exact, *ratio_ok)
    assert inc == 6
    st, (_, _, inc, _) = _hy_spec([4, 3], ids, [6, 1099, 22, 23, 24, 25], *ratio_ok)
    assert inc == 3                                 # row 2 (a delimiter) misses


@pytest.mark.parametrize("mode,k,margin,thresh", [
    ("topk", 3, 2.0, 0.5), ("topk", 1, 2.0, 0.5), ("topk", 8, 2.0, 0.9),
    ("adaptive", 3, 2.0, 0.5), ("adaptive", 3, 0.7, 0.95), ("adaptive", 3, 1.704, 0.8)])
def test_hunyuan_spec_modes_match_torch(mode, k, margin, thresh):
    """HunYuan's SPEC_MODE=topk / adaptive (H:1712-1736) as the reference
    writes them on bf16 logits rows, against the oracle's rank / second-best
    restatement.  Rows have no ties at the top-k boundary (torch leaves the
    order among equal values unspecified); the margin rows include exact
    bf16 boundary cases."""
    rng = np.random.default_rng(k * 100 + int(margin * 10))
    rows, vocab = 96, 256
    cfg = OA.StepConfig(variant="hunyuan", spec_mode=mode, spec_topk=k, spec_margin=margin)
    x = rng.normal(0.0, 3.0, (rows, vocab)).astype(np.float32)
    logits = torch.from_numpy(x).to(torch.bfloat16)
    # distinct values per row: a permutation of a bf16-exact ladder (steps
    # of 1/16 in [-8, 8) need at most 8 significant bits)
    ladder = (torch.arange(vocab, dtype=torch.float32) / 16.0 - 8.0).to(torch.bfloat16)
    for r in range(rows):
        logits[r] = ladder[torch.from_numpy(rng.permutation(vocab))]
        if r % 2:  # lift the maximum a random margin above the runner-up
            top = int(logits[r].float().argmax())
            lifted = torch.tensor(7.9375 + rng.uniform(0.0, 3.0)).to(torch.bfloat16)
            logits[r, top] = lifted
    dense = logits.float().numpy()
    pred_tok = logits.float().argmax(-1)             # first maximum, as the fused argmax keeps
    ref_tok = torch.from_numpy(np.where(rng.random(rows) < 0.5,
                                        dense.argsort(1)[:, -1 - rng.integers(0, 6, rows)]
                                        [np.arange(rows), np.arange(rows)],
                                        rng.integers(0, vocab, rows)))
    rr = torch.arange(rows)
    ref_l, pred_l = logits[rr, ref_tok], logits[rr, pred_tok]
    if mode == "topk":
        want = (logits.topk(k, dim=-1).indices == ref_tok[:, None]).any(-1).numpy()
    else:
        top2 = logits.topk(2, dim=-1).values
        mg = top2[:, 0] - top2[:, 1]
        want = ((((ref_l / pred_l) >= thresh) & (pred_l > 0))
                | ((mg < margin) & (ref_l > 0))).numpy()
    got = []
    for r in range(rows):
        rank, second = OA.rank_and_second(dense[r], int(ref_tok[r]), int(pred_tok[r]))
        got.append(OA.spec_mode_passes(cfg, dense[r, pred_tok[r]], dense[r, ref_tok[r]], thresh,
                                       rank, second))
    np.testing.assert_array_equal(np.array(got), want)


def test_rank_and_second_ties():
    """Equal logits: lower columns rank first; the second best may equal the
    best when the maximum repeats."""
    row = np.array([1.0, 3.0, 2.0, 3.0, 2.0], dtype=np.float32)
    assert OA.rank_and_second(row, 1, 1) == (0, np.float32(3.0))
    assert OA.rank_and_second(row, 3, 1) == (1, np.float32(3.0))
    assert OA.rank_and_second(row, 4, 1)[0] == 3
    assert OA.rank_and_second(row, 0, 1) == (4, np.float32(3.0))

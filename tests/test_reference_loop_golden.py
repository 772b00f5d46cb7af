"""The verification loop pinned to the reference's own ``batch_generate``.

``tests/golden/batch_generate.json`` was recorded by running the unmodified
reference loop (hsd/dots_ocr_pipeline/modeling_dots_ocr_hsd.py D:923-1810)
on the stand-in model and tokenizer of ``tests/golden/standin.py``
(``make_golden.py``): pages of region blocks plus a page block that emits
layout JSON, with tree decoding on and off, compaction periods 0-3, tight
packing and a speculative length cap.  Here the oracle's restatement of the
loop, page block included, must reproduce every forward bit for bit (packed
input ids, positions, the KV columns the previous compaction kept, the
dense mask) and the outputs (generated tokens, decode count, compaction
counters).  The page block's host module of the package is checked against
the oracle's on the same steps.
"""
import json
import os

import numpy as np
import pytest

from oracle import accept as OA
from oracle import loop as OL
from oracle import page as OP
from tests.golden import standin as SI

HERE = os.path.dirname(os.path.abspath(__file__))
CASES = json.load(open(os.path.join(HERE, "golden", "batch_generate.json")))


def _setup(case):
    tok = SI.CharTokenizer()
    prompts = [tok.encode(t) for t in case["prompts"]]
    texts = [tok.encode(t) for t in case["texts"]]
    drafts = [tok.encode(d) for d in case["drafts"]]
    cfg = OA.StepConfig(pad_token_id=SI.PAD, eos_token_ids=(SI.EOS,), min_input_length=128,
                        max_tree_depth=15, max_tree_len=256,
                        max_spec_len=int(case["max_spec_len"]),
                        tight_pack=bool(case["tight_pack"]),
                        enable_tree_decode=bool(case["tree"]),
                        spec_thresh=float(case["spec_thresh"]),
                        tree_thresh=float(case["tree_thresh"]))
    return tok, prompts, texts, drafts, cfg


def _graded(case):
    return case["spec_thresh"] < 1.0 or case["tree_thresh"] < 1.0


def _models(case, prompts, texts):
    """``(model, logits_model)`` arguments of the oracle loop for the case."""
    lm = SI.StandInLM(prompts, texts, graded=_graded(case))
    if _graded(case):
        return None, SI.oracle_logits_model(lm)
    return SI.oracle_model(lm), None


def _oracle_run(case):
    tok, prompts, texts, drafts, cfg = _setup(case)
    model, logits_model = _models(case, prompts, texts)
    page = OP.OraclePage(tok, [OP.to_halfwidth_clean(d) for d in case["drafts"]], cfg)
    gen, trace = OL.reference_loop(prompts, drafts + [[]], model, cfg,
                                   int(case["max_new_tokens"]),
                                   compact_period=int(case["compact_period"]),
                                   max_iters=5000, logits_model=logits_model, page=page)
    return gen, trace


@pytest.mark.parametrize("case", CASES, ids=[c["name"] for c in CASES])
def test_oracle_loop_reproduces_reference_batch_generate(case):
    gen, trace = _oracle_run(case)
    assert len(trace) == case["decode_times"]
    for i, (step, want) in enumerate(zip(trace, case["steps"])):
        assert SI.trace_digest(step) == want, f"step {i}"
    assert gen == case["generated"]
    calls = sum(1 for s in trace if s["action"] != "stop")
    skipped = sum(1 for s in trace if s["action"] == "mask")
    assert (calls, skipped) == (case["compact_calls"], case["compact_skipped"])


def test_fixture_cases_cover_the_page_block_modes():
    """The recorded pages drive the page block through select, bbox and
    text mode, tree and speculative inputs, and every region outcome (EOS,
    repetition stop)."""
    seen = set()
    for case in CASES:
        tok, prompts, texts, drafts, cfg = _setup(case)
        page = OP.OraclePage(tok, [], cfg)
        text = case["texts"][-1]
        for i in range(1, len(text) + 1):
            page.parser.feed(text[i - 1:i].encode())
            seen.add("text" if page.parser.text_mode else
                     "bbox" if page.parser.bbox_mode else "select")
    assert seen == {"text", "bbox", "select"}
    assert any(c["tree"] for c in CASES) and any(c["tight_pack"] for c in CASES)
    assert any(g == SI.CharTokenizer().encode(c["drafts"][1])
               for c in CASES for g in c["generated"][1:2])


@pytest.mark.parametrize("case", CASES, ids=[c["name"] for c in CASES])
def test_package_page_block_matches_oracle_page_block(case):
    """hsd_b200.page_block.PageBlock (the package's host side of the page
    block) gives the oracle's next input at every step of the recorded runs:
    same kind, ids, positions, valid rows, match count and tree parents."""
    from hsd_b200.page_block import PageBlock, halfwidth_clean

    tok, prompts, texts, drafts, cfg = _setup(case)
    model, logits_model = _models(case, prompts, texts)
    page = OP.OraclePage(tok, [OP.to_halfwidth_clean(d) for d in case["drafts"]], cfg)
    mine = PageBlock(tok, max_tree_depth=15, tree_cap=256, min_input_length=128,
                     tight_pack=cfg.tight_pack, max_spec_len=cfg.max_spec_len,
                     enable_tree_decode=cfg.enable_tree_decode,
                     norm_draft=[halfwidth_clean(d) for d in case["drafts"]])
    calls = []
    orig = page.next_input

    def both(gen, inc, mws, generated, finished, pos_base, nxt):
        want = orig(gen, inc, mws, generated, finished, pos_base, nxt)
        got = mine.next_input(list(gen), inc, mws, pos_base,
                              [list(g) for g in generated[:-1]], list(finished[:-1]), nxt)
        kind = {"causal": "spec", "tree": "tree", "single": "normal"}[want[2]]
        assert (got.kind, got.ids, got.pos, got.valid, got.matches) == (
            kind, want[0], want[1], want[3], want[4]), f"call {len(calls)}"
        if kind == "tree":
            assert got.parents == list(want[5][1])
        assert mine.parser.text_mode == page.parser.text_mode
        calls.append(kind)
        return want

    page.next_input = both
    OL.reference_loop(prompts, drafts + [[]], model, cfg,
                      int(case["max_new_tokens"]), compact_period=int(case["compact_period"]),
                      max_iters=5000, logits_model=logits_model, page=page)
    assert len(calls) == case["decode_times"] - 1
    if case["tree"]:
        assert "tree" in calls and "spec" in calls

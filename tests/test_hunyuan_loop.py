"""The HunYuan variant of the loop on the host side.

The HunYuan pipeline's module (hsd/hunyuan_ocr_pipeline/
modeling_hunyuan_vl_hsd.py) cannot be imported here, so its loop is checked
through the oracle's restatement (``oracle.page.OracleHunyuanPage`` and
``oracle.loop.reference_loop`` with ``variant="hunyuan"``): verified
generation reproduces every block's target text, and the package's
``HunyuanPageBlock`` gives the oracle's next input at every step.
"""
import pytest

from oracle import accept as OA
from oracle import loop as OL
from oracle import page as OP
from tests.golden import cases as GC
from tests.golden import standin as SI

CASES = GC.hunyuan_generate_cases()


def hunyuan_setup(case):
    tok = SI.CharTokenizer()
    prompts = [tok.encode(t) for t in case["prompts"]]
    texts = [tok.encode(t) for t in case["texts"]]
    norm = [OP.to_halfwidth_clean(d) for d in case["drafts"]]
    drafts = [tok.encode(d) for d in norm]
    cfg = OA.StepConfig(pad_token_id=SI.PAD, eos_token_ids=(SI.EOS,), min_input_length=128,
                        max_tree_depth=15, max_tree_len=128, max_spec_len=0,
                        tight_pack=bool(case["tight_pack"]),
                        enable_tree_decode=bool(case["tree"]), repeat_sentinel=41153,
                        variant="hunyuan")
    return tok, prompts, texts, drafts, norm, cfg


def oracle_hunyuan_run(case, hook=None):
    tok, prompts, texts, drafts, norm, cfg = hunyuan_setup(case)
    lm = SI.StandInLM(prompts, texts)
    page = OP.OracleHunyuanPage(tok, norm, cfg)
    if hook is not None:
        hook(page, norm, cfg, tok)
    return OL.reference_loop(prompts, drafts + [[]], SI.oracle_model(lm), cfg,
                             int(case["max_new_tokens"]),
                             compact_period=int(case["compact_period"]), max_iters=5000,
                             page=page)


@pytest.mark.parametrize("case", CASES, ids=[c["name"] for c in CASES])
def test_oracle_hunyuan_loop_reproduces_texts(case):
    tok = SI.CharTokenizer()
    gen, trace = oracle_hunyuan_run(case)
    for b, (g, t) in enumerate(zip(gen, case["texts"])):
        if case["name"].endswith("repeat") and b == 1:
            continue            # repetition stop: the draft replaces the output
        if b == len(gen) - 1:
            assert tok.decode(g) == t       # the page block ran to its end
        else:                               # the loop ends with the page block (H:2135)
            assert t.startswith(tok.decode(g)), b
    assert len(trace) < len(case["texts"][-1])   # the page block took multi-token steps


@pytest.mark.parametrize("case", CASES, ids=[c["name"] for c in CASES])
def test_package_hunyuan_page_block_matches_oracle(case):
    from hsd_b200.page_block import HunyuanPageBlock
    calls = []

    def hook(page, norm, cfg, tok):
        mine = HunyuanPageBlock(tok, max_tree_depth=15, tree_cap=128, min_input_length=128,
                                tight_pack=cfg.tight_pack,
                                enable_tree_decode=cfg.enable_tree_decode, norm_draft=norm)
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
            calls.append(kind)
            return want
        page.next_input = both

    oracle_hunyuan_run(case, hook)
    assert calls and "spec" in calls

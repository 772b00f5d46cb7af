"""The multi-step verification loop: oracle restatement and device loop.

The synthetic target model continues each block's true text whenever the
context matches it, so verified generation must reproduce the true texts
exactly (speculative decoding is lossless), whatever the drafts.  The device
loop must follow the oracle loop step by step: the same packed inputs and
positions, the same dense mask (read back from the device tile plan) and the
same generated tokens.
"""
import numpy as np
import pytest
import torch

from oracle import accept as OA
from oracle import loop as OL
from tests import loop_cases as LC

MIL = 16


def _cfg(tree=False, tight=False):
    return OA.StepConfig(pad_token_id=LC.PAD, eos_token_ids=(LC.EOS,), min_input_length=MIL,
                         enable_tree_decode=tree, tight_pack=tight)


@pytest.mark.parametrize("seed,tree", [(0, False), (1, False), (2, False), (3, True),
                                       (4, True)])
def test_oracle_loop_reproduces_true_texts(seed, tree):
    prompts, truths, drafts = LC.make_loop_case(seed)
    model = OL.true_text_model(prompts, truths, LC.VOCAB, LC.EOS)
    gen, trace = OL.reference_loop(prompts, drafts, model, _cfg(tree), max_new_tokens=10 ** 6)
    if tree:  # tree blocks were proposed and walked
        assert any(OA.TREE in s["modes"] for s in trace)
    for b, (g, t) in enumerate(zip(gen, truths)):
        if b % 4 == 3:   # repetition stop: the draft replaces the output
            assert g == drafts[b]
        else:
            assert g == list(map(int, t)), b
    # drafts save steps: fewer forwards than the longest text has tokens
    assert len(trace) < max(len(t) for t in truths)


@pytest.mark.parametrize("seed,tree", [(0, False), (2, False), (3, True)])
def test_oracle_tight_loop_reproduces_true_texts(seed, tree):
    """HSD_TIGHT_PACK: unpadded blocks, the packed input padded to a
    multiple of 128 rows (D:1619-1632); the texts are those of the padded
    loop, with fewer packed rows."""
    prompts, truths, drafts = LC.make_loop_case(seed)
    model = OL.true_text_model(prompts, truths, LC.VOCAB, LC.EOS)
    gen, trace = OL.reference_loop(prompts, drafts, model, _cfg(tree, tight=True),
                                   max_new_tokens=10 ** 6)
    gen_pad, trace_pad = OL.reference_loop(prompts, drafts, model, _cfg(tree),
                                           max_new_tokens=10 ** 6)
    assert gen == gen_pad
    for s in trace[1:]:
        assert len(s["input_ids"]) % OL.Q_BLOCK == 0
        assert (s["input_ids"][s["q_blocks"]:] == LC.PAD).all()
        assert not s["allowed"][s["q_blocks"]:, -len(s["input_ids"]):].any()
    assert sum(s["q_blocks"] for s in trace[1:]) < sum(len(s["input_ids"]) for s in trace_pad[1:])


@pytest.mark.gpu
@pytest.mark.parametrize("seed,period,tree,tight", [
    (0, 1, False, False), (1, 1, False, False), (2, 3, False, False), (3, 1, True, False),
    (4, 2, True, False), (0, 1, False, True), (2, 2, False, True), (3, 1, True, True)])
def test_device_loop_follows_oracle_loop(seed, period, tree, tight):
    """Same inputs, positions, mask and tokens at every step.  With tight
    packing the rows past the blocks see no column on the device (no block
    reads them, their columns are filtered); the block rows' masks match."""
    from hsd_b200.loop import VerifyLoop
    assert torch.cuda.is_available(), "GPU tests need a CUDA device"
    dev = torch.device("cuda:0")
    prompts, truths, drafts = LC.make_loop_case(seed)
    model = OL.true_text_model(prompts, truths, LC.VOCAB, LC.EOS)
    ref_gen, trace = OL.reference_loop(prompts, drafts, model, _cfg(tree, tight),
                                       max_new_tokens=10 ** 6, compact_period=period)
    loop = VerifyLoop(prompts, drafts, eos_token_id=LC.EOS, max_new_tokens=10 ** 6,
                      pad_token_id=LC.PAD, min_input_length=MIL, compact_period=period,
                      enable_tree_decode=tree, tight_pack=tight, device=dev)
    for it, ref in enumerate(trace):
        ids, pos, mask = loop.inputs()
        np.testing.assert_array_equal(ids.cpu().numpy(), ref["input_ids"], err_msg=f"step {it}")
        np.testing.assert_array_equal(pos.cpu().numpy(), ref["position_ids"])
        plan = mask.plan()
        allowed = plan.dense_allowed()
        plan.raise_on_device_error()
        assert allowed.shape == ref["allowed"].shape, (it, allowed.shape, ref["allowed"].shape)
        qb = ref["q_blocks"]
        np.testing.assert_array_equal(allowed[:qb], ref["allowed"][:qb], err_msg=f"mask, step {it}")
        assert not allowed[qb:].any(), it
        kv_tokens = loop.kv_tokens.cpu().numpy()
        nxt = model(ref["input_ids"], ref["position_ids"], allowed, kv_tokens)
        more = loop.step(torch.from_numpy(nxt).to(dev))
        assert more == (it + 1 < len(trace)), it
    assert loop.generated() == ref_gen


@pytest.mark.gpu
def test_batch_generate_returns_true_texts():
    from hsd_b200.loop import batch_generate
    dev = torch.device("cuda:0")
    prompts, truths, drafts = LC.make_loop_case(5)
    model = OL.true_text_model(prompts, truths, LC.VOCAB, LC.EOS)
    ref_gen, trace = OL.reference_loop(prompts, drafts, model, _cfg(), max_new_tokens=10 ** 6)

    def model_fn(ids, pos, mask, kv_tokens):
        allowed = mask.plan().dense_allowed()
        return torch.from_numpy(model(ids.cpu().numpy(), pos.cpu().numpy(), allowed,
                                      kv_tokens.cpu().numpy())).to(dev)

    gen, decode_times, timings = batch_generate(
        model_fn, prompts, drafts, eos_token_id=LC.EOS, max_new_tokens=10 ** 6,
        pad_token_id=LC.PAD, min_input_length=MIL, device=dev)
    assert gen == ref_gen
    assert decode_times == len(trace)
    assert len(timings) == 8 and timings[6] == decode_times - 1


@pytest.mark.gpu
@pytest.mark.parametrize("seed,period,tree", [(0, 1, False), (2, 3, False), (3, 1, True)])
def test_registered_caches_follow_the_loops_columns(seed, period, tree):
    """A model's K/V caches registered with the loop (``kv_planes``) are
    compacted in place with its columns: every row of every plane encodes
    the token of its KV column (and the plane's index), and after every
    step's compaction the rows in front of the new ones still spell the
    loop's ``kv_tokens`` exactly."""
    from hsd_b200.compaction import plane_pointers
    from hsd_b200.loop import VerifyLoop
    assert torch.cuda.is_available(), "GPU tests need a CUDA device"
    dev = torch.device("cuda:0")
    prompts, truths, drafts = LC.make_loop_case(seed)
    model = OL.true_text_model(prompts, truths, LC.VOCAB, LC.EOS)
    ref_gen, _ = OL.reference_loop(prompts, drafts, model, _cfg(tree), max_new_tokens=10 ** 6,
                                   compact_period=period)
    cap = 4096
    caches = [torch.zeros(2, cap, 128, dtype=torch.bfloat16, device=dev) for _ in range(4)]
    planes = plane_pointers(caches, device=dev)
    n_planes = 2 * len(caches)
    loop = VerifyLoop(prompts, drafts, eos_token_id=LC.EOS, max_new_tokens=10 ** 6,
                      pad_token_id=LC.PAD, min_input_length=MIL, compact_period=period,
                      enable_tree_decode=tree, kv_planes=planes, row_bytes=256,
                      kv_capacity=cap, device=dev)
    plane_id = torch.arange(n_planes, device=dev, dtype=torch.float32).view(4, 2, 1)

    def check(n, tokens):
        for t, c in enumerate(caches):
            rows = c[:, :n, :3].float()                         # [2, n, 3]
            got = (rows[..., 0] * 256 + rows[..., 1]).long()
            assert torch.equal(got, tokens.long().expand(2, n)), (t, n)
            assert torch.equal(rows[..., 2], plane_id[t].expand(2, n))

    for it in range(1000):
        ids, pos, mask = loop.inputs()
        kv_tokens = loop.kv_tokens
        total, q = kv_tokens.numel(), ids.numel()
        check(total - q, kv_tokens[:total - q])
        # the model's cache update: rows of the step's new columns
        vals = torch.zeros(q, 128, dtype=torch.float32, device=dev)
        vals[:, 0] = (ids // 256).float()
        vals[:, 1] = (ids % 256).float()
        for t, c in enumerate(caches):
            for h in range(2):
                vals[:, 2] = float(plane_id[t, h, 0])
                c[h, total - q:total] = vals.to(torch.bfloat16)
        allowed = mask.plan().dense_allowed()
        nxt = model(ids.cpu().numpy(), pos.cpu().numpy(), allowed, kv_tokens.cpu().numpy())
        if not loop.step(torch.from_numpy(nxt).to(dev)):
            break
    assert loop.generated() == ref_gen


RATIO_CASES = [(0, False, 0.3, 1.0, {1, 2, 4}), (3, True, 0.3, 0.3, {1, 2, 4}),
               (4, True, 1.0, 0.3, {0, 1, 2, 3, 4, 5}), (7, True, 0.5, 0.5, {0, 2, 3, 5})]


def _ratio_cfg(tree, spec_t, tree_t, variant="dots"):
    return OA.StepConfig(pad_token_id=LC.PAD, eos_token_ids=(LC.EOS,), min_input_length=MIL,
                         enable_tree_decode=tree, spec_thresh=spec_t, tree_thresh=tree_t,
                         variant=variant, formula_tokens=(3, 5))


@pytest.mark.parametrize("seed,tree,spec_t,tree_t,text", RATIO_CASES)
def test_oracle_ratio_loop_departs_from_exact(seed, tree, spec_t, tree_t, text):
    """Thresholds below 1 change what the loop generates (the rules are
    exercised), while a logits model at the default thresholds generates
    exactly what the token model does."""
    prompts, truths, drafts = LC.make_loop_case(seed)
    model = OL.true_text_model(prompts, truths, LC.VOCAB, LC.EOS)
    lm = LC.logits_model(model, seed)
    ratio, _ = OL.reference_loop(prompts, drafts, model, _ratio_cfg(tree, spec_t, tree_t), 400,
                                 logits_model=lm, text_mode=text)
    exact_lm, _ = OL.reference_loop(prompts, drafts, model, _ratio_cfg(tree, 1.0, 1.0), 400,
                                    logits_model=lm, text_mode=text)
    exact, _ = OL.reference_loop(prompts, drafts, model, _cfg(tree), 400)
    assert exact_lm == exact
    assert ratio != exact


HUNYUAN_CASES = [(3, True, 0.5, 1.0, {0, 1, 2, 3, 4, 5}, 0), (0, False, 0.3, 1.0, {5}, 2),
                 (8, True, 0.5, 1.0, {1, 3, 5}, 0)]


@pytest.mark.parametrize("seed,tree,spec_t,tree_t,text,period", HUNYUAN_CASES)
def test_oracle_hunyuan_loop_departs_from_dots(seed, tree, spec_t, tree_t, text, period):
    """The HunYuan rules (last-block ratio outside formulas, model tokens
    kept, tree fallback at threshold 1, period-0 compaction) generate
    differently from the dots rules on the same logits."""
    prompts, truths, drafts = LC.make_loop_case(seed)
    model = OL.true_text_model(prompts, truths, LC.VOCAB, LC.EOS)
    lm = LC.logits_model(model, seed)
    hy, hy_trace = OL.reference_loop(prompts, drafts, model,
                                     _ratio_cfg(tree, spec_t, tree_t, "hunyuan"), 400,
                                     compact_period=period, logits_model=lm, text_mode=text)
    dots, dots_trace = OL.reference_loop(prompts, drafts, model, _ratio_cfg(tree, spec_t, tree_t),
                                         400, compact_period=period, logits_model=lm,
                                         text_mode=text)
    assert hy != dots or [s["action"] for s in hy_trace] != [s["action"] for s in dots_trace]


SPEC_MODE_CASE = (1, False, 0.5, 1.0, {5}, 1)


@pytest.mark.parametrize("mode,k,margin", [("topk", 3, 2.0), ("adaptive", 3, 50.0)])
def test_oracle_hunyuan_spec_modes_depart_from_fmst(mode, k, margin):
    """SPEC_MODE=topk / adaptive (H:1712-1736) accept differently from the
    default logit ratio on the same logits model (whose top-2 margins are
    all above 2, so the adaptive case widens the margin)."""
    seed, tree, spec_t, tree_t, text, period = SPEC_MODE_CASE
    prompts, truths, drafts = LC.make_loop_case(seed)
    model = OL.true_text_model(prompts, truths, LC.VOCAB, LC.EOS)
    lm = LC.logits_model(model, seed)
    cfg = _ratio_cfg(tree, spec_t, tree_t, "hunyuan")
    fmst, fmst_trace = OL.reference_loop(prompts, drafts, model, cfg, 400, compact_period=period,
                                         logits_model=lm, text_mode=text)
    cfg.spec_mode, cfg.spec_topk, cfg.spec_margin = mode, k, margin
    got, trace = OL.reference_loop(prompts, drafts, model, cfg, 400, compact_period=period,
                                   logits_model=lm, text_mode=text)
    assert got != fmst or len(trace) != len(fmst_trace)


@pytest.mark.gpu
@pytest.mark.parametrize("seed,tree,spec_t,tree_t,text,variant,period,spec_mode",
                         [c + ("dots", 1, "fmst") for c in RATIO_CASES] +
                         [c[:5] + ("hunyuan", c[5], "fmst") for c in HUNYUAN_CASES] +
                         [SPEC_MODE_CASE[:5] + ("hunyuan", SPEC_MODE_CASE[5], m)
                          for m in ("topk", "adaptive")])
def test_device_ratio_loop_follows_oracle_loop(seed, tree, spec_t, tree_t, text, variant, period,
                                               spec_mode):
    """The device loop below the default thresholds (and with the HunYuan
    rules): per step the same inputs as the oracle loop, the logits it reads
    listed by ``logit_probes``, and the same generated tokens."""
    from hsd_b200.loop import VerifyLoop
    dev = torch.device("cuda:0")
    prompts, truths, drafts = LC.make_loop_case(seed)
    model = OL.true_text_model(prompts, truths, LC.VOCAB, LC.EOS)
    lm = LC.logits_model(model, seed)
    cfg = _ratio_cfg(tree, spec_t, tree_t, variant)
    cfg.spec_mode = spec_mode
    cfg.spec_margin = 50.0   # adaptive: the margin rule fires wherever the draft logit is > 0
    ref_gen, trace = OL.reference_loop(prompts, drafts, model, cfg, 400,
                                       compact_period=period, logits_model=lm, text_mode=text)
    loop = VerifyLoop(prompts, drafts, eos_token_id=LC.EOS, max_new_tokens=400,
                      pad_token_id=LC.PAD, min_input_length=MIL, enable_tree_decode=tree,
                      spec_thresh=spec_t, tree_thresh=tree_t, variant=variant,
                      formula_tokens=(3, 5), compact_period=period, spec_mode=spec_mode,
                      spec_margin=cfg.spec_margin, device=dev)
    flags = [b in text for b in range(len(prompts))]
    for it, ref in enumerate(trace):
        ids, pos, mask = loop.inputs()
        np.testing.assert_array_equal(ids.cpu().numpy(), ref["input_ids"], err_msg=f"step {it}")
        np.testing.assert_array_equal(pos.cpu().numpy(), ref["position_ids"])
        allowed = mask.plan().dense_allowed()
        dense = lm(ref["input_ids"], ref["position_ids"], allowed, loop.kv_tokens.cpu().numpy())
        nxt = np.argmax(dense, axis=1)
        rows, toks = (t.cpu().numpy() for t in loop.logit_probes())
        probe = np.where(toks >= 0, dense[rows, np.maximum(toks, 0)], 0).astype(np.float32)
        max_l = dense[np.arange(len(nxt)), nxt].astype(np.float32)
        extra = {}
        if spec_mode != "fmst":   # the rank pass's outputs, here from the dense logits
            q = len(nxt)
            rs = [OA.rank_and_second(dense[r], int(ref["input_ids"][r + 1]), int(nxt[r]))
                  for r in range(q - 1)] + [(0, -np.inf)]
            extra = dict(rank=torch.tensor([x[0] for x in rs], dtype=torch.int32, device=dev),
                         second=torch.tensor(np.float32([x[1] for x in rs]), device=dev))
        more = loop.step(torch.from_numpy(nxt).to(dev), max_logit=torch.from_numpy(max_l).to(dev),
                         probe_logit=torch.from_numpy(probe).to(dev), text_mode=flags, **extra)
        assert more == (it + 1 < len(trace)), it
    assert loop.generated() == ref_gen

"""The drop-in ``batch_generate`` against the reference's own runs
(including runs below the default logit-ratio thresholds, on graded bf16
logits).

``hsd_b200.generate.batch_generate`` has the signature and return value of
the reference's ``DotsOCRForCausalLM.batch_generate``
(hsd/dots_ocr_pipeline/modeling_dots_ocr_hsd.py D:923-1810).  Driven by the
same stand-in model and tokenizer as the recorded reference runs
(tests/golden/batch_generate.json, see make_golden.py), on the GPU, every
forward must receive bit-identical inputs -- packed input ids, positions,
the KV columns left by the previous compaction (the model's own cache,
compacted in place by the package) and the attention mask read back from
the device tile plan -- and the call must return the same generated tokens,
decode count and compaction counters.
"""
import json
import os

import pytest
import torch

from tests.golden import standin as SI

pytestmark = pytest.mark.gpu

HERE = os.path.dirname(os.path.abspath(__file__))
CASES = json.load(open(os.path.join(HERE, "golden", "batch_generate.json")))


@pytest.mark.parametrize("case", CASES, ids=[c["name"] for c in CASES])
def test_drop_in_batch_generate_matches_reference_runs(case, monkeypatch):
    from hsd_b200.generate import batch_generate
    assert torch.cuda.is_available(), "GPU tests need a CUDA device"
    dev = torch.device("cuda:0")
    monkeypatch.setenv("HSD_TIGHT_PACK", "1" if case["tight_pack"] else "0")
    monkeypatch.setenv("HSD_COMPACT_PERIOD", str(case["compact_period"]))
    monkeypatch.setenv("HSD_MAX_SPEC_LEN", str(case["max_spec_len"]))
    monkeypatch.setenv("HSD_SPEC_THRESH", str(case["spec_thresh"]))
    monkeypatch.setenv("HSD_TREE_THRESH", str(case["tree_thresh"]))
    tok = SI.CharTokenizer()
    prompts = [tok.encode(t) for t in case["prompts"]]
    texts = [tok.encode(t) for t in case["texts"]]
    graded = case["spec_thresh"] < 1.0 or case["tree_thresh"] < 1.0
    model = SI.StandInLM(prompts, texts, graded=graded)   # bf16 logits for the ratio rules
    ids, mask, pos, pointer = SI.packed_prefill(prompts, device=dev)
    drafts = [{"block_content": d, "raw_block_content": d} for d in case["drafts"]]
    gen, decode_times, stats = batch_generate(
        model, input_ids=ids, attention_mask=mask, position_ids=pos, pointer=pointer,
        tokenizer=tok, draft=drafts, enable_tree_decode=bool(case["tree"]),
        eos_token_id=[SI.EOS], max_new_tokens=int(case["max_new_tokens"]))
    assert model.model.config._attn_implementation == "eager"   # restored
    for i, (t, want) in enumerate(zip(model.trace, case["steps"])):
        assert SI.step_digest(t) == want, f"step {i}"
    assert len(model.trace) == len(case["steps"])
    assert gen == case["generated"]
    assert decode_times == case["decode_times"]
    assert (stats[6], stats[7]) == (case["compact_calls"], case["compact_skipped"])
    assert len(stats) == 8


HCASES = __import__("tests.golden.cases", fromlist=["x"]).hunyuan_generate_cases()


@pytest.mark.parametrize("case", HCASES, ids=[c["name"] for c in HCASES])
def test_hunyuan_drop_in_matches_oracle_loop(case, monkeypatch):
    """The HunYuan drop-in (``batch_generate_hunyuan``, the H:1426-1448
    signature) against the oracle's restatement of the HunYuan loop on the
    same stand-in model: bit-identical forwards (ids, row-0 positions of the
    ``[1, 4, Q]`` position ids, kept KV columns, mask) and the dict return
    of H:2324-2343."""
    from hsd_b200.generate import batch_generate_hunyuan
    from tests.test_hunyuan_loop import oracle_hunyuan_run
    dev = torch.device("cuda:0")
    monkeypatch.setenv("HSD_TIGHT_PACK", "1" if case["tight_pack"] else "0")
    monkeypatch.setenv("HSD_COMPACT_PERIOD", str(case["compact_period"]))
    gen_ref, trace = oracle_hunyuan_run(case)
    tok = SI.CharTokenizer()
    prompts = [tok.encode(t) for t in case["prompts"]]
    texts = [tok.encode(t) for t in case["texts"]]
    model = SI.StandInLM(prompts, texts)
    ids, mask, pos, pointer = SI.packed_prefill(prompts, device=dev)
    pos4 = pos[:, None].expand(1, 4, -1)
    drafts = [{"block_content": d} for d in case["drafts"]]
    out = batch_generate_hunyuan(
        model, input_ids=ids, attention_mask=mask, position_ids=pos4, pointer=pointer,
        tokenizer=tok, draft=drafts, enable_tree_decode=bool(case["tree"]),
        eos_token_id=[SI.EOS], max_new_tokens=int(case["max_new_tokens"]))
    assert len(model.trace) == len(trace)
    for i, (t, ref) in enumerate(zip(model.trace, trace)):
        assert SI.step_digest(t) == SI.trace_digest(ref), f"step {i}"
    assert out["generated_tokens"] == gen_ref
    assert out["decode_times"] == len(trace)
    assert out["decode_token_num"] == len(gen_ref[-1])
    used = out["used_time"]
    assert used["kv_compact_calls"] == sum(1 for s in trace if s["action"] != "stop")
    assert used["kv_compact_skipped"] == sum(1 for s in trace if s["action"] == "none")
    assert len(out["compute_intensity"]) == len(trace)


def _tiny_qwen2(dev):
    from transformers.models.qwen2.modeling_qwen2 import Qwen2Config, Qwen2ForCausalLM
    torch.manual_seed(0)
    cfg = Qwen2Config(vocab_size=SI.VOCAB, hidden_size=256, intermediate_size=512,
                      num_hidden_layers=2, num_attention_heads=2, num_key_value_heads=1,
                      head_dim=128, rope_theta=1e6, max_position_embeddings=8192,
                      initializer_range=0.5, tie_word_embeddings=False)
    return Qwen2ForCausalLM(cfg).to(dev, torch.bfloat16).eval()


@pytest.mark.parametrize("tree", [False, True])
def test_drop_in_on_a_transformers_qwen2(tree, monkeypatch):
    """The drop-in driving a real transformers decoder (a small random
    Qwen2ForCausalLM, head_dim 128, bf16): its attention layers run through
    the registered "hsd_b200" attention on the caller's dense prefill mask
    and then on each step's PackedMask, its DynamicCache is compacted in
    place, and the config's attention implementation is restored.  With
    ``fused_lm_head`` the decoder runs alone and the fused lm_head + argmax
    picks the tokens: the same run, token for token, as the logits path."""
    from hsd_b200.generate import batch_generate
    dev = torch.device("cuda:0")
    monkeypatch.setenv("HSD_TIGHT_PACK", "1")
    monkeypatch.setenv("HSD_COMPACT_PERIOD", "1")
    case = CASES[1]
    tok = SI.CharTokenizer()
    prompts = [tok.encode(t) for t in case["prompts"]]
    drafts = [{"block_content": d, "raw_block_content": d} for d in case["drafts"]]
    model = _tiny_qwen2(dev)
    impl = model.config._attn_implementation
    runs = []
    for fused in (False, True):
        ids, mask, pos, pointer = SI.packed_prefill(prompts, device=dev)
        gen, decode_times, stats = batch_generate(
            model, input_ids=ids, attention_mask=mask, position_ids=pos, pointer=pointer,
            tokenizer=tok, draft=drafts, enable_tree_decode=tree, eos_token_id=[SI.EOS],
            max_new_tokens=160, fused_lm_head=fused)
        runs.append((gen, decode_times, stats[6], stats[7]))
        assert model.config._attn_implementation == impl
        assert decode_times > 3 and stats[6] == decode_times - 1
    assert runs[0] == runs[1]

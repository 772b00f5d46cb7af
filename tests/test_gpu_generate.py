"""The drop-in ``batch_generate`` against the reference's own runs.

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
    tok = SI.CharTokenizer()
    prompts = [tok.encode(t) for t in case["prompts"]]
    texts = [tok.encode(t) for t in case["texts"]]
    model = SI.StandInLM(prompts, texts)
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

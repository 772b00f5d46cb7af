"""Generate the golden fixtures that pin the oracle to the reference.

Run in a container where the reference checkout is present:

    python tests/golden/make_golden.py /path/to/reference [kmp|blockmask|attention|batch_generate ...]

(or set ``HSD_REFERENCE_ROOT``).

It imports ``hsd/dots_ocr_pipeline/modeling_dots_ocr_hsd.py`` from the
reference and records, for seeded inputs:

* ``kmp.json``        -- ``compute_lps`` and ``find_all_matches_kmp`` outputs
                         (matches and the continuation trie) (D:543-618);
* ``blockmask.json``  -- ``create_block_mask(make_mask_mod(mask), ...,
                         BLOCK_SIZE=(128, 64))`` lists for several packed
                         masks (D:94-106, D:148-153);
* ``attention_*.npz`` -- ``flex_attention_forward`` outputs (D:72-135) with
                         the module's ``torch.compile``d FlexAttention swapped
                         for the eager one, because the compiled kernel
                         rejects ``return_lse`` on the CPU;
* ``batch_generate.json`` -- the unmodified ``DotsOCRForCausalLM.batch_generate``
                         (D:923-1810) driven by the stand-in model and
                         tokenizer of ``standin.py`` over packed pages of
                         region blocks and a layout-JSON page block: every
                         forward's packed input ids, positions, the KV
                         columns the previous compaction kept and a hash of
                         the dense mask, then the generated tokens, the
                         decode count and the compaction counters.

The fixtures are committed; tests read them without the reference.
"""
from __future__ import annotations

import json
import math
import os
import random
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))

from tests.golden.cases import (attention_cases, blockmask_cases,  # noqa: E402
                                kmp_cases)


def _import_reference(root):
    sys.path.insert(0, root)
    import hsd.dots_ocr_pipeline.modeling_dots_ocr_hsd as ref  # noqa: E402
    from torch.nn.attention.flex_attention import flex_attention
    ref.flex_attention = flex_attention  # eager: the compiled one cannot return LSE on CPU
    return ref


def _ser(node):
    return [node.value, [_ser(c) for c in node.children.values()]]


def make_kmp(ref):
    out = []
    for case in kmp_cases():
        lps = ref.compute_lps(case["pattern"])
        trie, matches = ref.find_all_matches_kmp(case["texts"], case["pattern"],
                                                 lps, case["depth"])
        out.append(dict(case, lps=lps, matches=[list(m) for m in matches],
                        trie=_ser(trie)))
    with open(os.path.join(HERE, "kmp.json"), "w") as f:
        json.dump(out, f)
    return len(out)


def make_blockmask(ref):
    from torch.nn.attention.flex_attention import create_block_mask
    out = []
    for name, mask in blockmask_cases():
        causal = mask[:, :, :, :mask.shape[-1]]
        mm = ref.make_mask_mod(causal, 128, 64)
        bm = create_block_mask(mm, None, None, mask.shape[-2], mask.shape[-1],
                               device="cpu", BLOCK_SIZE=(128, 64))
        kn = bm.kv_num_blocks[0, 0].tolist()
        fn = bm.full_kv_num_blocks[0, 0].tolist()
        ki = [bm.kv_indices[0, 0, i, :n].tolist() for i, n in enumerate(kn)]
        fi = [bm.full_kv_indices[0, 0, i, :n].tolist() for i, n in enumerate(fn)]
        out.append(dict(name=name, q=mask.shape[-2], kv=mask.shape[-1],
                        kv_num_blocks=kn, kv_indices=ki,
                        full_kv_num_blocks=fn, full_kv_indices=fi))
    with open(os.path.join(HERE, "blockmask.json"), "w") as f:
        json.dump(out, f)
    return len(out)


def make_attention(ref):
    n = 0
    for name, (q, k, v, mask, scale, sample_rows) in attention_cases():
        out, lse = ref.flex_attention_forward(None, q[None], k[None], v[None],
                                              mask, scaling=scale)
        out = out[0].float().numpy()            # [Q, Hq, D]
        g = torch.Generator().manual_seed(1234)
        proj = torch.randn(out.shape[-1], 2, generator=g).numpy()
        np.savez_compressed(
            os.path.join(HERE, f"attention_{name}.npz"),
            input_checksum=np.array([float(q.double().sum()),
                                     float(k.double().sum()),
                                     float(v.double().sum())]),
            lse=lse[0].float().numpy(),
            out_proj=(out @ proj).astype(np.float32),
            sample_rows=np.asarray(sample_rows, dtype=np.int64),
            out_rows=out[np.asarray(sample_rows)].astype(np.float32))
        n += 1
    return n


def run_reference_batch_generate(ref, case):
    """One ``DotsOCRForCausalLM.batch_generate`` call of the reference,
    unmodified, on the stand-in model and tokenizer (tests/golden/standin.py):
    returns its outputs and the per-forward trace.  The module-level switches
    the reference reads at import (HSD_TIGHT_PACK, HSD_COMPACT_PERIOD,
    HSD_MAX_SPEC_LEN, D:52-62) are set on the imported module; the page
    block's pre-tokenizer (D:625-645) is the stand-in tokenizer and the
    cached candidate trees are rebuilt for every call."""
    from tests.golden import standin as SI

    tok = SI.CharTokenizer()
    ref._HSD_TIGHT_PACK = bool(case["tight_pack"])
    ref._HSD_COMPACT_PERIOD = int(case["compact_period"])
    ref._HSD_MAX_SPEC_LEN = int(case["max_spec_len"])
    ref._HSD_MAX_TREE_LEN = 0
    ref._pre_tokenizer = tok
    ref.CACHED_SELECT_MODE_ONE_MATCHES_TREE = None
    ref.CACHED_BBOX_MODE_ONE_MATCHES_TREE = None
    prompts = [tok.encode(t) for t in case["prompts"]]
    texts = [tok.encode(t) for t in case["texts"]]
    graded = case["spec_thresh"] < 1.0 or case["tree_thresh"] < 1.0
    model = SI.StandInLM(prompts, texts, graded=graded)
    ids, mask, pos, pointer = SI.packed_prefill(prompts)
    drafts = [{"block_content": d, "raw_block_content": d} for d in case["drafts"]]
    # the reference reads the thresholds from the environment at call time (D:970-971)
    saved = {k: os.environ.get(k) for k in ("HSD_SPEC_THRESH", "HSD_TREE_THRESH")}
    os.environ["HSD_SPEC_THRESH"] = str(case["spec_thresh"])
    os.environ["HSD_TREE_THRESH"] = str(case["tree_thresh"])
    try:
        gen, decode_times, stats = ref.DotsOCRForCausalLM.batch_generate(
            model, input_ids=ids, attention_mask=mask, position_ids=pos, pointer=pointer,
            tokenizer=tok, draft=drafts, enable_tree_decode=bool(case["tree"]),
            eos_token_id=[SI.EOS], max_new_tokens=int(case["max_new_tokens"]))
    finally:
        for k, v in saved.items():
            if v is None:
                os.environ.pop(k, None)
            else:
                os.environ[k] = v
    return dict(generated=[list(map(int, g)) for g in gen], decode_times=int(decode_times),
                compact_calls=int(stats[6]), compact_skipped=int(stats[7]),
                steps=[SI.step_digest(t) for t in model.trace],
                first_steps=[dict(input_ids=t["input_ids"].tolist(),
                                  position_ids=t["position_ids"].tolist())
                             for t in model.trace[:6]])


def make_batch_generate(ref):
    import contextlib
    import io

    from tests.golden.cases import batch_generate_cases
    out = []
    for case in batch_generate_cases():
        with contextlib.redirect_stdout(io.StringIO()):   # the loop prints its statistics
            got = run_reference_batch_generate(ref, case)
        out.append(dict(case, **got))
    with open(os.path.join(HERE, "batch_generate.json"), "w") as f:
        json.dump(out, f, separators=(",", ":"))
    return len(out)


def main():
    root = sys.argv[1] if len(sys.argv) > 1 else os.environ.get("HSD_REFERENCE_ROOT")
    if not root:
        raise SystemExit("usage: make_golden.py <reference checkout> "
                         "(or set HSD_REFERENCE_ROOT)")
    ref = _import_reference(root)
    only = sys.argv[2:] or ["kmp", "blockmask", "attention", "batch_generate"]
    if "kmp" in only:
        print("kmp cases", make_kmp(ref))
    if "blockmask" in only:
        print("blockmask cases", make_blockmask(ref))
    if "attention" in only:
        print("attention cases", make_attention(ref))
    if "batch_generate" in only:
        print("batch_generate cases", make_batch_generate(ref))


if __name__ == "__main__":
    main()

"""Generate the golden fixtures that pin the oracle to the reference.

Run in a container where the reference checkout is present:

    python tests/golden/make_golden.py [/path/to/reference]

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
                         rejects ``return_lse`` on the CPU.

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


def main():
    root = sys.argv[1] if len(sys.argv) > 1 else "/root/reference"
    ref = _import_reference(root)
    print("kmp cases", make_kmp(ref))
    print("blockmask cases", make_blockmask(ref))
    print("attention cases", make_attention(ref))


if __name__ == "__main__":
    main()

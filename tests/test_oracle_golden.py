"""The oracle against the reference's own outputs (fixtures from make_golden.py)."""
import json
import os

import numpy as np
import pytest
import torch

from oracle import attention as A
from oracle import blockmask as B
from oracle import kmp as K
from tests.golden import cases as C

GOLD = os.path.join(os.path.dirname(__file__), "golden")


def _load(name):
    with open(os.path.join(GOLD, name)) as f:
        return json.load(f)


def test_kmp_matches_reference():
    for case in _load("kmp.json"):
        lps = K.compute_lps(case["pattern"])
        assert lps == case["lps"]
        trie, matches = K.find_all_matches_kmp(case["texts"], case["pattern"],
                                               lps, case["depth"])
        assert [list(m) for m in matches] == case["matches"], case
        assert K.serialize_trie(trie) == case["trie"]


def test_kmp_cases_regenerate():
    gold = _load("kmp.json")
    cases = C.kmp_cases()
    assert len(gold) == len(cases)
    for g, c in zip(gold, cases):
        assert g["texts"] == c["texts"] and g["pattern"] == c["pattern"]


def test_blockmask_matches_reference():
    gold = {g["name"]: g for g in _load("blockmask.json")}
    for name, mask in C.blockmask_cases():
        g = gold[name]
        allowed = B.allowed_from_dense(mask)
        kn, ki, fn, fi = B.block_mask_lists(allowed)
        assert kn == g["kv_num_blocks"], name
        assert fn == g["full_kv_num_blocks"], name
        assert [list(map(int, x)) for x in ki] == g["kv_indices"], name
        assert [list(map(int, x)) for x in fi] == g["full_kv_indices"], name


def test_cfg1_tile_counts():
    allowed = C.cfg1_mask()
    assert B.allowed_pairs(allowed) == 1_059_604
    assert B.executed_tiles(allowed) == 149


@pytest.mark.parametrize("name", ["cfg1", "step_gqa4", "masked_rows_mqa"])
def test_attention_matches_reference(name):
    case = dict(C.attention_cases())[name]
    q, k, v, mask, scale, rows = case
    g = np.load(os.path.join(GOLD, f"attention_{name}.npz"))
    chk = [float(q.double().sum()), float(k.double().sum()), float(v.double().sum())]
    np.testing.assert_allclose(chk, g["input_checksum"], rtol=1e-9, atol=1e-6)
    allowed = B.allowed_from_dense(mask)
    out, lse = A.attention_fp32(q, k, v, allowed, scale)
    gen = torch.Generator().manual_seed(1234)
    proj = torch.randn(out.shape[-1], 2, generator=gen).numpy()
    np.testing.assert_allclose(lse.numpy(), g["lse"], rtol=1e-5, atol=1e-5)
    np.testing.assert_allclose(out.numpy() @ proj, g["out_proj"], rtol=1e-4, atol=1e-5)
    np.testing.assert_allclose(out.numpy()[g["sample_rows"]], g["out_rows"],
                               rtol=1e-4, atol=1e-6)

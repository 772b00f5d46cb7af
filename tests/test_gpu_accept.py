"""GPU parity: acceptance + KMP re-alignment kernel vs the oracle (bit-exact).

Checks per block: result fields (finished, increment, pointer, next token,
match count / first start / next slice), the updated state (generated
tokens, window size, match count, mode), the step's filter bits, and the
block's new visibility row (= the mask row at its pointer, which the next
step inherits, D:1634-1667).
"""
import numpy as np
import pytest
import torch

from oracle import accept as OA
from tests import accept_cases as AC

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def dev():
    assert torch.cuda.is_available(), "GPU tests need a CUDA device"
    return torch.device("cuda:0")


def run_kernel(sc, dev, page_block=None, logits=None, text_mode=(), variant="dots",
               formula_tokens=(3, 1099), spec=None):
    from hsd_b200 import accept as A
    from hsd_b200.plan import pack_bits
    nb = len(sc["blocks"])
    kv_len = sc["kv_len"]
    stride = (kv_len + 63) // 64 + 1
    blocks = np.zeros((nb, 16), dtype=np.int32)
    gen_pool = np.zeros(nb * AC.CAP, dtype=np.int32)
    drafts, tree_tok, tree_par = [], [], []
    seg_bits = np.zeros((nb, stride), dtype=np.uint64)
    doff = toff = 0
    for i, blk in enumerate(sc["blocks"]):
        f = A.F
        blocks[i, f["mode"]] = blk["mode"]
        blocks[i, f["q_start"]] = blk["q_start"]
        blocks[i, f["q_len"]] = blk["q_len"]
        blocks[i, f["valid_count"]] = blk["valid"] or 0
        blocks[i, f["gen_off"]] = i * AC.CAP
        blocks[i, f["gen_len"]] = len(blk["gen"])
        blocks[i, f["gen_cap"]] = AC.CAP
        gen_pool[i * AC.CAP:i * AC.CAP + len(blk["gen"])] = blk["gen"]
        blocks[i, f["draft_off"]] = doff
        blocks[i, f["draft_len"]] = len(blk["draft"])
        drafts += blk["draft"]
        doff += len(blk["draft"])
        blocks[i, f["mws"]] = blk["mws"]
        blocks[i, f["matches_len"]] = blk["matches_len"]
        if blk["tree"]:
            toks, pars = blk["tree"]
            blocks[i, f["tree_off"]] = toff
            blocks[i, f["tree_nodes"]] = len(toks)
            tree_tok += list(toks)
            tree_par += list(pars)
            toff += len(toks)
        blocks[i, f["seg"]] = i
        blocks[i, f["flags"]] = ((A.FLAG_PAGE_BLOCK if i == page_block else 0) |
                                 (A.FLAG_TEXT_MODE if i in text_mode else 0))
        seg_bits[i, :(kv_len + 63) // 64] = pack_bits(blk["kv"])
    t = lambda a, dt=torch.int32: torch.as_tensor(np.asarray(a), dtype=dt).to(dev)
    cfg = A.make_config(nb, kv_len, sc["q_len"], stride, sc["eos"])
    d_blocks = t(blocks)
    d_gen = t(gen_pool)
    out_bits = torch.zeros((nb, stride), dtype=torch.int64, device=dev)
    filt = torch.zeros(stride, dtype=torch.int64, device=dev)
    status = torch.zeros(1, dtype=torch.int32, device=dev)
    res = A.accept_kmp(cfg, d_blocks, t(sc["next_ids"]), t(sc["input_ids"]), d_gen,
                       t(drafts or [0]), t(seg_bits.view(np.int64), torch.int64), out_bits, filt,
                       tree_tokens=t(tree_tok or [0]), tree_parents=t(tree_par or [0]),
                       status=status,
                       logits=None if logits is None else (
                           torch.from_numpy(logits[0]).to(dev), torch.from_numpy(logits[1]).to(dev),
                           logits[2], logits[3]),
                       variant=variant, formula_tokens=formula_tokens,
                       **({} if spec is None else dict(
                           spec, rank=t(spec["rank"]),
                           second=torch.from_numpy(spec["second"]).to(dev))))
    torch.cuda.synchronize()
    assert status.item() == 0, hex(status.item())
    return (res.cpu().numpy(), d_blocks.cpu().numpy(), d_gen.cpu().numpy(),
            out_bits.cpu().numpy(), filt.cpu().numpy())


def unpack(words, n):
    return np.unpackbits(np.ascontiguousarray(words).view(np.uint8), bitorder="little")[:n].astype(bool)


@pytest.mark.parametrize("seed", list(range(24)))
@pytest.mark.parametrize("tight", [False, True])
def test_accept_kmp_matches_oracle(dev, seed, tight):
    from hsd_b200 import accept as A
    sc = AC.make_scenario(seed, tight=tight)
    page = len(sc["blocks"]) - 1 if seed % 3 == 0 else None
    expect, filt = run_oracle_checked(sc, page)
    compare(sc, seed, expect, filt, run_kernel(sc, dev, page_block=page))


@pytest.mark.parametrize("n_blocks,seed", [(17, 6), (33, 0), (40, 1), (64, 2), (97, 3),
                                           (129, 7), (256, 4), (300, 5)])
def test_accept_kmp_many_blocks_matches_oracle(dev, n_blocks, seed):
    """More blocks than one CTA's 32 warps: the launch becomes a cluster of
    up to eight CTAs sharing the filter (and, past 256 blocks, warps take
    several blocks each)."""
    sc = AC.make_scenario(100 + seed, n_blocks=n_blocks, tight=bool(seed & 1))
    page = n_blocks - 1 if seed % 2 == 0 else None
    expect, filt = run_oracle_checked(sc, page)
    compare(sc, seed, expect, filt, run_kernel(sc, dev, page_block=page))


def compare(sc, seed, expect, filt, kernel_out):
    from hsd_b200 import accept as A
    res, blocks, gen, vis, kfilt = kernel_out
    for i, (r, st, row) in enumerate(expect):
        got = {k: int(res[i, A.R[k]]) for k in A.RESULT_FIELDS}
        assert got == r, (seed, i, got, r)
        if r["finished"] == 3:
            continue
        glen = int(blocks[i, A.F["gen_len"]])
        assert gen[i * AC.CAP:i * AC.CAP + glen].tolist() == st.gen, (seed, i)
        assert int(blocks[i, A.F["mws"]]) == st.mws, (seed, i)
        assert int(blocks[i, A.F["matches_len"]]) == st.matches_len, (seed, i)
        assert (int(blocks[i, A.F["mode"]]) == OA.FINISHED) == (st.mode == OA.FINISHED)
        np.testing.assert_array_equal(unpack(vis[i], sc["kv_len"]), row)
    np.testing.assert_array_equal(unpack(kfilt, sc["kv_len"]), filt)


def run_oracle_checked(sc, page):
    out, filt = AC.run_oracle(sc, page_block=page)
    return out, filt


@pytest.mark.parametrize("seed", list(range(16)))
@pytest.mark.parametrize("spec_thresh,tree_thresh", [(0.9, 1.0), (1.0, 0.5), (0.75, 0.9),
                                                     (0.3, 0.3)])
def test_accept_logit_ratio_matches_oracle(dev, seed, spec_thresh, tree_thresh):
    """Thresholds below 1 (D:1147-1174, D:1228-1266): the kernel's
    decisions on the same bf16 logits equal the oracle's, bit for bit
    (generated tokens, pointers, filter and visibility rows)."""
    sc = AC.make_scenario(seed, tight=bool(seed % 2))
    page = len(sc["blocks"]) - 1 if seed % 3 == 0 else None
    max_l, probe = AC.make_logits(sc, seed, min(spec_thresh, tree_thresh))
    rng = np.random.default_rng(seed)
    text_mode = {i for i in range(len(sc["blocks"])) if rng.random() < 0.6}
    expect, filt = AC.run_oracle(sc, page_block=page, logits=(max_l, probe),
                                 spec_thresh=spec_thresh, tree_thresh=tree_thresh,
                                 text_mode=text_mode)
    out = run_kernel(sc, dev, page_block=page, text_mode=text_mode,
                     logits=(max_l, probe, spec_thresh, tree_thresh))
    compare(sc, seed, expect, filt, out)


@pytest.mark.parametrize("seed", list(range(24)))
@pytest.mark.parametrize("spec_thresh", [0.5, 1.0])
def test_accept_hunyuan_rules_match_oracle(dev, seed, spec_thresh):
    """HunYuan's rules (H:1653-1858) bit-exact vs the oracle: the ratio on
    the last block only (made speculative), formula rows exact-only (the
    delimiters made frequent: tokens 3 and 5 on small vocabularies),
    accepted rows keeping the model's tokens, and the tree fallback in
    text-mode blocks at threshold 1."""
    sc = AC.make_scenario(seed, tight=bool(seed % 2), last_mode=OA.SPEC)
    formula = (3, 5) if seed % 4 else (3, 1099)
    max_l, probe = AC.make_logits(sc, seed, 0.5)
    rng = np.random.default_rng(seed)
    text_mode = {i for i in range(len(sc["blocks"])) if rng.random() < 0.6}
    expect, filt = AC.run_oracle(sc, logits=(max_l, probe), spec_thresh=spec_thresh,
                                 tree_thresh=1.0, text_mode=text_mode, variant="hunyuan",
                                 formula_tokens=formula)
    out = run_kernel(sc, dev, text_mode=text_mode, logits=(max_l, probe, spec_thresh, 1.0),
                     variant="hunyuan", formula_tokens=formula)
    compare(sc, seed, expect, filt, out)


@pytest.mark.parametrize("seed", list(range(16)))
@pytest.mark.parametrize("mode,k,margin", [("topk", 3, 2.0), ("topk", 1, 2.0),
                                           ("adaptive", 3, 2.0), ("adaptive", 3, 0.7)])
def test_accept_hunyuan_spec_modes_match_oracle(dev, seed, mode, k, margin):
    """HunYuan SPEC_MODE=topk / adaptive (H:1712-1736) bit-exact vs the
    oracle on the same per-row ranks and second-best logits: the last
    block's missed rows outside formulas pass when the draft token ranks
    below k, or (adaptive) by the ratio or a bf16 top-1 / top-2 margin below
    the bf16 threshold with a positive draft logit (some margins placed
    exactly at it)."""
    sc = AC.make_scenario(seed, tight=bool(seed % 2), last_mode=OA.SPEC)
    formula = (3, 5) if seed % 4 else (3, 1099)
    max_l, probe = AC.make_logits(sc, seed, 0.5)
    rng = np.random.default_rng(seed + 77)
    q = sc["q_len"]
    rank = rng.integers(0, 6, q).astype(np.int32)
    second = OA.bf16_f32((max_l - rng.uniform(0.0, 3.0, q)).astype(np.float32))
    at = rng.random(q) < 0.2
    second[at] = OA.bf16_f32((max_l[at] - OA.bf16_f32(np.float32(margin))).astype(np.float32))
    expect, filt = AC.run_oracle(sc, logits=(max_l, probe, rank, second), spec_thresh=0.5,
                                 tree_thresh=1.0, variant="hunyuan", formula_tokens=formula,
                                 spec_mode=mode, spec_topk=k, spec_margin=margin)
    out = run_kernel(sc, dev, logits=(max_l, probe, 0.5, 1.0), variant="hunyuan",
                     formula_tokens=formula,
                     spec=dict(spec_mode=mode, spec_topk=k, spec_margin=margin, rank=rank,
                               second=second))
    compare(sc, seed, expect, filt, out)

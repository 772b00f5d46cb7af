"""GPU parity: tile plans and verification attention against the oracle.

Tolerance (attention, bf16 inputs/outputs vs the fp32 CPU oracle):
max-abs <= 2e-2 and mean-abs <= 2e-3 on the output; LSE within 2e-2.
Tile classes, index lists and row masks are compared bit-exactly.
"""
import math

import numpy as np
import pytest
import torch

from oracle import attention as OA
from oracle import blockmask as OB
from oracle import masks as OM
from tests.golden import cases as C

pytestmark = pytest.mark.gpu

MAX_ABS, MEAN_ABS, LSE_ABS = 2e-2, 2e-3, 2e-2


@pytest.fixture(scope="module")
def dev():
    assert torch.cuda.is_available(), "GPU tests need a CUDA device"
    from hsd_b200 import _native
    _native.load()
    return torch.device("cuda:0")


def norm_lists(lists):
    kn, ki, fn, fi = lists
    return (list(map(int, kn)), [list(map(int, x)) for x in ki], list(map(int, fn)),
            [list(map(int, x)) for x in fi])


def _bf16(x, dev):
    return x.to(torch.bfloat16).to(dev)


def run_attention(q, k, v, mask_obj, scale, dev, balanced=True):
    from hsd_b200.attention import plan_for, verify_attention
    qd, kd, vd = _bf16(q, dev), _bf16(k, dev), _bf16(v, dev)
    plan = plan_for(mask_obj, q.shape[1], k.shape[1])
    out, lse = verify_attention(qd, kd, vd, plan, scale=scale, balanced=balanced)
    torch.cuda.synchronize()
    plan.raise_on_device_error()
    return out.float().cpu(), lse.cpu(), plan


def check_close(out, lse, q, k, v, allowed, scale):
    # the oracle sees the same bf16-rounded inputs
    ref_out, ref_lse = OA.attention_fp32(q.to(torch.bfloat16).float(),
                                         k.to(torch.bfloat16).float(),
                                         v.to(torch.bfloat16).float(), allowed, scale)
    err = (out - ref_out).abs()
    assert err.max().item() <= MAX_ABS, err.max().item()
    assert err.mean().item() <= MEAN_ABS, err.mean().item()
    fin = torch.isfinite(ref_lse)
    assert torch.equal(fin, torch.isfinite(lse))
    assert (lse[fin] - ref_lse[fin]).abs().max().item() <= LSE_ABS
    assert torch.all(lse[~fin] == -math.inf)
    dead = ~torch.as_tensor(allowed).any(1)
    if dead.any():
        assert out[dead].abs().max().item() == 0.0


@pytest.mark.parametrize("name", [n for n, _ in C.blockmask_cases()])
def test_dense_plan_matches_create_block_mask(dev, name):
    from hsd_b200.plan import plan_from_dense
    mask = dict(C.blockmask_cases())[name]
    allowed = OB.allowed_from_dense(mask)
    plan = plan_from_dense(mask.to(dev))
    torch.cuda.synchronize()
    assert plan.block_mask_lists() == norm_lists(OB.block_mask_lists(allowed))
    np.testing.assert_array_equal(plan.tile_class().cpu().numpy(), OB.tile_classes(allowed))
    np.testing.assert_array_equal(plan.dense_allowed(), allowed)


def cfg1_segments():
    n = 1512
    segs = [dict(q_start=0, q_len=1024, kind=OM.CAUSAL, kv=np.zeros(n, bool))]
    s = 1024
    prefix = np.zeros(n, bool)
    prefix[:1024] = True
    for L in [64, 96, 128, 200]:
        segs.append(dict(q_start=s, q_len=L, kind=OM.CAUSAL, kv=prefix.copy()))
        s += L
    return segs


def test_segment_plan_matches_dense(dev):
    from hsd_b200.plan import PackedMask
    segs = cfg1_segments()
    allowed = OM.segments_to_allowed(1512, 1512, segs)
    np.testing.assert_array_equal(allowed, C.cfg1_mask())
    pm = PackedMask(1512, 1512, segs, device=dev)
    plan = pm.plan()
    torch.cuda.synchronize()
    plan.raise_on_device_error()
    np.testing.assert_array_equal(plan.dense_allowed(), allowed)
    assert plan.block_mask_lists() == norm_lists(OB.block_mask_lists(allowed))
    assert int((plan.tile_class() != 0).sum()) == 149


def test_segment_plan_tree_single_none(dev):
    """Tree ancestor sets, single-token blocks and uncovered rows."""
    from hsd_b200.plan import PackedMask
    rng = np.random.default_rng(5)
    kv_old = 333
    parents = [-1, 0, 0, 1, 1, 2, 3, 3, 5, 8, 8, 0]
    segs_q = [(0, 128, OM.CAUSAL), (128, 128, OM.TREE), (256, 128, OM.SINGLE),
              (384, 37, OM.CAUSAL), (421, 20, OM.NONE)]
    q_len = 441 + 30  # 30 uncovered tail rows
    kv_len = kv_old + q_len
    segs = []
    for qs, ql, kind in segs_q:
        kv = np.zeros(kv_len, bool)
        lo = int(rng.integers(0, kv_old - 50))
        kv[lo:lo + int(rng.integers(1, 50))] = True
        kv[rng.integers(0, kv_old, 10)] = True
        d = dict(q_start=qs, q_len=ql, kind=kind, kv=kv)
        if kind == OM.TREE:
            d["parents"] = parents
        segs.append(d)
    # a later segment also sees an earlier segment's new columns (prefix tree)
    segs[3]["kv"][kv_old:kv_old + 128] = True
    allowed = OM.segments_to_allowed(q_len, kv_len, segs)
    pm = PackedMask(q_len, kv_len, segs, device=dev)
    plan = pm.plan()
    torch.cuda.synchronize()
    np.testing.assert_array_equal(plan.dense_allowed(), allowed)
    np.testing.assert_array_equal(plan.tile_class().cpu().numpy(), OB.tile_classes(allowed))
    q, k, v = C.qkv(4, 2, q_len, kv_len, seed=11)
    out, lse, _ = run_attention(q, k, v, pm, None, dev)
    check_close(out, lse, q, k, v, allowed, None)


@pytest.mark.parametrize("q_len,kv_old,seed", [(6000, 3000, 21), (4100, 9000, 22)])
def test_segment_plan_many_tiles(dev, q_len, kv_old, seed):
    """More query tiles than the ordering kernel has warps (each warp builds
    several tiles' lists) and the classification spread over several parts
    per tile: lists, classes, 128-column block list, tile order and prefix."""
    from hsd_b200.plan import PackedMask
    rng = np.random.default_rng(seed)
    kv_len = kv_old + q_len
    segs, qs = [], 0
    while qs < q_len - 40:
        ql = int(min(q_len - 40 - qs, rng.integers(1, 400)))
        kind = [OM.CAUSAL, OM.SINGLE, OM.NONE][int(rng.integers(0, 3))] if ql > 1 else OM.SINGLE
        kv = np.zeros(kv_len, bool)
        kv[:int(rng.integers(0, kv_old))] = True
        kv[rng.integers(0, kv_old + qs + 1, 20)] = True
        segs.append(dict(q_start=qs, q_len=ql, kind=kind, kv=kv))
        qs += ql
    allowed = OM.segments_to_allowed(q_len, kv_len, segs)
    pm = PackedMask(q_len, kv_len, segs, device=dev)
    plan = pm.plan()
    torch.cuda.synchronize()
    plan.raise_on_device_error()
    np.testing.assert_array_equal(plan.dense_allowed(), allowed)
    cls = OB.tile_classes(allowed)
    np.testing.assert_array_equal(plan.tile_class().cpu().numpy(), cls)
    assert plan.block_mask_lists() == norm_lists(OB.block_mask_lists(allowed))
    # 128-column blocks: present when either 64-column half is, flags per half
    cnt, lst = (t.cpu().numpy() for t in plan.blocks())
    nq, n64 = cls.shape
    for t in range(nq):
        want = []
        for b in range((n64 + 1) // 2):
            c0 = int(cls[t, 2 * b])
            c1 = int(cls[t, 2 * b + 1]) if 2 * b + 1 < n64 else 0
            if c0 or c1:
                want.append(b | (int(c0 != 0) << 24) | (int(c0 == 1) << 25)
                            | (int(c1 != 0) << 26) | (int(c1 == 1) << 27))
        assert int(cnt[t]) == len(want), t
        assert lst[t, :len(want)].astype(np.uint32).tolist() == want, t
    # order: block count descending, ties by tile; prefix over that order
    order = plan._view("tile_order", torch.int32, (nq,)).cpu().numpy()
    prefix = plan._view("blk_prefix", torch.int32, (nq + 1,)).cpu().numpy()
    want_order = sorted(range(nq), key=lambda t: (-int(cnt[t]), t))
    assert order.tolist() == want_order
    assert prefix.tolist() == np.concatenate([[0], np.cumsum(cnt[want_order])]).tolist()


@pytest.mark.parametrize("name", ["cfg1", "step_gqa4", "masked_rows_mqa"])
def test_attention_golden_cases(dev, name):
    q, k, v, mask, scale, _ = dict(C.attention_cases())[name]
    allowed = OB.allowed_from_dense(mask)
    out, lse, _ = run_attention(q, k, v, mask.to(dev), scale, dev)
    check_close(out, lse, q, k, v, allowed, scale)


@pytest.mark.parametrize("hq,hkv", [(12, 2), (16, 8), (3, 1), (2, 2), (5, 5)])
def test_attention_head_groupings(dev, hq, hkv):
    allowed = C.cfg1_mask()[:700, :700]
    q, k, v = C.qkv(hq, hkv, 700, 700, seed=hq * 31 + hkv)
    mask = C._dense(allowed).to(dev)
    out, lse, _ = run_attention(q, k, v, mask, None, dev)
    check_close(out, lse, q, k, v, allowed, None)


def test_attention_strided_query_layout(dev):
    """HF passes q as a transposed view [1, H, Q, D] of [1, Q, H, D]."""
    from hsd_b200.attention import flex_attention_forward
    allowed = C.cfg1_mask()[:520, :520]
    q, k, v = C.qkv(12, 2, 520, 520, seed=3)
    q_sh = q.transpose(0, 1).contiguous().to(torch.bfloat16).to(dev)  # [Q, H, D]
    q_view = q_sh.transpose(0, 1).unsqueeze(0)                         # [1, H, Q, D] strided
    out, lse = flex_attention_forward(None, q_view, _bf16(k, dev)[None], _bf16(v, dev)[None],
                                      C._dense(allowed).to(dev))
    torch.cuda.synchronize()
    assert out.shape == (1, 520, 12, 128) and lse.shape == (1, 12, 520)
    assert lse.dtype == torch.bfloat16
    ref_out, _ = OA.attention_fp32(q.to(torch.bfloat16).float(), k.to(torch.bfloat16).float(),
                                   v.to(torch.bfloat16).float(), allowed)
    err = (out[0].float().cpu() - ref_out).abs()
    assert err.max().item() <= MAX_ABS and err.mean().item() <= MEAN_ABS


def test_drop_in_fp32_model_cfg1(dev):
    """The reference's first config runs FlexAttention in fp32: the drop-in
    takes fp32 q/k/v (computed in bf16) and returns fp32, within the bf16
    tolerance of the fp32 reference."""
    from hsd_b200.attention import flex_attention_forward
    q, k, v, mask, scale, _ = dict(C.attention_cases())["cfg1"]
    allowed = OB.allowed_from_dense(mask)
    out, lse = flex_attention_forward(None, q[None].to(dev), k[None].to(dev), v[None].to(dev),
                                      mask.to(dev), scaling=scale)
    torch.cuda.synchronize()
    assert out.dtype == torch.float32 and lse.dtype == torch.float32
    ref_out, ref_lse = OA.attention_fp32(q, k, v, allowed, scale)
    err = (out[0].cpu() - ref_out).abs()
    assert err.max().item() <= MAX_ABS and err.mean().item() <= MEAN_ABS
    assert (lse[0].cpu() - ref_lse).abs().max().item() <= LSE_ABS


def test_attention_long_prefix_many_blocks(dev):
    """Stage-2 shape slice: one causal segment over a long cached prefix."""
    kv_old, ql = 2000, 300
    kv = kv_old + ql
    segs = [dict(q_start=0, q_len=ql, kind=OM.CAUSAL,
                 kv=np.concatenate([np.ones(kv_old, bool), np.zeros(ql, bool)]))]
    from hsd_b200.plan import PackedMask
    allowed = OM.segments_to_allowed(ql, kv, segs)
    q, k, v = C.qkv(12, 2, ql, kv, seed=9)
    out, lse, _ = run_attention(q, k, v, PackedMask(ql, kv, segs, device=dev), None, dev)
    check_close(out, lse, q, k, v, allowed, None)


def test_attention_large_scores_rescale(dev):
    """Growing maxima across blocks exercise the lazy O rescale."""
    allowed = np.ones((256, 1024), bool)
    torch.manual_seed(4)
    q = torch.randn(2, 256, 128)
    k = torch.randn(1, 1024, 128) * torch.linspace(0.1, 3.0, 1024)[None, :, None]
    v = torch.randn(1, 1024, 128)
    out, lse, _ = run_attention(q, k, v, C._dense(allowed).to(dev), 0.3, dev)
    check_close(out, lse, q, k, v, allowed, 0.3)


@pytest.mark.parametrize("balanced", [True, False])
@pytest.mark.parametrize("name", ["cfg1", "step_gqa4", "masked_rows_mqa"])
def test_attention_both_schedules(dev, name, balanced):
    """Stream-K (split items combined through the workspace) and one-CTA-per-item."""
    q, k, v, mask, scale, _ = dict(C.attention_cases())[name]
    allowed = OB.allowed_from_dense(mask)
    out, lse, _ = run_attention(q, k, v, mask.to(dev), scale, dev, balanced=balanced)
    check_close(out, lse, q, k, v, allowed, scale)


@pytest.mark.parametrize("qn,kvn", [(128, 256), (64, 70), (300, 5000)])
def test_attention_small_and_skewed(dev, qn, kvn):
    """Less work than SMs; one query tile much heavier than the others."""
    rng = np.random.default_rng(qn + kvn)
    allowed = rng.random((qn, kvn)) < 0.3
    allowed[: qn // 3] = False          # a fully masked band of rows
    if qn >= 256:
        allowed[:128] = False           # a whole query tile with nothing visible
        allowed[200:, :] = True         # and a dense one
    q, k, v = C.qkv(6, 2, qn, kvn, seed=qn)
    for balanced in (True, False):
        out, lse, _ = run_attention(q, k, v, C._dense(allowed).to(dev), None, dev, balanced)
        check_close(out, lse, q, k, v, allowed, None)


def test_attention_repeated_launches_reuse_workspace(dev):
    """Counters are left at zero: many launches in a row stay correct."""
    from hsd_b200.attention import plan_for, verify_attention
    allowed = C.cfg1_mask()
    q, k, v = C.qkv(12, 2, 1512, 1512, seed=21)
    qd, kd, vd = _bf16(q, dev), _bf16(k, dev), _bf16(v, dev)
    plan = plan_for(C._dense(allowed).to(dev), 1512, 1512)
    outs = [verify_attention(qd, kd, vd, plan)[0] for _ in range(6)]
    torch.cuda.synchronize()
    ref, _ = verify_attention(qd, kd, vd, plan, balanced=False)
    for o in outs[1:]:
        assert torch.equal(o, outs[0])
    err = (outs[0].float() - ref.float()).abs()
    assert err.max().item() <= 1e-2

"""GPU parity of the fused lm_head + argmax against the oracle.

The oracle sums the logits exactly and rounds them once to bf16; the kernel
sums in fp32 (as the reference's bf16 GEMM does, in its own order) before the
same rounding.  Ids must be equal except on rows whose exact top logits lie
within one bf16 step of each other (``oracle.lm_head.near_tie``), and such
rows must stay rare (at most 1 %).  Ties between equal logits (duplicate
weight rows) must go to the lowest id, across tiles and within one.
"""
import numpy as np
import pytest
import torch

from oracle import lm_head as OL

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def dev():
    assert torch.cuda.is_available(), "GPU tests need a CUDA device"
    from hsd_b200 import _native
    _native.load()
    return torch.device("cuda:0")


def _case(q, vocab, hd, seed):
    g = torch.Generator().manual_seed(seed)
    h = torch.randn(q, hd, generator=g).to(torch.bfloat16)
    w = (torch.randn(vocab, hd, generator=g) / hd ** 0.5).to(torch.bfloat16)
    return h, w


def _run(h, w, dev):
    from hsd_b200.lm_head import lm_head_argmax
    q = h.shape[0]
    ids32 = torch.empty(q, dtype=torch.int32, device=dev)
    mx = torch.empty(q, dtype=torch.float32, device=dev)
    status = torch.zeros(1, dtype=torch.int32, device=dev)
    ids = lm_head_argmax(h.to(dev), w.to(dev), out_int32=ids32, max_logit=mx, status=status)
    torch.cuda.synchronize()
    assert int(status.item()) == 0
    assert torch.equal(ids.int(), ids32)
    return ids.cpu().numpy(), mx.cpu().numpy()


def _check(got, got_max, h, w):
    want, want_max, exact = OL.lm_head_argmax(h, w)
    diff = np.nonzero(got != want)[0]
    assert len(diff) <= max(1, len(want) // 100), (len(diff), len(want))
    for r in diff:
        assert OL.near_tie(exact[r], got[r], want[r]), (r, got[r], want[r])
    same = got == want
    assert np.array_equal(got_max[same], want_max[same].astype(np.float32))


@pytest.mark.parametrize("q,vocab,hd,seed", [
    (300, 5003, 1536, 0),     # partial row tile and partial vocabulary tile
    (1, 777, 512, 1),
    (129, 4096, 200, 2),      # hidden size not a multiple of 64 (zero-filled tail)
    (640, 2560, 1536, 3),
])
def test_random_cases_match_oracle(dev, q, vocab, hd, seed):
    h, w = _case(q, vocab, hd, seed)
    ids, mx = _run(h, w, dev)
    _check(ids, mx, h, w)


def test_equal_logits_go_to_lowest_id(dev):
    h, w = _case(8, 5000, 1536, 4)
    pairs = [(100, 4000), (513, 700), (40, 41), (4990, 4999)]
    for r, (a, b) in enumerate(pairs):
        w[b] = w[a]
        h[r] = w[a].float() * 8
    ids, mx = _run(h, w, dev)
    assert ids[:len(pairs)].tolist() == [a for a, _ in pairs]
    _check(ids, mx, h, w)


def test_all_negative_logits_ignore_padding_columns(dev):
    g = torch.Generator().manual_seed(5)
    w = torch.randn(5003, 256, generator=g).abs().to(torch.bfloat16)
    h = (-torch.randn(200, 256, generator=g).abs()).to(torch.bfloat16)
    ids, mx = _run(h, w, dev)
    assert np.all(ids < 5003) and np.all(mx < 0)
    _check(ids, mx, h, w)


def test_repeat_calls_and_graph_capture(dev):
    from hsd_b200.lm_head import lm_head_argmax
    h, w = _case(256, 3000, 1536, 6)
    hd, wd = h.to(dev), w.to(dev)
    first = lm_head_argmax(hd, wd)
    second = lm_head_argmax(hd, wd)
    out = torch.empty(256, dtype=torch.int64, device=dev)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        lm_head_argmax(hd, wd, out=out)
    g.replay()
    torch.cuda.synchronize()
    assert torch.equal(first, second) and torch.equal(first, out)


def test_full_vocabulary_against_fp32_logits(dev):
    """Stage-1 page rows against the 151,936-token vocabulary: the fp32
    logits of torch (no TF32) rounded to bf16 stand in for the exact ones."""
    q, vocab, hd = 2176, 151936, 1536
    g = torch.Generator(device=dev).manual_seed(7)
    h = torch.randn(q, hd, generator=g, device=dev).to(torch.bfloat16)
    w = (torch.randn(vocab, hd, generator=g, device=dev) / hd ** 0.5).to(torch.bfloat16)
    from hsd_b200.lm_head import lm_head_argmax
    mx = torch.empty(q, dtype=torch.float32, device=dev)
    ids = lm_head_argmax(h, w, max_logit=mx)
    assert torch.backends.cuda.matmul.allow_tf32 is False
    ref = torch.empty(q, dtype=torch.int64, device=dev)
    near = torch.zeros(q, dtype=torch.bool, device=dev)
    for r0 in range(0, q, 512):
        lg = h[r0:r0 + 512].float() @ w.float().T
        lb = lg.to(torch.bfloat16)
        ref[r0:r0 + 512] = lb.argmax(-1)
        best = lg.gather(1, ref[r0:r0 + 512, None])[:, 0]
        step = torch.exp2(torch.floor(torch.log2(best.abs())) - 7)
        got = lg.gather(1, ids[r0:r0 + 512, None])[:, 0]
        near[r0:r0 + 512] = got >= best - step
    diff = ids != ref
    assert int(diff.sum()) <= q // 100
    assert bool(near[diff].all())
    same = ~diff
    ref_max = torch.empty(q, dtype=torch.float32, device=dev)
    for r0 in range(0, q, 512):
        lb = (h[r0:r0 + 512].float() @ w.float().T).to(torch.bfloat16)
        ref_max[r0:r0 + 512] = lb.max(-1).values.float()
    assert torch.equal(mx[same], ref_max[same])


def _one_step_off(exact, got, abs_sum, hd):
    """``got`` (bf16 value) is the exact logit rounded to bf16, or within
    one bf16 step of it plus the error bound of an fp32 sum of ``hd``
    products (``hd * 2^-24 * sum |a_i b_i|``, which dominates when the
    products cancel)."""
    want = OL.round_bf16(exact)
    _, e = np.frexp(np.maximum(np.abs(exact), 1e-30))
    step = np.ldexp(1.0, e - 8)
    return (got == want) | (np.abs(got - exact) <= step + hd * 2.0 ** -24 * abs_sum)


@pytest.mark.parametrize("q,vocab,hd,n,seed", [(300, 5003, 1536, 4000, 0), (7, 64, 8, 50, 1),
                                               (129, 4096, 200, 0, 2), (64, 151936, 1536, 512, 3)])
def test_probe_logits_match_exact_and_cublas(dev, q, vocab, hd, n, seed):
    """``probe_logits`` returns the bf16 logit the logits tensor holds:
    equal to the exact dot product rounded to bf16 (one bf16 step off at
    most, near rounding boundaries), and to torch's bf16 GEMM logits with
    fp32 reduction the same way; toks < 0 give 0.  (torch's default bf16
    GEMM may reduce partial sums in bf16 --
    ``allow_bf16_reduced_precision_reduction`` -- and then differs from the
    exactly rounded logit in a sizeable share of entries.)"""
    from hsd_b200.lm_head import probe_logits
    if hd % 8:
        hd += 8 - hd % 8
    h, w = _case(q, vocab, hd, seed)
    rng = np.random.default_rng(seed)
    rows = rng.integers(0, q, n).astype(np.int32)
    toks = rng.integers(0, vocab, n).astype(np.int32)
    toks[rng.random(n) < 0.1] = -1
    status = torch.zeros(1, dtype=torch.int32, device=dev)
    got = probe_logits(h.to(dev), w.to(dev), torch.from_numpy(rows).to(dev),
                       torch.from_numpy(toks).to(dev), status=status)
    torch.cuda.synchronize()
    assert int(status.item()) == 0
    got = got.cpu().numpy().astype(np.float64)
    if n == 0:
        assert got.size == 0
        return
    on = toks >= 0
    assert np.all(got[~on] == 0)
    hd64 = h.double().numpy()
    wd64 = w.double().numpy()
    exact = np.einsum("kh,kh->k", hd64[rows[on]], wd64[toks[on]])
    abs_sum = np.einsum("kh,kh->k", np.abs(hd64[rows[on]]), np.abs(wd64[toks[on]]))
    ok = _one_step_off(exact, got[on], abs_sum, hd)
    bad = np.nonzero(~ok)[0][:3]
    assert ok.all(), [(exact[i], got[on][i], abs_sum[i]) for i in bad]
    assert np.mean(got[on] == OL.round_bf16(exact)) > 0.97
    # torch's logits tensor, a bf16 GEMM with fp32 reduction
    flag = torch.backends.cuda.matmul.allow_bf16_reduced_precision_reduction
    torch.backends.cuda.matmul.allow_bf16_reduced_precision_reduction = False
    try:
        ref = (h.to(dev) @ w.to(dev).T)[torch.from_numpy(rows[on]).long().to(dev),
                                        torch.from_numpy(toks[on]).long().to(dev)]
        ref = ref.float().cpu().numpy().astype(np.float64)
    finally:
        torch.backends.cuda.matmul.allow_bf16_reduced_precision_reduction = flag
    assert np.mean(got[on] == ref) > 0.97
    assert _one_step_off(exact, ref, abs_sum, hd).all()


def test_probe_logits_bad_index_sets_status(dev):
    from hsd_b200.lm_head import probe_logits
    h, w = _case(8, 100, 64, 4)
    rows = torch.tensor([0, 8, 3], dtype=torch.int32, device=dev)
    toks = torch.tensor([5, 5, 100], dtype=torch.int32, device=dev)
    status = torch.zeros(1, dtype=torch.int32, device=dev)
    out = probe_logits(h.to(dev), w.to(dev), rows, toks, status=status)
    torch.cuda.synchronize()
    assert int(status.item()) & 0x20000
    o = out.cpu().numpy()
    assert np.isfinite(o[0]) and np.isnan(o[1]) and np.isnan(o[2])


@pytest.mark.parametrize("q,vocab,hd,seed", [(200, 3000, 512, 0), (64, 1000, 256, 1),
                                             (300, 151936 // 16, 1536, 2)])
def test_lm_head_rank_matches_torch(dev, q, vocab, hd, seed):
    """The rank pass against torch's bf16 logits: multiples of 1/4 in hidden
    and weight make every fp32 sum exact, so both sides round the same
    values to bf16 (with many equal logits).  rank = the draft token's
    position in the descending order with lower columns first among equal
    logits; second = the best logit outside the argmax column; rank < k
    agrees with topk(k) wherever the k-th and (k+1)-th logits differ."""
    from hsd_b200.lm_head import lm_head_argmax, lm_head_rank
    from oracle import accept as OA
    g = torch.Generator().manual_seed(seed)
    h = (torch.randint(-4, 5, (q, hd), generator=g).float() / 4).to(torch.bfloat16)
    w = (torch.randint(-4, 5, (vocab, hd), generator=g).float() / 4).to(torch.bfloat16)
    logits = (h.float() @ w.float().T).to(torch.bfloat16)        # exact sums, one rounding
    dense = logits.float().numpy()
    ids = lm_head_argmax(h.to(dev), w.to(dev)).cpu()
    np.testing.assert_array_equal(ids.numpy(), dense.argmax(1))
    rng = np.random.default_rng(seed)
    ref = np.where(rng.random(q) < 0.5, np.argsort(-dense, 1, kind="stable")[
        np.arange(q), rng.integers(0, 8, q)], rng.integers(0, vocab, q)).astype(np.int32)
    probe = dense[np.arange(q), ref].astype(np.float32)
    rank, second = lm_head_rank(h.to(dev), w.to(dev), torch.from_numpy(probe).to(dev),
                                torch.from_numpy(ref).to(dev),
                                ids.to(torch.int32).to(dev))
    want = [OA.rank_and_second(dense[r], int(ref[r]), int(ids[r])) for r in range(q)]
    np.testing.assert_array_equal(rank.cpu().numpy(), [x[0] for x in want])
    np.testing.assert_array_equal(second.cpu().numpy(), np.float32([x[1] for x in want]))
    for k in (1, 3, 5):
        top = logits.topk(k + 1, dim=-1).values.float().numpy()
        clear = top[:, k - 1] != top[:, k]          # no tie at the boundary
        in_topk = (logits.topk(k, dim=-1).indices.numpy() == ref[:, None]).any(1)
        np.testing.assert_array_equal((rank.cpu().numpy() < k)[clear], in_topk[clear])
    # a second call reuses the cleared workspace
    rank2, second2 = lm_head_rank(h.to(dev), w.to(dev), torch.from_numpy(probe).to(dev),
                                  torch.from_numpy(ref).to(dev), ids.to(torch.int32).to(dev))
    assert torch.equal(rank2, rank) and torch.equal(second2, second)


@pytest.mark.parametrize("q,vocab,hd,seed", [(256, 151936 // 8, 1536, 3), (96, 5000, 1024, 4)])
def test_lm_head_rank_with_probe_kernel_logits(dev, q, vocab, hd, seed):
    """The rank pass fed by hsd_probe_logits on random bf16 inputs, where the
    probe's summation order differs from the GEMM's and the two bf16 logits
    of the draft token may differ by one unit: the token must not count
    itself, so rank < k agrees with torch.topk(k) of the fp32-accumulated
    logits on every row whose k-th and (k+1)-th logits are more than two
    bf16 units apart and whose draft logit is not within two units of them."""
    from hsd_b200.lm_head import lm_head_argmax, lm_head_rank, probe_logits
    g = torch.Generator().manual_seed(seed)
    h = torch.randn(q, hd, generator=g).to(torch.bfloat16)
    w = (torch.randn(vocab, hd, generator=g) / hd ** 0.5).to(torch.bfloat16)
    logits = (h.float() @ w.float().T).to(torch.bfloat16).float()
    ids = lm_head_argmax(h.to(dev), w.to(dev)).to(torch.int32)
    rng = np.random.default_rng(seed)
    order = torch.argsort(logits, dim=1, descending=True, stable=True).numpy()
    ref = np.where(rng.random(q) < 0.7, order[np.arange(q), rng.integers(0, 6, q)],
                   rng.integers(0, vocab, q)).astype(np.int32)
    rows = torch.arange(q, dtype=torch.int32, device=dev)
    d_ref = torch.from_numpy(ref).to(dev)
    probe = probe_logits(h.to(dev), w.to(dev), rows, d_ref)
    rank, _ = lm_head_rank(h.to(dev), w.to(dev), probe, d_ref, ids)
    rank = rank.cpu().numpy()
    dense = logits.numpy()
    thr = dense[np.arange(q), ref]
    ulp = 2.0 * np.float32(2.0 ** -7) * np.maximum(np.abs(dense).max(1), 1e-3)
    checked = 0
    for k in (1, 3, 5):
        top = logits.topk(k + 1, dim=-1).values.numpy()
        clear = ((top[:, k - 1] - top[:, k]) > ulp) & (np.abs(thr - top[:, k - 1]) > ulp) \
            & (np.abs(thr - top[:, k]) > ulp)
        in_topk = (logits.topk(k, dim=-1).indices.numpy() == ref[:, None]).any(1)
        np.testing.assert_array_equal((rank < k)[clear], in_topk[clear])
        checked += int(clear.sum())
    assert checked > q  # most rows are decided away from a tie


def test_lm_head_rank_nan_probe_ranks_last(dev):
    """A NaN probe (hsd_probe_logits of a bad index) gives rank vocab - 1,
    never a rank that would accept the token."""
    from hsd_b200.lm_head import lm_head_argmax, lm_head_rank
    h, w = _case(16, 1000, 64, 5)
    ids = lm_head_argmax(h.to(dev), w.to(dev)).to(torch.int32)
    probe = torch.full((16,), float("nan"), device=dev)
    ref = torch.arange(16, dtype=torch.int32, device=dev)
    rank, _ = lm_head_rank(h.to(dev), w.to(dev), probe, ref, ids)
    assert (rank.cpu().numpy() == 999).all()

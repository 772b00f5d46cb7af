"""GPU parity of a whole verification step (``VerifyStep``) against the oracle.

One step of a packed page -- a small region page, and the three benchmarked
pages at their full sizes -- runs through the device path (KV
append, tile plan, attention on every layer, acceptance + KMP, keep indices,
in-place compaction, visibility remap) and is checked against the oracle's
restatement of the same iteration: per-block pointer / increment / finished
and the kept columns bit-exactly, the compacted caches bit-exactly against
``index_select`` of the appended caches, attention within the tolerance of
the attention tests.  The end-to-end form (pinned host buffers, Q copied
layer by layer on a copy stream) and its CUDA-graph capture must give the
same results as the device-resident form.
"""
import numpy as np
import pytest
import torch

from oracle import accept as OA
from oracle import attention as OAtt
from oracle import compact as OC
from oracle import masks as OM

pytestmark = pytest.mark.gpu

MAX_ABS, MEAN_ABS = 2e-2, 2e-3


@pytest.fixture(scope="module")
def page():
    assert torch.cuda.is_available(), "GPU tests need a CUDA device"
    from hsd_b200 import _native
    from hsd_b200 import workloads as W
    _native.load()
    return W.stage1_regions(seed=5, prefix=640, groups=3, drafts_per_group=2)


def _step(page, seed=0):
    from hsd_b200.verify_step import VerifyStep
    return VerifyStep(page, device="cuda:0", seed=seed)


def _oracle(page):
    from hsd_b200.workloads import segment_dicts
    allowed = OM.segments_to_allowed(page.q_len, page.kv_len, segment_dicts(page))
    cfg = OA.StepConfig(pad_token_id=-1, eos_token_ids=(2**31 - 1,), tight_pack=True)
    filt = np.zeros(page.kv_len, bool)
    base = page.kv_len - page.q_len
    nxt, ids = page.next_ids.tolist(), page.input_ids.tolist()
    rows = []
    for sg in page.segments:
        st = OA.BlockState(mode=OA.SPEC, gen=list(sg.gen), draft=list(sg.draft), mws=3,
                           matches_len=1, valid_count=sg.q_len)
        ptr, _, inc, fin = OA.accept_block(st, sg.q_start, sg.q_start + sg.q_len, nxt, ids,
                                           cfg, filt, base, lambda r: allowed[r], False)
        rows.append((ptr, inc, int(bool(fin))))
    active = [p for p, _, f in rows if not f]
    keep = OC.keep_columns(allowed, active, filt)
    return allowed, rows, OC.keep_indices(keep)


def test_step_matches_oracle(page):
    _check_step_against_oracle(page)


@pytest.mark.parametrize("name", ["stage1_regions", "stage2_page", "hunyuan_regions"])
def test_full_size_step_matches_oracle(name):
    """The benchmarked pages at their full sizes: stage-1 regions (Q 2176 over
    KV 4800, 761 tiles per head, 28 layers), the stage-2 page (one
    3072-token causal draft over a 4096-token prefix, KV 7168, 2136 tiles)
    and the HunYuan-scale regions (24 layers, 16 / 8 heads, tight-packed
    4096-row chunk): the stream-K split, the owner merge and the block walk
    at the lengths and tile counts the bench times.  Attention on the first
    and last layer (output and LSE) within the attention tolerance, the
    per-block results, kept columns and compacted caches bit-exact."""
    from hsd_b200 import workloads as W
    _check_step_against_oracle(W.WORKLOADS[name](seed=0))


def _check_step_against_oracle(page):
    from hsd_b200.accept import R
    s = _step(page)
    appended = s.cache.clone()
    appended[:, :, :, s.prefix:s.prefix + s.q_len] = s.new_kv
    q = s.q.clone()
    s.run()
    torch.cuda.synchronize()
    allowed, rows, idx = _oracle(page)

    res = s.results.cpu().numpy()
    got = [(int(r[R["pointer"]]), int(r[R["increment"]]), int(r[R["finished"]])) for r in res]
    assert got == rows

    n_keep, first = (int(x) for x in s.counts.cpu().tolist())
    assert n_keep == len(idx)
    moved = np.nonzero(idx != np.arange(len(idx)))[0]
    assert first == (int(moved[0]) if len(moved) else n_keep)
    it = torch.as_tensor(idx, device=appended.device)
    assert torch.equal(s.cache[:, :, :, :n_keep], appended.index_select(3, it))

    mask = torch.as_tensor(allowed)
    for l in (0, page.layers - 1):
        ref, ref_lse = OAtt.attention_fp32(q[l].cpu(), appended[l, 0].cpu(),
                                           appended[l, 1].cpu(), mask)
        err = (s.out[l].float().cpu() - ref).abs()
        assert err.max().item() <= MAX_ABS and err.mean().item() <= MEAN_ABS, (
            l, err.max().item(), err.mean().item())
        rows = mask.any(1)
        lerr = (s.lse[l].cpu()[:, rows] - ref_lse[:, rows]).abs()
        assert lerr.max().item() <= 2e-2, (l, lerr.max().item())
        assert torch.isneginf(s.lse[l].cpu()[:, ~rows]).all()
    assert int(s.status.item()) == 0


def _state(s):
    torch.cuda.synchronize()
    return [t.clone() for t in (s.results, s.counts, s.cache, s.out, s.lse, s.vis_next)]


def test_from_host_and_graph_match_device_form(page):
    """The end-to-end form (rows copied layer by layer into alternating
    device input sets, appended per layer) and its two- and four-step CUDA
    graphs give the device-resident form's state after the same number of
    steps."""
    a = _step(page)
    a.run()
    a.run()
    want = _state(a)
    a.run()
    a.run()
    want4 = _state(a)
    a.run()
    a.run()
    want6 = _state(a)

    b = _step(page)
    b.run_from_host(buffers=0)
    b.run_from_host(buffers=1)
    h = b.host_buffers()
    torch.cuda.synchronize()
    assert torch.equal(h["results"], b.results.cpu())
    assert torch.equal(h["counts"], b.counts.cpu())
    for x, y in zip(want, _state(b)):
        assert torch.equal(x, y)

    c = _step(page)
    c.run_from_host(buffers=0)
    c.run_from_host(buffers=1)
    g = c.capture(from_host=True)
    g.replay()
    for x, y in zip(want4, _state(c)):
        assert torch.equal(x, y)
    assert int(c.status.item()) == 0
    del g

    d = _step(page)            # four steps per graph: set 0 reused inside the capture
    d.run_from_host(buffers=0)
    d.run_from_host(buffers=1)
    g = d.capture(from_host=True, host_steps=4)
    g.replay()
    for x, y in zip(want6, _state(d)):
        assert torch.equal(x, y)
    assert int(d.status.item()) == 0
    del g

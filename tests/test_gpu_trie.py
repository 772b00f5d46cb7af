"""GPU parity of the device-built continuation trees against the oracle's
restatement of the reference's KMP trie + BFS packing (``oracle/kmp.py``:
``find_all_matches_kmp`` then ``trie_bfs``), node for node, and of their
ancestor rows against the parent links."""
import numpy as np
import pytest
import torch

from oracle import kmp as OK

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def dev():
    assert torch.cuda.is_available(), "GPU tests need a CUDA device"
    from hsd_b200 import _native
    _native.load()
    return torch.device("cuda:0")


def _oracle(draft, window, depth, cap):
    trie, _ = OK.find_all_matches_kmp([draft], window, OK.compute_lps(window), depth)
    return OK.trie_bfs(trie, cap)


def _cases(seed, count):
    rng = np.random.default_rng(seed)
    out = []
    for _ in range(count):
        alpha = int(rng.integers(2, 40))
        n = int(rng.integers(0, 600))
        draft = [int(x) for x in rng.integers(1, alpha + 1, n)]
        gen = [int(x) for x in rng.integers(1, alpha + 1, int(rng.integers(1, 12)))]
        out.append((draft, gen[-min(10, len(gen)):]))
    return out


@pytest.mark.parametrize("seed,depth,cap", [(0, 15, 256), (1, 4, 256), (2, 15, 40),
                                            (3, 1, 256), (4, 0, 256), (5, 15, 1),
                                            (6, 15, 1024), (7, 9, 100)])
def test_trees_match_oracle(dev, seed, depth, cap):
    from hsd_b200.trie import continuation_trees
    cases = _cases(seed, 24)
    pool, off, ln = [], [], []
    for draft, _ in cases:
        off.append(len(pool))
        ln.append(len(draft))
        pool += draft
    t = lambda x: torch.tensor(x or [0], dtype=torch.int32, device=dev)
    last = [w[-1] for _, w in cases]
    status = torch.zeros(1, dtype=torch.int32, device=dev)
    trees = continuation_trees(t(pool), t(off), t(ln), t(last), depth, cap, status=status)
    got = trees.host()
    assert int(status.item()) == 0
    anc = trees.anc.cpu().numpy().view(np.uint64)
    for i, (draft, window) in enumerate(cases):
        want = _oracle(draft, window, depth, cap)
        assert got[i] == (list(want[0]), list(want[1]), list(want[2])), i
        parents = want[2]
        for node in range(len(parents)):
            bits = np.zeros(anc.shape[2] * 64, dtype=bool)
            a = node
            while a >= 0:
                bits[a] = True
                a = parents[a]
            row = np.unpackbits(anc[i, node].view(np.uint8), bitorder="little").astype(bool)
            assert np.array_equal(row, bits), (i, node)


def test_repetitive_and_edge_drafts(dev):
    from hsd_b200.trie import continuation_tree
    cases = [
        ([], [5]),                       # empty draft: root only
        ([7], [7]),                      # root at the last position: no follower
        ([1, 2, 3], [9]),                # root absent
        ([4] * 300, [4]),                # one long chain of repeats
        ([1, 2] * 700, [2, 1, 2]),       # 700 occurrences, two-way alternation
        ([int(x) for x in np.random.default_rng(3).integers(1, 4, 3072)], [2]),
    ]
    for draft, window in cases:
        for depth, cap in ((15, 256), (3, 1024)):
            want = _oracle(draft, window, depth, cap)
            got = continuation_tree(draft, window[-1], depth, cap, device=dev)
            assert got == (list(want[0]), list(want[1]), list(want[2]))


def test_too_many_occurrences_reports_capacity(dev):
    from hsd_b200 import _native as N
    from hsd_b200.trie import continuation_trees
    draft = torch.full((5000,), 3, dtype=torch.int32, device=dev)
    z = torch.zeros(1, dtype=torch.int32, device=dev)
    status = torch.zeros(1, dtype=torch.int32, device=dev)
    trees = continuation_trees(draft, z, torch.tensor([5000], dtype=torch.int32, device=dev),
                               torch.tensor([3], dtype=torch.int32, device=dev), 15, 256,
                               status=status)
    torch.cuda.synchronize()
    assert int(status.item()) & N.HSD_DEV_CAPACITY
    assert int(trees.counts.item()) == 0

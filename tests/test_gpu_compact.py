"""GPU parity: in-place KV compaction, keep indices and bit remaps (bit-exact)."""
import numpy as np
import pytest
import torch

from oracle import compact as OC

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def dev():
    assert torch.cuda.is_available(), "GPU tests need a CUDA device"
    return torch.device("cuda:0")


def random_keep(kv, rng, dead_frac, first_dead=None):
    keep = rng.random(kv) > dead_frac
    if first_dead is not None:
        keep[:first_dead] = True
    return keep


@pytest.mark.parametrize("layers,hkv,kv,dead,first", [
    (1, 2, 1512, 0.3, None),        # cfg1: one fp32-sized layer
    (28, 2, 4800, 0.05, 2600),      # cfg2-like: prefix untouched, drafts compacted
    (24, 8, 2500, 0.2, 1600),       # cfg4-like
    (3, 1, 777, 0.9, 0),            # almost everything dead
    (2, 2, 1000, 0.0, None),        # nothing dead: no row moves
])
def test_compact_matches_index_select(dev, layers, hkv, kv, dead, first):
    from hsd_b200.compaction import compact_kv, keep_indices, plane_pointers
    rng = np.random.default_rng(layers * 1000 + kv)
    keep = random_keep(kv, rng, dead, first)
    ks = [torch.randn(1, hkv, kv, 128, device=dev).to(torch.bfloat16) for _ in range(layers)]
    vs = [torch.randn(1, hkv, kv, 128, device=dev).to(torch.bfloat16) for _ in range(layers)]
    ref_k, ref_v = OC.compact_layers([k.cpu() for k in ks], [v.cpu() for v in vs],
                                     OC.keep_indices(keep))
    live = torch.from_numpy(_pack(keep)).to(dev)[None]
    keep_bits, keep_idx, counts = keep_indices(live, None, kv)
    planes = plane_pointers(ks + vs)
    status = torch.zeros(1, dtype=torch.int32, device=dev)
    compact_kv(planes, 256, keep_idx, counts=counts, status=status)
    torch.cuda.synchronize()
    assert status.item() == 0
    n_keep = int(keep.sum())
    c = counts.cpu().tolist()
    assert c[0] == n_keep
    moved = np.nonzero(OC.keep_indices(keep) != np.arange(n_keep))[0]
    assert c[1] == (int(moved[0]) if len(moved) else n_keep)
    np.testing.assert_array_equal(keep_idx[:n_keep].cpu().numpy(), OC.keep_indices(keep))
    for k, rk in zip(ks, ref_k):
        assert torch.equal(k[:, :, :n_keep].cpu(), rk)
    for v, rv in zip(vs, ref_v):
        assert torch.equal(v[:, :, :n_keep].cpu(), rv)


@pytest.mark.parametrize("n_planes,row_bytes,kv,dead,first", [
    (64, 256, 12000, 0.1, 50),      # > 8192 moved rows: indices past the staged cache
    (80, 512, 3000, 0.3, 200),      # 512-byte rows (head dim 256), bulk kernel
    (70, 64 * 1024, 40, 0.4, 1),    # rows larger than a staging buffer: cluster kernel
    (4, 1024, 2000, 0.5, 10),       # few planes: cluster kernel
    (100, 256, 300, 0.2, 100),      # two CTAs per plane, one wave: the second has none
    (148, 1024, 5000, 0.3, 7),      # two CTAs per plane, one plane per SM, 32-row waves
    (149, 256, 2000, 0.3, 5),       # more planes than SMs: one CTA per plane
])
def test_compact_row_sizes_and_long_moves(dev, n_planes, row_bytes, kv, dead, first):
    """Planes of raw rows of any 16-byte multiple move like index_select,
    whichever kernel the plane count and row size pick."""
    from hsd_b200.compaction import compact_kv, keep_indices
    rng = np.random.default_rng(n_planes + row_bytes + kv)
    keep = random_keep(kv, rng, dead, first)
    data = torch.randint(0, 256, (n_planes, kv, row_bytes), dtype=torch.uint8, device=dev)
    ref = data[:, torch.as_tensor(OC.keep_indices(keep), device=dev)].clone()
    live = torch.from_numpy(_pack(keep)).to(dev)[None]
    _, keep_idx, counts = keep_indices(live, None, kv)
    planes = torch.tensor([data[i].data_ptr() for i in range(n_planes)], dtype=torch.int64,
                          device=dev)
    status = torch.zeros(1, dtype=torch.int32, device=dev)
    compact_kv(planes, row_bytes, keep_idx, counts=counts, status=status)
    torch.cuda.synchronize()
    assert status.item() == 0
    n_keep = int(keep.sum())
    assert torch.equal(data[:, :n_keep], ref)


def _pack(b):
    from hsd_b200.plan import pack_bits
    return pack_bits(b).view(np.int64)


def test_keep_indices_live_filter(dev):
    """keep = OR over active pointer rows & ~filtered (D:1679-1687)."""
    from hsd_b200.compaction import keep_indices
    rng = np.random.default_rng(3)
    kv = 3001
    rows = rng.random((5, kv)) > 0.6
    filt = rng.random(kv) > 0.8
    expect = OC.keep_columns(rows, [0, 2, 4], filt)
    live = torch.from_numpy(_pack(rows[[0, 2, 4]])).to(dev)
    _, keep_idx, counts = keep_indices(live, torch.from_numpy(_pack(filt)).to(dev), kv)
    torch.cuda.synchronize()
    n = int(expect.sum())
    assert counts[0].item() == n
    np.testing.assert_array_equal(keep_idx[:n].cpu().numpy(), np.nonzero(expect)[0])


def test_compact_bits_remaps_visibility(dev):
    from hsd_b200.compaction import compact_bits, keep_indices
    rng = np.random.default_rng(8)
    kv = 900
    keep = rng.random(kv) > 0.3
    vis = rng.random((7, kv)) > 0.5
    stride = 20
    vb = np.zeros((7, stride), dtype=np.int64)
    vb[:, :(kv + 63) // 64] = _pack(vis)
    _, keep_idx, counts = keep_indices(torch.from_numpy(_pack(keep)).to(dev)[None], None, kv)
    n = int(keep.sum())
    out = compact_bits(torch.from_numpy(vb).to(dev), keep_idx, counts, (n + 63) // 64)
    torch.cuda.synchronize()
    exp = vis[:, keep]
    got = np.unpackbits(out.cpu().numpy().view(np.uint8).reshape(7, stride, 8), axis=-1,
                        bitorder="little").reshape(7, stride * 64)[:, :n].astype(bool)
    np.testing.assert_array_equal(got, exp)


def test_kv_append_matches_slice_copy(dev):
    from hsd_b200.compaction import kv_append
    L, hkv, cap, q, d = 3, 2, 900, 333, 128
    cache = torch.randn(L, 2, hkv, cap, d, device=dev).to(torch.bfloat16)
    new = torch.randn(L, 2, hkv, q, d, device=dev).to(torch.bfloat16)
    ref = cache.clone()
    ref[:, :, :, 500:500 + q] = new
    dst = torch.tensor([cache[l, k, h].data_ptr() for l in range(L) for k in range(2)
                        for h in range(hkv)], dtype=torch.int64, device=dev)
    src = torch.tensor([new[l, k, h].data_ptr() for l in range(L) for k in range(2)
                        for h in range(hkv)], dtype=torch.int64, device=dev)
    kv_append(dst, src, d * 2, 500, q)
    torch.cuda.synchronize()
    assert torch.equal(cache, ref)

"""GPU parity of the fused RoPE + cache update: bit-identical to the oracle
and to transformers' ``apply_rotary_pos_emb`` + ``torch.cat`` on the device.

Layouts: q / k / v as column slices of one fused projection output (row
stride (Hq + 2 Hkv) * 128), caches [Hkv, KV, 128] with the new rows written
at an offset; rows outside it must stay untouched.
"""
import numpy as np
import pytest
import torch

from oracle import rope as OR

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def dev():
    assert torch.cuda.is_available(), "GPU tests need a CUDA device"
    from hsd_b200 import _native
    _native.load()
    return torch.device("cuda:0")


def _cos_sin(pos, d=128, theta=1e6):
    inv = 1.0 / theta ** (torch.arange(0, d, 2, dtype=torch.float32) / d)
    f = pos.float()[:, None] * inv[None, :]
    emb = torch.cat([f, f], dim=-1)
    return emb.cos().to(torch.bfloat16), emb.sin().to(torch.bfloat16)


@pytest.mark.parametrize("n,hq,hkv,kv,row0,seed", [
    (217, 12, 2, 600, 300, 0),
    (1, 12, 2, 64, 63, 1),
    (2176, 12, 2, 4800, 2624, 2),
    (130, 16, 8, 400, 0, 3),
])
def test_matches_oracle_and_transformers(dev, n, hq, hkv, kv, row0, seed):
    from transformers.models.qwen2.modeling_qwen2 import apply_rotary_pos_emb

    from hsd_b200.rope import rope_append
    g = torch.Generator().manual_seed(seed)
    w = (hq + 2 * hkv) * 128
    qkv = (torch.randn(n, w, generator=g) * 2).to(torch.bfloat16)
    cos, sin = _cos_sin(torch.randint(0, 10000, (n,), generator=g))
    kc = torch.randn(hkv, kv, 128, generator=g).to(torch.bfloat16)
    vc = torch.randn(hkv, kv, 128, generator=g).to(torch.bfloat16)
    q = qkv[:, :hq * 128].reshape(n, hq, 128).transpose(0, 1)
    k = qkv[:, hq * 128:(hq + hkv) * 128].reshape(n, hkv, 128).transpose(0, 1)
    v = qkv[:, (hq + hkv) * 128:].reshape(n, hkv, 128).transpose(0, 1)
    want_q, want_kc, want_vc = OR.rope_append(q, k, v, cos, sin, kc.float().numpy(),
                                              vc.float().numpy(), row0)

    d_qkv, d_kc, d_vc = qkv.to(dev), kc.to(dev), vc.to(dev)
    d_cos, d_sin = cos.to(dev), sin.to(dev)
    qv = rope_append(d_qkv[:, :hq * 128], d_qkv[:, hq * 128:(hq + hkv) * 128],
                     d_qkv[:, (hq + hkv) * 128:], d_cos, d_sin, d_kc, d_vc, row0)
    torch.cuda.synchronize()
    assert qv.shape == (1, hq, n, 128)
    assert np.array_equal(qv[0].float().cpu().numpy(), want_q)
    assert np.array_equal(d_kc.float().cpu().numpy(), want_kc)
    assert np.array_equal(d_vc.float().cpu().numpy(), want_vc)
    # the reference's own ops on the device
    qd, kd = qkv.to(dev), None
    q4 = qd[:, :hq * 128].reshape(1, n, hq, 128).transpose(1, 2)
    k4 = qd[:, hq * 128:(hq + hkv) * 128].reshape(1, n, hkv, 128).transpose(1, 2)
    qe, ke = apply_rotary_pos_emb(q4, k4, d_cos[None], d_sin[None])
    assert torch.equal(qe, qv)
    assert torch.equal(ke[0], d_kc[:, row0:row0 + n])


def test_keys_and_values_only(dev):
    from hsd_b200.rope import rope_append
    g = torch.Generator().manual_seed(9)
    n, hkv = 40, 2
    k = torch.randn(n, hkv * 128, generator=g).to(torch.bfloat16)
    v = torch.randn(n, hkv * 128, generator=g).to(torch.bfloat16)
    cos, sin = _cos_sin(torch.arange(100, 100 + n))
    kc = torch.zeros(hkv, 64, 128, dtype=torch.bfloat16)
    vc = torch.zeros(hkv, 64, 128, dtype=torch.bfloat16)
    _, want_kc, want_vc = OR.rope_append(np.zeros((0, n, 128), np.float32),
                                         k.reshape(n, hkv, 128).transpose(0, 1),
                                         v.reshape(n, hkv, 128).transpose(0, 1), cos, sin,
                                         kc.float().numpy(), vc.float().numpy(), 10)
    d_kc, d_vc = kc.to(dev), vc.to(dev)
    assert rope_append(None, k.to(dev), v.to(dev), cos.to(dev), sin.to(dev), d_kc, d_vc,
                       10) is None
    torch.cuda.synchronize()
    assert np.array_equal(d_kc.float().cpu().numpy(), want_kc)
    assert np.array_equal(d_vc.float().cpu().numpy(), want_vc)


def test_special_values_bitwise_like_transformers(dev):
    """Rounding edge cases: products and sums that overflow to infinity,
    bf16 subnormals, signed zeros, ties between two bf16 neighbours and
    infinite inputs, compared bit for bit (as int16) with transformers' ops
    on the device."""
    from transformers.models.qwen2.modeling_qwen2 import apply_rotary_pos_emb

    from hsd_b200.rope import rope_append
    g = torch.Generator().manual_seed(11)
    n, hq, hkv = 256, 4, 2
    w = (hq + 2 * hkv) * 128
    special = torch.tensor([3.0e38, -3.0e38, 1.7e38, 2.0e-39, -5.0e-40, 1.0e-38, 0.0, -0.0,
                            float("inf"), float("-inf"), 1.00390625, 65504.0, 1.5e-45, 7.0])
    qkv = torch.randn(n, w, generator=g)
    pick = torch.randint(0, len(special), (n, w), generator=g)
    mask = torch.rand(n, w, generator=g) < 0.5
    qkv = torch.where(mask, special[pick], qkv).to(torch.bfloat16)
    cs_special = torch.tensor([1.0, -1.0, 0.5, 0.99609375, 1.0e-38, 2.0e-39, 0.75, 0.0])
    cos = cs_special[torch.randint(0, len(cs_special), (n, 128), generator=g)]
    sin = cs_special[torch.randint(0, len(cs_special), (n, 128), generator=g)]
    cos, sin = cos.to(torch.bfloat16).to(dev), sin.to(torch.bfloat16).to(dev)
    qd = qkv.to(dev)
    kc = torch.zeros(hkv, n + 8, 128, dtype=torch.bfloat16, device=dev)
    vc = torch.zeros_like(kc)
    q4 = qd[:, :hq * 128].reshape(1, n, hq, 128).transpose(1, 2)
    k4 = qd[:, hq * 128:(hq + hkv) * 128].reshape(1, n, hkv, 128).transpose(1, 2)
    qe, ke = apply_rotary_pos_emb(q4.clone(), k4.clone(), cos[None], sin[None])
    qv = rope_append(qd[:, :hq * 128], qd[:, hq * 128:(hq + hkv) * 128],
                     qd[:, (hq + hkv) * 128:], cos, sin, kc, vc, 4)
    torch.cuda.synchronize()
    nan_q, nan_k = torch.isnan(qe), torch.isnan(ke[0])
    assert torch.equal(torch.isnan(qv), nan_q) and torch.equal(torch.isnan(kc[:, 4:4 + n]), nan_k)
    bits = lambda t: t.contiguous().view(torch.int16)
    assert torch.equal(bits(torch.where(nan_q, 0, qv)), bits(torch.where(nan_q, 0, qe)))
    got_k = kc[:, 4:4 + n]
    assert torch.equal(bits(torch.where(nan_k, 0, got_k)), bits(torch.where(nan_k, 0, ke[0])))
    assert torch.equal(bits(vc[:, 4:4 + n]),
                       bits(qd[:, (hq + hkv) * 128:].reshape(n, hkv, 128).transpose(0, 1)))

"""The RoPE + cache-update oracle against transformers' own
``apply_rotary_pos_emb`` (the function the reference calls, D:345-346), run
on the CPU in bf16: bit-identical."""
import numpy as np
import torch

from oracle import rope as OR


def _cos_sin(pos, d=128, theta=1e6):
    inv = 1.0 / theta ** (torch.arange(0, d, 2, dtype=torch.float32) / d)
    f = pos.float()[:, None] * inv[None, :]
    emb = torch.cat([f, f], dim=-1)
    return emb.cos().to(torch.bfloat16), emb.sin().to(torch.bfloat16)


def test_apply_rope_matches_transformers():
    from transformers.models.qwen2.modeling_qwen2 import apply_rotary_pos_emb
    g = torch.Generator().manual_seed(0)
    pos = torch.randint(0, 8000, (77,), generator=g)
    cos, sin = _cos_sin(pos)
    q = (torch.randn(1, 12, 77, 128, generator=g) * 3).to(torch.bfloat16)
    k = (torch.randn(1, 2, 77, 128, generator=g) * 3).to(torch.bfloat16)
    qe, ke = apply_rotary_pos_emb(q, k, cos[None], sin[None])
    assert np.array_equal(OR.apply_rope(q[0], cos, sin), qe[0].float().numpy())
    assert np.array_equal(OR.apply_rope(k[0], cos, sin), ke[0].float().numpy())


def test_rope_append_rows():
    g = torch.Generator().manual_seed(1)
    cos, sin = _cos_sin(torch.arange(10, 15))
    q = torch.randn(4, 5, 128, generator=g).to(torch.bfloat16)
    k = torch.randn(2, 5, 128, generator=g).to(torch.bfloat16)
    v = torch.randn(2, 5, 128, generator=g).to(torch.bfloat16)
    kc = torch.randn(2, 20, 128, generator=g).to(torch.bfloat16).float().numpy()
    vc = torch.randn(2, 20, 128, generator=g).to(torch.bfloat16).float().numpy()
    qr, kc2, vc2 = OR.rope_append(q, k, v, cos, sin, kc, vc, 7)
    assert np.array_equal(kc2[:, :7], kc[:, :7]) and np.array_equal(kc2[:, 12:], kc[:, 12:])
    assert np.array_equal(vc2[:, 7:12], v.float().numpy())
    assert np.array_equal(kc2[:, 7:12], OR.apply_rope(k, cos, sin))

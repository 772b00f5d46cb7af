"""The next-token oracle (lm_head + argmax) on the CPU: bf16 rounding, the
first-index tie rule and the near-tie criterion the GPU parity tests use."""
import numpy as np
import torch

from oracle import lm_head as OL


def test_round_bf16_single_rounding():
    # exactly representable, halfway cases (ties to even), and a value just
    # below a halfway point that a float32 round trip would push up
    assert OL.round_bf16([1.0, -2.5, 1.00390625, 1.01171875]).tolist() == \
        [1.0, -2.5, 1.0, 1.015625]
    assert OL.round_bf16([18.437499718946164])[0] == 18.375
    x = np.random.default_rng(1).standard_normal(20000) * 30
    r = OL.round_bf16(x)
    # every result is a bf16 value and the nearest one
    b = torch.tensor(r.astype(np.float32)).to(torch.bfloat16).double().numpy()
    assert np.array_equal(b, r)
    step = np.ldexp(1.0, np.frexp(r)[1] - 8)
    assert np.all(np.abs(r - x) <= step / 2 + 1e-12)


def test_argmax_first_index_on_ties():
    g = torch.Generator().manual_seed(0)
    w = torch.randn(700, 64, generator=g).to(torch.bfloat16)
    w[650] = w[20]          # duplicate rows: equal logits, the lower id wins
    h = w[20:21].float().clone()
    ids, mx, exact = OL.lm_head_argmax(h, w)
    assert ids.tolist() == [20]
    assert exact[0, 20] == exact[0, 650]


def test_all_negative_logits():
    g = torch.Generator().manual_seed(2)
    w = torch.randn(300, 64, generator=g).abs().to(torch.bfloat16)
    h = -torch.randn(3, 64, generator=g).abs()
    ids, mx, exact = OL.lm_head_argmax(h, w)
    assert np.all(mx < 0)
    assert np.array_equal(ids, OL.round_bf16(exact).argmax(1))


def test_near_tie_criterion():
    row = np.array([10.0, 10.05, 9.0, 10.1])
    assert OL.near_tie(row, 1, 3)          # within one bf16 step (1/16 at 10)
    assert not OL.near_tie(row, 2, 3)

"""fp32 masked GQA attention with log-sum-exp (test infrastructure only).

Restates what the reference's ``flex_attention_forward`` returns
(D:72-135, H:103-180): ``softmax(q k^T * scale + mask) v`` per query head,
with the KV heads repeated ``Hq / Hkv`` times (``repeat_kv``, D:137-146),
the output transposed to ``[Q, Hq, D]`` (D:134) and the LSE in natural log
``[Hq, Q]``.  FlexAttention gives fully masked rows an all-zero output and
an LSE of -inf (checked by ``tests/golden/make_golden.py``); so does this.
"""
from __future__ import annotations

import math

import numpy as np
import torch


def attention_fp32(q, k, v, allowed, scale=None):
    """Reference attention on the CPU in fp32.

    q: ``[Hq, Q, D]``; k, v: ``[Hkv, KV, D]``; allowed: bool ``[Q, KV]``.
    Returns ``(out [Q, Hq, D] float32, lse [Hq, Q] float32)``.
    """
    q = torch.as_tensor(q).float()
    k = torch.as_tensor(k).float()
    v = torch.as_tensor(v).float()
    allowed = torch.as_tensor(np.asarray(allowed), dtype=torch.bool)
    hq, qn, d = q.shape
    hkv = k.shape[0]
    rep = hq // hkv
    if scale is None:
        scale = 1.0 / math.sqrt(d)
    k = k.repeat_interleave(rep, dim=0)
    v = v.repeat_interleave(rep, dim=0)
    s = torch.matmul(q, k.transpose(-1, -2)) * scale
    s = s.masked_fill(~allowed[None], float("-inf"))
    lse = torch.logsumexp(s, dim=-1)
    p = torch.exp(s - lse[..., None])
    p = torch.nan_to_num(p, nan=0.0)
    out = torch.matmul(p, v)
    return out.transpose(0, 1).contiguous(), lse


def flex_attention_eager(q, k, v, allowed, scale=None):
    """The reference's own call (D:94-130) run eagerly on the CPU.

    ``create_block_mask`` with BLOCK_SIZE (128, 64) over the dense predicate,
    then ``flex_attention(..., return_lse=True)``; K/V are expanded with
    ``repeat_kv`` when Hq is not a power of two (D:108-115), otherwise
    ``enable_gqa`` is used.  Inputs as for :func:`attention_fp32`.
    """
    from torch.nn.attention.flex_attention import (create_block_mask,
                                                   flex_attention)

    q = torch.as_tensor(q).float()[None]
    k = torch.as_tensor(k).float()[None]
    v = torch.as_tensor(v).float()[None]
    pred = torch.as_tensor(np.asarray(allowed), dtype=torch.bool)
    qn, kvn = pred.shape

    def mask_mod(b, h, qi, ki):
        return pred[qi, ki]

    bm = create_block_mask(mask_mod, None, None, qn, kvn, device="cpu",
                           BLOCK_SIZE=(128, 64))
    hq = q.shape[1]
    gqa = (hq & (hq - 1)) == 0
    if not gqa:
        rep = hq // k.shape[1]
        k = k.repeat_interleave(rep, dim=1)
        v = v.repeat_interleave(rep, dim=1)
    out, lse = flex_attention(q, k, v, block_mask=bm, enable_gqa=gqa,
                              scale=scale, return_lse=True)
    return out[0].transpose(0, 1).contiguous(), lse[0]

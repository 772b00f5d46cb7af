"""Rotary position embedding + cache update on the CPU (test infrastructure
only).

Restates what the reference's patched Qwen2 attention does with a layer's new
rows (hsd/dots_ocr_pipeline/modeling_dots_ocr_hsd.py D:337-351):
transformers' ``apply_rotary_pos_emb`` -- ``q * cos + rotate_half(q) * sin``
with ``rotate_half(x) = cat(-x[..., d/2:], x[..., :d/2])`` -- evaluated as
torch's bf16 tensor ops evaluate it (each product rounded to bf16, the sum of
the two bf16 products formed in fp32 and rounded to bf16), then
``DynamicCache.update``'s ``torch.cat`` of key and value states onto the
layer's cache.  Arithmetic in numpy float32 with explicit bf16 rounding.
"""
from __future__ import annotations

import numpy as np
import torch


def _bf16(x):
    """float32 array -> nearest bf16 values (ties to even), as float32."""
    return torch.from_numpy(np.ascontiguousarray(x, dtype=np.float32)).to(
        torch.bfloat16).float().numpy()


def apply_rope(x, cos, sin):
    """x: [..., Q, D] bf16 values; cos, sin: [Q, D] (broadcast over leading
    dims).  Returns the rotated values as float32 (exactly bf16)."""
    x = torch.as_tensor(x).float().numpy()
    cos = torch.as_tensor(cos).float().numpy()
    sin = torch.as_tensor(sin).float().numpy()
    h = x.shape[-1] // 2
    rot = np.concatenate([-x[..., h:], x[..., :h]], axis=-1)
    return _bf16(_bf16(x * cos) + _bf16(rot * sin))


def rope_append(q, k, v, cos, sin, k_cache, v_cache, dst_row0):
    """Per-layer step: q [Hq, Q, D], k / v [Hkv, Q, D], caches [Hkv, KV, D]
    (numpy float32 holding bf16 values).  Returns (rotated q, new k cache,
    new v cache) with rows [dst_row0, dst_row0 + Q) of the caches replaced."""
    qr = apply_rope(q, cos, sin)
    kr = apply_rope(k, cos, sin)
    kc = np.array(k_cache, dtype=np.float32, copy=True)
    vc = np.array(v_cache, dtype=np.float32, copy=True)
    n = kr.shape[1]
    kc[:, dst_row0:dst_row0 + n] = kr
    vc[:, dst_row0:dst_row0 + n] = torch.as_tensor(v).float().numpy()
    return qr, kc, vc

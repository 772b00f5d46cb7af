"""Rotary position embedding of a layer's new rows fused with the cache update.

Drop-in for the two steps the reference's patched Qwen2 attention takes
between the projections and the attention call
(hsd/dots_ocr_pipeline/modeling_dots_ocr_hsd.py D:337-351):
``apply_rotary_pos_emb(query_states, key_states, cos, sin)`` and
``past_key_value.update(key_states, value_states, ...)`` (a ``torch.cat`` of
the whole layer cache).  One launch rotates the query rows in place in the
``q_proj`` output and writes the rotated key rows and the value rows into
preallocated cache planes; results are bit-identical to torch's bf16 ops.
"""
from __future__ import annotations

import torch

from . import _native as N


def _rows(t, name, width=None):
    t2 = t.reshape(-1, t.shape[-1]) if t.dim() != 2 else t
    if t2.dtype != torch.bfloat16 or not t2.is_cuda:
        raise TypeError(f"rope_append: {name} must be a bf16 CUDA tensor")
    if t2.stride(-1) != 1:
        raise ValueError(f"rope_append: {name} rows must be contiguous")
    if width is not None and t2.shape[-1] != width:
        raise ValueError(f"rope_append: {name} has {t2.shape[-1]} columns, expected {width}")
    return t2


def _cache(c, name):
    c3 = c.reshape(-1, c.shape[-2], c.shape[-1]) if c.dim() != 3 else c
    if c3.dtype != torch.bfloat16 or c3.shape[-1] != 128 or c3.stride(-1) != 1:
        raise ValueError(f"rope_append: {name} must be bf16 [..., Hkv, KV, 128] with contiguous rows")
    return c3


def rope_append(q, k, v, cos, sin, k_cache, v_cache, dst_row0, num_q_heads=None,
                num_kv_heads=None):
    """Rotate ``q`` in place and append rotated ``k`` and ``v`` to the caches.

    q: ``[..., Q, Hq * 128]`` (the ``q_proj`` output; may be a column slice of
    a fused projection) or None; k, v: ``[..., Q, Hkv * 128]``; cos, sin:
    ``[..., Q, 128]`` bf16 (the model's ``position_embeddings``); k_cache,
    v_cache: ``[..., Hkv, KV, 128]`` bf16, rows ``[dst_row0, dst_row0 + Q)``
    receive the new rows.  Returns the rotated queries as a
    ``[1, Hq, Q, 128]`` view (the reference's ``query_states`` layout), or
    None when q is None.  Asynchronous on the current stream.
    """
    kc, vc = _cache(k_cache, "k_cache"), _cache(v_cache, "v_cache")
    hkv = num_kv_heads or kc.shape[0]
    k2, v2 = _rows(k, "k", hkv * 128), _rows(v, "v", hkv * 128)
    n = k2.shape[0]
    if k2.stride(0) != v2.stride(0):
        raise ValueError("rope_append: k and v must share a row stride")
    c2, s2 = _rows(cos, "cos", 128), _rows(sin, "sin", 128)
    if c2.stride(0) != s2.stride(0) or c2.shape[0] != n or v2.shape[0] != n:
        raise ValueError("rope_append: cos / sin / k / v row counts or strides differ")
    if kc.stride() != vc.stride() or kc.shape != vc.shape or kc.shape[0] != hkv:
        raise ValueError("rope_append: k_cache and v_cache must have one layout")
    if dst_row0 < 0 or dst_row0 + n > kc.shape[1]:
        raise ValueError(f"rope_append: rows {dst_row0}..{dst_row0 + n} past the cache")
    hq, q2, qptr, qstride = 0, None, None, 0
    if q is not None:
        hq = num_q_heads or q.shape[-1] // 128
        q2 = _rows(q, "q", hq * 128)
        if q2.shape[0] != n:
            raise ValueError("rope_append: q and k row counts differ")
        qptr, qstride = N.ptr(q2), q2.stride(0)
    lib = N.load()
    N.check(lib.hsd_rope_append(qptr, qstride, N.ptr(k2), N.ptr(v2), k2.stride(0), N.ptr(c2),
                                N.ptr(s2), c2.stride(0), n, hq, hkv, 128, N.ptr(kc),
                                kc.stride(0), N.ptr(vc), vc.stride(0), kc.stride(1), dst_row0,
                                N.stream_handle()), "hsd_rope_append")
    if q2 is None:
        return None
    return q2.unflatten(-1, (hq, 128)).unsqueeze(0).transpose(1, 2)

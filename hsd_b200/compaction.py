"""KV-cache compaction (host side of subsystem 2).

Replaces the reference's per-layer ``index_select(-2, keep_indices)`` on K and
V (hsd/dots_ocr_pipeline/modeling_dots_ocr_hsd.py D:1705-1722,
hsd/hunyuan_ocr_pipeline/modeling_hunyuan_vl_hsd.py H:2262-2269) with one
in-place kernel over every (layer, K/V, KV head) plane that moves only the
rows at or after the first dropped one.
"""
from __future__ import annotations

import torch

from . import _native as N


def plane_pointers(tensors, device=None):
    """Device array of plane base addresses.

    ``tensors`` are per-layer K or V caches ``[1, Hkv, KV, D]`` / ``[Hkv, KV, D]``
    (contiguous rows); every KV head of every tensor is one plane.
    """
    addrs = []
    for t in tensors:
        x = t[0] if t.dim() == 4 else t
        if x.stride(-1) != 1 or x.stride(-2) != x.shape[-1]:
            raise ValueError("compaction needs contiguous [KV, D] rows per head")
        for h in range(x.shape[0]):
            addrs.append(x[h].data_ptr())
    dev = device or tensors[0].device
    return torch.tensor(addrs, dtype=torch.int64, device=dev)


def keep_indices(live_bits, filter_bits, kv_len, stream=None, out=None):
    """keep = OR(live rows) & ~filter -> (keep_bits, keep_idx, counts[2]) on device.

    ``out``: optional preallocated ``(keep_bits, keep_idx, counts)`` with at
    least ``ceil(kv_len / 64)`` words and ``kv_len`` indices."""
    lib = N.load()
    dev = live_bits.device
    n_live = live_bits.shape[0] if live_bits.dim() == 2 else 1
    stride = live_bits.shape[-1]
    nw = (kv_len + 63) // 64
    if out is not None:
        keep_bits, keep_idx, counts = out
        if keep_bits.numel() < nw or keep_idx.numel() < max(kv_len, 1) or counts.numel() < 2:
            raise ValueError("keep_indices: preallocated outputs too small")
    else:
        keep_bits = torch.empty(nw, dtype=torch.int64, device=dev)
        keep_idx = torch.empty(max(kv_len, 1), dtype=torch.int32, device=dev)
        counts = torch.empty(2, dtype=torch.int32, device=dev)
    N.check(lib.hsd_keep_indices(N.ptr(live_bits), n_live, stride, N.ptr(filter_bits), kv_len,
                                 N.ptr(keep_bits), N.ptr(keep_idx), N.ptr(counts),
                                 N.stream_handle(stream)), "hsd_keep_indices")
    return keep_bits, keep_idx, counts


def compact_kv(planes, row_bytes, keep_idx, n_keep=None, counts=None, status=None,
               stream=None):
    """In-place compaction of every plane: row i <- row keep_idx[i].

    ``planes``: int64 device tensor of plane addresses (:func:`plane_pointers`).
    Pass either the host ``n_keep`` or the device ``counts`` written by
    :func:`keep_indices` (then only rows from ``counts[1]`` on move).
    """
    lib = N.load()
    if keep_idx.dtype != torch.int32:
        keep_idx = keep_idx.to(torch.int32)
    N.check(lib.hsd_compact_kv(N.ptr(planes), planes.numel(), int(row_bytes), N.ptr(keep_idx),
                               -1 if n_keep is None else int(n_keep), N.ptr(counts),
                               N.ptr(status), N.stream_handle(stream)), "hsd_compact_kv")


def kv_append(dst_planes, src_planes, row_bytes, dst_row0, n_rows, stream=None):
    """Append ``n_rows`` rows of every source plane at ``dst_row0`` of its
    destination plane (the cache update ``DynamicCache.update`` does with
    ``torch.cat``)."""
    lib = N.load()
    N.check(lib.hsd_kv_append(N.ptr(dst_planes), N.ptr(src_planes), dst_planes.numel(),
                              int(row_bytes), int(dst_row0), int(n_rows),
                              N.stream_handle(stream)), "hsd_kv_append")


def compact_bits(in_bits, keep_idx, counts, out_words, out=None, stream=None):
    """Visibility rows after compaction: out[r] bit i = in[r] bit keep_idx[i]."""
    lib = N.load()
    if out is None:
        out = torch.zeros_like(in_bits)
    N.check(lib.hsd_compact_bits(N.ptr(in_bits), N.ptr(out), in_bits.shape[0], in_bits.shape[1],
                                 N.ptr(keep_idx), N.ptr(counts), int(out_words),
                                 N.stream_handle(stream)), "hsd_compact_bits")
    return out

"""Next tokens of the packed rows: fused lm_head + argmax.

Drop-in for the two lines of the reference's loop that turn the decoder's
final hidden states into next tokens, ``logits = outputs.logits`` (the
model's ``lm_head``, a bias-free bf16 linear layer) and
``all_next_tokens = logits.argmax(dim=-1)``
(hsd/dots_ocr_pipeline/modeling_dots_ocr_hsd.py D:1057-1064).  The kernel
never writes the ``[Q, vocab]`` logits: each 128 x 256 tile of the product
is reduced to a per-row (max, first column) in the epilogue, with the logits
rounded to bf16 as the logits tensor would hold them and ties going to the
lowest id, as ``torch.argmax`` does.
"""
from __future__ import annotations

import ctypes as C

import torch

from . import _native as N

_workspaces = {}


def _workspace(q_len, device):
    """Zero-filled per-device scratch, grown to fit ``q_len`` rows; every call
    leaves it zeroed again (calls sharing it must not overlap in time)."""
    need = N.load().hsd_lm_head_argmax_workspace_bytes(q_len)
    ws = _workspaces.get(device)
    if ws is None or ws[1] < need:
        buf = torch.zeros(need + 256, dtype=torch.uint8, device=device)
        ws = (buf, need)
        _workspaces[device] = ws
    buf, nbytes = ws
    return (buf.data_ptr() + 255) & ~255, nbytes


def lm_head_argmax(hidden, weight, *, out=None, out_int32=None, max_logit=None, status=None):
    """``argmax(hidden @ weight.T, dim=-1)`` with bf16 logits, without the logits.

    hidden: ``[..., H]`` bf16 (the decoder's final normed states); weight:
    ``[V, H]`` bf16 (``lm_head.weight``).  Returns int64 ids of shape
    ``hidden.shape[:-1]`` (or fills ``out``); ``out_int32`` (int32, same
    number of rows) receives the ids too, in the form the acceptance kernel
    reads; ``max_logit`` (fp32) the maximal bf16 logit per row.  Runs on the
    current stream without a host sync.
    """
    if hidden.dtype != torch.bfloat16 or weight.dtype != torch.bfloat16:
        raise TypeError("lm_head_argmax: hidden and weight must be bf16")
    if not hidden.is_cuda or hidden.device != weight.device:
        raise ValueError("lm_head_argmax: hidden and weight must be on the same CUDA device")
    hd = hidden.shape[-1]
    if weight.dim() != 2 or weight.shape[1] != hd:
        raise ValueError(f"lm_head_argmax: weight {tuple(weight.shape)} vs hidden dim {hd}")
    h2 = hidden.reshape(-1, hd)
    if h2.stride(-1) != 1:
        h2 = h2.contiguous()
    w = weight if weight.stride(-1) == 1 else weight.contiguous()
    q = h2.shape[0]
    lead = hidden.shape[:-1]
    if out is None:
        out = torch.empty(lead, dtype=torch.int64, device=hidden.device)
    for t, dt in ((out, torch.int64), (out_int32, torch.int32), (max_logit, torch.float32)):
        if t is not None and (t.dtype != dt or t.numel() != q or not t.is_contiguous()):
            raise ValueError(f"lm_head_argmax: output must be contiguous {dt} with {q} rows")
    if q == 0:
        return out
    lib = N.load()
    base, nbytes = _workspace(q, hidden.device)
    N.check(lib.hsd_lm_head_argmax(
        N.ptr(h2), h2.stride(0), N.ptr(w), w.stride(0), q, w.shape[0], hd, N.ptr(out_int32),
        N.ptr(out), N.ptr(max_logit), C.c_void_p(base), nbytes, N.ptr(status),
        N.stream_handle()), "hsd_lm_head_argmax")
    return out


def probe_logits(hidden, weight, rows, toks, *, out=None, status=None):
    """Single bf16 logits ``logits[rows[k], toks[k]]`` as float32, without
    the logits tensor: ``hidden[rows[k]] . weight[toks[k]]`` with fp32
    accumulation rounded to bf16 (``hsd_probe_logits``); ``toks[k] < 0``
    gives 0.  These are the entries the logit-ratio acceptance reads
    (D:1167-1168, D:1231-1232); :meth:`hsd_b200.loop.VerifyLoop.logit_probes`
    lists them for a step.  ``rows`` / ``toks``: int32 device tensors.
    """
    if hidden.dtype != torch.bfloat16 or weight.dtype != torch.bfloat16:
        raise TypeError("probe_logits: hidden and weight must be bf16")
    hd = hidden.shape[-1]
    if weight.dim() != 2 or weight.shape[1] != hd:
        raise ValueError(f"probe_logits: weight {tuple(weight.shape)} vs hidden dim {hd}")
    h2 = hidden.reshape(-1, hd)
    if h2.stride(-1) != 1:
        h2 = h2.contiguous()
    w = weight if weight.stride(-1) == 1 else weight.contiguous()
    n = rows.numel()
    if toks.numel() != n or rows.dtype != torch.int32 or toks.dtype != torch.int32:
        raise ValueError("probe_logits: rows and toks int32 of one length")
    rows, toks = rows.contiguous(), toks.contiguous()
    if out is None:
        out = torch.empty(n, dtype=torch.float32, device=hidden.device)
    if status is None:
        status = torch.zeros(1, dtype=torch.int32, device=hidden.device)
    if n == 0:
        return out
    N.check(N.load().hsd_probe_logits(
        N.ptr(h2), h2.stride(0), N.ptr(w), w.stride(0), h2.shape[0], w.shape[0], hd,
        N.ptr(rows), N.ptr(toks), n, N.ptr(out), N.ptr(status), N.stream_handle()),
        "hsd_probe_logits")
    return out


def lm_head_rank(hidden, weight, probe_logit, ref_col, excl_col, *, status=None):
    """Rank of a token among a row's bf16 logits and the row's second best,
    without the logits (``hsd_lm_head_rank``), for HunYuan's SPEC_MODE=topk /
    adaptive acceptance (H:1712-1736).

    For every row r of ``hidden`` (``[R, H]`` bf16, e.g. the last block's
    final states): ``rank[r]`` = the number of columns whose logit exceeds
    ``probe_logit[r]`` (= ``logits[r, ref_col[r]]``, :func:`probe_logits`)
    plus the columns below ``ref_col[r]`` with an equal logit, so
    ``rank[r] < k`` means ``ref_col[r]`` is among ``topk(k).indices``;
    ``second[r]`` = the largest logit outside column ``excl_col[r]`` (the
    row's argmax), ``topk(2).values[1]``.  ``probe_logit`` float32,
    ``ref_col`` / ``excl_col`` int32, one per row.  Returns ``(rank int32,
    second float32)``.
    """
    if hidden.dtype != torch.bfloat16 or weight.dtype != torch.bfloat16:
        raise TypeError("lm_head_rank: hidden and weight must be bf16")
    if not hidden.is_cuda or hidden.device != weight.device:
        raise ValueError("lm_head_rank: hidden and weight must be on the same CUDA device")
    hd = hidden.shape[-1]
    if weight.dim() != 2 or weight.shape[1] != hd:
        raise ValueError(f"lm_head_rank: weight {tuple(weight.shape)} vs hidden dim {hd}")
    h2 = hidden.reshape(-1, hd)
    if h2.stride(-1) != 1:
        h2 = h2.contiguous()
    w = weight if weight.stride(-1) == 1 else weight.contiguous()
    q = h2.shape[0]
    for t, dt in ((probe_logit, torch.float32), (ref_col, torch.int32), (excl_col, torch.int32)):
        if t.dtype != dt or t.numel() != q or not t.is_contiguous():
            raise ValueError(f"lm_head_rank: inputs must be contiguous {dt} with {q} rows")
    rank = torch.zeros(q, dtype=torch.int32, device=hidden.device)
    second = torch.full((q,), float("-inf"), dtype=torch.float32, device=hidden.device)
    if q == 0:
        return rank, second
    base, nbytes = _workspace(q, hidden.device)
    N.check(N.load().hsd_lm_head_rank(
        N.ptr(h2), h2.stride(0), N.ptr(w), w.stride(0), q, w.shape[0], hd, N.ptr(probe_logit),
        N.ptr(ref_col), N.ptr(excl_col), N.ptr(rank), N.ptr(second), C.c_void_p(base), nbytes,
        N.ptr(status), N.stream_handle()), "hsd_lm_head_rank")
    return rank, second

"""Verification attention: the drop-in for the reference's attention hook.

``flex_attention_forward`` keeps the signature and return convention of the
reference's hook (hsd/dots_ocr_pipeline/modeling_dots_ocr_hsd.py D:72-135,
hsd/hunyuan_ocr_pipeline/modeling_hunyuan_vl_hsd.py H:103-180), which the
patched Qwen2 / HunYuan attention calls per decoder layer (D:378-381,
H:1039-1042).  It accepts the same dense float mask (converted once per step
and cached by identity, as D:83-106 caches its BlockMask), a
:class:`~hsd_b200.plan.PackedMask`, or a prebuilt
:class:`~hsd_b200.plan.TilePlan`.  Grouped KV heads are consumed directly;
nothing is expanded the way ``repeat_kv`` (D:137-146) does.
"""
from __future__ import annotations

import contextlib
import ctypes
import math

import torch

from . import _native as N
from .plan import PackedMask, TilePlan, plan_from_dense

_cache = {"src": None, "plan": None}
_workspaces = {}


class AttentionWorkspace:
    """Device scratch of the load-balanced schedule (one per device and
    stream): the partial rows of items cut between two SMs' shares of the
    work, their ready flags and a launch generation.  Zero-filled once here;
    every call leaves it ready for the next.  Calls that share one workspace
    must not overlap on the GPU: launches on one stream never do, which is
    why the cache below keeps one workspace per stream."""

    def __init__(self, nbytes, device, stream=None):
        dev = torch.device(device)
        if stream is not None:
            with torch.cuda.stream(stream):
                self.buf = torch.zeros(nbytes + 256, dtype=torch.uint8, device=dev)
        else:
            self.buf = torch.zeros(nbytes + 256, dtype=torch.uint8, device=dev)
        self.base = (self.buf.data_ptr() + 255) & ~255
        self.nbytes = nbytes


def attention_workspace(q_len, hq, hkv, device, stream=None):
    """The cached workspace of (``device``, ``stream``; default the device's
    current stream), grown to fit (q_len, hq, hkv).  A workspace that grows
    is allocated on the same stream, and the caching allocator hands the old
    block to no other stream, so a launch still queued on that stream keeps
    valid scratch."""
    need = N.load().hsd_attention_workspace_bytes(int(q_len), int(hq), int(hkv))
    dev = torch.device(device)
    if dev.index is None:
        dev = torch.device("cuda", torch.cuda.current_device())
    s = stream if stream is not None else torch.cuda.current_stream(dev)
    key = (dev.index, int(s.cuda_stream))
    ws = _workspaces.get(key)
    if ws is None or ws.nbytes < need:
        ws = AttentionWorkspace(max(need, 1 << 20), dev, s)
        _workspaces[key] = ws
    return ws


def _as_heads(x, name):
    """[1, H, S, D] or [H, S, D] -> [H, S, D] view (strides kept)."""
    if x.dim() == 4:
        if x.shape[0] != 1:
            raise ValueError(f"{name}: batch must be 1 (packed verification)")
        x = x[0]
    if x.dim() != 3:
        raise ValueError(f"{name}: expected [1, H, S, D] or [H, S, D], got {tuple(x.shape)}")
    if x.dtype != torch.bfloat16:
        raise TypeError(f"{name}: bf16 required, got {x.dtype}")
    if x.stride(-1) != 1:
        x = x.contiguous()
    return x


def verify_attention(q, k, v, plan: TilePlan, scale=None, out=None, lse=None,
                     need_lse=True, stream=None, balanced=True):
    """Masked GQA attention over a tile plan.

    q: ``[Hq, Q, 128]`` (or ``[1, Hq, Q, 128]``) bf16, any row/head strides;
    k, v: ``[Hkv, KV, 128]`` likewise.  Returns ``(out [Q, Hq, 128] bf16,
    lse [Hq, Q] fp32 natural log or None)``.  ``balanced`` selects the
    stream-K schedule (equal work per SM through the workspace cached for
    this device and ``stream``; calls on one stream are ordered, calls on
    different streams get different workspaces); otherwise every (query
    tile, head pair) gets its own CTA.
    """
    lib = N.load()
    q = _as_heads(q, "query")
    k = _as_heads(k, "key")
    v = _as_heads(v, "value")
    hq, q_len, d = q.shape
    hkv, kv_len = k.shape[0], k.shape[1]
    if scale is None:
        scale = 1.0 / math.sqrt(d)
    if out is None:
        out = torch.empty((q_len, hq, d), dtype=torch.bfloat16, device=q.device)
    if need_lse and lse is None:
        lse = torch.empty((hq, q_len), dtype=torch.float32, device=q.device)
    ws_ptr, ws_bytes = None, 0
    if balanced:
        ws = attention_workspace(q_len, hq, hkv, q.device, stream)
        ws_ptr, ws_bytes = ctypes.c_void_p(ws.base), ws.nbytes
    N.check(lib.hsd_verify_attention(
        N.ptr(q), q.stride(1), q.stride(0), N.ptr(k), k.stride(1), k.stride(0),
        N.ptr(v), v.stride(1), v.stride(0), N.ptr(out), N.ptr(lse) if need_lse else None,
        q_len, kv_len, hq, hkv, d, float(scale), ctypes.byref(plan.struct), ws_ptr, ws_bytes,
        N.ptr(plan.status), N.stream_handle(stream)), "hsd_verify_attention")
    return out, lse


def plan_for(attention_mask, q_len, kv_len):
    """Tile plan for whatever mask object the caller passed.

    A dense mask tensor is converted once and the plan reused while the same
    tensor object comes back (every layer of one step), as D:83-106 reuses
    its BlockMask; like there, a mask changed in place between calls keeps
    its old plan, so pass a new tensor (or a PackedMask) for a new step."""
    if isinstance(attention_mask, TilePlan):
        return attention_mask
    if isinstance(attention_mask, PackedMask):
        return attention_mask.plan()
    if isinstance(attention_mask, torch.Tensor):
        if _cache["src"] is attention_mask and _cache["plan"] is not None \
                and _cache["plan"].kv_len == kv_len:
            return _cache["plan"]
        plan = plan_from_dense(attention_mask[..., :kv_len], kv_len)
        _cache["src"], _cache["plan"] = attention_mask, plan
        return plan
    raise TypeError(f"unsupported attention_mask type {type(attention_mask)!r}")


def flex_attention_forward(module, query, key, value, attention_mask, scaling=None,
                           softcap=None, head_mask=None, **kwargs):
    """Drop-in for the reference's ``flex_attention_forward``.

    Returns ``(attn_output [1, Q, Hq, D] contiguous, lse [1, Hq, Q])`` in the
    value dtype like D:131-135.  The kernel computes in bf16 (fp32
    accumulation): fp32 / fp16 models get their q, k, v cast to bf16 and the
    output cast back.  ``softcap`` and ``head_mask`` are not used by the
    reference's FlexAttention call either (D:118-130).
    """
    if attention_mask is None:
        raise ValueError("packed verification needs a mask (dense, PackedMask or TilePlan)")
    q_len, kv_len = query.shape[-2], key.shape[-2]
    plan = plan_for(attention_mask, q_len, kv_len)
    dtype = value.dtype
    if dtype != torch.bfloat16:
        query, key, value = (t.to(torch.bfloat16) for t in (query, key, value))
    out, lse = verify_attention(query, key, value, plan, scale=scaling)
    return out.to(dtype).unsqueeze(0), lse.to(dtype).unsqueeze(0)


# ---------------------------------------------------------------- transformers
ATTENTION_NAME = "hsd_b200"
_step = {"mask": None}


@contextlib.contextmanager
def step_attention_mask(mask):
    """Within the block, attention calls that receive no mask use ``mask``
    (a :class:`PackedMask` or :class:`TilePlan`).  transformers drops a mask
    object it cannot prepare for a custom attention implementation, so the
    verification loop hands each step's mask to the decoder layers this way;
    every layer of the step then reuses the one tile plan."""
    prev = _step["mask"]
    _step["mask"] = mask
    try:
        yield
    finally:
        _step["mask"] = prev


def transformers_attention(module, query, key, value, attention_mask, scaling=None,
                           dropout=0.0, **kwargs):
    """The attention callable registered with transformers' AttentionInterface
    under :data:`ATTENTION_NAME` (the role of D:378-381): the packed
    verification attention over the mask given, or the step's mask of
    :func:`step_attention_mask` when transformers passes none."""
    mask = attention_mask if attention_mask is not None else _step["mask"]
    return flex_attention_forward(module, query, key, value, mask, scaling)


def register_transformers_attention():
    """Register :func:`transformers_attention` as ``"hsd_b200"``; returns the name."""
    from transformers import AttentionInterface
    AttentionInterface.register(ATTENTION_NAME, transformers_attention)
    return ATTENTION_NAME

"""Acceptance + KMP re-alignment (host side of subsystem 3).

One kernel launch per verification step handles every packed block with one
warp each: the reference's per-block Python loop body
(hsd/dots_ocr_pipeline/modeling_dots_ocr_hsd.py D:1103-1336) at the default
exact-match thresholds, and with ``logits`` the logit-ratio rules below them
(HSD_SPEC_THRESH / HSD_TREE_THRESH < 1, D:1147-1174, D:1228-1266).  Block
state lives in an int32 tensor with the field order of ``hsd_block_t``;
results come back as ``hsd_block_result_t`` rows.
"""
from __future__ import annotations

import ctypes as C

import torch

from . import _native as N

BLOCK_FIELDS = [f for f, _ in N.Block._fields_]
RESULT_FIELDS = [f for f, _ in N.BlockResult._fields_]
F = {name: i for i, name in enumerate(BLOCK_FIELDS)}
R = {name: i for i, name in enumerate(RESULT_FIELDS)}

DOTS_SENTINEL = 20993     # D:1306
HUNYUAN_SENTINEL = 41153  # H:1873
FLAG_PAGE_BLOCK = 1       # hsd_block_t.flags: no repetition stop, no token KMP
FLAG_TEXT_MODE = 2        # parser.text_mode (D:1229): tree logit-ratio fallback on


def make_config(n_blocks, kv_len, q_len, words_stride, eos_ids, match_window_size=3,
                match_window_size_upper_bound=10, max_spec_len=0,
                repeat_sentinel=DOTS_SENTINEL):
    cfg = N.AcceptConfig()
    cfg.n_blocks = n_blocks
    cfg.kv_len = kv_len
    cfg.kv_base = kv_len - q_len
    cfg.kv_words_stride = words_stride
    cfg.match_window_size = match_window_size
    cfg.match_window_size_upper_bound = match_window_size_upper_bound
    cfg.max_spec_len = max_spec_len
    cfg.repeat_sentinel = repeat_sentinel
    eos = list(eos_ids)
    if len(eos) > 8:
        raise ValueError("at most 8 EOS ids")
    cfg.n_eos = len(eos)
    for i, e in enumerate(eos):
        cfg.eos_ids[i] = int(e)
    return cfg


def accept_kmp(cfg, blocks, next_ids, input_ids, gen_pool, draft_pool, seg_kv_bits,
               out_kv_bits, filter_bits, tree_tokens=None, tree_parents=None, results=None,
               status=None, stream=None, logits=None, variant="dots",
               formula_tokens=(3, 1099), spec_mode="fmst", spec_topk=3, spec_margin=2.0,
               rank=None, second=None):
    """Launch the acceptance kernel; all tensors are device int32 / int64.

    ``blocks``: int32 ``[n_blocks, 16]`` (updated in place);
    returns ``results`` int32 ``[n_blocks, 8]``.  ``logits = (max_logit,
    probe_logit, spec_thresh, tree_thresh)`` (float32 ``[Q]`` tensors, see
    ``hsd_accept_logits_t``) turns on the logit-ratio rules for thresholds
    below 1; ``variant="hunyuan"`` selects the HunYuan pipeline's rules
    (H:1653-1858) with its formula delimiters ``formula_tokens`` and its
    ``spec_mode`` (SPEC_MODE "fmst", "topk" or "adaptive", H:1668-1743):
    "topk" reads ``rank`` (int32 ``[Q]``) and ``spec_topk``, "adaptive"
    ``second`` (float32 ``[Q]``) and ``spec_margin``
    (:func:`hsd_b200.lm_head.lm_head_rank` computes both).
    """
    lib = N.load()
    if results is None:
        results = torch.empty((blocks.shape[0], len(RESULT_FIELDS)), dtype=torch.int32,
                              device=blocks.device)
    dummy = None
    if tree_tokens is None or tree_parents is None:
        dummy = torch.zeros(1, dtype=torch.int32, device=blocks.device)
    args = (C.byref(cfg), N.ptr(blocks), N.ptr(results), N.ptr(next_ids), N.ptr(input_ids),
            N.ptr(gen_pool), N.ptr(draft_pool),
            N.ptr(tree_tokens if tree_tokens is not None else dummy),
            N.ptr(tree_parents if tree_parents is not None else dummy), N.ptr(seg_kv_bits),
            N.ptr(out_kv_bits), N.ptr(filter_bits))
    if logits is None:
        N.check(lib.hsd_accept_kmp(*args, N.ptr(status), N.stream_handle(stream)),
                "hsd_accept_kmp")
        return results
    max_logit, probe_logit, spec_thresh, tree_thresh = logits
    for t in (max_logit, probe_logit):
        if t is not None and (t.dtype != torch.float32 or not t.is_contiguous()
                              or t.numel() < input_ids.numel()):
            raise ValueError("max_logit / probe_logit: contiguous float32, one per packed row")
    if variant not in ("dots", "hunyuan"):
        raise ValueError(f"variant must be 'dots' or 'hunyuan', not {variant!r}")
    if spec_mode not in N.SPEC_MODES:
        raise ValueError(f"spec_mode must be one of {sorted(N.SPEC_MODES)}, not {spec_mode!r}")
    for t, dt, need in ((rank, torch.int32, spec_mode == "topk"),
                        (second, torch.float32, spec_mode == "adaptive")):
        if variant == "hunyuan" and need and (t is None or t.dtype != dt or not t.is_contiguous()
                                              or t.numel() < input_ids.numel()):
            raise ValueError(f"spec_mode {spec_mode!r}: rank (int32) / second (float32), "
                             "contiguous, one per packed row")
    lg = N.AcceptLogits(N.ptr(max_logit), N.ptr(probe_logit), float(spec_thresh),
                        float(tree_thresh),
                        N.HSD_ACCEPT_HUNYUAN if variant == "hunyuan" else N.HSD_ACCEPT_DOTS,
                        (C.c_int32 * 2)(*[int(t) for t in formula_tokens]),
                        N.SPEC_MODES[spec_mode], int(spec_topk), float(spec_margin),
                        N.ptr(rank) if rank is not None else None,
                        N.ptr(second) if second is not None else None)
    N.check(lib.hsd_accept_kmp_logits(*args, C.byref(lg), N.ptr(status),
                                      N.stream_handle(stream)), "hsd_accept_kmp_logits")
    return results

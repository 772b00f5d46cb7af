"""``batch_generate`` with the reference's call surface, on this package.

Drop-in for ``DotsOCRForCausalLM.batch_generate``
(hsd/dots_ocr_pipeline/modeling_dots_ocr_hsd.py D:923-1810): the same
signature, keyword arguments (``eos_token_id`` and ``max_new_tokens`` in
``**kwargs``, D:953-956), environment switches (HSD_TIGHT_PACK,
HSD_COMPACT_PERIOD, HSD_MAX_SPEC_LEN, HSD_MAX_TREE_LEN, HSD_TREE_THRESH,
HSD_SPEC_THRESH, HSD_MATCH_WINDOW, D:50-62, D:970-975) and return value
``(generated_tokens, decode_times, (forward_s, outside_forward_s,
surround_s, prepare_s, first_forward_s, compaction_s, compaction_calls,
compactions_skipped))`` (D:1801-1810).  A maintainer rebinds it::

    from hsd_b200.generate import batch_generate
    DotsOCRForCausalLM.batch_generate = batch_generate

What changes underneath, per step:

* the mask never exists as a dense ``[1, 1, Q, KV]`` float tensor after the
  caller's prefill: a :class:`~hsd_b200.plan.PackedMask` of segment
  descriptors whose tile plan the decoder layers share
  (:func:`hsd_b200.attention.step_attention_mask`);
* acceptance, stop rules and KMP re-alignment of every block run in one
  kernel, the region blocks' continuation trees in another, keep indices and
  the in-place compaction of the model's own KV cache in two more
  (:class:`~hsd_b200.loop.VerifyLoop`);
* the page block (the last one) follows its layout-JSON parser on the host
  (:mod:`hsd_b200.page_block`) while the device builds the other blocks'
  trees.

``self`` must provide ``forward(input_ids=, attention_mask=, position_ids=,
past_key_values=, use_cache=)`` returning ``.logits`` ``[1, Q, V]`` and
``.past_key_values`` (a transformers cache: ``.layers[i].keys / .values`` or
``.key_cache / .value_cache``, each ``[1, H, KV, D]`` with contiguous rows),
and ``self.model.config`` whose ``_attn_implementation`` is switched to
``"hsd_b200"`` during the call, as the reference switches it to
``flex_attention`` (D:948-949).  The page block's candidate trees use
``pre_tokenizer=`` (keyword) or else ``tokenizer``; the reference loads the
same tokenizer again from the model files for them (D:625-645).

``fused_lm_head=True`` (keyword): after the prefill, each step runs the
decoder alone (``self.model``, which must return ``last_hidden_state`` and
``past_key_values``) and takes the next tokens from
:func:`hsd_b200.lm_head.lm_head_argmax` over ``self.lm_head.weight``, so the
``[Q, vocab]`` logits of D:1060 are never written; the logits the ratio
rules read come from :func:`hsd_b200.lm_head.probe_logits`.
"""
from __future__ import annotations

import os
import time

import numpy as np
import torch

from .attention import register_transformers_attention, step_attention_mask
from .compaction import compact_kv
from .lm_head import lm_head_argmax, probe_logits
from .loop import VerifyLoop
from .page_block import PageBlock, halfwidth_clean


def _env_int(name, default):
    return int(os.environ.get(name, str(default)))


def _env_float(name, default):
    return float(os.environ.get(name, str(default)))


def _cache_tensors(cache):
    """``(tensors, setter)``: every layer's keys and values of a transformers
    cache, and a function that replaces them (after compaction)."""
    if hasattr(cache, "layers"):
        layers = [lay for lay in cache.layers
                  if getattr(lay, "keys", None) is not None and lay.keys.numel()]
        tensors = [t for lay in layers for t in (lay.keys, lay.values)]

        def setter(new):
            for i, lay in enumerate(layers):
                lay.keys, lay.values = new[2 * i], new[2 * i + 1]
        return tensors, setter
    if hasattr(cache, "key_cache"):
        idx = [i for i in range(len(cache.key_cache)) if cache.key_cache[i].numel()]
        tensors = [t for i in idx for t in (cache.key_cache[i], cache.value_cache[i])]

        def setter(new):
            for j, i in enumerate(idx):
                cache.key_cache[i], cache.value_cache[i] = new[2 * j], new[2 * j + 1]
        return tensors, setter
    raise TypeError(f"unsupported cache type {type(cache)!r}")


def compact_model_cache(cache, keep_idx, counts, n_keep, status=None):
    """In-place compaction of every layer's keys and values of ``cache`` to
    the columns ``keep_idx`` (ascending, ``n_keep`` of them): one launch for
    all layers, K and V and heads (what D:1704-1722 does with one
    ``index_select`` per layer and tensor), then the tensors are narrowed to
    ``n_keep`` rows."""
    tensors, setter = _cache_tensors(cache)
    if not tensors:
        return
    row_bytes = tensors[0].shape[-1] * tensors[0].element_size()
    planes = []
    for t in tensors:
        if (t.dim() != 4 or t.shape[0] != 1 or t.stride(-1) != 1
                or t.stride(-2) != t.shape[-1]
                or t.shape[-1] * t.element_size() != row_bytes):
            raise ValueError("cache tensors must be [1, H, KV, D] with contiguous rows of one size")
        planes += [t[0, h].data_ptr() for h in range(t.shape[1])]
    d_planes = torch.tensor(planes, dtype=torch.int64, device=tensors[0].device)
    compact_kv(d_planes, row_bytes, keep_idx, counts=counts, status=status)
    setter([t[:, :, :n_keep] for t in tensors])


def _inherited_rows(attention_mask, pointer, kv_words):
    """Per block, the columns its pointer row of the caller's prefill mask
    sees outside the block's own rows (packed u64 words, int64 on the
    device): the visibility the block's next rows inherit (D:1634-1667)."""
    m = attention_mask
    while m.dim() > 2:
        m = m[0]
    dev = m.device
    ptr = pointer.to(device=dev, dtype=torch.long).reshape(-1)
    rows = m.index_select(0, ptr) > -0.1
    ends = ptr + 1
    starts = torch.cat([torch.zeros(1, dtype=torch.long, device=dev), ends[:-1]])
    col = torch.arange(rows.shape[1], device=dev)
    own = (col[None] >= starts[:, None]) & (col[None] < ends[:, None])
    rows = rows & ~own
    pad = kv_words * 64 - rows.shape[1]
    if pad > 0:
        rows = torch.cat([rows, torch.zeros((rows.shape[0], pad), dtype=torch.bool,
                                            device=dev)], 1)
    bits = rows[:, :kv_words * 64].reshape(rows.shape[0], kv_words, 64).long()
    weights = torch.ones(64, dtype=torch.long, device=dev) << torch.arange(64, device=dev)
    return (bits * weights).sum(-1)   # disjoint bits: the sum wraps to the bit pattern


@torch.no_grad()
def batch_generate(self, input_ids, inputs_embeds=None, pixel_values=None, image_grid_thw=None,
                   attention_mask=None, position_ids=None, pointer=None, use_cache=True,
                   match_window_size=3, match_window_size_upper_bound=10, max_tree_depth=15,
                   max_tree_len=256, min_input_length=128, max_input_length=128,
                   tokenizer=None, draft=None, enable_tree_decode=False, generation_config=None,
                   **kwargs):
    """``DotsOCRForCausalLM.batch_generate`` (D:923-1810) on the package's
    kernels; see the module docstring for the contract."""
    t_surround = time.time()
    config = getattr(getattr(self, "model", None), "config", None)
    original_impl = getattr(config, "_attn_implementation", None)
    if config is not None:
        config._attn_implementation = register_transformers_attention()
    try:
        return _run(self, input_ids, pixel_values, image_grid_thw, attention_mask,
                    position_ids, pointer, use_cache, match_window_size,
                    match_window_size_upper_bound, max_tree_depth, max_tree_len,
                    min_input_length, tokenizer, draft, enable_tree_decode, kwargs, t_surround)
    finally:
        if config is not None:
            config._attn_implementation = original_impl


def _run(self, input_ids, pixel_values, image_grid_thw, attention_mask, position_ids, pointer,
         use_cache, match_window_size, mws_ub, max_tree_depth, max_tree_len, min_input_length,
         tokenizer, draft, enable_tree_decode, kwargs, t_surround):
    tree_len_env = _env_int("HSD_MAX_TREE_LEN", 0)
    if tree_len_env > 0:
        max_tree_len = tree_len_env
    eos_token_id = kwargs.get("eos_token_id", None)
    max_new_tokens = kwargs.get("max_new_tokens", None)
    assert eos_token_id is not None, "eos_token_id must be provided for speculative generation."
    assert max_new_tokens is not None, \
        "max_new_tokens must be provided for speculative generation."
    eos = list(eos_token_id) if isinstance(eos_token_id, (list, tuple)) else [int(eos_token_id)]
    pre_tokenizer = kwargs.get("pre_tokenizer", None)
    fused = bool(kwargs.get("fused_lm_head", False))
    # the raw block content is tokenized so that tokens match the model's output (D:958-964)
    draft_raw = [item.get("raw_block_content", item["block_content"]) for item in draft]
    norm_draft = [halfwidth_clean(item["block_content"]) for item in draft]
    tokenized = [tokenizer.encode(r, add_special_tokens=False) for r in draft_raw]
    pad = tokenizer.pad_token_id
    tree_thresh = _env_float("HSD_TREE_THRESH", 1.0)
    spec_thresh = _env_float("HSD_SPEC_THRESH", 1.0)
    mw = _env_int("HSD_MATCH_WINDOW", 0)
    if mw > 0:
        match_window_size = mw
    tight = os.environ.get("HSD_TIGHT_PACK", "0") == "1"
    period = _env_int("HSD_COMPACT_PERIOD", 3)
    max_spec = _env_int("HSD_MAX_SPEC_LEN", 0)

    dev = input_ids.device
    nb = int(pointer.numel())
    drafts = [tokenized[b] if b < len(tokenized) else [] for b in range(nb - 1)] + [[]]
    ids_host = input_ids[0].cpu().numpy()
    pos_host = position_ids[0].cpu().numpy()
    ptr_host = pointer.reshape(-1).cpu().numpy()

    cache = {"kv": None}

    def hook(keep_idx, counts, n_keep):
        compact_model_cache(cache["kv"], keep_idx, counts, n_keep, status=loop.status)

    loop = VerifyLoop(None, drafts, eos_token_id=eos, max_new_tokens=int(max_new_tokens),
                      pad_token_id=pad, match_window_size=match_window_size,
                      match_window_size_upper_bound=mws_ub, min_input_length=min_input_length,
                      max_spec_len=max_spec, compact_period=period,
                      enable_tree_decode=enable_tree_decode, tight_pack=tight,
                      max_tree_depth=max_tree_depth, max_tree_len=max_tree_len,
                      spec_thresh=spec_thresh, tree_thresh=tree_thresh,
                      packed=(ids_host, pos_host, ptr_host, None), page_block=True,
                      pad_rows_inherit=True, compact_hook=hook, track_kv_tokens=False,
                      device=dev)
    loop.seg_bits[:] = 0
    vis = _inherited_rows(attention_mask, pointer, min(loop.stride, (ids_host.size + 63) // 64))
    loop.seg_bits[:, :vis.shape[1]] = vis
    page = PageBlock(tokenizer, pre_tokenizer, max_tree_depth=max_tree_depth,
                     tree_cap=max_tree_len, min_input_length=min_input_length,
                     tight_pack=tight, max_spec_len=max_spec,
                     enable_tree_decode=enable_tree_decode,
                     match_window_size_upper_bound=mws_ub, norm_draft=norm_draft)

    def others():
        gen = loop.generated()
        fin = loop.step_finished
        return gen[:-1], fin[:-1]

    def page_next(lp, gen, increment, mws, pos_base, next_token):
        return page.next_input(gen, increment, mws, pos_base, others, None, next_token)

    model_inputs = dict(input_ids=input_ids, pixel_values=pixel_values,
                        image_grid_thw=image_grid_thw, attention_mask=attention_mask,
                        position_ids=position_ids, use_cache=use_cache)
    t_surround = time.time() - t_surround
    t_fwd = t_out = first = 0.0
    decode_times = 0
    mask = attention_mask
    while True:
        decode_times += 1
        t0 = time.time()
        hidden = None
        with step_attention_mask(None if isinstance(mask, torch.Tensor) else mask):
            if fused and decode_times > 1:
                # the decoder alone: the lm_head GEMM and argmax are one kernel below
                dec = self.model(**model_inputs)
                hidden = dec.last_hidden_state[0]
                outputs = dec
            else:
                outputs = self.forward(**model_inputs)
        cache["kv"] = outputs.past_key_values
        if hidden is not None:
            weight = self.lm_head.weight
            max_l = torch.empty(hidden.shape[0], dtype=torch.float32, device=dev)
            next_ids = lm_head_argmax(hidden, weight, max_logit=max_l)
        else:
            logits = outputs.logits[0]
            next_ids = logits.argmax(dim=-1)
        torch.cuda.synchronize(dev)
        t1 = time.time()
        t_fwd += t1 - t0
        if decode_times == 1:
            first = t1 - t0
        extra = {}
        if loop.ratio:
            rows, toks = loop.logit_probes()
            if hidden is not None:
                probe = probe_logits(hidden, weight, rows, toks)
                extra = dict(max_logit=max_l, probe_logit=probe)
            else:
                probe = logits[rows.long(), toks.clamp(min=0).long()].float()
                probe = torch.where(toks >= 0, probe, torch.zeros_like(probe))
                extra = dict(max_logit=logits.gather(1, next_ids[:, None])[:, 0].float(),
                             probe_logit=probe)
        more = loop.step(next_ids, text_mode=[page.parser.text_mode] * nb,
                         page_next=page_next, **extra)
        if not more:
            t_out += time.time() - t1
            break
        ids, pos, mask = loop.inputs()
        model_inputs = dict(input_ids=ids[None].long(), attention_mask=mask,
                            position_ids=pos[None], past_key_values=cache["kv"],
                            use_cache=use_cache)
        t_out += time.time() - t1
    generated = loop.generated()
    return generated, decode_times, (t_fwd, t_out, t_surround, 0.0, first, loop.compaction_s,
                                     loop.compaction_calls, loop.compactions_skipped)


def _rank_and_second(logits, rows, toks, top):
    """Per packed row r with ``toks[r] >= 0``: the draft token's 0-based rank
    among the row's logits (lower columns first among equal values) and the
    best logit outside the row's argmax column -- what HunYuan's SPEC_MODE
    topk / adaptive read from ``logits.topk`` (H:1712-1736)."""
    q = logits.shape[0]
    tok = toks.clamp(min=0).long()
    thr = logits[torch.arange(q, device=logits.device), tok]
    col = torch.arange(logits.shape[1], device=logits.device)
    above = (logits > thr[:, None]) | ((logits == thr[:, None]) & (col[None] < tok[:, None]))
    rank = above.sum(-1).to(torch.int32)
    masked = logits.clone()
    masked[torch.arange(q, device=logits.device), top] = float("-inf")
    return rank, masked.max(-1).values.float()


@torch.no_grad()
def batch_generate_hunyuan(self, input_ids=None, attention_mask=None, position_ids=None,
                           imgs=None, imgs_pos=None, token_type_ids=None, pixel_values=None,
                           image_grid_thw=None, pointer=None,
                           match_window_size=int(os.environ.get("MATCH_WINDOW_SIZE", "3")),
                           match_window_size_upper_bound=10, max_tree_depth=15,
                           max_tree_len=128, min_input_length=128, max_input_length=128,
                           tokenizer=None, draft=None, enable_tree_decode=False, **kwargs):
    """Drop-in for the HunYuan pipeline's ``batch_generate``
    (hsd/hunyuan_ocr_pipeline/modeling_hunyuan_vl_hsd.py H:1426-1448), on the
    package's kernels.  Its differences from the dots loop are kept: the
    acceptance rules of H:1653-1858 (``variant="hunyuan"``: the logit ratio
    below SPEC_THRESH on the last block only, outside formulas, accepted rows
    keeping the model's tokens, SPEC_MODE fmst / topk / adaptive), the
    repetition sentinel 41153, the page block's text rule
    (:class:`~hsd_b200.page_block.HunyuanPageBlock`), drafts tokenized from
    their half-width form, no speculative length cap, period 0 compacting,
    tight-padding rows masked (H:2290-2293), the stop on the page block's own
    length (H:2133), the ``[1, 4, Q]`` position ids of every step (the xdrope
    rows, all equal for generated tokens, H:2033, H:2100, H:2128) and the
    returned dict (H:2324-2343).  The first forward embeds the tokens and the
    images as H:1481-1494 does when the model has ``model.embed_tokens``."""
    t0_all = time.time()
    config = getattr(getattr(self, "model", None), "config", None)
    original_impl = getattr(config, "_attn_implementation", None)
    if config is not None:
        config._attn_implementation = register_transformers_attention()
    try:
        return _run_hunyuan(self, input_ids, attention_mask, position_ids, pixel_values,
                            image_grid_thw, pointer, match_window_size,
                            match_window_size_upper_bound, max_tree_depth, max_tree_len,
                            min_input_length, tokenizer, draft, enable_tree_decode, kwargs,
                            t0_all)
    finally:
        if config is not None:
            config._attn_implementation = original_impl


def _run_hunyuan(self, input_ids, attention_mask, position_ids, pixel_values, image_grid_thw,
                 pointer, match_window_size, mws_ub, max_tree_depth, max_tree_len,
                 min_input_length, tokenizer, draft, enable_tree_decode, kwargs, t0_all):
    from .page_block import HunyuanPageBlock

    eos_token_id = kwargs.get("eos_token_id", None)
    max_new_tokens = kwargs.get("max_new_tokens", None)
    assert eos_token_id is not None, "eos_token_id must be provided for speculative generation."
    assert max_new_tokens is not None, \
        "max_new_tokens must be provided for speculative generation."
    eos = list(eos_token_id) if isinstance(eos_token_id, (list, tuple)) else [int(eos_token_id)]
    content = [item["block_content"] for item in draft]
    norm_draft = [halfwidth_clean(c) for c in content]
    tokenized = [tokenizer.encode(d, add_special_tokens=False) for d in norm_draft]
    pad = tokenizer.pad_token_id
    spec_thresh = _env_float("SPEC_THRESH", 1.0)
    spec_mode = os.environ.get("SPEC_MODE", "fmst")
    spec_topk = _env_int("SPEC_TOPK", 3)
    spec_margin = _env_float("SPEC_MARGIN", 2.0)
    tight = os.environ.get("HSD_TIGHT_PACK", "0") == "1"
    period = _env_int("HSD_COMPACT_PERIOD", 3)

    dev = input_ids.device
    nb = int(pointer.numel())
    drafts = [tokenized[b] if b < len(tokenized) else [] for b in range(nb - 1)] + [[]]
    pos_rows = position_ids[0] if position_ids.dim() == 3 else position_ids
    ids_host = input_ids[0].cpu().numpy()
    pos_host = pos_rows[0].cpu().numpy()
    ptr_host = pointer.reshape(-1).cpu().numpy()
    cache = {"kv": None}

    def hook(keep_idx, counts, n_keep):
        compact_model_cache(cache["kv"], keep_idx, counts, n_keep, status=loop.status)

    loop = VerifyLoop(None, drafts, eos_token_id=eos, max_new_tokens=int(max_new_tokens),
                      pad_token_id=pad, match_window_size=match_window_size,
                      match_window_size_upper_bound=mws_ub, min_input_length=min_input_length,
                      max_spec_len=0, compact_period=period,
                      enable_tree_decode=enable_tree_decode, tight_pack=tight,
                      max_tree_depth=max_tree_depth, max_tree_len=max_tree_len,
                      repeat_sentinel=41153, spec_thresh=spec_thresh, tree_thresh=1.0,
                      variant="hunyuan", spec_mode=spec_mode, spec_topk=spec_topk,
                      spec_margin=spec_margin, packed=(ids_host, pos_host, ptr_host, None),
                      page_block=True, pad_rows_inherit=False, compact_hook=hook, track_kv_tokens=False,
                      device=dev)
    loop.seg_bits[:] = 0
    vis = _inherited_rows(attention_mask, pointer, min(loop.stride, (ids_host.size + 63) // 64))
    loop.seg_bits[:, :vis.shape[1]] = vis
    page = HunyuanPageBlock(tokenizer, max_tree_depth=max_tree_depth, tree_cap=max_tree_len,
                            min_input_length=min_input_length, tight_pack=tight,
                            enable_tree_decode=enable_tree_decode,
                            match_window_size_upper_bound=mws_ub, norm_draft=norm_draft)

    def others():
        gen = loop.generated()
        return gen[:-1], loop.step_finished[:-1]

    def page_next(lp, gen, increment, mws, pos_base, next_token):
        return page.next_input(gen, increment, mws, pos_base, others, None, next_token)

    t_prefill0 = time.time()
    embed = getattr(getattr(self, "model", None), "embed_tokens", None)
    if embed is not None:
        inputs_embeds = embed(input_ids)
        vit = getattr(self, "vit", None)
        if vit is not None and pixel_values is not None:
            image_embeds = vit(pixel_values.to(torch.bfloat16), image_grid_thw).to(dev)
            image_mask, _ = self.get_placeholder_mask(input_ids, inputs_embeds=inputs_embeds,
                                                      image_features=image_embeds)
            inputs_embeds = inputs_embeds.masked_scatter(image_mask, image_embeds)
        model_inputs = dict(inputs_embeds=inputs_embeds, attention_mask=attention_mask,
                            position_ids=position_ids, use_cache=True)
    else:
        model_inputs = dict(input_ids=input_ids, attention_mask=attention_mask,
                            position_ids=position_ids, use_cache=True)
    prefill = time.time() - t_prefill0
    surround = time.time() - t0_all - prefill
    t_fwd = t_out = 0.0
    decode_times = 0
    intensity = []
    mask = attention_mask
    while True:
        decode_times += 1
        t0 = time.time()
        with step_attention_mask(None if isinstance(mask, torch.Tensor) else mask):
            outputs = self.forward(**model_inputs)
        cache["kv"] = outputs.past_key_values
        logits = outputs.logits[0]
        next_ids = logits.argmax(dim=-1)
        torch.cuda.synchronize(dev)
        t1 = time.time()
        t_fwd += t1 - t0
        if decode_times == 1:
            prefill += t1 - t0
        intensity.append((int(logits.shape[0]), int(logits.shape[0]), int(loop.kv_len), 0.0))
        extra = {}
        if loop.ratio:
            rows, toks = loop.logit_probes()
            probe = logits[rows.long(), toks.clamp(min=0).long()].float()
            probe = torch.where(toks >= 0, probe, torch.zeros_like(probe))
            extra = dict(max_logit=logits.gather(1, next_ids[:, None])[:, 0].float(),
                         probe_logit=probe)
            if spec_mode != "fmst":
                nxt_in = torch.roll(torch.as_tensor(loop.input_ids, device=dev), -1)
                rank, second = _rank_and_second(logits.float(), rows, nxt_in, next_ids)
                extra.update(rank=rank, second=second)
        # the HunYuan parser is never fed: no block is ever in text mode (H:1792)
        more = loop.step(next_ids, text_mode=[False] * nb, page_next=page_next, **extra)
        if not more:
            t_out += time.time() - t1
            break
        ids, pos, mask = loop.inputs()
        model_inputs = dict(input_ids=ids[None].long(), attention_mask=mask,
                            position_ids=pos[None, None].expand(1, 4, -1),
                            past_key_values=cache["kv"], use_cache=True)
        t_out += time.time() - t1
    generated = loop.generated()
    return {
        "generated_tokens": generated,
        "decode_times": decode_times,
        "decode_token_num": len(generated[-1]),
        "compute_intensity": intensity,
        "used_time": {
            "total_prefill_time": prefill,
            "total_surround_time": surround,
            "total_forward_time": t_fwd,
            "total_outside_forward_time": t_out,
            "phase_verify_loop": t_out - loop.compaction_s,
            "phase_kv_compact": loop.compaction_s,
            "phase_kv_layers": loop.compaction_s,
            "phase_mask_build": 0.0,
            "phase_reindex_mask": 0.0,
            "phase_cat_inputs": 0.0,
            "kv_compact_calls": loop.compaction_calls,
            "kv_compact_skipped": loop.compactions_skipped,
        },
    }

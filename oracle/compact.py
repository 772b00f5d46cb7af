"""KV-cache compaction (test infrastructure only).

Restates the fused compaction of the reference's loop: dots D:1586-1594 and
D:1669-1735, HunYuan H:2147-2151 and H:2225-2285.

``live``  = any over the active blocks' pointer rows of the mask (> -0.1);
``keep``  = live & ~filtered;
physical compaction ``index_select(-2, nonzero(keep))`` on every layer's K
and V (and the mask's columns) when the period rule fires, otherwise the
dead columns are ``masked_fill``-ed with -inf.  Kept rows stay in ascending
original order.
"""
from __future__ import annotations

import numpy as np
import torch


def pad_filter(filt, input_ids, pad_token_id):
    """Pad positions of the current query become filtered (D:1590-1594)."""
    q = len(input_ids)
    filt = filt.copy()
    filt[len(filt) - q:] |= np.asarray(input_ids) == pad_token_id
    return filt


def all_dead_filter(filt, allowed):
    """HunYuan only: columns no row can see are filtered (H:2147-2148)."""
    return filt | ~np.asarray(allowed).any(axis=0)


def keep_columns(allowed, active_pointers, filt):
    """``keep = any(mask[active pointers]) & ~filtered`` (D:1679-1687)."""
    allowed = np.asarray(allowed, dtype=bool)
    if len(active_pointers):
        live = allowed[np.asarray(active_pointers)].any(axis=0)
    else:
        live = np.zeros(allowed.shape[1], dtype=bool)
    return live & ~np.asarray(filt, dtype=bool)


def should_compact(kv_len, n_keep, decode_times, period, hunyuan=False):
    """Period / 20%-dead rule.

    dots (D:1693-1700): period 0 never compacts.  HunYuan (H:2253-2259):
    ``period <= 1`` -- 0 included -- compacts every iteration.
    """
    dead = kv_len - n_keep
    rule = (period <= 1) or (decode_times % period == 0) or (dead > kv_len * 0.2)
    if hunyuan:
        return rule
    return period > 0 and rule


def compaction_action(kv_len, n_keep, decode_times, period, hunyuan=False):
    """'compact' | 'mask' | 'none' as the reference branches (D:1704-1731)."""
    if should_compact(kv_len, n_keep, decode_times, period, hunyuan):
        return "compact" if n_keep < kv_len else "none"
    return "mask"


def keep_indices(keep):
    return np.nonzero(np.asarray(keep, dtype=bool))[0].astype(np.int64)


def compact_layers(layers_k, layers_v, keep_idx):
    """``index_select(-2, keep_idx)`` on every layer (D:1705-1722)."""
    idx = torch.as_tensor(keep_idx, dtype=torch.long)
    return ([k.index_select(-2, idx) for k in layers_k],
            [v.index_select(-2, idx) for v in layers_v])


def apply_to_mask(attention_mask, keep, action):
    """Column update of the dense mask for the chosen action."""
    keep_t = torch.as_tensor(np.asarray(keep, dtype=bool))
    if action == "compact":
        return attention_mask.index_select(-1, torch.nonzero(keep_t)[:, 0])
    if action == "mask":
        return attention_mask.masked_fill(~keep_t[None, None, None, :],
                                          float("-inf"))
    return attention_mask

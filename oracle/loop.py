"""The verification loop of ``batch_generate`` restated on the CPU (test
infrastructure only).

Composes the per-step restatements of this package into the reference's
iteration (hsd/dots_ocr_pipeline/modeling_dots_ocr_hsd.py):

* prefill packing: block-diagonal causal mask over the blocks' prompts,
  ``pointer`` = cumulative ends - 1 (RD:232-245), every block starts in
  ``normal`` mode (D:978-986);
* per iteration: target argmax for every packed row (D:1057-1064), the
  per-block acceptance / stop rules / KMP re-alignment / next input
  (D:1103-1567), the generation-finished test (D:1589-1591), the pad filter
  (D:1596-1599), keep columns and the compaction rule (D:1679-1731), the next
  dense mask (D:1634-1667, D:1737-1748) and the next pointer (D:1604-1606);
  with ``cfg.tight_pack`` (HSD_TIGHT_PACK) blocks are not padded and the
  packed input is padded to a multiple of 128 rows that belong to no block
  (D:1619-1632, D:1640-1644);
* the KV cache grows by the packed input of every forward (DynamicCache) and
  loses the compacted columns.

Without ``page`` every block is a region block; with it the last block is
the page block of :mod:`oracle.page` (its parser-driven candidates,
D:1337-1567, and the "last block finished" stop, D:1591-1592).  ``model(input_ids,
position_ids, allowed, kv_tokens)`` stands for the target forward + argmax:
``allowed`` is the step's [Q, KV] visibility, ``kv_tokens`` the token of
every KV column.
"""
from __future__ import annotations

import numpy as np
import torch

from .accept import (FINISHED, SPEC, TREE, BlockState, accept_block, next_block_input,
                     rank_and_second, realign_block)
from .compact import apply_to_mask, compaction_action, keep_columns, pad_filter
from .masks import (assemble_next_mask, initial_packed_mask, normal_block_mask,
                    spec_block_mask, tree_block_mask)

Q_BLOCK = 128  # _HSD_Q_BLOCK (D:53): tight-packed inputs are padded to a multiple of it


def ratio_logits(logits, next_ids, input_ids, spans, states):
    """``(max_logit, probe_logit)`` per packed row, the logits tensor's
    entries the logit-ratio rules read (D:1163-1168, D:1231-1232,
    D:1259-1260): ``logits[r, next[r]]``; a speculative row's draft token
    ``logits[r, input[r + 1]]``; a tree node's token at its parent's row."""
    q = len(input_ids)
    max_l = logits[np.arange(q), next_ids].astype(np.float32)
    probe = np.zeros(q, dtype=np.float32)
    for (bs, be), st in zip(spans, states):
        if st.mode == SPEC:
            for r in range(bs, be - 1):
                probe[r] = logits[r, input_ids[r + 1]]
        elif st.mode == TREE:
            for c in range(1, len(st.tree_tokens)):
                probe[bs + c] = logits[bs + st.tree_parents[c], st.tree_tokens[c]]
    return max_l, probe


def reference_loop(prompts, drafts, model, cfg, max_new_tokens, compact_period=1,
                   max_iters=1000, logits_model=None, text_mode=(), page=None):
    """Run the loop; returns ``(generated tokens per block, trace)``.

    ``trace`` holds, per iteration, the packed ``input_ids``,
    ``position_ids``, the bool ``allowed`` mask [Q, KV], the KV column ids
    the previous compaction kept (``kept_column_ids``: ids numbered in order
    of appearance), the blocks' modes and the compaction action taken after
    the step.  With ``logits_model`` (same arguments, returns float32 logits
    ``[Q, V]`` of bf16 values) the next tokens are its first argmax per row
    and the logit-ratio rules of ``cfg`` read its entries; ``text_mode``
    holds the blocks whose parser is in text mode.

    ``page`` (an :class:`oracle.page.OraclePage`) makes the last block the
    page block, as in the reference: no repetition stop for it (D:1306),
    its next input from the parser-driven candidates (D:1337-1567), the
    parser's text mode for every block's tree fallback (D:1229, D:1257), and
    the loop ends when it finishes (D:1591-1592).
    """
    nb = len(prompts)
    lens = [len(p) for p in prompts]
    input_ids = np.concatenate([np.asarray(p, dtype=np.int64) for p in prompts])
    position_ids = np.concatenate([np.arange(n, dtype=np.int64) for n in lens])
    mask = initial_packed_mask(lens)
    kv_tokens = input_ids.copy()
    kv_ids = np.arange(len(input_ids), dtype=np.int64)
    next_id = len(input_ids)
    kept_ids = np.zeros(0, dtype=np.int64)
    pointer = [int(x) for x in np.cumsum(lens) - 1]
    states = [BlockState(draft=list(d), mws=cfg.match_window_size) for d in drafts]
    new_tokens = 0
    trace = []
    for decode_times in range(1, max_iters + 1):
        allowed = (mask[0, 0] > -0.1).numpy()
        q = len(input_ids)
        kv = allowed.shape[1]
        logits = None
        if logits_model is not None:
            dense = logits_model(input_ids, position_ids, allowed, kv_tokens)
            next_ids = np.argmax(dense, axis=1).astype(np.int64)
            spans, b0 = [], 0
            for b in range(nb):
                spans.append((b0, pointer[b] + 1))
                b0 = pointer[b] + 1
            logits = ratio_logits(dense, next_ids, input_ids, spans, states)
            if cfg.variant == "hunyuan" and cfg.spec_mode != "fmst":
                # topk / adaptive: the draft token's rank and the second best
                # logit of every speculative row (H:1712-1736)
                rank = np.zeros(q, dtype=np.int32)
                second = np.full(q, -np.inf, dtype=np.float32)
                for r in range(q - 1):
                    rank[r], second[r] = rank_and_second(dense[r], int(input_ids[r + 1]),
                                                         int(next_ids[r]))
                logits = logits + (rank, second)
        else:
            next_ids = np.asarray(model(input_ids, position_ids, allowed, kv_tokens),
                                  dtype=np.int64)
        step = dict(input_ids=input_ids.copy(), position_ids=position_ids.copy(),
                    allowed=allowed.copy(), modes=[st.mode for st in states],
                    kept_column_ids=kept_ids.copy(),
                    q_blocks=pointer[-1] + 1)   # rows owned by blocks (the rest: tight padding)
        trace.append(step)
        kv_base = kv - q
        filt = np.zeros(kv, dtype=bool)
        next_list, input_list = next_ids.tolist(), input_ids.tolist()
        new_ids, new_pos = [], []
        new_lens, new_masks = [0] * nb, [None] * nb
        bs = 0
        for b in range(nb):
            be = pointer[b] + 1
            st = states[b]
            if st.mode == FINISHED:
                bs = be
                continue
            is_page = page is not None and b == nb - 1
            st.text_mode = (page.parser.text_mode if page is not None else b in text_mode)
            ptr, nxt, inc, fin = accept_block(st, bs, be, next_list, input_list, cfg, filt,
                                              kv_base, lambda row: allowed[row], is_page,
                                              logits=logits, is_last_block=(b == nb - 1))
            pointer[b] = ptr
            new_tokens += inc
            bs = be
            if fin:
                continue
            if is_page:                                        # D:1337-1567, last block
                ids, pos, kind, n_valid, n_match, tree = page.next_input(
                    st.gen, inc, st.mws, [x.gen for x in states],
                    [x.mode == FINISHED for x in states], int(position_ids[ptr]) + 1, nxt)
                st.matches_len = n_match
                st.valid_count = n_valid
                st.mode = {"causal": SPEC, "tree": TREE, "single": 0}[kind]
                st.tree_tokens, st.tree_parents = (tree if tree is not None else (None, None))
                n = len(ids)
            else:
                window, matches, trie = realign_block(st, cfg)
                ids, pos, kind, n = next_block_input(st, cfg, window, matches, trie, nxt,
                                                     int(position_ids[ptr]) + 1)
            new_ids.append(ids)
            new_pos.append(pos)
            new_lens[b] = n
            if kind == "causal":
                new_masks[b] = spec_block_mask(n)
            elif kind == "tree":
                new_masks[b] = tree_block_mask(st.tree_parents, n)
            else:
                new_masks[b] = normal_block_mask(n)
        # the HunYuan loop stops on the page block's own length (H:2133)
        produced = (len(states[-1].gen) if cfg.variant == "hunyuan" and page is not None
                    else new_tokens)
        if produced >= max_new_tokens or all(st.mode == FINISHED for st in states) or (
                page is not None and states[-1].mode == FINISHED):
            step["action"] = "stop"
            break
        filt = pad_filter(filt, input_ids, cfg.pad_token_id)
        active = [pointer[b] for b in range(nb) if states[b].mode != FINISHED]
        keep = keep_columns(allowed, active, filt)
        action = compaction_action(kv, int(keep.sum()), decode_times, compact_period,
                                   hunyuan=cfg.variant == "hunyuan")
        step["action"] = action
        mask = apply_to_mask(mask, keep, action)
        if action == "compact":
            kv_tokens = kv_tokens[keep]
            kv_ids = kv_ids[keep]
        # HSD_TIGHT_PACK: the packed input is padded to a multiple of
        # _HSD_Q_BLOCK with pad tokens at position 0 (D:1619-1632)
        pad_n = (-sum(new_lens)) % Q_BLOCK if cfg.tight_pack else 0
        mask = assemble_next_mask(mask, pointer, new_lens, new_masks, tight_pad_len=pad_n,
                                  hunyuan=cfg.variant == "hunyuan")
        if pad_n:
            new_ids.append([cfg.pad_token_id] * pad_n)
            new_pos.append([0] * pad_n)
        input_ids = np.concatenate([np.asarray(x, dtype=np.int64) for x in new_ids])
        position_ids = np.concatenate([np.asarray(x, dtype=np.int64) for x in new_pos])
        kept_ids = kv_ids.copy()
        kv_tokens = np.concatenate([kv_tokens, input_ids])
        kv_ids = np.concatenate([kv_ids, np.arange(next_id, next_id + len(input_ids))])
        next_id += len(input_ids)
        pointer = [int(x) for x in np.cumsum(new_lens) - 1]
    return [list(st.gen) for st in states], trace


def true_text_model(prompts, truths, vocab, eos_id):
    """Deterministic stand-in for the target model's argmax.

    A row's context is the token of every KV column it sees, in column order
    (its own column last).  The block is identified by its prompt (prompts
    are distinct); when the tokens after the prompt match a prefix of the
    block's true text, the model predicts the next true token (EOS past the
    end), otherwise a token hashed from the last four context tokens.  Rows
    that see nothing predict 0.
    """
    heads = {tuple(int(t) for t in p[:4]): b for b, p in enumerate(prompts)}

    def model(input_ids, position_ids, allowed, kv_tokens):
        kv_tokens = np.asarray(kv_tokens, dtype=np.int64)
        out = np.zeros(allowed.shape[0], dtype=np.int64)
        for r in range(allowed.shape[0]):
            ctx = kv_tokens[allowed[r]]
            if len(ctx) == 0:
                continue
            b = heads.get(tuple(int(t) for t in ctx[:4]))
            if b is not None:
                gen = ctx[len(prompts[b]):]
                truth = truths[b]
                if len(gen) <= len(truth) and np.array_equal(gen, truth[:len(gen)]):
                    out[r] = truth[len(gen)] if len(gen) < len(truth) else eos_id
                    continue
            tail = [int(t) for t in ctx[-4:]]
            h = 0
            for t in tail:
                h = (h * 1000003 + t + 1) % 2147483647
            out[r] = 1 + h % (vocab - 1)
        return out

    return model

"""The verification loop of ``batch_generate`` on the device.

Drives the reference's iteration (hsd/dots_ocr_pipeline/modeling_dots_ocr_hsd.py
D:923-1767) for region blocks with the kernels of this package:

* the packed mask of a step is a :class:`~hsd_b200.plan.PackedMask` whose
  per-block visibility rows stay in device memory: the acceptance kernel
  writes each block's row of its last accepted token (the row the
  reference's next mask inherits, D:1634-1667), and after compaction the
  rows are remapped with the keep indices (D:1723);
* acceptance, stop rules and KMP re-alignment run in one launch
  (:func:`hsd_b200.accept.accept_kmp`); only the 8-int result rows of the
  blocks come back to the host, which packs the next input (speculative
  draft slice, or the next token) as D:1421-1567 does;
* keep columns, the compaction rule and in-place compaction of the
  registered KV planes (D:1679-1731).

The target model stays outside: :meth:`VerifyLoop.inputs` gives the packed
``input_ids`` / ``position_ids`` and the step's :class:`PackedMask` (its
tile plan is what :func:`hsd_b200.attention.flex_attention_forward`
consumes), and :meth:`VerifyLoop.step` takes the model's argmax per packed
row.  With ``enable_tree_decode`` a block without exactly one KMP match
proposes its draft's continuation tree (D:1488-1543), built and packed on the
device for all such blocks in one launch (:mod:`hsd_b200.trie`); the tree's
node arrays feed the next acceptance kernel and its ancestor rows the next
mask without a host copy, and only tokens and depths come back to pack the
input.  Below the default thresholds (``spec_thresh`` / ``tree_thresh`` < 1,
HSD_SPEC_THRESH / HSD_TREE_THRESH, D:970-971) the logit-ratio rules apply:
:meth:`VerifyLoop.logit_probes` lists the logits they read, and
:meth:`VerifyLoop.step` takes them with the maximal logit per row.
With ``tight_pack`` (HSD_TIGHT_PACK) blocks are not padded to
``min_input_length`` and the packed input is padded to a multiple of 128
rows.  Not driven by this loop: the page block's tokenizer-driven parsers.
"""
from __future__ import annotations

import math
import time

import numpy as np
import torch

from . import _native as N
from .accept import DOTS_SENTINEL, FLAG_PAGE_BLOCK, FLAG_TEXT_MODE, F, R, accept_kmp, make_config
from .compaction import compact_bits, compact_kv, keep_indices
from .plan import SEG_CAUSAL, SEG_NONE, SEG_SINGLE, SEG_TREE, PackedMask, pack_bits
from .trie import continuation_trees

Q_BLOCK = 128  # _HSD_Q_BLOCK (D:53): tight-packed inputs are padded to a multiple of it


class VerifyLoop:
    """Region blocks verified in parallel, one :meth:`step` per forward.

    ``variant="hunyuan"`` applies the HunYuan pipeline's acceptance and
    compaction rules (H:1653-1858, H:2237-2285) in place of the dots ones.

    ``prompts[b]`` is block b's prefill input (its own prompt: blocks do not
    share KV columns, as in the reference's stage-1 packing, RD:232-245) and
    ``drafts[b]`` its tokenized draft.  ``kv_tokens`` (device int32, one
    token per KV column; ``track_kv_tokens=False`` skips it) is kept
    compacted alongside the mask; pass
    ``kv_planes`` (device int64 plane addresses, see
    :func:`hsd_b200.compaction.plane_pointers`) and ``row_bytes`` to have
    model caches compacted in place too.
    """

    def __init__(self, prompts, drafts, *, eos_token_id, max_new_tokens, pad_token_id=0,
                 match_window_size=3, match_window_size_upper_bound=10, min_input_length=128,
                 max_spec_len=0, compact_period=1, enable_tree_decode=False, tight_pack=False,
                 max_tree_depth=15, max_tree_len=256,
                 repeat_sentinel=DOTS_SENTINEL, kv_planes=None, row_bytes=0,
                 kv_capacity=None, spec_thresh=1.0, tree_thresh=1.0, variant="dots",
                 formula_tokens=(3, 1099), spec_mode="fmst", spec_topk=3, spec_margin=2.0,
                 packed=None, page_block=False, pad_rows_inherit=False, compact_hook=None,
                 track_kv_tokens=True, device="cuda"):
        if packed is not None:
            # the caller's packed prefill: (input_ids, position_ids, pointer)
            p_ids, p_pos, p_ptr = packed[:3]
            p_ids = np.asarray(p_ids, dtype=np.int64).reshape(-1)
            ends = np.asarray(p_ptr, dtype=np.int64).reshape(-1) + 1
            starts = np.concatenate([[0], ends[:-1]])
            prompts = [p_ids[a:b] for a, b in zip(starts, ends)]
        if len(prompts) != len(drafts) or not prompts:
            raise ValueError("one draft per prompt, at least one block")
        self.device = torch.device(device)
        dev = self.device
        self.nb = len(prompts)
        self.pad = int(pad_token_id)
        self.eos = list(eos_token_id) if isinstance(eos_token_id, (list, tuple)) else [
            int(eos_token_id)]
        self.max_new_tokens = int(max_new_tokens)
        self.mws0 = int(match_window_size)
        self.mws_ub = int(match_window_size_upper_bound)
        self.mil = int(min_input_length)
        self.max_spec_len = int(max_spec_len)
        self.tree_decode = bool(enable_tree_decode)
        self.tight = bool(tight_pack)
        self.tree_depth = int(max_tree_depth)
        self.tree_cap = (min(int(max_tree_len), self.max_spec_len) if self.max_spec_len > 0
                         else int(max_tree_len))
        self.period = int(compact_period)
        self.sentinel = int(repeat_sentinel)
        self.spec_thresh, self.tree_thresh = float(spec_thresh), float(tree_thresh)
        if variant not in ("dots", "hunyuan"):
            raise ValueError(f"variant must be 'dots' or 'hunyuan', not {variant!r}")
        self.variant, self.formula_tokens = variant, tuple(int(t) for t in formula_tokens)
        if spec_mode not in N.SPEC_MODES or (spec_mode != "fmst" and variant != "hunyuan"):
            raise ValueError("spec_mode 'topk' / 'adaptive' belong to the HunYuan rules; "
                             f"got {spec_mode!r} with variant {variant!r}")
        self.spec_mode, self.spec_topk = spec_mode, int(spec_topk)
        self.spec_margin = float(spec_margin)
        # HunYuan's tree fallback runs at any threshold in text mode (H:1791)
        self.ratio = (self.spec_thresh < 1.0 or self.tree_thresh < 1.0
                      or (variant == "hunyuan" and self.tree_decode))
        self.kv_planes, self.row_bytes = kv_planes, int(row_bytes)
        self.drafts = [list(map(int, d)) for d in drafts]
        lens = [len(p) for p in prompts]
        if kv_capacity is None:
            longest = max([self.mil] + [len(d) for d in self.drafts])
            kv_capacity = sum(lens) + self.max_new_tokens + 4 * self.nb * longest + 64
        self.kv_cap = int(kv_capacity)
        self.stride = (self.kv_cap + 63) // 64
        cap = self.max_new_tokens + max([len(d) for d in self.drafts] + [0]) + self.mil + 8
        self.gen_cap = cap

        # the last block is the page block: its next input comes from the
        # caller (page_next of step()), no repetition stop, no token KMP
        self.page_block = bool(page_block)
        self.pad_rows_inherit = bool(pad_rows_inherit)
        self.compact_hook = compact_hook
        if self.page_block:
            self.drafts[-1] = []
        self._drafts_np = [np.asarray(d, dtype=np.int64) for d in self.drafts]
        # host state of the current step
        self.input_ids = np.concatenate([np.asarray(p, dtype=np.int64) for p in prompts])
        if packed is not None:
            self.position_ids = np.asarray(packed[1], dtype=np.int64).reshape(-1).copy()
        else:
            self.position_ids = np.concatenate([np.arange(n, dtype=np.int64) for n in lens])
        self.q_start = np.concatenate([[0], np.cumsum(lens)[:-1]]).astype(np.int64)
        self.q_len = np.asarray(lens, dtype=np.int64)
        self.kinds = [SEG_CAUSAL] * self.nb
        self.trees = None                            # device trees of this step's TREE blocks
        self.tree_slot = [-1] * self.nb              # row of block b in self.trees
        self.tree_parents = [None] * self.nb         # host parents of block b's tree
        self.host_tree = [None] * self.nb            # (tokens, parents) of a host-built tree
        self.modes = [N.HSD_MODE_NORMAL] * self.nb   # D:978
        # non-pad rows per block (the reference counts them while
        # block_valid_counts is None, D:1108-1111)
        self.valid = [int(np.count_nonzero(np.asarray(p) != self.pad)) for p in prompts]
        self.kv_len = int(self.input_ids.size)       # the prefill forward fills the cache
        self.decode_times = 0
        self.new_tokens = 0
        self.done = False
        self.compaction_s = 0.0
        self.compaction_calls = 0
        self.compactions_skipped = 0

        # device state
        blocks = np.zeros((self.nb, 16), dtype=np.int32)
        doff = 0
        for b in range(self.nb):
            blocks[b, F["gen_off"]] = b * cap
            blocks[b, F["gen_cap"]] = cap
            blocks[b, F["draft_off"]] = doff
            blocks[b, F["draft_len"]] = len(self.drafts[b])
            blocks[b, F["mws"]] = self.mws0
            blocks[b, F["seg"]] = b
            doff += len(self.drafts[b])
        if self.page_block:
            blocks[self.nb - 1, F["flags"]] = FLAG_PAGE_BLOCK
        self.d_draft_off = torch.from_numpy(blocks[:, F["draft_off"]].copy()).to(dev)
        self.d_draft_len = torch.from_numpy(blocks[:, F["draft_len"]].copy()).to(dev)
        self.blocks = torch.from_numpy(blocks).to(dev)
        self.draft_pool = torch.tensor(sum(self.drafts, []) or [0], dtype=torch.int32, device=dev)
        self.gen_pool = torch.zeros(self.nb * cap, dtype=torch.int32, device=dev)
        self.seg_bits = torch.zeros((self.nb, self.stride), dtype=torch.int64, device=dev)
        self.out_bits = torch.zeros_like(self.seg_bits)
        self.filter = torch.zeros(self.stride, dtype=torch.int64, device=dev)
        self.results = torch.zeros((self.nb, len(R)), dtype=torch.int32, device=dev)
        self.status = torch.zeros(1, dtype=torch.int32, device=dev)
        self.kv_tokens = (torch.from_numpy(self.input_ids.astype(np.int32)).to(dev)
                          if track_kv_tokens else None)
        self.gen_host = [[] for _ in range(self.nb)]
        self._flags = blocks[:, F["flags"]].copy()
        self._upd_cols = torch.tensor([F["mode"], F["q_start"], F["q_len"], F["valid_count"],
                                       F["flags"], F["tree_off"], F["tree_nodes"]],
                                      dtype=torch.long, device=dev)
        self._zero_i32 = torch.zeros(1, dtype=torch.int32, device=dev)
        self._pinned = None
        self._copied = torch.cuda.Event()
        self._keep_out = (torch.empty(self.stride, dtype=torch.int64, device=dev),
                          torch.empty(self.kv_cap, dtype=torch.int32, device=dev),
                          torch.empty(2, dtype=torch.int32, device=dev))
        self._blk = blocks
        if packed is not None and len(packed) > 3 and packed[3] is not None:
            # visibility the blocks' rows inherit from outside their own prompt
            vis = packed[3]
            self.seg_bits[:, :vis.shape[1]] = vis
        self._mask = None

    # ------------------------------------------------------------------
    def inputs(self):
        """``(input_ids int32 [Q], position_ids int64 [Q], PackedMask)`` of this step."""
        if self._mask is None:
            q = int(self.input_ids.size)
            segs = np.zeros((self.nb, 6), dtype=np.int32)
            segs[:, 0], segs[:, 1], segs[:, 2] = self.q_start, self.q_len, self.kinds
            row_seg = np.full(q, -1, dtype=np.int32)
            nrows = int(self.q_len.sum())
            row_seg[:nrows] = np.repeat(np.arange(self.nb, dtype=np.int32), self.q_len)
            tree_rows, tree_off = [], 0
            for b in [b for b in range(self.nb) if self.kinds[b] == SEG_TREE]:
                qs, ql = int(self.q_start[b]), int(self.q_len[b])
                # node i sees itself and its ancestors (D:1506-1533), rows
                # from the tree kernel or the host tree; pad rows see nothing
                tw = (ql + 63) // 64
                n = int(self.valid[b])
                if self.host_tree[b] is not None:
                    anc = np.zeros((ql, tw * 64), dtype=bool)
                    par = self.host_tree[b][1]
                    for j in range(n):
                        a = j
                        while a >= 0:
                            anc[j, a] = True
                            a = par[a]
                    rows = torch.from_numpy(pack_bits(anc).view(np.int64)).to(self.device)
                else:
                    i = self.tree_slot[b]
                    rows = torch.zeros((ql, tw), dtype=torch.int64, device=self.device)
                    w = min(tw, self.trees.anc.shape[2])
                    rows[:n, :w] = self.trees.anc[i, :n, :w]
                tree_rows.append(rows.reshape(-1))
                segs[b, 3], segs[b, 4] = tree_off, tw
                tree_off += ql * tw
            kv_bits = self.seg_bits
            q_blocks = int(self.q_start[-1] + self.q_len[-1]) if self.nb else 0
            if self.pad_rows_inherit and q > q_blocks:
                # tight padding rows inherit the last block's row and see
                # none of the new columns (D:1640-1644)
                segs = np.concatenate([segs, np.asarray([[q_blocks, q - q_blocks, SEG_NONE,
                                                          0, 0, 0]], dtype=np.int32)])
                row_seg[q_blocks:] = self.nb
                kv_bits = torch.cat([self.seg_bits, self.seg_bits[self.nb - 1:self.nb]])
            tree_bits = torch.cat(tree_rows) if tree_rows else None
            self._mask = PackedMask.from_bits(q, self.kv_len, segs, row_seg, kv_bits,
                                              self.device, tree_bits)
            # the step's ids and positions go up once, with the mask
            self._ids = torch.from_numpy(self.input_ids.astype(np.int32)).to(self.device)
            self._pos = torch.from_numpy(self.position_ids).to(self.device)
        return self._ids, self._pos, self._mask

    def logit_probes(self):
        """``(rows, toks)``, int32 device ``[Q]``: the logits
        ``logits[rows[r], toks[r]]`` the logit-ratio rules read this step,
        one per packed row (``toks[r] = -1``: none).  A speculative block's
        row r probes its draft token ``input_ids[r + 1]`` (D:1166-1167); a
        tree block's node c (row bs + c) probes its own token at its
        parent's row, ``logits[bs + parent(c), token(c)]`` (D:1231, D:1259).
        :func:`hsd_b200.lm_head.probe_logits` computes them from the final
        hidden states."""
        q = int(self.input_ids.size)
        rows = np.arange(q, dtype=np.int32)
        toks = np.full(q, -1, dtype=np.int32)
        for b in range(self.nb):
            qs, ql = int(self.q_start[b]), int(self.q_len[b])
            if self.modes[b] == N.HSD_MODE_SPEC and ql > 1:
                toks[qs:qs + ql - 1] = self.input_ids[qs + 1:qs + ql]
            elif self.modes[b] == N.HSD_MODE_TREE and self.tree_parents[b] is not None:
                n = int(self.valid[b])
                par = np.asarray(self.tree_parents[b][:n], dtype=np.int32)
                rows[qs + 1:qs + n] = qs + par[1:]
                toks[qs + 1:qs + n] = self.input_ids[qs + 1:qs + n]
        return (torch.from_numpy(rows).to(self.device), torch.from_numpy(toks).to(self.device))

    def step(self, next_ids, max_logit=None, probe_logit=None, text_mode=None, rank=None,
             second=None, page_next=None):
        """Consume the target argmax of every packed row; prepare the next step.

        With thresholds below 1, ``max_logit`` (float32 ``[Q]``, the maximal
        bf16 logit per row: :func:`hsd_b200.lm_head.lm_head_argmax`'s
        ``max_logit``) and ``probe_logit`` (float32 ``[Q]``, the logits
        :meth:`logit_probes` lists) feed the logit-ratio rules, and
        ``text_mode[b]`` (the page parser's ``text_mode``, D:1229; default
        False) enables the tree fallback for block b.  Returns False once
        generation is finished (every block finished or ``max_new_tokens``
        generated, D:1589-1591).  HunYuan's ``spec_mode="topk"`` reads
        ``rank`` (int32 ``[Q]``: row r's draft token ``input_ids[r + 1]``
        ranked among the row's logits) and ``"adaptive"`` ``second`` (float32
        ``[Q]``: the row's second best logit);
        :func:`hsd_b200.lm_head.lm_head_rank` computes both for the last
        block's rows, the only rows these modes read.

        With a page block, ``page_next(loop, gen, increment, mws, pos_base,
        next_token)`` gives its next input (a :class:`hsd_b200.page_block.PageInput`) from
        its generated tokens ``gen`` after the step; it runs on the host
        while the device computes the other blocks' trees and keep indices.
        """
        if self.done:
            raise RuntimeError("the loop has finished")
        if self.ratio and (max_logit is None or probe_logit is None):
            raise ValueError("thresholds below 1 need max_logit and probe_logit")
        if self.ratio and self.spec_thresh < 1.0 and (
                (self.spec_mode == "topk" and rank is None)
                or (self.spec_mode == "adaptive" and second is None)):
            raise ValueError(f"spec_mode {self.spec_mode!r} needs "
                             f"{'rank' if self.spec_mode == 'topk' else 'second'}")
        dev = self.device
        self.decode_times += 1
        q = int(self.input_ids.size)
        kv = self.kv_len
        nb = self.nb
        if text_mode is not None:
            flags = np.asarray([FLAG_TEXT_MODE if t else 0 for t in text_mode], dtype=np.int32)
            if flags.size != nb:
                raise ValueError("text_mode: one flag per block")
            if self.page_block:
                flags[-1] |= FLAG_PAGE_BLOCK
            self._flags = flags
        # tree blocks read their nodes from the tree kernel's rows of the last
        # step; host-built trees (the page block's) follow them
        toff = np.zeros(nb, dtype=np.int32)
        tnodes = np.zeros(nb, dtype=np.int32)
        d_tok = d_par = self._zero_i32
        host_trees = [b for b in range(nb)
                      if self.modes[b] == N.HSD_MODE_TREE and self.host_tree[b] is not None]
        if self.trees is not None or host_trees:
            base = 0
            toks, pars = [], []
            if self.trees is not None:
                toks.append(self.trees.tokens.reshape(-1))
                pars.append(self.trees.parents.reshape(-1))
                base = int(self.trees.tokens.numel())
                for b in range(nb):
                    if self.modes[b] == N.HSD_MODE_TREE and self.host_tree[b] is None:
                        toff[b] = self.tree_slot[b] * self.trees.cap
                        tnodes[b] = self.valid[b]
            for b in host_trees:
                t, par = self.host_tree[b]
                toff[b], tnodes[b] = base, len(t)
                toks.append(torch.tensor(t, dtype=torch.int32, device=dev))
                pars.append(torch.tensor(par, dtype=torch.int32, device=dev))
                base += len(t)
            d_tok, d_par = torch.cat(toks), torch.cat(pars)
        # this step's block fields and pad columns: one upload each
        cols = np.stack([np.asarray(self.modes), self.q_start, self.q_len,
                         np.asarray(self.valid), self._flags, toff, tnodes], 1).astype(np.int32)
        self.blocks[:, self._upd_cols] = torch.from_numpy(cols).to(dev, non_blocking=True)
        pad_cols = np.zeros(self.stride * 64, dtype=bool)
        pad_cols[kv - q:kv] = self.input_ids == self.pad
        pad_words = np.packbits(pad_cols, bitorder="little").view(np.int64)  # 64 bits a word
        pad_dev = torch.from_numpy(pad_words).to(dev, non_blocking=True)
        self.filter.zero_()
        self.out_bits.zero_()
        cfg = make_config(nb, kv, q, self.stride, self.eos, self.mws0, self.mws_ub,
                          self.max_spec_len, self.sentinel)
        ids, _, _ = self.inputs()
        accept_kmp(cfg, self.blocks, next_ids.to(torch.int32), ids, self.gen_pool,
                   self.draft_pool, self.seg_bits, self.out_bits, self.filter,
                   tree_tokens=d_tok, tree_parents=d_par, results=self.results,
                   status=self.status,
                   logits=(max_logit, probe_logit, self.spec_thresh, self.tree_thresh)
                   if self.ratio else None, variant=self.variant,
                   formula_tokens=self.formula_tokens, spec_mode=self.spec_mode,
                   spec_topk=self.spec_topk, spec_margin=self.spec_margin,
                   rank=None if rank is None else rank.to(torch.int32).contiguous(),
                   second=None if second is None else second.to(torch.float32).contiguous())
        # pad columns of this step's input join the filter after the blocks'
        # own updates, as the reference ORs them in after its block loop (D:1596-1599)
        self.filter |= pad_dev

        # device work that needs no host decision: the continuation trees of
        # every live region block (the host keeps those of blocks without
        # exactly one match), the keep indices over every block's row (a
        # finished block's row is empty, or all filtered when it finished in
        # this step, so the active rows give the same keep, D:1679-1687) and
        # the new tokens of every block
        cand = [b for b in range(nb) if self.tree_decode and self.modes[b] != N.HSD_MODE_FINISHED
                and not (self.page_block and b == nb - 1)]
        new_trees = None
        if cand:
            idx = torch.tensor(cand, dtype=torch.long, device=dev)
            new_trees = continuation_trees(
                self.draft_pool, self.d_draft_off[idx].contiguous(),
                self.d_draft_len[idx].contiguous(),
                self.results[idx, R["next_token"]].contiguous(), self.tree_depth,
                self.tree_cap, status=self.status)
        keep_bits, keep_idx, counts = keep_indices(self.out_bits, self.filter, kv,
                                                   out=self._keep_out)
        live = [b for b in range(nb) if self.modes[b] != N.HSD_MODE_FINISHED]
        # gen-pool slots of every live block's rows, one run per block
        lens = self.q_len[live].astype(np.int64)
        first = np.asarray([b * self.gen_cap + len(self.gen_host[b]) for b in live],
                           dtype=np.int64)
        gidx = (np.arange(int(lens.sum()), dtype=np.int64)
                + np.repeat(first - (np.cumsum(lens) - lens), lens))
        gidx = np.minimum(gidx, self.gen_pool.numel() - 1)
        parts = [self.results.reshape(-1), self.status, counts, self.blocks.reshape(-1)]
        if gidx.size:
            parts.append(self.gen_pool[torch.from_numpy(gidx).to(dev, non_blocking=True)])
        if new_trees is not None:
            parts += [new_trees.counts, new_trees.tokens.reshape(-1),
                      new_trees.depths.reshape(-1), new_trees.parents.reshape(-1)]
        # ---- the step's one device -> host copy
        packed = torch.cat(parts)
        if self._pinned is None or self._pinned.numel() < packed.numel():
            self._pinned = torch.empty(max(packed.numel(), 4096) * 2, dtype=torch.int32,
                                       pin_memory=True)
        host = self._pinned[:packed.numel()]
        host.copy_(packed, non_blocking=True)
        self._copied.record()
        self._copied.synchronize()
        h = host.numpy()
        o = 0
        res = h[o:o + nb * len(R)].reshape(nb, len(R)).copy()
        o += nb * len(R)
        code = int(h[o])
        o += 1
        n_keep = int(h[o])
        o += 2
        blk = h[o:o + nb * 16].reshape(nb, 16).copy()
        o += nb * 16
        newtok = h[o:o + gidx.size]
        o += gidx.size
        if code:
            raise N.HSDError(f"device status 0x{code:x} in the verification loop")
        host_tree_lists = {}
        if new_trees is not None:
            cap, nt = new_trees.cap, len(cand)
            tcnt = h[o:o + nt]
            o += nt
            arr = [h[o + k * nt * cap:o + (k + 1) * nt * cap].reshape(nt, cap) for k in range(3)]
            for i, b in enumerate(cand):
                c = int(tcnt[i])
                host_tree_lists[b] = (arr[0][i, :c].tolist(), arr[1][i, :c].tolist(),
                                      arr[2][i, :c].tolist())
        # generated tokens on the host (EOS dropped, D:1303; the draft after
        # a repetition stop, D:1317)
        j = 0
        for b in live:
            n = int(self.q_len[b])
            r = res[b]
            inc = int(r[R["increment"]])
            if r[R["finished"]] == 2:
                self.gen_host[b] = list(self.drafts[b])
            else:
                self.gen_host[b] += newtok[j:j + inc].tolist()
                if r[R["finished"]] == 1:
                    self.gen_host[b].pop()
            j += n
        self._blk = blk

        want = [b for b in cand if not res[b][R["finished"]] and res[b][R["match_count"]] != 1]
        new_slot = [-1] * nb
        for b in want:
            new_slot[b] = cand.index(b)

        # stop rule and compaction first: they need only the copied results,
        # so the compaction runs on the device while the host does the page
        # block's parser and matching and packs the next input below
        self.step_finished = [self.modes[b] == N.HSD_MODE_FINISHED or bool(res[b][R["finished"]])
                              for b in range(nb)]
        for b in live:
            self.new_tokens += int(res[b][R["increment"]])
        if self.page_block and self.variant == "hunyuan":
            # the HunYuan loop counts the page block's own tokens (H:2133)
            produced = len(self.gen_host[nb - 1])
        else:
            produced = self.new_tokens
        if produced >= self.max_new_tokens or all(self.step_finished) or (
                self.page_block and self.step_finished[-1]):                  # D:1589-1592
            self.modes = [N.HSD_MODE_FINISHED if f else m
                          for f, m in zip(self.step_finished, self.modes)]
            self.done = True
            return False

        # the compaction rule (D:1693-1700, H:2253-2259) on the kept count
        t_c = time.perf_counter()
        self.compaction_calls += 1
        dead = kv - n_keep
        if self.variant == "hunyuan":   # period 0 compacts too (H:2253-2259)
            rule = (self.period <= 1 or self.decode_times % self.period == 0
                    or dead > kv * 0.2)
        else:                           # D:1693-1700
            rule = self.period > 0 and (self.period <= 1 or self.decode_times % self.period == 0
                                        or dead > kv * 0.2)
        nw = (kv + 63) // 64
        if rule and n_keep < kv:                      # compact (D:1704-1723)
            if self.kv_planes is not None:
                compact_kv(self.kv_planes, self.row_bytes, keep_idx, counts=counts,
                           status=self.status)
            if self.compact_hook is not None:
                self.compact_hook(keep_idx, counts, n_keep)
            if self.kv_tokens is not None:
                self.kv_tokens = self.kv_tokens[keep_idx[:n_keep].long()]
            self.seg_bits = compact_bits(self.out_bits, keep_idx, counts, self.stride)
            kv = n_keep
        elif not rule:                                # dead columns masked (D:1724-1729)
            self.seg_bits = self.out_bits.clone()
            self.seg_bits[:, :nw] &= keep_bits[None, :nw]
            if self.variant != "hunyuan":             # dots counts masked steps (D:1730)
                self.compactions_skipped += 1
        else:
            self.seg_bits = self.out_bits.clone()
            if self.variant == "hunyuan":             # HunYuan: nothing to drop (H:2275)
                self.compactions_skipped += 1
        self.compaction_s += time.perf_counter() - t_c


        # the page block's next input, from the host (D:1337-1567)
        page_in = None
        last = nb - 1
        if (self.page_block and page_next is not None
                and self.modes[last] != N.HSD_MODE_FINISHED and not res[last][R["finished"]]):
            r = res[last]
            page_in = page_next(self, list(self.gen_host[last]), int(r[R["increment"]]),
                                int(blk[last][F["mws"]]),
                                int(self.position_ids[int(r[R["pointer"]])]) + 1,
                                int(r[R["next_token"]]))
            self.blocks[last, F["matches_len"]] = int(page_in.matches)
        # next inputs (D:1421-1565) from the result rows
        new_ids, new_pos, new_lens = [], [], [0] * nb
        new_modes, new_valid, new_kinds = list(self.modes), [0] * nb, list(self.kinds)
        new_parents = [None] * nb
        new_host_tree = [None] * nb
        for b in range(nb):
            if self.modes[b] == N.HSD_MODE_FINISHED:
                new_kinds[b] = SEG_NONE   # no rows any more
                continue
            r = res[b]
            if r[R["finished"]]:
                new_modes[b], new_kinds[b] = N.HSD_MODE_FINISHED, SEG_NONE
                continue
            base = int(self.position_ids[int(r[R["pointer"]])]) + 1
            if page_in is not None and b == nb - 1:
                toks = np.asarray(page_in.ids, dtype=np.int64)
                pos = np.asarray(page_in.pos, dtype=np.int64)
                if page_in.kind == "spec":
                    new_modes[b], new_kinds[b] = N.HSD_MODE_SPEC, SEG_CAUSAL
                elif page_in.kind == "tree":
                    new_modes[b], new_kinds[b] = N.HSD_MODE_TREE, SEG_TREE
                    new_parents[b] = list(page_in.parents)
                    new_host_tree[b] = (toks[:page_in.valid].tolist(), list(page_in.parents))
                else:
                    new_modes[b], new_kinds[b] = N.HSD_MODE_NORMAL, SEG_SINGLE
                new_valid[b] = int(page_in.valid)
            elif r[R["match_count"]] == 1:
                toks = self._drafts_np[b][int(r[R["slice_begin"]]):int(r[R["slice_end"]])]
                n = len(toks)
                if not self.tight:
                    pad_n = math.ceil(n / self.mil) * self.mil - n
                    toks = np.concatenate([toks, np.full(pad_n, self.pad, dtype=np.int64)])
                new_modes[b], new_kinds[b], new_valid[b] = N.HSD_MODE_SPEC, SEG_CAUSAL, n
                pos = np.arange(base, base + len(toks), dtype=np.int64)
            else:
                tree = host_tree_lists.get(b) if b in want else None
                if tree is not None and len(tree[0]) > 1:    # D:1488-1543
                    tokens, depths, new_parents[b] = tree
                    n = len(tokens)
                    pad_n = 0 if self.tight else math.ceil(n / self.mil) * self.mil - n
                    toks = np.asarray(list(tokens) + [self.pad] * pad_n, dtype=np.int64)
                    pos = np.asarray([d + base for d in depths] + [0] * pad_n, dtype=np.int64)
                    new_modes[b], new_kinds[b], new_valid[b] = N.HSD_MODE_TREE, SEG_TREE, n
                else:                                        # D:1544-1565
                    fill = 0 if self.tight else self.mil - 1
                    toks = np.full(1 + fill, self.pad, dtype=np.int64)
                    toks[0] = int(r[R["next_token"]])
                    pos = np.zeros(1 + fill, dtype=np.int64)
                    pos[0] = base
                    new_modes[b], new_kinds[b], new_valid[b] = N.HSD_MODE_NORMAL, SEG_SINGLE, 1
            new_ids.append(toks)
            new_pos.append(pos)
            new_lens[b] = len(toks)
        # the next packed input and its KV columns; tight packing pads the
        # input to a multiple of 128 rows at position 0 that belong to no
        # block (D:1619-1632): with ``pad_rows_inherit`` they see the last
        # block's row (the dots loop, D:1640-1644), otherwise nothing (the
        # HunYuan loop, H:2290-2293); no block reads their outputs and the
        # pad filter drops their columns, so tokens and compaction are the same
        if self.tight and sum(new_lens) % Q_BLOCK:
            pad_n = Q_BLOCK - sum(new_lens) % Q_BLOCK
            new_ids.append(np.full(pad_n, self.pad, dtype=np.int64))
            new_pos.append(np.zeros(pad_n, dtype=np.int64))
        empty = np.zeros(0, dtype=np.int64)
        self.input_ids = np.concatenate(new_ids or [empty])
        self.position_ids = np.concatenate(new_pos or [empty])
        ends = np.cumsum(new_lens)
        self.q_len = np.asarray(new_lens, dtype=np.int64)
        self.q_start = ends - self.q_len
        self.modes, self.valid, self.kinds = new_modes, new_valid, new_kinds
        self.trees = new_trees if want else None
        self.tree_slot, self.tree_parents = new_slot, new_parents
        self.host_tree = new_host_tree
        self.kv_len = kv + int(self.input_ids.size)
        if self.kv_len > self.kv_cap:
            raise N.HSDError(f"KV columns {self.kv_len} exceed the loop's capacity {self.kv_cap}")
        if self.kv_tokens is not None:
            self.kv_tokens = torch.cat([self.kv_tokens,
                                        torch.from_numpy(self.input_ids.astype(np.int32)).to(dev)])
        self._mask = None
        return True

    def generated(self):
        """Generated tokens of every block (EOS dropped, D:1303), kept on the
        host from each step's copy of the blocks' new tokens."""
        return [list(g) for g in self.gen_host]

    def _check(self):
        code = int(self.status.item())
        if code:
            raise N.HSDError(f"device status 0x{code:x} in the verification loop")


def batch_generate(model_fn, prompts, drafts, *, eos_token_id, max_new_tokens, **loop_kwargs):
    """Run the loop to completion with ``model_fn(input_ids, position_ids,
    mask, kv_tokens) -> next_ids`` (the target forward + argmax per packed
    row; ``mask`` is the step's :class:`PackedMask`, ``kv_tokens`` the token
    of every KV column, which a model holding its own cache can ignore).
    Below the default thresholds (``spec_thresh`` / ``tree_thresh`` < 1)
    the call is ``model_fn(..., probes=(rows, toks)) -> (next_ids,
    max_logit, probe_logit)`` with the probes of
    :meth:`VerifyLoop.logit_probes`, optionally followed by ``text_mode``
    (one flag per block).

    Returns the reference's result shape (D:1801-1810): ``(generated_tokens,
    decode_times, (forward_s, outside_forward_s, 0.0, 0.0, first_forward_s,
    compaction_s, compaction_calls, compactions_skipped))`` -- the setup and
    preparation times have no counterpart here and are 0.
    """
    loop = VerifyLoop(prompts, drafts, eos_token_id=eos_token_id,
                      max_new_tokens=max_new_tokens, **loop_kwargs)
    t_fwd = t_out = first = 0.0
    while True:
        ids, pos, mask = loop.inputs()
        torch.cuda.synchronize(loop.device)
        t0 = time.perf_counter()
        if loop.ratio:
            out = model_fn(ids, pos, mask, loop.kv_tokens, probes=loop.logit_probes())
        else:
            out = (model_fn(ids, pos, mask, loop.kv_tokens),)
        torch.cuda.synchronize(loop.device)
        t1 = time.perf_counter()
        more = loop.step(*out)
        t2 = time.perf_counter()
        t_fwd += t1 - t0
        t_out += t2 - t1
        if loop.decode_times == 1:
            first = t1 - t0
        if not more:
            break
    return loop.generated(), loop.decode_times, (t_fwd, t_out, 0.0, 0.0, first,
                                                   loop.compaction_s, loop.compaction_calls,
                                                   loop.compactions_skipped)

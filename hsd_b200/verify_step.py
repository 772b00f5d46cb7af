"""One verification step of a packed page, entirely on the device.

This is the hot path of the reference's ``batch_generate`` iteration
(hsd/dots_ocr_pipeline/modeling_dots_ocr_hsd.py D:1053-1767) minus the dense
decoder GEMMs, which stay in the model:

1. KV append of the step's new rows into the layer caches (what
   ``DynamicCache.update`` does with ``torch.cat``, D:356-359),
2. tile plan from the segment descriptors (replaces the dense mask build and
   ``create_block_mask``, D:94-106, D:1634-1667),
3. packed verification attention on every layer (D:72-135),
4. acceptance + KMP re-alignment of every block (D:1103-1336),
5. keep indices and in-place compaction of every layer's K and V
   (D:1669-1735), plus the remap of each block's visibility row.

``VerifyStep.run()`` launches all of it on one stream without a host sync.
``VerifyStep.run_from_host()`` is the end-to-end form: the step's inputs come
from pinned host buffers and the per-block results go back to the host.
Both capture into CUDA graphs (``VerifyStep.capture``): every buffer and
launch argument is fixed, so a replay re-runs the step without host work.
"""
from __future__ import annotations

import ctypes as C

import numpy as np
import torch

from . import _native as N
from .accept import F as BF
from .accept import make_config
from .plan import PackedMask, TilePlan, pack_bits


class VerifyStep:
    def __init__(self, page, device="cuda", seed=0, period=1, device_rng=False):
        """Device buffers of one page's step.  The synthetic Q / K / V come
        from a CPU generator seeded with ``seed`` (the same on every machine),
        or, with ``device_rng``, from a generator on the device (fast when
        many pages are built)."""
        self.page = page
        self.device = torch.device(device)
        dev = self.device
        L, hq, hkv, d = page.layers, page.hq, page.hkv, page.head_dim
        self.L, self.hq, self.hkv, self.d = L, hq, hkv, d
        self.q_len, self.kv_len, self.prefix = page.q_len, page.kv_len, page.prefix
        gdev = dev if device_rng else torch.device("cpu")
        g = torch.Generator(device=gdev).manual_seed(seed)
        s = 1.0 / np.sqrt(d)

        def rnd(*shape):
            return (torch.randn(*shape, generator=g, device=gdev) * s).to(torch.bfloat16)

        # step inputs (device-resident for run(); mirrored in pinned host memory
        # for run_from_host())
        self.q = rnd(L, hq, self.q_len, d).to(dev)
        self.new_kv = rnd(L, 2, hkv, self.q_len, d).to(dev)
        # layer caches [L][K/V][Hkv][kv_len][D]; the prefix rows are resident state
        self.cache = torch.empty(L, 2, hkv, self.kv_len, d, dtype=torch.bfloat16, device=dev)
        self.cache[:, :, :, :self.prefix] = rnd(L, 2, hkv, self.prefix, d).to(dev)
        self.out = torch.empty(L, self.q_len, hq, d, dtype=torch.bfloat16, device=dev)
        self.lse = torch.empty(L, hq, self.q_len, dtype=torch.float32, device=dev)

        from .workloads import segment_dicts
        self.mask = PackedMask(self.q_len, self.kv_len, segment_dicts(page), device=dev)
        self.plan = TilePlan(self.q_len, self.kv_len, dev)
        from .attention import attention_workspace
        self.ws = attention_workspace(self.q_len, hq, hkv, dev)
        self.status = torch.zeros(1, dtype=torch.int32, device=dev)

        # acceptance inputs
        segs = page.segments
        nb = len(segs)
        self.n_blocks = nb
        self.stride = self.mask.stride
        cap = max(len(sg.gen) + sg.q_len + 8 for sg in segs)
        cap = max(cap, max(len(sg.draft) for sg in segs))
        blocks = np.zeros((nb, 16), dtype=np.int32)
        gen_pool = np.zeros(nb * cap, dtype=np.int32)
        drafts = []
        doff = 0
        for i, sg in enumerate(segs):
            blocks[i, BF["mode"]] = N.HSD_MODE_SPEC
            blocks[i, BF["q_start"]] = sg.q_start
            blocks[i, BF["q_len"]] = sg.q_len
            blocks[i, BF["valid_count"]] = sg.q_len
            blocks[i, BF["gen_off"]] = i * cap
            blocks[i, BF["gen_len"]] = len(sg.gen)
            blocks[i, BF["gen_cap"]] = cap
            gen_pool[i * cap:i * cap + len(sg.gen)] = sg.gen
            blocks[i, BF["draft_off"]] = doff
            blocks[i, BF["draft_len"]] = len(sg.draft)
            drafts += sg.draft
            doff += len(sg.draft)
            blocks[i, BF["mws"]] = 3
            blocks[i, BF["matches_len"]] = 1
            blocks[i, BF["seg"]] = i
        self.blocks0 = torch.from_numpy(blocks).to(dev)
        self.blocks = self.blocks0.clone()
        self.gen_pool = torch.from_numpy(gen_pool).to(dev)
        self.draft_pool = torch.from_numpy(np.asarray(drafts, dtype=np.int32)).to(dev)
        self.input_ids = torch.from_numpy(page.input_ids).to(dev)
        self.next_ids = torch.from_numpy(page.next_ids).to(dev)
        self.results = torch.zeros(nb, 8, dtype=torch.int32, device=dev)
        self.vis = torch.zeros(nb, self.stride, dtype=torch.int64, device=dev)
        self.vis_next = torch.zeros_like(self.vis)
        self.filter = torch.zeros(self.stride, dtype=torch.int64, device=dev)
        self.keep_bits = torch.zeros(self.stride, dtype=torch.int64, device=dev)
        self.keep_idx = torch.zeros(self.kv_len, dtype=torch.int32, device=dev)
        self.counts = torch.zeros(2, dtype=torch.int32, device=dev)
        self.tree_dummy = torch.zeros(1, dtype=torch.int32, device=dev)
        self.cfg = make_config(nb, self.kv_len, self.q_len, self.stride, [2**31 - 1])
        planes = []
        for l in range(L):
            for kv in range(2):
                for h in range(hkv):
                    planes.append(self.cache[l, kv, h].data_ptr())
        self.planes = torch.tensor(planes, dtype=torch.int64, device=dev)
        src = []
        for l in range(L):
            for kv in range(2):
                for h in range(hkv):
                    src.append(self.new_kv[l, kv, h].data_ptr())
        self.new_planes = torch.tensor(src, dtype=torch.int64, device=dev)
        self.row_bytes = d * 2
        self.period = period
        self.copy_layers = 4   # layers per host -> device copy in run_from_host
        self._host = None
        self._side = None  # second stream for the step's independent launches
        self.attn_launches_per_step = L
        # append 1 + plan 2 + attention L + accept 1 + keep 1 + compact 1 + bits 1
        self.kernel_launches_per_step = 1 + 2 + L + 4
        # the end-to-end form appends layer by layer: L appends instead of 1
        self.kernel_launches_per_host_step = L + 2 + L + 4

    # ------------------------------------------------------------------
    def _ptr(self, t):
        return C.c_void_p(t.data_ptr())

    def run(self, stream=None, attn_events=None, phase_events=None, layer_ready=None,
            buffers=0):
        """Launch one verification step on ``stream`` (no host sync).

        ``attn_events[l]`` (start, end) bracket layer l's attention call;
        ``phase_events`` (dict of name -> (start, end)) bracket the phases
        append / plan / accept / keep / compact / bits.  With
        ``layer_ready`` (one event per layer) the step reads its query and
        new K/V rows from input set ``buffers`` (see :meth:`run_from_host`)
        and appends and attends layer by layer, layer l waiting only for
        ``layer_ready[l]``.

        Independent launches run on a second stream: the KV append beside
        the tile plan (both feed the attention), the visibility-row remap
        beside the compaction (both follow the keep indices).  With
        ``phase_events`` every phase runs in order on ``stream``, so each
        pair of events brackets one phase alone.
        """
        lib = N.load()
        main = stream if stream is not None else torch.cuda.current_stream()
        st = N.stream_handle(main)
        p = self._ptr
        ev = phase_events or {}
        concurrent = not ev
        if concurrent and self._side is None:
            self._side = torch.cuda.Stream(device=self.device)
        side = self._side if concurrent else main
        sst = N.stream_handle(side)

        def mark(name, i):
            if name in ev:
                ev[name][i].record(main)
        # 1. KV append (the model's cache update), beside the plan
        if concurrent:
            side.wait_stream(main)
        mark("append", 0)
        if layer_ready is None:
            N.check(lib.hsd_kv_append(p(self.planes), p(self.new_planes), self.planes.numel(),
                                      self.row_bytes, self.prefix, self.q_len, sst),
                    "hsd_kv_append")
        mark("append", 1)
        with torch.cuda.stream(main):
            self.filter.zero_()
            self.blocks.copy_(self.blocks0)
        mark("plan", 0)
        # 2. tile plan
        m = self.mask
        N.check(lib.hsd_build_plan_segments(
            p(m.segs), m.n_segs, p(m.row_seg), p(m.kv_bits), m.stride, p(m.tree_bits),
            C.byref(self.plan.struct), p(self.status), st), "hsd_build_plan_segments")
        mark("plan", 1)
        if concurrent:
            main.wait_stream(side)
        # 3. attention, every layer (with its own append when the rows arrive per layer)
        self.run_attention(main, attn_events, layer_ready, buffers)
        # 4. acceptance + KMP
        mark("accept", 0)
        N.check(lib.hsd_accept_kmp(
            C.byref(self.cfg), p(self.blocks), p(self.results), p(self.next_ids),
            p(self.input_ids), p(self.gen_pool), p(self.draft_pool), p(self.tree_dummy),
            p(self.tree_dummy), p(m.kv_bits), p(self.vis), p(self.filter), p(self.status), st),
            "hsd_accept_kmp")
        mark("accept", 1)
        # 5. keep indices, in-place compaction, visibility remap
        mark("keep", 0)
        N.check(lib.hsd_keep_indices(p(self.vis), self.n_blocks, self.stride, p(self.filter),
                                     self.kv_len, p(self.keep_bits), p(self.keep_idx),
                                     p(self.counts), st), "hsd_keep_indices")
        mark("keep", 1)
        if concurrent:
            side.wait_stream(main)
        mark("compact", 0)
        N.check(lib.hsd_compact_kv(p(self.planes), self.planes.numel(), self.row_bytes,
                                   p(self.keep_idx), -1, p(self.counts), p(self.status), st),
                "hsd_compact_kv")
        mark("compact", 1)
        mark("bits", 0)
        N.check(lib.hsd_compact_bits(p(self.vis), p(self.vis_next), self.n_blocks, self.stride,
                                     p(self.keep_idx), p(self.counts), self.stride, sst),
                "hsd_compact_bits")
        mark("bits", 1)
        if concurrent:
            main.wait_stream(side)

    def run_attention(self, stream=None, attn_events=None, layer_ready=None, buffers=0):
        """The step's attention launches alone (every layer, current plan);
        with ``layer_ready`` each layer first waits for its event and
        appends its own new K/V rows from input set ``buffers``."""
        lib = N.load()
        st = N.stream_handle(stream)
        ts = stream if stream is not None else torch.cuda.current_stream()
        p = self._ptr
        scale = 1.0 / np.sqrt(self.d)
        ql, kvl, hq, hkv, d = self.q_len, self.kv_len, self.hq, self.hkv, self.d
        qset = self.q if buffers == 0 else self._alt["q"]
        per = 2 * hkv
        for l in range(self.L):
            q = qset[l]
            k = self.cache[l, 0]
            v = self.cache[l, 1]
            if layer_ready is not None:
                ts.wait_event(layer_ready[l])
                src = self.new_planes if buffers == 0 else self._alt["new_planes"]
                N.check(lib.hsd_kv_append(C.c_void_p(self.planes.data_ptr() + 8 * l * per),
                                          C.c_void_p(src.data_ptr() + 8 * l * per), per,
                                          self.row_bytes, self.prefix, self.q_len, st),
                        "hsd_kv_append")
            if attn_events is not None:
                attn_events[l][0].record(stream)
            N.check(lib.hsd_verify_attention(
                p(q), q.stride(1), q.stride(0), p(k), k.stride(1), k.stride(0), p(v), v.stride(1),
                v.stride(0), p(self.out[l]), p(self.lse[l]), ql, kvl, hq, hkv, d, scale,
                C.byref(self.plan.struct), C.c_void_p(self.ws.base), self.ws.nbytes,
                p(self.status), st), "hsd_verify_attention")
            if attn_events is not None:
                attn_events[l][1].record(stream)

    def compaction_bytes(self):
        """(bytes moved by the last compaction (read + write), rows moved, rows kept)."""
        n_keep, first = (int(x) for x in self.counts.cpu().tolist())
        moved = max(0, n_keep - first)
        return 2 * moved * self.row_bytes * self.planes.numel(), moved, n_keep

    # ------------------------------------------------------------------
    def host_buffers(self):
        """Pinned host copies of the step's inputs (end-to-end form)."""
        if self._host is None:
            self._host = dict(
                q=self.q.cpu().pin_memory(), new_kv=self.new_kv.cpu().pin_memory(),
                input_ids=self.input_ids.cpu().pin_memory(),
                next_ids=self.next_ids.cpu().pin_memory(),
                results=torch.empty_like(self.results, device="cpu").pin_memory(),
                counts=torch.empty_like(self.counts, device="cpu").pin_memory())
        return self._host

    def h2d_bytes(self):
        h = self.host_buffers()
        return sum(h[k].numel() * h[k].element_size() for k in ("q", "new_kv", "input_ids",
                                                                  "next_ids"))

    def d2h_bytes(self):
        h = self.host_buffers()
        return sum(h[k].numel() * h[k].element_size() for k in ("results", "counts"))

    def _second_input_set(self):
        if getattr(self, "_alt", None) is None:
            q2 = torch.empty_like(self.q)
            kv2 = torch.empty_like(self.new_kv)
            planes = [kv2[l, kv, h].data_ptr() for l in range(self.L) for kv in range(2)
                      for h in range(self.hkv)]
            self._alt = dict(q=q2, new_kv=kv2, new_planes=torch.tensor(
                planes, dtype=torch.int64, device=self.device))
        return self._alt

    def run_from_host(self, stream=None, buffers=0, fork=True):
        """End-to-end step: pinned host inputs -> device step -> results to host.

        Every layer's query rows and new K/V rows (all but a few KB of the
        step's bytes) go layer by layer on a copy stream into input set
        ``buffers`` (0 or 1); each layer's append and attention wait only for
        that layer's rows, so the copies overlap the step's kernels.  The
        copy stream waits for nothing else: alternating ``buffers`` between
        consecutive steps lets step i+1's copies run under step i's kernels
        (set k is rewritten only after the step that last read it, two steps
        back, has finished).  The token ids (KBs) go on the compute stream.
        Inside a CUDA graph capture the copy stream forks from the capturing
        stream when ``fork`` (the graph's first step); a later step whose input
        set an earlier step of the same capture read waits for that step's
        kernels, the graph's second step only for its own earlier copies
        (replays of a graph never overlap).
        """
        h = self.host_buffers()
        cs = stream if stream is not None else torch.cuda.current_stream()
        if getattr(self, "_copy_stream", None) is None:
            self._copy_stream = torch.cuda.Stream(device=self.device)
            self._ready = [[torch.cuda.Event() for _ in range(self.L)] for _ in range(2)]
            self._set_free = [torch.cuda.Event(), torch.cuda.Event()]
            self._set_used = [False, False]
        xs = self._copy_stream
        q, nkv = (self.q, self.new_kv) if buffers == 0 else (
            self._second_input_set()["q"], self._second_input_set()["new_kv"])
        capturing = torch.cuda.is_current_stream_capturing()
        if capturing:
            if fork:
                xs.wait_stream(cs)
                self._cap_used = [False, False]
                self._cap_free = [torch.cuda.Event(), torch.cuda.Event()]
            elif self._cap_used[buffers]:
                xs.wait_event(self._cap_free[buffers])  # recorded earlier in this capture
        elif self._set_used[buffers]:
            xs.wait_event(self._set_free[buffers])  # the step that last read this set is done
        else:
            xs.wait_stream(cs)
        with torch.cuda.stream(xs):
            # a few layers per copy: large enough for the link's full rate,
            # small enough that the first layers' kernels start early
            for l0 in range(0, self.L, self.copy_layers):
                l1 = min(self.L, l0 + self.copy_layers)
                q[l0:l1].copy_(h["q"][l0:l1], non_blocking=True)
                nkv[l0:l1].copy_(h["new_kv"][l0:l1], non_blocking=True)
                for l in range(l0, l1):
                    self._ready[buffers][l].record(xs)
        with torch.cuda.stream(cs):
            self.input_ids.copy_(h["input_ids"], non_blocking=True)
            self.next_ids.copy_(h["next_ids"], non_blocking=True)
        self.run(cs, layer_ready=self._ready[buffers], buffers=buffers)
        if capturing:
            self._cap_free[buffers].record(cs)
            self._cap_used[buffers] = True
        else:
            self._set_free[buffers].record(cs)
            self._set_used[buffers] = True
        with torch.cuda.stream(cs):
            h["results"].copy_(self.results, non_blocking=True)
            h["counts"].copy_(self.counts, non_blocking=True)

    def capture(self, from_host=False, attention_only=False, host_steps=2):
        """A CUDA graph of one whole step (``run`` or, ``from_host``,
        ``host_steps`` (even) consecutive ``run_from_host`` steps on
        alternating input sets, or only the step's attention launches): the
        launches replay with no host work between them.  Call :meth:`run`
        (and, for ``from_host``, :meth:`run_from_host` on both sets) once
        before capturing: first-call setup must not happen inside a
        capture."""
        if from_host and (host_steps < 2 or host_steps % 2):
            raise ValueError("host_steps: an even number of steps, at least 2")
        torch.cuda.synchronize(self.device)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            if attention_only:
                self.run_attention()
            elif from_host:
                for i in range(host_steps):
                    self.run_from_host(buffers=i % 2, fork=i == 0)
            else:
                self.run()
        torch.cuda.synchronize(self.device)
        return graph

    # ------------------------------------------------------------------
    def attention_flops(self):
        """(executed-tile FLOPs, allowed-pair FLOPs) per attention launch.

        Executed tiles are FlexAttention's 128x64 tiles (partial + full) of the
        plan: FLOPs = tiles * 128 * 64 * 4 * D * Hq; allowed pairs likewise
        count only unmasked (q, kv) pairs.
        """
        cls = self.plan.tile_class().cpu().numpy()
        tiles = int((cls != 0).sum())
        words = self.plan.mask_words().cpu().numpy().view(np.uint64)
        pairs = int(np.unpackbits(words.view(np.uint8)).sum())
        f = 4 * self.d * self.hq
        return tiles * 128 * 64 * f, pairs * f, tiles, pairs

    def raise_on_device_error(self):
        code = int(self.status.item())
        if code:
            raise N.HSDError(f"device status 0x{code:x} during the verification step")

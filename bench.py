"""Benchmark of the HSD verification hot path on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--workload stage1_regions|stage2_page|hunyuan_regions]
                    [--multi-pages P]

A step is one verification iteration of one packed page (per GPU): KV
append, tile plan, packed verification attention over every decoder layer,
acceptance + KMP re-alignment of every block, keep indices and in-place KV
compaction (see hsd_b200/verify_step.py).  The default workload is Stage-1
region verification at dots.ocr scale (28 layers, 12/2 heads, 2624-token
page prefix, 32 drafts in a depth-2 prefix tree), seeded synthetic data.

Metric: verified draft tokens per second (non-pad packed query tokens of all
pages / step time), whole job.  With N GPUs every rank verifies a page of the
same shape with its own seeded Q / K / V: weak scaling, no collective on the
hot path; the step time is the max over ranks of CUDA-event time.  The same
line carries ``multi_page``: a fixed set of seeded pages (region counts
U[8, 64], prefix lengths U[1024, 4096]) shared out over the ranks, results
gathered to rank 0 (strong scaling).

``--impl reference`` times the reference's CPU path on the host cores (the
oracle restatement: eager FlexAttention with the 128x64 block mask and
repeat_kv, the acceptance loop with KMP, index_select compaction) on rank 0:
each step is one decoder layer's share of a page step, really run, credited
with that share of the page's tokens.
"""
from __future__ import annotations

import argparse
import datetime
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

FALLBACK_PEAKS = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}
E2E_STEPS = 8  # consecutive end-to-end steps per CUDA graph replay


def load_peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(path):
        with open(path) as f:
            d = json.load(f)
        return d, "measured"
    return FALLBACK_PEAKS, "fallback"


def profile_traffic(name):
    """DRAM bytes per launch recorded by the committed ncu summary, or None."""
    path = os.path.join(ROOT, "profiles", f"{name}.md")
    if not os.path.exists(path):
        return None
    for line in open(path):
        if line.strip().startswith("traffic_bytes_per_launch:"):
            try:
                return float(line.split(":", 1)[1].strip())
            except ValueError:
                return None
    return None


class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled every 20 ms; ``stop()``
    keeps the samples taken between ``mark_start()`` and ``mark_end()`` (the
    timed region), or all of them if the region was shorter than one
    sampling interval."""

    FIELDS = ("timestamp,index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index):
        self.gpu = gpu_index
        self.proc = None
        self.path = None
        self.t0 = self.t1 = None

    def mark_start(self):
        self.t0 = datetime.datetime.now()

    def mark_end(self):
        self.t1 = datetime.datetime.now()

    def start(self):
        fd, self.path = tempfile.mkstemp(suffix=".csv")
        os.close(fd)
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "20"],
                stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
        except (OSError, FileNotFoundError):
            self.proc = None

    def stop(self):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        rows = []
        for line in open(self.path):
            parts = [p.strip() for p in line.split(",")]
            if len(parts) >= 10 and parts[2].replace(".", "").isdigit():
                try:
                    ts = datetime.datetime.strptime(parts[0], "%Y/%m/%d %H:%M:%S.%f")
                except ValueError:
                    ts = None
                rows.append((ts, parts[1:]))
        os.unlink(self.path)
        inside = [r for ts, r in rows if ts is not None and self.t0 is not None
                  and self.t1 is not None and self.t0 <= ts <= self.t1]
        window = "timed region" if inside else "around the timed region"
        rows = inside or [r for _, r in rows]
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no samples"]}
        sm = [float(r[1]) for r in rows]
        mx = max(float(r[2]) for r in rows)
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i in range(4) if r[5 + i] == "Active"})
        loaded = [s for s in sm if s > 0.5 * mx] or sm
        return {"sm_mhz": statistics.median(loaded), "sm_max_mhz": mx, "reasons": reasons,
                "samples": len(rows), "window": window,
                "power_w_max": max(float(r[3]) for r in rows)}


# ---------------------------------------------------------------- CPU side
def page_config(page):
    """``config`` of a bench line: the workload only, identical for both arms."""
    return {"workload": page.name, "layers": page.layers, "q_len": page.q_len,
            "kv_len": page.kv_len, "heads": [page.hq, page.hkv],
            "verified_tokens_per_step_per_gpu": page.verified_tokens,
            "pages_per_gpu": 1}


class ReferenceSample:
    """The reference's CPU path over a page, one decoder layer per call.

    The oracle restates the reference's own ops (test infrastructure only):
    eager FlexAttention with the 128x64 block mask and ``repeat_kv``
    (D:72-135), the acceptance loop with KMP (D:1103-1336) and
    ``index_select`` compaction (D:1704-1723).  One :meth:`step` is the
    page's work divided by its decoder layers: the dense mask build, one
    layer's attention over every query row, that layer's K and V compaction
    (bf16) and the acceptance + KMP of every block; it is credited with
    ``verified_tokens / layers`` tokens.  The mask build and acceptance are
    charged in full on every call (about 0.05 % of a call)."""

    def __init__(self, page, seed=0):
        import torch

        from hsd_b200.workloads import segment_dicts
        from oracle import masks as OM

        self.page = page
        self.segs = segment_dicts(page)
        g = torch.Generator().manual_seed(seed)
        s = 1.0 / np.sqrt(page.head_dim)
        self.q = torch.randn(page.hq, page.q_len, page.head_dim, generator=g) * s
        self.k = torch.randn(page.hkv, page.kv_len, page.head_dim, generator=g) * s
        self.v = torch.randn(page.hkv, page.kv_len, page.head_dim, generator=g) * s
        self.kc = torch.randn(page.hkv, page.kv_len, page.head_dim,
                              generator=g).to(torch.bfloat16)
        self.vc = torch.randn(page.hkv, page.kv_len, page.head_dim,
                              generator=g).to(torch.bfloat16)
        self.allowed = OM.segments_to_allowed(page.q_len, page.kv_len, self.segs)
        self.tokens_per_step = page.verified_tokens / page.layers

    def step(self):
        import torch

        from oracle import accept as OA
        from oracle import attention as OAtt
        from oracle import compact as OC
        from oracle import masks as OM

        page = self.page
        parts = {}
        t0 = time.perf_counter()
        allowed = OM.segments_to_allowed(page.q_len, page.kv_len, self.segs)
        t1 = time.perf_counter()
        OAtt.flex_attention_eager(self.q, self.k, self.v, allowed)
        t2 = time.perf_counter()
        cfg = OA.StepConfig(pad_token_id=-1, eos_token_ids=(2**31 - 1,), tight_pack=True)
        filt = np.zeros(page.kv_len, bool)
        base = page.kv_len - page.q_len
        nxt, ids = page.next_ids.tolist(), page.input_ids.tolist()
        pointers = []
        for sg in page.segments:
            st = OA.BlockState(mode=OA.SPEC, gen=list(sg.gen), draft=list(sg.draft), mws=3,
                               matches_len=1, valid_count=sg.q_len)
            ptr, _, _, fin = OA.accept_block(st, sg.q_start, sg.q_start + sg.q_len, nxt, ids,
                                             cfg, filt, base, lambda r: allowed[r], False)
            if not fin:
                pointers.append(ptr)
                OA.realign_block(st, cfg)
        t3 = time.perf_counter()
        it = torch.as_tensor(OC.keep_indices(OC.keep_columns(allowed, pointers, filt)))
        self.kc.index_select(-2, it)
        self.vc.index_select(-2, it)
        t4 = time.perf_counter()
        parts = {"mask_build_s": t1 - t0, "attention_layer_s": t2 - t1,
                 "accept_kmp_s": t3 - t2, "compaction_layer_s": t4 - t3}
        return t4 - t0, parts

    def sample_text(self):
        p = self.page
        return (f"1/{p.layers} of a page step per step: dense mask build, one layer's eager "
                f"FlexAttention over all {p.q_len} query rows x {p.kv_len} columns, that "
                f"layer's index_select compaction of K and V, acceptance + KMP of all "
                f"{len(p.segments)} blocks; credited {p.verified_tokens}/{p.layers} tokens")


def cpu_parity_check(step, page):
    """Outputs of the timed device step against the oracle (CPU, fp32):
    attention of the first and last layer within max-abs 2e-2 / mean-abs
    2e-3, the per-block result rows (pointer, increment, finished) and the
    kept-column count bit-exact.  Runs after the timed region, on rank 0."""
    import torch

    from hsd_b200.accept import R
    from hsd_b200.workloads import segment_dicts
    from oracle import accept as OA
    from oracle import attention as OAtt
    from oracle import compact as OC
    from oracle import masks as OM

    allowed = OM.segments_to_allowed(page.q_len, page.kv_len, segment_dicts(page))
    mask = torch.as_tensor(allowed)
    errs = {}
    ok = True
    for l in (0, page.layers - 1):
        k = torch.cat([step.cache[l, 0, :, :page.prefix].cpu(), step.new_kv[l, 0].cpu()], 1)
        v = torch.cat([step.cache[l, 1, :, :page.prefix].cpu(), step.new_kv[l, 1].cpu()], 1)
        ref, _ = OAtt.attention_fp32(step.q[l].cpu(), k, v, mask)
        e = (step.out[l].float().cpu() - ref).abs()
        errs[f"layer{l}"] = {"max_abs": float(e.max()), "mean_abs": float(e.mean())}
        ok &= float(e.max()) <= 2e-2 and float(e.mean()) <= 2e-3
    cfg = OA.StepConfig(pad_token_id=-1, eos_token_ids=(2**31 - 1,), tight_pack=True)
    filt = np.zeros(page.kv_len, bool)
    base = page.kv_len - page.q_len
    nxt, ids = page.next_ids.tolist(), page.input_ids.tolist()
    rows, active = [], []
    for sg in page.segments:
        st = OA.BlockState(mode=OA.SPEC, gen=list(sg.gen), draft=list(sg.draft), mws=3,
                           matches_len=1, valid_count=sg.q_len)
        ptr, _, inc, fin = OA.accept_block(st, sg.q_start, sg.q_start + sg.q_len, nxt, ids,
                                           cfg, filt, base, lambda r: allowed[r], False)
        rows.append((ptr, inc, int(bool(fin))))
        if not fin:
            active.append(ptr)
    res = step.results.cpu().numpy()
    got = [(int(r[R["pointer"]]), int(r[R["increment"]]), int(r[R["finished"]])) for r in res]
    n_keep = len(OC.keep_indices(OC.keep_columns(allowed, active, filt)))
    results_ok = got == rows and int(step.counts[0].item()) == n_keep
    return {"parity_checked": bool(ok and results_ok), "attention": errs,
            "results_bit_exact": bool(results_ok),
            "tolerance": {"max_abs": 2e-2, "mean_abs": 2e-3},
            "oracle": "fp32 masked softmax attention, restated acceptance + keep rule"}


def run_reference(args):
    import torch
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return 0
    # torchrun sets OMP_NUM_THREADS=1; the reference arm uses every host core
    torch.set_num_threads(os.cpu_count() or 1)
    from hsd_b200 import workloads as W
    page = W.WORKLOADS[args.workload](seed=0)
    ref = ReferenceSample(page)
    for _ in range(args.warmup):
        ref.step()
    times, parts = [], None
    t_wall = time.perf_counter()
    for _ in range(args.steps):
        t, parts = ref.step()
        times.append(t)
    wall = time.perf_counter() - t_wall
    per_step = sum(times) / len(times)
    value = ref.tokens_per_step / per_step
    cores = torch.get_num_threads()
    line = {
        "impl": "reference", "metric": "verified_draft_tokens_per_s", "value": value,
        "unit": "tokens/s", "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": per_step * 1e3, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": page_config(page),
        "timed_region_s": wall,
        "cpu_baseline": {"value": value, "unit": "tokens/s", "cores": cores,
                         "kind": "port", "sample": ref.sample_text(), "parts": parts,
                         "os_cpu_count": os.cpu_count()},
        "e2e": {"value": value, "unit": "tokens/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


# ---------------------------------------------------------------- GPU side
def measure_next_tokens(page, dev, steps, warmup, seed=0):
    """Fused lm_head + argmax on the page's packed rows (hidden = Hq x head
    dim: 1536, the dots.ocr decoder's, on the stage-1 workload; the
    151,936-token vocabulary), against the reference's two ops on the same
    device: ``F.linear`` (cuBLAS bf16, fp32 accumulation, bf16 logits)
    then ``argmax(-1)``.  The weight (467 MB) exceeds L2, so no flush."""
    import torch

    from hsd_b200.lm_head import lm_head_argmax
    from hsd_b200.workloads import VOCAB

    q, hd = page.q_len, page.hq * page.head_dim
    g = torch.Generator(device=dev).manual_seed(1000 + seed)
    h = torch.randn(q, hd, generator=g, device=dev).to(torch.bfloat16)
    w = (torch.randn(VOCAB, hd, generator=g, device=dev) / hd ** 0.5).to(torch.bfloat16)
    out = torch.empty(q, dtype=torch.int64, device=dev)
    n = max(5, min(steps, 50))

    def timed(fn):
        for _ in range(max(3, warmup)):
            fn()
        torch.cuda.synchronize()
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(n):
            fn()
        e1.record()
        torch.cuda.synchronize()
        return e0.elapsed_time(e1) / n

    ours_ms = timed(lambda: lm_head_argmax(h, w, out=out))
    ref_ms = timed(lambda: torch.nn.functional.linear(h, w).argmax(-1))
    agree = float((out == torch.nn.functional.linear(h, w).argmax(-1)).float().mean())
    flops = 2.0 * q * VOCAB * hd
    # HunYuan SPEC_MODE=topk / adaptive: the rank pass over one region
    # block's rows (512, the draft cap), against the reference's
    # F.linear + topk(3) on the same rows
    from hsd_b200.lm_head import lm_head_rank
    rr = min(512, q)
    hr = h[q - rr:]
    ids32 = out[q - rr:].to(torch.int32)
    ref_col = torch.randint(0, VOCAB, (rr,), generator=g, device=dev, dtype=torch.int32)
    probe = torch.nn.functional.linear(hr, w).float()[torch.arange(rr, device=dev),
                                                      ref_col.long()].contiguous()
    rank_ms = timed(lambda: lm_head_rank(hr, w, probe, ref_col, ids32))
    topk_ms = timed(lambda: torch.nn.functional.linear(hr, w).topk(3, dim=-1))
    del h, w
    return {"kernel": "lm_head_argmax_kernel", "rows": q, "hidden": hd, "vocab": VOCAB,
            "launches": n, "ms": ours_ms, "tflops": flops / (ours_ms * 1e-3) / 1e12,
            "torch_linear_argmax_ms": ref_ms, "speedup_vs_torch": ref_ms / ours_ms,
            "ids_agree_with_torch": agree,
            "logits_bytes_not_written": q * VOCAB * 2,
            "rank_pass": {"rows": rr, "ms": rank_ms,
                          "tflops": 2.0 * rr * VOCAB * hd / (rank_ms * 1e-3) / 1e12,
                          "torch_linear_topk3_ms": topk_ms}}


def measure_rope_append(page, dev, steps, warmup, seed=0):
    """Fused RoPE + cache update of one step's new rows on every layer,
    against the reference's ops on the same device: transformers'
    ``apply_rotary_pos_emb`` on the query / key states and ``torch.cat`` of
    key and value states onto the layer cache (DynamicCache.update).  q / k /
    v are column slices of one fused projection output; the cache holds the
    page prefix and receives the step's rows after it."""
    import torch
    from transformers.models.qwen2.modeling_qwen2 import apply_rotary_pos_emb

    from hsd_b200.rope import rope_append

    n, hq, hkv, L = page.q_len, page.hq, page.hkv, page.layers
    g = torch.Generator(device=dev).manual_seed(2000 + seed)
    qkv = torch.randn(L, n, (hq + 2 * hkv) * 128, generator=g, device=dev).to(torch.bfloat16)
    pos = torch.arange(page.prefix, page.prefix + n, device=dev).float()
    inv = 1.0 / 1e6 ** (torch.arange(0, 128, 2, device=dev).float() / 128)
    emb = torch.cat([pos[:, None] * inv, pos[:, None] * inv], dim=-1)
    cos, sin = emb.cos().to(torch.bfloat16), emb.sin().to(torch.bfloat16)
    kc = torch.zeros(L, hkv, page.kv_len, 128, dtype=torch.bfloat16, device=dev)
    vc = torch.zeros_like(kc)
    prev_k = torch.randn(L, 1, hkv, page.prefix, 128, generator=g, device=dev).to(torch.bfloat16)
    prev_v = torch.randn_like(prev_k)
    a, b = hq * 128, (hq + hkv) * 128
    n_iter = max(5, min(steps, 50))

    def ours():
        for l in range(L):
            rope_append(qkv[l, :, :a], qkv[l, :, a:b], qkv[l, :, b:], cos, sin, kc[l], vc[l],
                        page.prefix)

    def floor():
        # the same launches on one row each: what a launch costs in the graph
        # (launch, programmatic wait on the previous kernel, ramp) with no data
        for l in range(L):
            rope_append(qkv[l, :1, :a], qkv[l, :1, a:b], qkv[l, :1, b:], cos[:1], sin[:1], kc[l],
                        vc[l], page.prefix)

    def ref():
        for l in range(L):
            q4 = qkv[l, :, :a].reshape(1, n, hq, 128).transpose(1, 2)
            k4 = qkv[l, :, a:b].reshape(1, n, hkv, 128).transpose(1, 2)
            v4 = qkv[l, :, b:].reshape(1, n, hkv, 128).transpose(1, 2)
            qe, ke = apply_rotary_pos_emb(q4, k4, cos[None], sin[None])
            torch.cat([prev_k[l], ke], dim=-2)
            torch.cat([prev_v[l], v4], dim=-2)

    def timed(fn):
        # both paths as CUDA graphs of their per-layer launches, so the
        # device time is measured rather than Python's per-call overhead
        fn()
        torch.cuda.synchronize()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            fn()
        for _ in range(max(3, warmup)):
            graph.replay()
        torch.cuda.synchronize()
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(n_iter):
            graph.replay()
        e1.record()
        torch.cuda.synchronize()
        del graph
        return e0.elapsed_time(e1) / n_iter

    ours_ms, ref_ms, floor_ms = timed(ours), timed(ref), timed(floor)
    per_row = hq * 256 * 2 + hkv * 256 * 2 * 2 + 2 * 256  # q r/w, k and v r/w, cos + sin
    algo = n * per_row
    return {"kernel": "rope_append_kernel", "rows": n, "layers": L, "launches_per_step": L,
            "timing": "CUDA graph of the 28 per-layer launches (both paths)",
            "ms_all_layers": ours_ms, "us_per_launch": ours_ms * 1e3 / L,
            "bytes_per_launch": algo,
            "achieved_gbs": algo / (ours_ms * 1e-3 / L) / 1e9,
            "torch_rope_cat_ms_all_layers": ref_ms, "speedup_vs_torch": ref_ms / ours_ms,
            "launch_floor_us": floor_ms * 1e3 / L,
            "achieved_gbs_beyond_floor": algo / max((ours_ms - floor_ms) * 1e-3 / L, 1e-9) / 1e9}


def measure_compaction(step, steps, warmup, copies=4):
    """The compaction launch timed alone, as the attention is: a CUDA graph
    of back-to-back ``hsd_compact_kv`` launches over every layer's K and V
    planes, rotating over ``copies`` scratch copies of the step's cache so
    that consecutive launches touch different memory (together larger than
    the 126 MB L2: each launch reads its rows from HBM), with the step's keep
    indices (every launch moves the same rows, so each does the step's
    algorithmic traffic).  Returns ms per launch."""
    import ctypes as C

    import torch

    from hsd_b200 import _native as N

    lib = N.load()
    scratch = [step.cache.clone() for _ in range(copies)]
    tables = [torch.tensor([c[l, kv, h].data_ptr() for l in range(step.L) for kv in range(2)
                            for h in range(step.hkv)], dtype=torch.int64, device=c.device)
              for c in scratch]
    status = torch.zeros(1, dtype=torch.int32, device=step.cache.device)
    p = lambda t: C.c_void_p(t.data_ptr())

    def launch(i):
        t = tables[i % copies]
        N.check(lib.hsd_compact_kv(p(t), t.numel(), step.row_bytes, p(step.keep_idx), -1,
                                   p(step.counts), p(status), N.stream_handle()),
                "hsd_compact_kv")
    n = copies * max(3, min(steps, 40) // copies)
    for i in range(copies):
        launch(i)
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        for i in range(n):
            launch(i)
    for _ in range(max(3, warmup)):
        graph.replay()
    torch.cuda.synchronize()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(5):
        graph.replay()
    e1.record()
    torch.cuda.synchronize()
    if int(status.item()):
        raise N.HSDError(f"device status 0x{int(status.item()):x} in the compaction timing")
    del graph, scratch
    return e0.elapsed_time(e1) / (5 * n)


def measure_h2d_link(dev, nbytes=256 << 20, reps=10):
    """Plain pinned host -> device copy bandwidth of this rank's link (GB/s):
    the bound of the end-to-end step, whose inputs cross it every step."""
    import torch
    h = torch.empty(nbytes, dtype=torch.uint8).pin_memory()
    d = torch.empty(nbytes, dtype=torch.uint8, device=dev)
    d.copy_(h, non_blocking=True)
    torch.cuda.synchronize()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(reps):
        d.copy_(h, non_blocking=True)
    e1.record()
    torch.cuda.synchronize()
    return nbytes * reps / (e0.elapsed_time(e1) * 1e-3) / 1e9


def measure_trees(page, dev, steps, warmup, depth=15, cap=256):
    """Continuation trees of every block of the page in one launch (root =
    the block's last generated token), against the oracle's restatement of
    the reference's host code (kmp_search's trie insertion + BFS packing,
    D:573-586, D:1488-1543) on one host core."""
    import torch

    from hsd_b200.trie import continuation_trees
    from oracle import kmp as OK

    drafts = [list(map(int, sg.draft)) for sg in page.segments]
    roots = [int(sg.gen[-1]) if len(sg.gen) else int(sg.draft[0]) for sg in page.segments]
    off = np.cumsum([0] + [len(d) for d in drafts[:-1]]).tolist()
    t = lambda x: torch.tensor(x, dtype=torch.int32, device=dev)
    pool, d_off, d_len, d_root = t(sum(drafts, [])), t(off), t([len(d) for d in drafts]), \
        t(roots)
    n = max(5, min(steps, 100))
    for _ in range(max(3, warmup)):
        continuation_trees(pool, d_off, d_len, d_root, depth, cap)
    torch.cuda.synchronize()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(n):
        trees = continuation_trees(pool, d_off, d_len, d_root, depth, cap)
    e1.record()
    torch.cuda.synchronize()
    dev_ms = e0.elapsed_time(e1) / n
    got = trees.host()
    t0 = time.perf_counter()
    want = []
    for d, r in zip(drafts, roots):
        trie, _ = OK.find_all_matches_kmp([d], [r], OK.compute_lps([r]), depth)
        want.append(OK.trie_bfs(trie, cap))
    cpu_ms = (time.perf_counter() - t0) * 1e3
    same = all(g == (list(w[0]), list(w[1]), list(w[2])) for g, w in zip(got, want))
    return {"kernel": "trie_kernel", "trees": len(drafts), "depth": depth, "cap": cap,
            "nodes": int(sum(len(g[0]) for g in got)), "ms": dev_ms,
            "host_python_ms": cpu_ms, "equal_to_oracle": same,
            "timing": "CUDA events around back-to-back launches (includes the launch)"}


def measure_loop(page, dev, iters=30):
    """The verification loop's own cost per iteration: ``VerifyLoop.inputs``
    + ``step`` (device tile plan, acceptance + KMP, keep / compaction rule, the
    8-int result rows to the host and the host packing of the next inputs),
    on the page's drafts with 64-token seeded prompts.  The target model is
    replaced by a stand-in on the device (each packed row predicts the next
    packed input token, so a speculative block accepts its whole draft
    slice); its time is excluded."""
    import torch

    from hsd_b200.loop import VerifyLoop
    from hsd_b200.workloads import EOS_ID

    rng = np.random.default_rng(7)
    drafts = [list(map(int, sg.draft)) for sg in page.segments]
    prompts = [[int(x) for x in rng.integers(1, 150000, 64)] for _ in drafts]
    loop = VerifyLoop(prompts, drafts, eos_token_id=EOS_ID, max_new_tokens=10 ** 7,
                      kv_capacity=65536, track_kv_tokens=False, device=dev)
    times, rows, tokens = [], [], []
    for _ in range(iters + 3):
        t0 = time.perf_counter()
        ids, pos, mask = loop.inputs()
        nxt = torch.roll(ids, -1)                 # the stand-in target model
        before = loop.new_tokens
        more = loop.step(nxt)
        torch.cuda.synchronize(dev)
        times.append(time.perf_counter() - t0)
        rows.append(int(ids.numel()))
        tokens.append(loop.new_tokens - before)
        if not more:
            break
    t, r, k = times[3:], rows[3:], tokens[3:]   # first iterations: setup, allocation
    if not t:
        return None
    return {"blocks": len(drafts), "iterations": len(t),
            "ms_per_iteration": 1e3 * sum(t) / len(t),
            "packed_rows_per_iteration": sum(r) / len(r),
            "new_tokens_per_iteration": sum(k) / len(k),
            "timing": "host wall clock around inputs() + step(), device synchronised"}


def measure_multi_page(args, world, rank, dev):
    """The multi-page throughput run: ``args.multi_pages`` seeded pages (region
    counts U[8, 64], prefix lengths U[1024, 4096], 28 layers) shared out over
    the ranks by LPT on the estimated tile work, every rank verifying its pages
    one after another with one page resident at a time, and the per-page result
    rows gathered to rank 0.  Per page: its buffers are built (device RNG, not
    timed), one untimed step, then ``reps`` steps bracketed by CUDA events;
    a rank's time is the sum of its pages' timed steps.  ``value`` = tokens of
    all pages x reps / the slowest rank's time (fixed page set: strong
    scaling).  Returns the section on rank 0, None elsewhere."""
    import torch
    import torch.distributed as dist

    from hsd_b200 import sharding as S
    from hsd_b200 import workloads as W
    from hsd_b200.verify_step import VerifyStep

    n_pages = int(args.multi_pages)
    if n_pages <= 0:
        return None
    reps = 3
    costs = [S.page_cost(W.multi_page(i)) for i in range(n_pages)]
    mine = S.shard_pages(costs, world)[rank]
    dev_ms, tokens, results = 0.0, 0.0, {}
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    status_ok = True
    for i in mine:
        page = W.multi_page(i)
        st = VerifyStep(page, device=dev, seed=i, device_rng=True)
        st.run()
        torch.cuda.synchronize()
        e0.record()
        for _ in range(reps):
            st.run()
        e1.record()
        torch.cuda.synchronize()
        dev_ms += e0.elapsed_time(e1)
        tokens += reps * page.verified_tokens
        status_ok &= int(st.status.item()) == 0
        results[i] = st.results.reshape(-1).to(torch.int64).clone()
        del st
    stats = torch.tensor([dev_ms, tokens, float(sum(costs[i] for i in mine)), len(mine),
                          float(status_ok)], dtype=torch.float64, device=dev)
    per_rank = [stats]
    if world > 1:
        per_rank = [torch.zeros_like(stats) for _ in range(world)]
        dist.all_gather(per_rank, stats)
        gathered = S.gather_page_results(results, n_pages, dst=0, device=dev)
    else:
        gathered = results
    if rank != 0:
        return None
    ms_max = max(float(t[0]) for t in per_rank)
    slow = max(range(world), key=lambda r: float(per_rank[r][0]))
    tok = sum(float(t[1]) for t in per_rank)
    return {"metric": "verified_draft_tokens_per_s", "value": tok / (ms_max * 1e-3),
            "unit": "tokens/s", "scaling": "strong", "pages": n_pages,
            "steps_per_page": reps,
            "workload": "multi_page: region counts U[8,64], prefix U[1024,4096], 28 layers, "
                        "12/2 heads (seeded)",
            "sharding": "LPT on estimated tile work (sharding.shard_pages)",
            "device_ms_slowest_rank": ms_max, "slowest_rank": slow,
            "per_rank": [{"rank": r, "device_ms": float(t[0]), "tokens": float(t[1]),
                          "estimated_cost": float(t[2]), "pages": int(t[3]),
                          "status_ok": bool(t[4])} for r, t in enumerate(per_rank)],
            "pages_gathered_on_rank0": len(gathered) if gathered is not None else 0,
            "timing": "per page: CUDA events around its timed steps (plain launches); page "
                      "set-up between pages is not timed"}


def run_ours(args):
    import torch
    import torch.distributed as dist

    from hsd_b200 import workloads as W
    from hsd_b200.verify_step import VerifyStep

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world != args.gpus:
        raise SystemExit(f"--gpus {args.gpus} but WORLD_SIZE={world}")
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        import datetime
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=dev)
    # every rank verifies a page of the same shape (tile structure, drafts,
    # acceptance) with its own seeded Q / K / V: equal work per GPU, so the
    # weak-scaling curve measures the hardware, not page-size imbalance
    page = W.WORKLOADS[args.workload](seed=0)
    step = VerifyStep(page, device=dev, seed=rank)
    stream = torch.cuda.current_stream()
    for _ in range(args.warmup):
        step.run(stream)
    torch.cuda.synchronize()
    step.raise_on_device_error()

    # per-launch attention events of the timed steps (same stream)
    ev = [[[torch.cuda.Event(enable_timing=True) for _ in range(2)] for _ in range(step.L)]
          for _ in range(args.steps)]
    phases = ("append", "plan", "accept", "keep", "compact", "bits")
    pev = [{k: [torch.cuda.Event(enable_timing=True) for _ in range(2)] for k in phases}
           for _ in range(args.steps)]
    gpu_index = local
    vis = os.environ.get("CUDA_VISIBLE_DEVICES")
    if vis:
        try:
            gpu_index = int(vis.split(",")[local])
        except ValueError:
            pass
    # instrumented pass (plain launches with per-layer and per-phase events):
    # the per-launch attention time of the roofline and the phase breakdown
    torch.cuda.synchronize()
    for i in range(args.steps):
        step.run(stream, attn_events=ev[i], phase_events=pev[i])
    torch.cuda.synchronize()
    step.raise_on_device_error()

    # timed region: the whole step captured once as a CUDA graph and replayed
    graph = step.capture()
    for _ in range(args.warmup):
        graph.replay()
    torch.cuda.synchronize()
    step.raise_on_device_error()
    sampler = ClockSampler(gpu_index)
    sampler.start()
    time.sleep(0.3)
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    t_start = torch.cuda.Event(enable_timing=True)
    t_end = torch.cuda.Event(enable_timing=True)
    sampler.mark_start()
    t_start.record(stream)
    for i in range(args.steps):
        graph.replay()
    t_end.record(stream)
    torch.cuda.synchronize()
    sampler.mark_end()
    if world > 1:
        dist.barrier()
    clocks = sampler.stop()
    step.raise_on_device_error()
    ms = t_start.elapsed_time(t_end) / args.steps
    attn_ms = [ev[i][l][0].elapsed_time(ev[i][l][1]) for i in range(args.steps)
               for l in range(step.L)]
    attn_event_ms = sum(attn_ms) / len(attn_ms)
    breakdown = {k: sum(pev[i][k][0].elapsed_time(pev[i][k][1]) for i in range(args.steps))
                 / args.steps for k in phases}
    breakdown["attention_all_layers"] = attn_event_ms * step.L

    # attention launch time for the roofline: the step's attention launches
    # alone, as a graph of back-to-back launches, over the same step count
    graph_attn = step.capture(attention_only=True)
    for _ in range(args.warmup):
        graph_attn.replay()
    torch.cuda.synchronize()
    a0 = torch.cuda.Event(enable_timing=True)
    a1 = torch.cuda.Event(enable_timing=True)
    a0.record(stream)
    for _ in range(args.steps):
        graph_attn.replay()
    a1.record(stream)
    torch.cuda.synchronize()
    attn_avg_ms = a0.elapsed_time(a1) / (args.steps * step.L)
    comp_bytes, comp_moved, comp_kept = step.compaction_bytes()
    comp_ms = measure_compaction(step, args.steps, args.warmup)

    # end to end: pinned host inputs in, results out, every step (graph
    # replay; one replay = E2E_STEPS consecutive steps on alternating input
    # sets, so the link idles only once per replay)
    step.host_buffers()
    step.run_from_host(stream, buffers=0)
    step.run_from_host(stream, buffers=1)
    graph_e2e = step.capture(from_host=True, host_steps=E2E_STEPS)
    for _ in range(max(1, args.warmup)):
        graph_e2e.replay()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    n_e2e = max(1, args.steps // E2E_STEPS)
    e0.record(stream)
    for _ in range(n_e2e):
        graph_e2e.replay()
    e1.record(stream)
    torch.cuda.synchronize()
    step.raise_on_device_error()
    e2e_ms = e0.elapsed_time(e1) / (E2E_STEPS * n_e2e)
    link_gbs = measure_h2d_link(dev)

    next_tokens = measure_next_tokens(page, dev, args.steps, args.warmup, seed=rank)
    rope = measure_rope_append(page, dev, args.steps, args.warmup, seed=rank)
    trees = measure_trees(page, dev, args.steps, args.warmup)
    loop_cost = measure_loop(page, dev)

    tokens = float(page.verified_tokens)
    stats = torch.tensor([ms, e2e_ms, tokens, attn_avg_ms], dtype=torch.float64, device=dev)
    per_rank = [stats]
    if world > 1:
        per_rank = [torch.zeros_like(stats) for _ in range(world)]
        dist.all_gather(per_rank, stats)
    ms = max(float(t[0]) for t in per_rank)
    e2e_ms = max(float(t[1]) for t in per_rank)
    tokens = sum(float(t[2]) for t in per_rank)
    flops_exec, flops_pairs, tiles, pairs = step.attention_flops()
    multi = measure_multi_page(args, world, rank, dev)
    if rank == 0:
        peaks, peaks_src = load_peaks()
        # the attention is timed alone (a graph of its launches): burst peak
        peak = peaks.get("bf16_tflops", FALLBACK_PEAKS["bf16_tflops"])
        peak_sus = peaks.get("bf16_tflops_sustained", FALLBACK_PEAKS["bf16_tflops_sustained"])
        achieved = flops_exec / (attn_avg_ms * 1e-3) / 1e12
        line = {
            "metric": "verified_draft_tokens_per_s", "value": tokens / (ms * 1e-3),
            "unit": "tokens/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": ms, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
            "config": page_config(page),
            "timing": {"parallelism": f"page-sharded x{world} (no hot-path collective)",
                       "launch": f"one CUDA graph per step "
                                 f"({step.kernel_launches_per_step} kernels)",
                       "l2": "inputs exceed L2 (all layers' Q/K/V per step, no flush needed)",
                       "per_rank": [{"rank": r, "ms_per_step": float(t[0]),
                                     "e2e_ms_per_step": float(t[1]), "tokens": float(t[2]),
                                     "attention_ms_per_launch": float(t[3])}
                                    for r, t in enumerate(per_rank)]},
            "roofline": {"bound": "tensor", "achieved": achieved, "peak": peak,
                         "unit": "TFLOP/s", "frac": achieved / peak,
                         "peak_source": f"{peaks_src} bf16_tflops (burst: the attention "
                                        f"launches are timed alone)",
                         "frac_of_sustained": achieved / peak_sus,
                         "kernel": "verify_attn_kernel",
                         "flops_per_launch": flops_exec, "executed_tiles_128x64": tiles,
                         "allowed_pairs": pairs,
                         "pair_flops_tflops": flops_pairs / (attn_avg_ms * 1e-3) / 1e12,
                         "avg_launch_ms": attn_avg_ms,
                         "avg_launch_ms_single_events": attn_event_ms,
                         "traffic": profile_traffic("verify_attn_stage1_regions")},
            "e2e": {"value": tokens / (e2e_ms * 1e-3), "unit": "tokens/s",
                    "h2d_bytes_per_step": step.h2d_bytes(),
                    "d2h_bytes_per_step": step.d2h_bytes(),
                    "h2d_gbs_per_rank": step.h2d_bytes() / (e2e_ms * 1e-3) / 1e9,
                    "h2d_link_gbs_rank0": link_gbs,
                    "link_bound_tokens_per_s_per_rank":
                        page.verified_tokens / (step.h2d_bytes() / (link_gbs * 1e9)),
                    "timing": f"graph of {E2E_STEPS} consecutive steps on alternating "
                              "device input sets; every layer's query and new K/V rows copied from "
                              "pinned host memory on a copy stream, each layer's append and "
                              "attention waiting for its own rows; results and counts "
                              "copied back every step"},
            "breakdown_ms_per_step": breakdown,
            "latency_bound": {
                "accept_kmp_us": breakdown["accept"] * 1e3,
                "blocks": step.n_blocks,
                "blocks_per_s": step.n_blocks / (breakdown["accept"] * 1e-3),
                "plan_us": breakdown["plan"] * 1e3,
                "query_tiles": int(step.plan.struct.n_qtiles),
                "segments_per_s": len(page.segments) / (breakdown["plan"] * 1e-3)},
            "compaction": {"bound": "hbm", "bytes_per_launch": comp_bytes,
                           "rows_moved": comp_moved, "rows_kept": comp_kept,
                           "planes": int(step.planes.numel()),
                           "avg_launch_ms": comp_ms,
                           "timing": "CUDA graph of back-to-back launches on a scratch copy "
                                     "of the cache (the attention's method); the step's "
                                     "own event pair, launch latency included: "
                                     f"{breakdown['compact']:.4f} ms",
                           "achieved_gbs": comp_bytes / (comp_ms * 1e-3) / 1e9,
                           "peak_gbs": peaks.get("hbm_gbs", FALLBACK_PEAKS["hbm_gbs"]),
                           "frac": comp_bytes / (comp_ms * 1e-3) / 1e9
                           / peaks.get("hbm_gbs", FALLBACK_PEAKS["hbm_gbs"]),
                           "frac_in_step": comp_bytes / (breakdown["compact"] * 1e-3) / 1e9
                           / peaks.get("hbm_gbs", FALLBACK_PEAKS["hbm_gbs"]),
                           "traffic": profile_traffic("compact_kv_stage1_regions")},
            "gpu_launches": args.steps * step.kernel_launches_per_step,
            "gpu_launches_e2e_region": E2E_STEPS * n_e2e * step.kernel_launches_per_host_step,
            "clocks": clocks,
            "next_tokens": dict(next_tokens, peak_tflops=peak,
                                frac=next_tokens["tflops"] / peak,
                                frac_of_sustained=next_tokens["tflops"] / peak_sus,
                                traffic=profile_traffic("lm_head_argmax_stage1_rows")),
            "trees": trees,
            "loop": loop_cost,
            "rope_append": dict(rope, peak_gbs=peaks.get("hbm_gbs", FALLBACK_PEAKS["hbm_gbs"]),
                                traffic=profile_traffic("rope_append_stage1_rows"),
                                frac=rope["achieved_gbs"]
                                / peaks.get("hbm_gbs", FALLBACK_PEAKS["hbm_gbs"]),
                                frac_beyond_floor=rope["achieved_gbs_beyond_floor"]
                                / peaks.get("hbm_gbs", FALLBACK_PEAKS["hbm_gbs"])),
        }
        if multi is not None:
            line["multi_page"] = multi
        if world == 1 and not args.no_cpu_baseline:
            line["parity"] = cpu_parity_check(step, page)
            torch.set_num_threads(os.cpu_count() or 1)
            ref = ReferenceSample(page)
            ref.step()  # first-call setup of eager FlexAttention
            ts = [ref.step() for _ in range(2)]
            t = sum(x[0] for x in ts) / len(ts)
            line["cpu_baseline"] = {
                "value": ref.tokens_per_step / t, "unit": "tokens/s",
                "cores": torch.get_num_threads(), "kind": "port",
                "sample": ref.sample_text() + "; 2 calls after 1 warm-up",
                "parts": ts[-1][1]}
        print(json.dumps(line), flush=True)
    del graph, graph_e2e, graph_attn
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    return 0


def run_pages(args):
    """Multi-page mode: ``--pages K`` seeded pages of the multi-page shape
    (region count U[8, 64], prefix U[1024, 4096]) are shared out over the
    ranks by LPT on the estimated tile work; every timed iteration verifies
    one step of every page, each rank its own pages one after another (one
    CUDA graph per page).  ``value`` = tokens of all pages / the slowest
    rank's time; the page set is fixed, so the scaling is strong.  The
    per-page results are gathered to rank 0 afterwards (not timed)."""
    import torch
    import torch.distributed as dist

    from hsd_b200 import sharding as S
    from hsd_b200 import workloads as W
    from hsd_b200.verify_step import VerifyStep

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world != args.gpus:
        raise SystemExit(f"--gpus {args.gpus} but WORLD_SIZE={world}")
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        import datetime
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=dev)
    pages = [W.multi_page(i) for i in range(args.pages)]
    costs = [S.page_cost(p) for p in pages]
    mine = S.shard_pages(costs, world)[rank]
    steps = {i: VerifyStep(pages[i], device=dev, seed=i, device_rng=True) for i in mine}
    graphs = {}
    for i, st in steps.items():
        for _ in range(args.warmup):
            st.run()
        torch.cuda.synchronize()
        st.raise_on_device_error()
        graphs[i] = st.capture()
    torch.cuda.synchronize()
    n_iter = max(3, min(args.steps, 50))
    for _ in range(args.warmup):
        for i in mine:
            graphs[i].replay()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(n_iter):
        for i in mine:
            graphs[i].replay()
    e1.record()
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / n_iter
    for st in steps.values():
        st.raise_on_device_error()
    tokens = float(sum(pages[i].verified_tokens for i in mine))
    stats = torch.tensor([ms, tokens, float(sum(costs[i] for i in mine))], dtype=torch.float64,
                         device=dev)
    per_rank = [torch.zeros_like(stats) for _ in range(world)]
    if world > 1:
        dist.all_gather(per_rank, stats)
    else:
        per_rank = [stats]
    # per-page results (8 int32 per block) to rank 0, as a serving job would
    results = {i: steps[i].results.reshape(-1).to(torch.int64) for i in mine}
    gathered = S.gather_page_results(results, args.pages, dst=0, device=dev) if world > 1 \
        else results
    if rank == 0:
        ms_max = max(float(t[0]) for t in per_rank)
        tok = sum(float(t[1]) for t in per_rank)
        line = {
            "metric": "verified_draft_tokens_per_s", "value": tok / (ms_max * 1e-3),
            "unit": "tokens/s", "n_gpus": world, "steps": n_iter, "warmup": args.warmup,
            "ms_per_step": ms_max, "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
            "config": {"workload": "multi_page", "pages": args.pages,
                       "parallelism": f"LPT page sharding x{world} (no hot-path collective)",
                       "launch": "one CUDA graph per page step",
                       "per_rank": [{"ms": float(t[0]), "tokens": float(t[1]),
                                     "estimated_cost": float(t[2])} for t in per_rank]},
            "pages_gathered": len(gathered),
        }
        print(json.dumps(line), flush=True)
    del graphs
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    return 0


def main():
    ap = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=300)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--workload", default="stage1_regions",
                    choices=["stage1_regions", "stage2_page", "hunyuan_regions"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--pages", type=int, default=0,
                    help="multi-page mode: this many seeded pages shared out over the ranks")
    ap.add_argument("--multi-pages", type=int, default=256,
                    help="pages of the multi-page section of the default run (0: skip)")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    if args.impl == "reference":
        return run_reference(args)
    if args.pages > 0:
        return run_pages(args)
    return run_ours(args)


if __name__ == "__main__":
    sys.exit(main())

"""Page-wise sharding across the GPUs of one node, and the result gather.

Pages of a document batch are independent verification problems (the
reference runs them one after another in one process, RD:346-410), so the
multi-GPU design has no collective on the hot path: every rank verifies its
own shard of pages on its own HBM, and only the per-page results travel to
rank 0 at the end (``torch.distributed`` over NCCL on GPUs, gloo on CPUs).

Sharding is size-balanced: pages are assigned longest-first to the rank with
the least estimated work (LPT), with the verification-attention tile count as
the cost estimate.
"""
from __future__ import annotations

import heapq

import torch
import torch.distributed as dist


def page_cost(page) -> int:
    """Estimated verification work of a page: 128x64 tiles of its packed mask
    times query heads (the attention dominates a step)."""
    prefix = page.prefix
    rows = page.q_len
    # every query row sees the prefix plus at most its own group's columns
    tiles = -(-rows // 128) * (-(-prefix // 64) + 2)
    return tiles * page.hq * page.layers


def shard_pages(costs, world: int):
    """LPT assignment: list (per rank) of page indices, ascending.

    Deterministic: ties on cost break by page index, ties on load by rank.
    """
    if world <= 0:
        raise ValueError("world must be positive")
    order = sorted(range(len(costs)), key=lambda i: (-costs[i], i))
    heap = [(0, r) for r in range(world)]
    heapq.heapify(heap)
    shards = [[] for _ in range(world)]
    for i in order:
        load, r = heapq.heappop(heap)
        shards[r].append(i)
        heapq.heappush(heap, (load + costs[i], r))
    return [sorted(s) for s in shards]


def run_shard(pages, fn):
    """Verify this rank's pages one after another, as the reference's
    per-image loop does (hsd/hunyuan_ocr_pipeline/run_hunyuan_ocr_hsd.py
    RH:264-280): a page whose ``fn(page)`` raises is recorded as failed (its
    result is ``None``, its message kept) and the next page runs.

    Returns ``(results {page: 1-D int tensor or None}, errors {page: str})``.
    """
    results, errors = {}, {}
    for i in pages:
        try:
            results[i] = torch.as_tensor(fn(i), dtype=torch.int64).reshape(-1)
        except Exception as e:  # noqa: BLE001 -- any failure of one page
            results[i] = None
            errors[i] = f"{type(e).__name__}: {e}"
    return results, errors


def gather_page_results(local: dict, n_pages: int, dst: int = 0, device=None):
    """Gather ``{page_index: 1-D int tensor or None}`` from every rank to ``dst``.

    Variable-length results travel as (lengths, padded buffer): one gather of
    the per-page lengths, then one of the padded token buffers; a failed page
    (``None``) travels as length -2 and comes back as ``None``.  Returns the
    full ``{page_index: tensor or None}`` on ``dst`` and ``None`` elsewhere;
    a page that no rank reported raises on ``dst``.  Collectives that a dead
    rank never joins end with the process group's timeout error.
    """
    world = dist.get_world_size()
    rank = dist.get_rank()
    device = device or torch.device("cpu")
    idx = sorted(local)
    n_local = torch.tensor([len(idx)], dtype=torch.int64, device=device)
    counts = [torch.zeros_like(n_local) for _ in range(world)]
    dist.all_gather(counts, n_local)
    max_n = int(max(c.item() for c in counts))
    if max_n == 0:          # no rank holds a page: nothing more to gather
        if n_pages > 0 and rank == dst:
            raise RuntimeError(f"pages without results after the gather: "
                               f"{list(range(n_pages))[:8]}")
        return {} if rank == dst else None
    lens = torch.full((max_n, 2), -1, dtype=torch.int64, device=device)
    for j, i in enumerate(idx):
        lens[j, 0] = i
        lens[j, 1] = -2 if local[i] is None else local[i].numel()
    all_lens = [torch.zeros_like(lens) for _ in range(world)]
    dist.all_gather(all_lens, lens)
    max_len = max(1, int(max(t[:, 1].max().item() for t in all_lens)))
    buf = torch.zeros((max_n, max_len), dtype=torch.int64, device=device)
    for j, i in enumerate(idx):
        if local[i] is not None:
            buf[j, :local[i].numel()] = local[i].to(device=device, dtype=torch.int64)
    all_buf = [torch.zeros_like(buf) for _ in range(world)]
    dist.all_gather(all_buf, buf)
    if rank != dst:
        return None
    out = {}
    for lens_r, buf_r in zip(all_lens, all_buf):
        for j in range(max_n):
            page, n = int(lens_r[j, 0]), int(lens_r[j, 1])
            if page >= 0:
                out[page] = None if n == -2 else buf_r[j, :n].clone()
    missing = set(range(n_pages)) - set(out)
    if missing:
        raise RuntimeError(f"pages without results after the gather: {sorted(missing)[:8]}")
    return out

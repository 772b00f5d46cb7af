"""Page sharding and the rank-0 result gather, on CPU ranks over gloo."""
import os
import socket
import time

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from hsd_b200 import sharding as S


def test_lpt_sharding_covers_every_page_once_and_balances():
    costs = [((i * 7919) % 97) + 1 for i in range(256)]
    for world in (1, 2, 4, 8):
        shards = S.shard_pages(costs, world)
        flat = sorted(i for s in shards for i in s)
        assert flat == list(range(256))
        loads = [sum(costs[i] for i in s) for s in shards]
        assert max(loads) - min(loads) <= max(costs)


def test_sharding_is_deterministic():
    costs = [5, 5, 3, 3, 8, 1, 1, 9]
    assert S.shard_pages(costs, 3) == S.shard_pages(list(costs), 3)


def test_page_cost_orders_by_size():
    from hsd_b200 import workloads as W
    small, large = W.multi_page(0), W.multi_page(1)
    pages = sorted([small, large], key=lambda p: p.q_len * p.prefix)
    assert S.page_cost(pages[0]) <= S.page_cost(pages[1])


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _worker(rank, world, port, n_pages, q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        costs = [(i % 5) + 1 for i in range(n_pages)]
        mine = S.shard_pages(costs, world)[rank]
        # each page's "result" is a deterministic variable-length token list
        local = {i: torch.arange(i % 7 + 1) + 1000 * i for i in mine}
        out = S.gather_page_results(local, n_pages, dst=0)
        if rank == 0:
            q.put({k: v.tolist() for k, v in out.items()})
        else:
            q.put(None if out is None else "unexpected")
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world,n_pages", [(2, 11), (3, 11), (2, 1), (2, 0)])
def test_gather_to_rank0_over_gloo(world, n_pages):
    """Every page's result reaches rank 0, including with fewer pages than
    ranks (a rank with no page) and with no page at all (an empty dict)."""
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, n_pages, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = [q.get(timeout=120) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    gathered = [r for r in results if isinstance(r, dict)]
    assert len(gathered) == 1 and all(r is None for r in results if not isinstance(r, dict))
    got = gathered[0]
    assert sorted(got) == list(range(n_pages))
    for i in range(n_pages):
        assert got[i] == [1000 * i + t for t in range(i % 7 + 1)]


def _worker_failures(rank, world, port, n_pages, q):
    import datetime
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=20))
    try:
        mine = S.shard_pages([1] * n_pages, world)[rank]

        def verify(i):
            if i % 4 == 3:
                raise RuntimeError(f"page {i} could not be verified")
            return list(range(i + 1))

        local, errors = S.run_shard(mine, verify)
        out = S.gather_page_results(local, n_pages, dst=0)
        q.put((rank, None if out is None else {k: (None if v is None else v.tolist())
                                               for k, v in out.items()}, sorted(errors)))
    finally:
        dist.destroy_process_group()


def test_failed_pages_are_reported_and_the_rest_gathered():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port, world, n_pages = _free_port(), 2, 10
    procs = [ctx.Process(target=_worker_failures, args=(r, world, port, n_pages, q))
             for r in range(world)]
    for p in procs:
        p.start()
    results = sorted([q.get(timeout=120) for _ in range(world)], key=lambda x: x[0])
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    got = results[0][1]
    assert sorted(got) == list(range(n_pages))
    for i in range(n_pages):
        assert got[i] == (None if i % 4 == 3 else list(range(i + 1)))
    assert sorted(results[0][2] + results[1][2]) == [3, 7]


def _worker_dead_rank(rank, world, port, q):
    import datetime
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=5))
    if rank == 1:
        os._exit(0)  # leaves between steps, never joins the gather
    t0 = time.time()
    try:
        S.gather_page_results({0: torch.arange(3)}, 2, dst=0)
        q.put(("no error", time.time() - t0))
    except Exception as e:  # noqa: BLE001
        q.put((type(e).__name__, time.time() - t0))


def test_dead_rank_ends_the_gather_with_an_error():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker_dead_rank, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    kind, dt = q.get(timeout=120)
    for p in procs:
        p.join(timeout=60)
    assert kind != "no error" and dt < 60

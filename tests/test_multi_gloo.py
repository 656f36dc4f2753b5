"""The N>1 path on CPU: two gloo ranks each search their row shard (oracle stand-in for the
shard search), all-gather, merge, and must equal the single-process exact search."""

import os
import socket

import numpy as np
import pytest
import torch.multiprocessing as mp


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, n, d, nq, k, metric, out):
    import torch
    import torch.distributed as dist

    from oracle import oracle
    from vectoraccelerate_b200.sharded import ShardedSearch, merge_lists_host, shard_bounds

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        x = oracle.gen_gaussian(n, d, 0)
        q = oracle.gen_gaussian(nq, d, 1, row0=1 << 31)
        row0, nl = shard_bounds(n, world, rank)

        def local(nq_, k_):
            ids, vals = oracle.knn(q, x[row0:row0 + nl], k_, metric=metric)
            ids = np.where(ids == 0xFFFFFFFF, ids, ids + row0).astype(np.uint32)
            return torch.from_numpy(vals), torch.from_numpy(ids.view(np.int32))

        def merge(gv, gi):
            v, i = merge_lists_host(gv.numpy(), gi.numpy().view(np.uint32), 1 if metric == 2 else 0)
            return torch.from_numpy(v), torch.from_numpy(i.view(np.int32))

        fv, fi = ShardedSearch(world, local, merge).search(nq, k)
        if rank == 0:
            out.put((fv.numpy(), fi.numpy().view(np.uint32)))
    except Exception as e:  # surface worker failures to the test instead of a queue timeout
        out.put(e)
        raise
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world,metric,n", [(2, 0, 1001), (2, 2, 640), (3, 0, 500)])
def test_sharded_gather_merge_equals_single(world, metric, n):
    from oracle import oracle
    ctx = mp.get_context("spawn")
    out = ctx.Queue()
    port = _free_port()
    d, nq, k = 32, 17, 7
    procs = [ctx.Process(target=_worker, args=(r, world, port, n, d, nq, k, metric, out)) for r in range(world)]
    for p in procs:
        p.start()
    got = out.get(timeout=120)
    if isinstance(got, Exception):
        for p in procs:
            p.join(timeout=30)
        raise got
    fv, fi = got
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    x = oracle.gen_gaussian(n, d, 0)
    q = oracle.gen_gaussian(nq, d, 1, row0=1 << 31)
    tids, tvals = oracle.knn(q, x, k, metric=metric)
    assert np.array_equal(fi, tids)
    np.testing.assert_array_equal(fv, tvals)


def test_shard_bounds_cover_rows():
    from vectoraccelerate_b200.sharded import shard_bounds
    for n in (1, 7, 10_000_000, 50_000_001):
        for world in (1, 2, 3, 4, 8):
            if n < world:
                continue
            spans = [shard_bounds(n, world, r) for r in range(world)]
            assert spans[0][0] == 0
            for (a, na), (b, _) in zip(spans, spans[1:]):
                assert a + na == b
            assert spans[-1][0] + spans[-1][1] == n


# ------------------------------------------------------------------------------------------------ failures
def _join_or_fail(rank, world, port, mode, out):
    """mode 'never_joins': rank 1 exits without joining; 'raises': rank 1 joins, then raises before
    the gather. Rank 0 reports how its next step ended and after how long."""
    import time

    import torch
    import torch.distributed as dist
    from datetime import timedelta

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    if mode == "never_joins" and rank == 1:
        return
    t0 = time.time()
    try:
        dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=4))
        if mode == "raises" and rank == 1:
            dist.destroy_process_group()
            raise SystemExit(3)
        from vectoraccelerate_b200.sharded import ShardedSearch

        def local(nq, k):
            return torch.zeros((nq, k)), torch.zeros((nq, k), dtype=torch.int32)

        ShardedSearch(world, local, lambda gv, gi: (gv[0], gi[0])).search(4, 2)
        out.put(("completed", time.time() - t0))
    except Exception as e:  # the bounded error this test expects
        out.put((type(e).__name__, time.time() - t0))


@pytest.mark.parametrize("mode", ["never_joins", "raises"])
def test_missing_rank_gives_a_bounded_error(mode):
    ctx = mp.get_context("spawn")
    out = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_join_or_fail, args=(r, 2, port, mode, out)) for r in range(2)]
    for p in procs:
        p.start()
    what, seconds = out.get(timeout=120)
    for p in procs:
        p.join(timeout=60)
        if p.is_alive():
            p.kill()
    assert what != "completed", "rank 0 finished a collective without its peer"
    assert seconds < 60, f"rank 0 waited {seconds:.1f} s"

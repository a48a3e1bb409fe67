"""The multi-GPU host logic on CPU: two gloo ranks (world size 2)."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, q):
    import sys
    sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    import oracle
    from tiler_b200 import provider, sharding
    try:
        count = 1 << 18
        x = (np.random.default_rng(1).standard_normal(count) * 100).astype(np.float32)
        lo, hi = sharding.row_range(count, rank, world)  # contiguous contributor shard
        g = provider.plan_grid_grouping(1, hi - lo)

        def local_sum(t):
            st, y = oracle.grid_fold(t.numpy(), g)
            assert st == 0
            return torch.from_numpy(y)
        total = sharding.sum_across_ranks(torch.from_numpy(x[lo:hi].copy()), local_sum)

        m, k, n = 16, 32, 24
        rng = np.random.default_rng(2)
        a = torch.from_numpy(rng.standard_normal((m, k)).astype(np.float32))
        w = torch.from_numpy(rng.standard_normal((n, k)).astype(np.float32))
        c0, c1 = sharding.row_range(n, rank, world)
        c = sharding.gemm_n_sharded(a, w[c0:c1].contiguous(), lambda aa, ww: aa @ ww.t())
        q.put((rank, np.float32(total).view(np.uint32).item(), c.numpy(), g))
    except Exception as exc:  # report instead of leaving the peer waiting
        q.put((rank, None, repr(exc), None))
        raise
    finally:
        dist.destroy_process_group()


def test_two_rank_sum_and_n_sharded_contraction(oracle_lib):
    world, port = 2, _free_port()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = [q.get(timeout=120) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    results.sort(key=lambda r: r[0])
    assert all(r[1] is not None for r in results), results
    # the declared multi-GPU order: per-shard grid folds, then a strict fold in rank order
    count = 1 << 18
    x = (np.random.default_rng(1).standard_normal(count) * 100).astype(np.float32)
    partials = []
    for r in range(world):
        lo, hi = r * count // world, (r + 1) * count // world
        _, y = oracle_lib.grid_fold(x[lo:hi], results[r][3])
        partials.append(y[0])
    _, want = oracle_lib.strict_sum(np.array(partials, np.float32))
    assert results[0][1] == results[1][1] == np.float32(want[0]).view(np.uint32).item()
    # N-sharded contraction assembles the full product on every rank
    rng = np.random.default_rng(2)
    a = rng.standard_normal((16, 32)).astype(np.float32)
    w = rng.standard_normal((24, 32)).astype(np.float32)
    for r in range(world):
        np.testing.assert_allclose(results[r][2], a @ w.T, rtol=1e-5, atol=1e-5)

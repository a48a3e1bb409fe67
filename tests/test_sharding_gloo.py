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

        # the fused form's host logic: every rank's buffer mapped in rank order,
        # the fused GEMM called with them, then the ordering collective
        opened, closed, calls = [], [], []

        def export(t):
            return bytes([rank]) * 64, 16 * rank

        def open_peer(handle, offset):
            opened.append((handle[0], offset))
            return 1000 + 10 * handle[0] + offset

        blocks = sharding.PeerBlocks(torch.zeros(world, m, c1 - c0), export, open_peer,
                                     lambda p, o: closed.append((p, o)))

        def fused(aa, ww, ptrs, r, nw):
            calls.append((list(ptrs), r, nw))
            blocks.local[r] = aa @ ww.t()
        got = sharding.gemm_n_sharded_fused(a, w[c0:c1].contiguous(), blocks, fused)
        blocks.close()
        peer = 1 - rank
        assert opened == [(peer, 16 * peer)] and closed == [(1000 + 10 * peer + 16 * peer, 16 * peer)]
        want_ptrs = [blocks.local.data_ptr() if q_ == rank else 1000 + 10 * q_ + 16 * q_ for q_ in range(world)]
        assert calls == [(want_ptrs, rank, world)]
        assert got is blocks.local and torch.equal(got[rank], a @ w[c0:c1].t())

        # the multicast form's host logic: one call with this rank's buffer and its
        # multicast address, between the two ordering all-reduces (gloo here)
        import types
        mb = types.SimpleNamespace(local=torch.zeros(world, m, c1 - c0), local_ptr=11, multicast_ptr=22,
                                   rank=rank, world=world)
        mcalls = []

        def fused_mc(aa, ww, lp, mp, r, nw):
            mcalls.append((lp, mp, r, nw))
            mb.local[r] = aa @ ww.t()
        got = sharding.gemm_n_sharded_multicast(a, w[c0:c1].contiguous(), mb, fused_mc)
        assert mcalls == [(11, 22, rank, world)] and got is mb.local
        assert torch.equal(got[rank], a @ w[c0:c1].t())

        # a mapping failure on one rank is raised on every rank alike
        def export_fails_on_1(t):
            if rank == 1:
                raise OSError("no IPC here")
            return export(t)
        try:
            sharding.PeerBlocks(torch.zeros(world, 2, 2), export_fails_on_1, open_peer)
            raise AssertionError("expected a RuntimeError")
        except RuntimeError as exc:
            assert "rank 1" in str(exc)
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

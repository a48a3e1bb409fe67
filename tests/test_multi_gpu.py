"""Multi-GPU parity of the sharded families (one process per GPU, NCCL).

Runs at every world size in {2, 4, 8} that the box's GPUs allow; a 1-GPU box
skips it.  Each world checks, on every rank:

* the fused GEMM + all-gather (peer stores from the GEMM epilogue) against the
  local GEMM followed by an NCCL all-gather, bit for bit, on two calls in a
  row with different operands, each result read before the next call;
* row-sharded RMS norm and causal softmax (rank r owns ``row_range``; the
  softmax shard passes its global first row as ``row_offset``) against the
  same family run over all rows on one GPU, bit for bit;
* the rank-ordered sum (per-shard grid groupings, partials all-gathered over
  NCCL and folded strictly in rank order) against the oracle's evaluation of
  that declared grouping.
"""
import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _checks(rank, world):
    import numpy as np

    import oracle
    from tiler_b200 import families as fam, sharding
    results = {}
    gen = torch.Generator("cuda").manual_seed(4)  # the same operands on every rank

    # fused GEMM + all-gather, two calls in a row with different A
    m, n, k = 1024, 256 * world * 2, 512
    w = (torch.randn(n, k, device="cuda", generator=gen) * 0.1).to(torch.bfloat16)
    c0, c1 = sharding.row_range(n, rank, world)
    ws = w[c0:c1].contiguous()
    blocks = sharding.PeerBlocks(torch.full((world, m, c1 - c0), -1.0, device="cuda", dtype=torch.bfloat16),
                                 fam.ipc_export, fam.ipc_open, fam.ipc_close)
    ok = True
    for call in range(2):
        a = (torch.randn(m, k, device="cuda", generator=gen) * 0.1).to(torch.bfloat16)
        want = sharding.gemm_n_sharded(a, ws, lambda aa, ww: fam.gemm_bf16(aa, ww, "silu"), assemble=False)
        got = sharding.gemm_n_sharded_fused(
            a, ws, blocks, lambda aa, ww, p, r, nw: fam.gemm_bf16_allgather(aa, ww, p, r, nw, "silu"))
        ok = ok and torch.equal(got.view(torch.int16), want.view(torch.int16))  # read before the next call
    torch.distributed.barrier()
    blocks.close()
    results["gemm_fused_allgather"] = bool(ok)

    # the same exchange through an NVLink multicast mapping, where the box has one
    try:
        mblocks = sharding.MulticastBlocks((world, m, c1 - c0), torch.bfloat16, "cuda")
        multicast = mblocks.available
    except Exception:  # noqa: BLE001 - no symmetric memory on this box
        multicast = False
    results["multicast_available"] = multicast
    if multicast:
        ok = True
        for call in range(2):
            a = (torch.randn(m, k, device="cuda", generator=gen) * 0.1).to(torch.bfloat16)
            want = sharding.gemm_n_sharded(a, ws, lambda aa, ww: fam.gemm_bf16(aa, ww, "silu"), assemble=False)
            got = sharding.gemm_n_sharded_multicast(
                a, ws, mblocks,
                lambda aa, ww, lp, mp, r, nw: fam.gemm_bf16_allgather_multicast(aa, ww, lp, mp, r, nw, "silu"))
            ok = ok and torch.equal(got.view(torch.int16), want.view(torch.int16))
        torch.distributed.barrier()
        results["gemm_multicast_allgather"] = bool(ok)

    # row-sharded RMS norm [8192, 4096] f32
    x = torch.randn(8192, 4096, device="cuda", generator=gen)
    wr = torch.rand(4096, device="cuda", generator=gen) + 0.5
    full = fam.rms_norm(x, wr)
    r0, r1 = sharding.row_range(8192, rank, world)
    part = fam.rms_norm(x[r0:r1].contiguous(), wr)
    results["rms_row_shard"] = bool(torch.equal(part.view(torch.int32), full[r0:r1].view(torch.int32)))
    del x, full, part

    # row-sharded causal softmax [8192, 2048] (shards start inside mask blocks at W = 8)
    z = torch.randn(8192, 2048, device="cuda", generator=gen) * 3
    full = fam.softmax(z, causal_period=2048)
    part = fam.softmax(z[r0:r1].contiguous(), causal_period=2048,
                       row_offset=sharding.causal_row_offset(8192, rank, world))
    results["softmax_row_shard"] = bool(torch.equal(part.view(torch.int32), full[r0:r1].view(torch.int32)))
    del z, full, part

    # the rank-ordered sum of 2^24 contributors
    count = 1 << 24
    s = torch.rand(count, device="cuda", generator=gen) * 2 - 1
    s0, s1 = sharding.row_range(count, rank, world)
    shard = s[s0:s1].contiguous()
    got = sharding.sum_across_ranks(shard, lambda t: fam.sum_f32(t, fam.plan_grouping(1, t.numel())))
    host = s.cpu().numpy()
    partials = []
    for q in range(world):
        q0, q1 = sharding.row_range(count, q, world)
        _, v = oracle.grid_fold(host[q0:q1], fam.plan_grouping(1, q1 - q0))
        partials.append(np.float32(np.asarray(v).ravel()[0]))
    want = sharding._strict_fold(np.array(partials, np.float32))
    results["sum_rank_ordered"] = bool(np.float32(got).view(np.uint32) == np.float32(want).view(np.uint32))

    # the same sum with the exchange in one kernel over NVLink, on four calls in a row
    xch = sharding.SumExchange(1, "cuda", fam.ipc_export, fam.ipc_open, fam.ipc_close)
    ok = True
    for call in range(4):
        part = fam.sum_f32(shard, fam.plan_grouping(1, shard.numel())).reshape(1)
        res = xch(part, device_count=call >= 2).cpu().numpy()  # host seq 1, 2, then the buffer's count
        ok = ok and bool(res.view(np.uint32)[0] == np.float32(want).view(np.uint32))
    torch.distributed.barrier()
    xch.close()
    results["sum_exchange_kernel"] = ok
    return results


def _worker(rank, world, port, q):
    import sys
    sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    import torch.distributed as dist
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=torch.device("cuda", rank))
    try:
        q.put((rank, _checks(rank, world)))
    except Exception as exc:  # report instead of leaving the peers waiting
        q.put((rank, repr(exc)))
        raise
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 4, 8])
def test_sharded_families_match_one_gpu(world):
    if not torch.cuda.is_available() or torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    port = _free_port()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = sorted((q.get(timeout=600) for _ in range(world)), key=lambda t: t[0])
    for p in procs:
        p.join(timeout=120)
    want = {"gemm_fused_allgather": True, "rms_row_shard": True, "softmax_row_shard": True,
            "sum_rank_ordered": True, "sum_exchange_kernel": True}
    for r, res in results:
        assert isinstance(res, dict), (r, res)
        if res.pop("multicast_available"):
            want_r = dict(want, gemm_multicast_allgather=True)
        else:
            want_r = want
        assert res == want_r, (r, res)
    assert [r for r, _ in results] == list(range(world))

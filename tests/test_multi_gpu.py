"""Two-GPU parity of the fused GEMM + all-gather (one process per GPU, NCCL).

Runs only where two GPUs are visible; the single-GPU suite skips it.  The
fused form (the all-gather done by peer stores from the GEMM epilogue) must
give the same blocks, bit for bit, as the local GEMM followed by an NCCL
all-gather.
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


def _worker(rank, world, port, q):
    import sys
    sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    import torch.distributed as dist
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=torch.device("cuda", rank))
    from tiler_b200 import families as fam, sharding
    try:
        m, n, k = 1024, 2048, 512
        gen = torch.Generator("cuda").manual_seed(4)  # the same operands on every rank
        a = (torch.randn(m, k, device="cuda", generator=gen) * 0.1).to(torch.bfloat16)
        w = (torch.randn(n, k, device="cuda", generator=gen) * 0.1).to(torch.bfloat16)
        c0, c1 = sharding.row_range(n, rank, world)
        ws = w[c0:c1].contiguous()
        want = sharding.gemm_n_sharded(a, ws, lambda aa, ww: fam.gemm_bf16(aa, ww, "silu"), assemble=False)
        blocks = sharding.PeerBlocks(torch.full((world, m, c1 - c0), -1.0, device="cuda", dtype=torch.bfloat16),
                                     fam.ipc_export, fam.ipc_open, fam.ipc_close)
        ok = True
        for _ in range(3):  # repeated launches into the same buffers
            got = sharding.gemm_n_sharded_fused(
                a, ws, blocks, lambda aa, ww, p, r, nw: fam.gemm_bf16_allgather(aa, ww, p, r, nw, "silu"))
            torch.cuda.synchronize()
            ok = ok and torch.equal(got.view(torch.int16), want.view(torch.int16))
        dist.barrier()
        blocks.close()
        q.put((rank, bool(ok)))
    except Exception as exc:  # report instead of leaving the peer waiting
        q.put((rank, repr(exc)))
        raise
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_fused_gemm_allgather_equals_gemm_then_nccl_allgather():
    world, port = 2, _free_port()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = sorted(q.get(timeout=300) for _ in range(world))
    for p in procs:
        p.join(timeout=120)
    assert results == [(0, True), (1, True)], results

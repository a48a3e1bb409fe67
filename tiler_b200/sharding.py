"""One process per GPU: how the hot-path families spread over the GPUs of a node.

The reference is single-device; these are the backend's multi-GPU
realizations, each a declared, deterministic order (so results stay
bit-identical to a single-GPU run of the same declared grouping):

* row families (RMS norm, softmax, quantize/decode, gather, maps): rank r of
  W owns the contiguous row block ``row_range(rows, r, W)``; no collective;
* the sum: rank r folds its contiguous shard of the contributor sequence
  under the shard's grid grouping, the W partials are all-gathered and folded
  strictly in rank order (partition r = rank r: a strict_partitioned_sum over
  W partitions whose partition folds are the shard groupings);
* the contraction: W is split along N; rank r computes C[:, shard r] on its
  tensor cores and one all-gather assembles C (rank-major column blocks).

The collective is torch.distributed (NCCL on GPUs, gloo in the CPU tests).
The local compute is injected so the host logic is testable without a GPU.
"""
from __future__ import annotations

import numpy as np
import torch
import torch.distributed as dist


def row_range(rows: int, rank: int, world: int):
    """Contiguous row block of `rank`: [rows*rank//world, rows*(rank+1)//world)."""
    return rows * rank // world, rows * (rank + 1) // world


def causal_row_offset(rows: int, rank: int, world: int) -> int:
    """The global row index of the shard's first row: a softmax shard passes
    it as ``row_offset`` so the causal mask keeps ``global_row mod period``."""
    return row_range(rows, rank, world)[0]


def _strict_fold(values: np.ndarray) -> np.float32:
    """Strict left fold seeded at the first value (evaluate.rs:555-585), NaN
    canonicalized."""
    acc = np.float32(values[0])
    with np.errstate(invalid="ignore", over="ignore"):
        for v in values[1:]:
            acc = np.float32(acc + np.float32(v))
    if np.isnan(acc):
        return np.array([0x7FC00000], np.uint32).view(np.float32)[0]
    return acc


def sum_across_ranks(shard: torch.Tensor, local_sum, group=None) -> np.float32:
    """The multi-GPU sum: ``local_sum(shard)`` is this rank's partial (a
    0-d or 1-element tensor); the partials are all-gathered and folded in
    rank order.  Every rank returns the same bits."""
    world = dist.get_world_size(group)
    partial = local_sum(shard).reshape(1).to(torch.float32)
    gathered = torch.empty(world, dtype=torch.float32, device=partial.device)
    dist.all_gather_into_tensor(gathered, partial, group=group)
    return _strict_fold(gathered.cpu().numpy())


class PeerBlocks:
    """A [world, m, n] block buffer on every rank, each mapped into every
    rank's process (the target of the fused GEMM + all-gather).  ``export``
    and ``open_peer`` are the IPC calls (injected so the host logic runs
    without a GPU in tests); ``ptrs[q]`` is rank q's buffer in this process."""

    def __init__(self, local: torch.Tensor, export, open_peer, close_peer=None, group=None, blocks=True):
        self.world, self.rank = dist.get_world_size(group), dist.get_rank(group)
        assert not blocks or (local.dim() == 3 and local.shape[0] == self.world)
        self.local = local
        self._close = close_peer
        self._opened = []
        self.ptrs = []
        # every rank learns of a failure on any rank (no rank is left waiting
        # in a collective the others skipped)
        try:
            info = export(local)
        except Exception as exc:  # noqa: BLE001 - reported to every rank below
            info = ("error", repr(exc))
        infos = [None] * self.world
        dist.all_gather_object(infos, info, group=group)
        failed = [q for q, i in enumerate(infos) if i[0] == "error"]
        error = None if not failed else f"export failed on rank {failed[0]}: {infos[failed[0]][1]}"
        if error is None:
            try:
                for q, (handle, offset) in enumerate(infos):
                    if q == self.rank:
                        self.ptrs.append(local.data_ptr())
                    else:
                        p = open_peer(handle, offset)
                        self._opened.append((p, offset))
                        self.ptrs.append(p)
            except Exception as exc:  # noqa: BLE001
                error = f"open failed on rank {self.rank}: {exc!r}"
        errors = [None] * self.world
        dist.all_gather_object(errors, error, group=group)
        bad = [e for e in errors if e]
        if bad:
            self.close()
            raise RuntimeError(bad[0])

    def close(self):
        if self._close:
            for p, offset in self._opened:
                self._close(p, offset)
        self._opened = []


class SumExchange:
    """The multi-GPU sum's exchange without a library collective: each rank's
    partial sums go into every rank's exchange buffer over NVLink (peer
    stores) and every rank folds the W partials in rank order in one kernel
    (``tiler_cuda_sum_f32_exchange``).  The buffers are mapped into every rank
    once (``PeerBlocks`` over a byte buffer); ``__call__`` runs one exchange
    and returns the [rows] result on the device."""

    def __init__(self, rows: int, device, export, open_peer, close_peer=None, group=None):
        from . import _native as N
        self.rows = rows
        nbytes = int(N.lib().tiler_cuda_sum_exchange_buffer_bytes(rows))
        self.buffer = torch.zeros(nbytes, dtype=torch.uint8, device=device)
        self.peers = PeerBlocks(self.buffer, export, open_peer, close_peer, group=group, blocks=False)
        self.seq = 0

    def __call__(self, partial: torch.Tensor, out: torch.Tensor | None = None, check: bool = True,
                 device_count: bool = False):
        """One exchange; ``device_count`` takes the call number from the
        buffer's own counter (seq 0), so the launch can be graph-captured."""
        import ctypes as C

        from . import _native as N
        from . import families as F
        self.seq += 1
        seq = 0 if device_count else self.seq
        out = torch.empty(self.rows, dtype=torch.float32, device=partial.device) if out is None else out
        arr = (C.c_void_p * self.peers.world)(*self.peers.ptrs)
        st = F._status() if check else None
        F._check(N.lib().tiler_cuda_sum_f32_exchange(F.context(), F._stream(), st.ptr if st else 0,
                                                       partial.data_ptr(), self.rows, self.peers.rank,
                                                       self.peers.world, arr, seq, out.data_ptr()),
                 "sum_f32_exchange")
        if st:
            F._raise_from(st, "sum_f32_exchange")
        return out

    def close(self):
        self.peers.close()


class MulticastBlocks:
    """A [world, m, n] block buffer in torch symmetric memory on every rank,
    with its NVLink multicast address when the GPUs and driver offer one
    (``available``).  The fused GEMM's multicast stores into it reach every
    rank's copy at once."""

    def __init__(self, shape, dtype, device, group=None):
        import torch.distributed._symmetric_memory as symm_mem
        self.world, self.rank = dist.get_world_size(group), dist.get_rank(group)
        assert shape[0] == self.world
        group = group or dist.group.WORLD
        name = group.group_name
        if hasattr(symm_mem, "enable_symm_mem_for_group"):
            try:
                symm_mem.enable_symm_mem_for_group(name)
            except Exception:  # noqa: BLE001 - newer releases enable it themselves
                pass
        self.local = symm_mem.empty(shape, dtype=dtype, device=device)
        self.handle = symm_mem.rendezvous(self.local, name)
        base = int(self.handle.multicast_ptr or 0)
        self.available = base != 0
        self.local_ptr = self.local.data_ptr()
        offset = self.local_ptr - int(self.handle.buffer_ptrs[self.handle.rank])
        self.multicast_ptr = base + offset if self.available else 0


def gemm_n_sharded_multicast(a: torch.Tensor, w_shard: torch.Tensor, blocks: MulticastBlocks, fused_gemm, group=None):
    """``gemm_n_sharded_fused`` over multicast: ``fused_gemm(a, w_shard,
    local_ptr, multicast_ptr, rank, world)`` stores this rank's columns once,
    and the switch delivers them to every rank.  The same two one-element
    all-reduces order the call (before: every rank has finished reading the
    previous result; after: every rank's stores have landed)."""
    ready = torch.zeros(1, device=a.device)
    dist.all_reduce(ready, group=group)
    fused_gemm(a, w_shard, blocks.local_ptr, blocks.multicast_ptr, blocks.rank, blocks.world)
    done = torch.zeros(1, device=a.device)
    dist.all_reduce(done, group=group)
    return blocks.local


def gemm_n_sharded_fused(a: torch.Tensor, w_shard: torch.Tensor, blocks: PeerBlocks, fused_gemm, group=None):
    """The contraction's multi-GPU form with the exchange fused into the GEMM:
    ``fused_gemm(a, w_shard, ptrs, rank, world)`` writes this rank's columns
    into every rank's block buffer.  Two one-element all-reduces on the stream
    order the exchange: the one before the launch holds every rank's kernel
    until all ranks have reached this call, so no rank overwrites a peer's
    blocks while that peer still reads the previous call's result (reads the
    caller enqueued on this stream before the call); the one after orders every
    rank's kernel before anyone reads.  Returns the local [world, m, n/world]
    blocks (the layout ``gemm_n_sharded(assemble=False)`` returns); they stay
    valid until this rank's next call."""
    ready = torch.zeros(1, device=a.device)
    dist.all_reduce(ready, group=group)
    fused_gemm(a, w_shard, blocks.ptrs, blocks.rank, blocks.world)
    done = torch.zeros(1, device=a.device)
    dist.all_reduce(done, group=group)
    return blocks.local


def gemm_n_sharded(a: torch.Tensor, w_shard: torch.Tensor, local_gemm, group=None, assemble: bool = True):
    """C = local_gemm(a, w_shard) on every rank ([M, N/W] each), then one
    all-gather.  Returns [M, N] (assemble=True) or the rank-major blocks
    [W, M, N/W] as gathered."""
    world = dist.get_world_size(group)
    c_local = local_gemm(a, w_shard).contiguous()
    m, n_local = c_local.shape
    flat = torch.empty((world * m, n_local), dtype=c_local.dtype, device=c_local.device)
    dist.all_gather_into_tensor(flat, c_local, group=group)
    blocks = flat.view(world, m, n_local)
    if not assemble:
        return blocks
    return blocks.permute(1, 0, 2).reshape(m, world * n_local)

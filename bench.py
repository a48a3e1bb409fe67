"""Benchmark of the tiler-cuda hot path on B200 (the driver's contract).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl tiler|reference]

Headline workload (the metric's first config that
fits one GPU): RMS normalization, x f32 [8192, 4096] ~ N(0,1), w f32 [4096]
~ U[0.5, 1.5], eps = 1e-6 (bits 0x358637bd).  A step is one pass of the RMS
kernel over one [8192, 4096] batch; steps rotate over enough input/output
batches that the working set (>= 768 MB) is far larger than L2.

`value` is algorithmic HBM bytes (read x + w, write y) over device time, in
GB/s, summed over ranks (one process per GPU, each normalizing its own
batches: weak scaling, no collective on the data path).  `e2e` measures the
same metric through the public C-ABI entry point with the batch starting
and ending in pinned host memory.  `families` carries the other BASELINE
configs measured the same way (device time, CUDA events on the launching
stream).  With --impl reference the CPU restatement of tiler-reference
(oracle/, the only reference implementation runnable here) is timed on the
host cores for the same metric.
"""
from __future__ import annotations

import argparse
import json
import os
import re
import statistics
import subprocess
import sys
import tempfile
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

EPS_BITS = 0x358637BD
RMS_ROWS, RMS_EXTENT = 8192, 4096
RMS_BYTES = RMS_ROWS * RMS_EXTENT * 4 * 2 + RMS_EXTENT * 4  # read x, read w, write y
METRIC = "rms_norm_f32 HBM GB/s (per-family HBM GB/s; bf16 contraction TFLOP/s)"


def sustained_tflops():
    """The bf16 GEMM figure measured back to back for seconds under the power
    cap (MEASURED_PEAKS.json bf16_tflops_sustained), else the fallback 1400."""
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            v = json.load(f).get("bf16_tflops_sustained")
        if v:
            return float(v)
    return 1400.0


def measured_peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            d = json.load(f)
        return float(d["hbm_gbs"]), float(d["bf16_tflops"]), "measured"
    return 6650.0, 1590.0, "fallback"


def committed_traffic(name):
    """DRAM bytes per launch from the committed ncu summary profiles/<name>.txt
    (line `traffic_bytes_per_launch: N`), else None."""
    p = os.path.join(ROOT, "profiles", name + ".txt")
    if not os.path.exists(p):
        return None
    m = re.search(r"traffic_bytes_per_launch:\s*([0-9.eE+]+)", open(p).read())
    return float(m.group(1)) if m else None


class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled during the timed region."""

    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device_index):
        self.dev = device_index
        self.proc = None
        self.path = None

    def __enter__(self):
        fd, self.path = tempfile.mkstemp(suffix=".csv")
        os.close(fd)
        try:
            self.proc = subprocess.Popen(["nvidia-smi", "-i", str(self.dev), f"--query-gpu={self.Q}",
                                          "--format=csv,noheader,nounits", "-lms", "100"],
                                         stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
        except OSError:
            self.proc = None
        time.sleep(0.3)
        return self

    def __exit__(self, *a):
        if self.proc:
            self.proc.terminate()
            self.proc.wait()

    def summary(self):
        rows = []
        if self.path and os.path.exists(self.path):
            for line in open(self.path):
                parts = [p.strip() for p in line.split(",")]
                if len(parts) >= 9:
                    rows.append(parts)
            os.unlink(self.path)
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        sm = [float(r[1]) for r in rows if r[1].replace(".", "").isdigit()]
        mx = [float(r[2]) for r in rows if r[2].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({n for r in rows for n, v in zip(names, r[5:9]) if v.lower() == "active"})
        loaded = [s for s in sm if mx and s > 0.5 * max(mx)] or sm
        return {"sm_mhz": statistics.median(loaded) if loaded else None,
                "sm_max_mhz": max(mx) if mx else None, "reasons": reasons, "samples": len(rows)}


def dist_setup(n_gpus):
    import torch
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import torch.distributed as dist
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", device_id=torch.device("cuda", local))
    else:
        torch.cuda.set_device(0)
    return rank, world, local


def barrier(world):
    if world > 1:
        import torch.distributed as dist
        dist.barrier()


def max_over_ranks(v, world):
    if world == 1:
        return v
    import torch
    import torch.distributed as dist
    t = torch.tensor([v], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def cur_stream():
    import torch
    return torch.cuda.current_stream().cuda_stream


GRAPH_CHUNK = 192  # launches per captured graph (a multiple of the rotating-buffer counts 2, 3, 4, 6, 8)


def time_device(fn, steps, warmup, world, clocks=None, graph=False):
    """Runs warmup untimed steps, then times exactly `steps` calls of fn(i)
    with CUDA events on the current stream, barrier + synchronize on both
    sides; returns (ms total, max over ranks).  graph=True issues the timed
    steps from CUDA graphs of GRAPH_CHUNK captured launches (and one graph for
    the remainder), replayed back to back: the same kernels on the same
    buffers, without the per-launch host overhead.  fn must launch on the
    current stream only and must not synchronize."""
    import torch
    for i in range(warmup):
        fn(i)
    torch.cuda.synchronize()
    replays = []
    if graph:
        try:
            chunk = min(steps, GRAPH_CHUNK)
            full, rest = divmod(steps, chunk)
            cap = torch.cuda.Stream()
            g_full = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g_full, stream=cap, capture_error_mode="thread_local"):
                for i in range(chunk):
                    fn(i)
            replays = [g_full] * full
            if rest:
                g_rest = torch.cuda.CUDAGraph()
                with torch.cuda.graph(g_rest, stream=cap, capture_error_mode="thread_local"):
                    for i in range(rest):
                        fn(full * chunk + i)
                replays.append(g_rest)
            for g in set(replays):  # one untimed replay of each (uploads the graphs)
                g.replay()
        except Exception:  # noqa: BLE001 - capture refused: time plain launches
            replays = []
        torch.cuda.synchronize()
    barrier(world)
    torch.cuda.synchronize()
    s = torch.cuda.current_stream()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ctx = clocks if clocks is not None else _Null()
    with ctx:
        e0.record(s)
        if replays:
            for g in replays:
                g.replay()
        else:
            for i in range(steps):
                fn(i)
        e1.record(s)
        torch.cuda.synchronize()
    barrier(world)
    torch.cuda.synchronize()
    return max_over_ranks(e0.elapsed_time(e1), world)


class _Null:
    def __enter__(self):
        return self

    def __exit__(self, *a):
        pass


def cpu_baseline_rms(nthreads, min_seconds=3.0):
    """The oracle's RMS (tiler-reference semantics) on the host cores over a
    bounded sample: the full [8192, 4096] batch, repeated until min_seconds."""
    import numpy as np

    import oracle
    oracle.build()
    rng = np.random.default_rng(0)
    x = rng.standard_normal((RMS_ROWS, RMS_EXTENT), dtype=np.float32)
    w = rng.uniform(0.5, 1.5, RMS_EXTENT).astype(np.float32)
    reps, t0 = 0, time.perf_counter()
    while True:
        oracle.rms_norm_f32(x, w, EPS_BITS, nthreads=nthreads)
        reps += 1
        el = time.perf_counter() - t0
        if el >= min_seconds:
            break
    return RMS_BYTES * reps / el / 1e9, f"{reps} x full [8192,4096] batch, {el:.1f} s"


def run_reference(args):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return 0
    import numpy as np

    import oracle
    oracle.build()
    cores = os.cpu_count() or 1
    rng = np.random.default_rng(0)
    sample_rows = 1024  # bounded sample: 1/8 of the batch per step
    x = rng.standard_normal((sample_rows, RMS_EXTENT), dtype=np.float32)
    w = rng.uniform(0.5, 1.5, RMS_EXTENT).astype(np.float32)
    for _ in range(args.warmup):
        oracle.rms_norm_f32(x, w, EPS_BITS, nthreads=cores)
    t0 = time.perf_counter()
    for _ in range(args.steps):
        oracle.rms_norm_f32(x, w, EPS_BITS, nthreads=cores)
    el = time.perf_counter() - t0
    bytes_per_step = sample_rows * RMS_EXTENT * 8 + RMS_EXTENT * 4
    v = bytes_per_step * args.steps / el / 1e9
    line = {"impl": "reference", "metric": METRIC, "value": round(v, 3), "unit": "GB/s", "n_gpus": args.gpus,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": el * 1e3 / args.steps,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic (seeded N(0,1) x, U[0.5,1.5] w)",
            "config": {"workload": "rms_norm_f32 [8192,4096] eps=1e-6", "sample": f"{sample_rows} rows per step",
                       "parallelism": f"{cores} host threads"},
            "cpu_baseline": {"value": round(v, 3), "unit": "GB/s", "cores": cores, "kind": "port",
                             "sample": f"{sample_rows} of 8192 rows per step, {args.steps} steps"},
            "e2e": {"value": round(v, 3), "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
            "note": "tiler-reference is Rust (nightly) and cannot be built here; its C++ restatement "
                    "(oracle/, bit-identical results) is the reference arm"}
    print(json.dumps(line), flush=True)
    return 0


def family_suite(fam, torch, world, steps_small, warmup):
    """Per-family device throughput at the BASELINE configs (each config's own
    algorithmic bytes / FLOPs; rotating buffers so inputs exceed L2)."""
    hbm, tflops, _ = measured_peaks()
    # the strong-scaled lines first, at the clocks the headline ran at (after
    # the power-heavy contraction they measured up to 30 % slower)
    strong = strong_scaled_suite(fam, torch, world, steps_small, warmup)
    out = {}
    gen = torch.Generator("cuda").manual_seed(7)
    dev = "cuda"

    def rec(name, unit, per_step, ms, steps, peak, launches=1):
        v = per_step * steps / (ms / 1e3) / (1e9 if unit == "GB/s" else 1e12)
        out[name] = {"value": round(v, 2), "unit": unit, "frac": round(v / peak, 4),
                     "us_per_launch": round(ms * 1e3 / steps / launches, 2)}

    # two-level grouped sum, x f32 [2^24]
    n = 1 << 24
    xs = [torch.rand(n, device=dev, generator=gen) * 2 - 1 for _ in range(4)]
    g = fam.plan_grouping(1, n)
    ws = fam.grouped_workspace(1, g)
    o = torch.empty(1, device=dev)
    from tiler_b200 import _native as N
    import ctypes as C
    gs = N.Grouping.from_dict(g)
    ctx, L = fam.context(), N.lib()
    stream = torch.cuda.current_stream().cuda_stream

    def run_sum(i):
        L.tiler_cuda_sum_f32(ctx, cur_stream(), xs[i % 4].data_ptr(), 1, n, C.byref(gs), ws.data_ptr(), ws.numel(),
                             o.data_ptr())
    ms = time_device(run_sum, steps_small * 4, warmup, world, graph=True)
    rec("sum_f32_2^24", "GB/s", n * 4, ms, steps_small * 4, hbm)
    out["sum_f32_2^24"]["grouping"] = g
    del xs

    # RMS bf16 [8192, 4096]
    xb = [torch.randn(RMS_ROWS, RMS_EXTENT, device=dev, generator=gen).to(torch.bfloat16) for _ in range(6)]
    wb = (torch.rand(RMS_EXTENT, device=dev, generator=gen) + 0.5).to(torch.bfloat16)
    yb = [torch.empty_like(xb[0]) for _ in range(2)]
    ms = time_device(lambda i: fam.rms_norm(xb[i % 6], wb, out=yb[i % 2], check=False), steps_small * 4, warmup, world,
                     graph=True)
    rec("rms_norm_bf16_8192x4096", "GB/s", RMS_ROWS * RMS_EXTENT * 4 + RMS_EXTENT * 2, ms, steps_small * 4, hbm)
    del xb, yb

    # elementwise maps f32 [8192, 4096]: certified SiLU, and (x*a)+b with rank-0 a, b
    xm = [torch.randn(RMS_ROWS, RMS_EXTENT, device=dev, generator=gen) * 4 for _ in range(3)]
    ym = [torch.empty_like(xm[0]) for _ in range(2)]
    ms = time_device(lambda i: fam.silu(xm[i % 3], out=ym[i % 2], check=False), steps_small * 2, warmup, world, graph=True)
    rec("silu_f32_8192x4096", "GB/s", RMS_ROWS * RMS_EXTENT * 8, ms, steps_small * 2, hbm)
    sa, sb = torch.tensor(1.5, device=dev), torch.tensor(-0.25, device=dev)
    ms = time_device(lambda i: fam.scale_bias(xm[i % 3], sa, sb, out=ym[i % 2]), steps_small * 2, warmup, world, graph=True)
    rec("scale_bias_f32_8192x4096", "GB/s", RMS_ROWS * RMS_EXTENT * 8, ms, steps_small * 2, hbm)
    del xm, ym

    # softmax f32 [65536, 2048] with the causal block mask
    xsm = torch.randn(65536, 2048, device=dev, generator=gen) * 3
    ysm = torch.empty_like(xsm)
    ms = time_device(lambda i: fam.softmax(xsm, causal_period=2048, out=ysm, check=False), steps_small, warmup, world,
                     graph=True)
    rec("softmax_f32_65536x2048_causal", "GB/s", 65536 * 2048 * 8, ms, steps_small, hbm)
    # the same causal mask as a program tensor [2048, 2048] (0 / -inf), added in the kernel
    col = torch.arange(2048, device=dev)
    mask = torch.where(col[None, :] > col[:, None], float("-inf"), 0.0).contiguous()
    ms = time_device(lambda i: fam.softmax_masked(xsm, mask, out=ysm, check=False), steps_small, warmup, world,
                     graph=True)
    rec("softmax_masked_f32_65536x2048_mask_tensor", "GB/s", 65536 * 2048 * 8 + 2048 * 2048 * 4, ms, steps_small, hbm)
    del mask
    del xsm, ysm

    # quantize / decode f32 [16384, 4096]
    xq = [torch.randn(16384, 4096, device=dev, generator=gen) for _ in range(2)]
    codes, scales = fam.quantize_i8_rows(xq[0])
    # outputs rotate over 3 x 64 MB so the codes do not stay in L2 between steps
    qout = [(torch.empty_like(codes), torch.empty_like(scales)) for _ in range(3)]
    ms = time_device(lambda i: fam.quantize_i8_rows(xq[i % 2], check=False, out=qout[i % 3]), steps_small * 3,
                     warmup, world, graph=True)
    qbytes = 16384 * 4096 * 5 + 16384 * 4
    rec("quantize_i8_16384x4096", "GB/s", qbytes, ms, steps_small * 3, hbm)
    del qout
    yq = torch.empty(16384, 4096, device=dev)
    cd = torch.empty_like(codes)

    # fused RMS norm -> int8 quantize over the RMS config (x read once, y never written)
    xr = [torch.randn(RMS_ROWS, RMS_EXTENT, device=dev, generator=gen) for _ in range(2)]
    wr_ = torch.rand(RMS_EXTENT, device=dev, generator=gen) + 0.5
    fout = [(torch.empty(RMS_ROWS, RMS_EXTENT, device=dev, dtype=torch.int8), torch.empty(RMS_ROWS, device=dev))
            for _ in range(4)]
    ms = time_device(lambda i: fam.rms_norm_quantize_i8(xr[i % 2], wr_, check=False, out=fout[i % 4]),
                     steps_small * 4, warmup, world, graph=True)
    rec("rms_norm_quantize_i8_8192x4096", "GB/s", RMS_ROWS * RMS_EXTENT * 5 + RMS_EXTENT * 4 + RMS_ROWS * 4, ms,
        steps_small * 4, hbm)
    del xr, fout

    def run_dec(i):
        L.tiler_cuda_dequantize_i8_rows(ctx, cur_stream(), None, codes.data_ptr(), scales.data_ptr(), 16384, 4096,
                                        yq.data_ptr())
    ms = time_device(run_dec, steps_small, warmup, world, graph=True)
    rec("dequantize_i8_16384x4096", "GB/s", qbytes, ms, steps_small, hbm)
    del xq, yq, codes, cd

    # gather: ids i32 [8192] from bf16 table [128256, 4096]
    table = (torch.randn(128256, 4096, device=dev, generator=gen) * 0.02).to(torch.bfloat16)
    idss = [torch.randint(0, 128256, (8192,), device=dev, dtype=torch.int32, generator=gen) for _ in range(8)]
    # outputs rotate over 4 x 64 MB so the rows written do not stay in L2 between steps
    gas = [torch.empty(8192, 4096, device=dev, dtype=torch.bfloat16) for _ in range(4)]
    ga = gas[0]
    ms = time_device(lambda i: fam.gather_rows(table, idss[i % 8], out=gas[i % 4], check=False), steps_small * 4,
                     warmup, world, graph=True)
    rec("gather_bf16_8192_of_128256x4096", "GB/s", 8192 * 4 + 8192 * 4096 * 4, ms, steps_small * 4, hbm)

    # bf16 contraction [8192,4096] x [4096,14336] + SiLU (W stored [N,K])
    wt = (torch.randn(14336, 4096, device=dev, generator=gen) * 0.02).to(torch.bfloat16)
    cc = torch.empty(8192, 14336, device=dev, dtype=torch.bfloat16)
    gsteps = max(2, steps_small // 2)
    ms = time_device(lambda i: fam.gemm_bf16(ga, wt, "silu", out=cc, check=False), gsteps, warmup, world, graph=True)
    rec("gemm_bf16_silu_8192x4096x14336", "TFLOP/s", 2.0 * 8192 * 4096 * 14336, ms, gsteps, tflops)
    # the same against the sustained (power-capped) GEMM figure: the launches
    # run back to back, so the power cap governs their clocks as it does there
    g_ = out["gemm_bf16_silu_8192x4096x14336"]
    g_["frac_of_sustained"] = round(g_["value"] / sustained_tflops(), 4)
    if world > 1:
        # N-sharded contraction: each rank computes [8192, 14336/W] on its
        # tensor cores, one NCCL all-gather assembles C (strong scaling; the
        # whole-job FLOPs are the single contraction's)
        from tiler_b200 import sharding
        rank = torch.distributed.get_rank()
        c0, c1 = sharding.row_range(14336, rank, world)
        if (c1 - c0) % 256 == 0:
            ws_ = wt[c0:c1].contiguous()
            cl = torch.empty(8192, c1 - c0, device=dev, dtype=torch.bfloat16)
            ms = time_device(lambda i: fam.gemm_bf16(ga, ws_, "silu", out=cl, check=False), gsteps, warmup, world,
                             graph=True)
            rec("gemm_bf16_silu_nsharded_local", "TFLOP/s", 2.0 * 8192 * 4096 * 14336, ms, gsteps, tflops * world)
            ms = time_device(lambda i: sharding.gemm_n_sharded(
                ga, ws_, lambda a_, w_: fam.gemm_bf16(a_, w_, "silu", out=cl, check=False), assemble=False),
                gsteps, warmup, world)
            rec("gemm_bf16_silu_nsharded_allgather", "TFLOP/s", 2.0 * 8192 * 4096 * 14336, ms, gsteps,
                tflops * world)
            # the all-gather fused into the epilogue (peer stores over NVLink);
            # PeerBlocks raises on every rank alike if any rank cannot map the buffers
            try:
                blocks = sharding.PeerBlocks(torch.empty(world, 8192, c1 - c0, device=dev, dtype=torch.bfloat16),
                                             fam.ipc_export, fam.ipc_open, fam.ipc_close)
            except RuntimeError as exc:
                blocks = None
                out["gemm_bf16_silu_nsharded_fused_allgather"] = {"unavailable": str(exc)[:200]}
            if blocks is not None:
                ms = time_device(lambda i: sharding.gemm_n_sharded_fused(
                    ga, ws_, blocks, lambda a_, w_, p_, r_, n_: fam.gemm_bf16_allgather(a_, w_, p_, r_, n_, "silu",
                                                                                       check=False)),
                    gsteps, warmup, world)
                rec("gemm_bf16_silu_nsharded_fused_allgather", "TFLOP/s", 2.0 * 8192 * 4096 * 14336, ms, gsteps,
                    tflops * world)
                blocks.close()
            # the all-gather as multicast stores into an NVLink multicast mapping (each box
            # crosses NVLink once); available where torch symmetric memory offers one
            try:
                mblocks = sharding.MulticastBlocks((world, 8192, c1 - c0), torch.bfloat16, dev)
            except Exception as exc:  # noqa: BLE001
                mblocks = None
                out["gemm_bf16_silu_nsharded_multicast_allgather"] = {"unavailable": str(exc)[:200]}
            if mblocks is not None and not mblocks.available:
                out["gemm_bf16_silu_nsharded_multicast_allgather"] = {"unavailable": "no multicast mapping"}
            elif mblocks is not None:
                ms = time_device(lambda i: sharding.gemm_n_sharded_multicast(
                    ga, ws_, mblocks, lambda a_, w_, lp, mp, r_, n_: fam.gemm_bf16_allgather_multicast(
                        a_, w_, lp, mp, r_, n_, "silu", check=False)), gsteps, warmup, world)
                rec("gemm_bf16_silu_nsharded_multicast_allgather", "TFLOP/s", 2.0 * 8192 * 4096 * 14336, ms, gsteps,
                    tflops * world)
    del table, ga, gas, wt, cc
    torch.cuda.empty_cache()
    # the committed ncu summary each family's counters reproduce from
    for name, prof in (("sum_f32_2^24", "dequantize_sum_gather_launch_metrics.txt"),
                       ("dequantize_i8_16384x4096", "dequantize_sum_gather_launch_metrics.txt"),
                       ("gather_bf16_8192_of_128256x4096", "dequantize_sum_gather_launch_metrics.txt"),
                       ("silu_f32_8192x4096", "silu_f32_8192x4096.txt"),
                       ("rms_norm_bf16_8192x4096", "rms_norm_bf16_8192x4096.txt"),
                       ("softmax_f32_65536x2048_causal", "softmax_f32_65536x2048_causal.txt"),
                       ("quantize_i8_16384x4096", "quantize_i8_16384x4096.txt"),
                       ("gemm_bf16_silu_8192x4096x14336", "gemm_bf16_silu_pair_2048x14336x4096.txt")):
        if name in out and os.path.exists(os.path.join(ROOT, "profiles", prof)):
            out[name]["profile"] = "profiles/" + prof
    out.update(strong)
    return out


def strong_scaled_suite(fam, torch, world, steps_small, warmup):
    """The row families and the sum split over the ranks (strong scaling: the
    whole job is the one BASELINE config; rank r takes sharding.row_range of
    its rows).  `value` is the whole job's algorithmic bytes over the max over
    ranks of the device time, so the driver's per-N values give the
    strong-scaling efficiency directly; `us_per_launch` shows the floor that
    launch latency sets once a shard is small."""
    import ctypes as C

    from tiler_b200 import _native as N
    from tiler_b200 import sharding
    hbm, _, _ = measured_peaks()
    rank = torch.distributed.get_rank() if world > 1 else 0
    gen = torch.Generator("cuda").manual_seed(11)
    dev = "cuda"
    out = {}

    def rec(name, total_bytes, ms, steps, shard):
        v = total_bytes * steps / (ms / 1e3) / 1e9
        out[name] = {"value": round(v, 2), "unit": "GB/s", "frac_per_gpu": round(v / world / hbm, 4),
                     "us_per_launch": round(ms * 1e3 / steps, 2), "scaling": "strong", "shard": shard}

    # RMS f32: rows [r0, r1) of the [8192, 4096] batch
    r0, r1 = sharding.row_range(RMS_ROWS, rank, world)
    shard_bytes = (r1 - r0) * RMS_EXTENT * 4
    nb = max(3, -(-3 * 126 * 2 ** 20 // (2 * shard_bytes)))  # rotation well past L2
    xs = [torch.randn(r1 - r0, RMS_EXTENT, device=dev, generator=gen) for _ in range(nb)]
    ys = [torch.empty_like(xs[0]) for _ in range(nb)]
    w = torch.rand(RMS_EXTENT, device=dev, generator=gen) + 0.5
    steps = steps_small * 8
    ms = time_device(lambda i: fam.rms_norm(xs[i % nb], w, out=ys[i % nb], check=False), steps, warmup, world,
                     graph=True)
    rec("strong_rms_norm_f32_8192x4096", RMS_BYTES, ms, steps, f"{r1 - r0} rows per rank")
    del xs, ys

    # causal softmax: rows [r0, r1) of [65536, 2048]; the shard keeps its global row offset
    r0, r1 = sharding.row_range(65536, rank, world)
    nb = 2 if world > 1 else 1
    zs = [torch.randn(r1 - r0, 2048, device=dev, generator=gen) * 3 for _ in range(nb)]
    zo = [torch.empty_like(zs[0]) for _ in range(nb)]
    ms = time_device(lambda i: fam.softmax(zs[i % nb], causal_period=2048, row_offset=r0, out=zo[i % nb],
                                           check=False), steps_small * 2, warmup, world, graph=True)
    rec("strong_softmax_f32_65536x2048_causal", 65536 * 2048 * 8, ms, steps_small * 2, f"{r1 - r0} rows per rank")
    del zs, zo

    # the sum of 2^24: each rank's shard under its grid grouping, the W partials
    # all-gathered over NCCL and folded strictly in rank order on the device
    n = 1 << 24
    s0, s1 = sharding.row_range(n, rank, world)
    shards = [torch.rand(s1 - s0, device=dev, generator=gen) * 2 - 1 for _ in range(4)]
    g = fam.plan_grouping(1, s1 - s0)
    gs = N.Grouping.from_dict(g)
    ws = fam.grouped_workspace(1, g)
    part = torch.empty(1, device=dev)
    gathered = torch.empty(world, device=dev)
    total = torch.empty(1, device=dev)
    ctx, L = fam.context(), N.lib()

    def run_sum(i):
        L.tiler_cuda_sum_f32(ctx, cur_stream(), shards[i % 4].data_ptr(), 1, s1 - s0, C.byref(gs), ws.data_ptr(),
                             ws.numel(), part.data_ptr())
        if world > 1:
            torch.distributed.all_gather_into_tensor(gathered, part)
            L.tiler_cuda_strict_sum_f32(ctx, cur_stream(), gathered.data_ptr(), 1, world, total.data_ptr())
    steps = steps_small * 8
    ms = time_device(run_sum, steps, warmup, world)
    rec("strong_sum_f32_2^24_rank_ordered_nccl", n * 4, ms, steps, f"{s1 - s0} contributors per rank")
    # the exchange as one kernel: partials stored over NVLink into every rank's
    # buffer, each rank folding the W partials in rank order
    xch = None
    if world > 1:
        try:
            xch = sharding.SumExchange(1, dev, fam.ipc_export, fam.ipc_open, fam.ipc_close)
        except RuntimeError as exc:
            out["strong_sum_f32_2^24_rank_ordered"] = {"unavailable": str(exc)[:200]}

    def run_sum_xch(i):
        L.tiler_cuda_sum_f32(ctx, cur_stream(), shards[i % 4].data_ptr(), 1, s1 - s0, C.byref(gs), ws.data_ptr(),
                             ws.numel(), part.data_ptr())
        if xch is not None:
            xch(part, out=total, check=False, device_count=True)
    if world == 1 or xch is not None:
        ms = time_device(run_sum_xch, steps, warmup, world, graph=True)
        rec("strong_sum_f32_2^24_rank_ordered", n * 4, ms, steps, f"{s1 - s0} contributors per rank")
    if xch is not None:
        torch.distributed.barrier()
        xch.close()
    del shards
    return out


def run_tiler(args):
    import torch

    from tiler_b200 import families as fam
    from tiler_b200 import _native as N
    import ctypes as C

    rank, world, local = dist_setup(args.gpus)
    hbm, tflops, peak_kind = measured_peaks()
    ctx, L = fam.context(), N.lib()
    gen = torch.Generator("cuda").manual_seed(1234 + rank)
    nbuf = 3
    xs = [torch.randn(RMS_ROWS, RMS_EXTENT, device="cuda", generator=gen) for _ in range(nbuf)]
    w = torch.rand(RMS_EXTENT, device="cuda", generator=gen) + 0.5
    ys = [torch.empty_like(xs[0]) for _ in range(nbuf)]
    stream = torch.cuda.current_stream().cuda_stream

    def step(i):
        L.tiler_cuda_rms_norm_f32(ctx, cur_stream(), None, xs[i % nbuf].data_ptr(), w.data_ptr(), 0, RMS_ROWS,
                                  RMS_EXTENT, EPS_BITS, ys[i % nbuf].data_ptr())

    clocks = ClockSampler(local) if rank == 0 else None
    ms = time_device(step, args.steps, args.warmup, world, clocks=clocks, graph=True)
    ms_step = ms / args.steps
    value = RMS_BYTES * world * args.steps / (ms / 1e3) / 1e9
    per_gpu = RMS_BYTES / (ms_step / 1e3) / 1e9
    clk = clocks.summary() if clocks else None

    # end to end through the public entry point: pinned host x -> device ->
    # RMS -> pinned host y, every step
    hx = torch.empty(RMS_ROWS, RMS_EXTENT, dtype=torch.float32, pin_memory=True)
    hx.copy_(xs[0])
    hy = torch.empty_like(hx, pin_memory=True)
    dx, dy = xs[0], ys[0]

    def e2e_step(i):
        # upload, kernel and download chunked and overlapped inside the entry point
        L.tiler_cuda_rms_norm_host(ctx, stream, None, 0, hx.data_ptr(), dx.data_ptr(), w.data_ptr(), 0, RMS_ROWS,
                                   RMS_EXTENT, EPS_BITS, dy.data_ptr(), hy.data_ptr(), 0)
    e2e_steps = max(3, min(args.steps, 20))
    ms_e2e = time_device(e2e_step, e2e_steps, 2, world)
    e2e_value = RMS_BYTES * world * e2e_steps / (ms_e2e / 1e3) / 1e9
    del hx, hy

    families = None
    if not args.no_families:
        del xs, ys
        torch.cuda.empty_cache()
        families = family_suite(fam, torch, world, args.family_steps, max(3, args.warmup))

    if rank == 0:
        cpu_v, cpu_sample = (None, None)
        if world == 1 and not args.no_cpu_baseline:
            cpu_v, cpu_sample = cpu_baseline_rms(os.cpu_count() or 1)
        line = {
            "metric": METRIC, "value": round(value, 2), "unit": "GB/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(ms_step, 5), "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "f32", "data": "synthetic (seeded N(0,1) x, U[0.5,1.5] w)",
            "config": {"workload": "rms_norm_f32 [8192,4096] eps=1e-6 (BASELINE configs[1])",
                       "l2": f"{nbuf} rotating input/output batches ({nbuf * 256} MB) > 126 MB L2",
                       "parallelism": f"dp{world} (one [8192,4096] batch per GPU per step)",
                       "timing": f"CUDA events around CUDA graphs of {GRAPH_CHUNK} captured launches replayed back to "
                                 "back (one launch per step); e2e from plain launches"},
            "gpu_launches": args.steps,
            "e2e": {"value": round(e2e_value, 2), "unit": "GB/s",
                    "h2d_bytes_per_step": RMS_ROWS * RMS_EXTENT * 4, "d2h_bytes_per_step": RMS_ROWS * RMS_EXTENT * 4,
                    "steps": e2e_steps,
                    "path": "tiler_cuda_rms_norm_host (pinned host x -> device -> RMS -> pinned host y, 8 chunks, "
                            "upload / kernel / download overlapped)"},
            "roofline": {"bound": "hbm", "achieved": round(per_gpu, 2), "peak": hbm, "unit": "GB/s",
                         "frac": round(per_gpu / hbm, 4), "traffic": committed_traffic("rms_norm_f32_8192x4096"),
                         "peak_source": f"{peak_kind} (MEASURED_PEAKS.json hbm_gbs)" if peak_kind == "measured"
                         else "fallback 6.65 TB/s",
                         "algorithmic_bytes_per_launch": RMS_BYTES},
            "clocks": clk,
        }
        if cpu_v is not None:
            line["cpu_baseline"] = {"value": round(cpu_v, 3), "unit": "GB/s", "cores": os.cpu_count() or 1,
                                    "kind": "port", "sample": cpu_sample}
        if families is not None:
            line["families"] = families
        print(json.dumps(line), flush=True)
    if world > 1:
        import torch.distributed as dist
        dist.destroy_process_group()
    return 0


def run_profile_case(family: str, launches: int):
    """A few launches of one family at its BASELINE config, for ncu captures
    (profiles/*.txt name this command)."""
    import torch

    from tiler_b200 import families as fam
    torch.cuda.set_device(0)
    g = torch.Generator("cuda").manual_seed(3)
    dev = "cuda"
    if family in ("rms_f32", "rms_bf16"):
        dt = torch.float32 if family == "rms_f32" else torch.bfloat16
        x = torch.randn(RMS_ROWS, RMS_EXTENT, device=dev, generator=g).to(dt)
        w = (torch.rand(RMS_EXTENT, device=dev, generator=g) + 0.5).to(dt)
        y = torch.empty_like(x)
        run = lambda: fam.rms_norm(x, w, out=y, check=False)
    elif family == "softmax":
        x = torch.randn(65536, 2048, device=dev, generator=g) * 3
        y = torch.empty_like(x)
        run = lambda: fam.softmax(x, causal_period=2048, out=y, check=False)
    elif family in ("silu", "scale_bias"):
        x = torch.randn(RMS_ROWS, RMS_EXTENT, device=dev, generator=g) * 4
        y = torch.empty_like(x)
        sa, sb = torch.tensor(1.5, device=dev), torch.tensor(-0.25, device=dev)
        run = (lambda: fam.silu(x, out=y, check=False)) if family == "silu" else \
            (lambda: fam.scale_bias(x, sa, sb, out=y))
    elif family == "sum":
        x = torch.rand(1 << 24, device=dev, generator=g) * 2 - 1
        gr = fam.plan_grouping(1, 1 << 24)
        ws = fam.grouped_workspace(1, gr)
        run = lambda: fam.sum_f32(x, gr, ws)
    elif family in ("quantize", "dequantize"):
        x = torch.randn(16384, 4096, device=dev, generator=g)
        codes, scales = fam.quantize_i8_rows(x)
        run = (lambda: fam.quantize_i8_rows(x, check=False)) if family == "quantize" else \
            (lambda: fam.dequantize_i8_rows(codes, scales, check=False))
    elif family == "gather":
        table = (torch.randn(128256, 4096, device=dev, generator=g) * 0.02).to(torch.bfloat16)
        ids = torch.randint(0, 128256, (8192,), device=dev, dtype=torch.int32, generator=g)
        out = torch.empty(8192, 4096, device=dev, dtype=torch.bfloat16)
        run = lambda: fam.gather_rows(table, ids, out=out, check=False)
    elif family in ("gemm", "gemm_small"):
        m = 8192 if family == "gemm" else 2048
        a = (torch.randn(m, 4096, device=dev, generator=g) * 0.02).to(torch.bfloat16)
        w = (torch.randn(14336, 4096, device=dev, generator=g) * 0.02).to(torch.bfloat16)
        c = torch.empty(m, 14336, device=dev, dtype=torch.bfloat16)
        run = lambda: fam.gemm_bf16(a, w, "silu", out=c, check=False)
    else:
        raise SystemExit(f"unknown family {family}")
    for _ in range(launches):
        run()
    torch.cuda.synchronize()
    print(json.dumps({"profile_case": family, "launches": launches}))
    return 0


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20000)
    ap.add_argument("--warmup", type=int, default=50)
    ap.add_argument("--impl", default="tiler", choices=["tiler", "reference"])
    ap.add_argument("--family-steps", type=int, default=20)
    ap.add_argument("--no-families", action="store_true")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--profile", default=None, help="launch one family's kernel a few times (for ncu)")
    ap.add_argument("--launches", type=int, default=4)
    args = ap.parse_args()
    if args.profile:
        return run_profile_case(args.profile, args.launches)
    args.warmup = max(3, args.warmup)
    if args.impl == "reference":
        return run_reference(args)
    return run_tiler(args)


if __name__ == "__main__":
    sys.exit(main())

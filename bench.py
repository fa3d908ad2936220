#!/usr/bin/env python
"""Benchmark of the block-scaled GEMM path on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--workload moe|fp8_prefill|fp4_decode|moe_stack|act_quant|fp4_act_quant|
                                hc_sinkhorn|sparse_attn|indexer]

Default workload (one "step"): the grouped FP8 x FP4 MoE layer -- 1024 tokens,
hidden 4096, inter 2048, 256 experts, top-8 -- through the library's
single-kernel layer; at N>1 GPUs expert parallel (each rank its own tokens and
E/N experts, rows exchanged over NVLink peer memory inside the layer's
kernels), total batch fixed (strong scaling).  The same line carries the
4096^3 prefill fp8_gemm / fp4_gemm rates (one GPU).

Rank 0 prints one JSON line.  ``value`` is device-timed (CUDA events on the
launching stream, max over ranks) with inputs resident in HBM; every step
streams all expert weights (GiBs, far above L2).  ``roofline`` is the
dominant kernel's algorithmic bytes over its event-timed duration.  ``e2e``
times the public API from pinned host tokens and logits to a pinned host
copy of the output.  ``--impl reference`` times the reference's CPU
arithmetic (a torch restatement, oracle/torch_cpu.py) on the host cores.
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)
PKG = "deepseek-v4-experimental-platform-on-dgx-spark_b200"

# DRAM bytes (read + write) per launch of the dominant kernel, taken from one
# ncu capture of the same kernel at the same size (dram__bytes_read.sum +
# dram__bytes_write.sum); a recorded figure, not measured by this run.
# Output writes still in L2 when the kernel ends are not counted by ncu.
NCU_TRAFFIC = {
    "fp8_gemm_4096x4096x4096": 34_120_960 + 2_532_864,
    "fp4_decode_16x4096x4096": 9_046_784 + 0,
    "moe_layer_1024x256": None,
    # dram__bytes.sum.per_second x duration
    "act_quant_16384x7168": 325_000_000,
    "fp4_act_quant_16384x7168": 410_000_000,
}

PEAKS_FILE = os.path.join(ROOT, "MEASURED_PEAKS.json")
FALLBACK_PEAKS = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}


def load_peaks():
    try:
        with open(PEAKS_FILE) as f:
            return json.load(f), "measured"
    except Exception:
        return dict(FALLBACK_PEAKS), "fallback"


# ---------------------------------------------------------------------------
# distributed plumbing
# ---------------------------------------------------------------------------

def dist_env():
    ws = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return ws, rank, local


class Clocks:
    """Samples nvidia-smi during the timed region (SM clock, throttle reasons)."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "100"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except Exception:
            self.proc = None

    def stop(self):
        if self.proc is None:
            return None
        time.sleep(0.25)
        self.proc.terminate()
        try:
            out, _ = self.proc.communicate(timeout=5)
        except Exception:
            self.proc.kill()
            return None
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in out.strip().splitlines():
            f = [x.strip() for x in line.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx = float(f[2])
            except ValueError:
                continue
            for n, v in zip(names, f[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        if not sm:
            return None
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(sm)}


# ---------------------------------------------------------------------------
# workloads
# ---------------------------------------------------------------------------

def make_fp8_prefill(torch, dev, M, N, K, seed, n_sets):
    """Config-2 operands generated on the device (seeded)."""
    pkg = __import__("importlib").import_module(PKG)
    g = torch.Generator(device=dev)
    g.manual_seed(seed)
    sets = []
    for _ in range(n_sets):
        x = torch.randn(M, K, generator=g, device=dev, dtype=torch.float32).to(torch.bfloat16)
        a, a_s = pkg.act_quant(x, 128)
        w = torch.randn(N, K, generator=g, device=dev, dtype=torch.float32) * 0.02
        wb = w.view(N // 128, 128, K // 128, 128)
        s = (wb.abs().amax(dim=(1, 3)).clamp(min=1e-4) / 448.0)
        b = (wb / s[:, None, :, None]).clamp(-448, 448).to(torch.float8_e4m3fn).view(N, K)
        sets.append((a, a_s, b, s.contiguous(), x))
    return sets


class pipelined_e2e:
    """Single-GPU e2e steps on three streams with two buffers: step i copies
    the pinned host inputs in (stream in), runs `compute(i, *inputs_dev)`
    through the public API (stream compute) and copies the result out to
    pinned host memory (stream out).  Step i+2 reuses step i's buffers only
    after step i's compute and copy-out are done, so steps overlap without
    sharing data.  `x_host` is one pinned tensor or a tuple of them."""

    def __init__(self, torch, x_host, out_shape, compute):
        self.torch, self.compute = torch, compute
        self.x_host = tuple(x_host) if isinstance(x_host, (tuple, list)) else (x_host,)
        dev = torch.device("cuda", torch.cuda.current_device())
        self.x_dev = [[torch.empty(h.shape, dtype=h.dtype, device=dev) for h in self.x_host] for _ in range(2)]
        self.o_host = [torch.empty(out_shape, dtype=torch.bfloat16).pin_memory() for _ in range(2)]
        self.s_in, self.s_comp, self.s_out = (torch.cuda.Stream() for _ in range(3))
        self.in_done = [torch.cuda.Event() for _ in range(2)]
        self.comp_done = [torch.cuda.Event() for _ in range(2)]
        self.out_done = [torch.cuda.Event() for _ in range(2)]
        main = torch.cuda.current_stream()
        for s in (self.s_in, self.s_comp, self.s_out):
            s.wait_stream(main)
        for e in self.comp_done + self.out_done:
            e.record(main)

    def __call__(self, i):
        torch, b = self.torch, i & 1
        with torch.cuda.stream(self.s_in):
            self.s_in.wait_event(self.comp_done[b])          # step i-2 has read x_dev[b]
            for d, h in zip(self.x_dev[b], self.x_host):
                d.copy_(h, non_blocking=True)
            self.in_done[b].record()
        with torch.cuda.stream(self.s_comp):
            self.s_comp.wait_event(self.in_done[b])
            self.s_comp.wait_event(self.out_done[b])         # step i-2's result has left its buffer
            c = self.compute(i, *self.x_dev[b])
            c.record_stream(self.s_out)
            self.comp_done[b].record()
        with torch.cuda.stream(self.s_out):
            self.s_out.wait_event(self.comp_done[b])
            self.o_host[b].copy_(c, non_blocking=True)
            self.out_done[b].record()

    def start(self):
        """Order the streams after everything already on the current stream
        (the start event of a timed region)."""
        main = self.torch.cuda.current_stream()
        for s in (self.s_in, self.s_comp, self.s_out):
            s.wait_stream(main)

    def join(self):
        main = self.torch.cuda.current_stream()
        for s in (self.s_in, self.s_comp, self.s_out):
            main.wait_stream(s)


def bench_fp8_prefill(args, torch, dist, ws, rank, dev):
    pkg = __import__("importlib").import_module(PKG)
    M = N = K = 4096
    if N % (ws * 128):
        raise SystemExit("N must split into 128-row blocks per rank")
    n_local = N // ws
    n_sets = 5  # 5 x (16 MiB A + 16/ws MiB B) rotating: inputs >> L2 across consecutive steps
    sets = make_fp8_prefill(torch, dev, M, N, K, 1234, n_sets)
    # this rank's column shard of every weight copy
    shards = [(a, a_s, b[rank * n_local:(rank + 1) * n_local].contiguous(),
               s[rank * n_local // 128:(rank + 1) * n_local // 128].contiguous()) for a, a_s, b, s, _ in sets]
    outs = [torch.empty(M, n_local, device=dev, dtype=torch.bfloat16) for _ in range(2)]
    gathered = torch.empty(ws, M, n_local, device=dev, dtype=torch.bfloat16)
    full = torch.empty(M, N, device=dev, dtype=torch.bfloat16)
    lib = pkg._lib.load()
    stream = torch.cuda.current_stream()
    # N > 1: the GEMM epilogue stores every tile into all ranks' C over NVLink
    # (fused), or the shard is gathered afterwards with NCCL (nccl)
    fused = ws > 1 and args.tp_gather == "fused"
    tpg = None
    if fused:
        tpg = __import__("importlib").import_module(PKG + ".tp").TPGemm(M, N, K, device=dev)

    def gemm(i, out):
        a, a_s, b, s = shards[i % n_sets]
        if fused:
            # the fused kernel alone (no barrier): timing of the GEMM + peer stores
            pkg._lib.check(lib.bs_fp8_gemm_allgather(
                a.data_ptr(), a_s.data_ptr(), pkg._lib.DT_F32, b.data_ptr(), s.data_ptr(), pkg._lib.DT_F32,
                M, n_local, K, tpg.ptrs[i & 1], ws, N, tpg.col0, stream.cuda_stream))
            return
        pkg._lib.check(lib.bs_fp8_gemm(a.data_ptr(), a_s.data_ptr(), pkg._lib.DT_F32, b.data_ptr(), s.data_ptr(),
                                       pkg._lib.DT_F32, M, n_local, K, out.data_ptr(), stream.cuda_stream))

    def step(i):
        if fused:
            a, a_s, b, s = shards[i % n_sets]
            tpg(a, a_s, b, s)
            return
        out = outs[i & 1]
        gemm(i, out)
        if ws > 1:
            dist.all_gather_into_tensor(gathered, out)
            full.view(M, ws, n_local).copy_(gathered.permute(1, 0, 2))

    for i in range(args.warmup):
        step(i)
    torch.cuda.synchronize()

    # kernel-only timing of the GEMM (roofline numerator), separate short loop
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(args.steps)]
    for i in range(args.steps):
        ev[i][0].record()
        gemm(i, outs[i & 1])
        ev[i][1].record()
    torch.cuda.synchronize()
    kern_ms = statistics.mean(e0.elapsed_time(e1) for e0, e1 in ev)

    clocks = Clocks(torch.cuda.current_device())
    if dist is not None:
        dist.barrier()
    torch.cuda.synchronize()
    clocks.start()
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t0.record()
    for i in range(args.steps):
        step(i)
    t1.record()
    torch.cuda.synchronize()
    if dist is not None:
        dist.barrier()
    clk = clocks.stop()
    ms = t0.elapsed_time(t1) / args.steps
    ms = max_over_ranks(torch, dist, ms)
    kern_ms = max_over_ranks(torch, dist, kern_ms)
    flops = 2.0 * M * N * K
    value = flops / (ms * 1e-3) / 1e12

    # end to end through the public API: pinned host bf16 activations ->
    # act_quant -> fp8_gemm (local shard) [-> all-gather] -> pinned host output
    x_host = sets[0][4].cpu().pin_memory()
    o_host = torch.empty(M, N if ws > 1 else n_local, dtype=torch.bfloat16).pin_memory()
    x_dev = torch.empty_like(sets[0][4])
    b_loc, s_loc = shards[0][2], shards[0][3]

    def e2e_step(i=0):
        x_dev.copy_(x_host, non_blocking=True)
        a, a_s = pkg.act_quant(x_dev, 128)
        if fused:
            c = tpg(a, a_s, b_loc, s_loc)
        else:
            c = pkg.fp8_gemm(a, a_s, b_loc, s_loc)
            if ws > 1:
                dist.all_gather_into_tensor(gathered, c)
                full.view(M, ws, n_local).copy_(gathered.permute(1, 0, 2))
                c = full
        if rank == 0:      # every rank holds the gathered C: the job reads it out once
            o_host.copy_(c, non_blocking=True)

    if ws == 1:
        # one GPU: consecutive steps overlap on three streams (inputs in,
        # compute, result out; two buffers each), as a serving loop would run
        # them; every step still copies its own input in and its result out
        e2e_step = pipelined_e2e(torch, x_host, o_host.shape,
                                 lambda i, xd: pkg.fp8_gemm(*pkg.act_quant(xd, 128), b_loc, s_loc))
    for i in range(2):
        e2e_step(i)
    torch.cuda.synchronize()
    if dist is not None:
        dist.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    if ws == 1:
        e2e_step.start()
    for i in range(args.steps):
        e2e_step(i)
    if ws == 1:
        e2e_step.join()
    e1.record()
    torch.cuda.synchronize()
    e2e_ms = max_over_ranks(torch, dist, e0.elapsed_time(e1) / args.steps)

    if tpg is not None:
        torch.cuda.synchronize()
        pkg._lib.device_error_check()
        tpg.close()
    peaks, src = load_peaks()
    peak = 2.0 * peaks["bf16_tflops"]  # dense e4m3 rate = 2x the measured dense bf16 rate
    local_flops = 2.0 * M * n_local * K
    achieved = local_flops / (kern_ms * 1e-3) / 1e12
    nvlink = None
    if fused:
        # fused GEMM + all-gather: the kernel cannot beat the slower of its math
        # at the tensor peak and the gathered bytes it must receive (and send)
        # over NVLink at the measured 770 GB/s per direction
        gathered_bytes = (ws - 1) * M * n_local * 2
        t_math = local_flops / (peak * 1e12)
        t_link = gathered_bytes / 770e9
        peak = local_flops / max(t_math, t_link) / 1e12
        nvlink = {"bytes_per_gpu": gathered_bytes, "gbs_per_direction": 770.0,
                  "target_ms": round(max(t_math, t_link) * 1e3, 4),
                  "bound_by": "nvlink" if t_link > t_math else "tensor"}
    traffic = NCU_TRAFFIC.get(f"fp8_gemm_{M}x{n_local}x{K}")
    line = {
        "metric": "block-scaled FP8 GEMM TFLOP/s (dense fp8_gemm, 1x128 act + 128x128 weight fp32 scales)",
        "value": round(value, 2), "unit": "TFLOP/s", "n_gpus": ws, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(ms, 4), "higher_is_better": True, "scaling": "strong" if ws > 1 else "weak",
        "vs_baseline": None, "dtype": "e4m3", "data": "synthetic (seeded N(0,1) activations, N(0,0.02) weights)",
        "config": {"workload": f"fp8_gemm M=N=K={M}" + (
                       (f", column-sharded TP{ws}, all-gather fused into the GEMM epilogue (NVLink peer stores)"
                        if fused else f", column-sharded TP{ws} + NCCL all-gather") if ws > 1 else ""),
                   "M": M, "N": N, "K": K, "parallelism": f"tp{ws}" if ws > 1 else "none",
                   "l2": f"{n_sets} rotating input sets ({n_sets * (M * K + n_local * K) // 2**20} MiB) > L2"},
        "e2e": {"value": round(flops / (e2e_ms * 1e-3) / 1e12, 2), "unit": "TFLOP/s",
                "h2d_bytes_per_step": M * K * 2, "d2h_bytes_per_step": M * (N if ws > 1 else n_local) * 2,
                "ms_per_step": round(e2e_ms, 4),
                "path": "act_quant + fp8_gemm public API, pinned host I/O" + (
                    "; consecutive steps overlapped on copy-in / compute / copy-out streams" if ws == 1 else
                    "; every rank copies its input in, rank 0 copies the gathered C out")},
        "roofline": {"bound": "tensor", "achieved": round(achieved, 1), "peak": round(peak, 1), "unit": "TFLOP/s",
                     "frac": round(achieved / peak, 3), "traffic": traffic,
                     "kernel": "bsg_kernel<normal,fp8,BN=256>" + (" + peer stores" if fused else ""),
                     "kernel_ms": round(kern_ms, 4),
                     "peak_source": f"2 x bf16_tflops of {src} MEASURED_PEAKS.json (dense e4m3 rate)"
                                    + ("; min with NVLink 770 GB/s per direction for the gathered bytes"
                                       if fused else ""),
                     "nvlink": nvlink},
        "gpu_launches": args.steps * (2 if fused else 1),
        "clocks": clk,
    }
    return line


def bench_fp4_decode(args, torch, dist, ws, rank, dev):
    """Config-3 decode sweep point (M tokens, K=4096, N), HBM-bound."""
    pkg = __import__("importlib").import_module(PKG)
    M, N, K = args.m, args.n, 4096
    g = torch.Generator(device=dev)
    g.manual_seed(77)
    n_sets = max(8, int(np.ceil(400e6 / (N * K // 2))))  # >= 400 MB of distinct weights: no L2 reuse
    x = torch.randn(M, K, generator=g, device=dev).to(torch.bfloat16)
    a, a_s = pkg.act_quant(x, 128)
    ws_ = [(torch.randint(0, 256, (N, K // 2), generator=g, device=dev, dtype=torch.uint8),
            (127 - torch.randint(0, 7, (N, K // 32), generator=g, device=dev, dtype=torch.uint8)))
           for _ in range(n_sets)]
    out = torch.empty(M, N, device=dev, dtype=torch.bfloat16)
    lib = pkg._lib.load()
    st = torch.cuda.current_stream().cuda_stream

    def step(i):
        b, bs = ws_[i % n_sets]
        pkg._lib.check(lib.bs_fp4_gemm(a.data_ptr(), a_s.data_ptr(), pkg._lib.DT_F32, b.data_ptr(), bs.data_ptr(),
                                       pkg._lib.DT_E8M0, M, N, K, out.data_ptr(), st))

    for i in range(max(args.warmup, n_sets)):
        step(i)
    torch.cuda.synchronize()
    # Decode GEMMs run back to back inside a captured CUDA graph, as a decode
    # step does: host launch cost leaves the timed region, and programmatic
    # dependent launch lets each GEMM stream its weights while the previous
    # one drains.  One replay = `steps` calls over rotating weight copies.
    steps = max(args.steps, 2 * n_sets)
    graph = torch.cuda.CUDAGraph()
    cap = torch.cuda.Stream()
    cap.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(cap):
        st = cap.cuda_stream
        with torch.cuda.graph(graph, stream=cap):
            for i in range(steps):
                b, bs = ws_[i % n_sets]
                pkg._lib.check(lib.bs_fp4_gemm(a.data_ptr(), a_s.data_ptr(), pkg._lib.DT_F32, b.data_ptr(),
                                               bs.data_ptr(), pkg._lib.DT_E8M0, M, N, K, out.data_ptr(),
                                               cap.cuda_stream))
    torch.cuda.current_stream().wait_stream(cap)
    for _ in range(2):
        graph.replay()
    torch.cuda.synchronize()
    reps = 5
    clocks = Clocks(torch.cuda.current_device())
    clocks.start()
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t0.record()
    for _ in range(reps):
        graph.replay()
    t1.record()
    torch.cuda.synchronize()
    clk = clocks.stop()
    ms = t0.elapsed_time(t1) / (reps * steps)
    # the same sequence launched call by call from Python (host-bound)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for i in range(steps):
        step(i)
    e1.record()
    torch.cuda.synchronize()
    ms_eager = e0.elapsed_time(e1) / steps
    # end to end through the public API, as a decode loop runs it: each call
    # copies its bf16 activations in from pinned host memory, runs act_quant
    # and fp4_gemm (rotating resident weights) and copies its output back to
    # pinned host memory; the calls are captured once in a CUDA graph
    wv = [(b.view(torch.float4_e2m1fn_x2), bs.view(torch.float8_e8m0fnu)) for b, bs in ws_]
    x_host = x.cpu().pin_memory()
    o_host = torch.empty(M, N, dtype=torch.bfloat16).pin_memory()
    x_dev = torch.empty_like(x)

    def e2e_call(i):
        x_dev.copy_(x_host, non_blocking=True)
        o_host.copy_(pkg.fp4_gemm(*pkg.act_quant(x_dev, 128), *wv[i % n_sets]), non_blocking=True)

    for i in range(2):
        e2e_call(i)
    torch.cuda.synchronize()
    g_e2e = torch.cuda.CUDAGraph()
    cap.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(cap):
        with torch.cuda.graph(g_e2e, stream=cap):
            for i in range(steps):
                e2e_call(i)
    torch.cuda.current_stream().wait_stream(cap)
    g_e2e.replay()
    torch.cuda.synchronize()
    e0.record()
    for _ in range(reps):
        g_e2e.replay()
    e1.record()
    torch.cuda.synchronize()
    e2e_ms = e0.elapsed_time(e1) / (reps * steps)
    nbytes = N * K // 2 + N * K // 32 + M * K + 4 * M * K // 128 + 2 * M * N
    gbs = nbytes / (ms * 1e-3) / 1e9
    peaks, src = load_peaks()
    return {"metric": "fp4_gemm decode HBM GB/s", "value": round(gbs, 1), "unit": "GB/s", "n_gpus": 1,
            "steps": steps, "warmup": args.warmup, "ms_per_step": round(ms, 5), "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "e4m3 x e2m1",
            "data": "synthetic", "config": {"workload": f"fp4_gemm decode M={M} N={N} K={K}",
                                            "l2": f"{n_sets} rotating weight copies"},
            "roofline": {"bound": "hbm", "achieved": round(gbs, 1), "peak": peaks["hbm_gbs"], "unit": "GB/s",
                         "frac": round(gbs / peaks["hbm_gbs"], 3),
                         "traffic": NCU_TRAFFIC.get(f"fp4_decode_{M}x{N}x{K}"), "peak_source": src},
            "e2e": {"value": round(nbytes / (e2e_ms * 1e-3) / 1e9, 1), "unit": "GB/s",
                    "h2d_bytes_per_step": M * K * 2, "d2h_bytes_per_step": M * N * 2,
                    "ms_per_step": round(e2e_ms, 5),
                    "path": "act_quant + fp4_gemm public API per call with pinned host copies in and out, "
                            "calls replayed from one CUDA graph"},
            "gpu_launches": steps * reps, "clocks": clk,
            "eager_ms_per_call": round(ms_eager, 5)}


def moe_weights(torch, dev, El, H, I, seed):
    """One rank's experts: packed e2m1 codes uniform over all 16 values,
    ue8m0 1x32 scales with exponents uniform in [-6, 0]."""
    g = torch.Generator(device=dev)
    g.manual_seed(seed)
    w13 = torch.randint(0, 256, (El, 2 * I, H // 2), generator=g, device=dev, dtype=torch.uint8)
    w13_s = 127 - torch.randint(0, 7, (El, 2 * I, H // 32), generator=g, device=dev, dtype=torch.uint8)
    w2 = torch.randint(0, 256, (El, H, I // 2), generator=g, device=dev, dtype=torch.uint8)
    w2_s = 127 - torch.randint(0, 7, (El, H, I // 32), generator=g, device=dev, dtype=torch.uint8)
    return w13, w13_s, w2, w2_s


def prefill_gemm_rates(torch, dev, peaks):
    """Device-timed 4096^3 prefill GEMMs through the C ABI: fp8_gemm (1x128
    activation, 128x128 weight fp32 scales: the dense projection shape) and
    fp4_gemm (1x128 fp32 activation scales, packed e2m1 weights with ue8m0 1x32
    scales); five rotating operand sets (> L2)."""
    pkg = __import__("importlib").import_module(PKG)
    lib = pkg._lib.load()
    M = N = K = 4096
    sets = make_fp8_prefill(torch, dev, M, N, K, 1234, 5)
    g = torch.Generator(device=dev)
    g.manual_seed(99)
    w4 = [(torch.randint(0, 256, (N, K // 2), generator=g, device=dev, dtype=torch.uint8),
           127 - torch.randint(0, 7, (N, K // 32), generator=g, device=dev, dtype=torch.uint8)) for _ in sets]
    out = torch.empty(M, N, device=dev, dtype=torch.bfloat16)
    st = torch.cuda.current_stream().cuda_stream
    res = {}
    for name in ("fp8_gemm", "fp4_gemm"):
        def call(i):
            a, a_s, b, s, _ = sets[i % len(sets)]
            if name == "fp8_gemm":
                pkg._lib.check(lib.bs_fp8_gemm(a.data_ptr(), a_s.data_ptr(), pkg._lib.DT_F32, b.data_ptr(),
                                               s.data_ptr(), pkg._lib.DT_F32, M, N, K, out.data_ptr(), st))
            else:
                b4, s4 = w4[i % len(w4)]
                pkg._lib.check(lib.bs_fp4_gemm(a.data_ptr(), a_s.data_ptr(), pkg._lib.DT_F32, b4.data_ptr(),
                                               s4.data_ptr(), pkg._lib.DT_E8M0, M, N, K, out.data_ptr(), st))
        for i in range(5):
            call(i)
        n = 20
        t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        torch.cuda.synchronize()
        t0.record()
        for i in range(n):
            call(i)
        t1.record()
        torch.cuda.synchronize()
        ms = t0.elapsed_time(t1) / n
        tf = 2.0 * M * N * K / (ms * 1e-3) / 1e12
        res[name] = {"tflops": round(tf, 1), "ms": round(ms, 4), "frac": round(tf / (2.0 * peaks["bf16_tflops"]), 3),
                     "shape": "M=N=K=4096"}
    res["peak_note"] = "frac of 2 x measured dense bf16 (the e4m3 / e2m1 tensor rate)"
    return res


def cpu_moe_sample(torch, x, logits, weights_cpu_fetch, E, k, budget_s=12.0, min_experts=4, max_experts=None,
                   seed=0):
    """The reference's CPU arithmetic for the MoE layer (oracle/torch_cpu.py:
    act_quant + three LUT-dequant bf16 fp4_gemm per active expert) on the
    host cores, over a sample of the active experts (seeded order) until
    `budget_s` is spent.  Returns (layer seconds extrapolated to every active
    expert, experts timed, active experts)."""
    from oracle import torch_cpu as tc
    idx = torch.topk(logits, k, dim=1).indices
    active = torch.unique(idx).tolist()
    order = torch.randperm(len(active), generator=torch.Generator().manual_seed(seed)).tolist()
    xs = x.float().to(torch.bfloat16)
    w = torch.softmax(torch.topk(logits, k, dim=1).values, dim=1)
    out = torch.zeros(x.shape, dtype=torch.float32)
    done, t_total = 0, 0.0
    for o in order:
        e = active[o]
        W = weights_cpu_fetch(e)
        t = time.perf_counter()
        tc.moe_experts(xs, idx, w, [e], *({e: t} for t in W), out)
        t_total += time.perf_counter() - t
        done += 1
        if (t_total >= budget_s and done >= min_experts) or (max_experts and done >= max_experts):
            break
    return t_total * len(active) / done, done, len(active)


def bench_moe(args, torch, dist, ws, rank, dev):
    """MoE layer (the grouped FP8 x FP4 form): T tokens in total (default
    1024), H=4096, I=2048, E=256 experts, top-8 of N(0,1) gate logits,
    weights = softmax over the top 8.

    One GPU: the whole layer (bs_moe_forward: one kernel whose phases are
    quantise + route + dispatch, the grouped GEMMs, and the combine).  N
    GPUs: expert parallel -- rank r owns tokens [r*T/N, (r+1)*T/N) and
    experts [r*E/N, (r+1)*E/N); rows travel to the expert owners and back
    over NVLink peer memory inside the layer's own kernels (or, with
    --ep-transport nccl, by NCCL all-to-all); strong scaling: the total
    batch is fixed.
    """
    import importlib
    pkg = importlib.import_module(PKG)
    moe = importlib.import_module(PKG + ".moe")
    lib = pkg._lib.load()
    T, H, I, E, k = args.tokens, 4096, 2048, args.experts, 8
    if T % ws or E % ws:
        raise SystemExit("tokens and experts must split evenly over the ranks")
    g = torch.Generator(device=dev)
    g.manual_seed(4)
    x = torch.randn(T, H, generator=g, device=dev).to(torch.bfloat16)        # same on every rank
    logits = torch.randn(T, E, generator=g, device=dev)
    El, tl = E // ws, T // ws
    w13, w13_s, w2, w2_s = moe_weights(torch, dev, El, H, I, 1000 + rank)     # this rank's experts
    weights = moe.MoEWeights(w13, w13_s, w2, w2_s)
    xl, ll = x[rank * tl:(rank + 1) * tl].contiguous(), logits[rank * tl:(rank + 1) * tl].contiguous()
    outs = [torch.empty(tl, H, dtype=torch.bfloat16, device=dev) for _ in range(2)]
    layer, graph = None, None
    if ws == 1:
        def call(xd, ld, o):
            return moe.moe_forward(xd, ld, weights, k, out=o)
        launches = 1
    else:
        ep = importlib.import_module(PKG + ".ep")
        layer = ep.EPMoE(weights, E, k, max_tokens=tl, transport=args.ep_transport)

        def call(xd, ld, o):
            return layer.forward(xd, ld, out=o)
        launches = 1 if args.ep_transport == "peer" else 9
    step = lambda: call(xl, ll, outs[0])                                        # noqa: E731
    if ws > 1 and args.ep_transport == "peer":
        # no host sync inside the layer: capture it once, replay one graph per step
        for _ in range(2):
            step()
        torch.cuda.synchronize()
        graph = torch.cuda.CUDAGraph()
        cap = torch.cuda.Stream()
        cap.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(cap):
            with torch.cuda.graph(graph, stream=cap):
                step()
        torch.cuda.current_stream().wait_stream(cap)
        step = graph.replay
    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    if dist is not None:
        dist.barrier()
    clocks = Clocks(torch.cuda.current_device())
    clocks.start()
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t0.record()
    for _ in range(args.steps):
        step()
    t1.record()
    torch.cuda.synchronize()
    if dist is not None:
        dist.barrier()
    clk = clocks.stop()
    ms = max_over_ranks(torch, dist, t0.elapsed_time(t1) / args.steps)

    # the layer kernel (all of the layer's work), timed live with events the
    # library records around it on the launching stream
    kern_ms = None
    if args.ep_transport == "peer" or ws == 1:
        evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(args.steps)]
        for e0, e1 in evs:
            e0.record()
            e1.record()                       # creates the events
        torch.cuda.synchronize()
        if dist is not None:
            dist.barrier()
        for e0, e1 in evs:
            lib.bs_moe_time_layer(e0.cuda_event, e1.cuda_event)
            call(xl, ll, outs[0])
        torch.cuda.synchronize()
        kern_ms = max_over_ranks(torch, dist, statistics.mean(e0.elapsed_time(e1) for e0, e1 in evs))
    # rows this rank's experts receive (routing is a pure function of the logits)
    top = torch.topk(logits, k, dim=1).indices
    recv = int(((top >= rank * El) & (top < (rank + 1) * El)).sum().item())
    wbytes = w13.numel() + w13_s.numel() + w2.numel() + w2_s.numel()            # this rank's weights + scales
    # activation bytes of this rank's HBM: its bf16 tokens and fp32 logits in,
    # received e4m3 rows + scale words written (by the dispatch) and read (by
    # the GEMMs), hidden rows written and read, its rows' bf16 expert outputs
    # written (by the owners) and read (by the combine), bf16 output out
    abytes = (tl * (H * 2 + E * 4) + 2 * recv * (H + H // 32) + 2 * recv * (I + I // 32) + 2 * tl * k * H * 2
              + tl * H * 2)
    kbytes = wbytes + abytes
    peaks, src = load_peaks()
    gbs = kbytes / (kern_ms * 1e-3) / 1e9 if kern_ms else None
    traffic = NCU_TRAFFIC.get(f"moe_layer_{T // ws}x{E // ws}") if ws == 1 else None

    # end to end through the public API: pinned host bf16 tokens and fp32 gate
    # logits -> device -> the layer -> pinned host output, consecutive steps
    # overlapped on copy-in / compute / copy-out streams
    x_host, l_host = xl.cpu().pin_memory(), ll.cpu().pin_memory()
    e2e_step = pipelined_e2e(torch, (x_host, l_host), (tl, H), lambda i, xd, ld: call(xd, ld, outs[i & 1]))
    for i in range(2):
        e2e_step(i)
    torch.cuda.synchronize()
    if dist is not None:
        dist.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    e2e_step.start()
    for i in range(args.steps):
        e2e_step(i)
    e2e_step.join()
    e1.record()
    torch.cuda.synchronize()
    e2e_ms = max_over_ranks(torch, dist, e0.elapsed_time(e1) / args.steps)
    if ws > 1:
        del graph
        torch.cuda.synchronize()
        pkg._lib.device_error_check()
        layer.close()
    line = {"metric": "MoE-layer tokens/s", "value": round(T / (ms * 1e-3), 1), "unit": "tokens/s", "n_gpus": ws,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms, 4), "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "e4m3 x e2m1",
            "data": "synthetic (seeded N(0,1) tokens and gate logits, uniform e2m1 codes, ue8m0 exponents in [-6,0])",
            "config": {"workload": f"MoE layer T={T} H={H} I={I} E={E} top-{k} (grouped FP8xFP4 GEMMs)",
                       "parallelism": f"ep{ws}" if ws > 1 else "none",
                       "exchange": (("NVLink peer memory inside the layer's kernels (no NCCL, no host sync)"
                                     if args.ep_transport == "peer" else "NCCL all-to-all") if ws > 1 else None),
                       "l2": f"expert weights {wbytes * ws / 2**30:.2f} GiB >> L2 (every step streams them)"},
            "roofline": {"bound": "hbm", "achieved": round(gbs, 1) if gbs else None, "peak": peaks["hbm_gbs"],
                         "unit": "GB/s", "frac": round(gbs / peaks["hbm_gbs"], 3) if gbs else None,
                         "traffic": traffic,
                         "traffic_source": "recorded ncu capture of this kernel at this size (not measured in this "
                                           "run)" if traffic else None,
                         "kernel": "mf::layer_kernel (the whole layer: quantise + route + dispatch, persistent "
                                   "W1|W3 + W2 grouped GEMMs, combine)",
                         "kernel_ms": round(kern_ms, 4) if kern_ms else None,
                         "algorithmic_bytes": kbytes,
                         "note": "this rank's expert weights + scales, tokens + logits in, received rows written and "
                                 "read, hidden rows written and read, returned outputs written and read, output out, "
                                 "per launch / the kernel's event-timed duration (max over ranks)",
                         "peak_source": f"hbm_gbs of {src} MEASURED_PEAKS.json"},
            "e2e": {"value": round(T / (e2e_ms * 1e-3), 1), "unit": "tokens/s",
                    "h2d_bytes_per_step": ws * tl * (H * 2 + E * 4), "d2h_bytes_per_step": ws * tl * H * 2,
                    "ms_per_step": round(e2e_ms, 4),
                    "path": "moe_forward / EPMoE.forward public API, pinned host tokens + logits in, output out; "
                            "consecutive steps overlapped on copy-in / compute / copy-out streams"},
            "gpu_launches": args.steps * launches, "clocks": clk}
    if ws == 1:
        line["prefill_gemm"] = prefill_gemm_rates(torch, dev, peaks)
    if rank == 0 and ws == 1 and not args.no_cpu_baseline:
        torch.set_num_threads(cpu_threads())
        xc, lc = x.cpu(), logits.cpu()
        fetch = lambda e: (w13[e].cpu(), w13_s[e].cpu().view(torch.float8_e8m0fnu), w2[e].cpu(),   # noqa: E731
                           w2_s[e].cpu().view(torch.float8_e8m0fnu))
        layer_s, n_done, n_act = cpu_moe_sample(torch, xc, lc, fetch, E, k)
        line["cpu_baseline"] = {"value": round(T / layer_s, 2), "unit": "tokens/s", "cores": cpu_threads(),
                                "kind": "port",
                                "sample": f"{n_done} of the {n_act} active experts with all their routed tokens "
                                          f"through the torch restatement of the reference's CPU ops (act_quant + "
                                          f"LUT-dequant bf16 fp4_gemm x3 per expert); layer time extrapolated to "
                                          f"all active experts: {layer_s:.2f} s"}
    return line


def bench_quant(args, torch, dist, ws, rank, dev):
    """The quantisers that feed the GEMMs, on bf16 [rows, 7168] (rows = --tokens, default 16384):
    act_quant (1x128 blocks, e4m3 + fp32 scales; 3 B per element + 4 B per block) or the
    in-place fp4_act_quant (blocks of 32; 4 B per element).  One step = one call; the calls run
    from one CUDA graph over three rotating inputs, each larger than L2.  N GPUs: independent
    replicas (weak scaling), value = all ranks' bytes / the slowest rank's time."""
    pkg = __import__("importlib").import_module(PKG)
    lib = pkg._lib.load()
    fp4 = args.workload == "fp4_act_quant"
    R, K = args.tokens, 7168
    n_sets = 3
    g = torch.Generator(device=dev)
    g.manual_seed(5 + rank)
    xs = [torch.randn(R, K, generator=g, device=dev).to(torch.bfloat16) for _ in range(n_sets)]
    y = torch.empty(R, K, dtype=torch.uint8, device=dev)
    s_ = torch.empty(R, K // 128, dtype=torch.float32, device=dev)

    def call(i, st):
        x = xs[i % n_sets]
        if fp4:
            pkg._lib.check(lib.bs_fp4_act_quant_inplace(x.data_ptr(), pkg._lib.DT_BF16, R, K, 32, st))
        else:
            pkg._lib.check(lib.bs_act_quant(x.data_ptr(), pkg._lib.DT_BF16, R, K, 128, 0, y.data_ptr(),
                                            s_.data_ptr(), pkg._lib.DT_F32, st))

    cur = torch.cuda.current_stream().cuda_stream
    for i in range(max(args.warmup, n_sets)):
        call(i, cur)
    torch.cuda.synchronize()
    steps = max(args.steps, 2 * n_sets)
    graph = torch.cuda.CUDAGraph()
    cap = torch.cuda.Stream()
    cap.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(cap):
        with torch.cuda.graph(graph, stream=cap):
            for i in range(steps):
                call(i, cap.cuda_stream)
    torch.cuda.current_stream().wait_stream(cap)
    graph.replay()
    torch.cuda.synchronize()
    if dist is not None:
        dist.barrier()
    reps = 3
    clocks = Clocks(torch.cuda.current_device())
    clocks.start()
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t0.record()
    for _ in range(reps):
        graph.replay()
    t1.record()
    torch.cuda.synchronize()
    clk = clocks.stop()
    ms = max_over_ranks(torch, dist, t0.elapsed_time(t1) / (reps * steps))
    nbytes = R * K * 4 if fp4 else R * K * 3 + R * (K // 128) * 4
    gbs = ws * nbytes / (ms * 1e-3) / 1e9
    # end to end through the public API: bf16 rows in from pinned host memory, the result back
    x_host = xs[0].cpu().pin_memory()
    x_dev = torch.empty_like(xs[0])
    y_host = torch.empty(R, K, dtype=torch.bfloat16 if fp4 else torch.uint8).pin_memory()
    s_host = torch.empty(R, K // 128, dtype=torch.float32).pin_memory()

    def e2e_call():
        x_dev.copy_(x_host, non_blocking=True)
        if fp4:
            y_host.copy_(pkg.fp4_act_quant(x_dev, 32, True), non_blocking=True)
        else:
            yq, sq = pkg.act_quant(x_dev, 128)
            y_host.copy_(yq.view(torch.uint8), non_blocking=True)
            s_host.copy_(sq, non_blocking=True)

    e2e_call()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e2e_steps = 3
    e0.record()
    for _ in range(e2e_steps):
        e2e_call()
    e1.record()
    torch.cuda.synchronize()
    e2e_ms = max_over_ranks(torch, dist, e0.elapsed_time(e1) / e2e_steps)
    d2h = R * K * (2 if fp4 else 1) + (0 if fp4 else R * (K // 128) * 4)
    peaks, src = load_peaks()
    name = "fp4_act_quant bf16 block 32 (in place)" if fp4 else "act_quant bf16 1x128 -> e4m3 + fp32 scales"
    key = f"{args.workload}_{R}x{K}"
    line = {"metric": f"{args.workload} HBM GB/s", "value": round(gbs, 1), "unit": "GB/s", "n_gpus": ws,
            "steps": steps, "warmup": args.warmup, "ms_per_step": round(ms, 5), "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "bf16 -> e2m1 grid" if fp4 else "bf16 -> e4m3",
            "data": "synthetic (seeded N(0,1))",
            "config": {"workload": f"{name}, [{R}, {K}]", "l2": f"{n_sets} rotating inputs of {R * K * 2 >> 20} MiB",
                       "parallelism": f"replicas x{ws}" if ws > 1 else "none"},
            "roofline": {"bound": "hbm", "achieved": round(nbytes / (ms * 1e-3) / 1e9, 1), "peak": peaks["hbm_gbs"],
                         "unit": "GB/s", "frac": round(nbytes / (ms * 1e-3) / 1e9 / peaks["hbm_gbs"], 3),
                         "traffic": NCU_TRAFFIC.get(key), "peak_source": src},
            "e2e": {"value": round(ws * nbytes / (e2e_ms * 1e-3) / 1e9, 1), "unit": "GB/s",
                    "h2d_bytes_per_step": R * K * 2, "d2h_bytes_per_step": d2h, "ms_per_step": round(e2e_ms, 4),
                    "path": ("fp4_act_quant" if fp4 else "act_quant") +
                            " public API with the rows copied in from and the result out to pinned host memory"},
            "gpu_launches": steps * reps, "clocks": clk}
    if rank == 0 and ws == 1 and not args.no_cpu_baseline:
        from oracle import blockscaled as ob
        rows = 512
        xh = xs[0][:rows].view(torch.int16).cpu().numpy().view(np.uint16)
        t = time.perf_counter()
        if fp4:
            ob.fp4_act_quant_inplace(xh, ob.DT_BF16, 32)
        else:
            ob.act_quant(xh, ob.DT_BF16, 128, None, ob.DT_F32)
        dt = time.perf_counter() - t
        line["cpu_baseline"] = {"value": round(rows * nbytes / R / dt / 1e9, 3), "unit": "GB/s", "cores": 1,
                                "kind": "port", "sample": f"{rows} of the {R} rows through the numpy port of the "
                                                          f"reference's quantiser ({dt * 1e3:.0f} ms)"}
    return line


def bench_attn_side(args, torch, dist, ws, rank, dev):
    """The attention-side consumers (one GPU; N GPUs run replicas, weak scaling):
    hc_split_sinkhorn on [1, 65536, 24] fp32 mixes (hc=4, 20 iterations;
    HBM GB/s of mixes in + pre/post/comb out), sparse_attn on a 4096-query
    prefill (16 heads x 576, 512 keys per query from a 1024-row cache, bf16;
    TFLOP/s of the two contractions), the Indexer's score -> top-k on 4096
    queries x 1024 keys (64 heads x 128, fp32; TFLOP/s of the scores)."""
    pkg = __import__("importlib").import_module(PKG)
    kern = pkg.kernel
    g = torch.Generator(device=dev)
    g.manual_seed(31 + rank)
    peaks, src = load_peaks()
    if args.workload == "hc_sinkhorn":
        n, hc = 65536, 4
        mix = torch.randn(1, n, (2 + hc) * hc, generator=g, device=dev)
        sc = torch.rand(3, generator=g, device=dev) + 0.5
        base = torch.randn((2 + hc) * hc, generator=g, device=dev)
        call = lambda: kern.hc_split_sinkhorn(mix, sc, base, hc, 20, 1e-6)       # noqa: E731
        work, unit, metric = n * 2 * (2 + hc) * hc * 4, "GB/s", "hc_split_sinkhorn HBM GB/s"
        bound, peak = "hbm", peaks["hbm_gbs"]
        cfg = f"hc_split_sinkhorn mixes [1, {n}, {(2 + hc) * hc}] fp32, hc={hc}, 20 iterations"
        h2d, d2h = n * (2 + hc) * hc * 4, n * (2 + hc) * hc * 4
    elif args.workload == "sparse_attn":
        b, sq, h, d, nk, k = 1, 4096, 16, 576, 1024, 512
        q = torch.randn(b, sq, h, d, generator=g, device=dev).to(torch.bfloat16)
        kv = torch.randn(b, nk, d, generator=g, device=dev).to(torch.bfloat16)
        sink = torch.randn(h, generator=g, device=dev)
        idx = torch.randint(0, nk, (b, sq, k), generator=g, device=dev)
        call = lambda: kern.sparse_attn(q, kv, sink, idx, d ** -0.5)             # noqa: E731
        work, unit, metric = 4.0 * b * sq * h * k * d, "TFLOP/s", "sparse_attn TFLOP/s"
        bound, peak = "tensor", peaks["bf16_tflops"]
        cfg = f"sparse_attn q [{b}, {sq}, {h}, {d}] bf16, kv [{b}, {nk}, {d}], {k} keys per query"
        h2d, d2h = q.numel() * 2 + idx.numel() * 8, q.numel() * 2
    else:
        sq, h, d, t, k = 4096, 64, 128, 1024, 512
        q = torch.randn(1, sq, h, d, generator=g, device=dev)
        kv = torch.randn(1, t, d, generator=g, device=dev)
        w = torch.randn(1, sq, h, generator=g, device=dev)
        call = lambda: kern.indexer_topk(q, kv, w, k, 4, 0, 0)                   # noqa: E731
        work, unit, metric = 2.0 * sq * h * d * t, "TFLOP/s", "Indexer score+top-k TFLOP/s"
        bound, peak = "tensor", peaks["bf16_tflops"]
        cfg = f"Indexer q [1, {sq}, {h}, {d}] fp32, kv [1, {t}, {d}], top-{k}, ratio 4, prefill"
        h2d, d2h = q.numel() * 4 + w.numel() * 4, sq * k * 8
    for _ in range(args.warmup):
        call()
    torch.cuda.synchronize()
    if dist is not None:
        dist.barrier()
    clocks = Clocks(torch.cuda.current_device())
    clocks.start()
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t0.record()
    for _ in range(args.steps):
        call()
    t1.record()
    torch.cuda.synchronize()
    clk = clocks.stop()
    ms = max_over_ranks(torch, dist, t0.elapsed_time(t1) / args.steps)
    scale = 1e9 if unit == "GB/s" else 1e12
    rate = work / (ms * 1e-3) / scale
    return {"metric": metric, "value": round(ws * rate, 3), "unit": unit, "n_gpus": ws, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(ms, 4), "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "fp32 arithmetic", "data": "synthetic (seeded)",
            "config": {"workload": cfg, "parallelism": f"replicas x{ws}" if ws > 1 else "none"},
            "roofline": {"bound": bound, "achieved": round(rate, 3), "peak": peak, "unit": unit,
                         "frac": round(rate / peak, 4), "traffic": None,
                         "peak_source": f"{'hbm_gbs' if bound == 'hbm' else 'bf16_tflops'} of {src} "
                                        "MEASURED_PEAKS.json"},
            "e2e": None, "io_bytes_per_step": {"h2d": h2d, "d2h": d2h}, "gpu_launches": args.steps, "clocks": clk}


def max_over_ranks(torch, dist, v):
    if dist is None:
        return v
    t = torch.tensor([v], device="cuda", dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


# ---------------------------------------------------------------------------
# CPU legs: the oracle port of the reference algorithm on the host cores
# ---------------------------------------------------------------------------

def cpu_threads():
    return len(os.sched_getaffinity(0))


def cpu_fp4_decode(M: int, N: int, K: int = 4096, steps: int = 3):
    """The oracle's fp4_gemm (the reference CPU path: LUT dequant of all of B ->
    bf16 -> matmul) on the decode shape; GB/s of the same bytes the GPU line
    counts."""
    from oracle import blockscaled as ob
    rng = np.random.default_rng(77)
    x = ob.f32_to_bf16(rng.standard_normal((M, K)).astype(np.float32))
    a, a_s = ob.act_quant(x, ob.DT_BF16, 128, None, ob.DT_F32)
    b = rng.integers(0, 256, size=(N, K // 2), dtype=np.uint8)
    b_s = (127 - rng.integers(0, 7, size=(N, K // 32))).astype(np.uint8)
    ob.fp4_gemm(a, a_s, b, b_s, ob.DT_F32, ob.DT_E8M0)
    times = []
    for _ in range(steps):
        t = time.perf_counter()
        ob.fp4_gemm(a, a_s, b, b_s, ob.DT_F32, ob.DT_E8M0)
        times.append(time.perf_counter() - t)
    s = min(times)
    byts = N * K // 2 + N * K // 32 + M * K + 4 * M * K // 128 + 2 * M * N
    return byts / s / 1e9, s


def zipf_bias(torch, E, seed):
    """Expert popularity skew of the long-prefill config: -1.2*ln(1 + rank of e)
    under a seeded permutation of the experts (a Zipf(1.2)-like stand-in)."""
    perm = torch.randperm(E, generator=torch.Generator().manual_seed(seed))
    return -1.2 * torch.log1p(perm.float())


def bench_moe_stack(args, torch, dist, ws, rank, dev):
    """Config-5 long-prefill stack: T=8192 tokens, 4 layers, each an fp8_gemm
    4096->4096 projection (1x128 activation, 128x128 weight scales) followed by
    the config-4 MoE (256 experts, top-8) under Zipf-skewed expert popularity.

    One GPU: the whole stack.  N GPUs: rank r owns tokens [r*T/N, (r+1)*T/N)
    (its projections run on its own tokens with a full copy of the small dense
    weights) and experts [r*E/N, (r+1)*E/N) of every layer; the MoE rows
    travel over NVLink peer memory.  Metric: token-layers per second
    (T x 4 / stack time), strong scaling.
    """
    import importlib
    pkg = importlib.import_module(PKG)
    moe = importlib.import_module(PKG + ".moe")
    T, H, I, E, k, L = args.tokens, 4096, 2048, args.experts, 8, 4
    if T % ws or E % ws:
        raise SystemExit("tokens and experts must split evenly over the ranks")
    El, tl = E // ws, T // ws
    g = torch.Generator(device=dev)
    g.manual_seed(5)
    x_all = torch.randn(T, H, generator=g, device=dev).to(torch.bfloat16)
    bias = zipf_bias(torch, E, 11).to(dev)
    logits = [(torch.randn(T, E, generator=g, device=dev) + bias)[rank * tl:(rank + 1) * tl].contiguous()
              for _ in range(L)]
    proj = []
    for _ in range(L):
        w = torch.randn(H, H, generator=g, device=dev) * 0.02
        wb = w.view(H // 128, 128, H // 128, 128)
        sc = wb.abs().amax(dim=(1, 3)).clamp(min=1e-4) / 448.0
        proj.append(((wb / sc[:, None, :, None]).clamp(-448, 448).to(torch.float8_e4m3fn).view(H, H), sc.contiguous()))
    g.manual_seed(2000 + rank)
    layers = []
    for _ in range(L):
        w13 = torch.randint(0, 256, (El, 2 * I, H // 2), generator=g, device=dev, dtype=torch.uint8)
        w13_s = 127 - torch.randint(0, 7, (El, 2 * I, H // 32), generator=g, device=dev, dtype=torch.uint8)
        w2 = torch.randint(0, 256, (El, H, I // 2), generator=g, device=dev, dtype=torch.uint8)
        w2_s = 127 - torch.randint(0, 7, (El, H, I // 32), generator=g, device=dev, dtype=torch.uint8)
        layers.append(moe.MoEWeights(w13, w13_s, w2, w2_s))
        del w13, w13_s, w2, w2_s
    x0 = x_all[rank * tl:(rank + 1) * tl].contiguous()
    del x_all
    if ws > 1:
        ep = importlib.import_module(PKG + ".ep")
        eps = [ep.EPMoE(W, E, k, max_tokens=tl, transport=args.ep_transport) for W in layers]
    outs = [torch.empty(tl, H, dtype=torch.bfloat16, device=dev) for _ in range(2)]

    def stack(x):
        for l in range(L):
            a, a_s = pkg.act_quant(x, 128)
            h = pkg.fp8_gemm(a, a_s, proj[l][0], proj[l][1])
            out = outs[l & 1]
            if ws > 1:
                eps[l].forward(h, logits[l], out=out)
            else:
                moe.moe_forward(h, logits[l], layers[l], k, out=out)
            x = out
        return x

    for _ in range(args.warmup):
        stack(x0)
    torch.cuda.synchronize()
    if dist is not None:
        dist.barrier()
    clocks = Clocks(torch.cuda.current_device())
    clocks.start()
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t0.record()
    for _ in range(args.steps):
        stack(x0)
    t1.record()
    torch.cuda.synchronize()
    if dist is not None:
        dist.barrier()
    clk = clocks.stop()
    ms = max_over_ranks(torch, dist, t0.elapsed_time(t1) / args.steps)
    # load balance: rows each rank's experts receive per layer, max / mean over
    # the owners; routing is a pure function of the logits
    per_owner = torch.zeros(L, ws, dtype=torch.float64, device=dev)
    for l in range(L):
        owner = torch.topk(logits[l], k, dim=1).indices // El
        per_owner[l] = torch.bincount(owner.flatten(), minlength=ws).double()
    if dist is not None:
        dist.all_reduce(per_owner)
    imbalance = [round(float(r.max() / r.mean()), 3) for r in per_owner]
    # end to end: pinned host tokens in, the last layer's output out
    x_host = x0.cpu().pin_memory()
    o_host = torch.empty(tl, H, dtype=torch.bfloat16).pin_memory()
    x_dev = torch.empty_like(x0)

    def e2e_step():
        x_dev.copy_(x_host, non_blocking=True)
        o_host.copy_(stack(x_dev), non_blocking=True)

    e2e_step()
    torch.cuda.synchronize()
    if dist is not None:
        dist.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(args.steps):
        e2e_step()
    e1.record()
    torch.cuda.synchronize()
    e2e_ms = max_over_ranks(torch, dist, e0.elapsed_time(e1) / args.steps)
    if ws > 1:
        pkg._lib.device_error_check()
        for m in eps:
            m.close()
    peaks, src = load_peaks()
    flops = L * (2.0 * T * H * H + T * k * (2.0 * H * 2 * I + 2.0 * I * H))
    achieved = flops / ws / (ms * 1e-3) / 1e12
    peak = 2.0 * peaks["bf16_tflops"]
    return {"metric": "MoE stack token-layers/s (long prefill)", "value": round(T * L / (ms * 1e-3), 1),
            "unit": "token-layers/s", "n_gpus": ws, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": round(ms, 3), "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
            "dtype": "e4m3 x e2m1 (MoE), e4m3 (projections)", "data": "synthetic (Zipf-skewed gate logits)",
            "config": {"workload": f"{L} layers x (fp8_gemm {H}->{H} + MoE E={E} top-{k} I={I}), T={T}",
                       "parallelism": f"ep{ws} (+ token-parallel projections)" if ws > 1 else "none",
                       "exchange": ("NVLink peer memory" if args.ep_transport == "peer" else "NCCL all-to-all")
                       if ws > 1 else None,
                       "load_imbalance_max_over_mean": imbalance},
            "e2e": {"value": round(T * L / (e2e_ms * 1e-3), 1), "unit": "token-layers/s",
                    "h2d_bytes_per_step": T * H * 2, "d2h_bytes_per_step": T * H * 2, "ms_per_step": round(e2e_ms, 3)},
            "roofline": {"bound": "tensor", "achieved": round(achieved, 1), "peak": round(peak, 1), "unit": "TFLOP/s",
                         "frac": round(achieved / peak, 3), "traffic": None,
                         "note": "per-GPU FLOP of the stack / stack time vs the dense e4m3 rate"},
            "gpu_launches": args.steps * L * (2 + (3 if ws == 1 or args.ep_transport == "peer" else 9)),
            "clocks": clk}


def reference_moe(args, ws):
    """The MoE workload on the host CPU: each step runs a bounded sample of the
    layer (8 of the active experts, all their routed tokens) through the
    torch restatement of the reference's CPU ops, and the step's layer time
    is that sample's time scaled to every active expert."""
    import torch
    torch.set_num_threads(cpu_threads())
    T, H, I, E, k = args.tokens, 4096, 2048, args.experts, 8
    g = torch.Generator().manual_seed(4)
    x = torch.randn(T, H, generator=g).to(torch.bfloat16)
    logits = torch.randn(T, E, generator=g)
    cache = {}

    def fetch(e):
        if e not in cache:
            ge = torch.Generator().manual_seed(50_000 + e)
            cache[e] = (torch.randint(0, 256, (2 * I, H // 2), generator=ge, dtype=torch.uint8),
                        (127 - torch.randint(0, 7, (2 * I, H // 32), generator=ge, dtype=torch.uint8)).view(
                            torch.float8_e8m0fnu),
                        torch.randint(0, 256, (H, I // 2), generator=ge, dtype=torch.uint8),
                        (127 - torch.randint(0, 7, (H, I // 32), generator=ge, dtype=torch.uint8)).view(
                            torch.float8_e8m0fnu))
        return cache[e]

    per_step = 8
    for w in range(args.warmup):
        cpu_moe_sample(torch, x, logits, fetch, E, k, budget_s=0.0, min_experts=per_step, max_experts=per_step,
                       seed=w)
    times = []
    for i in range(args.steps):
        layer_s, _, n_act = cpu_moe_sample(torch, x, logits, fetch, E, k, budget_s=0.0, min_experts=per_step,
                                           max_experts=per_step, seed=100 + i)
        times.append(layer_s)
    layer_s = statistics.mean(times)
    v = T / layer_s
    return {"impl": "reference", "metric": "MoE-layer tokens/s", "value": round(v, 3), "unit": "tokens/s",
            "n_gpus": ws, "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(layer_s * 1e3, 1),
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "e4m3 x e2m1",
            "data": "synthetic (seeded N(0,1) tokens and gate logits, uniform e2m1 codes, ue8m0 exponents in [-6,0])",
            "config": {"workload": f"MoE layer T={T} H={H} I={I} E={E} top-{k} (grouped FP8xFP4 GEMMs)",
                       "parallelism": "host CPU"},
            "cpu_baseline": {"value": round(v, 3), "unit": "tokens/s", "cores": cpu_threads(), "kind": "port",
                             "sample": f"per step {per_step} of the {n_act} active experts with all their routed "
                                       "tokens (act_quant + LUT-dequant bf16 fp4_gemm x3 per expert, torch on the "
                                       "host cores); layer time scaled to all active experts"},
            "e2e": {"value": round(v, 3), "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}


def reference_fp8(args, ws):
    """The dense fp8_gemm (M=N=K=4096) through the torch restatement of the
    reference's CPU branch: dequantise both operands, round to bf16, one
    bf16 torch.mm."""
    import torch
    from oracle import torch_cpu as tc
    torch.set_num_threads(cpu_threads())
    sys.path.insert(0, os.path.join(ROOT, "tests", "golden"))
    import cases
    c = cases.cfg2_fp8(M=4096)
    a = torch.from_numpy(c["a"]).view(torch.float8_e4m3fn)
    a_s = torch.from_numpy(c["a_s"])
    b = torch.from_numpy(c["b"]).view(torch.float8_e4m3fn)
    b_s = torch.from_numpy(c["b_s"])
    for _ in range(args.warmup):
        tc.fp8_gemm(a, a_s, b, b_s)
    times = []
    for _ in range(args.steps):
        t = time.perf_counter()
        tc.fp8_gemm(a, a_s, b, b_s)
        times.append(time.perf_counter() - t)
    s = statistics.mean(times)
    v = 2.0 * 4096 ** 3 / s / 1e12
    return {"impl": "reference",
            "metric": "block-scaled FP8 GEMM TFLOP/s (dense fp8_gemm, 1x128 act + 128x128 weight fp32 scales)",
            "value": round(v, 4), "unit": "TFLOP/s", "n_gpus": ws, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": round(s * 1e3, 2), "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": "e4m3", "data": "synthetic",
            "config": {"workload": "fp8_gemm M=N=K=4096 on the host CPU", "M": 4096, "N": 4096, "K": 4096},
            "cpu_baseline": {"value": round(v, 4), "unit": "TFLOP/s", "cores": cpu_threads(), "kind": "port",
                             "sample": "one full 4096^3 fp8_gemm per step: dequantise -> bf16 -> torch.mm (torch)"},
            "e2e": {"value": round(v, 4), "unit": "TFLOP/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--workload", choices=["moe", "fp8_prefill", "fp4_decode", "moe_stack", "act_quant",
                                           "fp4_act_quant", "hc_sinkhorn", "sparse_attn", "indexer"], default="moe")
    ap.add_argument("--tokens", type=int, default=None,
                    help="moe: 1024, moe_stack: 8192, act_quant / fp4_act_quant: 16384 rows")
    ap.add_argument("--experts", type=int, default=256)
    ap.add_argument("--m", type=int, default=16)
    ap.add_argument("--n", type=int, default=4096)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--ep-transport", choices=["peer", "nccl"], default="peer",
                    help="moe at N>1: rows exchanged over NVLink peer memory, or by NCCL all-to-all")
    ap.add_argument("--tp-gather", choices=["fused", "nccl"], default="fused",
                    help="fp8_prefill at N>1: all-gather fused into the GEMM epilogue, or NCCL after it")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)
    if args.tokens is None:
        args.tokens = {"moe_stack": 8192, "act_quant": 16384, "fp4_act_quant": 16384}.get(args.workload, 1024)
    ws, rank, local = dist_env()

    if args.impl == "reference":
        # the reference's CPU arithmetic on the host cores, rank 0 only; other ranks exit
        if rank != 0:
            return
        if args.workload == "moe":
            print(json.dumps(reference_moe(args, ws)), flush=True)
        else:
            print(json.dumps(reference_fp8(args, ws)), flush=True)
        return

    import torch
    dist = None
    if ws > 1:
        import datetime
        import torch.distributed as dist_mod
        torch.cuda.set_device(local)
        dist_mod.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                    device_id=torch.device("cuda", local))
        dist = dist_mod
    else:
        torch.cuda.set_device(0)
    dev = torch.device("cuda", torch.cuda.current_device())
    importlib = __import__("importlib")
    importlib.import_module(PKG)._lib.load()

    if args.workload == "fp8_prefill":
        line = bench_fp8_prefill(args, torch, dist, ws, rank, dev)
    elif args.workload == "moe":
        line = bench_moe(args, torch, dist, ws, rank, dev)
    elif args.workload == "moe_stack":
        line = bench_moe_stack(args, torch, dist, ws, rank, dev)
    elif args.workload in ("act_quant", "fp4_act_quant"):
        line = bench_quant(args, torch, dist, ws, rank, dev)
    elif args.workload in ("hc_sinkhorn", "sparse_attn", "indexer"):
        line = bench_attn_side(args, torch, dist, ws, rank, dev)
    else:
        line = bench_fp4_decode(args, torch, dist, ws, rank, dev)

    if rank == 0 and ws == 1 and args.workload == "fp4_decode" and not args.no_cpu_baseline:
        torch.set_num_threads(cpu_threads())
        v, s = cpu_fp4_decode(args.m, args.n)
        line["cpu_baseline"] = {"value": round(v, 3), "unit": "GB/s", "cores": cpu_threads(), "kind": "port",
                                "sample": f"fp4_gemm M={args.m} N={args.n} K=4096 on the host ({s * 1e3:.1f} ms per "
                                          "call): LUT dequant of all of B -> bf16 -> fp32 matmul (numpy), best of 3"}
    if rank == 0 and ws == 1 and args.workload == "fp8_prefill" and not args.no_cpu_baseline:
        r = reference_fp8(argparse.Namespace(steps=2, warmup=1), 1)
        line["cpu_baseline"] = r["cpu_baseline"]
    pkg = importlib.import_module(PKG)
    pkg._lib.device_error_check()
    if rank == 0:
        print(json.dumps(line), flush=True)
    if dist is not None:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()

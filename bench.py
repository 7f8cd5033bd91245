#!/usr/bin/env python3
"""W4A16 decode benchmark on B200 (one JSON line on rank 0).

Workload (config "decode", the headline): Llama-3-8B decode at M = 1.  One
step = one token through the 7 projections of all 32 layers
(q 4096x4096, k/v 4096x1024, o 4096x4096, gate/up 4096x14336, down 14336x4096),
signed INT4 weights (full-range random words), group-128 fp16 scales
|N(0,0.02)|+1e-3, fp16 activations N(0,1).  The layers' weights rotate through
a pool of distinct buffers at least 4x the L2 size, so every launch streams
its weights from HBM (inputs larger than L2; no flush needed).

value = algorithmic bytes / second over all ranks, algorithmic bytes per
projection = K*N/2 + (K/128)*N*2 + M*K*2 + M*N*2.

With --gpus N > 1 (torchrun, one process per GPU) every projection is
column-sharded N ways and the outputs are gathered by the decode kernel itself
(peer stores over NVLink, t4_cuda_b200.shard.P2PGatherGroup; --nccl-gather
uses NCCL all-gather instead): the same token, so "scaling" is "strong".

The line also carries "decode_batch" (one GPU): the four projection shapes
at M in {1, 4, 8, 16}, one launch at a time; "gemm_sweep" (one GPU): the
same shapes at M in {512, 2048, 4096} on the tcgen05 GEMM; and
"sharded_70b": Llama-3-70B layer projections column-sharded over the same
N GPUs at M in {1, 16, 256, 4096} (see sharded_70b); "fp8_gemm" (one GPU): the
FP8-E4M3 weight GEMM at the four shapes, M = 1 and M = 4096.

--impl reference times the reference's CPU dequant + matmul path
(tests/test_fused_gemm_correctness.py:22-36, restated in oracle/cpu_path.py)
on the host cores, one projection per step.
"""

import argparse
import json
import math
import os
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

import torch  # noqa: E402

METRIC = "W4A16 GEMV HBM GB/s (% of 8 TB/s) at M=1; GEMM TFLOPS at M=4096"
WORKLOAD = "decode: Llama-3-8B token, 32 layers x 7 projections, M=1, s4 g128"
GROUP = 128
N_LAYERS = 32
PROJ = [("q", 4096, 4096), ("k", 4096, 1024), ("v", 4096, 1024), ("o", 4096, 4096),
        ("gate", 4096, 14336), ("up", 4096, 14336), ("down", 14336, 4096)]
# projections that read the same activation share one all-gather
GATHERS = [("x", ["q", "k", "v"]), ("attn", ["o"]), ("x", ["gate", "up"]), ("h", ["down"])]
ACT_K = {"x": 4096, "attn": 4096, "h": 14336}
# Llama-3-70B layer: hidden 8192, intermediate 28672, 64 query / 8 KV heads of 128
PROJ_70B = [("q", 8192, 8192), ("k", 8192, 1024), ("v", 8192, 1024), ("o", 8192, 8192),
            ("gate", 8192, 28672), ("up", 8192, 28672), ("down", 28672, 8192)]
ACT_K_70B = {"x": 8192, "attn": 8192, "h": 28672}
M_70B = (1, 16, 256, 4096)


def alg_bytes(M, K, N, group=GROUP):
    return K * N // 2 + (K // group) * N * 2 + M * K * 2 + M * N * 2


def load_peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            d = json.load(f)
        return {"hbm_gbs": d["hbm_gbs"], "bf16_tflops": d["bf16_tflops"], "source": "measured"}
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "source": "fallback"}


def load_gemm_traffic():
    """DRAM bytes of one prefill GEMM launch (M = K = N = 4096) from the committed
    ncu summary (profiles/gemm_w4_tc_pair_4096.md, line
    'traffic_bytes_per_launch <name> <bytes>')."""
    p = os.path.join(ROOT, "profiles", "gemm_w4_tc_pair_4096.md")
    if os.path.exists(p):
        for line in open(p):
            parts = line.strip().strip("`").split()
            if len(parts) == 3 and parts[0] == "traffic_bytes_per_launch":
                return float(parts[2])
    return None


def load_traffic():
    """DRAM bytes of one decode step from the committed ncu summary
    (profiles/gemv_w4_decode.md, line 'traffic_bytes_per_step <name> <bytes>');
    the roofline reports it per launch (divided by the launches of a step)."""
    p = os.path.join(ROOT, "profiles", "gemv_w4_decode.md")
    out = {}
    if os.path.exists(p):
        for line in open(p):
            parts = line.strip().strip("`").split()
            if len(parts) == 3 and parts[0] == "traffic_bytes_per_step":
                out[parts[1]] = float(parts[2])
    return out


class ClockSampler:
    """Polls NVML (SM clock, throttle reasons) on a thread while the timed
    region runs; the region is too short for nvidia-smi's 200 ms cadence."""

    BITS = {0x4: "sw_power_cap", 0x8: "hw_slowdown", 0x20: "sw_thermal_slowdown", 0x40: "hw_thermal_slowdown",
            0x80: "hw_power_brake_slowdown", 0x1: "gpu_idle", 0x2: "applications_clocks_setting"}

    def __init__(self, device_index):
        self.samples, self.reasons, self.max_mhz, self.ok = [], 0, None, False
        self._stop = threading.Event()
        try:
            import pynvml
            pynvml.nvmlInit()
            uuid = torch.cuda.get_device_properties(device_index).uuid
            self.h = None
            for i in range(pynvml.nvmlDeviceGetCount()):
                hh = pynvml.nvmlDeviceGetHandleByIndex(i)
                if str(uuid).replace("GPU-", "") in str(pynvml.nvmlDeviceGetUUID(hh)):
                    self.h = hh
            if self.h is None:
                self.h = pynvml.nvmlDeviceGetHandleByIndex(device_index)
            self.nv = pynvml
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self.h, pynvml.NVML_CLOCK_SM)
            self._reasons_fn = getattr(pynvml, "nvmlDeviceGetCurrentClocksEventReasons", None) or \
                pynvml.nvmlDeviceGetCurrentClocksThrottleReasons
            self.ok = True
        except Exception:
            self.ok = False

    def _run(self):
        nv = self.nv
        while not self._stop.is_set():
            try:
                self.samples.append(nv.nvmlDeviceGetClockInfo(self.h, nv.NVML_CLOCK_SM))
                self.reasons |= self._reasons_fn(self.h)
            except Exception:
                pass
            time.sleep(0.002)

    def __enter__(self):
        if self.ok:
            self.t = threading.Thread(target=self._run, daemon=True)
            self.t.start()
        return self

    def __exit__(self, *exc):
        if self.ok:
            self._stop.set()
            self.t.join()

    def summary(self):
        if not self.ok or not self.samples:
            return None
        s = sorted(self.samples)
        return {"sm_mhz": s[len(s) // 2], "sm_max_mhz": self.max_mhz, "samples": len(s),
                "reasons": [n for b, n in self.BITS.items() if self.reasons & b and n != "gpu_idle"]}


# ----------------------------------------------------------------------------- our arm
def make_layer(rank, world, M, dev, gen):
    layer = {}
    for name, K, N in PROJ:
        n = N // world
        W = torch.randint(-2 ** 31, 2 ** 31 - 1, (K // 8, n), dtype=torch.int32, device=dev, generator=gen)
        S = (torch.randn((K // GROUP, n), device=dev, generator=gen).abs() * 0.02 + 1e-3).half()
        layer[name] = (W, S)
    return layer


def prefill_gemm(dev, M=4096, steps=5, warmup=3):
    """Second half of the metric: the tcgen05 prefill GEMM at M = 4096 over the
    seven projections of one Llama-3-8B layer (one step = all seven), timed
    with CUDA events on the current stream; TFLOP/s = 2 M K N / time."""
    from t4_cuda_b200 import ops
    gen = torch.Generator(device=dev).manual_seed(11)
    layer = {}
    for name, K, N in PROJ:
        W = torch.randint(-2 ** 31, 2 ** 31 - 1, (K // 8, N), dtype=torch.int32, device=dev, generator=gen)
        S = (torch.randn((K // GROUP, N), device=dev, generator=gen).abs() * 0.02 + 1e-3).half()
        layer[name] = (W, S)
    acts = {k: torch.randn((M, kk), device=dev, generator=gen).half() for k, kk in (("x", 4096), ("h", 14336))}

    def step():
        for name, K, N in PROJ:
            ops.fused_w4a16_gemm_s4(acts["h"] if name == "down" else acts["x"], layer[name][0], layer[name][1], None)

    for _ in range(warmup):
        step()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(steps):
        step()
    e1.record()
    e1.synchronize()
    ms = e0.elapsed_time(e1) / steps
    flops = sum(2.0 * M * K * N for _, K, N in PROJ)
    per_shape = {}
    for name, K, N in PROJ:
        a = acts["h"] if name == "down" else acts["x"]
        f0, f1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        f0.record()
        for _ in range(steps):
            ops.fused_w4a16_gemm_s4(a, layer[name][0], layer[name][1], None)
        f1.record()
        f1.synchronize()
        us = f0.elapsed_time(f1) * 1e3 / steps
        per_shape[f"{name}_{K}x{N}"] = {"us": round(us, 2), "TFLOP/s": round(2.0 * M * K * N / us / 1e6, 1)}
    tflops = flops / (ms * 1e-3) / 1e12
    return {"metric": "GEMM TFLOPS at M=4096", "value": round(tflops, 1), "unit": "TFLOP/s",
            "ms_per_step": round(ms, 4), "steps": steps, "warmup": warmup,
            "config": {"workload": "prefill: one Llama-3-8B layer, 7 projections at M=4096, s4 g128", "M": M},
            "kernel": "gemm_w4_tc_kernel (tcgen05.mma kind::f16, 128x256 tiles, TMEM accumulator)",
            "per_shape": per_shape}


def _graph_us(dev, calls, reps=20):
    """Average device time of one call in a CUDA graph of `calls` (a list of
    zero-argument callables, replayed `reps` times after warm-up)."""
    s = torch.cuda.Stream(dev)
    s.wait_stream(torch.cuda.current_stream(dev))
    with torch.cuda.stream(s):
        for f in calls:
            f()
    torch.cuda.current_stream(dev).wait_stream(s)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        for f in calls:
            f()
    for _ in range(3):
        g.replay()
    torch.cuda.synchronize(dev)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(reps):
        g.replay()
    e1.record()
    e1.synchronize()
    us = e0.elapsed_time(e1) * 1e3 / (reps * len(calls))
    del g
    return us


def int3_and_dequant(dev):
    """The other hot-path kernels at BASELINE-config shapes, device time per
    launch in a graph, inputs rotating through >= 4x L2:
      * H17 INT3 GEMV, M = 1, K in {4100, 14340} (4096 / 14336 padded to a
        multiple of 10), N in {4096, 14336}, group 128, no zero points; bytes
        = (K/10) N 4 + ceil(K/128) N 2 + 2 K + 2 N; and the same shapes at
        M = 512 and 4096 (the tcgen05 INT3 GEMM, TFLOP/s);
      * flat dequantization (s4 and s3 magic, fp8) of a 4096 x 14336 weight's
        words with per-word scales / zero points; bytes = read + written."""
    from t4_cuda_b200 import ops
    gen = torch.Generator(device=dev).manual_seed(9)
    l2 = torch.cuda.get_device_properties(dev).L2_cache_size
    out = {"int3_gemv": {}, "dequant": {}}
    for K, N in ((4100, 4096), (4100, 14336), (14340, 4096), (14340, 14336)):
        G = -(-K // 128)
        wbytes = (K // 10) * N * 4
        pool = max(4, (4 * l2) // wbytes + 1)
        Ws = [torch.randint(0, 2 ** 30, (K // 10, N), dtype=torch.int32, device=dev, generator=gen) for _ in range(pool)]
        S = (torch.randn((G, N), device=dev, generator=gen).abs() * 0.02).half()
        A = torch.randn((1, K), device=dev, generator=gen).half()
        Z = torch.empty(0, dtype=torch.float16, device=dev)
        us = _graph_us(dev, [lambda W=W: ops.fused_h17_gemv_s3(A, W, S, Z, group_size=128) for W in Ws])
        alg = wbytes + G * N * 2 + K * 2 + N * 2
        out["int3_gemv"][f"{K}x{N}"] = {"us": round(us, 3), "GB/s": round(alg / us / 1e3, 1)}
        del Ws
    # INT3 prefill (M > 16: the tcgen05 INT3 GEMM), TFLOP/s = 2 M K N / time,
    # a CUDA graph of 5 launches on one weight set (compute-bound)
    out["int3_gemm"] = {}
    for K, N in ((4100, 4096), (4100, 14336), (14340, 4096), (14340, 14336)):
        G = -(-K // 128)
        W = torch.randint(0, 2 ** 30, (K // 10, N), dtype=torch.int32, device=dev, generator=gen)
        S = (torch.randn((G, N), device=dev, generator=gen).abs() * 0.02 + 1e-3).half()
        Z = torch.empty(0, dtype=torch.float16, device=dev)
        row = {}
        for M in (512, 4096):
            A = torch.randn((M, K), device=dev, generator=gen).half()
            us = _graph_us(dev, [lambda: ops.fused_h17_gemv_s3(A, W, S, Z, group_size=128)] * 5, reps=4)
            row[f"M={M}"] = {"us": round(us, 2), "TFLOP/s": round(2.0 * M * K * N / us / 1e6, 1)}
        out["int3_gemm"][f"{K}x{N}"] = row
        del W
    words = 4096 // 8 * 14336
    for kind, per_word, fn in (("s4", 8, ops.dequantize_s4), ("s3", 10, ops.dequantize_s3), ("fp8", 4, None)):
        pool = max(4, (4 * l2) // (words * (4 + 4 + 2 * per_word)) + 1)
        Ws = [torch.randint(0, 2 ** 30, (words,), dtype=torch.int32, device=dev, generator=gen) for _ in range(pool)]
        S = (torch.randn(words, device=dev, generator=gen) * 0.02).half()
        Zp = torch.zeros(words, device=dev, dtype=torch.float16)
        if kind == "fp8":
            calls = [lambda W=W: ops.dequantize_fp8(W, S, mode="magic") for W in Ws]
            byts = words * (4 + 2 + 2 * per_word)
        else:
            calls = [lambda W=W, fn=fn: fn(W, S, Zp, mode="magic") for W in Ws]
            byts = words * (4 + 2 + 2 + 2 * per_word)
        us = _graph_us(dev, calls)
        out["dequant"][kind] = {"words": words, "us": round(us, 3), "GB/s": round(byts / us / 1e3, 1)}
        del Ws
    return out


def fp8_gemm(dev, reps=5):
    """The FP8-E4M3 weight GEMM (tcgen05, E4M3 -> fp16 dequant stage) at the
    Llama-3-8B projection shapes: M = 1 (decode; weights rotate through a pool
    >= 4x L2; GB/s of algorithmic bytes K N + (K/128) N 2 + 2 M K + 2 M N) and
    M = 4096 (prefill; TFLOP/s = 2 M K N), each a CUDA graph, CUDA events."""
    from t4_cuda_b200 import ops
    gen = torch.Generator(device=dev).manual_seed(13)
    l2 = torch.cuda.get_device_properties(dev).L2_cache_size
    out = {"decode_M=1": {}, "prefill_M=4096": {}}
    for K, N in ((4096, 4096), (4096, 1024), (4096, 14336), (14336, 4096)):
        pool = max(2, math.ceil(4 * l2 / (K * N)))
        # random E4M3 codes without the two NaN codes (0x7F, 0xFF)
        Ws = [(torch.randint(0, 2 ** 31 - 1, (K // 4, N), dtype=torch.int32, device=dev, generator=gen)
               & 0x7E7E7E7E) for _ in range(pool)]
        S = (torch.randn((K // GROUP, N), device=dev, generator=gen).abs() * 0.02 + 1e-3).half()
        A1 = torch.randn((1, K), device=dev, generator=gen).half()
        us = _graph_us(dev, [lambda W=W: ops.fused_w8a16_gemm_fp8(A1, W, S) for W in Ws])
        byts = K * N + (K // GROUP) * N * 2 + K * 2 + N * 2
        out["decode_M=1"][f"{K}x{N}"] = {"us": round(us, 3), "GB/s": round(byts / us / 1e3, 1)}
        A4 = torch.randn((4096, K), device=dev, generator=gen).half()
        us = _graph_us(dev, [lambda: ops.fused_w8a16_gemm_fp8(A4, Ws[0], S)] * reps, reps=4)
        out["prefill_M=4096"][f"{K}x{N}"] = {"us": round(us, 2), "TFLOP/s": round(2.0 * 4096 * K * N / us / 1e6, 1)}
        del Ws, A4
    return out


def gemm_sweep(dev, Ms=(512, 2048, 4096), reps=5):
    """The prefill configuration in full: the four Llama-3-8B projection shapes
    at M in {512, 2048, 4096} through the public op (tcgen05 GEMM), a CUDA
    graph of `reps` launches timed with CUDA events (short kernels launched
    one by one from Python would measure the host); TFLOP/s = 2 M K N / time."""
    from t4_cuda_b200 import ops
    gen = torch.Generator(device=dev).manual_seed(12)
    out = {}
    for K, N in ((4096, 4096), (4096, 1024), (4096, 14336), (14336, 4096)):
        W = torch.randint(-2 ** 31, 2 ** 31 - 1, (K // 8, N), dtype=torch.int32, device=dev, generator=gen)
        S = (torch.randn((K // GROUP, N), device=dev, generator=gen).abs() * 0.02 + 1e-3).half()
        row = {}
        for M in Ms:
            A = torch.randn((M, K), device=dev, generator=gen).half()
            us = _graph_us(dev, [lambda: ops.fused_w4a16_gemm_s4(A, W, S, None)] * reps, reps=4)
            row[f"M={M}"] = {"us": round(us, 2), "TFLOP/s": round(2.0 * M * K * N / us / 1e6, 1)}
        out[f"{K}x{N}"] = row
        del W
    return out


def decode_batch(dev, Ms=(1, 4, 8, 16), reps=10):
    """The decode skinny-GEMM configuration in full: the four Llama-3-8B
    projection shapes at M in {1, 4, 8, 16} through the public op, each a CUDA
    graph over a pool of distinct weights >= 4x L2, CUDA events; GB/s of
    algorithmic bytes per launch."""
    from t4_cuda_b200 import ops
    gen = torch.Generator(device=dev).manual_seed(1)
    l2 = torch.cuda.get_device_properties(dev).L2_cache_size
    out = {}
    for K, N in ((4096, 4096), (4096, 1024), (4096, 14336), (14336, 4096)):
        pool = max(2, math.ceil(4 * l2 / (K * N // 2)))
        Ws = [torch.randint(-2 ** 31, 2 ** 31 - 1, (K // 8, N), dtype=torch.int32, device=dev, generator=gen)
              for _ in range(pool)]
        S = (torch.randn((K // GROUP, N), device=dev, generator=gen).abs() * 0.02 + 1e-3).half()
        row = {}
        for M in Ms:
            A = torch.randn((M, K), device=dev, generator=gen).half()
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g):
                for W in Ws:
                    ops.fused_w4a16_gemm_s4(A, W, S, None)
            for _ in range(3):
                g.replay()
            torch.cuda.synchronize()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            for _ in range(reps):
                g.replay()
            e1.record()
            e1.synchronize()
            us = e0.elapsed_time(e1) * 1e3 / (reps * pool)
            row[f"M={M}"] = {"us": round(us, 3), "GB/s": round(alg_bytes(M, K, N) / us / 1e3, 1)}
            del g
        out[f"{K}x{N}"] = row
        del Ws
    return out


def _pct(sorted_vals, q):
    """q-th percentile (nearest rank) of an ascending list."""
    if not sorted_vals:
        return float("nan")
    k = max(0, min(len(sorted_vals) - 1, int(round(q / 100.0 * (len(sorted_vals) - 1)))))
    return sorted_vals[k]


def _max_over_ranks(dist, dev, ms):
    if dist is None:
        return ms
    t = torch.tensor([ms], device=dev, dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def sharded_70b(dev, world, rank, dist, l2, nccl_gather=False, steps=10, warmup=3):
    """Llama-3-70B layer projections column-sharded over the ranks at
    M in {1, 16, 256, 4096}; one step = the seven projections of a layer with
    every output gathered to every rank (max over ranks, CUDA events).
    M <= 16 rotates the layers' weights through a pool >= 4x L2 and reports
    HBM GB/s (algorithmic bytes of the full, unsharded layer); M >= 256 runs
    one layer and reports TFLOP/s (2 M K N).  Gathers: the decode kernel's own
    (P2PGatherGroup; the whole step one CUDA graph) where it takes the shape,
    else one NCCL all-gather per group from the host (ShardedGroup; the local
    projections of a group as one CUDA graph at M <= 16)."""
    from t4_cuda_b200 import ops
    from t4_cuda_b200.shard import P2PGatherGroup, ShardedGroup, ShardedLinear

    gen = torch.Generator(device=dev).manual_seed(4 + 1000 * rank)

    def make():
        L = {}
        for name, K, N in PROJ_70B:
            n = N // world
            W = torch.randint(-2 ** 31, 2 ** 31 - 1, (K // 8, n), dtype=torch.int32, device=dev, generator=gen)
            S = (torch.randn((K // GROUP, n), device=dev, generator=gen).abs() * 0.02 + 1e-3).half()
            L[name] = ShardedLinear(W, S, None, "s4")
        return L

    layer_bytes_local = sum(K * (N // world) // 2 + (K // GROUP) * (N // world) * 2 for _, K, N in PROJ_70B)
    pool = min(16, max(2, math.ceil(4 * l2 / layer_bytes_local)))
    layers = [make() for _ in range(pool)]

    def time_steps(run, reps):
        for _ in range(warmup):
            run()
        torch.cuda.synchronize()
        if dist is not None:
            dist.barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(reps):
            run()
        e1.record()
        e1.synchronize()
        return _max_over_ranks(dist, dev, e0.elapsed_time(e1) / reps)

    cases = {}
    for M in M_70B:
        acts = {a: torch.randn((M, k), device=dev, generator=gen).half() for a, k in ACT_K_70B.items()}
        decode = M <= 16
        use = layers if decode else layers[:1]
        mode, groups, graph = "single GPU", None, None
        if world > 1 and decode and not nccl_gather:
            built = []
            try:
                for L in use:
                    built.append([])
                    for _, names in GATHERS:
                        built[-1].append(P2PGatherGroup([L[n] for n in names], M))
                groups, mode = built, "fused"
            except RuntimeError:     # the same shapes on every rank: every rank falls back together
                for row in built:    # nothing was launched on these buffers
                    for grp in row:
                        grp.close()
        if world > 1 and groups is None:
            groups = [[ShardedGroup([L[n] for n in names]) for _, names in GATHERS] for L in use]
            mode = "nccl"
            if decode:
                for row in groups:
                    for g, (a, _) in enumerate(GATHERS):
                        row[g].capture_local(acts[a])

        def step():
            for li, L in enumerate(use):
                for g, (a, names) in enumerate(GATHERS):
                    if groups is None:
                        for n in names:
                            ops.fused_w4a16_gemm_s4(acts[a], L[n].W, L[n].S, None)
                    else:
                        groups[li][g](acts[a])

        run = step
        if decode and mode != "nccl":
            side = torch.cuda.Stream()
            side.wait_stream(torch.cuda.current_stream())
            with torch.cuda.stream(side):
                step()
                step()
            torch.cuda.current_stream().wait_stream(side)
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph):
                step()
            run = graph.replay
        ms = time_steps(run, steps if decode else 3)
        per_layer = ms / len(use)
        case = {"gather": mode, "ms_per_layer": round(per_layer, 4), "layers_per_step": len(use)}
        if decode:
            byts = sum(alg_bytes(M, K, N) for _, K, N in PROJ_70B)
            case["GB/s"] = round(byts / (per_layer * 1e-3) / 1e9, 1)
        else:
            flops = sum(2.0 * M * K * N for _, K, N in PROJ_70B)
            case["TFLOP/s"] = round(flops / (per_layer * 1e-3) / 1e12, 1)
        cases[f"M={M}"] = case
        del graph
        torch.cuda.synchronize()
        if dist is not None:
            dist.barrier()       # no rank still writes into another's gather buffers
        if groups is not None:
            for row in groups:
                for grp in row:
                    if isinstance(grp, P2PGatherGroup):
                        grp.close()
                    else:
                        grp.release_graph()
        torch.cuda.synchronize()
    return {"workload": "Llama-3-70B layer projections (q 8192x8192, k/v 8192x1024, o 8192x8192, "
                        "gate/up 8192x28672, down 28672x8192), s4 g128, column-sharded", "n_gpus": world,
            "distinct_weight_layers": pool, "weight_pool_bytes_per_gpu": pool * layer_bytes_local,
            "scaling": "strong", "cases": cases}


def run_ours(args):
    from t4_cuda_b200 import ops
    from t4_cuda_b200.shard import P2PGatherGroup, ShardedGroup, ShardedLinear

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    dist = None
    if world > 1:
        import datetime
        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)
    M = args.m
    gen = torch.Generator(device=dev).manual_seed(1234 + rank)

    layer_bytes_local = sum(K * (N // world) // 2 + (K // GROUP) * (N // world) * 2 for _, K, N in PROJ)
    l2 = torch.cuda.get_device_properties(dev).L2_cache_size
    pool = max(2, math.ceil(4 * l2 / layer_bytes_local))
    pool = min(pool, N_LAYERS)
    layers = [make_layer(rank, world, M, dev, gen) for _ in range(pool)]
    acts = {a: torch.randn((M, k), device=dev, generator=gen).half() for a, k in ACT_K.items()}
    # N > 1: the all-gather is fused into the decode GEMV (peer stores over
    # NVLink, no collective in the step); if that cannot be set up, each
    # group's local projections replay as a CUDA graph with NCCL all-gathers
    # between them from the host
    gather_mode = "single GPU"
    pg_layers = None
    if world > 1 and not args.nccl_gather:
        try:
            pg_layers = [{g: P2PGatherGroup([ShardedLinear(L[n][0], L[n][1], None, "s4") for n in names], M)
                          for g, (a, names) in enumerate(GATHERS)} for L in layers]
            gather_mode = "fused"
        except Exception as e:          # noqa: BLE001 -- reported in the JSON line
            print(f"rank {rank}: fused gather unavailable ({e}); NCCL all-gather", file=sys.stderr)
            pg_layers = None
    if pg_layers is None:
        pg_layers = [{g: ShardedGroup([ShardedLinear(L[n][0], L[n][1], None, "s4") for n in names])
                      for g, (a, names) in enumerate(GATHERS)} for L in layers]
        if world > 1:
            gather_mode = "nccl"

    def token(act):
        outs = []
        for li in range(N_LAYERS):
            groups = pg_layers[li % pool]
            for g, (a, names) in enumerate(GATHERS):
                outs.extend(groups[g](act[a]))
        return outs

    step_bytes = N_LAYERS * sum(alg_bytes(M, K, N) for _, K, N in PROJ)
    # one launch per projection, or one per group where ShardedGroup makes a
    # grouped call that the decode kernel takes as one launch
    def group_launches(grp, act, names):
        if getattr(grp, "_grouped", None) is None:
            return len(names)
        Ns = [N // world for n, _, N in PROJ if n in names]
        return 1 if ops.grouped_plan(Ns, M, ACT_K[act], GROUP) is not None else len(names)
    launches_per_step = N_LAYERS * sum(group_launches(pg_layers[0][g], a, names)
                                       for g, (a, names) in enumerate(GATHERS))

    use_graph = gather_mode in ("single GPU", "fused")
    if use_graph:
        s = torch.cuda.Stream()
        s.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s):
            for _ in range(2):
                token(acts)
        torch.cuda.current_stream().wait_stream(s)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            token(acts)
        run_step = graph.replay
    else:
        # NCCL path: each rank's local projections of a gather group replay as
        # one CUDA graph; the all-gathers run between them from the host
        for groups in pg_layers:
            for g, (a, names) in enumerate(GATHERS):
                groups[g].capture_local(acts[a])

        def run_step():
            token(acts)

    def barrier_sync():
        torch.cuda.synchronize()
        if dist is not None:
            dist.barrier()
        torch.cuda.synchronize()

    for _ in range(args.warmup):
        run_step()
    # one event between consecutive steps: the whole region and every step
    evs = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps + 1)]
    # NVML set-up and the sampling thread start before the barrier: their
    # time differs by rank and would otherwise skew the ranks' starts
    clk = ClockSampler(local)
    with clk:
        barrier_sync()
        evs[0].record()
        for i in range(args.steps):
            run_step()
            evs[i + 1].record()
        evs[-1].synchronize()
    barrier_sync()
    ms = evs[0].elapsed_time(evs[-1])
    step_ms = sorted(evs[i].elapsed_time(evs[i + 1]) for i in range(args.steps))
    if dist is not None:
        t = torch.tensor([ms], device=dev, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    ms_per_step = ms / args.steps
    value = step_bytes * args.steps / (ms * 1e-3) / 1e9

    # ---- the same step through the reference's op surface: one
    # fused_w4a16_gemm_s4 call per projection (one GPU, a CUDA graph)
    per_proj = None
    if world == 1:
        def token_single(act):
            outs = []
            for li in range(N_LAYERS):
                groups = pg_layers[li % pool]
                for g, (a, names) in enumerate(GATHERS):
                    outs.extend(lin.local(act[a]) for lin in groups[g].linears)
            return outs
        g1 = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g1):
            token_single(acts)
        for _ in range(args.warmup):
            g1.replay()
        torch.cuda.synchronize()
        p0, p1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        p0.record()
        for _ in range(args.steps):
            g1.replay()
        p1.record()
        p1.synchronize()
        pms = p0.elapsed_time(p1) / args.steps
        per_proj = {"ms_per_step": round(pms, 4), "GB/s": round(step_bytes / (pms * 1e-3) / 1e9, 1),
                    "launches_per_step": N_LAYERS * len(PROJ),
                    "api": "fused_w4a16_gemm_s4, one call per projection (the reference's op surface)"}
        del g1

    # ---- per-shape breakdown (one GPU): a graph of `pool` launches of one shape
    per_shape = {}
    if world == 1:
        for name, K, N in PROJ:
            a = acts["h"] if name == "down" else acts["x"]
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g):
                for L in layers:
                    ops.fused_w4a16_gemm_s4(a, L[name][0], L[name][1], None)
            for _ in range(3):
                g.replay()
            torch.cuda.synchronize()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            reps = 20
            e0.record()
            for _ in range(reps):
                g.replay()
            e1.record()
            e1.synchronize()
            us = e0.elapsed_time(e1) * 1e3 / (reps * len(layers))
            per_shape[f"{name}_{K}x{N}"] = {"us": round(us, 3), "GB/s": round(alg_bytes(M, K, N) / us / 1e3, 1)}
            del g
        # the grouped launches of the step: one call per group, a graph over the pool
        for a_name, names in GATHERS:
            grp0 = pg_layers[0][GATHERS.index((a_name, names))]
            if len(names) < 2 or getattr(grp0, "_grouped", None) is None:
                continue
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g):
                for li in range(pool):
                    pg_layers[li][GATHERS.index((a_name, names))](acts[a_name])
            for _ in range(3):
                g.replay()
            torch.cuda.synchronize()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            reps = 20
            e0.record()
            for _ in range(reps):
                g.replay()
            e1.record()
            e1.synchronize()
            us = e0.elapsed_time(e1) * 1e3 / (reps * pool)
            byts = sum(alg_bytes(M, K, N) for n, K, N in PROJ if n in names)
            per_shape["+".join(names) + "_grouped"] = {"us": round(us, 3), "GB/s": round(byts / us / 1e3, 1)}
            del g

    # ---- second half of the metric: prefill GEMM at M = 4096 (one GPU)
    gemm = None
    if world == 1 and not args.no_gemm:
        gemm = prefill_gemm(dev)
    others = None
    if world == 1 and not args.no_gemm:
        others = int3_and_dequant(dev)
    batch = decode_batch(dev) if world == 1 else None
    sweep = gemm_sweep(dev) if world == 1 and not args.no_gemm else None
    fp8 = fp8_gemm(dev) if world == 1 and not args.no_gemm else None

    # ---- end to end through the public API, host buffers, copies timed
    pin = {a: t.cpu().pin_memory() for a, t in acts.items()}
    dev_in = {a: torch.empty_like(t) for a, t in acts.items()}
    outs_eager = token(dev_in)
    n_out = sum(o.numel() for o in outs_eager)
    out_host = torch.empty(n_out, dtype=torch.float16).pin_memory()
    h2d = sum(t.numel() * 2 for t in acts.values())
    d2h = n_out * 2

    def e2e_step():
        for a in acts:
            dev_in[a].copy_(pin[a], non_blocking=True)
        outs = token(dev_in)
        # every output of the step comes back to the host: gathered into one
        # device buffer, then one copy (the same bytes as one copy per output)
        out_host.copy_(torch.cat([o.reshape(-1) for o in outs]), non_blocking=True)

    for _ in range(max(1, args.warmup)):
        e2e_step()
    barrier_sync()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(args.steps):
        e2e_step()
    e1.record()
    e1.synchronize()
    barrier_sync()
    e2e_ms = e0.elapsed_time(e1)
    if dist is not None:
        t = torch.tensor([e2e_ms], device=dev, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e2e_ms = float(t.item())
    e2e_value = step_bytes * args.steps / (e2e_ms * 1e-3) / 1e9
    e2e_lib = {"value": round(e2e_value, 1), "unit": "GB/s", "h2d_bytes_per_step": h2d,
               "d2h_bytes_per_step": d2h, "ms_per_step": round(e2e_ms / args.steps, 4),
               "api": {"single GPU": "t4_cuda_b200.shard.ShardedGroup: fused_w4a16_gemm_grouped for q/k/v and "
                                     "gate/up, fused_w4a16_gemm_s4 for o and down",
                       "fused": "t4_cuda_b200.shard.P2PGatherGroup (t4b_fused_w4a16_gemv_allgather_grouped)",
                       "nccl": "t4_cuda_b200.shard.ShardedGroup"}[gather_mode] + " (eager, pinned host buffers)"}

    # ---- the same end to end through the drop-in op, one call per projection
    e2e_single = None
    if world == 1:
        import t4_kernels

        def e2e_step_single():
            for a in acts:
                dev_in[a].copy_(pin[a], non_blocking=True)
            outs = []
            for li in range(N_LAYERS):
                L = layers[li % pool]
                for name, K, N in PROJ:
                    a = "h" if name == "down" else ("attn" if name == "o" else "x")
                    outs.append(t4_kernels.fused_w4a16_gemm_s4(dev_in[a], L[name][0], L[name][1], None))
            out_host.copy_(torch.cat([o.reshape(-1) for o in outs]), non_blocking=True)

        for _ in range(max(1, args.warmup)):
            e2e_step_single()
        torch.cuda.synchronize()
        e0.record()
        for _ in range(args.steps):
            e2e_step_single()
        e1.record()
        e1.synchronize()
        sms = e0.elapsed_time(e1) / args.steps
        e2e_single = {"value": round(step_bytes / (sms * 1e-3) / 1e9, 1), "unit": "GB/s", "ms_per_step": round(sms, 4),
                      "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                      "api": "t4_kernels.fused_w4a16_gemm_s4, one call per projection (eager, pinned host buffers)"}

    # a bounded wait that ran out or a launch that aborted sets the library's
    # device error word; the line reports it (max over ranks)
    dev_err = int(ops.device_error(dev))
    if dist is not None:
        t = torch.tensor([dev_err], device=dev, dtype=torch.int64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        dev_err = int(t.item())

    sh70 = None
    if not args.no_70b:
        sh70 = sharded_70b(dev, world, rank, dist, l2, nccl_gather=args.nccl_gather)

    if use_graph:
        del graph
    torch.cuda.synchronize()
    if dist is not None:
        dist.barrier()          # no rank still writes into another's gather buffers
    for groups in pg_layers:
        for grp in groups.values():
            if isinstance(grp, P2PGatherGroup):
                grp.close()
            else:
                grp.release_graph()
    torch.cuda.synchronize()
    if dist is not None:
        dist.barrier()
        dist.destroy_process_group()
    if rank != 0:
        return

    peaks = load_peaks()
    traffic = load_traffic()
    achieved = step_bytes / (ms_per_step * 1e-3) / 1e9 if world == 1 else None
    roof = None
    if world == 1:
        tr = traffic.get("decode_step")
        roof = {"bound": "hbm", "kernel": "gemv_w4_decode_kernel", "achieved": round(achieved, 1),
                "peak": peaks["hbm_gbs"], "unit": "GB/s", "frac": round(achieved / peaks["hbm_gbs"], 4),
                "peak_source": f"{peaks['source']} (MEASURED_PEAKS.json hbm_gbs)" if peaks["source"] == "measured"
                else "fallback 6650 GB/s",
                "traffic": (tr / launches_per_step) if tr else None,
                "algorithmic_bytes_per_launch": step_bytes / launches_per_step,
                "note": "timed region holds only gemv_w4_decode_kernel launches; duration per launch = region / launches"}
    line = {
        "metric": METRIC, "value": round(value, 1), "unit": "GB/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(ms_per_step, 4),
        "step_ms_rank0": {"median": round(_pct(step_ms, 50), 4), "p5": round(_pct(step_ms, 5), 4),
                          "p95": round(_pct(step_ms, 95), 4)},
        "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "f16 (int4 weights, fp32 accumulate)",
        "data": "synthetic",
        "config": {"workload": WORKLOAD,
                   "M": M, "group": GROUP, "layers_per_step": N_LAYERS, "distinct_weight_layers": pool,
                   "weight_pool_bytes": pool * layer_bytes_local, "l2_bytes": l2,
                   "l2_policy": "weights rotate through a pool >= 4x L2 (inputs larger than L2)",
                   "parallelism": {"single GPU": "single GPU",
                                   "fused": f"column-shard x{world}, all-gather fused into the decode GEMV "
                                            "(epoch-tagged column pairs stored into peer memory over NVLink; "
                                            "whole step one CUDA graph)",
                                   "nccl": f"column-shard x{world} + NCCL all-gather (local projections of each "
                                           "gather group replayed as a CUDA graph, all-gathers from the host)"}[gather_mode],
                   "frac_of_8TBs": round(value / 8000.0, 4)},
        "gpu_launches": launches_per_step * args.steps,
        "device_error": dev_err,
        # one GPU: e2e through the reference's op surface (t4_kernels, one
        # call per projection); the grouped calls' end to end beside it
        "e2e": e2e_single if e2e_single is not None else e2e_lib,
        "e2e_grouped": e2e_lib if e2e_single is not None else None,
        "per_shape": per_shape,
        "roofline": roof,
        "per_projection_step": per_proj,
        "clocks": clk.summary(),
    }
    if gemm is not None:
        pk = peaks["bf16_tflops"]
        gemm["roofline"] = {"bound": "tensor", "achieved": gemm["value"], "peak": pk, "unit": "TFLOP/s",
                            "frac": round(gemm["value"] / pk, 4),
                            "peak_source": "measured (MEASURED_PEAKS.json bf16_tflops, burst)" if peaks["source"] == "measured"
                            else "fallback 1590 TFLOP/s", "traffic": load_gemm_traffic(),
                            "traffic_note": "DRAM bytes of one 4096 x 4096 x 4096 launch (ncu, "
                                            "profiles/gemm_w4_tc_pair_4096.md); the seven projections differ in shape",
                            "timing": "CUDA events around 5 eager steps on one fixed weight set (compute-bound)"}
        line["gemm"] = gemm
    if others is not None:
        line["other_kernels"] = others
    if batch is not None:
        line["decode_batch"] = batch
    if sweep is not None:
        line["gemm_sweep"] = sweep
    if fp8 is not None:
        line["fp8_gemm"] = fp8
    if sh70 is not None:
        line["sharded_70b"] = sh70
    if world == 1 and not args.no_cpu_baseline:
        line["cpu_baseline"] = cpu_baseline(budget_s=args.cpu_budget)
    print(json.dumps(line), flush=True)


# ----------------------------------------------------------------------------- CPU path
def cpu_projection(name, K, N, M, gen):
    A = torch.randn((M, K), generator=gen).half()
    W = torch.randint(-2 ** 31, 2 ** 31 - 1, (K // 8, N), dtype=torch.int32, generator=gen)
    S = (torch.randn((K // GROUP, N), generator=gen).abs() * 0.02 + 1e-3).half()
    return A, W, S


def cpu_baseline(budget_s=12.0, M=1):
    """The reference's CPU dequant + matmul (oracle/cpu_path.py) over the 7
    projections of a layer, layer after layer (the same weights; they are
    far larger than the CPU caches) until the time budget is spent."""
    from oracle import cpu_path
    torch.set_num_threads(os.cpu_count() or 1)
    gen = torch.Generator().manual_seed(7)
    inputs = [(K, N, cpu_projection(name, K, N, M, gen)) for name, K, N in PROJ]
    cpu_path.w4_gemm(*cpu_projection("warm", 512, 512, M, gen), None, True)
    nbytes, secs, layers = 0, 0.0, 0
    while secs < budget_s:
        for K, N, (A, W, S) in inputs:
            t0 = time.perf_counter()
            cpu_path.w4_gemm(A, W, S, None, True)
            secs += time.perf_counter() - t0
            nbytes += alg_bytes(M, K, N)
        layers += 1
    return {"value": round(nbytes / secs / 1e9, 3), "unit": "GB/s", "cores": torch.get_num_threads(),
            "kind": "port", "seconds": round(secs, 2),
            "sample": f"{layers} passes over the 7 Llama-3-8B layer projections q/k/v/o/gate/up/down at M={M} "
                      "(one pass = 1/32 of a step), torch CPU dequant (q*s -> fp16) + fp32 matmul as "
                      "tests/test_fused_gemm_correctness.py:22-36"}


def run_reference(args):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    from oracle import cpu_path
    torch.set_num_threads(os.cpu_count() or 1)
    gen = torch.Generator().manual_seed(7)
    M = args.m
    inputs = [cpu_projection(n, K, N, M, gen) for n, K, N in PROJ]
    for i in range(args.warmup):
        A, W, S = inputs[i % len(PROJ)]
        cpu_path.w4_gemm(A, W, S, None, True)
    nbytes, secs = 0, 0.0
    for i in range(args.steps):
        (name, K, N), (A, W, S) = PROJ[i % len(PROJ)], inputs[i % len(PROJ)]
        t0 = time.perf_counter()
        cpu_path.w4_gemm(A, W, S, None, True)
        secs += time.perf_counter() - t0
        nbytes += alg_bytes(M, K, N)
    value = nbytes / secs / 1e9
    line = {"impl": "reference", "metric": METRIC, "value": round(value, 3), "unit": "GB/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(secs * 1e3 / args.steps, 3),
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f32 (fp16 weights)",
            "data": "synthetic",
            "config": {"workload": WORKLOAD, "M": M, "group": GROUP, "layers_per_step": N_LAYERS,
                       "reference_step": "a bounded sample: one projection per step, rotating q,k,v,o,gate,up,down "
                                         "(GB/s of algorithmic bytes, the same unit as the full step)"},
            "cpu_baseline": {"value": round(value, 3), "unit": "GB/s", "cores": torch.get_num_threads(),
                             "kind": "port",
                             "sample": "one Llama-3-8B projection per step, rotating q,k,v,o,gate,up,down"},
            "e2e": {"value": round(value, 3), "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def run_case(spec, launches=6):
    """Profiling driver (no JSON line): a few launches of ONE kernel on one
    case, for ncu captures of a single kernel.  Weights rotate through a pool
    of >= 4x L2 (except gemm), so every launch reads them from HBM.
      decode:K:N:M   s4 group-128 GEMV / skinny GEMM (default dispatch)
      stream:K:N:M   the same through the split-tile stream kernel
      gemm:M:K:N     s4 group-128 prefill GEMM (tcgen05)
      int3:K:N       H17 INT3 GEMV, M = 1, group 128 (K a multiple of 10)
      int3gemm:M:K:N H17 INT3 prefill GEMM (tcgen05), group 128
      dequant:KIND:W flat dequant (KIND s4, s3 or fp8; magic mode) of W words
      grouped:K:N1+N2+..:M  one grouped decode call of projections N1, N2, .."""
    from t4_cuda_b200 import ops
    kind, *dims = spec.split(":")
    dev = torch.device("cuda", int(os.environ.get("LOCAL_RANK", "0")))
    torch.cuda.set_device(dev)
    gen = torch.Generator(device=dev).manual_seed(5)
    l2 = torch.cuda.get_device_properties(dev).L2_cache_size

    def pool_of(nbytes, make):
        return [make() for _ in range(max(4, (4 * l2) // nbytes + 1))]

    if kind in ("decode", "stream"):
        K, N, M = (int(x) for x in dims)
        Ws = pool_of(K * N // 2, lambda: torch.randint(-2 ** 31, 2 ** 31 - 1, (K // 8, N), dtype=torch.int32,
                                                         device=dev, generator=gen))
    elif kind == "gemm":
        M, K, N = (int(x) for x in dims)
        Ws = [torch.randint(-2 ** 31, 2 ** 31 - 1, (K // 8, N), dtype=torch.int32, device=dev, generator=gen)]
    elif kind == "int3":
        K, N = (int(x) for x in dims)
        Ws = pool_of((K // 10) * N * 4, lambda: torch.randint(0, 2 ** 30, (K // 10, N), dtype=torch.int32,
                                                                device=dev, generator=gen))
        S = (torch.randn((-(-K // 128), N), device=dev, generator=gen).abs() * 0.02).half()
        A = torch.randn((1, K), device=dev, generator=gen).half()
        Z = torch.empty(0, dtype=torch.float16, device=dev)
        for i in range(launches):
            C = ops.fused_h17_gemv_s3(A, Ws[i % len(Ws)], S, Z, group_size=128)
    elif kind == "int3gemm":
        M, K, N = (int(x) for x in dims)
        W = torch.randint(0, 2 ** 30, (K // 10, N), dtype=torch.int32, device=dev, generator=gen)
        S = (torch.randn((-(-K // 128), N), device=dev, generator=gen).abs() * 0.02 + 1e-3).half()
        A = torch.randn((M, K), device=dev, generator=gen).half()
        Z = torch.empty(0, dtype=torch.float16, device=dev)
        for _ in range(launches):
            C = ops.fused_h17_gemv_s3(A, W, S, Z, group_size=128)
    elif kind == "grouped":
        K, Ns, M = int(dims[0]), [int(x) for x in dims[1].split("+")], int(dims[2])
        sets = pool_of(sum(K * N // 2 for N in Ns), lambda: [
            torch.randint(-2 ** 31, 2 ** 31 - 1, (K // 8, N), dtype=torch.int32, device=dev, generator=gen)
            for N in Ns])
        Ss = [(torch.randn((K // GROUP, N), device=dev, generator=gen).abs() * 0.02 + 1e-3).half() for N in Ns]
        A = torch.randn((M, K), device=dev, generator=gen).half()
        for i in range(launches):
            C = ops.fused_w4a16_gemm_grouped(A, sets[i % len(sets)], Ss)[0]
    elif kind == "dequant":
        dk, words = dims[0], int(dims[1])
        per = {"s4": 8, "s3": 10, "fp8": 4}[dk]
        Ws = pool_of(words * (8 + 2 * per), lambda: torch.randint(0, 2 ** 30, (words,), dtype=torch.int32,
                                                                    device=dev, generator=gen))
        S = (torch.randn(words, device=dev, generator=gen) * 0.02).half()
        Zp = torch.zeros(words, device=dev, dtype=torch.float16)
        for i in range(launches):
            W = Ws[i % len(Ws)]
            C = (ops.dequantize_fp8(W, S, mode="magic") if dk == "fp8" else
                 getattr(ops, f"dequantize_{dk}")(W, S, Zp, mode="magic"))
    else:
        raise SystemExit(f"unknown case {spec!r}")
    if kind in ("decode", "stream", "gemm"):
        S = (torch.randn((K // GROUP, N), device=dev, generator=gen).abs() * 0.02 + 1e-3).half()
        A = torch.randn((M, K), device=dev, generator=gen).half()
        prev = ops.set_gemv_kernel("stream") if kind == "stream" else None
        for i in range(launches):
            C = ops.fused_w4a16_gemm_s4(A, Ws[i % len(Ws)], S, None)
        if prev is not None:
            ops.set_gemv_kernel(prev)
    torch.cuda.synchronize()
    err = ops.device_error(dev)
    print(f"case {spec}: {launches} launches, mean |C| {float(C.float().abs().mean()):.4f}, device error {err}")
    if err:
        raise SystemExit(1)


def main():
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--no-gemm", action="store_true", help="skip the M=4096 prefill GEMM half of the metric")
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--m", type=int, default=1, help="activation rows (decode batch)")
    ap.add_argument("--cpu-budget", type=float, default=12.0, help="seconds of CPU baseline work")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--nccl-gather", action="store_true", help="N > 1: NCCL all-gather instead of the fused one")
    ap.add_argument("--no-70b", action="store_true", help="skip the column-sharded Llama-3-70B layer section")
    ap.add_argument("--case", help="profiling driver, comma-separated cases (see run_case; a few launches, no JSON)")
    ap.add_argument("--launches", type=int, default=6, help="launches for --case")
    args = ap.parse_args()
    if args.case:
        for spec in args.case.split(","):
            run_case(spec, args.launches)
            torch.cuda.empty_cache()
        return
    args.warmup = max(3, args.warmup)     # at least 3 untimed warm-up steps
    if args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()

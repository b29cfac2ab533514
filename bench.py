#!/usr/bin/env python3
"""Benchmark of the B200 k-quant decode path. Prints ONE JSON line (rank 0).

Headline metric: Q4_K GEMV HBM GB/s on the BASELINE config-2 shape (2048 rows x 6144, bf16 x,
M = 1). A step is one pass over a batch of `--matrices` distinct weight matrices (1.8 GB by default,
far larger than the 126 MB L2, so no L2 flush is needed) applied to the same activation row, as ONE
grouped launch (aipu_q4k_gemm_grouped), replayed as a CUDA graph. value = algorithmic bytes
(weights + x + y) of all GEMVs of all ranks / device time (max over ranks). The same GEMVs as one
launch per matrix (decode-style stream, programmatic dependent launch) are reported as
"single_launch".

Also reported: roofline of the GEMV kernel against MEASURED_PEAKS.json, the CPU baseline (the C
restatement of the reference's contract on the host cores), the end-to-end number through the public
API with host buffers, SM clocks sampled through NVML during the timed region, and the MoE-layer
decode throughput of BASELINE config 3 (1 GPU).

--impl reference times the reference's CPU implementation of the path (its C restatement, all host
threads) on the same config and metric.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

N_ROWS, K_COLS = 2048, 6144
GEMV_W_BYTES = N_ROWS * (K_COLS // 256) * 144            # 7,077,888
GEMV_BYTES = GEMV_W_BYTES + K_COLS * 2 + N_ROWS * 2       # + x bf16 + y bf16 = 7,094,272
METRIC = "Q4_K GEMV HBM GB/s"


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=400)
    ap.add_argument("--warmup", type=int, default=20)
    ap.add_argument("--impl", default="aipu", choices=["aipu", "reference"])
    ap.add_argument("--matrices", type=int, default=256, help="distinct weight matrices per step")
    ap.add_argument("--no-moe", action="store_true", help="skip the MoE decode measurement")
    ap.add_argument("--no-cpu", action="store_true", help="skip the CPU baseline")
    ap.add_argument("--stream-layers", type=int, default=75,
                    help="layers of the full-depth expert-parallel decode stream (BASELINE config 5) at N > 1, "
                         "capped by device memory; 0 skips it")
    return ap.parse_args()


def peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        d = json.load(open(p))
        return float(d["hbm_gbs"]), float(d["bf16_tflops"]), "measured"
    return 6650.0, 1590.0, "fallback"


def traffic_from_profile():
    """dram bytes per launch of the GEMV kernel from the committed ncu summary, if present."""
    p = os.path.join(ROOT, "profiles", "gemv_q4k_2048x6144.md")
    if not os.path.exists(p):
        return None
    for line in open(p):
        if line.strip().startswith("traffic_bytes_per_launch:"):
            try:
                return int(line.split(":")[1].strip().split()[0])
            except ValueError:
                return None
    return None


class _Null:
    def __enter__(self):
        return self

    def __exit__(self, *a):
        return False


class ClockSampler:
    """Samples SM clock and throttle reasons through NVML while running."""

    def __init__(self, index: int):
        self.index = index
        self.samples = []
        self.reasons = set()
        self._stop = threading.Event()
        self.ok = False
        self.max_mhz = None

    def __enter__(self):
        try:
            import pynvml as nv

            nv.nvmlInit()
            self.nv = nv
            self.h = nv.nvmlDeviceGetHandleByIndex(self.index)
            self.max_mhz = nv.nvmlDeviceGetMaxClockInfo(self.h, nv.NVML_CLOCK_SM)
            self.ok = True
            self.t = threading.Thread(target=self._run, daemon=True)
            self.t.start()
        except Exception:
            self.ok = False
        return self

    def _run(self):
        nv = self.nv
        names = {
            "hw_slowdown": getattr(nv, "nvmlClocksEventReasonHwSlowdown", 0x8),
            "hw_thermal_slowdown": getattr(nv, "nvmlClocksEventReasonHwThermalSlowdown", 0x40),
            "sw_thermal_slowdown": getattr(nv, "nvmlClocksEventReasonSwThermalSlowdown", 0x20),
            "sw_power_cap": getattr(nv, "nvmlClocksEventReasonSwPowerCap", 0x4),
            "hw_power_brake_slowdown": getattr(nv, "nvmlClocksEventReasonHwPowerBrakeSlowdown", 0x80),
        }
        while not self._stop.is_set():
            try:
                self.samples.append(nv.nvmlDeviceGetClockInfo(self.h, nv.NVML_CLOCK_SM))
                r = nv.nvmlDeviceGetCurrentClocksEventReasons(self.h)
                for k, bit in names.items():
                    if r & bit:
                        self.reasons.add(k)
            except Exception:
                pass
            time.sleep(0.005)

    def __exit__(self, *a):
        self._stop.set()
        if self.ok:
            self.t.join(timeout=1)

    def summary(self):
        if not self.ok or not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": self.max_mhz, "reasons": ["nvml unavailable"], "samples": 0}
        return {"sm_mhz": statistics.median(self.samples), "sm_max_mhz": self.max_mhz,
                "reasons": sorted(self.reasons), "samples": len(self.samples)}


def dist_setup(n_gpus):
    import torch

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import torch.distributed as dist

        import datetime

        torch.cuda.set_device(local)
        # a rank that fails leaves the others blocked in their next collective until this expires
        dist.init_process_group("nccl", device_id=torch.device("cuda", local),
                                timeout=datetime.timedelta(seconds=300))
    else:
        torch.cuda.set_device(0)
    return world, rank, local


def cpu_baseline_gemv(seconds=10.0, w=None, x=None):
    """The C restatement on all host cores: full 2048 x 6144 Q4_K GEMVs for ~`seconds`."""
    import numpy as np

    from aipu_b200 import formats as F
    from oracle import cpu

    if w is None:
        w = F.random_rows_np(F.Q4_K, N_ROWS, K_COLS, seed=0)
        x = np.random.default_rng(0).standard_normal((1, K_COLS)).astype(np.float32)
    cores = os.cpu_count() or 1
    cpu.gemm(F.Q4_K, w, N_ROWS, K_COLS, x, nthreads=cores)
    n, t0 = 0, time.perf_counter()
    while True:
        cpu.gemm(F.Q4_K, w, N_ROWS, K_COLS, x, nthreads=cores)
        n += 1
        dt = time.perf_counter() - t0
        if dt >= seconds:
            break
    return {"value": round(GEMV_BYTES * n / dt / 1e9, 4), "unit": "GB/s", "cores": cores, "kind": "port",
            "sample": f"{n} full Q4_K GEMVs 2048x6144 (M=1) by oracle/q4k_oracle.c, {cores} threads, {dt:.1f} s"}


def run_reference(args):
    """--impl reference: the reference's CPU implementation of the path (C restatement), rank 0 only."""
    import numpy as np

    from aipu_b200 import formats as F
    from oracle import cpu

    if int(os.environ.get("RANK", "0")) != 0:
        return
    cores = os.cpu_count() or 1
    w = F.random_rows_np(F.Q4_K, N_ROWS, K_COLS, seed=0)
    x = np.random.default_rng(0).standard_normal((1, K_COLS)).astype(np.float32)
    for _ in range(max(args.warmup, 1)):
        cpu.gemm(F.Q4_K, w, N_ROWS, K_COLS, x, nthreads=cores)
    t0 = time.perf_counter()
    for _ in range(args.steps):
        cpu.gemm(F.Q4_K, w, N_ROWS, K_COLS, x, nthreads=cores)
    dt = time.perf_counter() - t0
    v = GEMV_BYTES * args.steps / dt / 1e9
    line = {"metric": METRIC, "value": round(v, 4), "unit": "GB/s", "n_gpus": args.gpus, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(dt / args.steps * 1e3, 4), "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic", "impl": "reference",
            "config": {"workload": "Q4_K GEMV 2048x6144, x bf16-valued fp32 [1,6144], y bf16 (BASELINE config 2, "
                                   "Q4_K, M=1)", "step": "one GEMV"},
            "cpu_baseline": {"value": round(v, 4), "unit": "GB/s", "cores": cores, "kind": "port",
                             "sample": f"{args.steps} GEMVs, oracle/q4k_oracle.c (restatement of tools/q4k_ref.py)"},
            "e2e": {"value": round(v, 4), "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def moe_decode(M_list=(1, 4), reps=200):
    """BASELINE config 3 on one GPU: tokens/s of the MoE layer (CUDA graph replays)."""
    import numpy as np
    import torch

    from aipu_b200 import formats as F
    from aipu_b200 import ops

    d = torch.device("cuda", torch.cuda.current_device())
    H, Fd, E, T = 6144, 2048, 256, 8
    W = moe_layer_weights(d)
    ctx = ops.Context(d)
    out = {}
    expert_bytes = 2 * Fd * (H // 256) * 144 + H * (Fd // 256) * 210
    for M in M_list:
        x = (torch.randn((M, H), device=d, generator=torch.Generator(device=d).manual_seed(100 + M))).to(torch.bfloat16)
        y = torch.empty((M, H), dtype=torch.bfloat16, device=d)
        _, sel, _ = ops.moe_layer(W, x, ctx=ctx, out=y, return_routing=True)
        torch.cuda.synchronize()
        union = len(set(sel.cpu().numpy().reshape(-1).tolist()))
        g = torch.cuda.CUDAGraph()
        s = torch.cuda.Stream()
        with torch.cuda.stream(s):
            ops.moe_layer(W, x, ctx=ctx, out=y)
            torch.cuda.synchronize()
            with torch.cuda.graph(g, stream=s):
                ops.moe_layer(W, x, ctx=ctx, out=y)
        for _ in range(10):
            g.replay()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(reps):
            g.replay()
        e1.record()
        torch.cuda.synchronize()
        t = e0.elapsed_time(e1) / reps / 1e3
        byts = H * E * 4 + (union + 1) * expert_bytes
        out[f"M{M}"] = {"us_per_layer": round(t * 1e6, 2), "tokens_per_s": round(M / t, 1), "union_experts": union,
                        "hbm_bytes": byts, "hbm_gbs": round(byts / t / 1e9, 1)}
    out["prefill"] = moe_prefill(W)
    del W
    torch.cuda.empty_cache()
    return out


def moe_layer_weights(d):
    """BASELINE configs 3/4 weights: 256 routed experts + 1 shared, hidden 6144, FFN 2048."""
    import torch

    from aipu_b200 import formats as F
    from aipu_b200 import ops

    H, Fd, E, T = 6144, 2048, 256, 8
    return ops.MoeLayerWeights(
        hidden=H, ffn=Fd, n_experts=E, topk=T, router_wtype=F.F32,
        router_w=torch.randn((H, E), device=d, generator=torch.Generator(device=d).manual_seed(1)) * 0.02,
        router_bias=torch.randn((E,), device=d, generator=torch.Generator(device=d).manual_seed(2)) * 0.01,
        gate_w=F.random_rows_dev(F.Q4_K, E * Fd, H, seed=11, device=d),
        up_w=F.random_rows_dev(F.Q4_K, E * Fd, H, seed=12, device=d),
        down_w=F.random_rows_dev(F.Q6_K, E * H, Fd, seed=13, device=d),
        shared_gate_w=F.random_rows_dev(F.Q4_K, Fd, H, seed=14, device=d),
        shared_up_w=F.random_rows_dev(F.Q4_K, Fd, H, seed=15, device=d),
        shared_down_w=F.random_rows_dev(F.Q6_K, H, Fd, seed=16, device=d))


def moe_prefill(W, M=2048, reps=10):
    """BASELINE config 4 on one GPU: one MoE layer over 2048 tokens (router, per-expert token lists,
    tcgen05 SwiGLU and down GEMMs grouped by expert, shared expert, combine), CUDA-graph replays.
    Tensor FLOPs counted = 2 * (token-expert pairs + tokens for the shared expert) * 3 * H * F."""
    import torch

    from aipu_b200 import ops

    d = torch.device("cuda", torch.cuda.current_device())
    H, Fd, T = W.hidden, W.ffn, W.topk
    ctx = ops.Context(d)
    x = torch.randn((M, H), device=d, generator=torch.Generator(device=d).manual_seed(4)).to(torch.bfloat16)
    y = torch.empty((M, H), dtype=torch.bfloat16, device=d)
    s = torch.cuda.Stream()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.stream(s):
        ops.moe_layer(W, x, ctx=ctx, out=y)
        torch.cuda.synchronize()
        with torch.cuda.graph(g, stream=s):
            ops.moe_layer(W, x, ctx=ctx, out=y)
    for _ in range(3):
        g.replay()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(reps):
        g.replay()
    e1.record()
    torch.cuda.synchronize()
    t = e0.elapsed_time(e1) / reps / 1e3
    flops = 2.0 * (M * T + M) * 3 * H * Fd
    _, tf_peak, kind = peaks()
    return {"tokens": M, "ms_per_layer": round(t * 1e3, 3), "tokens_per_s": round(M / t, 1),
            "tensor_tflops": round(flops / t / 1e12, 1), "frac_of_bf16_peak": round(flops / t / 1e12 / tf_peak, 4),
            "peak_source": kind, "flops": flops}


def _time_ep_layer(layer, x, reps):
    """Device time per call of an expert-parallel layer (CUDA graph when capture works), max over ranks."""
    import torch
    import torch.distributed as dist

    d = x.device
    for _ in range(5):
        layer(x)
    torch.cuda.synchronize()
    run, graphed = (lambda: layer(x)), False
    try:
        gr = torch.cuda.CUDAGraph()
        s = torch.cuda.Stream()
        s.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s):
            layer(x)
            torch.cuda.synchronize()
            with torch.cuda.graph(gr, stream=s):
                layer(x)
        torch.cuda.synchronize()
        run, graphed = gr.replay, True
    except Exception:  # capture unsupported here: time eager calls
        torch.cuda.synchronize()
    for _ in range(5):
        run()
    torch.cuda.synchronize()
    dist.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(reps):
        run()
    e1.record()
    torch.cuda.synchronize()
    t = torch.tensor([e0.elapsed_time(e1) / reps / 1e3], device=d, dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return {"t": float(t.item()), "graphed": graphed}


def moe_decode_ep(world, rank, M_list=(1, 4), reps=100):
    """BASELINE config 3/5 decode layer with the 256 routed experts sharded over the N ranks
    (256/N per GPU, NCCL all-gather dispatch and all-to-all return); every rank decodes M tokens.
    tokens/s = N * M / (max-over-ranks device time per layer)."""
    import torch
    import torch.distributed as dist

    from aipu_b200 import ep
    from aipu_b200 import formats as F
    from aipu_b200 import ops

    d = torch.device("cuda", torch.cuda.current_device())
    H, Fd, E, T = 6144, 2048, 256, 8
    n = E // world
    g = torch.Generator(device=d)
    local = ops.MoeLayerWeights(
        hidden=H, ffn=Fd, n_experts=n, topk=T, router_wtype=F.F32,
        router_w=torch.randn((H, E), device=d, generator=g.manual_seed(1)) * 0.02,
        router_bias=torch.randn((E,), device=d, generator=g.manual_seed(2)) * 0.01,
        gate_w=F.random_rows_dev(F.Q4_K, n * Fd, H, seed=11 + 100 * rank, device=d),
        up_w=F.random_rows_dev(F.Q4_K, n * Fd, H, seed=12 + 100 * rank, device=d),
        down_w=F.random_rows_dev(F.Q6_K, n * H, Fd, seed=13 + 100 * rank, device=d),
        shared_gate_w=F.random_rows_dev(F.Q4_K, Fd, H, seed=14, device=d),
        shared_up_w=F.random_rows_dev(F.Q4_K, Fd, H, seed=15, device=d),
        shared_down_w=F.random_rows_dev(F.Q6_K, H, Fd, seed=16, device=d))
    sharded = ep.ShardedMoeWeights(local, rank * n, E)
    layers = {"nccl": ep.ExpertParallelMoE(sharded, backend=ep.CudaBackend(ops.Context(d))),
              "peer": ep.PeerExpertParallelMoE(sharded, max_tokens=max(M_list))}
    expert_bytes = 2 * Fd * (H // 256) * 144 + H * (Fd // 256) * 210
    out = {}
    for kind, layer in layers.items():
        for M in M_list:
            x = torch.randn((M, H), device=d, generator=g.manual_seed(100 + M + 7 * rank)).to(torch.bfloat16)
            r = _time_ep_layer(layer, x, reps)
            t = r["t"]
            # experts this rank touched in one layer (union of its local experts over all N*M tokens)
            sel_all = torch.empty((world * M, T), dtype=torch.int32, device=d)
            sel, _, _ = ops.moe_router(F.F32, local.router_w, x, E, T, bias=local.router_bias)
            dist.all_gather_into_tensor(sel_all, sel)
            touched = len(set(v for v in sel_all.cpu().numpy().reshape(-1).tolist() if rank * n <= v < (rank + 1) * n))
            byts = H * E * 4 + (touched + 1) * expert_bytes
            out[f"{kind}_M{M}"] = {"us_per_layer": round(t * 1e6, 2), "tokens_per_s": round(world * M / t, 1),
                                   "tokens_per_rank": M, "experts_per_gpu": n, "rank0_touched_experts": touched,
                                   "cuda_graph": r["graphed"], "rank0_hbm_gbs": round(byts / t / 1e9, 1)}
    layers["peer"].close()
    return out


def moe_decode_stream(world, rank, layers_req=75, M_list=(1, 4), reps=10):
    """the full-depth decode weight stream, `layers_req` MoE layers (256 routed
    experts + 1 shared each, hidden 6144, FFN 2048) with the routed experts sharded over the N ranks,
    run back to back for M tokens per rank (each layer's output feeds the next), over the NVLink
    peer exchange and over NCCL. The layer count is capped by free device memory and by ~64 GB of
    weights per GPU (75 layers fit at N = 8; fewer at N < 8, reported).
    tokens/s = N * M / (max-over-ranks device time of one pass through all layers)."""
    import torch
    import torch.distributed as dist

    from aipu_b200 import ep
    from aipu_b200 import formats as F
    from aipu_b200 import ops

    d = torch.device("cuda", torch.cuda.current_device())
    H, Fd, E, T = 6144, 2048, 256, 8
    n = E // world
    expert_bytes = 2 * Fd * F.row_bytes(F.Q4_K, H) + H * F.row_bytes(F.Q6_K, Fd)
    per_layer = (n + 1) * expert_bytes + H * E * 4 + E * 4
    torch.cuda.empty_cache()
    free = torch.cuda.mem_get_info(d)[0]
    cap = torch.tensor([max(0, int((free - 8e9) // per_layer))], device=d, dtype=torch.int64)
    dist.all_reduce(cap, op=dist.ReduceOp.MIN)
    # at most ~64 GB of weights per GPU (the config-5 share at N = 8), so every N takes similar time
    L = min(layers_req, int(cap.item()), int(64e9 // per_layer))
    if L < 1:
        return {"skipped": f"not enough device memory for one layer ({per_layer / 1e9:.1f} GB per layer per GPU)"}
    g = torch.Generator(device=d)
    layers = []
    for l in range(L):
        s0 = 100000 * (l + 1)
        local = ops.MoeLayerWeights(
            hidden=H, ffn=Fd, n_experts=n, topk=T, router_wtype=F.F32,
            router_w=torch.randn((H, E), device=d, generator=g.manual_seed(s0 + 1)) * 0.02,
            router_bias=torch.randn((E,), device=d, generator=g.manual_seed(s0 + 2)) * 0.01,
            gate_w=F.random_rows_dev(F.Q4_K, n * Fd, H, seed=s0 + 11 + 100 * rank, device=d),
            up_w=F.random_rows_dev(F.Q4_K, n * Fd, H, seed=s0 + 12 + 100 * rank, device=d),
            down_w=F.random_rows_dev(F.Q6_K, n * H, Fd, seed=s0 + 13 + 100 * rank, device=d),
            shared_gate_w=F.random_rows_dev(F.Q4_K, Fd, H, seed=s0 + 14, device=d),
            shared_up_w=F.random_rows_dev(F.Q4_K, Fd, H, seed=s0 + 15, device=d),
            shared_down_w=F.random_rows_dev(F.Q6_K, H, Fd, seed=s0 + 16, device=d))
        layers.append(ep.ShardedMoeWeights(local, rank * n, E))
    out = {"layers": L, "full_depth": L == 75, "experts_per_gpu": n,
           "weights_gb_per_gpu": round(L * per_layer / 1e9, 1)}
    for kind in ("peer", "nccl"):
        stream = ep.DecodeStream(layers, exchange=kind, max_tokens=max(M_list),
                                 backend=ep.CudaBackend(ops.Context(d)) if kind == "nccl" else None)
        for M in M_list:
            x = torch.randn((M, H), device=d, generator=g.manual_seed(7 + M + 31 * rank)).to(torch.bfloat16)
            r = _time_ep_layer(stream, x, reps)
            t = r["t"]
            out[f"{kind}_M{M}"] = {"ms_per_pass": round(t * 1e3, 3), "us_per_layer": round(t / L * 1e6, 2),
                                   "tokens_per_s": round(world * M / t, 1), "cuda_graph": r["graphed"]}
        stream.close()
    del layers
    torch.cuda.empty_cache()
    return out


def main():
    args = parse()
    if args.impl == "reference":
        run_reference(args)
        return
    import numpy as np
    import torch

    from aipu_b200 import formats as F
    from aipu_b200 import ops

    world, rank, local = dist_setup(args.gpus)
    d = torch.device("cuda", torch.cuda.current_device())
    L = args.matrices
    Wt = F.random_rows_dev(F.Q4_K, L * N_ROWS, K_COLS, seed=1234 + rank, device=d)
    rb = F.row_bytes(F.Q4_K, K_COLS)
    mats = [Wt[l * N_ROWS:(l + 1) * N_ROWS] for l in range(L)]
    x = torch.randn((1, K_COLS), device=d, generator=torch.Generator(device=d).manual_seed(7)).to(torch.bfloat16)
    y = torch.empty((L, 1, N_ROWS), dtype=torch.bfloat16, device=d)
    ctx = ops.Context(d).set_flags(pdl=True)

    def issue_grouped():
        ops.gemm_grouped(F.Q4_K, Wt, L, N_ROWS, K_COLS, x, ctx=ctx, out=y)

    def issue_single():
        for l in range(L):
            ops.gemm(F.Q4_K, mats[l], N_ROWS, K_COLS, x, ctx=ctx, out=y[l])

    def capture(fn):
        g = torch.cuda.CUDAGraph()
        with torch.cuda.stream(s):
            fn()
            torch.cuda.synchronize()
            with torch.cuda.graph(g, stream=s):
                fn()
        torch.cuda.synchronize()
        return g

    def timed(g, steps, warmup, sampler=None):
        for _ in range(max(warmup, 3)):
            g.replay()
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        with (sampler if sampler is not None else _Null()):
            torch.cuda.synchronize()
            e0.record()
            for _ in range(steps):
                g.replay()
            e1.record()
            torch.cuda.synchronize()
        t = e0.elapsed_time(e1) / 1e3
        if world > 1:
            tt = torch.tensor([t], device=d, dtype=torch.float64)
            dist.all_reduce(tt, op=dist.ReduceOp.MAX)
            t = float(tt.item())
        return t / steps

    s = torch.cuda.Stream()
    if world > 1:
        import torch.distributed as dist
    g = capture(issue_grouped)
    clk = ClockSampler(d.index)
    step = timed(g, args.steps, args.warmup, clk)
    value = world * L * GEMV_BYTES / step / 1e9
    hbm_peak, _, peak_kind = peaks()
    achieved = L * GEMV_BYTES / step / 1e9
    # the same GEMVs as one launch per matrix (decode-style stream), back to back with PDL
    gs = capture(issue_single)
    step_single = timed(gs, max(10, args.steps // 4), args.warmup)
    single = {"us_per_launch": round(step_single / L * 1e6, 3),
              "gbs": round(L * GEMV_BYTES / step_single / 1e9, 1),
              "note": "one kernel launch per 2048x6144 matrix, CUDA graph, programmatic dependent launch"}
    del gs

    # ---- end to end through the public API with host buffers (x in, all y out, every step)
    x_host = torch.empty((1, K_COLS), dtype=torch.bfloat16, pin_memory=True).copy_(x.cpu())
    y_host = torch.empty((L, 1, N_ROWS), dtype=torch.bfloat16, pin_memory=True)
    e2e_steps = max(10, args.steps // 4)
    torch.cuda.synchronize()
    with torch.cuda.stream(s):
        for _ in range(3):
            x.copy_(x_host, non_blocking=True)
            g.replay()
            y_host.copy_(y, non_blocking=True)
        s.synchronize()
        t0 = time.perf_counter()
        for _ in range(e2e_steps):
            x.copy_(x_host, non_blocking=True)
            g.replay()
            y_host.copy_(y, non_blocking=True)
        s.synchronize()
        te = (time.perf_counter() - t0) / e2e_steps
    if world > 1:
        tt = torch.tensor([te], device=d, dtype=torch.float64)
        dist.all_reduce(tt, op=dist.ReduceOp.MAX)
        te = float(tt.item())
    e2e = {"value": round(world * L * GEMV_BYTES / te / 1e9, 2), "unit": "GB/s",
           "h2d_bytes_per_step": K_COLS * 2, "d2h_bytes_per_step": L * N_ROWS * 2,
           "path": "ops.gemm_grouped -> aipu_q4k_gemm_grouped (C ABI), replayed as a CUDA graph; pinned host x in, "
                   "all y out, every step"}

    del Wt, mats
    torch.cuda.empty_cache()
    moe = None
    if rank == 0 and world == 1 and not args.no_moe:
        moe = moe_decode()
    moe_ep = None
    moe_stream = None
    if world > 1 and not args.no_moe:
        moe_ep = moe_decode_ep(world, rank)
        if args.stream_layers > 0:
            try:
                moe_stream = moe_decode_stream(world, rank, args.stream_layers)
            except Exception as e:  # reported in the line; the GEMV metric above stands
                moe_stream = {"error": f"{type(e).__name__}: {e}"[:300]}
    cpu_base = None
    if rank == 0 and world == 1 and not args.no_cpu:
        cpu_base = cpu_baseline_gemv()
    if rank == 0:
        line = {
            "metric": METRIC, "value": round(value, 2), "unit": "GB/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(step * 1e3, 4), "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": {"workload": "Q4_K GEMV 2048x6144, x bf16 [1,6144] ~N(0,1), y bf16 (BASELINE config 2, Q4_K, "
                                   "M=1); a step = one grouped launch over the batch of matrices",
                       "matrices_per_step": L, "bytes_per_gemv": GEMV_BYTES,
                       "l2": f"inputs larger than L2: {L * GEMV_W_BYTES / 1e9:.2f} GB of distinct weights per step",
                       "parallelism": f"replicas x{world}"},
            "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": hbm_peak, "unit": "GB/s",
                         "frac": round(achieved / hbm_peak, 4), "traffic": traffic_from_profile(),
                         "peak_source": peak_kind, "kernel": "aipu_kq_gemv_kernel<Q4_K,bf16,store> (grouped launch)",
                         "us_per_launch": round(step * 1e6, 3)},
            "single_launch": single,
            "cpu_baseline": cpu_base, "e2e": e2e, "gpu_launches": args.steps,
            "clocks": clk.summary(), "moe_decode": moe, "moe_decode_ep": moe_ep,
            "moe_decode_stream": moe_stream,
        }
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.destroy_process_group()


if __name__ == "__main__":
    main()

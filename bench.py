#!/usr/bin/env python3
"""Benchmark of the B200 k-quant decode path. Prints ONE JSON line (rank 0).

Headline: Q4_K GEMV HBM GB/s on 4096 x 4096 Q4_K weights (16 super-blocks per
row), x fp32 [1, 4096] ~ N(0, 1) drawn with numpy seed 0, bf16 out. A step is ONE grouped launch
(aipu_q4k_gemm_grouped) over `--matrices` distinct seeded matrices (64 x 9.4 MB = 604 MB, more than
twice the 126 MB L2, so no flush is needed), replayed as a CUDA graph. value = algorithmic bytes
(weights + x + y) of all GEMVs of all ranks / device time (max over ranks). The same GEMVs as one
launch per matrix are reported as "single_launch".

Also reported: the roofline of the GEMV kernel against MEASURED_PEAKS.json; the CPU baselines (the C
restatement of the reference's contract on all host cores, and the numpy restatement on a sample);
the end-to-end number through the public API with host buffers; SM clocks sampled through NVML during
the timed region; the Q6_K decode GEMV (6144 x 2048, grouped) with its parity; the MoE layer of
BASELINE configs 3 (decode, M = 1 and 4) and 4 (prefill, 2048 tokens) on the default bit-exact path,
the exact-gate/up + GEMV-down path and the tensor-core path, each with parity against the
oracle computed in the same run (the oracle's timed CPU run of the same sampled tokens is the CPU
baseline of that layer); at N > 1 the expert-parallel decode layer and the full-depth decode stream.

--impl reference times the reference's CPU implementation of the path (its C restatement, all host
threads) on the same config, inputs and per-step work.
--case {gemv,chain,tc,moe,router} runs one small workload for a profiler capture and exits.
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

# BASELINE config 1
C1_N, C1_K = 4096, 4096
C1_W_BYTES = C1_N * (C1_K // 256) * 144                # 9,437,184
C1_BYTES = C1_W_BYTES + C1_K * 4 + C1_N * 2             # + x fp32 + y bf16 = 9,461,760
METRIC = "Q4_K GEMV HBM GB/s"
# DRAM bytes per C1 GEMV of the grouped kernel, from one ncu capture (dram__bytes_read.sum +
# dram__bytes_write.sum = 75,807,744 + 2,077,696 B) of an 8-matrix C1 launch
# (`bench.py --case gemv --x-f32 --groups 8`) divided by 8; the full launch reads every weight byte
# once, so its traffic is this times the matrices per launch.
C1_TRAFFIC_PER_GEMV = 9_735_680
MOE_H, MOE_F, MOE_E, MOE_T = 6144, 2048, 256, 8


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=100)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", default="aipu", choices=["aipu", "reference"])
    ap.add_argument("--matrices", type=int, default=64, help="distinct 4096x4096 Q4_K matrices per step")
    ap.add_argument("--no-moe", action="store_true", help="skip the MoE measurements")
    ap.add_argument("--no-cpu", action="store_true", help="skip the CPU baselines")
    ap.add_argument("--stream-layers", type=int, default=75,
                    help="layers of the full-depth expert-parallel decode stream (BASELINE config 5) at N > 1, "
                         "capped by device memory; 0 skips it")
    ap.add_argument("--case", default=None, choices=["gemv", "chain", "tc", "moe", "router"],
                    help="run one small workload for a profiler capture and exit")
    ap.add_argument("--wtype", type=int, default=0)
    ap.add_argument("--n", type=int, default=4096)
    ap.add_argument("--k", type=int, default=4096)
    ap.add_argument("--m", type=int, default=1)
    ap.add_argument("--x-f32", action="store_true")
    ap.add_argument("--groups", type=int, default=8)
    ap.add_argument("--experts", type=int, default=64)
    ap.add_argument("--tokens", type=int, default=512)
    return ap.parse_args()


def peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        d = json.load(open(p))
        return float(d["hbm_gbs"]), float(d["bf16_tflops"]), "measured"
    return 6650.0, 1590.0, "fallback"


def q6k_grouped(F, ops, ctx, s, timed, hbm_peak, rank0, L=64, N=6144, K=2048):
    """The Q6_K decode GEMV (MoE down-projection shape 6144 x 2048, bf16 x, M = 1) as one grouped
    launch over L distinct seeded matrices (0.66 GB > L2), with the parity of matrix 0 against the
    oracle (checker use, rank 0)."""
    import numpy as np
    import torch

    d = torch.device("cuda", torch.cuda.current_device())
    w = F.random_rows_dev(F.Q6_K, L * N, K, seed=21, device=d)
    x = torch.randn((1, K), device=d, generator=torch.Generator(device=d).manual_seed(22)).to(torch.bfloat16)
    y = torch.empty((L, 1, N), dtype=torch.bfloat16, device=d)
    g = _graph(lambda: ops.gemm_grouped(F.Q6_K, w, L, N, K, x, ctx=ctx, out=y), s)
    t = timed(g, 20, 3)
    byts = L * (N * (K // 256) * 210 + K * 2 + N * 2)
    out = {"matrices": L, "shape": f"{N}x{K}", "us_per_launch": round(t * 1e6, 2), "gbs": round(byts / t / 1e9, 1),
           "frac": round(byts / t / 1e9 / hbm_peak, 4),
           "kernel": "aipu_kq_gemv_kernel<Q6_K, bf16 x, store> (integer dot engine)"}
    if rank0:
        from oracle import q4k_oracle as qo

        ref = qo.gemm(F.Q6_K, w[:N].cpu().numpy(), N, K, x.float().cpu().numpy())
        got = _bf16_np(y[0])
        st = qo.parity_stats(got, ref)
        out["parity"] = {k: (round(v, 6) if isinstance(v, float) else v) for k, v in st.items()}
    del g, w
    return out


def c1_inputs(L):
    """BASELINE config 1 inputs, identical in both arms: x = numpy default_rng(0) N(0,1) fp32 [1, 4096];
    matrix l = formats.random_rows_np(Q4_K, 4096, 4096, seed=1000 + l)."""
    import numpy as np

    from aipu_b200 import formats as F

    x = np.random.default_rng(0).standard_normal((1, C1_K)).astype(np.float32)
    w = np.empty((L, C1_N, F.row_bytes(F.Q4_K, C1_K)), np.uint8)
    for l in range(L):
        w[l] = F.random_rows_np(F.Q4_K, C1_N, C1_K, seed=1000 + l)
    return x, w


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
        self._names = names
        i = 0
        while not self._stop.is_set():
            try:
                self.samples.append(nv.nvmlDeviceGetClockInfo(self.h, nv.NVML_CLOCK_SM))
                # the reasons query is the slower one: every fourth sample, and always the first
                if i % 4 == 0:
                    r = nv.nvmlDeviceGetCurrentClocksEventReasons(self.h)
                    for k, bit in names.items():
                        if r & bit:
                            self.reasons.add(k)
            except Exception:
                pass
            i += 1
            time.sleep(0.0002)

    def __exit__(self, *a):
        self._stop.set()
        if self.ok:
            self.t.join(timeout=1)
            try:  # the reasons at the end of the region too
                r = self.nv.nvmlDeviceGetCurrentClocksEventReasons(self.h)
                for k, bit in self._names.items():
                    if r & bit:
                        self.reasons.add(k)
            except Exception:
                pass

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


def cpu_baseline_c1(x, w, seconds=10.0):
    """CPU baselines of the headline workload on the host cores: (a) the C restatement of the
    reference's contract (oracle/q4k_oracle.c) on all cores over the distinct matrices for ~`seconds`;
    (b) the numpy restatement (oracle/q4k_oracle.py, vectorised over rows, sequential over K) on a
    256-row sample of one matrix, its rate scaled to GB/s of the same workload."""
    import numpy as np

    from aipu_b200 import formats as F
    from oracle import cpu
    from oracle import q4k_oracle as qo

    cores = os.cpu_count() or 1
    L = w.shape[0]
    cpu.gemm(F.Q4_K, w[0], C1_N, C1_K, x, nthreads=cores)
    n, t0 = 0, time.perf_counter()
    while True:
        cpu.gemm(F.Q4_K, w[n % L], C1_N, C1_K, x, nthreads=cores)
        n += 1
        dt = time.perf_counter() - t0
        if dt >= seconds:
            break
    out = {"value": round(C1_BYTES * n / dt / 1e9, 4), "unit": "GB/s", "cores": cores, "kind": "port",
           "sample": f"{n} full C1 GEMVs (Q4_K 4096x4096, x fp32) by oracle/q4k_oracle.c on {cores} threads, "
                     f"{dt:.1f} s"}
    rows = 256
    t0 = time.perf_counter()
    qo.gemm(F.Q4_K, w[0][:rows], rows, C1_K, x)
    dt = time.perf_counter() - t0
    out["numpy"] = {"value": round(C1_BYTES * rows / C1_N / dt / 1e9, 5), "unit": "GB/s", "cores": 1,
                    "kind": "port", "sample": f"{rows} of 4096 rows of one C1 GEMV by oracle/q4k_oracle.py "
                                               f"(numpy, one core), {dt:.2f} s, rate scaled to the full GEMV"}
    return out


def run_reference(args):
    """--impl reference: the reference's contract on the host cores (the C restatement), rank 0 only,
    on the same inputs and per-step work as the GPU arm (one step = the GEMVs of all matrices)."""
    if int(os.environ.get("RANK", "0")) != 0:
        return
    from aipu_b200 import formats as F
    from oracle import cpu

    cores = os.cpu_count() or 1
    L = args.matrices
    x, w = c1_inputs(L)
    for _ in range(max(args.warmup, 1)):
        cpu.gemm(F.Q4_K, w[0], C1_N, C1_K, x, nthreads=cores)
    t0 = time.perf_counter()
    for _ in range(args.steps):
        for l in range(L):
            cpu.gemm(F.Q4_K, w[l], C1_N, C1_K, x, nthreads=cores)
    dt = time.perf_counter() - t0
    v = L * C1_BYTES * args.steps / dt / 1e9
    line = {"metric": METRIC, "value": round(v, 4), "unit": "GB/s", "n_gpus": args.gpus, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(dt / args.steps * 1e3, 4), "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic", "impl": "reference",
            "config": c1_config(L, args.gpus),
            "cpu_baseline": {"value": round(v, 4), "unit": "GB/s", "cores": cores, "kind": "port",
                             "sample": f"{args.steps} steps x {L} C1 GEMVs, oracle/q4k_oracle.c (the C restatement "
                                       f"of tools/q4k_ref.py matmul_q4k_col) on {cores} threads"},
            "e2e": {"value": round(v, 4), "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def c1_config(L, world):
    return {"workload": "BASELINE config 1: Q4_K GEMV, W 4096 rows x 4096 (16 super-blocks per row), x fp32 [1,4096] "
                        "~N(0,1) (numpy seed 0), y bf16; a step = the GEMVs of all matrices (one grouped launch)",
            "matrices_per_step": L, "bytes_per_gemv": C1_BYTES,
            "l2": f"inputs larger than L2: {L * C1_W_BYTES / 1e9:.2f} GB of distinct weights per step",
            "parallelism": f"replicas x{world}"}


def _graph(fn, stream):
    import torch

    g = torch.cuda.CUDAGraph()
    with torch.cuda.stream(stream):
        fn()
        torch.cuda.synchronize()
        with torch.cuda.graph(g, stream=stream):
            fn()
    torch.cuda.synchronize()
    return g


def _time_graph(g, reps, stream):
    import torch

    with torch.cuda.stream(stream):
        for _ in range(3):
            g.replay()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(reps):
            g.replay()
        e1.record(stream)
        torch.cuda.synchronize()
    return e0.elapsed_time(e1) / reps / 1e3


def moe_layer_weights(d):
    """BASELINE configs 3/4 weights: 256 routed experts + 1 shared, hidden 6144, FFN 2048."""
    import torch

    from aipu_b200 import formats as F
    from aipu_b200 import ops

    H, Fd, E, T = MOE_H, MOE_F, MOE_E, MOE_T
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


def _bf16_np(t):
    import numpy as np

    return (t.view(__import__("torch").int16).cpu().numpy().astype(np.uint16).astype(np.uint32) << 16).view(np.float32)


def moe_oracle_check(W, x_bf, y, sel, sw, rows):
    """CPU baseline leg of the MoE layer: the oracle layer (C restatement GEMMs on packed rows) on the
    sampled token rows, timed on the host cores; its outputs against the GPU's give the parity object."""
    import numpy as np

    from oracle import moe_oracle as mo
    from oracle import q4k_oracle as qo

    H, Fd, E, T = W.hidden, W.ffn, W.n_experts, W.topk
    xs = _bf16_np(x_bf)[rows]
    gv, uv, dv = W.gate_w.view(E, Fd, -1), W.up_w.view(E, Fd, -1), W.down_w.view(E, H, -1)

    def experts(e):
        return gv[e].cpu().numpy(), uv[e].cpu().numpy(), dv[e].cpu().numpy()

    shared = (W.shared_gate_w.cpu().numpy(), W.shared_up_w.cpu().numpy(), W.shared_down_w.cpu().numpy())
    wr = W.router_w.cpu().numpy().T.copy()
    bias = W.router_bias.cpu().numpy()
    t0 = time.perf_counter()
    y_ref, sel_ref, sw_ref = mo.moe_layer_packed(xs, wr, experts, shared, T, bias=bias, gate_wtype=W.gate_wtype,
                                                 down_wtype=W.down_wtype)
    dt = time.perf_counter() - t0
    got = _bf16_np(y)[rows]
    st = qo.parity_stats(got, y_ref)
    parity = {"tokens_checked": int(len(rows)), "frac_within_1ulp": round(st["frac_within_1ulp"], 6),
              "max_rel": round(st["max_rel"], 6), "max_ulp": st["max_ulp"],
              "bit_exact": bool(np.array_equal(got.view(np.uint32), y_ref.view(np.uint32))),
              "topk_exact": bool(np.array_equal(sel.cpu().numpy()[rows], sel_ref)),
              "weights_exact": bool(np.array_equal(_bf16_np(sw)[rows].view(np.uint32), sw_ref.view(np.uint32)))}
    cpu = {"value": round(len(rows) / dt, 3), "unit": "tokens/s", "cores": os.cpu_count() or 1, "kind": "port",
           "sample": f"{len(rows)} token rows through oracle/moe_oracle.py moe_layer_packed (C restatement GEMMs, "
                     f"all cores), {dt:.1f} s including the host copies of the experts"}
    return parity, cpu


def moe_bench(check=True):
    """BASELINE config 3 (decode, M = 1 and 4) and config 4 (prefill, 2048 tokens) on one GPU, on the
    default bit-exact path and on the tensor-core path, CUDA-graph replays, with parity."""
    import numpy as np
    import torch

    from aipu_b200 import ops

    d = torch.device("cuda", torch.cuda.current_device())
    H, Fd, E, T = MOE_H, MOE_F, MOE_E, MOE_T
    W = moe_layer_weights(d)
    s = torch.cuda.Stream()
    hbm, tf_peak, kind = peaks()
    expert_bytes = 2 * Fd * (H // 256) * 144 + H * (Fd // 256) * 210
    out = {}
    paths = {"exact": {}, "exact_gateup_fast_down": {"fast_down": True}, "tensor_core": {"tc_decode": True}}
    for M in (1, 4):
        x = (torch.randn((M, H), device=d, generator=torch.Generator(device=d).manual_seed(100 + M))).to(torch.bfloat16)
        y = torch.empty((M, H), dtype=torch.bfloat16, device=d)
        for name, flags in paths.items():
            ctx = ops.Context(d).set_flags(**flags)
            yy, sel, sw = ops.moe_layer(W, x, ctx=ctx, out=y, return_routing=True)
            torch.cuda.synchronize()
            union = len(set(sel.cpu().numpy().reshape(-1).tolist()))
            g = _graph(lambda: ops.moe_layer(W, x, ctx=ctx, out=y), s)
            t = _time_graph(g, 100, s)
            byts = H * E * 4 + (union + 1) * expert_bytes
            ent = {"us_per_layer": round(t * 1e6, 2), "tokens_per_s": round(M / t, 1), "union_experts": union,
                   "hbm_bytes": byts, "hbm_gbs": round(byts / t / 1e9, 1),
                   "roofline_frac": round(byts / t / 1e9 / hbm, 4)}
            if check:
                ent["parity"], ent["cpu_baseline"] = moe_oracle_check(W, x, y, sel, sw, np.arange(M))
            out[f"{name}_M{M}"] = ent
            del g
            ctx.close()
    out["prefill"] = moe_prefill_bench(W, check)
    del W
    torch.cuda.empty_cache()
    return out


def moe_prefill_bench(W, check):
    """BASELINE config 4 on one GPU: one MoE layer over 2048 tokens, CUDA-graph replays. Tensor-core
    path (default for >= 64 tokens) and the bit-exact chain path (AIPU_FLAG_STRICT). Tensor FLOPs
    counted = 2 * (token-expert pairs + tokens for the shared expert) * 3 * H * F."""
    import numpy as np
    import torch

    from aipu_b200 import ops

    d = torch.device("cuda", torch.cuda.current_device())
    H, Fd, T = W.hidden, W.ffn, W.topk
    M = 2048
    x = torch.randn((M, H), device=d, generator=torch.Generator(device=d).manual_seed(4)).to(torch.bfloat16)
    y = torch.empty((M, H), dtype=torch.bfloat16, device=d)
    s = torch.cuda.Stream()
    flops = 2.0 * (M * T + M) * 3 * H * Fd
    _, tf_peak, kind = peaks()
    out = {"tokens": M, "flops": flops, "peak_source": kind}
    rows = np.sort(np.random.default_rng(7).choice(M, 16, replace=False))
    for name, flags, reps in (("tensor_core", {}, 10), ("exact", {"strict": True}, 2)):
        ctx = ops.Context(d).set_flags(**flags)
        yy, sel, sw = ops.moe_layer(W, x, ctx=ctx, out=y, return_routing=True)
        torch.cuda.synchronize()
        g = _graph(lambda: ops.moe_layer(W, x, ctx=ctx, out=y), s)
        t = _time_graph(g, reps, s)
        ent = {"ms_per_layer": round(t * 1e3, 3), "tokens_per_s": round(M / t, 1),
               "tensor_tflops": round(flops / t / 1e12, 1), "frac_of_bf16_peak": round(flops / t / 1e12 / tf_peak, 4)}
        if check:
            ent["parity"], ent["cpu_baseline"] = moe_oracle_check(W, x, y, sel, sw, rows)
        out[name] = ent
        del g
        ctx.close()
    return out


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


def _ep_local_weights(d, world, rank):
    """Rank `rank`'s share of the BASELINE config 3/4 layer: experts [r*E/N, (r+1)*E/N), the router and
    the shared expert replicated."""
    import torch

    from aipu_b200 import formats as F
    from aipu_b200 import ops

    H, Fd, E, T = MOE_H, MOE_F, MOE_E, MOE_T
    n = E // world
    g = torch.Generator(device=d)
    return ops.MoeLayerWeights(
        hidden=H, ffn=Fd, n_experts=n, topk=T, router_wtype=F.F32,
        router_w=torch.randn((H, E), device=d, generator=g.manual_seed(1)) * 0.02,
        router_bias=torch.randn((E,), device=d, generator=g.manual_seed(2)) * 0.01,
        gate_w=F.random_rows_dev(F.Q4_K, n * Fd, H, seed=11 + 100 * rank, device=d),
        up_w=F.random_rows_dev(F.Q4_K, n * Fd, H, seed=12 + 100 * rank, device=d),
        down_w=F.random_rows_dev(F.Q6_K, n * H, Fd, seed=13 + 100 * rank, device=d),
        shared_gate_w=F.random_rows_dev(F.Q4_K, Fd, H, seed=14, device=d),
        shared_up_w=F.random_rows_dev(F.Q4_K, Fd, H, seed=15, device=d),
        shared_down_w=F.random_rows_dev(F.Q6_K, H, Fd, seed=16, device=d))


def _one_gpu_layer_us(d, M, reps=50, **flags):
    """Device time of the whole BASELINE config 3/4 layer (all 256 experts) on this GPU for M tokens."""
    import torch

    from aipu_b200 import ops

    W = moe_layer_weights(d)
    x = torch.randn((M, MOE_H), device=d, generator=torch.Generator(device=d).manual_seed(55)).to(torch.bfloat16)
    y = torch.empty((M, MOE_H), dtype=torch.bfloat16, device=d)
    ctx = ops.Context(d).set_flags(**flags)
    s = torch.cuda.Stream()
    ops.moe_layer(W, x, ctx=ctx, out=y)
    torch.cuda.synchronize()
    g = _graph(lambda: ops.moe_layer(W, x, ctx=ctx, out=y), s)
    t = _time_graph(g, reps, s)
    del g, W
    ctx.close()
    torch.cuda.empty_cache()
    return t


def moe_decode_ep(world, rank, M_list=(1, 4), reps=100):
    """BASELINE config 3 decode layer with the 256 routed experts sharded over the N ranks (256/N per
    GPU); every rank decodes M tokens. Exchanges: NCCL (all-gather dispatch, all-to-all return) and
    the NVLink peer-memory exchange inside the library. tokens/s = N * M / (max-over-ranks device time
    per layer). Per rank: the HBM bytes it streams (router, the local experts its ranks' tokens
    touched, the shared expert) and their fraction of the measured HBM peak; efficiency_vs_n1 = the
    one-GPU layer's time for all N * M tokens / (N * the expert-parallel time)."""
    import torch
    import torch.distributed as dist

    from aipu_b200 import ep
    from aipu_b200 import formats as F
    from aipu_b200 import ops

    d = torch.device("cuda", torch.cuda.current_device())
    H, Fd, E, T = MOE_H, MOE_F, MOE_E, MOE_T
    n = E // world
    hbm, _, _ = peaks()
    local = _ep_local_weights(d, world, rank)
    sharded = ep.ShardedMoeWeights(local, rank * n, E)
    layers = {"nccl": ep.ExpertParallelMoE(sharded, backend=ep.CudaBackend(ops.Context(d))),
              "peer": ep.PeerExpertParallelMoE(sharded, max_tokens=max(M_list))}
    expert_bytes = 2 * Fd * (H // 256) * 144 + H * (Fd // 256) * 210
    g = torch.Generator(device=d)
    out = {}
    t1 = {}
    for M in M_list:
        x = torch.randn((M, H), device=d, generator=g.manual_seed(100 + M + 7 * rank)).to(torch.bfloat16)
        sel_all = torch.empty((world * M, T), dtype=torch.int32, device=d)
        sel, _, _ = ops.moe_router(F.F32, local.router_w, x, E, T, bias=local.router_bias)
        dist.all_gather_into_tensor(sel_all, sel)
        touched = len(set(v for v in sel_all.cpu().numpy().reshape(-1).tolist() if rank * n <= v < (rank + 1) * n))
        byts = H * E * 4 + (touched + 1) * expert_bytes
        for kind, layer in layers.items():
            r = _time_ep_layer(layer, x, reps)
            t = r["t"]
            out[f"{kind}_M{M}"] = {"us_per_layer": round(t * 1e6, 2), "tokens_per_s": round(world * M / t, 1),
                                   "tokens_per_rank": M, "experts_per_gpu": n, "rank0_touched_experts": touched,
                                   "cuda_graph": r["graphed"], "rank0_hbm_gbs": round(byts / t / 1e9, 1),
                                   "rank0_hbm_frac": round(byts / t / 1e9 / hbm, 4)}
    layers["peer"].close()
    del layers, local, sharded
    torch.cuda.empty_cache()
    if rank == 0:
        for M in M_list:
            t1[M] = _one_gpu_layer_us(d, world * M)
            for kind in ("nccl", "peer"):
                ent = out[f"{kind}_M{M}"]
                ent["one_gpu_us_for_all_tokens"] = round(t1[M] * 1e6, 2)
                ent["efficiency_vs_n1"] = round(t1[M] / (world * ent["us_per_layer"] * 1e-6), 4)
    dist.barrier()
    return out


def moe_prefill_ep(world, rank, M=2048, reps=3):
    """BASELINE config 4 expert-parallel: 2048 tokens per rank, all-to-all dispatch of each token to the
    ranks owning its experts (NCCL), the tensor-core expert GEMMs on every rank's received tokens,
    all-to-all return of the per-slot outputs, slot-order combine. tokens/s = N * 2048 / (max-over-
    ranks time); efficiency_vs_n1 = the one-GPU layer's time for 2048 tokens / the expert-parallel
    time (the same tokens per GPU)."""
    import torch
    import torch.distributed as dist

    from aipu_b200 import ep
    from aipu_b200 import ops

    d = torch.device("cuda", torch.cuda.current_device())
    n = MOE_E // world
    local = _ep_local_weights(d, world, rank)
    layer = ep.ExpertParallelMoE(ep.ShardedMoeWeights(local, rank * n, MOE_E), backend=ep.CudaBackend(ops.Context(d)),
                                 dispatch="alltoall")
    x = torch.randn((M, MOE_H), device=d, generator=torch.Generator(device=d).manual_seed(9 + rank)).to(torch.bfloat16)
    for _ in range(2):
        layer(x)
    torch.cuda.synchronize()
    dist.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(reps):
        layer(x)
    e1.record()
    torch.cuda.synchronize()
    t = torch.tensor([e0.elapsed_time(e1) / reps / 1e3], device=d, dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    t = float(t.item())
    flops = 2.0 * (M * MOE_T + M) * 3 * MOE_H * MOE_F * world
    _, tf_peak, _ = peaks()
    out = {"tokens_per_rank": M, "ms_per_layer": round(t * 1e3, 3), "tokens_per_s": round(world * M / t, 1),
           "dispatch": "all-to-all (NCCL), tokens only to the ranks owning their experts",
           "tensor_tflops_total": round(flops / t / 1e12, 1),
           "per_gpu_frac_of_bf16_peak": round(flops / world / t / 1e12 / tf_peak, 4)}
    del layer, local
    torch.cuda.empty_cache()
    if rank == 0:
        t1 = _one_gpu_layer_us(d, M, reps=3)
        out["one_gpu_ms_same_tokens_per_gpu"] = round(t1 * 1e3, 3)
        out["efficiency_vs_n1"] = round(t1 / t, 4)
    dist.barrier()
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


def run_case(a):
    """Small workloads for a profiler capture (a few GB on the device at most, inputs larger than L2)."""
    import torch

    from aipu_b200 import formats as F
    from aipu_b200 import ops

    d = torch.device("cuda", 0)
    torch.cuda.set_device(0)
    if a.case in ("gemv", "chain"):
        w = F.random_rows_dev(a.wtype, a.groups * a.n * 4, a.k, seed=1, device=d)
        x = torch.randn((a.m, a.k), device=d)
        if not a.x_f32:
            x = x.to(torch.bfloat16)
        for i in range(6):
            sub = w[(i % 4) * a.groups * a.n:((i % 4) + 1) * a.groups * a.n]
            if a.case == "chain":
                y = ops.gemm(a.wtype, sub[:a.n], a.n, a.k, x, mode="strict")
            elif a.groups > 1:
                y = ops.gemm_grouped(a.wtype, sub, a.groups, a.n, a.k, x)
            else:
                y = ops.gemm(a.wtype, sub, a.n, a.k, x)
    elif a.case == "tc":
        w = F.random_rows_dev(a.wtype, a.n, a.k, seed=3, device=d)
        x = torch.randn((a.m, a.k), device=d).to(torch.bfloat16)
        for _ in range(3):
            y = ops.gemm_tc(a.wtype, w, a.n, a.k, x)
    elif a.case == "router":
        g = torch.Generator(device=d)
        w = torch.randn((MOE_H, MOE_E), device=d, generator=g.manual_seed(1)) * 0.02
        b = torch.randn((MOE_E,), device=d, generator=g.manual_seed(2)) * 0.01
        x = torch.randn((a.tokens, MOE_H), device=d, generator=g.manual_seed(3)).to(torch.bfloat16)
        for _ in range(4):
            y, _, _ = ops.moe_router(F.F32, w, x, MOE_E, MOE_T, bias=b)
    else:
        g = torch.Generator(device=d)
        E = a.experts
        W = ops.MoeLayerWeights(
            hidden=MOE_H, ffn=MOE_F, n_experts=E, topk=MOE_T, router_wtype=F.F32,
            router_w=torch.randn((MOE_H, E), device=d, generator=g.manual_seed(1)) * 0.02,
            router_bias=torch.randn((E,), device=d, generator=g.manual_seed(2)) * 0.01,
            gate_w=F.random_rows_dev(F.Q4_K, E * MOE_F, MOE_H, seed=11, device=d),
            up_w=F.random_rows_dev(F.Q4_K, E * MOE_F, MOE_H, seed=12, device=d),
            down_w=F.random_rows_dev(F.Q6_K, E * MOE_H, MOE_F, seed=13, device=d),
            shared_gate_w=F.random_rows_dev(F.Q4_K, MOE_F, MOE_H, seed=14, device=d),
            shared_up_w=F.random_rows_dev(F.Q4_K, MOE_F, MOE_H, seed=15, device=d),
            shared_down_w=F.random_rows_dev(F.Q6_K, MOE_H, MOE_F, seed=16, device=d))
        x = torch.randn((a.tokens, MOE_H), device=d, generator=g.manual_seed(3)).to(torch.bfloat16)
        for _ in range(3):
            y = ops.moe_layer(W, x)
    torch.cuda.synchronize()
    print(a.case, "ok", float(y.float().abs().mean()), flush=True)


def main():
    args = parse()
    if args.case:
        run_case(args)
        return
    if args.impl == "reference":
        run_reference(args)
        return
    import torch

    from aipu_b200 import formats as F
    from aipu_b200 import ops

    world, rank, local = dist_setup(args.gpus)
    if world > 1:
        import torch.distributed as dist
    d = torch.device("cuda", torch.cuda.current_device())
    L = args.matrices
    x_np, w_np = c1_inputs(L)
    Wt = torch.from_numpy(w_np.reshape(L * C1_N, -1)).to(d)
    x = torch.from_numpy(x_np).to(d)
    y = torch.empty((L, 1, C1_N), dtype=torch.bfloat16, device=d)
    mats = [Wt[l * C1_N:(l + 1) * C1_N] for l in range(L)]
    ctx = ops.Context(d).set_flags(pdl=True)
    s = torch.cuda.Stream()

    def issue_grouped():
        ops.gemm_grouped(F.Q4_K, Wt, L, C1_N, C1_K, x, ctx=ctx, out=y)

    def issue_single():
        for l in range(L):
            ops.gemm(F.Q4_K, mats[l], C1_N, C1_K, x, ctx=ctx, out=y[l])

    def timed(g, steps, warmup, sampler=None):
        with torch.cuda.stream(s):
            for _ in range(max(warmup, 3)):
                g.replay()
            torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        with (sampler if sampler is not None else _Null()):
            with torch.cuda.stream(s):
                torch.cuda.synchronize()
                e0.record(s)
                for _ in range(steps):
                    g.replay()
                e1.record(s)
                # wait by polling with sleeps (the clock sampler thread runs meanwhile)
                while not e1.query():
                    time.sleep(0.0002)
                torch.cuda.synchronize()
        t = e0.elapsed_time(e1) / 1e3
        if world > 1:
            tt = torch.tensor([t], device=d, dtype=torch.float64)
            dist.all_reduce(tt, op=dist.ReduceOp.MAX)
            t = float(tt.item())
        return t / steps

    g = _graph(issue_grouped, s)
    clk = ClockSampler(d.index)
    step = timed(g, args.steps, args.warmup, clk)
    value = world * L * C1_BYTES / step / 1e9
    hbm_peak, _, peak_kind = peaks()
    achieved = L * C1_BYTES / step / 1e9
    # parity of the timed kernel's outputs against the C restatement, on one matrix (checker use)
    gs = _graph(issue_single, s)
    step_single = timed(gs, max(10, args.steps // 4), args.warmup)
    single = {"us_per_launch": round(step_single / L * 1e6, 3), "gbs": round(L * C1_BYTES / step_single / 1e9, 1),
              "frac": round(L * C1_BYTES / step_single / 1e9 / hbm_peak, 4),
              "note": "one kernel launch per 4096x4096 matrix, CUDA graph, programmatic dependent launch"}
    del gs
    q6k = q6k_grouped(F, ops, ctx, s, timed, hbm_peak, rank0=(int(os.environ.get("RANK", "0")) == 0))

    # ---- end to end through the public API with host buffers (x in, all y out, every step). Steps
    # alternate between two activation and two output buffers, with the host-to-device copy of x on one
    # copy stream and the device-to-host copy of y on another, so that the copies of neighbouring
    # steps overlap the GEMVs; every step still copies its x in and all its y out.
    x_host = torch.from_numpy(x_np).pin_memory()
    y_hosts = [torch.empty((L, 1, C1_N), dtype=torch.bfloat16, pin_memory=True) for _ in range(2)]
    xs_ = [x, torch.empty_like(x)]
    ys = [y, torch.empty_like(y)]

    def issue_grouped_into(b):
        return lambda: ops.gemm_grouped(F.Q4_K, Wt, L, C1_N, C1_K, xs_[b], ctx=ctx, out=ys[b])

    gb = [_graph(issue_grouped_into(0), s), _graph(issue_grouped_into(1), s)]
    hs, ds = torch.cuda.Stream(), torch.cuda.Stream()
    ev_x = [torch.cuda.Event() for _ in range(2)]
    ev_k = [torch.cuda.Event() for _ in range(2)]
    ev_c = [torch.cuda.Event() for _ in range(2)]
    e2e_steps = max(10, args.steps // 2)

    def e2e_step(i):
        b = i & 1
        hs.wait_event(ev_k[b])  # the GEMVs two steps back have read this x buffer
        with torch.cuda.stream(hs):
            xs_[b].copy_(x_host, non_blocking=True)
            ev_x[b].record(hs)
        s.wait_event(ev_x[b])
        s.wait_event(ev_c[b])  # the copy out of this y buffer two steps back is done
        with torch.cuda.stream(s):
            gb[b].replay()
            ev_k[b].record(s)
        ds.wait_event(ev_k[b])
        with torch.cuda.stream(ds):
            y_hosts[b].copy_(ys[b], non_blocking=True)
            ev_c[b].record(ds)

    torch.cuda.synchronize()
    for i in range(4):
        e2e_step(i)
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    for i in range(e2e_steps):
        e2e_step(i)
    torch.cuda.synchronize()
    te = (time.perf_counter() - t0) / e2e_steps
    if world > 1:
        tt = torch.tensor([te], device=d, dtype=torch.float64)
        dist.all_reduce(tt, op=dist.ReduceOp.MAX)
        te = float(tt.item())
    e2e = {"value": round(world * L * C1_BYTES / te / 1e9, 2), "unit": "GB/s",
           "h2d_bytes_per_step": C1_K * 4, "d2h_bytes_per_step": L * C1_N * 2,
           "path": "ops.gemm_grouped -> aipu_q4k_gemm_grouped (C ABI), replayed as a CUDA graph; pinned host x in, "
                   "all y out, every step (double-buffered x and y, copies on their own streams overlapping the neighbouring "
                   "steps' GEMVs)"}
    y_first = y[0].clone()
    del Wt, mats, gb, ys
    torch.cuda.empty_cache()

    cpu_base = None
    if rank == 0 and world == 1 and not args.no_cpu:
        from oracle import cpu
        from oracle import q4k_oracle as qo

        cpu_base = cpu_baseline_c1(x_np, w_np)
        # checker: the timed kernel's outputs for matrix 0 against the C restatement's
        ref = cpu.gemm(F.Q4_K, w_np[0], C1_N, C1_K, x_np)
        st = qo.parity_stats(_bf16_np(y_first), ref)
        cpu_base["parity_of_timed_gemv"] = {k: (round(v, 6) if isinstance(v, float) else v) for k, v in st.items()}
    del w_np
    moe = None
    if rank == 0 and world == 1 and not args.no_moe:
        moe = moe_bench(check=not args.no_cpu)
    moe_ep = None
    moe_stream = None
    moe_pre_ep = None
    if world > 1 and not args.no_moe:
        moe_ep = moe_decode_ep(world, rank)
        try:
            moe_pre_ep = moe_prefill_ep(world, rank)
        except Exception as e:  # reported in the line; the GEMV metric above stands
            moe_pre_ep = {"error": f"{type(e).__name__}: {e}"[:300]}
        if args.stream_layers > 0:
            try:
                moe_stream = moe_decode_stream(world, rank, args.stream_layers)
            except Exception as e:  # reported in the line; the GEMV metric above stands
                moe_stream = {"error": f"{type(e).__name__}: {e}"[:300]}
    if rank == 0:
        traffic = None if C1_TRAFFIC_PER_GEMV is None else int(C1_TRAFFIC_PER_GEMV * L)
        line = {
            "metric": METRIC, "value": round(value, 2), "unit": "GB/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(step * 1e3, 4), "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": c1_config(L, world),
            "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": hbm_peak, "unit": "GB/s",
                         "frac": round(achieved / hbm_peak, 4), "traffic": traffic, "peak_source": peak_kind,
                         "kernel": "aipu_kq_gemv_kernel<Q4_K, fp32 x, store> (grouped launch)",
                         "us_per_launch": round(step * 1e6, 3),
                         "algorithmic_bytes_per_launch": L * C1_BYTES},
            "single_launch": single,
            "q6k_grouped": q6k,
            "cpu_baseline": cpu_base, "e2e": e2e, "gpu_launches": args.steps,
            "clocks": clk.summary(), "moe": moe, "moe_decode_ep": moe_ep, "moe_prefill_ep": moe_pre_ep,
            "moe_decode_stream": moe_stream,
        }
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.destroy_process_group()


if __name__ == "__main__":
    main()

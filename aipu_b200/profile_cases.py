"""Small, self-contained GPU workloads for profiling single kernels of this library.

Each case builds seeded synthetic inputs on cuda:0, runs the operation a few times and prints one
line. Sizes are chosen so that a profiler capture of one launch stays small (a few GB on the
device at most, inputs larger than L2).

    python -m aipu_b200.profile_cases gemv --wtype 0 --m 1 --groups 8
    python -m aipu_b200.profile_cases tc --wtype 1 --n 49152 --k 2048 --m 64
    python -m aipu_b200.profile_cases moe --experts 64 --tokens 512
    python -m aipu_b200.profile_cases router --tokens 1
"""
from __future__ import annotations

import argparse

import torch

from . import formats as F
from . import ops


def case_gemv(wtype: int, m: int, groups: int, n: int = 2048, k: int = 6144) -> None:
    d = torch.device("cuda", 0)
    w = F.random_rows_dev(wtype, groups * n * 4, k, seed=1, device=d)
    x = torch.randn((m, k), device=d).to(torch.bfloat16)
    for i in range(6):
        sub = w[(i % 4) * groups * n:((i % 4) + 1) * groups * n]
        y = ops.gemm_grouped(wtype, sub, groups, n, k, x) if groups > 1 else ops.gemm(wtype, sub, n, k, x)
    torch.cuda.synchronize()
    print("gemv ok", float(y.float().abs().mean()))


def case_tc(wtype: int, n: int, k: int, m: int) -> None:
    d = torch.device("cuda", 0)
    w = F.random_rows_dev(wtype, n, k, seed=3, device=d)
    x = torch.randn((m, k), device=d).to(torch.bfloat16)
    for _ in range(3):
        y = ops.gemm_tc(wtype, w, n, k, x)
    torch.cuda.synchronize()
    print("tc ok", float(y.float().abs().mean()))


def case_moe(experts: int, tokens: int, hidden: int = 6144, ffn: int = 2048, topk: int = 8) -> None:
    d = torch.device("cuda", 0)
    g = torch.Generator(device=d)
    W = ops.MoeLayerWeights(
        hidden=hidden, ffn=ffn, n_experts=experts, topk=topk, router_wtype=F.F32,
        router_w=torch.randn((hidden, experts), device=d, generator=g.manual_seed(1)) * 0.02,
        router_bias=torch.randn((experts,), device=d, generator=g.manual_seed(2)) * 0.01,
        gate_w=F.random_rows_dev(F.Q4_K, experts * ffn, hidden, seed=11, device=d),
        up_w=F.random_rows_dev(F.Q4_K, experts * ffn, hidden, seed=12, device=d),
        down_w=F.random_rows_dev(F.Q6_K, experts * hidden, ffn, seed=13, device=d),
        shared_gate_w=F.random_rows_dev(F.Q4_K, ffn, hidden, seed=14, device=d),
        shared_up_w=F.random_rows_dev(F.Q4_K, ffn, hidden, seed=15, device=d),
        shared_down_w=F.random_rows_dev(F.Q6_K, hidden, ffn, seed=16, device=d))
    x = torch.randn((tokens, hidden), device=d, generator=g.manual_seed(3)).to(torch.bfloat16)
    for _ in range(3):
        y = ops.moe_layer(W, x)
    torch.cuda.synchronize()
    print("moe ok", float(y.float().abs().mean()))


def case_router(tokens: int, hidden: int = 6144, experts: int = 256, topk: int = 8) -> None:
    d = torch.device("cuda", 0)
    g = torch.Generator(device=d)
    w = torch.randn((hidden, experts), device=d, generator=g.manual_seed(1)) * 0.02
    b = torch.randn((experts,), device=d, generator=g.manual_seed(2)) * 0.01
    x = torch.randn((tokens, hidden), device=d, generator=g.manual_seed(3)).to(torch.bfloat16)
    for _ in range(4):
        sel, _, _ = ops.moe_router(F.F32, w, x, experts, topk, bias=b)
    torch.cuda.synchronize()
    print("router ok", int(sel.sum()))


def main() -> None:
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    sub = ap.add_subparsers(dest="case", required=True)
    a = sub.add_parser("gemv")
    a.add_argument("--wtype", type=int, default=F.Q4_K)
    a.add_argument("--m", type=int, default=1)
    a.add_argument("--groups", type=int, default=8)
    a.add_argument("--n", type=int, default=2048)
    a.add_argument("--k", type=int, default=6144)
    a = sub.add_parser("tc")
    a.add_argument("--wtype", type=int, default=F.Q4_K)
    a.add_argument("--n", type=int, default=32768)
    a.add_argument("--k", type=int, default=6144)
    a.add_argument("--m", type=int, default=128)
    a = sub.add_parser("moe")
    a.add_argument("--experts", type=int, default=64)
    a.add_argument("--tokens", type=int, default=512)
    a = sub.add_parser("router")
    a.add_argument("--tokens", type=int, default=1)
    args = ap.parse_args()
    if args.case == "gemv":
        case_gemv(args.wtype, args.m, args.groups, args.n, args.k)
    elif args.case == "tc":
        case_tc(args.wtype, args.n, args.k, args.m)
    elif args.case == "router":
        case_router(args.tokens)
    else:
        case_moe(args.experts, args.tokens)


if __name__ == "__main__":
    main()

"""Expert-parallel pieces on the GPU: aipu_moe_experts + aipu_moe_combine.

* one GPU: G shards emulated in one process (each shard's experts on the same gathered tokens,
  the all-to-all done by indexing), checked bit for bit against the one-GPU layer in strict mode and
  within the reference SwiGLU tolerance against the oracle in fast mode, for few tokens (grouped
  GEMV) and many (tcgen05);
* two GPUs (skipped with fewer): ExpertParallelMoE over NCCL and PeerExpertParallelMoE over NVLink
  peer memory in child processes, strict mode bit for bit against the one-GPU layer.
"""
import os
import socket

import numpy as np
import pytest
import torch

from aipu_b200 import formats as F
from aipu_b200 import ops
from oracle import moe_oracle as mo
from oracle import q4k_oracle as qo

pytestmark = pytest.mark.gpu
F32 = np.float32


def _bf16_np(t):
    return (t.view(torch.int16).cpu().numpy().astype(np.uint16).astype(np.uint32) << 16).view(F32)


def _layer(d, H, Fd, E, T, seed):
    rng = np.random.default_rng(seed)
    return ops.MoeLayerWeights(
        hidden=H, ffn=Fd, n_experts=E, topk=T, router_wtype=F.F32,
        router_w=torch.from_numpy(rng.normal(0, 0.02, (H, E)).astype(F32)).to(d),
        router_bias=torch.from_numpy(rng.normal(0, 0.01, E).astype(F32)).to(d),
        gate_w=F.random_rows_dev(F.Q4_K, E * Fd, H, seed=seed + 1, device=d),
        up_w=F.random_rows_dev(F.Q4_K, E * Fd, H, seed=seed + 2, device=d),
        down_w=F.random_rows_dev(F.Q6_K, E * H, Fd, seed=seed + 3, device=d),
        shared_gate_w=F.random_rows_dev(F.Q4_K, Fd, H, seed=seed + 4, device=d),
        shared_up_w=F.random_rows_dev(F.Q4_K, Fd, H, seed=seed + 5, device=d),
        shared_down_w=F.random_rows_dev(F.Q6_K, H, Fd, seed=seed + 6, device=d))


def _emulated_ep(W, xs, G, ctx):
    """xs: per-rank token batches [M, H] (bf16 device). Returns per-rank outputs."""
    M = xs[0].shape[0]
    n = W.n_experts // G
    routes = [ops.moe_router(W.router_wtype, W.router_w, x, W.n_experts, W.topk, bias=W.router_bias, ctx=ctx)[:2]
              for x in xs]
    x_all = torch.cat(xs)
    sel_all = torch.cat([r[0] for r in routes])
    y_by_rank, ysh_by_rank = [], []
    for r in range(G):
        y_slots, y_sh = ops.moe_experts(ops.expert_slice(W, r * n, n), r * n, x_all, sel_all,
                                        shared_range=(r * M, M), ctx=ctx)
        y_by_rank.append(y_slots.view(G, M, W.topk, W.hidden))
        ysh_by_rank.append(y_sh)
    outs = []
    for q in range(G):  # all-to-all: rank q receives rows [q*M, (q+1)*M) of every rank's y_slots
        pieces = torch.stack([y_by_rank[r][q] for r in range(G)])
        outs.append(ops.moe_combine(routes[q][0], routes[q][1], n, pieces, ysh_by_rank[q], ctx=ctx))
    return outs


@pytest.mark.parametrize("M,H,Fd,E,G", [(2, 6144, 2048, 256, 4), (40, 512, 256, 16, 2), (96, 512, 256, 16, 2)])
def test_expert_parallel_emulated_strict_matches_one_gpu(M, H, Fd, E, G):
    d = torch.device("cuda", 0)
    W = _layer(d, H, Fd, E, 8, seed=100 + M)
    ctx = ops.Context(d).set_flags(strict=True)
    rng = np.random.default_rng(M)
    xs = [torch.from_numpy(qo.bf16_round(rng.standard_normal((M, H)).astype(F32))).to(d).to(torch.bfloat16)
          for _ in range(G)]
    outs = _emulated_ep(W, xs, G, ctx)
    for q in range(G):
        ref = ops.moe_layer(W, xs[q], ctx=ctx)
        torch.cuda.synchronize()
        assert torch.equal(outs[q].view(torch.int16), ref.view(torch.int16)), f"rank {q}"


@pytest.mark.parametrize("M", [4, 96])
def test_expert_parallel_emulated_fast_within_reference_tolerance(M):
    """Fast mode (grouped GEMV for 4 tokens, tcgen05 for 2 x 96 gathered tokens) against the oracle."""
    d = torch.device("cuda", 0)
    H, Fd, E, G, T = 512, 256, 16, 2, 8
    W = _layer(d, H, Fd, E, T, seed=7)
    ctx = ops.Context(d)
    rng = np.random.default_rng(3 + M)
    xn = [qo.bf16_round(rng.standard_normal((M, H)).astype(F32)) for _ in range(G)]
    xs = [torch.from_numpy(a).to(d).to(torch.bfloat16) for a in xn]
    outs = _emulated_ep(W, xs, G, ctx)
    torch.cuda.synchronize()
    gv, uv, dv = (W.gate_w.view(E, Fd, -1).cpu().numpy(), W.up_w.view(E, Fd, -1).cpu().numpy(),
                  W.down_w.view(E, H, -1).cpu().numpy())

    def deq(e):
        return (qo.dequant_rows(F.Q4_K, gv[e], Fd, H), qo.dequant_rows(F.Q4_K, uv[e], Fd, H),
                qo.dequant_rows(F.Q6_K, dv[e], H, Fd))

    shared = (qo.dequant_rows(F.Q4_K, W.shared_gate_w.cpu().numpy(), Fd, H),
              qo.dequant_rows(F.Q4_K, W.shared_up_w.cpu().numpy(), Fd, H),
              qo.dequant_rows(F.Q6_K, W.shared_down_w.cpu().numpy(), H, Fd))
    wr_t = W.router_w.cpu().numpy().T.copy()
    for q in range(G):
        ref, _, _, mag = mo.moe_layer(xn[q], wr_t, deq, shared, T, bias=W.router_bias.cpu().numpy(), want_mag=True)
        got = _bf16_np(outs[q]).astype(np.float64)
        tol = np.maximum(np.maximum(0.06 * np.abs(ref), 0.02 * mag), 0.03)
        assert not (np.abs(got - ref) > tol).any()


def _nccl_worker(rank, world, port, q, dispatch="allgather"):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    import torch.distributed as dist

    from aipu_b200 import ep
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=torch.device("cuda", rank))
    try:
        d = torch.device("cuda", rank)
        W = _layer(d, 6144, 2048, 256, 8, seed=55)
        ctx = ops.Context(d).set_flags(strict=True)
        rng = np.random.default_rng(1000 + rank)
        x = torch.from_numpy(qo.bf16_round(rng.standard_normal((3, 6144)).astype(F32))).to(d).to(torch.bfloat16)
        layer = ep.ExpertParallelMoE(ep.shard(W, rank, world), backend=ep.CudaBackend(ctx), dispatch=dispatch)
        out = layer(x)
        ref = ops.moe_layer(W, x, ctx=ctx)
        torch.cuda.synchronize()
        q.put((rank, bool(torch.equal(out.view(torch.int16), ref.view(torch.int16)))))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("dispatch", ["allgather", "alltoall"])
def test_expert_parallel_two_gpus_nccl_strict(dispatch):
    """NCCL expert parallelism on 2 GPUs equals the one-GPU layer bit for bit, with the all-gather
    dispatch and with the all-to-all dispatch (tokens only to the ranks that own their experts)."""
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    procs = [ctx.Process(target=_nccl_worker, args=(r, 2, port, q, dispatch)) for r in range(2)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=600) for _ in procs)
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    assert res == {0: True, 1: True}


def _p2p_worker(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    import torch.distributed as dist

    from aipu_b200 import ep
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=torch.device("cuda", rank))
    res = {}
    try:
        d = torch.device("cuda", rank)
        W = _layer(d, 6144, 2048, 256, 8, seed=77)
        for strict in (True, False):
            ctx = ops.Context(d).set_flags(strict=strict)
            layer = ep.PeerExpertParallelMoE(ep.shard(W, rank, world), max_tokens=4, ctx=ctx)
            ok = True
            for call, M in enumerate((3, 1, 4)):  # several calls: the flags advance per call
                rng = np.random.default_rng(2000 + 10 * rank + call)
                x = torch.from_numpy(qo.bf16_round(rng.standard_normal((M, 6144)).astype(F32))).to(d).to(torch.bfloat16)
                out = layer(x)
                ref = ops.moe_layer(W, x, ctx=ctx)
                torch.cuda.synchronize()
                if strict:
                    ok = ok and bool(torch.equal(out.view(torch.int16), ref.view(torch.int16)))
                else:
                    ud = qo.ulp_diff_bf16(_bf16_np(out), _bf16_np(ref))
                    ok = ok and float(np.mean(ud <= 1)) >= 0.99
            assert ctx.status() == 0
            layer.close()
            res["strict" if strict else "fast"] = ok
        q.put((rank, res))
    finally:
        dist.destroy_process_group()


def test_expert_parallel_two_gpus_peer_memory():
    """The NVLink peer-memory exchange: strict mode equals the one-GPU layer bit for bit, fast mode
    within 1 ulp of it on >= 99 % of outputs, over several calls."""
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    procs = [ctx.Process(target=_p2p_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=600) for _ in procs)
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    assert res == {0: {"strict": True, "fast": True}, 1: {"strict": True, "fast": True}}


def _stream_worker(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    import torch.distributed as dist

    from aipu_b200 import ep
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=torch.device("cuda", rank))
    res = {}
    try:
        d = torch.device("cuda", rank)
        Ws = [_layer(d, 512, 256, 16, 4, seed=300 + 10 * l) for l in range(3)]
        ctx = ops.Context(d).set_flags(strict=True)
        rng = np.random.default_rng(4000 + rank)
        x = torch.from_numpy(qo.bf16_round(rng.standard_normal((2, 512)).astype(F32))).to(d).to(torch.bfloat16)
        ref = x
        for W in Ws:
            ref = ops.moe_layer(W, ref, ctx=ctx)
        for kind in ("peer", "nccl"):
            stream = ep.DecodeStream([ep.shard(W, rank, world) for W in Ws], exchange=kind, max_tokens=2, ctx=ctx,
                                     backend=ep.CudaBackend(ctx))
            out = stream(x)
            out2 = stream(x)  # a second call through the same exchange state
            torch.cuda.synchronize()
            res[kind] = bool(torch.equal(out.view(torch.int16), ref.view(torch.int16))) and \
                bool(torch.equal(out2.view(torch.int16), ref.view(torch.int16)))
            stream.close()
        res["status"] = ctx.status()
        q.put((rank, res))
    finally:
        dist.destroy_process_group()


def test_decode_stream_two_gpus_strict():
    """Three expert-parallel layers back to back, over the peer exchange and over NCCL, equal the
    one-GPU layers applied in turn (strict mode, bit for bit), on two successive calls."""
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    procs = [ctx.Process(target=_stream_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=600) for _ in procs)
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    assert res == {0: {"peer": True, "nccl": True, "status": 0}, 1: {"peer": True, "nccl": True, "status": 0}}

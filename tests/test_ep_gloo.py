"""Expert-parallel MoE orchestration (aipu_b200.ep) on CPU: two gloo ranks, the compute steps
restated by the oracle, checked bit for bit against the one-process oracle layer. This covers the
dispatch (all-gather), the expert sharding, the all-to-all return and the slot-order combine."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from aipu_b200 import ep
from aipu_b200 import formats as F
from aipu_b200 import ops
from oracle import moe_oracle as mo
from oracle import q4k_oracle as qo

F32 = np.float32
H, FD, E, T, M = 256, 256, 4, 2, 3


def _bf16_t(a):
    return torch.from_numpy((np.asarray(a, F32).view(np.uint32) >> 16).astype(np.uint16).view(np.int16)).view(
        torch.bfloat16)


def _np(t):
    return (t.view(torch.int16).numpy().astype(np.uint16).astype(np.uint32) << 16).view(F32)


class OracleBackend:
    """Host restatement of the three compute steps (test double for the CUDA backend)."""

    def route(self, R, x):
        sel, sw, _ = mo.moe_router(_np(x), R.router_w.numpy().view(F32).reshape(H, -1).T.copy(), R.topk,
                                   None if R.router_bias is None else R.router_bias.numpy(), R.scale)
        return torch.from_numpy(sel.astype(np.int32)), _bf16_t(sw)

    def experts(self, W, lo, x, sel, shared_range):
        xs, s = _np(x), sel.numpy()
        n = W.n_experts
        y = np.zeros((xs.shape[0], W.topk, H), F32)
        g = W.gate_w.numpy().reshape(n, FD, -1)
        u = W.up_w.numpy().reshape(n, FD, -1)
        d = W.down_w.numpy().reshape(n, H, -1)
        for m in range(xs.shape[0]):
            for k in range(W.topk):
                le = int(s[m, k]) - lo
                if 0 <= le < n:
                    hh = mo.swiglu_hidden(xs[m:m + 1], qo.dequant_rows(F.Q4_K, g[le], FD, H),
                                          qo.dequant_rows(F.Q4_K, u[le], FD, H))
                    y[m, k] = qo.matmul_seq(hh, qo.dequant_rows(F.Q6_K, d[le], H, FD))[0]
        t0, cnt = shared_range
        hh = mo.swiglu_hidden(xs[t0:t0 + cnt], qo.dequant_rows(F.Q4_K, W.shared_gate_w.numpy(), FD, H),
                              qo.dequant_rows(F.Q4_K, W.shared_up_w.numpy(), FD, H))
        ysh = qo.matmul_seq(hh, qo.dequant_rows(F.Q6_K, W.shared_down_w.numpy(), H, FD))
        return _bf16_t(y), _bf16_t(ysh)

    def combine(self, sel, sw, epp, pieces, y_sh):
        s, w, p = sel.numpy(), _np(sw), _np(pieces)
        Mloc = s.shape[0]
        y_slots = np.stack([np.stack([p[int(s[m, k]) // epp, m, k] for k in range(s.shape[1])]) for m in range(Mloc)])
        return _bf16_t(mo.combine(w, y_slots, _np(y_sh)))


def _weights(seed):
    rng = np.random.default_rng(seed)
    W = ops.MoeLayerWeights(
        hidden=H, ffn=FD, n_experts=E, topk=T, router_wtype=F.F32,
        router_w=torch.from_numpy(rng.normal(0, 0.05, (H, E)).astype(F32).view(np.uint8).reshape(-1)),
        router_bias=torch.from_numpy(rng.normal(0, 0.01, E).astype(F32)),
        gate_w=torch.from_numpy(F.random_rows_np(F.Q4_K, E * FD, H, seed=seed + 1)),
        up_w=torch.from_numpy(F.random_rows_np(F.Q4_K, E * FD, H, seed=seed + 2)),
        down_w=torch.from_numpy(F.random_rows_np(F.Q6_K, E * H, FD, seed=seed + 3)),
        shared_gate_w=torch.from_numpy(F.random_rows_np(F.Q4_K, FD, H, seed=seed + 4)),
        shared_up_w=torch.from_numpy(F.random_rows_np(F.Q4_K, FD, H, seed=seed + 5)),
        shared_down_w=torch.from_numpy(F.random_rows_np(F.Q6_K, H, FD, seed=seed + 6)))
    xs = [qo.bf16_round(rng.standard_normal((M, H)).astype(F32)) for _ in range(2)]
    return W, xs


def _worker(rank, world, port, q, dispatch="allgather"):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        W, xs = _weights(7)
        layer = ep.ExpertParallelMoE(ep.shard(W, rank, world), backend=OracleBackend(), dispatch=dispatch)
        out = layer(_bf16_t(xs[rank]))
        q.put((rank, _np(out)))
    finally:
        dist.destroy_process_group()


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.parametrize("dispatch", ["allgather", "alltoall"])
def test_expert_parallel_two_gloo_ranks_match_one_process_layer(dispatch):
    """Both dispatches: all-gather of every token, and all-to-all of each token to the ranks owning its
    experts with only the local slots' outputs returned."""
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q, dispatch)) for r in range(2)]
    for p in procs:
        p.start()
    got = dict(q.get(timeout=240) for _ in procs)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    W, xs = _weights(7)
    wr_t = W.router_w.numpy().view(F32).reshape(H, E).T.copy()
    gv, uv, dv = W.gate_w.numpy().reshape(E, FD, -1), W.up_w.numpy().reshape(E, FD, -1), W.down_w.numpy().reshape(E, H, -1)

    def deq(e):
        return (qo.dequant_rows(F.Q4_K, gv[e], FD, H), qo.dequant_rows(F.Q4_K, uv[e], FD, H),
                qo.dequant_rows(F.Q6_K, dv[e], H, FD))

    shared = (qo.dequant_rows(F.Q4_K, W.shared_gate_w.numpy(), FD, H),
              qo.dequant_rows(F.Q4_K, W.shared_up_w.numpy(), FD, H),
              qo.dequant_rows(F.Q6_K, W.shared_down_w.numpy(), H, FD))
    for r in range(2):
        ref, _, _ = mo.moe_layer(xs[r], wr_t, deq, shared, T, bias=W.router_bias.numpy())
        assert np.array_equal(got[r].view(np.uint32), ref.view(np.uint32)), f"rank {r}"


def _stream_worker(rank, world, port, q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        Ws = [_weights(7 + 10 * l)[0] for l in range(3)]
        _, xs = _weights(7)
        stream = ep.DecodeStream([ep.shard(W, rank, world) for W in Ws], exchange="nccl", backend=OracleBackend())
        out = stream(_bf16_t(xs[rank]))
        q.put((rank, _np(out)))
    finally:
        dist.destroy_process_group()


def test_decode_stream_two_gloo_ranks_three_layers():
    """Three expert-parallel layers back to back (each layer's output is the next one's input)
    equal the one-process oracle layers applied in turn."""
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_stream_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    got = dict(q.get(timeout=240) for _ in procs)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    Ws = [_weights(7 + 10 * l)[0] for l in range(3)]
    _, xs = _weights(7)
    for r in range(2):
        x = xs[r]
        for W in Ws:
            wr_t = W.router_w.numpy().view(F32).reshape(H, E).T.copy()
            gv, uv, dv = (W.gate_w.numpy().reshape(E, FD, -1), W.up_w.numpy().reshape(E, FD, -1),
                          W.down_w.numpy().reshape(E, H, -1))

            def deq(e, gv=gv, uv=uv, dv=dv):
                return (qo.dequant_rows(F.Q4_K, gv[e], FD, H), qo.dequant_rows(F.Q4_K, uv[e], FD, H),
                        qo.dequant_rows(F.Q6_K, dv[e], H, FD))

            shared = (qo.dequant_rows(F.Q4_K, W.shared_gate_w.numpy(), FD, H),
                      qo.dequant_rows(F.Q4_K, W.shared_up_w.numpy(), FD, H),
                      qo.dequant_rows(F.Q6_K, W.shared_down_w.numpy(), H, FD))
            x, _, _ = mo.moe_layer(x, wr_t, deq, shared, T, bias=W.router_bias.numpy())
        assert np.array_equal(got[r].view(np.uint32), x.view(np.uint32)), f"rank {r}"


def test_decode_stream_rejects_mismatched_layers():
    W1, _ = _weights(7)
    W2, _ = _weights(8)
    W2.topk = 1
    with pytest.raises(ValueError):
        ep.DecodeStream([ep.shard(W1, 0, 2), ep.shard(W2, 0, 2)], exchange="nccl")
    with pytest.raises(ValueError):
        ep.DecodeStream([], exchange="nccl")

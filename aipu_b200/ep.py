"""Expert-parallel MoE layer: the routed experts sharded over the ranks of a process group (one
process per GPU, NCCL over NVLink), the router and the shared expert replicated.

One layer call on every rank, for that rank's M tokens (the same M on every rank):

  1. route the local tokens (bit-exact router kernel);
  2. dispatch: all-gather the tokens and their selections (G*M rows);
  3. each rank runs its experts [r*E/G, (r+1)*E/G) on every gathered token that selected one of them
     (aipu_moe_experts: the grouped GEMV for few tokens, the tcgen05 path for many) and the shared
     expert on its own tokens;
  4. combine: an all-to-all returns to each owner the per-slot expert outputs of its tokens, and the
     owner combines them in slot order (aipu_moe_combine), the reference's order, so the result is
     the one-GPU layer's.

The compute steps go through ``backend`` (the CUDA library by default); the communication uses
torch.distributed, so the same orchestration runs with the gloo backend on CPU in tests, with a
host backend that restates the compute. ``PeerExpertParallelMoE`` is the same layer with the
exchange done inside the library over NVLink peer memory (decode sizes).
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass
from typing import Optional, Sequence

import torch
import torch.distributed as dist

from . import _lib as L
from . import ops


class CudaBackend:
    """The library's kernels on the current CUDA device."""

    def __init__(self, ctx: Optional[ops.Context] = None):
        self.ctx = ctx

    def route(self, W: ops.MoeLayerWeights, x: torch.Tensor):
        sel, sw, _ = ops.moe_router(W.router_wtype, W.router_w, x, W.n_experts_total, W.topk, bias=W.router_bias,
                                    scale=W.scale, ctx=self.ctx)
        return sel, sw

    def experts(self, W_local: ops.MoeLayerWeights, expert_lo: int, x: torch.Tensor, sel: torch.Tensor,
                shared_range: tuple):
        return ops.moe_experts(W_local, expert_lo, x, sel, shared_range=shared_range, ctx=self.ctx)

    def combine(self, sel, sel_w, experts_per_piece, pieces, y_shared):
        return ops.moe_combine(sel, sel_w, experts_per_piece, pieces, y_shared, ctx=self.ctx)


@dataclass
class ShardedMoeWeights:
    """Routed experts [expert_lo, expert_lo + local.n_experts) of an E-expert layer, plus the
    replicated router and shared expert (held in ``local``)."""
    local: ops.MoeLayerWeights
    expert_lo: int
    n_experts_total: int

    @property
    def topk(self):
        return self.local.topk

    @property
    def hidden(self):
        return self.local.hidden


def shard(W: ops.MoeLayerWeights, rank: int, world: int) -> ShardedMoeWeights:
    """Rank ``rank``'s share of a full layer (views of W's expert tensors)."""
    if W.n_experts % world:
        raise ValueError("experts must divide evenly over the ranks")
    n = W.n_experts // world
    return ShardedMoeWeights(ops.expert_slice(W, rank * n, n), rank * n, W.n_experts)


class _RouterView:
    """The router fields of a sharded layer, with the global expert count."""

    def __init__(self, S: ShardedMoeWeights):
        L = S.local
        self.router_wtype, self.router_w, self.router_bias = L.router_wtype, L.router_w, L.router_bias
        self.n_experts_total, self.topk, self.scale = S.n_experts_total, L.topk, L.scale


class ExpertParallelMoE:
    """The MoE branch of a decoder block with experts sharded over ``group`` (default: WORLD).

    dispatch: "allgather" -- every rank receives every token and its selections (fixed sizes, so a
    CUDA graph can capture the layer; the decode path); "alltoall" -- each token goes only to the
    ranks that own one of its experts, and only the per-slot outputs of those experts come back
    (variable sizes: the per-peer counts are exchanged first; the prefill path); "auto" -- all-to-all
    from ``a2a_min_tokens`` tokens per rank."""

    def __init__(self, weights: ShardedMoeWeights, group=None, backend=None, dispatch: str = "auto",
                 a2a_min_tokens: int = 64):
        self.W = weights
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        if weights.n_experts_total != weights.local.n_experts * self.world:
            raise ValueError("every rank must hold n_experts_total / world experts")
        if dispatch not in ("auto", "allgather", "alltoall"):
            raise ValueError("dispatch must be 'auto', 'allgather' or 'alltoall'")
        self.backend = backend or CudaBackend()
        self.router = _RouterView(weights)
        self.dispatch = dispatch
        self.a2a_min_tokens = a2a_min_tokens

    def __call__(self, x: torch.Tensor) -> torch.Tensor:
        M = x.shape[0]
        use_a2a = self.world > 1 and (self.dispatch == "alltoall" or
                                      (self.dispatch == "auto" and M >= self.a2a_min_tokens))
        sel, sw = self.backend.route(self.router, x)
        return self._alltoall(x, sel, sw) if use_a2a else self._allgather(x, sel, sw)

    def _allgather(self, x, sel, sw):
        W, G, r = self.W, self.world, self.rank
        M, H = x.shape
        T = W.topk
        # dispatch: every rank sees every token and its selection
        x_all = torch.empty((G * M, H), dtype=x.dtype, device=x.device)
        sel_all = torch.empty((G * M, T), dtype=sel.dtype, device=sel.device)
        dist.all_gather_into_tensor(x_all, x.contiguous(), group=self.group)
        dist.all_gather_into_tensor(sel_all, sel.contiguous(), group=self.group)
        # local experts on all tokens, shared expert on this rank's tokens
        y_slots, y_sh = self.backend.experts(W.local, W.expert_lo, x_all, sel_all, (r * M, M))
        # combine: rows [q*M, (q+1)*M) of y_slots go back to rank q
        pieces = torch.empty((G, M, T, H), dtype=y_slots.dtype, device=y_slots.device)
        dist.all_to_all_single(pieces.view(G * M, T, H), y_slots.contiguous(), group=self.group)
        return self.backend.combine(sel, sw, W.local.n_experts, pieces, y_sh)

    def _alltoall(self, x, sel, sw):
        W, G, r = self.W, self.world, self.rank
        M, H = x.shape
        T = W.topk
        n = W.local.n_experts
        dev = x.device
        owner = (sel.long() // n).clamp_(0, G - 1)                        # [M, T]
        # tokens for each destination rank, ascending token order within a destination
        need = torch.zeros((G, M), dtype=torch.bool, device=dev)
        need[owner.reshape(-1), torch.arange(M, device=dev).repeat_interleave(T)] = True
        send_tok = [torch.nonzero(need[q]).reshape(-1) for q in range(G)]
        send_counts = torch.tensor([int(t.numel()) for t in send_tok], dtype=torch.int64)
        recv_counts = torch.empty_like(send_counts)
        c_dev = send_counts.to(dev)
        rc_dev = torch.empty_like(c_dev)
        dist.all_to_all_single(rc_dev, c_dev, group=self.group)
        recv_counts = rc_dev.cpu()
        idx = torch.cat(send_tok)
        sc, rcv = send_counts.tolist(), recv_counts.tolist()
        Mr = sum(rcv)
        x_recv = torch.empty((Mr, H), dtype=x.dtype, device=dev)
        sel_recv = torch.empty((Mr, T), dtype=sel.dtype, device=dev)
        dist.all_to_all_single(x_recv, x.index_select(0, idx).contiguous(), rcv, sc, group=self.group)
        dist.all_to_all_single(sel_recv, sel.index_select(0, idx).contiguous(), rcv, sc, group=self.group)
        # local experts on the received tokens; this rank's own tokens ride along only for the shared
        # expert (their selections pointed at another rank's experts, so no routed work is done)
        other = (W.expert_lo + n) % W.n_experts_total
        x_cat = torch.cat([x_recv, x])
        sel_cat = torch.cat([sel_recv, torch.full_like(sel, other)])
        y_slots, y_sh = self.backend.experts(W.local, W.expert_lo, x_cat, sel_cat, (Mr, M))
        # return the outputs of the local slots only, (token, slot) order per source rank
        local = (sel_recv.long() // n) == r                               # [Mr, T]
        rows = y_slots[:Mr][local]                                        # [P_r, H]
        per_src = local.sum(dim=1)
        ret_send = [int(c.sum()) for c in torch.split(per_src, rcv)]
        ret_recv = [int(v) for v in (owner == torch.arange(G, device=dev).view(G, 1, 1)).reshape(G, -1).sum(1).tolist()]
        back = torch.empty((sum(ret_recv), H), dtype=y_slots.dtype, device=dev)
        dist.all_to_all_single(back, rows.contiguous(), ret_recv, ret_send, group=self.group)
        # pieces[q][m, s] = the output of expert sel[m, s] when its owner is q
        pieces = torch.zeros((G, M, T, H), dtype=y_slots.dtype, device=dev)
        off = 0
        for q in range(G):
            mask = owner == q
            cnt = ret_recv[q]
            if cnt:
                pieces[q][mask] = back[off:off + cnt]
            off += cnt
        return self.backend.combine(sel, sw, n, pieces, y_sh)


class PeerExpertParallelMoE:
    """The same layer with the exchange done by the library over NVLink peer memory (CUDA IPC):
    tokens and selections are stored straight into every peer's inbox and the per-slot expert outputs
    straight into each owner's outbox, with sequence-numbered flags (bounded device waits) instead of
    NCCL collectives. Decode sizes: at most ``max_tokens`` (<= 64) tokens per rank and call; every
    rank calls with the same number of tokens. torch.distributed is used once, to exchange the IPC
    handles."""

    def __init__(self, weights: ShardedMoeWeights, max_tokens: int = 8, group=None, ctx: Optional[ops.Context] = None):
        self.W = weights
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        if weights.n_experts_total != weights.local.n_experts * self.world:
            raise ValueError("every rank must hold n_experts_total / world experts")
        if weights.expert_lo != self.rank * weights.local.n_experts:
            raise ValueError("rank r must hold experts [r * E_local, (r + 1) * E_local)")
        d = torch.device("cuda", torch.cuda.current_device())
        self.ctx = ctx or ops.Context(d)
        self._cs = weights.local.cstruct()
        self._cs.n_experts = weights.local.n_experts
        h = ctypes.create_string_buffer(64)
        ep = ctypes.c_void_p()
        L.check(L.lib().aipu_ep_create(self.ctx.handle, self.world, self.rank, max_tokens, weights.hidden,
                                       weights.topk, ctypes.byref(ep), h))
        self._ep = ep
        mine = torch.frombuffer(bytearray(h.raw), dtype=torch.uint8).to(d)
        allh = torch.empty((self.world, 64), dtype=torch.uint8, device=d)
        dist.all_gather_into_tensor(allh, mine, group=group)
        handles = allh.cpu().numpy().tobytes()
        L.check(L.lib().aipu_ep_connect(self._ep, handles))
        dist.barrier(group=group)

    def __call__(self, x: torch.Tensor, out: Optional[torch.Tensor] = None) -> torch.Tensor:
        if x.dtype != torch.bfloat16 or not x.is_cuda:
            raise ValueError("tokens must be bf16 on the GPU")
        M = x.shape[0]
        if out is None:
            out = torch.empty((M, self.W.hidden), dtype=torch.bfloat16, device=x.device)
        L.check(L.lib().aipu_ep_moe_layer(self._ep, ctypes.byref(self._cs), self.W.expert_lo, x.data_ptr(), M,
                                          out.data_ptr(), torch.cuda.current_stream(x.device).cuda_stream))
        return out

    def close(self):
        if self._ep:
            L.lib().aipu_ep_destroy(self._ep)
            self._ep = None


class DecodeStream:
    """Full-depth expert-parallel decode: L MoE layers run back to back for this rank's M tokens, the
    output of layer l feeding layer l + 1 (the MoE branch of every decoder block; the attention and
    norms between blocks are outside this library's path).

    ``layers``: one ShardedMoeWeights per layer (same hidden size, top-k and expert split on every
    layer). ``exchange``: "peer" (one NVLink peer-memory exchange buffer shared by all layers, like
    PeerExpertParallelMoE) or "nccl" (ExpertParallelMoE per layer). Every rank calls with the same M.
    """

    def __init__(self, layers: Sequence[ShardedMoeWeights], exchange: str = "peer", max_tokens: int = 8,
                 group=None, ctx: Optional[ops.Context] = None, backend=None):
        if not layers:
            raise ValueError("a decode stream needs at least one layer")
        H, T = layers[0].hidden, layers[0].topk
        for S in layers:
            if S.hidden != H or S.topk != T or S.n_experts_total != layers[0].n_experts_total \
                    or S.expert_lo != layers[0].expert_lo or S.local.n_experts != layers[0].local.n_experts:
                raise ValueError("all layers of a decode stream must share hidden size, top-k and expert split")
        self.layers = list(layers)
        self.exchange = exchange
        self.hidden = H
        self._bufs = {}
        if exchange == "peer":
            self._peer = PeerExpertParallelMoE(self.layers[0], max_tokens=max_tokens, group=group, ctx=ctx)
            self._cs = []
            for S in self.layers:
                cs = S.local.cstruct()
                cs.n_experts = S.local.n_experts
                self._cs.append(cs)
        elif exchange == "nccl":
            self._peer = None
            self._nccl = [ExpertParallelMoE(S, group=group, backend=backend) for S in self.layers]
        else:
            raise ValueError("exchange must be 'peer' or 'nccl'")

    def _pingpong(self, x: torch.Tensor):
        key = (x.shape[0], x.device)
        if key not in self._bufs:
            self._bufs[key] = [torch.empty((x.shape[0], self.hidden), dtype=torch.bfloat16, device=x.device)
                               for _ in range(2)]
        return self._bufs[key]

    def __call__(self, x: torch.Tensor, out: Optional[torch.Tensor] = None) -> torch.Tensor:
        if self.exchange == "nccl":
            for layer in self._nccl:
                x = layer(x)
            if out is not None:
                out.copy_(x)
                return out
            return x
        if x.dtype != torch.bfloat16 or not x.is_cuda:
            raise ValueError("tokens must be bf16 on the GPU")
        M = x.shape[0]
        bufs = self._pingpong(x)
        stream = torch.cuda.current_stream(x.device).cuda_stream
        cur = x
        for i, cs in enumerate(self._cs):
            dst = out if (out is not None and i == len(self._cs) - 1) else bufs[i & 1]
            if dst is cur:  # never write the tokens being read
                dst = bufs[(i + 1) & 1]
            L.check(L.lib().aipu_ep_moe_layer(self._peer._ep, ctypes.byref(cs), self.layers[i].expert_lo,
                                              cur.data_ptr(), M, dst.data_ptr(), stream))
            cur = dst
        return cur

    def close(self):
        if self._peer is not None:
            self._peer.close()
            self._peer = None

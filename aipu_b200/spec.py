"""Speculative batched verify over the MoE decode stack (M = K + 1 token rows in one pass).

The reference's speculative system (src/glm_q4k_spec_system.v:30-61) verifies K draft tokens in one
pass of the model over the batch {cur_tok, d_1, .., d_K}: the pass yields the greedy tokens
m_1 .. m_{K+1} (row j's argmax), the drafts are accepted while d_j == m_j, the longest accepted
prefix p commits m_1 .. m_{p+1}, and the next pass starts from m_{p+1}. Because a row is accepted only
when its input is the token greedy decoding would have fed there, the committed stream equals greedy
decoding for any draft quality; the drafts only set how many tokens commit per weight stream.

This module runs that pass over the part of the model this library computes: token rows (an embedding
table lookup), the MoE branch of every layer in turn (one GPU: ops.moe_layer on the bit-exact decode
path; several GPUs: an ep.DecodeStream), then the LM head under the reference's bf16 dot contract
(ops.bf16_dot_gemv) and the argmax. The attention, norms and residuals between blocks -- and with them
the KV-cache write-back of the accepted rows and the AIPUDevice.step backend that drives a full model
(host/aipu_device.py:222-316) -- are outside this library's path; ``stack`` can be any callable that
maps [rows, H] bf16 hidden states to the next ones, so a caller that owns those parts plugs them in.
Every row is computed independently and bit-exactly, so a row's result does not depend on how many
rows share the pass (M = K + 1 rows give the same bits as K + 1 single-row passes).
"""
from __future__ import annotations

from dataclasses import dataclass, field
from typing import Callable, List, Optional, Sequence

import torch

from . import ops


def longest_accepted_prefix(drafts: Sequence[int], truth: Sequence[int]) -> int:
    """p = number of leading drafts equal to the verified tokens: d_j == m_j for j = 1..p
    (src/glm_q4k_spec_system.v:41-45). truth holds m_1 .. m_{K+1}."""
    p = 0
    while p < len(drafts) and p < len(truth) and int(drafts[p]) == int(truth[p]):
        p += 1
    return p


@dataclass
class SpecStats:
    """Bookkeeping over passes: passes run, drafts offered, drafts accepted, tokens committed."""
    passes: int = 0
    drafted: int = 0
    accepted: int = 0
    committed: int = 0
    accepted_per_pass: List[int] = field(default_factory=list)

    @property
    def acceptance_rate(self) -> float:
        return self.accepted / self.drafted if self.drafted else 0.0

    @property
    def tokens_per_pass(self) -> float:
        return self.committed / self.passes if self.passes else 0.0


class SpecVerifier:
    """Verify passes of K drafts over the MoE decode stack.

    emb: bf16 [V, H] token rows; lm_head: bf16 [V, H] (rows of the output projection);
    stack: list of ops.MoeLayerWeights (applied in turn on one GPU) or a callable [M, H] -> [M, H].
    """

    def __init__(self, emb: torch.Tensor, lm_head: torch.Tensor, stack, ctx: Optional[ops.Context] = None):
        if emb.dtype != torch.bfloat16 or lm_head.dtype != torch.bfloat16 or emb.dim() != 2 or lm_head.dim() != 2:
            raise ValueError("emb and lm_head must be bf16 [V, H]")
        if emb.shape[1] != lm_head.shape[1]:
            raise ValueError("emb and lm_head must have the same hidden size")
        self.emb = emb
        self.lm_head = lm_head
        self.ctx = ctx
        if callable(stack):
            self._stack: Callable[[torch.Tensor], torch.Tensor] = stack
        else:
            layers = list(stack)

            def run(x):
                for W in layers:
                    x = ops.moe_layer(W, x, ctx=self.ctx)
                return x

            self._stack = run
        self.stats = SpecStats()

    def greedy_tokens(self, rows: Sequence[int]) -> List[int]:
        """m_j = argmax of the LM head over the stack's output for token row j (lowest index on ties)."""
        idx = torch.as_tensor(list(rows), dtype=torch.long, device=self.emb.device)
        h = self._stack(self.emb.index_select(0, idx).contiguous())
        logits = ops.bf16_dot_gemv(self.lm_head, h, ctx=self.ctx)
        return [int(v) for v in logits.float().argmax(dim=1).cpu().tolist()]

    def verify(self, cur_tok: int, drafts: Sequence[int]):
        """One pass over {cur_tok, d_1..d_K}: returns (committed tokens m_1..m_{p+1}, p)."""
        truth = self.greedy_tokens([cur_tok] + list(drafts))
        p = longest_accepted_prefix(drafts, truth)
        committed = truth[:p + 1]
        s = self.stats
        s.passes += 1
        s.drafted += len(drafts)
        s.accepted += p
        s.committed += len(committed)
        s.accepted_per_pass.append(p)
        return committed, p

    def generate(self, cur_tok: int, n_tokens: int, draft_fn: Callable[[int, int], Sequence[int]], k: int):
        """Commit n_tokens tokens after cur_tok with K-draft verify passes; draft_fn(tok, k) proposes
        the next k tokens after tok."""
        out: List[int] = []
        tok = cur_tok
        while len(out) < n_tokens:
            committed, _ = self.verify(tok, list(draft_fn(tok, k))[:k])
            out.extend(committed)
            tok = committed[-1]
        return out[:n_tokens]

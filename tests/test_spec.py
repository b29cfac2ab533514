"""Speculative batched verify (aipu_b200/spec.py): acceptance bookkeeping on the host (CPU tests, a
token map standing in for the model) and a verify pass over a real MoE decode stack on the GPU whose
committed stream equals greedy one-token decoding and whose K+1-row pass equals K+1 single-row passes
bit for bit."""
import numpy as np
import pytest
import torch

from aipu_b200 import spec


def test_longest_accepted_prefix():
    assert spec.longest_accepted_prefix([], [5]) == 0
    assert spec.longest_accepted_prefix([1, 2, 3], [1, 2, 3, 4]) == 3
    assert spec.longest_accepted_prefix([1, 9, 3], [1, 2, 3, 4]) == 1
    assert spec.longest_accepted_prefix([7, 2, 3], [1, 2, 3, 4]) == 0


class _Table(spec.SpecVerifier):
    """A verifier whose 'model' is a fixed next-token table (host only)."""

    def __init__(self, nxt):
        self.nxt = nxt
        self.stats = spec.SpecStats()

    def greedy_tokens(self, rows):
        return [int(self.nxt[r]) for r in rows]


@pytest.mark.parametrize("quality", [0.0, 0.5, 1.0])
def test_spec_stream_equals_greedy_for_any_draft_quality(quality):
    rng = np.random.default_rng(1)
    V = 64
    nxt = rng.integers(0, V, V)
    v = _Table(nxt)

    def draft(tok, k):  # right with probability `quality`, else a wrong token
        out, t = [], tok
        for _ in range(k):
            t = int(nxt[t]) if rng.random() < quality else int((nxt[t] + 1) % V)
            out.append(t)
        return out

    got = v.generate(3, 40, draft, k=4)
    greedy, t = [], 3
    for _ in range(40):
        t = int(nxt[t])
        greedy.append(t)
    assert got == greedy
    s = v.stats
    assert s.committed >= 40 and s.accepted <= s.drafted
    if quality == 1.0:
        assert s.acceptance_rate == 1.0 and s.tokens_per_pass == 5.0
    if quality == 0.0:
        assert s.accepted == 0 and s.tokens_per_pass == 1.0


@pytest.mark.gpu
def test_verify_pass_over_moe_stack_gpu():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from aipu_b200 import formats as F
    from aipu_b200 import ops

    d = torch.device("cuda", 0)
    H, Fd, E, T, V, K = 512, 256, 16, 4, 384, 4
    g = torch.Generator(device=d)
    layers = []
    for l in range(3):
        s0 = 100 * (l + 1)
        layers.append(ops.MoeLayerWeights(
            hidden=H, ffn=Fd, n_experts=E, topk=T, router_wtype=F.F32,
            router_w=torch.randn((H, E), device=d, generator=g.manual_seed(s0)) * 0.02,
            router_bias=torch.randn((E,), device=d, generator=g.manual_seed(s0 + 1)) * 0.01,
            gate_w=F.random_rows_dev(F.Q4_K, E * Fd, H, seed=s0 + 2, device=d),
            up_w=F.random_rows_dev(F.Q4_K, E * Fd, H, seed=s0 + 3, device=d),
            down_w=F.random_rows_dev(F.Q4_K, E * H, Fd, seed=s0 + 4, device=d), down_wtype=F.Q4_K,
            shared_gate_w=F.random_rows_dev(F.Q4_K, Fd, H, seed=s0 + 5, device=d),
            shared_up_w=F.random_rows_dev(F.Q4_K, Fd, H, seed=s0 + 6, device=d),
            shared_down_w=F.random_rows_dev(F.Q4_K, H, Fd, seed=s0 + 7, device=d)))
    emb = torch.randn((V, H), device=d, generator=g.manual_seed(7)).to(torch.bfloat16)
    lm = (torch.randn((V, H), device=d, generator=g.manual_seed(8)) * 0.05).to(torch.bfloat16)
    v = spec.SpecVerifier(emb, lm, layers)
    # a K+1-row pass gives the same tokens as single-row passes (rows are exact and independent)
    rows = [5, 17, 200, 3, 99]
    assert v.greedy_tokens(rows) == [v.greedy_tokens([r])[0] for r in rows]
    # greedy reference stream, one row per pass
    greedy, t = [], 11
    for _ in range(12):
        t = v.greedy_tokens([t])[0]
        greedy.append(t)
    nxt = {}
    prev = 11
    for tok in greedy:
        nxt[prev] = tok
        prev = tok
    rng = np.random.default_rng(0)

    def draft(tok, k):  # the true continuation where known, corrupted with probability 1/3
        out, cur = [], tok
        for _ in range(k):
            cur = nxt.get(cur, 0)
            out.append(cur if rng.random() > 1 / 3 else (cur + 1) % V)
        return out

    v.stats = spec.SpecStats()
    got = v.generate(11, 12, draft, k=K)
    assert got == greedy
    assert v.stats.passes < 12  # some drafts were accepted

"""The K1 ops are safe to capture in a CUDA graph: no host synchronisation, no allocation
outside torch's allocator, and the forward's scratch counters are left zeroed by every
launch, so a replayed graph recomputes the same bits as eager calls.  Covers the autograd
op (forward + backward), the GRPO window node with temperature and the forward-only call,
on shapes that select the one-block-per-SM forward, the row-group forward and the split
block forward."""
import pytest
import torch

import kernel_opt
from _gpu import seeded_logits, seeded_targets

pytestmark = pytest.mark.gpu

SHAPES = [(1024, 152064), (12000, 4096), (300, 32000)]


def _warm_then_capture(fn, stream):
    stream.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(stream):
        for _ in range(3):
            fn()
    torch.cuda.current_stream().wait_stream(stream)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=stream):
        out = fn()
    return g, out


@pytest.mark.parametrize("rows,vocab", SHAPES)
def test_fwd_bwd_replay_equals_eager(rows, vocab):
    x = seeded_logits((rows, vocab), torch.bfloat16, 3.0, seed=rows).cuda()
    t = seeded_targets((rows,), vocab, seed=rows + 1).cuda()
    t[3] = -100
    gl = torch.full((rows,), -1.0 / rows, device="cuda")
    gh = torch.full((rows,), -0.01 / rows, device="cuda")

    def step():
        xx = x.detach().requires_grad_(True)
        lp, h, l = kernel_opt.fused_logprob_entropy(xx, t)
        (d,) = torch.autograd.grad((lp, h), xx, (gl, gh))
        return lp.detach(), h.detach(), l.detach(), d

    eager = step()
    g, static = _warm_then_capture(step, torch.cuda.Stream())
    for _ in range(3):
        g.replay()
        torch.cuda.synchronize()
        for a, b in zip(static, eager):
            torch.testing.assert_close(a, b, rtol=0, atol=0)
    # new inputs copied into the captured buffers give the eager results of those inputs
    x.copy_(seeded_logits((rows, vocab), torch.bfloat16, 2.0, seed=rows + 7).cuda())
    eager2 = step()
    g.replay()
    torch.cuda.synchronize()
    for a, b in zip(static, eager2):
        torch.testing.assert_close(a, b, rtol=0, atol=0)


def test_grpo_window_replay_equals_eager():
    from kernel_opt import grpo
    B, L, V, K = 4, 257, 65536, 200
    parent = seeded_logits((B, L, V), torch.bfloat16, 2.5, seed=5).cuda()
    ids = seeded_targets((B, K), V, seed=6).cuda()
    g_lp = torch.randn(B, K, device="cuda")

    def step():
        p = parent.detach().requires_grad_(True)
        lp, ent = grpo.window_logps_and_entropies(p, ids, K, temperature=0.7)
        (d,) = torch.autograd.grad(lp, p, g_lp)
        return lp.detach(), ent, d

    eager = step()
    g, static = _warm_then_capture(step, torch.cuda.Stream())
    g.replay()
    torch.cuda.synchronize()
    for a, b in zip(static, eager):
        torch.testing.assert_close(a, b, rtol=0, atol=0)

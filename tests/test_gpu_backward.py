"""Backward parity on the GPU vs the fp64 oracle, plus the reference's autograd tests
(tests/test_logprob.py:170-252, tests/test_compile.py:24-65)."""
import numpy as np
import pytest
import torch

import kernel_opt
from _gpu import GRAD_FLOOR, GRAD_RTOL, check_grad, grads_like, seeded_logits, seeded_targets
from _helpers import assert_close_nan, golden_cases
from kernel_opt import _C
from oracle import oracle

pytestmark = pytest.mark.gpu
DTYPES = [torch.float32, torch.bfloat16, torch.float16]
CASES = golden_cases()


def autograd_grad(x_cpu, t_cpu, g, which=(0, 1, 2)):
    x = x_cpu.cuda().requires_grad_(True)
    outs = kernel_opt.fused_logprob_entropy(x, t_cpu.cuda())
    used = [outs[i] for i in which]
    grads = [g[i].cuda() for i in which]
    (d,) = torch.autograd.grad(used, x, grads)
    assert d.dtype == x_cpu.dtype and d.shape == x_cpu.shape
    return d


@pytest.mark.parametrize("name", sorted(n for n in CASES if "d_logits" in CASES[n]))
def test_golden_cases(name):
    c = CASES[name]
    g = tuple(torch.from_numpy(c[k]).float() for k in ("g_logp", "g_ent", "g_lse"))
    d = autograd_grad(c["logits"], c["targets_t"], g)
    dt = c["logits"].dtype
    ref = c["d_logits"]
    scale = np.abs(ref[np.isfinite(ref)]).max()
    atol = max(1e-7 * scale, GRAD_FLOOR[dt])
    assert_close_nan(d.cpu().double().numpy(), ref, atol, GRAD_RTOL[dt], name)


@pytest.mark.parametrize("dtype", DTYPES)
@pytest.mark.parametrize("shape", [(2, 4, 256), (1, 8, 4096), (3, 16, 8192), (2, 7, 1003)])
def test_backward_matches_oracle(dtype, shape):
    """Reference tests/test_logprob.py:170-206 (random upstream grads x0.5, seed 7)."""
    x = seeded_logits(shape, dtype, 1.0, seed=7)
    t = seeded_targets(shape[:-1], shape[-1], seed=8)
    g = grads_like(shape[:-1], seed=9)
    d = autograd_grad(x, t, g)
    check_grad(d, x, t, *g, what=f"{dtype} {shape}")


def test_backward_only_logprob_grad():
    """Reference tests/test_logprob.py:209-231: entropy / lse unused -> None grads."""
    x = seeded_logits((2, 8, 4096), torch.float32, 1.0, seed=8)
    t = seeded_targets((2, 8), 4096)
    g = grads_like((2, 8), seed=10)
    d = autograd_grad(x, t, g, which=(0,))
    check_grad(d, x, t, g[0], None, None, what="logp only")


def test_gradcheck_small():
    """Reference tests/test_logprob.py:234-252."""
    torch.manual_seed(9)
    t = torch.randint(0, 64, (1, 2), device="cuda")

    def fn(x_double):
        lp, h, l = kernel_opt.fused_logprob_entropy(x_double.float(), t)
        return lp.double(), h.double(), l.double()

    x = torch.randn(1, 2, 64, device="cuda", dtype=torch.float64, requires_grad=True)
    assert torch.autograd.gradcheck(fn, (x,), eps=1e-3, atol=1e-2, rtol=1e-2, nondet_tol=1e-3)


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_compile_forward_and_backward_match_eager(dtype):
    """Reference tests/test_compile.py:24-65 (backend aot_eager)."""
    x0 = seeded_logits((2, 8, 4096), dtype, 1.0, seed=0).cuda()
    t = seeded_targets((2, 8), 4096).cuda()

    def loss_fn(x, t):
        lp, h, _l = kernel_opt.fused_logprob_entropy(x, t)
        return (lp + 0.1 * h).sum()

    eager = kernel_opt.fused_logprob_entropy(x0, t)
    comp = torch.compile(lambda a, b: kernel_opt.fused_logprob_entropy(a, b),
                         backend="aot_eager", dynamic=False)(x0, t)
    for e, c in zip(eager, comp):
        torch.testing.assert_close(e, c, rtol=0, atol=0)
    xe = x0.clone().requires_grad_(True)
    loss_fn(xe, t).backward()
    xc = x0.clone().requires_grad_(True)
    torch.compile(loss_fn, backend="aot_eager", dynamic=False)(xc, t).backward()
    torch.testing.assert_close(xc.grad, xe.grad, rtol=0, atol=0)


def test_in_place_and_strided_gradient_outputs():
    """d_logits may alias logits (in-place) or be a strided view into a larger buffer."""
    B, L, V = 3, 9, 4096
    x = seeded_logits((B, L, V), torch.bfloat16, 2.0, seed=21)
    t = seeded_targets((B, L), V, seed=22)
    g = grads_like((B, L), seed=23)
    xg, tg = x.cuda(), t.cuda()
    lp, h, l = kernel_opt.fused_logprob_entropy_forward(xg, tg)
    ref = torch.empty_like(xg)
    _C.fused_logprob_entropy_v1_backward(xg, tg, l, h, *(a.cuda() for a in g), ref)
    check_grad(ref, x, t, *g, what="plain")
    inplace = xg.clone()
    _C.fused_logprob_entropy_v1_backward(inplace, tg, l, h, *(a.cuda() for a in g), inplace)
    torch.testing.assert_close(inplace, ref, rtol=0, atol=0)
    parent = torch.full((B, L + 1, V), 7.0, dtype=torch.bfloat16, device="cuda")
    view = parent[:, 1:, :]
    _C.fused_logprob_entropy_v1_backward(xg, tg, l, h, *(a.cuda() for a in g), view)
    torch.testing.assert_close(view, ref, rtol=0, atol=0)
    assert (parent[:, 0, :] == 7.0).all()


def test_strided_logits_autograd():
    """Gradient through the GRPO window view logits[:, :-1] (single launch)."""
    B, L, V = 2, 17, 8192
    parent = seeded_logits((B, L, V), torch.bfloat16, 2.0, seed=24).cuda().requires_grad_(True)
    win = parent[:, :-1, :]
    t = seeded_targets((B, L - 1), V, seed=25).cuda()
    g = grads_like((B, L - 1), seed=26)
    lp, h, l = kernel_opt.fused_logprob_entropy(win, t)
    (lp * g[0].cuda() + h * g[1].cuda() + l * g[2].cuda()).sum().backward()
    assert parent.grad.shape == parent.shape
    assert (parent.grad[:, -1, :] == 0).all()
    check_grad(parent.grad[:, :-1, :], win.detach().cpu(), t.cpu(), *g, what="window")


def test_target_edges_and_confident_targets():
    """Out-of-range targets get no one-hot term; a target holding ~all the mass keeps its
    gradient g_logp (1 - p) to relative precision; -inf logits get a zero gradient (the
    reference kernel returns NaN there)."""
    V = 4096
    x = seeded_logits((6, V), torch.float32, 1.0, seed=27)
    x[0, 11] += 30.0
    x[1, 12] += 45.0
    x[4, ::5] = float("-inf")
    t = torch.tensor([11, 12, -100, V, 3, 4])
    g = (torch.ones(6), torch.full((6,), 0.3), torch.full((6,), -0.2))
    d = autograd_grad(x, t, g)
    check_grad(d, x, t, *g, what="edges")
    assert torch.isfinite(d).all()
    assert (d[4, ::5] == 0).all()


@pytest.mark.parametrize("dtype", DTYPES)
def test_backward_ragged_and_split(dtype):
    for n, V in ((1, 152064), (5, 1003), (37, 17), (2, 1)):
        x = seeded_logits((n, V), dtype, 3.0, seed=n + V)
        t = seeded_targets((n,), V, seed=n)
        g = grads_like((n,), seed=V)
        d = autograd_grad(x, t, g)
        check_grad(d, x, t, *g, what=f"{dtype} {n}x{V}")


def test_no_ring_wait_ran_out():
    """The bulk-copy ring bounds every barrier wait; none may have run out in this run."""
    x = seeded_logits((64, 32000), torch.bfloat16, 3.0, seed=60)
    t = seeded_targets((64,), 32000)
    autograd_grad(x, t, grads_like((64,), seed=61))
    torch.cuda.synchronize()
    assert _C.ring_status() == 0


def test_custom_op_opcheck():
    """torch.library.opcheck: schema, fake tensor, autograd registration, AOT dispatch."""
    from kernel_opt import ops
    x = seeded_logits((2, 4, 1000), torch.float32, 1.0, seed=70).cuda().requires_grad_(True)
    t = seeded_targets((2, 4), 1000, seed=71).cuda()
    torch.library.opcheck(ops._fwd_op, (x, t))


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_compile_fullgraph_no_graph_break(dtype):
    """With the custom op, a compiled loss containing K1 is one graph (fullgraph=True would
    raise on a graph break) and matches eager in value and gradient."""
    x0 = seeded_logits((2, 8, 4096), dtype, 1.0, seed=72).cuda()
    t = seeded_targets((2, 8), 4096, seed=73).cuda()

    def loss_fn(x, t):
        lp, h, _l = kernel_opt.fused_logprob_entropy(x, t)
        return (lp + 0.1 * h).sum()

    xe = x0.clone().requires_grad_(True)
    le = loss_fn(xe, t)
    le.backward()
    xc = x0.clone().requires_grad_(True)
    lc = torch.compile(loss_fn, backend="aot_eager", fullgraph=True)(xc, t)
    lc.backward()
    torch.testing.assert_close(lc, le, rtol=1e-6, atol=1e-6)
    torch.testing.assert_close(xc.grad, xe.grad, rtol=0, atol=0)

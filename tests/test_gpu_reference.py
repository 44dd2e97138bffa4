"""Parity against the reference's own CUDA kernels, rebuilt for sm_100a from the reference
sources (oracle/build_ref.py -> oracle/_ref).  This pins the fp64 oracle to the reference
implementation itself and checks this implementation against it on identical inputs,
with the reference tests' tolerances (tests/test_logprob.py:44-47, 127-130, 199-203)."""
import numpy as np
import pytest
import torch

import kernel_opt
from _gpu import grads_like, seeded_logits, seeded_targets
from _helpers import assert_close_nan
from oracle import oracle, reference_k1

pytestmark = pytest.mark.gpu
REF = reference_k1.load()
needs_ref = pytest.mark.skipif(REF is None, reason="reference K1 build (oracle/_ref) absent")

FWD_TOL = {torch.float32: 1e-4, torch.bfloat16: 5e-3, torch.float16: 5e-3}
BWD_TOL = {torch.float32: 1e-4, torch.bfloat16: 1e-2, torch.float16: 1e-2}


@needs_ref
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16, torch.float16])
@pytest.mark.parametrize("shape", [(2, 16, 4096), (1, 1, 32000), (3, 8, 8192), (4, 64, 128256)])
def test_oracle_and_ours_match_reference_forward(dtype, shape):
    x = seeded_logits(shape, dtype, 2.0, seed=2)
    t = seeded_targets(shape[:-1], shape[-1], seed=3)
    xg, tg = x.cuda(), t.cuda()
    ref = [o.cpu().double().numpy() for o in reference_k1.forward(xg, tg)]
    orc = oracle.forward(x, t)
    ours = [o.cpu().double().numpy() for o in kernel_opt.fused_logprob_entropy_forward(xg, tg)]
    tol = FWD_TOL[dtype]
    for name, r, o, k in zip(("logp", "entropy", "lse"), ref, orc, ours):
        assert_close_nan(o, r, tol, tol, f"oracle vs reference {name}")
        assert_close_nan(k, r, tol, tol, f"ours vs reference {name}")


@needs_ref
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("shape", [(2, 4, 256), (1, 8, 4096), (3, 16, 8192)])
def test_oracle_and_ours_match_reference_backward(dtype, shape):
    x = seeded_logits(shape, dtype, 1.0, seed=7)
    t = seeded_targets(shape[:-1], shape[-1], seed=8)
    g = [a.cuda() for a in grads_like(shape[:-1], seed=9)]
    xg, tg = x.cuda(), t.cuda()
    lp, h, l = reference_k1.forward(xg, tg)
    ref = reference_k1.backward(xg, tg, l, h, *g).cpu().double().numpy()
    lp0, h0, l0 = oracle.forward(x, t)
    orc = oracle.backward(x, t, l0, h0, *(a.cpu() for a in g))
    xo = xg.clone().requires_grad_(True)
    outs = kernel_opt.fused_logprob_entropy(xo, tg)
    (ours,) = torch.autograd.grad(outs, xo, g)
    tol = BWD_TOL[dtype]
    assert_close_nan(orc, ref, tol, tol, "oracle vs reference d_logits")
    assert_close_nan(ours.cpu().double().numpy(), ref, tol, tol, "ours vs reference d_logits")


@needs_ref
def test_reference_edge_semantics_are_followed():
    """Out-of-range targets (logit read as 0) and -inf entries skipped in the forward:
    same outputs as the reference kernel."""
    V = 1024
    x = seeded_logits((4, V), torch.float32, 2.0, seed=30)
    x[1, ::4] = float("-inf")
    t = torch.tensor([-100, 3, V + 2, 5])
    xg, tg = x.cuda(), t.cuda()
    ref = [o.cpu().double().numpy() for o in reference_k1.forward(xg, tg)]
    ours = [o.cpu().double().numpy() for o in kernel_opt.fused_logprob_entropy_forward(xg, tg)]
    for r, o in zip(ref, ours):
        assert_close_nan(o, r, 1e-4, 1e-4, "edge")
    np.testing.assert_array_equal(np.isfinite(ref[0]), np.isfinite(ours[0]))


@needs_ref
def test_minus_inf_logits_gradient_deliberately_differs():
    """The one deliberate difference from the reference: at a -inf logit the reference's
    backward computes 0 * inf = NaN (p = 0 times (x - lse) = -inf), where this build writes
    0, the limit of the gradient.  Everywhere else in the row both agree."""
    V = 2048
    x = seeded_logits((3, V), torch.float32, 2.0, seed=31)
    x[1, ::8] = float("-inf")
    t = torch.tensor([5, 9, 700])
    g = [a.cuda() for a in grads_like((3,), seed=32)]
    xg, tg = x.cuda(), t.cuda()
    lp, h, l = reference_k1.forward(xg, tg)
    ref = reference_k1.backward(xg, tg, l, h, *g).cpu()
    xo = xg.clone().requires_grad_(True)
    (ours,) = torch.autograd.grad(kernel_opt.fused_logprob_entropy(xo, tg), xo, g)
    ours = ours.cpu()
    neg = torch.isinf(x) & (x < 0)
    assert torch.isnan(ref[neg]).all(), "the reference no longer returns NaN at -inf logits"
    assert (ours[neg] == 0).all()
    keep = ~neg
    assert_close_nan(ours[keep].double().numpy(), ref[keep].double().numpy(), 1e-4, 1e-4,
                     "d_logits away from the -inf entries")

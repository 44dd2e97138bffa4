"""Temperature folded into K1 (`_C.fused_logprob_entropy_scaled*`) and the GRPO
completion-window node (`kernel_opt.grpo.window_logps_and_entropies`).

The reference trainer divides the sliced window in place by the temperature and then runs
K1 (python/kernel_opt/trainer.py:96-127).  The scaled kernels must reproduce that sequence
bit for bit: the forward equals K1 on `x.div_(T)`, the backward equals K1's backward on
the divided logits followed by torch's division backward.  The window node must give the
parent [B, L, V] gradient that autograd computes through slice + `div_` + K1, bit for bit,
with zeros outside the window.
"""
import pytest
import torch

import kernel_opt
from _gpu import check_forward_outputs, check_grad, grads_like, seeded_logits, seeded_targets
from kernel_opt import _C, grpo

pytestmark = pytest.mark.gpu
DTYPES = [torch.bfloat16, torch.float16, torch.float32]
TEMPS = [0.7, 1.3, 0.85]


def _outs(n, dev="cuda"):
    return tuple(torch.empty(n, device=dev) for _ in range(3))


def _equal(a, b, what):
    torch.testing.assert_close(a, b, rtol=0, atol=0, equal_nan=True, msg=what)


def _inputs(dtype, shape, seed, neg_inf=False):
    x = seeded_logits(shape, dtype, 3.0, seed=seed)
    if neg_inf:
        x.view(-1, shape[-1])[1, ::7] = float("-inf")
    t = seeded_targets(shape[:-1], shape[-1], seed=seed + 1)
    t.view(-1)[0] = -100  # ignore index
    return x.cuda(), t.cuda()


@pytest.mark.parametrize("dtype", DTYPES)
@pytest.mark.parametrize("T", TEMPS)
@pytest.mark.parametrize("shape", [(4, 8, 8192), (3, 5, 1001), (2, 64, 151936)])
def test_scaled_forward_equals_div_then_k1(dtype, T, shape):
    x, t = _inputs(dtype, shape, seed=11, neg_inf=True)
    s = grpo.temperature_scale(T)
    y = x.clone().div_(T)
    ref = _outs(t.shape)
    _C.fused_logprob_entropy_v1(y, t, *ref)
    got = _outs(t.shape)
    _C.fused_logprob_entropy_scaled(x, t, *got, s)
    for a, b, w in zip(got, ref, ("logprob", "entropy", "lse")):
        _equal(a, b, f"{dtype} T={T} {shape} {w}")


@pytest.mark.parametrize("dtype", DTYPES)
@pytest.mark.parametrize("T", TEMPS)
@pytest.mark.parametrize("shape", [(4, 8, 8192), (3, 5, 1001), (2, 64, 151936)])
@pytest.mark.parametrize("inplace", [False, True])
def test_scaled_backward_equals_k1_backward_then_div(dtype, T, shape, inplace):
    x, t = _inputs(dtype, shape, seed=21, neg_inf=True)
    s = grpo.temperature_scale(T)
    gl, ge, gs = (g.cuda() for g in grads_like(shape[:-1], seed=22))
    y = x.clone().div_(T)
    lp, h, l = _outs(t.shape)
    _C.fused_logprob_entropy_v1(y, t, lp, h, l)
    dy = torch.empty_like(y)
    _C.fused_logprob_entropy_v1_backward(y, t, l, h, gl, ge, gs, dy)
    ref = dy / T  # the division's backward
    if inplace:
        d = x.clone()
        _C.fused_logprob_entropy_scaled_backward(d, t, l, h, gl, ge, gs, d, s)
    else:
        d = torch.empty_like(x)
        _C.fused_logprob_entropy_scaled_backward(x, t, l, h, gl, ge, gs, d, s)
    _equal(d, ref, f"{dtype} T={T} {shape} inplace={inplace}")


@pytest.mark.parametrize("dtype", DTYPES)
def test_scaled_against_oracle(dtype):
    """The scaled path against the fp64 oracle on the divided logits (tolerances of the
    north star)."""
    shape = (2, 6, 32000)
    x, t = _inputs(dtype, shape, seed=31)
    T = 0.6
    y_cpu = x.clone().div_(T).cpu()
    outs = _outs(t.shape)
    _C.fused_logprob_entropy_scaled(x, t, *outs, grpo.temperature_scale(T))
    check_forward_outputs(outs, y_cpu, t.cpu(), f"scaled {dtype}")
    g = grads_like(shape[:-1], seed=32)
    lp, h, l = outs
    d = torch.empty_like(x)
    _C.fused_logprob_entropy_scaled_backward(x, t, l, h, *(v.cuda() for v in g), d,
                                              grpo.temperature_scale(T))
    # d = dL/dy / T: compare d * T with the oracle's dL/dy on y (within the bf16 tolerance,
    # widened by the extra rounding of the division)
    check_grad((d.double() * T).cpu(), y_cpu, t.cpu(), *g, what=f"scaled {dtype}")


def test_scale_one_is_the_unscaled_kernel():
    x, t = _inputs(torch.bfloat16, (2, 4, 4096), seed=41)
    a, b = _outs(t.shape), _outs(t.shape)
    _C.fused_logprob_entropy_v1(x, t, *a)
    _C.fused_logprob_entropy_scaled(x, t, *b, 1.0)
    for u, v in zip(a, b):
        _equal(u, v, "scale 1")


def test_bad_scale_rejected():
    x, t = _inputs(torch.bfloat16, (1, 2, 64), seed=42)
    for s in (0.0, -1.0, float("inf"), float("nan")):
        with pytest.raises(RuntimeError, match="scale must be positive"):
            _C.fused_logprob_entropy_scaled(x, t, *_outs(t.shape), s)
    with pytest.raises(ValueError):
        grpo.temperature_scale(0.0)


# ---------------------------------------------------------------------------------------
# The GRPO window node
# ---------------------------------------------------------------------------------------
def _parent(dtype, B, L, V, seed):
    g = torch.Generator().manual_seed(seed)
    base = (torch.randn(B, L, V, generator=g) * 3).to(dtype).cuda().requires_grad_(True)
    return base


def _reference_flow(base, ids, K, T, gl, ge):
    """What the reference trainer does (slice, div_ in place, K1), in one K1 launch on the
    window (our kernel on the same layout), differentiated by autograd."""
    logits = base * 1  # a non-leaf, like a model output
    w = grpo.completion_window(logits, K)
    w.div_(T)
    lp, h, _ = kernel_opt.fused_logprob_entropy(w, ids.contiguous())
    (d,) = torch.autograd.grad((lp, h), base, (gl, ge))
    return lp.detach(), h.detach(), d


@pytest.mark.parametrize("dtype", DTYPES)
@pytest.mark.parametrize("B,L,V,K", [(3, 17, 8192, 16), (2, 40, 4099, 12), (4, 9, 151936, 8)])
def test_window_node_equals_reference_flow(dtype, B, L, V, K):
    base = _parent(dtype, B, L, V, seed=51)
    ids = torch.randint(0, V, (B, L), generator=torch.Generator().manual_seed(52)).cuda()
    cids = ids[:, -K:]
    T = 0.7
    g = torch.Generator().manual_seed(53)
    gl = torch.randn(B, K, generator=g).cuda()
    ge = torch.randn(B, K, generator=g).cuda() * 0.1
    lp0, h0, d0 = _reference_flow(base, cids, K, T, gl, ge)
    logits = base * 1
    lp, h, _ = grpo._WindowLogprobEntropy.apply(logits, cids, K, grpo.temperature_scale(T), False)
    (d,) = torch.autograd.grad((lp, h), base, (gl, ge))
    _equal(lp.detach(), lp0, "logprob")
    _equal(h.detach(), h0, "entropy")
    _equal(d, d0, "parent gradient")
    lo = L - 1 - K
    assert torch.count_nonzero(d[:, L - 1:]) == 0
    if lo > 0:
        assert torch.count_nonzero(d[:, :lo]) == 0


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_window_node_inplace(dtype):
    B, L, V, K = 2, 12, 8192, 11
    base = _parent(dtype, B, L, V, seed=61)
    cids = torch.randint(0, V, (B, K), generator=torch.Generator().manual_seed(62)).cuda()
    gl = torch.randn(B, K, generator=torch.Generator().manual_seed(63)).cuda()

    lp, _ = grpo.window_logps_and_entropies(base * 1, cids, K, 0.8, False)
    (d_ref,) = torch.autograd.grad(lp, base, gl)

    logits = base * 1
    ptr = logits.data_ptr()
    lp2, ents = grpo.window_logps_and_entropies(logits, cids, K, 0.8, True, inplace_backward=True)
    assert ents is not None and not ents.requires_grad
    _equal(lp2.detach(), lp.detach(), "forward")
    lp2.backward(gl, retain_graph=True)
    _equal(base.grad, d_ref, "in-place gradient")
    # the gradient went through the logits' own storage
    _equal(logits.detach(), d_ref, "logits storage holds the gradient")
    assert logits.data_ptr() == ptr
    # the logits are consumed: a second backward through the retained graph fails loudly
    with pytest.raises(RuntimeError, match="modified by an inplace operation"):
        lp2.backward(gl)


def test_window_node_inplace_rejects_leaf():
    base = _parent(torch.bfloat16, 1, 4, 256, seed=71)
    cids = torch.zeros(1, 3, dtype=torch.long, device="cuda")
    with pytest.raises(ValueError, match="leaf"):
        grpo.window_logps_and_entropies(base, cids, 3, 1.0, inplace_backward=True)


def test_window_node_matches_oracle_bf16():
    """Window node vs the fp64 oracle on the divided window (parity with the reference's
    math, not only with our own unfused sequence)."""
    B, L, V, K, T = 2, 10, 32000, 7, 0.75
    base = _parent(torch.bfloat16, B, L, V, seed=81)
    cids = torch.randint(0, V, (B, K), generator=torch.Generator().manual_seed(82)).cuda()
    lp, h, lse = grpo._WindowLogprobEntropy.apply(base * 1, cids, K, grpo.temperature_scale(T),
                                                 False)
    y = grpo.completion_window(base.detach().clone(), K).div_(T).cpu()
    check_forward_outputs((lp, h, lse), y, cids.cpu(), "window")


@pytest.mark.parametrize("dtype", DTYPES)
def test_public_scaled_op_equals_division_then_k1(dtype):
    x, t = _inputs(dtype, (3, 7, 4099), seed=91)
    g = grads_like(t.shape, seed=92)
    T = 0.85
    xa = x.clone().requires_grad_(True)
    outs = kernel_opt.fused_logprob_entropy_scaled(xa, t, T)
    da = torch.autograd.grad(outs, xa, tuple(v.cuda() for v in g))[0]
    xb = x.clone().requires_grad_(True)
    ref = kernel_opt.fused_logprob_entropy(xb / T, t)
    db = torch.autograd.grad(ref, xb, tuple(v.cuda() for v in g))[0]
    for a, b in zip(outs, ref):
        _equal(a.detach(), b.detach(), "outputs")
    _equal(da, db, "gradient")

"""LM head fused with K1 (`kernel_opt.lm_head.fused_linear_logprob_entropy`).

The chunked path must give exactly K1 on the logits that the same GEMMs produce (chunk by
chunk), its gradients must equal autograd through materialised logits up to the fp32
accumulation order of dW, and its forward must meet the north-star tolerances against the
fp64 oracle on those logits.
"""
import pytest
import torch

from _gpu import check_forward_outputs
from kernel_opt import _C, grpo, lm_head

pytestmark = pytest.mark.gpu


def _problem(N, H, V, dtype, seed=0):
    g = torch.Generator().manual_seed(seed)
    h = (torch.randn(N, H, generator=g) * 0.5).to(dtype).cuda()
    w = (torch.randn(V, H, generator=g) * (3.0 / H ** 0.5)).to(dtype).cuda()
    t = torch.randint(0, V, (N,), generator=g).cuda()
    t[3] = -100
    gl = torch.randn(N, generator=g).cuda()
    ge = torch.randn(N, generator=g).cuda() * 0.1
    return h, w, t, gl, ge


def _chunk_logits(h, w, c):
    return torch.cat([h[a:a + c] @ w.t() for a in range(0, h.shape[0], c)])


def _outs(n):
    return tuple(torch.empty(n, device="cuda") for _ in range(3))


def _k1_chunked(z, t, scale, c):
    """K1 launched chunk by chunk like the fused path (a row's result depends on how the
    launch splits it between thread blocks, in the last bits only)."""
    outs = _outs(z.shape[0])
    for a in range(0, z.shape[0], c):
        _C.fused_logprob_entropy_scaled(z[a:a + c], t[a:a + c], *(o[a:a + c] for o in outs), scale)
    return outs


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16, torch.float32])
@pytest.mark.parametrize("T", [1.0, 0.7])
def test_forward_equals_k1_on_the_chunk_logits(dtype, T):
    N, H, V, c = 300, 128, 5003, 128
    h, w, t, _, _ = _problem(N, H, V, dtype)
    got = lm_head.fused_linear_logprob_entropy(h, w, t, T, chunk_rows=c)
    z = _chunk_logits(h, w, c)
    ref = _k1_chunked(z, t, grpo.temperature_scale(T), c)
    for a, b in zip(got, ref):
        torch.testing.assert_close(a, b, rtol=0, atol=0)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_forward_against_oracle(dtype):
    N, H, V, c, T = 200, 256, 32000, 64, 0.8
    h, w, t, _, _ = _problem(N, H, V, dtype, seed=1)
    lp, ent, lse = lm_head.fused_linear_logprob_entropy(h, w, t, T, chunk_rows=c)
    y = _chunk_logits(h, w, c).div_(T).cpu()
    check_forward_outputs((lp, ent, lse), y, t.cpu(), f"lm_head {dtype}")


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
@pytest.mark.parametrize("T", [1.0, 0.7])
def test_gradients_match_materialised_logits(dtype, T):
    N, H, V, c = 300, 128, 5003, 128
    h, w, t, gl, ge = _problem(N, H, V, dtype, seed=2)
    hx, wx = h.clone().requires_grad_(True), w.clone().requires_grad_(True)
    lp, ent, _ = lm_head.fused_linear_logprob_entropy(hx, wx, t, T, chunk_rows=c)
    dh, dw = torch.autograd.grad((lp, ent), (hx, wx), (gl, ge))

    # reference: the same chunk GEMMs materialised, divided by T, K1 + autograd; dW from
    # the materialised dz in fp32
    import kernel_opt
    hr, wr = h.clone().requires_grad_(True), w.clone().requires_grad_(True)
    z = _chunk_logits(hr, wr, c)
    parts = [kernel_opt.fused_logprob_entropy(z[a:a + c] / T, t[a:a + c])
             for a in range(0, N, c)]
    lp0 = torch.cat([p[0] for p in parts])
    ent0 = torch.cat([p[1] for p in parts])
    dh0, dz = torch.autograd.grad((lp0, ent0), (hr, z), (gl, ge))
    torch.testing.assert_close(lp.detach(), lp0.detach(), rtol=0, atol=0)
    torch.testing.assert_close(ent.detach(), ent0.detach(), rtol=0, atol=0)
    # dh: same per-chunk GEMMs on the same dz -> same bits
    torch.testing.assert_close(dh, dh0, rtol=0, atol=0)
    dw_ref = (dz.float().t() @ h.float())
    tol = 1e-5 if dtype == torch.float32 else 1e-2
    scale = float(dw_ref.abs().max())
    torch.testing.assert_close(dw.float(), dw_ref, rtol=tol, atol=1e-3 * scale)
    assert dw.dtype == w.dtype and dh.dtype == h.dtype


def test_frozen_head_and_no_hidden_grad():
    N, H, V = 130, 64, 3001
    h, w, t, gl, _ = _problem(N, H, V, torch.bfloat16, seed=3)
    hx = h.clone().requires_grad_(True)
    lp, _, _ = lm_head.fused_linear_logprob_entropy(hx, w, t, chunk_rows=64)
    (dh,) = torch.autograd.grad(lp, hx, gl)
    assert dh.shape == h.shape
    wx = w.clone().requires_grad_(True)
    lp, _, _ = lm_head.fused_linear_logprob_entropy(h, wx, t, chunk_rows=64)
    (dw,) = torch.autograd.grad(lp, wx, gl)
    assert dw.shape == w.shape


def test_leading_dims_and_default_chunk():
    B, K, H, V = 3, 50, 64, 4096
    g = torch.Generator().manual_seed(4)
    h = torch.randn(B, K + 1, H, generator=g).to(torch.bfloat16).cuda()[:, :-1]  # a view
    w = (torch.randn(V, H, generator=g) * 0.3).to(torch.bfloat16).cuda()
    t = torch.randint(0, V, (B, K), generator=g).cuda()
    lp, ent, lse = lm_head.fused_linear_logprob_entropy(h, w, t)
    assert lp.shape == (B, K)
    ref = _outs(B * K)
    _C.fused_logprob_entropy_v1((h.reshape(-1, H) @ w.t()), t.reshape(-1), *ref)
    for a, b in zip((lp, ent, lse), ref):
        torch.testing.assert_close(a.reshape(-1), b, rtol=0, atol=0)

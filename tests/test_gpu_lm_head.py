"""LM head fused with K1 (`kernel_opt.lm_head.fused_linear_logprob_entropy`).

fp16 / fp32 heads (library GEMMs and K1 on row chunks) must give exactly K1 on the logits
that the same GEMMs produce, chunk by chunk, and gradients equal to autograd through
materialised logits up to the fp32 accumulation order of dW.

bf16 heads run on the tensor-core kernel (tcgen05, K1 in the GEMM epilogue).  Its logits
must be the library GEMM's (bf16 of an fp32 accumulation: equal except for rare one-ulp
differences of the summation order), its statistics must meet the north-star tolerances
against K1 and against the fp64 oracle on those logits, its recomputed gradient must be
K1's backward on them bit for bit, and its autograd gradients must match materialised
logits.
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


@pytest.mark.parametrize("dtype", [torch.float16, torch.float32])
@pytest.mark.parametrize("T", [1.0, 0.7])
def test_forward_equals_k1_on_the_chunk_logits(dtype, T):
    N, H, V, c = 300, 128, 5003, 128
    h, w, t, _, _ = _problem(N, H, V, dtype)
    got = lm_head.fused_linear_logprob_entropy(h, w, t, T, chunk_rows=c)
    z = _chunk_logits(h, w, c)
    ref = _k1_chunked(z, t, grpo.temperature_scale(T), c)
    for a, b in zip(got, ref):
        torch.testing.assert_close(a, b, rtol=0, atol=0)


@pytest.mark.parametrize("dtype", [torch.float16, torch.float32])
def test_forward_against_oracle(dtype):
    N, H, V, c, T = 200, 256, 32000, 64, 0.8
    h, w, t, _, _ = _problem(N, H, V, dtype, seed=1)
    lp, ent, lse = lm_head.fused_linear_logprob_entropy(h, w, t, T, chunk_rows=c)
    y = _chunk_logits(h, w, c).div_(T).cpu()
    check_forward_outputs((lp, ent, lse), y, t.cpu(), f"lm_head {dtype}")


@pytest.mark.parametrize("dtype", [torch.float16, torch.float32])
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
    tol = 1e-5 if dtype == torch.float32 else 2e-2
    scale = float(dw_ref.abs().max())
    torch.testing.assert_close(dw.float(), dw_ref, rtol=tol, atol=1e-3 * scale)
    assert dw.dtype == w.dtype and dh.dtype == h.dtype


def test_frozen_head_and_no_hidden_grad():
    N, H, V = 130, 64, 3001
    for dtype in (torch.bfloat16, torch.float16):
        h, w, t, gl, _ = _problem(N, H, V, dtype, seed=3)
        hx = h.clone().requires_grad_(True)
        lp, _, _ = lm_head.fused_linear_logprob_entropy(hx, w, t, chunk_rows=64)
        (dh,) = torch.autograd.grad(lp, hx, gl)
        assert dh.shape == h.shape and torch.isfinite(dh.float()).all()
        wx = w.clone().requires_grad_(True)
        lp, _, _ = lm_head.fused_linear_logprob_entropy(h, wx, t, chunk_rows=64)
        (dw,) = torch.autograd.grad(lp, wx, gl)
        assert dw.shape == w.shape and torch.isfinite(dw.float()).all()


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
    torch.testing.assert_close(lse.reshape(-1), ref[2], rtol=0, atol=1e-5)
    torch.testing.assert_close(lp.reshape(-1), ref[0], rtol=0, atol=1e-5)
    torch.testing.assert_close(ent.reshape(-1), ref[1], rtol=1e-4, atol=1e-7)


# ---------------------------------------------------------------------------------------
# bf16: the tensor-core kernel
# ---------------------------------------------------------------------------------------
# H = 136 and 64: the last pipeline stage's second 64-wide K box lies wholly beyond H
# (read as zeros by the tensor copy).  Row stores: V = 32768 and 2064 take 32-byte stores
# (2064: a 16-column tail stored element by element), 1000, 3000 and 1544 16-byte
# stores, 777 and 4099 element by element.
TC_SHAPES = [(300, 256, 1000), (257, 200, 777), (640, 512, 3000), (129, 3584, 4099),
             (1024, 1024, 32768), (200, 136, 1544), (1000, 64, 2064)]


def _tc_problem(N, H, V, seed):
    g = torch.Generator(device="cuda").manual_seed(seed)
    h = (torch.randn(N, H, generator=g, device="cuda") * 0.5).to(torch.bfloat16)
    w = (torch.randn(V, H, generator=g, device="cuda") * (2.5 / H ** 0.5)).to(torch.bfloat16)
    t = torch.randint(0, V, (N,), generator=g, device="cuda")
    t[0], t[1] = -100, V  # outside the vocabulary: logprob = -lse, no one-hot term
    return h, w, t


def _tc_forward(h, w, t, scale, keep=True):
    outs = _outs(h.shape[0])
    z = torch.empty((h.shape[0], w.shape[0]), dtype=torch.bfloat16, device="cuda") if keep else None
    _C.lm_head_forward(h, w, t, *outs, scale, z)
    return outs, z


@pytest.mark.parametrize("shape", TC_SHAPES)
def test_tc_logits_are_the_rounded_product(shape):
    """z = bf16 of the fp32-accumulated product: within one bf16 ulp of the exact (fp64)
    product plus the fp32 accumulation error (2^-20 of the sum of |h_k w_k|, which matters
    only for logits near zero).  (The library GEMM rounds fp32 sums taken in another
    order -- split over K for few rows -- so its bits are not the reference here.)"""
    h, w, t = _tc_problem(*shape, seed=10)
    _, z = _tc_forward(h, w, t, 1.0)
    exact = h.double() @ w.double().t()
    _, e = torch.frexp(exact)
    ulp = torch.ldexp(torch.ones_like(exact), e - 8)  # bf16: 8 significant bits
    acc = (h.double().abs() @ w.double().abs().t()) * 2.0 ** -20
    assert bool(((z.double() - exact).abs() <= ulp + acc).all()), "a logit is off by > 1 ulp"


@pytest.mark.parametrize("shape", TC_SHAPES)
@pytest.mark.parametrize("T", [1.0, 0.7])
def test_tc_statistics_match_k1_and_oracle(shape, T):
    h, w, t = _tc_problem(*shape, seed=11)
    scale = grpo.temperature_scale(T)
    (lp, ent, lse), z = _tc_forward(h, w, t, scale)
    ref = _outs(h.shape[0])
    _C.fused_logprob_entropy_scaled(z, t, *ref, scale)
    torch.testing.assert_close(lse, ref[2], rtol=0, atol=1e-5)
    torch.testing.assert_close(lp, ref[0], rtol=0, atol=1e-5)
    torch.testing.assert_close(ent, ref[1], rtol=1e-4, atol=1e-7)
    assert torch.equal(lp[:2], -lse[:2])
    rows = torch.linspace(0, h.shape[0] - 1, min(64, h.shape[0])).round().long().unique().cuda()
    y = (z[rows].float() * scale).to(torch.bfloat16).cpu() if T != 1.0 else z[rows].cpu()
    check_forward_outputs((lp[rows], ent[rows], lse[rows]), y, t[rows].cpu(), f"tc {shape} T={T}")
    # the statistics-only launch (logits never written) gives the same bits
    (lp2, ent2, lse2), _ = _tc_forward(h, w, t, scale, keep=False)
    assert torch.equal(lp2, lp) and torch.equal(ent2, ent) and torch.equal(lse2, lse)


@pytest.mark.parametrize("shape", TC_SHAPES[:4] + TC_SHAPES[5:])
@pytest.mark.parametrize("T", [1.0, 0.7])
def test_tc_recomputed_gradient_is_k1_backward(shape, T):
    h, w, t = _tc_problem(*shape, seed=12)
    scale = grpo.temperature_scale(T)
    (lp, ent, lse), z = _tc_forward(h, w, t, scale)
    g = torch.Generator(device="cuda").manual_seed(5)
    gl = torch.randn(h.shape[0], generator=g, device="cuda") * 1e-3
    ge = torch.randn(h.shape[0], generator=g, device="cuda") * 1e-4
    d = torch.full_like(z, 7.0)
    _C.lm_head_backward(h, w, t, lse, ent, gl, ge, None, d, scale)
    dk = torch.empty_like(z)
    _C.fused_logprob_entropy_scaled_backward(z, t, lse, ent, gl, ge, None, dk, scale)
    assert torch.equal(d, dk)


@pytest.mark.parametrize("keep", [False, True])
@pytest.mark.parametrize("T", [1.0, 0.7])
def test_tc_gradients_match_materialised_logits(keep, T):
    N, H, V, c = 300, 256, 5003, 128
    h, w, t, gl, ge = _problem(N, H, V, torch.bfloat16, seed=2)
    hx, wx = h.clone().requires_grad_(True), w.clone().requires_grad_(True)
    lp, ent, _ = lm_head.fused_linear_logprob_entropy(hx, wx, t, T, chunk_rows=c,
                                                      keep_logits=keep)
    dh, dw = torch.autograd.grad((lp, ent), (hx, wx), (gl, ge))
    import kernel_opt
    hr, wr = h.clone().requires_grad_(True), w.clone().requires_grad_(True)
    z = hr @ wr.t()
    lp0, ent0, _ = kernel_opt.fused_logprob_entropy_scaled(z, t, T)
    dh0, dw0 = torch.autograd.grad((lp0, ent0), (hr, wr), (gl, ge))
    # the reference's logits come from the library GEMM, whose bf16 rounding differs from
    # the kernel's in rare elements (another summation order): results agree to that
    # rounding, not bit for bit (exact parity on the kernel's own logits is pinned above)
    torch.testing.assert_close(lp.detach(), lp0.detach(), rtol=1e-5, atol=1e-4)
    torch.testing.assert_close(ent.detach(), ent0.detach(), rtol=1e-4, atol=1e-5)
    for a, b in ((dh, dh0), (dw, dw0)):
        scale = float(b.float().abs().max())
        torch.testing.assert_close(a.float(), b.float(), rtol=2e-2, atol=1e-3 * scale)
        assert a.dtype == torch.bfloat16


def _shards(V, S):
    from kernel_opt import parallel
    return [parallel.vocab_shard(V, S, k) for k in range(S)]


@pytest.mark.parametrize("shape,S", [((300, 256, 1000), 3), ((129, 3584, 4099), 2),
                                     ((257, 200, 2064), 4)])
@pytest.mark.parametrize("T", [1.0, 0.7])
def test_tc_vocab_shards_combine_to_the_full_head(shape, S, T):
    """The head split over the vocabulary: each shard's partials (from the tensor-core
    kernel's epilogue), combined, give the full head's statistics within the north-star
    tolerances; each shard's recomputed gradient, from the combined lse / entropy, is the
    full head's gradient on the shard's columns bit for bit."""
    h, w, t = _tc_problem(*shape, seed=13)
    N, V = h.shape[0], w.shape[0]
    t[2] = V - 1          # the last column, in the last shard
    t[3] = _shards(V, S)[-1].start  # the first column of the last shard
    scale = grpo.temperature_scale(T)
    (lp0, ent0, lse0), z = _tc_forward(h, w, t, scale)
    parts, zs = [], []
    for cols in _shards(V, S):
        p = torch.empty((N, 4), dtype=torch.float64, device="cuda")
        _C.lm_head_shard_partials(h, w[cols], t, cols.start, p, scale)
        # the same launch also storing the shard's logits: the same partials, and the full
        # head's logits on those columns
        p2 = torch.empty_like(p)
        zk = torch.empty((N, cols.stop - cols.start), dtype=torch.bfloat16, device="cuda")
        _C.lm_head_shard_partials(h, w[cols], t, cols.start, p2, scale, zk)
        assert torch.equal(p2, p) and torch.equal(zk, z[:, cols])
        parts.append(p)
        zs.append(zk)
    gathered = torch.stack(parts)
    lp, ent, lse = _outs(N)
    _C.vocab_combine(gathered, S, lp, ent, lse)
    torch.testing.assert_close(lse, lse0, rtol=0, atol=1e-5)
    torch.testing.assert_close(lp, lp0, rtol=0, atol=1e-5)
    torch.testing.assert_close(ent, ent0, rtol=1e-4, atol=1e-7)
    assert torch.equal(lp[:2], -lse[:2])
    rows = torch.linspace(0, N - 1, min(64, N)).round().long().unique().cuda()
    y = (z[rows].float() * scale).to(torch.bfloat16).cpu() if T != 1.0 else z[rows].cpu()
    check_forward_outputs((lp[rows], ent[rows], lse[rows]), y, t[rows].cpu(), f"shards {shape}")

    g = torch.Generator(device="cuda").manual_seed(6)
    gl = torch.randn(N, generator=g, device="cuda") * 1e-3
    ge = torch.randn(N, generator=g, device="cuda") * 1e-4
    d_full = torch.empty_like(z)
    _C.lm_head_backward(h, w, t, lse, ent, gl, ge, None, d_full, scale)
    for cols, zk in zip(_shards(V, S), zs):
        d = torch.full((N, cols.stop - cols.start), 7.0, dtype=torch.bfloat16, device="cuda")
        _C.lm_head_shard_backward(h, w[cols], t, cols.start, lse, ent, gl, ge, None, d, scale)
        assert torch.equal(d, d_full[:, cols]), f"shard {cols} gradient differs"
        # K1's scaled backward in place on the kept shard (the keep_logits path): the same
        _C.vocab_shard_backward(zk, t, cols.start, lse, ent, gl, ge, None, zk, scale)
        assert torch.equal(zk, d_full[:, cols]), f"shard {cols} in-place gradient differs"


@pytest.mark.parametrize("keep", [False, True])
def test_tc_vocab_parallel_head_in_one_process(keep):
    """Without a process group the vocab-parallel head over the whole weight (one shard)
    equals the single-GPU fused head, forward and gradients (keep_logits: the shard's
    logits stored in the forward, K1's backward in place on them)."""
    from kernel_opt import parallel
    N, H, V, c = 300, 256, 5003, 128
    h, w, t, gl, ge = _problem(N, H, V, torch.bfloat16, seed=4)
    outs = []
    for fn in (lambda hx, wx: parallel.vocab_parallel_fused_linear_logprob_entropy(
                   hx, wx, t, 0, 0.7, chunk_rows=c, keep_logits=keep),
               lambda hx, wx: lm_head.fused_linear_logprob_entropy(hx, wx, t, 0.7, chunk_rows=c,
                                                                   keep_logits=keep)):
        hx, wx = h.clone().requires_grad_(True), w.clone().requires_grad_(True)
        lp, ent, lse = fn(hx, wx)
        dh, dw = torch.autograd.grad((lp, ent), (hx, wx), (gl, ge))
        outs.append((lp.detach(), ent.detach(), lse.detach(), dh, dw))
    (lp, ent, lse, dh, dw), (lp0, ent0, lse0, dh0, dw0) = outs
    torch.testing.assert_close(lse, lse0, rtol=0, atol=1e-5)
    torch.testing.assert_close(lp, lp0, rtol=0, atol=1e-5)
    torch.testing.assert_close(ent, ent0, rtol=1e-4, atol=1e-7)
    # the same d_logits; dh is rounded once from an fp32 product here and straight from the
    # library GEMM's bf16 output there (with keep_logits), which differ in rare elements by
    # the GEMM's own rounding (the tolerance of the library-GEMM comparisons above); dw is
    # formed identically
    torch.testing.assert_close(dh.float(), dh0.float(), rtol=2e-2, atol=2e-3 * float(dh0.float().abs().max()))
    assert torch.equal(dw, dw0)

"""Host-buffer streaming API: chunked H2D / K1 forward+backward / D2H on three streams must
give exactly the device-API results, for ragged chunking and for an in-place gradient."""
import pytest
import torch

import kernel_opt
from _gpu import grads_like, seeded_logits, seeded_targets
from kernel_opt import _C
from kernel_opt.host import fused_logprob_entropy_fwd_bwd_host

pytestmark = pytest.mark.gpu


def device_reference(x, t, g):
    xg, tg = x.cuda(), t.cuda()
    lp, h, l = kernel_opt.fused_logprob_entropy_forward(xg, tg)
    d = torch.empty_like(xg)
    _C.fused_logprob_entropy_v1_backward(xg, tg, l, h, *(a.cuda() for a in g), d)
    return [a.cpu() for a in (lp, h, l, d)]


@pytest.mark.parametrize("chunk_rows", [None, 7, 64])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_host_streaming_matches_device_api(chunk_rows, dtype):
    N, V = 150, 32000
    x = seeded_logits((N, V), dtype, 3.0, seed=50).pin_memory()
    t = seeded_targets((N,), V, seed=51)
    g = grads_like((N,), seed=52)
    ref = device_reference(x, t, g)
    got = fused_logprob_entropy_fwd_bwd_host(x, t, *g, chunk_rows=chunk_rows)
    if chunk_rows is None:  # one chunk: the same launch as the device API, same bits
        for a, b in zip(got, ref):
            torch.testing.assert_close(a, b, rtol=0, atol=0)
        return
    # Other row counts per launch split rows between thread blocks elsewhere, so the fp64
    # merge order differs: equal to within 2 ulp of fp32 outputs, and of the gradient's
    # dtype (the gradient reads lse / entropy).
    for a, b in zip(got[:3], ref[:3]):
        torch.testing.assert_close(a, b, rtol=2.4e-7, atol=0)
    # a 1-ulp change of lse moves gradient elements whose coefficient passes through zero
    # by a large relative amount: absolute floor of 1e-6 of the largest gradient
    rt = 2e-6 if dtype == torch.float32 else 8e-3
    torch.testing.assert_close(got[3], ref[3], rtol=rt,
                               atol=1e-6 * float(ref[3].float().abs().max()))


def test_host_streaming_in_place_and_shapes():
    B, S, V = 3, 40, 8192
    x = seeded_logits((B, S, V), torch.bfloat16, 2.0, seed=53).pin_memory()
    t = seeded_targets((B, S), V, seed=54)
    g = grads_like((B, S), seed=55)
    ref = device_reference(x.view(-1, V), t.view(-1), [a.view(-1) for a in g])
    buf = x.clone().pin_memory()
    lp, h, l, d = fused_logprob_entropy_fwd_bwd_host(buf, t, g[0], g[1], g[2], d_logits=buf,
                                                     chunk_rows=16)
    assert d.data_ptr() == buf.data_ptr() and lp.shape == (B, S)
    # chunked launches split rows between thread blocks differently from the one-call
    # reference (fp64 merge order): outputs within 2 ulp, gradients within bf16 rounding
    torch.testing.assert_close(lp.view(-1), ref[0], rtol=2.4e-7, atol=0)
    scale = float(ref[3].float().abs().max())
    torch.testing.assert_close(d.view(-1, V).float(), ref[3].float(), rtol=8e-3, atol=1e-6 * scale)


@pytest.mark.parametrize("chunk_rows", [None, 9])
def test_host_streaming_gradient_stays_on_device(chunk_rows):
    """d_logits on the device: each chunk's backward writes straight into it and only the
    per-row outputs come back to the host."""
    N, V = 120, 32000
    x = seeded_logits((N, V), torch.bfloat16, 3.0, seed=60).pin_memory()
    t = seeded_targets((N,), V, seed=61)
    g = grads_like((N,), seed=62)
    ref = device_reference(x, t, g)
    d_dev = torch.empty((N, V), dtype=x.dtype, device="cuda")
    lp, h, l, d = fused_logprob_entropy_fwd_bwd_host(x, t, *g, d_logits=d_dev,
                                                     chunk_rows=chunk_rows)
    assert d is d_dev and not lp.is_cuda
    if chunk_rows is None:
        for a, b in zip((lp, h, l, d.cpu()), ref):
            torch.testing.assert_close(a, b, rtol=0, atol=0)
    else:
        for a, b in zip((lp, h, l), ref[:3]):
            torch.testing.assert_close(a, b, rtol=2.4e-7, atol=0)
        scale = float(ref[3].float().abs().max())
        torch.testing.assert_close(d.cpu().float(), ref[3].float(), rtol=8e-3, atol=1e-6 * scale)
    with pytest.raises(ValueError):
        fused_logprob_entropy_fwd_bwd_host(x, t, *g, d_logits=d_dev[:, :100])

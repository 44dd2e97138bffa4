"""The fp64 C oracle against the golden vectors and the reference's known answers.

The golden answers are the reference tests' ground truth restated in torch fp64
(tests/golden/make_golden.py); the oracle is an independent two-pass C restatement.
"""
import numpy as np
import pytest
import torch

from _helpers import assert_close_nan, golden_cases
from oracle import oracle

CASES = golden_cases()


@pytest.mark.parametrize("name", sorted(CASES))
def test_oracle_forward_matches_golden(name):
    c = CASES[name]
    lp, h, l = oracle.forward(c["logits"], c["targets_t"])
    assert_close_nan(l, c["lse"], 1e-12, 1e-12, f"{name} lse")
    assert_close_nan(lp, c["logp"], 1e-12, 1e-12, f"{name} logp")
    assert_close_nan(h, c["entropy"], 1e-12, 1e-10, f"{name} entropy")


@pytest.mark.parametrize("name", sorted(n for n in CASES if "d_logits" in CASES[n]))
def test_oracle_backward_matches_golden(name):
    c = CASES[name]
    lp, h, l = oracle.forward(c["logits"], c["targets_t"])
    d = oracle.backward(c["logits"], c["targets_t"], l, h, c["g_logp"], c["g_ent"], c["g_lse"])
    scale = np.abs(c["d_logits"]).max()
    assert_close_nan(d, c["d_logits"], 1e-13 * scale, 1e-10, f"{name} d_logits")


def test_uniform_logits_entropy_equals_logV():
    """Reference tests/test_logprob.py:140-152."""
    V = 4096
    lp, h, l = oracle.forward(torch.zeros(1, 1, V), torch.zeros(1, 1, dtype=torch.int64))
    assert abs(h.item() - np.log(V)) < 1e-12
    assert abs(l.item() - np.log(V)) < 1e-12
    assert abs(lp.item() + np.log(V)) < 1e-12


def test_extreme_values_finite():
    """Reference tests/test_logprob.py:101-111."""
    x = torch.randn(1, 4, 1024, generator=torch.Generator().manual_seed(3)) + 60.0
    t = torch.randint(0, 1024, (1, 4))
    for a in oracle.forward(x, t):
        assert np.isfinite(a).all()


def test_out_of_range_target_reads_zero_logit():
    """Reference v1 leaves the shared target logit at 0.0 when no column matches
    (csrc/fused_logprob.cu:179-185): logprob = -lse, and no one-hot gradient."""
    x = torch.randn(3, 50, generator=torch.Generator().manual_seed(4))
    t = torch.tensor([-100, 50, 7])
    lp, h, l = oracle.forward(x, t)
    np.testing.assert_allclose(lp[:2], -l[:2], rtol=0, atol=0)
    g = np.ones(3)
    d = oracle.backward(x, t, l, h, g, None, None)
    p = np.exp(x.double().numpy() - l[:, None])
    np.testing.assert_allclose(d[0], -p[0], rtol=1e-12, atol=1e-15)
    np.testing.assert_allclose(d[2, 7], 1 - p[2, 7], rtol=1e-12)


def test_special_rows():
    """-inf entries are skipped; an all -inf row gives lse=-inf, H=NaN; NaN poisons."""
    x = torch.randn(4, 16, generator=torch.Generator().manual_seed(5))
    x[0, 3] = float("-inf")
    x[1, :] = float("-inf")
    x[2, 5] = float("nan")
    x[3, 2] = float("inf")
    t = torch.tensor([1, 1, 1, 1])
    lp, h, l = oracle.forward(x, t)
    ref = torch.logsumexp(x[0].double().masked_fill(torch.isinf(x[0]), -1e300), -1).item()
    assert abs(l[0] - ref) < 1e-12 and np.isfinite(h[0])
    assert l[1] == -np.inf and np.isnan(h[1]) and np.isnan(lp[1])
    assert np.isnan(l[2]) and np.isnan(h[2]) and np.isnan(lp[2])
    assert np.isnan(l[3]) and np.isnan(h[3])


def test_near_one_hot_entropy_relative_precision():
    """The case a plain fp32 accumulator gets wrong: one logit 40 above the rest."""
    V = 4096
    x = torch.randn(1, V, generator=torch.Generator().manual_seed(6)) * 2.0
    x[0, 100] += 40.0
    lp, h, l = oracle.forward(x, torch.tensor([100]))
    h_ref = decimal_entropy(x[0].tolist())
    assert h[0] > 0 and abs(h[0] - h_ref) / h_ref < 1e-9


def decimal_entropy(xs):
    """Entropy of softmax(xs) with 50-digit decimal arithmetic."""
    import decimal
    ctx = decimal.Context(prec=50)
    D = [ctx.create_decimal(repr(v)) for v in xs]
    m = max(D)
    e = [ctx.exp(d - m) for d in D]
    z = sum(e, ctx.create_decimal(0))
    return float(ctx.ln(z) - sum(ei * (d - m) for ei, d in zip(e, D)) / z)


def test_shard_partials_combine_equals_full():
    """Vocab-parallel restatement: sharded partials merged == unsharded oracle."""
    gen = torch.Generator().manual_seed(7)
    V, N = 1000, 6
    x = (torch.randn(N, V, generator=gen) * 3).to(torch.bfloat16)
    t = torch.tensor([0, 999, 250, 251, -100, 700])
    bounds = [0, 250, 251, 600, 1000]
    words = np.stack([oracle.shard_partials(x[:, a:b], t, a) for a, b in zip(bounds, bounds[1:])])
    lp, h, l = oracle.combine(words)
    lp0, h0, l0 = oracle.forward(x, t)
    np.testing.assert_allclose(l, l0, rtol=1e-13, atol=1e-13)
    np.testing.assert_allclose(h, h0, rtol=1e-11, atol=1e-13)
    np.testing.assert_allclose(lp, lp0, rtol=1e-13, atol=1e-13)

"""GPU parity helpers: run the CUDA path, compare with the fp64 oracle.

Tolerances (north star of this port, against fp64 ground truth):
  * logprob and lse: 1e-5 absolute (fp32 accumulation, whatever the input dtype);
  * entropy: 1e-4 relative (plus 1e-7 absolute for rows whose entropy is exactly 0);
  * d_logits: 1e-5 relative for fp32, 1e-2 relative for bf16 / fp16, with an absolute
    floor of 1e-7 x the largest gradient magnitude (elements whose coefficient
    g_lse - g_logp - g_ent (log p + H) passes through zero have no relative accuracy in
    any fp32 evaluation) and, for fp16, half of fp16's subnormal spacing (2.98e-8),
    below which fp16 cannot represent the value at all.  The floor covers cancellations
    only: every element whose value is not cancelled by more than 20x against the size
    of its terms must meet the relative tolerance alone (check_grad returns the worst).
"""
from __future__ import annotations

import numpy as np
import torch

from _helpers import assert_close_nan
from oracle import oracle

LOGP_ATOL = 1e-5
ENT_RTOL = 1e-4
ENT_ATOL = 1e-7
GRAD_RTOL = {torch.float32: 1e-5, torch.bfloat16: 1e-2, torch.float16: 1e-2}
GRAD_FLOOR = {torch.float32: 0.0, torch.bfloat16: 0.0, torch.float16: 2.98e-8}


def check_forward_outputs(outs, logits_cpu, targets_cpu, what=""):
    lp, h, l = (o.detach().cpu().double().numpy() for o in outs)
    lp0, h0, l0 = oracle.forward(logits_cpu, targets_cpu)
    assert_close_nan(l, l0, LOGP_ATOL, 0.0, f"{what} lse")
    assert_close_nan(lp, lp0, LOGP_ATOL, 0.0, f"{what} logprob")
    assert_close_nan(h, h0, ENT_ATOL, ENT_RTOL, f"{what} entropy")
    return lp0, h0, l0


def check_grad(d, logits_cpu, targets_cpu, g_logp=None, g_ent=None, g_lse=None, what="",
               fwd=None):
    if fwd is None:
        fwd = oracle.forward(logits_cpu, targets_cpu)
    _, h0, l0 = fwd
    d0 = oracle.backward(logits_cpu, targets_cpu, l0, h0, g_logp, g_ent, g_lse)
    dt = logits_cpu.dtype
    finite = np.isfinite(d0)
    scale = float(np.abs(d0[finite]).max()) if finite.any() else 0.0
    atol = max(1e-7 * scale, GRAD_FLOOR[dt])
    got = d.detach().cpu().double().numpy()
    assert_close_nan(got, d0, atol, GRAD_RTOL[dt], f"{what} d_logits")
    # The floor may only cover elements whose value is a cancellation: d = p k with
    # k = g_lse - g_logp - g_ent (x - lse + H) (+ g_logp on the target column), whose fp32
    # evaluation errs by ~eps times the size of its terms.  Every element not cancelled by
    # more than 20x (|d| >= p (|c0| + |g_ent| |x - lse|) / 20) must meet the relative
    # tolerance alone; the worst such error is returned so callers can report it.
    x = logits_cpu.double().numpy().reshape(d0.shape)
    rows = d0.shape[:-1]
    z = lambda g: np.zeros(rows) if g is None else np.asarray(g, np.float64).reshape(rows)
    gl, ge, gs = z(g_logp), z(g_ent), z(g_lse)
    l0r, h0r = np.asarray(l0, np.float64).reshape(rows), np.asarray(h0, np.float64).reshape(rows)
    with np.errstate(invalid="ignore", over="ignore"):
        dx = x - l0r[..., None]
        pr = np.exp(dx)
        c0 = np.abs(gs - gl - ge * h0r)[..., None]
        terms = pr * (c0 + np.abs(ge)[..., None] * np.abs(dx)) + np.abs(gl)[..., None] * pr
        t = np.asarray(targets_cpu, np.int64).reshape(rows)
        onehot = (np.arange(x.shape[-1]) == t[..., None])
        terms = terms + onehot * np.abs(gl)[..., None]
    # below the dtype's smallest normal number the output format itself has no relative
    # precision (fp16 subnormals): the absolute floor covers those
    tiny = float(torch.finfo(dt).tiny)
    plain = finite & np.isfinite(got) & (d0 != 0) & np.isfinite(terms) & \
        (np.abs(d0) >= terms / 20.0) & (np.abs(d0) >= max(GRAD_FLOOR[dt], tiny))
    worst = float((np.abs(got[plain] - d0[plain]) / np.abs(d0[plain])).max()) if plain.any() else 0.0
    assert worst <= GRAD_RTOL[dt], \
        f"{what} d_logits: relative error {worst:.3g} on an element without cancellation"
    return worst


def seeded_logits(shape, dtype, scale=2.0, seed=0, offset=0.0):
    g = torch.Generator().manual_seed(seed)
    return (torch.randn(shape, generator=g) * scale + offset).to(dtype)


def seeded_targets(shape, vocab, seed=1):
    g = torch.Generator().manual_seed(seed)
    return torch.randint(0, vocab, shape, generator=g)


def grads_like(shape, seed=2, scale=0.5):
    g = torch.Generator().manual_seed(seed)
    return tuple(torch.randn(shape, generator=g) * scale for _ in range(3))

"""GPU parity helpers: run the CUDA path, compare with the fp64 oracle.

Tolerances (north star of this port, against fp64 ground truth):
  * logprob and lse: 1e-5 absolute (fp32 accumulation, whatever the input dtype);
  * entropy: 1e-4 relative (plus 1e-7 absolute for rows whose entropy is exactly 0);
  * d_logits: 1e-5 relative for fp32, 1e-2 relative for bf16 / fp16, with an absolute
    floor of 1e-7 x the largest gradient magnitude (elements whose coefficient
    g_lse - g_logp - g_ent (log p + H) passes through zero have no relative accuracy in
    any fp32 evaluation) and, for fp16, half of fp16's subnormal spacing (2.98e-8),
    below which fp16 cannot represent the value at all.  Elements 100x above the floor
    must meet the relative tolerance alone (check_grad returns their worst error).
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
    # The absolute floor only covers elements near it: those 100x above it must meet the
    # relative tolerance on their own.  Returned so callers can report it.
    big = finite & (np.abs(d0) >= 100.0 * atol) & np.isfinite(got)
    worst = float((np.abs(got[big] - d0[big]) / np.abs(d0[big])).max()) if big.any() else 0.0
    assert worst <= GRAD_RTOL[dt], f"{what} d_logits: relative error {worst:.3g} above the floor"
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

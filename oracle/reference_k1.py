"""TEST INFRASTRUCTURE ONLY.  Loader for the reference's own K1 kernels rebuilt for
sm_100a by oracle/build_ref.py.  Returns None when the build is absent.

The reference binding takes contiguous CUDA tensors and out-parameters
(reference csrc/bindings.cpp:17-26):
  fused_logprob_entropy_v1(logits, targets, logprob, entropy, lse)
  fused_logprob_entropy_naive(logits, targets, logprob, entropy, lse)
  fused_logprob_entropy_v1_backward(logits, targets, lse, entropy, g_logp, g_ent, g_lse,
                                    d_logits)
"""
from __future__ import annotations

import importlib.util
import os

from .build_ref import NAME, built_path

_mod = None


def load():
    global _mod
    if _mod is None:
        path = built_path()
        if path is None or not os.path.exists(path):
            return None
        import torch  # noqa: F401  (torch libraries first)
        spec = importlib.util.spec_from_file_location(NAME, path)
        _mod = importlib.util.module_from_spec(spec)
        spec.loader.exec_module(_mod)
    return _mod


def forward(logits, targets):
    """Reference v1 forward on contiguous CUDA tensors -> (logp, entropy, lse) fp32."""
    import torch
    m = load()
    lp = torch.empty(targets.shape, device=logits.device, dtype=torch.float32)
    h, l = torch.empty_like(lp), torch.empty_like(lp)
    m.fused_logprob_entropy_v1(logits.contiguous(), targets.contiguous(), lp, h, l)
    return lp, h, l


def backward(logits, targets, lse, entropy, g_logp, g_ent, g_lse):
    import torch
    m = load()
    d = torch.empty_like(logits.contiguous())
    m.fused_logprob_entropy_v1_backward(logits.contiguous(), targets.contiguous(), lse, entropy,
                                        g_logp.contiguous(), g_ent.contiguous(),
                                        g_lse.contiguous(), d)
    return d


def autograd_function():
    """torch.autograd.Function over the reference kernels, following the reference's own
    wrapper (python/kernel_opt/ops.py:49-89): forward saves (logits, targets, lse,
    entropy); backward replaces missing upstream gradients by zero tensors, allocates
    d_logits with empty_like and calls the reference backward kernel.  Returns None when
    the build is absent."""
    import torch
    if load() is None:
        return None

    class RefFusedLogprobEntropy(torch.autograd.Function):
        @staticmethod
        def forward(ctx, logits, targets):
            lp, h, l = forward(logits, targets)
            ctx.save_for_backward(logits, targets, l, h)
            return lp, h, l

        @staticmethod
        def backward(ctx, g_logp, g_ent, g_lse):
            logits, targets, l, h = ctx.saved_tensors
            z = torch.zeros_like(l)
            g_logp = z if g_logp is None else g_logp.float().contiguous()
            g_ent = z if g_ent is None else g_ent.float().contiguous()
            g_lse = z if g_lse is None else g_lse.float().contiguous()
            return backward(logits, targets, l, h, g_logp, g_ent, g_lse), None

    return RefFusedLogprobEntropy

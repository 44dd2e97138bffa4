"""Generate tests/golden/k1_golden.npz -- small, seeded K1 cases with fp64 answers.

The answers come from the reference tests' own ground truth, restated in torch fp64:
`_ref_fp32` (log_softmax -> gather, -sum p log p, logsumexp; reference
tests/test_logprob.py:17-25) and autograd through `_ref_forward_pt` with the loss
sum(logp g_logp + H g_ent + lse g_lse) (tests/test_logprob.py:160-167,184-189).  This
is independent of the C oracle, which the CPU tests check against these files.
Edge rules that torch cannot express directly follow the reference kernels: a target
outside [0, V) reads a logit of 0 (csrc/fused_logprob.cu:179-185), and -inf logits
contribute nothing (csrc/fused_logprob.cu:141-143).

Inputs are stored as raw bits (bf16 / fp16 as uint16, fp32 as float32) so the files do
not depend on torch's RNG.  Run: python tests/golden/make_golden.py
"""
from __future__ import annotations

import os

import numpy as np
import torch
import torch.nn.functional as F

OUT = os.path.join(os.path.dirname(os.path.abspath(__file__)), "k1_golden.npz")
DT = {"f32": torch.float32, "f16": torch.float16, "bf16": torch.bfloat16}


def ground_truth(logits: torch.Tensor, targets: torch.Tensor, g=None):
    """fp64 (logp, H, lse[, d_logits]) with the reference kernels' edge rules."""
    x = logits.detach().double().requires_grad_(g is not None)
    V = x.shape[-1]
    logz = torch.logsumexp(x, dim=-1)
    log_probs = x - logz.unsqueeze(-1)
    p = log_probs.exp()
    # p log p -> 0 where p == 0 (x = -inf); the inner where keeps autograd free of 0 * inf
    plogp = p * torch.where(p > 0, log_probs, torch.zeros_like(log_probs))
    ent = -plogp.sum(-1)
    valid = (targets >= 0) & (targets < V)
    safe_t = torch.where(valid, targets, torch.zeros_like(targets))
    x_t = torch.where(valid, x.gather(-1, safe_t.unsqueeze(-1)).squeeze(-1), torch.zeros_like(logz))
    logp = x_t - logz
    out = [logp.detach(), ent.detach(), logz.detach()]
    if g is not None:
        g_logp, g_ent, g_lse = (t.double() for t in g)
        loss = (logp * g_logp + ent * g_ent + logz * g_lse).sum()
        (d,) = torch.autograd.grad(loss, x)
        out.append(d)
    return [o.numpy() for o in out]


def raw_bits(t: torch.Tensor) -> np.ndarray:
    if t.dtype == torch.float32:
        return t.numpy().copy()
    return t.view(torch.int16).numpy().view(np.uint16).copy()


def main():
    cases = {}

    def add(name, logits, targets, g=None):
        gt = ground_truth(logits, targets, g)
        cases[f"{name}/x"] = raw_bits(logits)
        cases[f"{name}/dtype"] = np.array(str(logits.dtype).replace("torch.", ""))
        cases[f"{name}/shape"] = np.array(logits.shape, np.int64)
        cases[f"{name}/targets"] = targets.numpy()
        cases[f"{name}/logp"], cases[f"{name}/entropy"], cases[f"{name}/lse"] = gt[:3]
        if g is not None:
            for k, v in zip(("g_logp", "g_ent", "g_lse"), g):
                cases[f"{name}/{k}"] = v.numpy()
            cases[f"{name}/d_logits"] = gt[3]

    gen = torch.Generator().manual_seed(0)
    # Shapes and value spreads of the reference's forward tests (tests/test_logprob.py:28-35,
    # 114-122), scaled down to keep the fixture small.
    for dt, shape in (("f32", (2, 3, 1000)), ("bf16", (1, 4, 4096)), ("f16", (1, 2, 8192)),
                      ("bf16", (1, 1, 32000))):
        x = (torch.randn(shape, generator=gen) * 2.0).to(DT[dt])
        t = torch.randint(0, shape[-1], shape[:-1], generator=gen)
        g = tuple(torch.randn(shape[:-1], generator=gen) * 0.5 for _ in range(3))
        add(f"rand_{dt}_{'x'.join(map(str, shape))}", x, t, g)

    # Known answer: zero logits -> H = lse = log V (tests/test_logprob.py:140-152).
    add("uniform_f32_4096", torch.zeros(1, 1, 4096), torch.zeros(1, 1, dtype=torch.int64))

    # Large offset must stay finite (tests/test_logprob.py:101-111).
    x = torch.randn(1, 4, 1024, generator=gen) + 60.0
    add("offset60_f32", x, torch.randint(0, 1024, (1, 4), generator=gen))

    # Edge rows: targets out of range, -inf entries, one near-one-hot row, V not a
    # multiple of the 16-byte vector, a single column.
    V = 1003
    x = torch.randn(5, V, generator=gen) * 2.0
    x[1, ::7] = float("-inf")
    x[2, 17] += 40.0
    t = torch.tensor([-100, 5, 17, V, V - 1])
    g = tuple(torch.randn(5, generator=gen) * 0.5 for _ in range(3))
    add("edge_f32_1003", x, t, g)
    xb = x.to(torch.bfloat16)
    add("edge_bf16_1003", xb, t, g)
    add("single_col_f32", torch.randn(3, 1, generator=gen), torch.tensor([0, 0, -1]))

    np.savez_compressed(OUT, **cases)
    print(f"wrote {OUT}: {len([k for k in cases if k.endswith('/x')])} cases")


if __name__ == "__main__":
    main()

"""TEST INFRASTRUCTURE / CPU BASELINE ONLY.  Restatement of the path K1 replaces:
TRL 1.4's `selective_log_softmax` + `entropy_from_logits`, run eagerly with torch.

TRL (pinned at 1.4.0 by the reference, notes/stage1_findings.md:6) is not installed
here, so this is written from the reference's own description of that code
(notes/stage1_findings.md:24-62, REPORT.md:19-30), not from TRL's source:
  * log-probs, bf16 / fp16 input: a Python loop over the leading batch dimension, each
    step a full log_softmax of one [L, V] slice in the input dtype, then a gather;
  * log-probs, fp32 / fp64 input: gather minus a per-batch-element logsumexp;
  * entropy: the flattened [N, V] rows in chunks of 128; per chunk log_softmax,
    then -(exp(logp) * logp).sum(-1), output in the input dtype.
The backward is torch autograd through that forward.  The reference's call sites are
tests/test_logprob.py:68,78-79 and bench/bench_micro.py:103-106.
"""
from __future__ import annotations

import torch
import torch.nn.functional as F


def selective_log_softmax(logits: torch.Tensor, index: torch.Tensor) -> torch.Tensor:
    if logits.dtype in (torch.float32, torch.float64):
        picked = torch.gather(logits, -1, index.unsqueeze(-1)).squeeze(-1)
        norm = torch.stack([torch.logsumexp(row, dim=-1) for row in logits])
        return picked - norm
    rows = []
    for row_logits, row_index in zip(logits, index):
        row_logp = F.log_softmax(row_logits, dim=-1)
        rows.append(row_logp.gather(-1, row_index.unsqueeze(-1)).squeeze(-1))
    return torch.stack(rows)


def entropy_from_logits(logits: torch.Tensor, chunk_size: int = 128) -> torch.Tensor:
    flat = logits.reshape(-1, logits.shape[-1])
    parts = []
    for chunk in flat.split(chunk_size, dim=0):
        logp = F.log_softmax(chunk, dim=-1)
        parts.append(-(torch.exp(logp) * logp).sum(-1))
    return torch.cat(parts).reshape(logits.shape[:-1])


def forward(logits: torch.Tensor, targets: torch.Tensor):
    """(logp, entropy) the way the TRL path computes them."""
    return selective_log_softmax(logits, targets), entropy_from_logits(logits)


def forward_backward(logits: torch.Tensor, targets: torch.Tensor, g_logp: torch.Tensor,
                     g_ent: torch.Tensor):
    """One forward + backward step; returns (logp, entropy, d_logits)."""
    x = logits.detach().requires_grad_(True)
    logp, ent = forward(x, targets)
    loss = (logp.float() * g_logp).sum() + (ent.float() * g_ent).sum()
    loss.backward()
    return logp.detach(), ent.detach(), x.grad

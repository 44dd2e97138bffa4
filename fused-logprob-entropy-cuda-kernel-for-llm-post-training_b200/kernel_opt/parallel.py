"""Multi-GPU K1 on one node: one process per GPU, torch.distributed over NCCL.

Two modes (no counterpart in the reference, which is single-GPU only):

Row-sharded.  Rows (B*S) are independent, so each rank runs K1 on its own contiguous
block of rows and nothing is exchanged.  `row_shard` gives the block.

Vocab-parallel (tensor-parallel LM head layout).  Rank k holds the columns
[vocab_offset_k, vocab_offset_k + V_k) of every row.  The forward is
  1. per-row partial state of the local shard (m, z, t, target logit if owned) --
     one streaming pass over the shard (`_C.vocab_shard_partials`);
  2. ONE collective: all-gather of the [N, 4] float64 partials (32 bytes per row);
  3. the associative merge of the gathered partials into (logprob, entropy, lse),
     identical on every rank (`_C.vocab_combine`).
A single all-gather carries everything: NCCL has no reduction operator for the
(max, sum-exp, sum-exp*x) triple, so a one-collective all-reduce is not available, and
the max + sum pair of all-reduces would be two collectives.  The backward is local to
each shard, with the one-hot term applied only on the rank that owns the target.
"""
from __future__ import annotations

import torch
import torch.distributed as dist

from kernel_opt import _C

PARTIAL_WORDS = 4  # one k1_partial (include/k1_logprob.h) = 4 float64 words


def row_shard(n_rows: int, world_size: int, rank: int) -> slice:
    """Contiguous, near-equal block of rows owned by `rank` (first n_rows % world_size
    ranks get one extra row)."""
    if world_size < 1 or not (0 <= rank < world_size):
        raise ValueError(f"bad rank {rank} for world size {world_size}")
    base, extra = divmod(n_rows, world_size)
    start = rank * base + min(rank, extra)
    return slice(start, start + base + (1 if rank < extra else 0))


def vocab_shard(vocab: int, world_size: int, rank: int) -> slice:
    """Contiguous columns of the full vocabulary held by `rank` (same rule as rows)."""
    return row_shard(vocab, world_size, rank)


def exchange_partials(partials: torch.Tensor, group=None) -> torch.Tensor:
    """Step 2: all-gather [N, 4] float64 partials into [world, N, 4] (rank-major).  Without
    an initialised process group (one process holding the whole vocabulary) there is
    nothing to exchange: [1, N, 4]."""
    n = partials.shape[0]
    if group is None and not (dist.is_available() and dist.is_initialized()):
        return partials.contiguous().view((1, n) + tuple(partials.shape[1:]))
    world = dist.get_world_size(group)
    out = torch.empty((world * n,) + tuple(partials.shape[1:]), dtype=partials.dtype,
                      device=partials.device)
    dist.all_gather_into_tensor(out, partials.contiguous(), group=group)
    return out.view((world, n) + tuple(partials.shape[1:]))


class _VocabParallelLogprobEntropy(torch.autograd.Function):
    @staticmethod
    def forward(ctx, logits_shard, targets, vocab_offset, group):
        assert logits_shard.is_cuda and targets.is_cuda
        assert targets.dtype == torch.int64
        assert logits_shard.shape[:-1] == targets.shape
        targets = targets.contiguous()
        n_rows = targets.numel()
        partials = torch.empty((n_rows, PARTIAL_WORDS), dtype=torch.float64,
                               device=logits_shard.device)
        _C.vocab_shard_partials(logits_shard, targets, int(vocab_offset), partials)
        gathered = exchange_partials(partials, group)
        shape = targets.shape
        logprob = torch.empty(shape, dtype=torch.float32, device=targets.device)
        entropy = torch.empty_like(logprob)
        lse = torch.empty_like(logprob)
        _C.vocab_combine(gathered, gathered.shape[0], logprob, entropy, lse)
        ctx.save_for_backward(logits_shard, targets, lse, entropy)
        ctx.vocab_offset = int(vocab_offset)
        ctx.set_materialize_grads(False)
        return logprob, entropy, lse

    @staticmethod
    def backward(ctx, g_logp, g_ent, g_lse):
        logits_shard, targets, lse, entropy = ctx.saved_tensors

        def _prep(g):
            return None if g is None else g.to(torch.float32, copy=False).contiguous()

        d_logits = torch.empty_like(logits_shard)
        _C.vocab_shard_backward(logits_shard, targets, ctx.vocab_offset, lse, entropy,
                                _prep(g_logp), _prep(g_ent), _prep(g_lse), d_logits)
        return d_logits, None, None, None


def vocab_parallel_fused_logprob_entropy(logits_shard: torch.Tensor, targets: torch.Tensor,
                                         vocab_offset: int, group=None):
    """K1 over a vocabulary-sharded [..., V_k] slice of the logits.

    `targets` hold global token ids (identical on every rank); `vocab_offset` is the
    global id of this shard's first column.  Returns the full-vocabulary
    (logprob, entropy, lse) on every rank; gradients flow to `logits_shard` only.
    Every rank of `group` must call this with the same row count.
    """
    return _VocabParallelLogprobEntropy.apply(logits_shard, targets, vocab_offset, group)

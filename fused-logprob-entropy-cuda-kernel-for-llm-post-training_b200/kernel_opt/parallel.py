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

Vocab-parallel LM head (`vocab_parallel_fused_linear_logprob_entropy`).  The same split
one step earlier: rank k holds rows [vocab_offset_k, vocab_offset_k + V_k) of the head's
weight, and step 1 computes the shard's partials in the epilogue of the tensor-core
LM-head kernel, so no rank writes logits in the forward.  The backward recomputes the
shard's logits gradient on the tensor cores; the hidden state's gradient is the sum of
the shards' parts, one all-reduce.
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


class _VocabParallelLinearLogprobEntropy(torch.autograd.Function):
    """The tensor-parallel LM head fused with K1 (bf16): this rank holds rows
    [vocab_offset, vocab_offset + V_k) of the head's [V, H] weight; `hidden` is the same on
    every rank.  No rank ever holds an [N, V] or [N, V_k] logits tensor in the forward."""

    @staticmethod
    def forward(ctx, hidden, weight_shard, targets, vocab_offset, scale, group, chunk_rows,
                keep_logits):
        n = hidden.shape[0]
        partials = torch.empty((n, PARTIAL_WORDS), dtype=torch.float64, device=hidden.device)
        grad = ctx.needs_input_grad[0] or ctx.needs_input_grad[1]
        z = torch.empty((n, weight_shard.shape[0]), dtype=hidden.dtype, device=hidden.device) \
            if (keep_logits and grad) else None
        _C.lm_head_shard_partials(hidden, weight_shard, targets, int(vocab_offset), partials,
                                  scale, z)
        gathered = exchange_partials(partials, group)
        logprob = torch.empty((n,), dtype=torch.float32, device=hidden.device)
        entropy = torch.empty_like(logprob)
        lse = torch.empty_like(logprob)
        _C.vocab_combine(gathered, gathered.shape[0], logprob, entropy, lse)
        ctx.save_for_backward(hidden, weight_shard, targets, lse, entropy,
                              z if z is not None else lse.new_empty(0))
        ctx.keep = z is not None
        ctx.vocab_offset = int(vocab_offset)
        ctx.scale = scale
        ctx.group = group
        ctx.chunk_rows = chunk_rows
        ctx.set_materialize_grads(False)
        ctx.mark_non_differentiable(lse)
        return logprob, entropy, lse

    @staticmethod
    def backward(ctx, g_logp, g_ent, _g_lse):
        from .lm_head import _chunks, default_chunk_rows

        hidden, w, targets, lse, entropy, z = ctx.saved_tensors
        need_h, need_w = ctx.needs_input_grad[0], ctx.needs_input_grad[1]
        if (g_logp is None and g_ent is None) or not (need_h or need_w):
            return None, None, None, None, None, None, None, None
        gl = None if g_logp is None else g_logp.to(torch.float32).contiguous()
        ge = None if g_ent is None else g_ent.to(torch.float32).contiguous()
        distributed = ctx.group is not None or (dist.is_available() and dist.is_initialized())
        if ctx.keep:
            # K1's backward in place on the kept logits shard, then the library GEMMs
            _C.vocab_shard_backward(z, targets, ctx.vocab_offset, lse, entropy, gl, ge, None, z,
                                    ctx.scale)
            dh = None
            if need_h:
                dh32 = torch.mm(z, w, out_dtype=torch.float32)
                if distributed:
                    dist.all_reduce(dh32, group=ctx.group)
                dh = dh32.to(hidden.dtype)
            dw = torch.mm(z.t(), hidden) if need_w else None
            return dh, dw, None, None, None, None, None, None
        n, vk = hidden.shape[0], w.shape[0]
        c = min(max(1, n), ctx.chunk_rows or default_chunk_rows(n, vk, w.element_size()))
        dz = torch.empty((c, vk), dtype=hidden.dtype, device=hidden.device)
        dh32 = torch.empty(hidden.shape, dtype=torch.float32, device=hidden.device) if need_h else None
        dw32 = torch.zeros(w.shape, dtype=torch.float32, device=w.device) if need_w else None
        for a, b in _chunks(n, c):
            d = dz[: b - a]
            _C.lm_head_shard_backward(hidden[a:b], w, targets[a:b], ctx.vocab_offset, lse[a:b],
                                      entropy[a:b], None if gl is None else gl[a:b],
                                      None if ge is None else ge[a:b], None, d, ctx.scale)
            if need_h:
                dh32[a:b] = torch.mm(d, w, out_dtype=torch.float32)
            if need_w:
                torch.addmm(dw32, d.t(), hidden[a:b], out_dtype=torch.float32, out=dw32)
        dh = None
        if need_h:
            # this shard's part of dL/dhidden; the sum over the shards is the gradient
            if distributed:
                dist.all_reduce(dh32, group=ctx.group)
            dh = dh32.to(hidden.dtype)
        dw = dw32.to(w.dtype) if need_w else None
        return dh, dw, None, None, None, None, None, None


def vocab_parallel_fused_linear_logprob_entropy(hidden: torch.Tensor, weight_shard: torch.Tensor,
                                                targets: torch.Tensor, vocab_offset: int,
                                                temperature: float = 1.0, group=None,
                                                chunk_rows: int | None = None,
                                                keep_logits: bool = False):
    """The LM head fused with K1, split over the vocabulary (tensor-parallel layout).

    hidden: [..., H] bf16, identical on every rank of `group`; weight_shard: [V_k, H] bf16,
    rows [vocab_offset, vocab_offset + V_k) of the head's [V, H] weight; targets: [...]
    int64 global token ids.  Returns the full-vocabulary (logprob, entropy, lse) of
    softmax((hidden @ W.T) / temperature) on every rank, shaped like `targets`.

    Forward: each rank computes its shard's per-row partial state on the tensor cores (the
    logits never reach memory), ONE all-gather of the [N, 4] float64 partials, and the
    combine.  Backward: each rank recomputes its shard's logits gradient row chunk by row
    chunk (`chunk_rows`, default at most 1 GiB of gradient), forms dL/dweight_shard locally
    and its part of dL/dhidden, and ONE all-reduce (fp32) sums the parts, so every rank
    gets the full dL/dhidden.  `keep_logits=True` trades memory for time as in
    `fused_linear_logprob_entropy`: the forward also stores this rank's [N, V_k] logits shard
    and the backward runs K1's backward in place on it instead of recomputing the GEMM.
    Every rank must call this with the same shapes and the same requires_grad flags (the
    collectives pair up across ranks).
    """
    from .grpo import temperature_scale

    lead = targets.shape
    h2 = hidden.reshape(-1, hidden.shape[-1])
    if not h2.is_contiguous():
        h2 = h2.contiguous()
    w = weight_shard if weight_shard.is_contiguous() else weight_shard.contiguous()
    t1 = targets.reshape(-1).contiguous()
    lp, ent, lse = _VocabParallelLinearLogprobEntropy.apply(
        h2, w, t1, int(vocab_offset), temperature_scale(temperature), group, chunk_rows,
        bool(keep_logits))
    return lp.view(lead), ent.view(lead), lse.view(lead)

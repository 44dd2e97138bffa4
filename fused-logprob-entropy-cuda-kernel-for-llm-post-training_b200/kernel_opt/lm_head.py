"""LM head + K1 without the [N, V] logits tensor.

The reference computes K1 on logits that the model has already materialised
(`model(**inputs).logits`, python/kernel_opt/trainer.py:96); it names fusing the LM-head
projection with K1 as the follow-up that would remove that tensor (README.md:135-136,
docs/FINAL_REPORT.md:490-494).

bf16 heads (the training case) run on the tensor-core kernel of csrc/k1_lmhead.cuh
(`_C.lm_head_forward` / `_C.lm_head_backward`): a tcgen05 GEMM whose epilogue folds every
128 x 256 tile of the logits straight into K1's per-row statistics, so the forward never
writes the logits to memory, and whose backward mode recomputes the tiles and writes K1's
gradient w.r.t. them.

  forward           z = bf16(h W^T), K1 statistics of bf16(z / T) in the GEMM epilogue
  backward          per row chunk: dz = K1 gradient from the recomputed tiles (tensor
                    cores), then dh_c = dz W, dW += dz^T h_c (library GEMMs, fp32 dW)
  keep_logits=True  the forward also writes z; the backward is K1's in-place backward on
                    it and two library GEMMs (memory of materialised logits, one GEMM less)

Other dtypes (fp16, fp32) keep the composition of library GEMMs and K1 kernels on row
chunks: each chunk's logits are produced into one reused buffer and consumed there by K1.

Chunk size (the backward's dz buffer, and the whole path for other dtypes) is a memory
budget (default 1 GiB), in multiples of 256 rows and equalised: every chunk's GEMMs
stream all of W and read and write the fp32 dW accumulator, so chunks small enough to
stay in L2 would make the GEMMs memory-bound.
"""
from __future__ import annotations

import torch

from kernel_opt import _C

from .grpo import temperature_scale
from .ops import _alloc_outputs

CHUNK_BUDGET_BYTES = 1 << 30  # logits buffer of one chunk
ROW_QUANTUM = 256             # chunk rows are a multiple of the GEMM's M tiles


def default_chunk_rows(n_rows: int, vocab: int, elem_size: int,
                       budget_bytes: int = CHUNK_BUDGET_BYTES) -> int:
    """Rows per chunk: split n_rows into the fewest chunks whose logits fit budget_bytes,
    equal sizes rounded up to a multiple of ROW_QUANTUM (at least one quantum)."""
    per_row = max(1, vocab * elem_size)
    cap = max(ROW_QUANTUM, (budget_bytes // per_row) // ROW_QUANTUM * ROW_QUANTUM)
    n_chunks = max(1, -(-n_rows // cap))
    rows = -(-n_rows // n_chunks)
    return min(cap, max(ROW_QUANTUM, -(-rows // ROW_QUANTUM) * ROW_QUANTUM))


def _chunks(n: int, c: int):
    for a in range(0, n, c):
        yield a, min(n, a + c)


class _LinearLogprobEntropy(torch.autograd.Function):
    @staticmethod
    def forward(ctx, hidden, weight, targets, scale, chunk_rows):
        if hidden.dim() != 2 or weight.dim() != 2 or hidden.shape[1] != weight.shape[1]:
            raise ValueError(f"hidden [N, H] and weight [V, H] expected, got "
                             f"{tuple(hidden.shape)} and {tuple(weight.shape)}")
        if hidden.dtype != weight.dtype:
            raise ValueError("hidden and weight must have the same dtype")
        if targets.shape != hidden.shape[:1]:
            raise ValueError("targets must have one entry per hidden row")
        N, V = hidden.shape[0], weight.shape[0]
        targets = targets.contiguous()
        logprob, entropy, lse = _alloc_outputs(targets)
        c = min(max(1, N), chunk_rows)
        zbuf = torch.empty((c, V), dtype=hidden.dtype, device=hidden.device)
        wt = weight.t()
        for a, b in _chunks(N, c):
            z = zbuf[: b - a]
            torch.mm(hidden[a:b], wt, out=z)
            _C.fused_logprob_entropy_scaled(z, targets[a:b], logprob[a:b], entropy[a:b],
                                            lse[a:b], scale)
        ctx.save_for_backward(hidden, weight, targets, lse, entropy)
        ctx.scale = scale
        ctx.chunk_rows = c
        ctx.set_materialize_grads(False)
        ctx.mark_non_differentiable(lse)
        return logprob, entropy, lse

    @staticmethod
    def backward(ctx, g_logp, g_ent, _g_lse):
        hidden, weight, targets, lse, entropy = ctx.saved_tensors
        need_h, need_w = ctx.needs_input_grad[0], ctx.needs_input_grad[1]
        if (g_logp is None and g_ent is None) or not (need_h or need_w):
            return None, None, None, None, None
        gl = None if g_logp is None else g_logp.to(torch.float32).contiguous()
        ge = None if g_ent is None else g_ent.to(torch.float32).contiguous()
        N, V = hidden.shape[0], weight.shape[0]
        c = ctx.chunk_rows
        zbuf = torch.empty((c, V), dtype=hidden.dtype, device=hidden.device)
        dh = torch.empty_like(hidden) if need_h else None
        dw32 = torch.zeros(weight.shape, dtype=torch.float32, device=weight.device) if need_w else None
        wt = weight.t()
        for a, b in _chunks(N, c):
            z = zbuf[: b - a]
            torch.mm(hidden[a:b], wt, out=z)
            _C.fused_logprob_entropy_scaled_backward(
                z, targets[a:b], lse[a:b], entropy[a:b],
                None if gl is None else gl[a:b], None if ge is None else ge[a:b], None,
                z, ctx.scale)
            if need_h:
                torch.mm(z, weight, out=dh[a:b])
            if need_w:
                if weight.dtype == torch.float32:
                    dw32.addmm_(z.t(), hidden[a:b])
                else:
                    torch.addmm(dw32, z.t(), hidden[a:b], out_dtype=torch.float32, out=dw32)
        dw = None
        if need_w:
            dw = dw32 if weight.dtype == torch.float32 else dw32.to(weight.dtype)
        return dh, dw, None, None, None


def tensor_core_head(hidden: torch.Tensor, weight: torch.Tensor) -> bool:
    """Whether the tcgen05 kernel serves this head: bf16 [N, H] x [V, H], H % 8 == 0."""
    return (hidden.dtype == torch.bfloat16 and weight.dtype == torch.bfloat16 and
            hidden.is_cuda and weight.is_cuda and hidden.shape[-1] % 8 == 0)


class _TCLinearLogprobEntropy(torch.autograd.Function):
    """The tensor-core path (bf16).  See the module docstring."""

    @staticmethod
    def forward(ctx, hidden, weight, targets, scale, chunk_rows, keep_logits):
        N, V = hidden.shape[0], weight.shape[0]
        targets = targets.contiguous()
        logprob, entropy, lse = _alloc_outputs(targets)
        grad = ctx.needs_input_grad[0] or ctx.needs_input_grad[1]
        z = torch.empty((N, V), dtype=hidden.dtype, device=hidden.device) \
            if (keep_logits and grad) else None
        _C.lm_head_forward(hidden, weight, targets, logprob, entropy, lse, scale, z)
        ctx.save_for_backward(hidden, weight, targets, lse, entropy,
                              z if z is not None else lse.new_empty(0))
        ctx.keep = z is not None
        ctx.scale = scale
        ctx.chunk_rows = min(max(1, N), chunk_rows)
        ctx.set_materialize_grads(False)
        ctx.mark_non_differentiable(lse)
        return logprob, entropy, lse

    @staticmethod
    def backward(ctx, g_logp, g_ent, _g_lse):
        hidden, weight, targets, lse, entropy, z = ctx.saved_tensors
        need_h, need_w = ctx.needs_input_grad[0], ctx.needs_input_grad[1]
        if (g_logp is None and g_ent is None) or not (need_h or need_w):
            return None, None, None, None, None, None
        gl = None if g_logp is None else g_logp.to(torch.float32).contiguous()
        ge = None if g_ent is None else g_ent.to(torch.float32).contiguous()
        if ctx.keep:
            # K1's backward in place on the kept logits, then the two library GEMMs that
            # autograd would run for z = h W^T
            _C.fused_logprob_entropy_scaled_backward(z, targets, lse, entropy, gl, ge, None, z,
                                                     ctx.scale)
            dh = torch.mm(z, weight) if need_h else None
            dw = torch.mm(z.t(), hidden) if need_w else None
            return dh, dw, None, None, None, None
        N, V = hidden.shape[0], weight.shape[0]
        c = ctx.chunk_rows
        dz = torch.empty((c, V), dtype=hidden.dtype, device=hidden.device)
        dh = torch.empty_like(hidden) if need_h else None
        dw32 = torch.zeros(weight.shape, dtype=torch.float32, device=weight.device) if need_w else None
        for a, b in _chunks(N, c):
            d = dz[: b - a]
            _C.lm_head_backward(hidden[a:b], weight, targets[a:b], lse[a:b], entropy[a:b],
                                None if gl is None else gl[a:b], None if ge is None else ge[a:b],
                                None, d, ctx.scale)
            if need_h:
                torch.mm(d, weight, out=dh[a:b])
            if need_w:
                torch.addmm(dw32, d.t(), hidden[a:b], out_dtype=torch.float32, out=dw32)
        dw = dw32.to(weight.dtype) if need_w else None
        return dh, dw, None, None, None, None


# Config attributes that make the logits something other than hidden @ W^T
_LOGIT_TRANSFORMS = ("final_logit_softcapping", "logit_scale", "logits_scaling",
                     "output_multiplier_scale")


def fused_head_parts(model):
    """(decoder, head weight) when `model`'s logits are exactly decoder(x) @ W^T, else None."""
    get_dec = getattr(model, "get_decoder", None)
    get_head = getattr(model, "get_output_embeddings", None)
    if get_dec is None or get_head is None:
        return None
    head = get_head()
    dec = get_dec()
    if not isinstance(head, torch.nn.Linear) or head.bias is not None or dec is None:
        return None
    cfg = getattr(model, "config", None)
    if any(getattr(cfg, a, None) not in (None, 1, 1.0) for a in _LOGIT_TRANSFORMS):
        return None
    return dec, head.weight


def fused_linear_logprob_entropy(hidden: torch.Tensor, weight: torch.Tensor,
                                 targets: torch.Tensor, temperature: float = 1.0,
                                 chunk_rows: int | None = None, keep_logits: bool = False):
    """Per-row log-prob of `targets`, entropy and log-sum-exp of
    softmax((hidden @ weight.T) / temperature), with gradients to `hidden` and `weight`.

    hidden: [..., H], weight: [V, H] (an nn.Linear's weight, no bias), same dtype;
    targets: [...] int64 (ignore index -100 allowed).  Returns (logprob, entropy, lse)
    shaped like `targets`.  The logits are rounded to the weight's dtype (as a model's
    logits are) and divided by the temperature with the rounding of an in-place
    `div_(temperature)`, so results equal K1 on the materialised, divided logits.

    bf16 heads run on the tensor-core kernel: the forward never writes the logits; the
    backward recomputes them chunk by chunk (`chunk_rows` rows of gradient at a time;
    default: the fewest equal chunks of at most 1 GiB).  `keep_logits=True` trades memory
    for time: the forward also writes the [N, V] logits and the backward reuses them.
    Other dtypes run library GEMMs and K1 kernels on row chunks.
    """
    lead = targets.shape
    h2 = hidden.reshape(-1, hidden.shape[-1])
    if not h2.is_contiguous():
        h2 = h2.contiguous()
    t1 = targets.reshape(-1)
    c = chunk_rows or default_chunk_rows(h2.shape[0], weight.shape[0], weight.element_size())
    scale = temperature_scale(temperature)
    if tensor_core_head(h2, weight):
        w = weight if weight.is_contiguous() else weight.contiguous()
        lp, h, l = _TCLinearLogprobEntropy.apply(h2, w, t1, scale, c, bool(keep_logits))
    else:
        lp, h, l = _LinearLogprobEntropy.apply(h2, weight, t1, scale, c)
    return lp.view(lead), h.view(lead), l.view(lead)

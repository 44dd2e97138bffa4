"""The K1 call inside GRPO's logprob method, usable without `trl`.

The reference trainer slices the model's [B, L, V] logits to the completion window,
which leaves a view whose batch stride is still L*V, divides that view by the sampling
temperature in place and then calls K1 once per batch element to avoid copying it
(python/kernel_opt/trainer.py:96-127).  Its backward therefore runs K1's backward per
element, the in-place division's backward (a clone of the parent-shaped gradient plus a
scaled copy of the window) and the slice's backward (a zero-filled parent-shaped
gradient and a copy of the window into it).

`window_logps_and_entropies` does the same computation as one autograd node on the
parent tensor: one forward launch over the strided window with the temperature applied
while the logits stream in (every logit rounded exactly as the in-place division rounds
it), and one backward launch that writes the gradient of the window straight into a
parent-shaped buffer (zeroing only the rows outside the window).  With
`inplace_backward=True` that buffer is the logits' own storage, so the loss block needs
no second [B, L, V] tensor at all.
"""
from __future__ import annotations

import numpy as np
import torch

from kernel_opt import _C

from .ops import _alloc_outputs, _check_inputs

MULTIMODAL_KWARGS = (
    "pixel_values", "image_grid_thw", "num_images",
    "pixel_attention_mask", "image_sizes",
    "token_type_ids", "mm_token_type_ids", "image_position_ids",
)


def completion_window(logits: torch.Tensor, logits_to_keep: int) -> torch.Tensor:
    """Drop the last position and keep the completion window, as TRL does
    (reference trainer.py:98-99).  Returns a view; no copy."""
    logits = logits[:, :-1, :]
    return logits[:, -logits_to_keep:, :]


def temperature_scale(temperature: float) -> float:
    """The factor torch multiplies by when it divides a CUDA tensor by the Python scalar
    `temperature`: 1 / temperature taken in double precision, then rounded to fp32
    (not 1.0f / (float)temperature, which differs in the last bit for e.g. 0.85)."""
    t = float(temperature)
    if not (np.isfinite(t) and t > 0):
        raise ValueError(f"temperature must be positive and finite, got {temperature!r}")
    s = np.float32(1.0 / t)
    if not (np.isfinite(s) and s > 0):
        raise ValueError(f"temperature {temperature!r} has no finite positive fp32 reciprocal")
    return float(s)


def _prep(g):
    return None if g is None else g.to(torch.float32, copy=False).contiguous()


class _WindowLogprobEntropy(torch.autograd.Function):
    """K1 on completion_window(logits, k) scaled by `scale`, differentiated with respect
    to the whole parent tensor `logits` [B, L, V]."""

    @staticmethod
    def forward(ctx, logits, completion_ids, logits_to_keep, scale, inplace_backward):
        if logits.dim() != 3:
            raise ValueError(f"logits must be [B, L, V], got shape {tuple(logits.shape)}")
        if inplace_backward and logits.is_leaf and logits.requires_grad:
            raise ValueError("inplace_backward overwrites the logits during backward; it needs "
                             "logits produced by an op, not a leaf tensor that requires grad")
        window = completion_window(logits, logits_to_keep)
        targets = completion_ids.contiguous()
        _check_inputs(window, targets)
        logprob, entropy, lse = _alloc_outputs(targets)
        _C.fused_logprob_entropy_scaled(window, targets, logprob, entropy, lse, scale)
        ctx.save_for_backward(logits, targets, lse, entropy)
        ctx.logits_to_keep = logits_to_keep
        ctx.scale = scale
        ctx.inplace = bool(inplace_backward)
        ctx.set_materialize_grads(False)
        ctx.mark_non_differentiable(lse)
        return logprob, entropy, lse

    @staticmethod
    def backward(ctx, g_logp, g_ent, _g_lse):
        logits, targets, lse, entropy = ctx.saved_tensors
        grad = logits if ctx.inplace else torch.empty_like(logits)
        window = completion_window(logits, ctx.logits_to_keep)
        _C.fused_logprob_entropy_scaled_backward(
            window, targets, lse, entropy, _prep(g_logp), _prep(g_ent), None,
            completion_window(grad, ctx.logits_to_keep), ctx.scale)
        # rows outside the window get no gradient
        L, n = logits.shape[1], window.shape[1]
        if L - 1 - n > 0:
            grad[:, :L - 1 - n].zero_()
        grad[:, L - 1:].zero_()
        if ctx.inplace:
            # the logits are gone: any other saved reference to them now fails loudly
            torch.autograd.graph.increment_version(logits)
        return grad, None, None, None, None


def window_logps_and_entropies(logits: torch.Tensor, completion_ids: torch.Tensor,
                               logits_to_keep: int, temperature: float = 1.0,
                               compute_entropy: bool = True, inplace_backward: bool = False):
    """Per-token log-probs and entropies of the GRPO completion window of the model's
    logits [B, L, V], as the reference trainer computes them (slice, in-place division by
    the temperature, K1; reference trainer.py:96-127) but in one launch each way.

    Returns (logps [B, K] with grad to `logits`, entropies [B, K] detached or None).
    Forward results are bit-identical to K1 on `completion_window(logits, K).div_(T)`, and
    so is the gradient written into the window of `logits`; the other rows of the
    gradient are zero.  `logits` itself is not modified by the forward.

    inplace_backward: the backward writes the gradient into the logits' own storage and
    returns it as the gradient (no second [B, L, V] buffer).  Only valid when nothing else
    needs the logits' values afterwards -- true for an LM head's output, whose producer
    (a matmul) saves its inputs, not its output.  The logits' version counter is bumped,
    so a later use of a saved reference to them raises instead of reading gradients.
    """
    logps, ents, _lse = _WindowLogprobEntropy.apply(
        logits, completion_ids, logits_to_keep, temperature_scale(temperature),
        inplace_backward)
    return logps, (ents.detach() if compute_entropy else None)

"""The K1 call inside GRPO's logprob method, usable without `trl`.

The reference trainer slices the model's [B, L, V] logits to the completion window,
which leaves a view whose batch stride is still L*V, and then calls K1 once per batch
element to avoid copying it (python/kernel_opt/trainer.py:104-127).  The kernels here
accept that two-level strided layout directly, so the whole window is one launch.
"""
from __future__ import annotations

import torch

from .ops import fused_logprob_entropy

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


def k1_logps_and_entropies(logits: torch.Tensor, completion_ids: torch.Tensor,
                           compute_entropy: bool):
    """Per-token log-probs (with grad) and detached entropies of a [B, L', V] window
    in one K1 launch.  Returns (logps [B, L'], entropies [B, L'] or None)."""
    logps, ents, _lse = fused_logprob_entropy(logits, completion_ids.contiguous())
    return logps, (ents.detach() if compute_entropy else None)

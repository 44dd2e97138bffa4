"""KernelOptGRPOTrainer -- trl.GRPOTrainer with the logprob/entropy block replaced by K1.

Same override as the reference (python/kernel_opt/trainer.py:1-131): only
`_get_per_token_logps_and_entropies` changes, which is TRL's single entry point for the
policy, old-policy and reference log-prob computations.  Multimodal inputs fall back to
the parent.  Unlike the reference, each chunk is one K1 launch on the strided [B, L', V]
completion window instead of a loop over batch elements, the temperature is applied
inside the kernels instead of by an in-place division, and the backward writes the
parent-shaped logits gradient directly (`grpo.window_logps_and_entropies`).  Results are
bit-identical to the reference's slice + `div_` + K1 sequence.

`k1_inplace_backward=True` (constructor keyword) lets the backward overwrite the model's
logits with their gradient, which removes the second [B, L, V] buffer of the loss block.

`k1_fused_lm_head=True` (constructor keyword) skips the logits tensor altogether: the
decoder's last hidden state of the completion window goes through
`kernel_opt.lm_head.fused_linear_logprob_entropy` (LM-head GEMM in L2-sized row chunks, K1
on each chunk).  Only for models whose head is a plain bias-free linear map of the final
hidden state; other models (logit soft-capping or scaling, a head bias) keep the standard
path, with a warning.

Requires `trl` (imported at module load, as in the reference); `kernel_opt` imports
this module lazily.
"""
from __future__ import annotations

import warnings

import torch
from trl import GRPOTrainer

from .grpo import MULTIMODAL_KWARGS, window_logps_and_entropies
from .lm_head import fused_head_parts, fused_linear_logprob_entropy


class KernelOptGRPOTrainer(GRPOTrainer):
    """trl.GRPOTrainer with the inner logprob+entropy block replaced by K1."""

    def __init__(self, *args, k1_inplace_backward: bool = False, k1_fused_lm_head: bool = False,
                 **kwargs):
        super().__init__(*args, **kwargs)
        self.k1_inplace_backward = k1_inplace_backward
        self.k1_fused_lm_head = k1_fused_lm_head

    def _get_per_token_logps_and_entropies(
        self,
        model,
        input_ids,
        attention_mask,
        logits_to_keep,
        batch_size=None,
        compute_entropy=False,
        pixel_values=None,
        image_grid_thw=None,
        num_images=None,
        pixel_attention_mask=None,
        image_sizes=None,
        token_type_ids=None,
        mm_token_type_ids=None,
        image_position_ids=None,
    ) -> tuple[torch.Tensor, torch.Tensor | None]:
        extra = dict(
            pixel_values=pixel_values, image_grid_thw=image_grid_thw, num_images=num_images,
            pixel_attention_mask=pixel_attention_mask, image_sizes=image_sizes,
            token_type_ids=token_type_ids, mm_token_type_ids=mm_token_type_ids,
            image_position_ids=image_position_ids,
        )
        assert set(extra) == set(MULTIMODAL_KWARGS)
        if any(v is not None for v in extra.values()):
            return super()._get_per_token_logps_and_entropies(
                model, input_ids, attention_mask, logits_to_keep,
                batch_size=batch_size, compute_entropy=compute_entropy, **extra)

        parts = None
        if getattr(self, "k1_fused_lm_head", False):
            parts = fused_head_parts(model)
            if parts is None:
                warnings.warn("k1_fused_lm_head: this model's logits are not a plain linear map "
                              "of the decoder output; using the logits path", stacklevel=2)
        bsz = batch_size or input_ids.size(0)
        all_logps: list[torch.Tensor] = []
        all_entropies: list[torch.Tensor] = []
        for start in range(0, input_ids.size(0), bsz):
            input_ids_batch = input_ids[start:start + bsz]
            attention_mask_batch = attention_mask[start:start + bsz]
            if parts is not None:
                # hidden states of the completion window -> fused LM head + K1
                decoder, weight = parts
                out = decoder(input_ids=input_ids_batch, attention_mask=attention_mask_batch,
                              use_cache=False)
                hidden = out[0][:, -(logits_to_keep + 1):-1, :]
                completion_ids = input_ids_batch[:, -logits_to_keep:]
                logps, ents, _ = fused_linear_logprob_entropy(hidden, weight, completion_ids,
                                                              self.temperature)
                all_logps.append(logps)
                if compute_entropy:
                    all_entropies.append(ents.detach())
                continue
            model_inputs = {"input_ids": input_ids_batch,
                            "attention_mask": attention_mask_batch}
            if "logits_to_keep" in self.model_kwarg_keys:
                # +1 because the last position is dropped below
                model_inputs["logits_to_keep"] = logits_to_keep + 1
            model_inputs["use_cache"] = False

            logits = model(**model_inputs).logits
            completion_ids = input_ids_batch[:, -logits_to_keep:]
            # completion window, temperature and K1 in one launch each way
            logps, ents = window_logps_and_entropies(
                logits, completion_ids, logits_to_keep, self.temperature, compute_entropy,
                inplace_backward=getattr(self, "k1_inplace_backward", False) and torch.is_grad_enabled())
            all_logps.append(logps)
            if compute_entropy:
                all_entropies.append(ents)

        logps = torch.cat(all_logps, dim=0)
        entropies = torch.cat(all_entropies, dim=0) if compute_entropy else None
        return logps, entropies

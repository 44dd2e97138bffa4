"""Python wrappers around the K1 kernels (kernel_opt._C -> libk1_b200.so).

Public entry points, with the reference's names and contracts
(python/kernel_opt/ops.py:1-111):
  - fused_logprob_entropy(logits, targets)          autograd-aware; training code
  - fused_logprob_entropy_forward(logits, targets)  forward only, no autograd graph
  - fused_logprob_entropy_naive(logits, targets)    one thread per row; correctness anchor

Differences from the reference, all widening what is accepted:
  - logits may be a strided view (unit stride on the vocab axis, leading dims that
    collapse to two stride levels, e.g. logits[:, :-1, :]); no copy is made;
  - targets may be non-contiguous (they are made contiguous, N int64 values);
  - unused outputs get no zero-filled gradient tensors: the kernel treats a missing
    upstream gradient as zero.
"""
import torch

from kernel_opt import _C


def _check_inputs(logits: torch.Tensor, targets: torch.Tensor):
    """Reference ops.py:16-21, minus the logits contiguity requirement."""
    assert logits.is_cuda and targets.is_cuda
    assert targets.dtype == torch.int64
    assert logits.shape[:-1] == targets.shape, \
        f"logits[...,V]={logits.shape} vs targets[...]={targets.shape}"


def _alloc_outputs(targets: torch.Tensor):
    """Three fp32 tensors shaped like targets (reference ops.py:24-30)."""
    out_shape = targets.shape
    return (
        torch.empty(out_shape, device=targets.device, dtype=torch.float32),
        torch.empty(out_shape, device=targets.device, dtype=torch.float32),
        torch.empty(out_shape, device=targets.device, dtype=torch.float32),
    )


def fused_logprob_entropy_naive(logits: torch.Tensor, targets: torch.Tensor):
    """One-thread-per-row forward in fp64 (reference ops.py:33-38). Never fast."""
    _check_inputs(logits, targets)
    targets = targets.contiguous()
    logprob, entropy, lse = _alloc_outputs(targets)
    _C.fused_logprob_entropy_naive(logits, targets, logprob, entropy, lse)
    return logprob, entropy, lse


def fused_logprob_entropy_forward(logits: torch.Tensor, targets: torch.Tensor):
    """K1 forward only (no autograd). Reference ops.py:41-46."""
    _check_inputs(logits, targets)
    targets = targets.contiguous()
    logprob, entropy, lse = _alloc_outputs(targets)
    _C.fused_logprob_entropy_v1(logits, targets, logprob, entropy, lse)
    return logprob, entropy, lse


class _FusedLogprobEntropy(torch.autograd.Function):
    """K1 forward + backward as a torch autograd op (reference ops.py:49-89).

    Forward saves (logits, targets, lse, entropy).  Backward recomputes
    p = exp(x - lse) in a single streaming pass -- no [B,S,V] intermediate.
    """

    @staticmethod
    def forward(ctx, logits, targets):
        _check_inputs(logits, targets)
        targets = targets.contiguous()
        logprob, entropy, lse = _alloc_outputs(targets)
        _C.fused_logprob_entropy_v1(logits, targets, logprob, entropy, lse)
        ctx.save_for_backward(logits, targets, lse, entropy)
        # Unused outputs arrive as None instead of materialised zero tensors.
        ctx.set_materialize_grads(False)
        return logprob, entropy, lse

    @staticmethod
    def backward(ctx, g_logp, g_ent, g_lse):
        logits, targets, lse, entropy = ctx.saved_tensors

        def _prep(g):
            if g is None:
                return None
            return g.to(torch.float32, copy=False).contiguous()

        d_logits = torch.empty_like(logits)
        _C.fused_logprob_entropy_v1_backward(
            logits, targets, lse, entropy,
            _prep(g_logp), _prep(g_ent), _prep(g_lse), d_logits)
        # targets has no grad
        return d_logits, None


class _FusedLogprobEntropyScaled(torch.autograd.Function):
    """K1 on logits divided by a temperature, the division done inside the kernels with
    the rounding of `logits.div_(T)` (see k1_fused_logprob_entropy_scaled)."""

    @staticmethod
    def forward(ctx, logits, targets, scale):
        _check_inputs(logits, targets)
        targets = targets.contiguous()
        logprob, entropy, lse = _alloc_outputs(targets)
        _C.fused_logprob_entropy_scaled(logits, targets, logprob, entropy, lse, scale)
        ctx.save_for_backward(logits, targets, lse, entropy)
        ctx.scale = scale
        ctx.set_materialize_grads(False)
        return logprob, entropy, lse

    @staticmethod
    def backward(ctx, g_logp, g_ent, g_lse):
        logits, targets, lse, entropy = ctx.saved_tensors

        def _prep(g):
            return None if g is None else g.to(torch.float32, copy=False).contiguous()

        d_logits = torch.empty_like(logits)
        _C.fused_logprob_entropy_scaled_backward(
            logits, targets, lse, entropy, _prep(g_logp), _prep(g_ent), _prep(g_lse), d_logits,
            ctx.scale)
        return d_logits, None, None


def fused_logprob_entropy_scaled(logits: torch.Tensor, targets: torch.Tensor,
                                 temperature: float = 1.0):
    """`fused_logprob_entropy(logits / temperature, targets)` without the division pass:
    same results and gradient (w.r.t. the undivided logits) bit for bit, one launch each
    way.  No counterpart in the reference, whose trainer divides in place first
    (python/kernel_opt/trainer.py:101)."""
    from .grpo import temperature_scale
    return _FusedLogprobEntropyScaled.apply(logits, targets, temperature_scale(temperature))


# ---------------------------------------------------------------------------------------
# torch.library registration: under torch.compile K1 is one opaque op with a fake (meta)
# implementation and an autograd formula, so compiled graphs contain it without a graph
# break.  (The reference's pybind call graph-breaks: REPORT.md:315-318.)
# ---------------------------------------------------------------------------------------
@torch.library.custom_op("kernel_opt::fused_logprob_entropy_fwd", mutates_args=())
def _fwd_op(logits: torch.Tensor, targets: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor,
                                                                   torch.Tensor]:
    targets = targets.contiguous()
    logprob, entropy, lse = _alloc_outputs(targets)
    _C.fused_logprob_entropy_v1(logits, targets, logprob, entropy, lse)
    return logprob, entropy, lse


@_fwd_op.register_fake
def _(logits, targets):
    return tuple(torch.empty(targets.shape, device=targets.device, dtype=torch.float32)
                 for _ in range(3))


@torch.library.custom_op("kernel_opt::fused_logprob_entropy_bwd", mutates_args=())
def _bwd_op(logits: torch.Tensor, targets: torch.Tensor, lse: torch.Tensor,
            entropy: torch.Tensor, g_logp: torch.Tensor | None, g_ent: torch.Tensor | None,
            g_lse: torch.Tensor | None) -> torch.Tensor:
    d_logits = torch.empty_like(logits)
    _C.fused_logprob_entropy_v1_backward(logits, targets.contiguous(), lse, entropy,
                                         g_logp, g_ent, g_lse, d_logits)
    return d_logits


@_bwd_op.register_fake
def _(logits, targets, lse, entropy, g_logp, g_ent, g_lse):
    return torch.empty_like(logits)


def _op_setup_context(ctx, inputs, output):
    logits, targets = inputs
    _logprob, entropy, lse = output
    ctx.save_for_backward(logits, targets, lse, entropy)


def _op_backward(ctx, g_logp, g_ent, g_lse):
    logits, targets, lse, entropy = ctx.saved_tensors

    def _prep(g):
        return None if g is None else g.to(torch.float32).contiguous()

    return _bwd_op(logits, targets, lse, entropy, _prep(g_logp), _prep(g_ent), _prep(g_lse)), None


_fwd_op.register_autograd(_op_backward, setup_context=_op_setup_context)


def fused_logprob_entropy_op(logits: torch.Tensor, targets: torch.Tensor):
    """K1 through the registered custom op `kernel_opt::fused_logprob_entropy_fwd` (same
    results and gradients as `fused_logprob_entropy`)."""
    _check_inputs(logits, targets)
    return _fwd_op(logits, targets)


def fused_logprob_entropy(logits: torch.Tensor, targets: torch.Tensor):
    """K1 (production), autograd-aware.  Reference ops.py:92-111.

    Replaces `selective_log_softmax(logits, targets)` + `entropy_from_logits(logits)`
    with one streaming pass per row, plus a streaming backward that recomputes the
    softmax from the saved lse.

    Args:
        logits:  [..., V] bf16 / fp16 / fp32 on CUDA, unit stride along V.
        targets: [...]    int64 on CUDA.  Ids outside [0, V) read a target logit of
                 0 (logprob = -lse) and get no one-hot gradient, as in the reference.

    Returns:
        (logprob, entropy, lse), each [...] fp32 on CUDA.
            logprob[i] = logits[i, targets[i]] - logsumexp(logits[i])
            entropy[i] = -sum_v softmax(logits[i])[v] * log_softmax(logits[i])[v]
            lse[i]     = logsumexp(logits[i])

    `targets` has no gradient.  Under torch.compile the call goes through the registered
    custom op (one node in the graph, no graph break); eagerly it is an autograd.Function.
    """
    if torch.compiler.is_compiling():
        return fused_logprob_entropy_op(logits, targets)
    return _FusedLogprobEntropy.apply(logits, targets)

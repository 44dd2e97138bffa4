"""kernel_opt -- B200-native (sm_100a) K1: per-token log-prob, entropy and log-sum-exp
over [..., V] logits, forward and backward, in one streaming pass each.

Drop-in for the reference package of the same name (python/kernel_opt/__init__.py:1-15):
the same public functions, the same `_C` binding names, and the lazily imported
`KernelOptGRPOTrainer` (needs `trl`).  Multi-GPU helpers live in `kernel_opt.parallel`,
the GRPO completion-window node in `kernel_opt.grpo`, the LM head fused with K1 in
`kernel_opt.lm_head`.
"""
import torch  # noqa: F401  (loads libc10 / libtorch before the extension)

try:
    from . import _C  # noqa: F401
except ImportError as e:  # fail loudly: there is no fallback implementation
    raise ImportError(
        "kernel_opt._C is not built; run `python build.py` in the package root "
        "(requires nvcc for sm_100a)") from e

from .ops import (  # noqa: F401
    fused_logprob_entropy,
    fused_logprob_entropy_forward,
    fused_logprob_entropy_naive,
    fused_logprob_entropy_scaled,
)
from .lm_head import fused_linear_logprob_entropy  # noqa: F401


def set_check_waits(on: bool = True) -> None:
    """Debug switch: raise a RuntimeError from any K1 call whose kernel's bounded wait ran
    out.  Every wait inside the kernels is bounded; one that runs out (it cannot in correct
    operation) leaves NaN in the outputs it could not finish and sets a device status word.
    With the switch on, each call synchronises its stream and reads that word.  Also set by
    K1_CHECK_WAITS=1 in the environment.  No counterpart in the reference."""
    _C.set_check_waits(bool(on))


def check_waits() -> bool:
    """Whether K1 calls check the kernels' bounded waits (see set_check_waits)."""
    return bool(_C.check_waits())


def __getattr__(name):
    # Lazy import so users without trl can still use the kernels.
    if name == "KernelOptGRPOTrainer":
        from .trainer import KernelOptGRPOTrainer
        return KernelOptGRPOTrainer
    raise AttributeError(f"module 'kernel_opt' has no attribute {name!r}")


__version__ = "0.1.0"

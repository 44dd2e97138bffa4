"""TEST INFRASTRUCTURE ONLY.  Build the reference's own K1 CUDA extension for sm_100a.

Compiles the reference sources where they lie (csrc/bindings.cpp and
csrc/fused_logprob.cu of the reference checkout; nothing is copied into this
repository) with torch.utils.cpp_extension.load and the reference's own nvcc flags
(setup.py:5-11: -O3 --use_fast_math -std=c++17), retargeted from sm_89 to sm_100a.
The reference's setup.py is not used: its MSVC-only cxx flags do not work with gcc.
Output: oracle/_ref/k1_reference*.so (git-ignored; it travels to the GPU box with the
rest of the tree).  Used only by GPU tests to pin the oracle and the kernels against the
reference kernels' actual outputs.
"""
from __future__ import annotations

import glob
import os
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
OUT = os.path.join(HERE, "_ref")
NAME = "k1_reference"


def reference_root() -> str | None:
    """The reference checkout: $K1_REFERENCE_ROOT, else a directory named `reference` beside
    this repository; None when neither holds the K1 sources."""
    env = os.environ.get("K1_REFERENCE_ROOT")
    cands = [env] if env else [os.path.join(os.path.dirname(os.path.dirname(HERE)), "reference")]
    for c in cands:
        if c and os.path.exists(os.path.join(c, "csrc", "fused_logprob.cu")):
            return c
    return None


def built_path() -> str | None:
    hits = sorted(glob.glob(os.path.join(OUT, NAME + "*.so")))
    return hits[0] if hits else None


def build(ref_root: str | None = None, force: bool = False) -> str | None:
    ref_root = ref_root or reference_root()
    if ref_root is None:
        return built_path()
    srcs = [os.path.join(ref_root, "csrc", "bindings.cpp"),
            os.path.join(ref_root, "csrc", "fused_logprob.cu")]
    if not all(os.path.exists(s) for s in srcs):
        return built_path()
    have = built_path()
    if have and not force and all(os.path.getmtime(have) >= os.path.getmtime(s) for s in srcs):
        return have
    os.makedirs(OUT, exist_ok=True)
    os.environ["TORCH_CUDA_ARCH_LIST"] = "10.0a"
    from torch.utils import cpp_extension
    cpp_extension.load(
        name=NAME,
        sources=srcs,
        extra_cflags=["-O3", "-std=c++17"],
        extra_cuda_cflags=["-O3", "--use_fast_math", "-std=c++17"],
        build_directory=OUT,
        verbose=False,
    )
    return built_path()


if __name__ == "__main__":
    p = build(force="--force" in sys.argv)
    print(p if p else "reference sources not found; nothing built")

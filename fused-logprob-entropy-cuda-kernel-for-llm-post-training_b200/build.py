"""Build recipe for the B200 K1 package (in-tree, sm_100a only).

Produces
  kernel_opt/lib/libk1_b200.so   C ABI (include/k1_logprob.h), CUDA kernels, no torch
  kernel_opt/_C<ext>.so          torch extension mirroring the reference's `_C`
                                 binding, linked against libk1_b200.so
  kernel_opt/lib/libk1_b200_waittest.so
                                 the C ABI with short wait limits and test knobs, for
                                 the wait-timeout GPU test only

Run `python build.py` (or `build()` from Python).  Outputs are rebuilt only when a
source is newer than the output, unless force=True.
"""
from __future__ import annotations

import os
import subprocess
import sys
import sysconfig

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
PKG = os.path.join(HERE, "kernel_opt")
LIBDIR = os.path.join(PKG, "lib")
INCLUDE = os.path.join(REPO, "include")

CAPI_SOURCES = ["k1_capi.cu", "k1_kernels.cuh", "k1_common.cuh", "k1_ring.cuh", "k1_fwd_sm.cuh",
                "k1_lmhead.cuh"]
CAPI_LIB = os.path.join(LIBDIR, "libk1_b200.so")
BINDING_SOURCE = "k1_torch_binding.cpp"

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-lineinfo", "-O3", "-std=c++17",
    "-Xcompiler", "-fPIC", "-shared",
]


def _nvcc() -> str:
    cuda_home = os.environ.get("CUDA_HOME", "/usr/local/cuda")
    cand = os.path.join(cuda_home, "bin", "nvcc")
    return cand if os.path.exists(cand) else "nvcc"


def _stale(output: str, sources: list[str]) -> bool:
    if not os.path.exists(output):
        return True
    t = os.path.getmtime(output)
    return any(os.path.getmtime(s) > t for s in sources)


def _run(cmd: list[str]) -> None:
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        sys.stderr.write(r.stdout + r.stderr)
        raise RuntimeError(f"build step failed: {' '.join(cmd[:3])} ... (exit {r.returncode})")


def build_capi(force: bool = False, verbose_ptxas: bool = False) -> str:
    srcs = [os.path.join(CSRC, s) for s in CAPI_SOURCES] + [os.path.join(INCLUDE, "k1_logprob.h")]
    if force or _stale(CAPI_LIB, srcs):
        os.makedirs(LIBDIR, exist_ok=True)
        cmd = [_nvcc(), *NVCC_FLAGS, "-I", INCLUDE, os.path.join(CSRC, "k1_capi.cu"),
               "-o", CAPI_LIB]
        if verbose_ptxas:
            cmd.insert(1, "-Xptxas=-v")
        _run(cmd)
    return CAPI_LIB


# The wait-timeout test library: the same C ABI built with short wait limits and the
# K1_WAIT_TEST knobs (k1_test_set_knobs), so a GPU test can make a kernel's bounded waits
# run out and check that the kernel returns, reports the status bit and writes NaN.  The
# product never loads it.
WAIT_TEST_LIB = os.path.join(LIBDIR, "libk1_b200_waittest.so")
WAIT_TEST_FLAGS = ["-DK1_WAIT_TEST", "-DK1_RING_MAX_TRIES=16", "-DK1_SM_MAX_POLLS=4096"]


def build_wait_test_lib(force: bool = False) -> str:
    srcs = [os.path.join(CSRC, s) for s in CAPI_SOURCES] + [os.path.join(INCLUDE, "k1_logprob.h")]
    if force or _stale(WAIT_TEST_LIB, srcs):
        os.makedirs(LIBDIR, exist_ok=True)
        _run([_nvcc(), *NVCC_FLAGS, *WAIT_TEST_FLAGS, "-I", INCLUDE,
              os.path.join(CSRC, "k1_capi.cu"), "-o", WAIT_TEST_LIB])
    return WAIT_TEST_LIB


def binding_path() -> str:
    suffix = sysconfig.get_config_var("EXT_SUFFIX") or ".so"
    return os.path.join(PKG, "_C" + suffix)


def build_binding(force: bool = False) -> str:
    import torch
    from torch.utils import cpp_extension

    out = binding_path()
    srcs = [os.path.join(CSRC, BINDING_SOURCE), os.path.join(INCLUDE, "k1_logprob.h"), CAPI_LIB]
    if not (force or _stale(out, srcs)):
        return out
    incs = cpp_extension.include_paths(device_type="cuda")
    libs = cpp_extension.library_paths(device_type="cuda")
    abi = int(torch._C._GLIBCXX_USE_CXX11_ABI)
    cmd = ["g++", "-O2", "-std=c++17", "-fPIC", "-shared", "-w",
           f"-D_GLIBCXX_USE_CXX11_ABI={abi}",
           "-DTORCH_API_INCLUDE_EXTENSION_H", "-DTORCH_EXTENSION_NAME=_C",
           "-I", INCLUDE, "-I", sysconfig.get_paths()["include"]]
    for d in incs:
        cmd += ["-I", d]
    cmd += [os.path.join(CSRC, BINDING_SOURCE), "-o", out]
    for d in libs:
        cmd += ["-L", d]
    cmd += ["-L", LIBDIR, "-lk1_b200", "-lc10", "-ltorch", "-ltorch_cpu", "-ltorch_python",
            "-lc10_cuda", "-ltorch_cuda", "-Wl,-rpath,$ORIGIN/lib"]
    _run(cmd)
    return out


def build(force: bool = False) -> None:
    build_capi(force=force)
    build_binding(force=force)
    build_wait_test_lib(force=force)


if __name__ == "__main__":
    build(force="--force" in sys.argv)
    print(CAPI_LIB)
    print(binding_path())

"""Test helpers: golden-fixture loading, seeded inputs, tolerance checks."""
from __future__ import annotations

import os
import re

import numpy as np
import torch

from conftest import PKG_ROOT, REPO

GOLDEN = os.path.join(REPO, "tests", "golden", "k1_golden.npz")
HEADER = os.path.join(REPO, "include", "k1_logprob.h")
CAPI_LIB = os.path.join(PKG_ROOT, "kernel_opt", "lib", "libk1_b200.so")
# the same C ABI built with short wait limits and the K1_WAIT_TEST knobs (test only)
WAIT_TEST_LIB = os.path.join(PKG_ROOT, "kernel_opt", "lib", "libk1_b200_waittest.so")

TORCH_DT = {"float32": torch.float32, "float16": torch.float16, "bfloat16": torch.bfloat16}


def golden_cases():
    z = np.load(GOLDEN)
    names = sorted({k.split("/")[0] for k in z.files})
    out = {}
    for n in names:
        c = {k.split("/", 1)[1]: z[k] for k in z.files if k.startswith(n + "/")}
        dt = TORCH_DT[str(c["dtype"])]
        shape = tuple(int(s) for s in c["shape"])
        raw = c["x"]
        if dt == torch.float32:
            x = torch.from_numpy(raw.astype(np.float32)).reshape(shape)
        else:
            x = torch.from_numpy(raw.view(np.int16)).view(dt).reshape(shape)
        c["logits"] = x
        c["targets_t"] = torch.from_numpy(c["targets"].astype(np.int64))
        out[n] = c
    return out


def header_functions():
    """Names of the functions declared in include/k1_logprob.h."""
    text = open(HEADER).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(k1_[a-z0-9_]+)\s*\(", text)))


def assert_close_nan(actual, expected, atol, rtol, what):
    """allclose with NaN == NaN and inf == inf; reports the worst element."""
    a = np.asarray(actual, np.float64)
    e = np.asarray(expected, np.float64)
    assert a.shape == e.shape, f"{what}: shape {a.shape} != {e.shape}"
    both_nan = np.isnan(a) & np.isnan(e)
    same_inf = np.isinf(a) & np.isinf(e) & (np.sign(a) == np.sign(e))
    ok = both_nan | same_inf | (np.abs(a - e) <= atol + rtol * np.abs(e))
    if not ok.all():
        i = np.unravel_index(np.argmax(~ok), ok.shape)
        raise AssertionError(f"{what}: {int((~ok).sum())} mismatches; first at {i}: "
                             f"got {a[i]!r}, want {e[i]!r} (atol {atol}, rtol {rtol})")

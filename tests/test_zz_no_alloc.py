"""The allocation-free forward entry point, k1_fused_logprob_entropy_v1_noalloc.

It exists for callers that cannot call cudaMalloc or provide device scratch of their own --
for example a plugin running inside a host framework whose memory pool is the only
allocator, or latency-critical code that must avoid cudaMalloc's implicit device
synchronisation.  Instead of a caller-provided workspace it uses scratch that the library
keeps in a static device array.  These tests call it through the C ABI and check that two
calls in a row give exactly what the workspace-taking entry point gives, also for row
counts that split rows between thread blocks (the case that uses the scratch).  The file
is named so that pytest collects it last.
"""
import ctypes

import pytest
import torch

from _gpu import check_forward_outputs, seeded_logits, seeded_targets
from _helpers import CAPI_LIB

pytestmark = pytest.mark.gpu

DTYPE_CODE = {torch.float32: 0, torch.float16: 1, torch.bfloat16: 2}


def capi():
    lib = ctypes.CDLL(CAPI_LIB)
    i64, p, c_int = ctypes.c_int64, ctypes.c_void_p, ctypes.c_int
    lib.k1_fused_logprob_entropy_v1.argtypes = [p, c_int, i64, i64, i64, i64, i64, p, p, p, p, p,
                                                ctypes.c_size_t, p]
    lib.k1_fused_logprob_entropy_v1_noalloc.argtypes = [p, c_int, i64, i64, i64, i64, i64, p, p,
                                                        p, p, p]
    lib.k1_forward_workspace_bytes.argtypes = [i64, i64, c_int, c_int]
    lib.k1_forward_workspace_bytes.restype = ctypes.c_size_t
    lib.k1_last_error.restype = ctypes.c_char_p
    return lib


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
@pytest.mark.parametrize("shape", [(3, 152064), (1024, 32000), (37, 1003)])
def test_noalloc_matches_workspace_entry_point(dtype, shape):
    lib = capi()
    N, V = shape
    x_cpu = seeded_logits(shape, dtype, 3.0, seed=N + V)
    t_cpu = seeded_targets((N,), V, seed=N)
    x, t = x_cpu.cuda(), t_cpu.cuda()
    stream = torch.cuda.current_stream().cuda_stream
    dt = DTYPE_CODE[dtype]

    ws_bytes = lib.k1_forward_workspace_bytes(N, V, dt, torch.cuda.current_device())
    ws = torch.zeros(ws_bytes, dtype=torch.uint8, device="cuda")
    ref = [torch.empty(N, device="cuda") for _ in range(3)]
    rc = lib.k1_fused_logprob_entropy_v1(x.data_ptr(), dt, N, V, N, V, 0, t.data_ptr(),
                                         *(o.data_ptr() for o in ref), ws.data_ptr(), ws_bytes,
                                         stream)
    assert rc == 0, lib.k1_last_error()

    for _ in range(2):  # two calls in a row share (and must re-clear) the static scratch
        out = [torch.full((N,), float("nan"), device="cuda") for _ in range(3)]
        rc = lib.k1_fused_logprob_entropy_v1_noalloc(x.data_ptr(), dt, N, V, N, V, 0,
                                                     t.data_ptr(), *(o.data_ptr() for o in out),
                                                     stream)
        assert rc == 0, lib.k1_last_error()
        for a, b in zip(out, ref):
            torch.testing.assert_close(a, b, rtol=0, atol=0)
        check_forward_outputs(out, x_cpu, t_cpu, "noalloc")


def test_noalloc_rejects_bad_arguments():
    lib = capi()
    rc = lib.k1_fused_logprob_entropy_v1_noalloc(1024, 7, 4, 16, 4, 16, 0, 2048, 4096, 4096,
                                                 4096, None)
    assert rc == 2 and b"bf16, fp16, or fp32" in lib.k1_last_error()

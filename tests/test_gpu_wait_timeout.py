"""Bounded waits that run out: the kernel returns, reports a status bit and leaves NaN.

Every wait inside the K1 kernels is bounded (the backward's bulk-copy ring, the
one-block-per-SM forward's row slots).  In correct operation none can run out.  These
tests use the wait-timeout test library (the same C ABI built with -DK1_WAIT_TEST and
short wait limits) and its knobs to make one block's waits run out on purpose:

  * backward: block 0's producer issues no bulk copy from chunk 3 on, so its consumers'
    waits for chunk 3 run out;
  * forward: block 0 drops one grab of row 0, so row 0 never completes and the grabs of
    the next row that needs its slot wait until their waits run out;
  * tensor-core LM head: CTA 0 stops issuing tile copies, so its MMA's wait runs out.

Nothing faults or hangs: the waits give up after a few milliseconds, the producer drains
the copies it issued, and the kernel returns.  Each test checks the status bit through
k1_ring_status, that the unfinished outputs are NaN, that every other output equals the
product library's bit for bit, and that a following call on the same context is clean.
"""
import ctypes

import pytest
import torch

from _helpers import CAPI_LIB, WAIT_TEST_LIB
from kernel_opt import _C

pytestmark = pytest.mark.gpu

BF16 = 2


def test_lib():
    lib = ctypes.CDLL(WAIT_TEST_LIB)
    i64, p, c_int = ctypes.c_int64, ctypes.c_void_p, ctypes.c_int
    lib.k1_test_set_knobs.argtypes = [ctypes.c_longlong, ctypes.c_longlong]
    lib.k1_fused_logprob_entropy_v1.argtypes = [p, c_int, i64, i64, i64, i64, i64, p, p, p, p, p,
                                                ctypes.c_size_t, p]
    lib.k1_fused_logprob_entropy_v1_backward.argtypes = [p, c_int, i64, i64, i64, i64, i64, p, p,
                                                         p, p, p, p, p, i64, i64, p]
    lib.k1_forward_workspace_bytes.argtypes = [i64, i64, c_int, c_int]
    lib.k1_forward_workspace_bytes.restype = ctypes.c_size_t
    lib.k1_ring_status.argtypes = [ctypes.POINTER(ctypes.c_uint)]
    lib.k1_last_error.restype = ctypes.c_char_p
    return lib


def status(lib):
    v = ctypes.c_uint(0)
    assert lib.k1_ring_status(ctypes.byref(v)) == 0, lib.k1_last_error()
    return v.value


def inputs(N=600, V=65536, seed=11):
    g = torch.Generator(device="cuda").manual_seed(seed)
    x = (torch.randn((N, V), generator=g, device="cuda") * 3.0).to(torch.bfloat16)
    t = torch.randint(0, V, (N,), generator=g, device="cuda")
    return x, t


def forward(lib, x, t):
    N, V = x.shape
    ws_bytes = lib.k1_forward_workspace_bytes(N, V, BF16, torch.cuda.current_device())
    ws = torch.zeros(ws_bytes, dtype=torch.uint8, device="cuda")
    out = [torch.full((N,), 7.0, device="cuda") for _ in range(3)]
    rc = lib.k1_fused_logprob_entropy_v1(x.data_ptr(), BF16, N, V, N, V, 0, t.data_ptr(),
                                         *(o.data_ptr() for o in out), ws.data_ptr(), ws_bytes,
                                         torch.cuda.current_stream().cuda_stream)
    assert rc == 0, lib.k1_last_error()
    torch.cuda.synchronize()
    return out


def backward(lib, x, t, lse, ent, gl, gh):
    N, V = x.shape
    d = torch.full_like(x, 7.0)
    rc = lib.k1_fused_logprob_entropy_v1_backward(
        x.data_ptr(), BF16, N, V, N, V, 0, t.data_ptr(), lse.data_ptr(), ent.data_ptr(),
        gl.data_ptr(), gh.data_ptr(), None, d.data_ptr(), V, 0,
        torch.cuda.current_stream().cuda_stream)
    assert rc == 0, lib.k1_last_error()
    torch.cuda.synchronize()
    return d


def product_outputs(x, t):
    out = [torch.empty(x.shape[0], device="cuda") for _ in range(3)]
    _C.fused_logprob_entropy_v1(x, t, *out)
    return out


def test_backward_ring_wait_runs_out():
    lib = test_lib()
    x, t = inputs()
    lp, h, l = product_outputs(x, t)
    N = x.shape[0]
    gl = torch.full((N,), -1.0 / N, device="cuda")
    gh = torch.full((N,), -0.01 / N, device="cuda")
    ref = torch.empty_like(x)
    _C.fused_logprob_entropy_v1_backward(x, t, l, h, gl, gh, None, ref)
    torch.cuda.synchronize()
    assert status(lib) == 0

    assert lib.k1_test_set_knobs(3, -1) == 0
    try:
        d = backward(lib, x, t, l, h, gl, gh)
        st = status(lib)
    finally:
        assert lib.k1_test_set_knobs(-1, -1) == 0
    assert st & 1, f"status {st}: the ring's wait did not report running out"
    flat, want = d.view(-1), ref.view(-1)
    bad = torch.isnan(flat)
    assert bad.any(), "no NaN written where the wait ran out"
    idx = bad.nonzero().view(-1)
    # block 0 computed its first 3 chunks (3 x 1024 vectors of 8 logits), then NaN up to
    # the end of its range: one contiguous run
    first, last = int(idx[0]), int(idx[-1])
    assert first == 3 * 1024 * 8
    assert int(idx.numel()) == last - first + 1
    assert torch.equal(flat[~bad], want[~bad])

    # the context is still usable: the same call without the knob is clean and exact
    d2 = backward(lib, x, t, l, h, gl, gh)
    assert status(lib) == 0
    assert torch.equal(d2, ref)


def test_forward_row_slot_wait_runs_out():
    lib = test_lib()
    x, t = inputs()
    ref = product_outputs(x, t)
    torch.cuda.synchronize()
    assert status(lib) == 0
    assert lib.k1_test_set_knobs(-1, 0) == 0
    try:
        out = forward(lib, x, t)
        st = status(lib)
    finally:
        assert lib.k1_test_set_knobs(-1, -1) == 0
    assert st & 4, f"status {st}: the row slot's wait did not report running out"
    G = torch.cuda.get_device_properties(0).multi_processor_count
    # block 0 owns rows 0, G, 2G, ...; row 0 lost a grab, and row 4G (the next row of
    # slot 0 of 4) could not park its grabs
    stuck = {0, 4 * G}
    for o, r in zip(out, ref):
        nan_rows = set(torch.isnan(o).nonzero().view(-1).tolist())
        assert nan_rows == stuck, f"NaN rows {sorted(nan_rows)}, expected {sorted(stuck)}"
        keep = ~torch.isnan(o)
        assert torch.equal(o[keep], r[keep])

    out2 = forward(lib, x, t)
    assert status(lib) == 0
    for o, r in zip(out2, ref):
        assert torch.equal(o, r)


def test_check_waits_switch_is_quiet_when_nothing_runs_out():
    """With the debug switch on, ordinary calls of the product library still pass (each
    reads the status word after its launch)."""
    import kernel_opt
    x, t = inputs(N=300, V=32768)
    was = kernel_opt.check_waits()
    kernel_opt.set_check_waits(True)
    try:
        xr = x.detach().requires_grad_(True)
        lp, h, _ = kernel_opt.fused_logprob_entropy(xr, t)
        (d,) = torch.autograd.grad((lp, h), xr, (torch.ones_like(lp), torch.ones_like(h)))
        torch.cuda.synchronize()
        assert torch.isfinite(d).all()
    finally:
        kernel_opt.set_check_waits(was)


def _lmh_api(lib):
    i64, p, f32 = ctypes.c_int64, ctypes.c_void_p, ctypes.c_float
    lib.k1_lm_head_workspace_bytes.argtypes = [i64, i64, i64, ctypes.c_int]
    lib.k1_lm_head_workspace_bytes.restype = ctypes.c_size_t
    lib.k1_lm_head_forward.argtypes = [p, p, i64, i64, i64, f32, p, p, p, p, p, i64, p,
                                       ctypes.c_size_t, p]
    lib.k1_lm_head_backward.argtypes = [p, p, i64, i64, i64, f32, p, p, p, p, p, p, p, i64, p]
    return lib


def _lmh_run(lib, h, w, t, scale, lse=None, ent=None, gl=None):
    N, H = h.shape
    V = w.shape[0]
    s = torch.cuda.current_stream().cuda_stream
    if lse is None:
        ws = torch.empty(lib.k1_lm_head_workspace_bytes(N, H, V, 0), dtype=torch.uint8,
                         device="cuda")
        out = [torch.full((N,), 7.0, device="cuda") for _ in range(3)]
        rc = lib.k1_lm_head_forward(h.data_ptr(), w.data_ptr(), N, H, V, scale, t.data_ptr(),
                                    *(o.data_ptr() for o in out), None, V, ws.data_ptr(),
                                    ws.numel(), s)
        assert rc == 0, lib.k1_last_error()
        torch.cuda.synchronize()
        return out
    d = torch.full((N, V), 7.0, dtype=torch.bfloat16, device="cuda")
    rc = lib.k1_lm_head_backward(h.data_ptr(), w.data_ptr(), N, H, V, scale, t.data_ptr(),
                                 lse.data_ptr(), ent.data_ptr(), gl.data_ptr(), None, None,
                                 d.data_ptr(), V, s)
    assert rc == 0, lib.k1_last_error()
    torch.cuda.synchronize()
    return d


def test_lm_head_wait_runs_out():
    """The tensor-core LM head: CTA 0 issues no tile copy from its 2nd stage on (every tile
    here takes two stages: H = 256 in K blocks of 128), so its MMA's wait for that stage
    runs out; the kernel returns, sets bit 3, the forward's statistics become NaN (a unit
    is missing, so every row is) and the gradient's unfinished tiles NaN."""
    lib = _lmh_api(test_lib())
    prod = _lmh_api(ctypes.CDLL(CAPI_LIB))
    g = torch.Generator(device="cuda").manual_seed(21)
    N, H, V = 512, 256, 4096
    h = (torch.randn(N, H, generator=g, device="cuda") * 0.5).to(torch.bfloat16)
    w = (torch.randn(V, H, generator=g, device="cuda") * 0.15).to(torch.bfloat16)
    t = torch.randint(0, V, (N,), generator=g, device="cuda")
    gl = torch.full((N,), -1.0 / N, device="cuda")
    ref = _lmh_run(prod, h, w, t, 1.0)
    dref = _lmh_run(prod, h, w, t, 1.0, ref[2], ref[1], gl)
    assert status(lib) == 0

    assert lib.k1_test_set_knobs(1, -1) == 0
    try:
        out = _lmh_run(lib, h, w, t, 1.0)
        st_f = status(lib)
        d = _lmh_run(lib, h, w, t, 1.0, ref[2], ref[1], gl)
        st_b = status(lib)
    finally:
        assert lib.k1_test_set_knobs(-1, -1) == 0
    assert st_f & 8 and st_b & 8, f"status {st_f}, {st_b}: the LM head's wait did not report"
    for o in out:
        assert torch.isnan(o).all()
    bad = torch.isnan(d.float())
    assert bad.any()
    assert torch.equal(d[~bad], dref[~bad])

    # the same context, knob off: clean and identical to the product library
    out2 = _lmh_run(lib, h, w, t, 1.0)
    d2 = _lmh_run(lib, h, w, t, 1.0, ref[2], ref[1], gl)
    assert status(lib) == 0
    for a, b in zip(out2, ref):
        assert torch.equal(a, b)
    assert torch.equal(d2, dref)

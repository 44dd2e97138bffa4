"""The C-ABI library (libk1_b200.so) loads without a GPU, exports every function that
include/k1_logprob.h declares, and rejects bad arguments before touching the device."""
import ctypes

import pytest

from _helpers import CAPI_LIB, WAIT_TEST_LIB, header_functions

K1_OK, K1_ERR_INVALID, K1_ERR_DTYPE, K1_ERR_WS = 0, 1, 2, 3


@pytest.fixture(scope="module")
def lib():
    return ctypes.CDLL(CAPI_LIB)


def test_header_declares_expected_entry_points():
    names = header_functions()
    for n in ("k1_fused_logprob_entropy_v1", "k1_fused_logprob_entropy_naive",
              "k1_fused_logprob_entropy_v1_backward", "k1_vocab_shard_partials",
              "k1_vocab_combine", "k1_vocab_shard_backward", "k1_forward_workspace_bytes",
              "k1_last_error", "k1_abi_version"):
        assert n in names


def test_every_declared_symbol_is_exported(lib):
    missing = [n for n in header_functions() if not hasattr(lib, n)]
    assert not missing, f"declared but not exported: {missing}"


def test_wait_test_knobs_only_in_the_test_library(lib):
    """The wait-timeout knobs are compiled into the test library alone; the product library
    has no way to make a kernel's wait run out."""
    assert not hasattr(lib, "k1_test_set_knobs")
    test_lib = ctypes.CDLL(WAIT_TEST_LIB)
    assert hasattr(test_lib, "k1_test_set_knobs")
    missing = [n for n in header_functions() if not hasattr(test_lib, n)]
    assert not missing


def test_abi_version(lib):
    lib.k1_abi_version.restype = ctypes.c_int
    assert lib.k1_abi_version() == 2


def _fwd(lib, dtype=2, n_rows=4, vocab=16, inner_rows=4, inner_stride=16, outer=0,
         logits=1024, targets=2048, out=4096, ws=8192, ws_bytes=1 << 20):
    f = lib.k1_fused_logprob_entropy_v1
    i64, p = ctypes.c_int64, ctypes.c_void_p
    f.argtypes = [p, ctypes.c_int, i64, i64, i64, i64, i64, p, p, p, p, p, ctypes.c_size_t, p]
    f.restype = ctypes.c_int
    return f(logits, dtype, n_rows, vocab, inner_rows, inner_stride, outer, targets, out, out,
             out, ws, ws_bytes, None)


def _err(lib):
    lib.k1_last_error.restype = ctypes.c_char_p
    return lib.k1_last_error().decode()


def test_rejects_bad_dtype(lib):
    assert _fwd(lib, dtype=7) == K1_ERR_DTYPE
    assert "bf16, fp16, or fp32" in _err(lib)


def test_rejects_bad_shapes(lib):
    assert _fwd(lib, vocab=0) == K1_ERR_INVALID
    assert "vocab" in _err(lib)
    assert _fwd(lib, n_rows=5, inner_rows=2) == K1_ERR_INVALID
    assert "inner_rows" in _err(lib)
    assert _fwd(lib, n_rows=-1) == K1_ERR_INVALID
    assert _fwd(lib, inner_stride=-3) == K1_ERR_INVALID


def test_rejects_null_and_misaligned_pointers(lib):
    assert _fwd(lib, logits=0) == K1_ERR_INVALID
    assert "NULL" in _err(lib)
    assert _fwd(lib, logits=1025) == K1_ERR_INVALID  # bf16 needs 2-byte alignment
    assert "aligned" in _err(lib)
    assert _fwd(lib, targets=0) == K1_ERR_INVALID


def test_zero_rows_is_a_no_op(lib):
    assert _fwd(lib, n_rows=0, logits=0, targets=0, out=0, ws=0) == K1_OK


def test_backward_and_combine_validation(lib):
    i64, p, c_int = ctypes.c_int64, ctypes.c_void_p, ctypes.c_int
    b = lib.k1_fused_logprob_entropy_v1_backward
    b.argtypes = [p, c_int, i64, i64, i64, i64, i64, p, p, p, p, p, p, p, i64, i64, p]
    b.restype = c_int
    assert b(1024, 9, 4, 16, 4, 16, 0, 2048, 4096, 4096, None, None, None, 8192, 16, 0,
             None) == K1_ERR_DTYPE
    assert b(1024, 2, 4, 16, 4, 16, 0, 2048, 4096, 4096, None, None, None, 0, 16, 0,
             None) == K1_ERR_INVALID
    c = lib.k1_vocab_combine
    c.argtypes = [p, c_int, i64, p, p, p, p]
    c.restype = c_int
    assert c(1024, 0, 4, 4096, 4096, 4096, None) == K1_ERR_INVALID
    v = lib.k1_vocab_shard_partials
    v.argtypes = [p, c_int, i64, i64, i64, i64, i64, i64, p, p, p, ctypes.c_size_t, p]
    v.restype = c_int
    assert v(1024, 2, 4, 16, 4, 16, 0, -5, 2048, 4096, 8192, 1 << 20, None) == K1_ERR_INVALID


def test_scaled_entry_points_validate_scale(lib):
    """The scaled forward / backward reject a scale that is not positive and finite
    before any device call (so this runs without a GPU)."""
    i64, p, c_int, c_float = ctypes.c_int64, ctypes.c_void_p, ctypes.c_int, ctypes.c_float
    f = lib.k1_fused_logprob_entropy_scaled
    f.argtypes = [p, c_int, i64, i64, i64, i64, i64, c_float, p, p, p, p, p, ctypes.c_size_t, p]
    f.restype = c_int
    b = lib.k1_fused_logprob_entropy_scaled_backward
    b.argtypes = [p, c_int, i64, i64, i64, i64, i64, c_float, p, p, p, p, p, p, p, i64, i64, p]
    b.restype = c_int
    for s in (0.0, -0.5, float("inf"), float("nan")):
        assert f(1024, 2, 4, 16, 4, 16, 0, s, 2048, 4096, 4096, 4096, 8192, 1 << 20,
                 None) == K1_ERR_INVALID
        assert "scale" in _err(lib)
        assert b(1024, 2, 4, 16, 4, 16, 0, s, 2048, 4096, 4096, None, None, None, 8192, 16, 0,
                 None) == K1_ERR_INVALID
        assert "scale" in _err(lib)
    # dtype is still checked first, and zero rows are a no-op
    assert f(1024, 7, 4, 16, 4, 16, 0, 1.5, 2048, 4096, 4096, 4096, 8192, 1 << 20,
             None) == K1_ERR_DTYPE
    assert f(0, 2, 0, 16, 1, 16, 0, 1.5, 0, 0, 0, 0, 0, 0, None) == K1_OK


def test_lm_head_entry_points_validate_before_the_device(lib):
    """The tensor-core LM head rejects bad sizes, pointers and scales before any device
    call (so this runs without a GPU)."""
    i64, p, c_float = ctypes.c_int64, ctypes.c_void_p, ctypes.c_float
    f = lib.k1_lm_head_forward
    f.argtypes = [p, p, i64, i64, i64, c_float, p, p, p, p, p, i64, p, ctypes.c_size_t, p]
    f.restype = ctypes.c_int
    b = lib.k1_lm_head_backward
    b.argtypes = [p, p, i64, i64, i64, c_float, p, p, p, p, p, p, p, i64, p]
    b.restype = ctypes.c_int
    ok = dict(h=4096, w=8192, n=4, hd=64, v=100, s=1.0)

    def fwd(**kw):
        a = {**ok, **kw}
        return f(a["h"], a["w"], a["n"], a["hd"], a["v"], a["s"], 1 << 16, 1 << 17, 1 << 17,
                 1 << 17, None, a["v"], 1 << 18, 1 << 20, None)

    assert fwd(h=0) == K1_ERR_INVALID and "NULL" in _err(lib)
    assert fwd(hd=60) == K1_ERR_INVALID and "multiple of 8" in _err(lib)
    assert fwd(w=8200) == K1_ERR_INVALID and "aligned" in _err(lib)
    assert fwd(v=0) == K1_ERR_INVALID
    for s in (0.0, -1.0, float("inf"), float("nan")):
        assert fwd(s=s) == K1_ERR_INVALID and "scale" in _err(lib)
    assert fwd(n=0) == K1_OK
    assert b(4096, 8192, 4, 64, 100, 1.0, 1 << 16, 1 << 17, 1 << 17, None, None, None,
             1 << 18, 99, None) == K1_ERR_INVALID and "d_stride" in _err(lib)
    lib.k1_lm_head_workspace_bytes.argtypes = [i64, i64, i64, ctypes.c_int]
    lib.k1_lm_head_workspace_bytes.restype = ctypes.c_size_t
    assert lib.k1_lm_head_workspace_bytes(0, 64, 100, 0) == 0


def test_lm_head_shard_entry_points_validate_before_the_device(lib):
    """The vocab-parallel LM head entry points reject a negative vocabulary offset, a NULL
    partials buffer and the LM head's own bad arguments before any device call."""
    i64, p, c_float = ctypes.c_int64, ctypes.c_void_p, ctypes.c_float
    f = lib.k1_lm_head_shard_partials
    f.argtypes = [p, p, i64, i64, i64, i64, c_float, p, p, p, i64, p, ctypes.c_size_t, p]
    f.restype = ctypes.c_int
    b = lib.k1_lm_head_shard_backward
    b.argtypes = [p, p, i64, i64, i64, i64, c_float, p, p, p, p, p, p, p, i64, p]
    b.restype = ctypes.c_int
    assert f(4096, 8192, 4, 64, 100, -1, 1.0, 1 << 16, 1 << 17, None, 100, 1 << 18, 1 << 20,
             None) == K1_ERR_INVALID and "vocab_offset" in _err(lib)
    assert f(4096, 8192, 4, 64, 100, 200, 1.0, 1 << 16, None, None, 100, 1 << 18, 1 << 20,
             None) == K1_ERR_INVALID and "partials" in _err(lib)
    assert f(4096, 8192, 4, 60, 100, 200, 1.0, 1 << 16, 1 << 17, None, 100, 1 << 18, 1 << 20,
             None) == K1_ERR_INVALID and "multiple of 8" in _err(lib)
    assert f(4096, 8192, 4, 64, 100, 200, 1.0, 1 << 16, 1 << 17, 1 << 19, 99, 1 << 18, 1 << 20,
             None) == K1_ERR_INVALID and "logits_stride" in _err(lib)
    assert f(4096, 8192, 0, 64, 100, 200, 1.0, 1 << 16, None, None, 0, None, 0, None) == K1_OK
    sb = lib.k1_vocab_shard_scaled_backward
    sb.argtypes = [p, ctypes.c_int, i64, i64, i64, i64, i64, i64, c_float, p, p, p, p, p, p, p,
                   i64, i64, p]
    sb.restype = ctypes.c_int
    for s in (0.0, float("nan")):
        assert sb(1024, 2, 4, 16, 4, 16, 0, 0, s, 2048, 4096, 4096, None, None, None, 8192, 16, 0,
                  None) == K1_ERR_INVALID and "scale" in _err(lib)
    assert sb(1024, 2, 4, 16, 4, 16, 0, -3, 1.5, 2048, 4096, 4096, None, None, None, 8192, 16, 0,
              None) == K1_ERR_INVALID and "vocab_offset" in _err(lib)
    assert b(4096, 8192, 4, 64, 100, -5, 1.0, 1 << 16, 1 << 17, 1 << 17, None, None, None,
             1 << 18, 100, None) == K1_ERR_INVALID and "vocab_offset" in _err(lib)
    assert b(4096, 8192, 4, 64, 100, 200, 0.0, 1 << 16, 1 << 17, 1 << 17, None, None, None,
             1 << 18, 100, None) == K1_ERR_INVALID and "scale" in _err(lib)

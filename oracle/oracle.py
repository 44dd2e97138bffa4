"""TEST INFRASTRUCTURE ONLY.  ctypes front end of the fp64 C oracle (k1_oracle.c).

Every function takes CPU torch tensors (bf16 / fp16 / fp32 logits as stored, int64
targets) and returns float64 numpy arrays.  Logits are handed to C as a contiguous
[N, V] copy, so the checker never depends on the product's stride handling.
"""
from __future__ import annotations

import ctypes
import os

import numpy as np
import torch

from .build import LIB, build

_DTYPE = {torch.float32: 0, torch.float16: 1, torch.bfloat16: 2}
_lib = None


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        if not os.path.exists(LIB):
            build()
        L = ctypes.CDLL(LIB)
        i64, p, c_int = ctypes.c_int64, ctypes.c_void_p, ctypes.c_int
        L.k1o_forward.argtypes = [p, c_int, i64, i64, i64, i64, i64, p, p, p, p, c_int]
        L.k1o_backward.argtypes = [p, c_int, i64, i64, i64, i64, i64, p, p, p, p, p, p, p, c_int]
        L.k1o_shard_partials.argtypes = [p, c_int, i64, i64, i64, i64, i64, i64, p, p, p, p, p,
                                         p, c_int]
        L.k1o_combine.argtypes = [p, p, p, p, p, c_int, i64, p, p, p]
        for f in (L.k1o_forward, L.k1o_backward, L.k1o_shard_partials, L.k1o_combine):
            f.restype = c_int
        _lib = L
    return _lib


def _ptr(a) -> int:
    if isinstance(a, torch.Tensor):
        return a.data_ptr()
    return a.ctypes.data


def _rows(logits: torch.Tensor):
    x = logits.detach().to("cpu").contiguous()
    V = x.shape[-1]
    x2 = x.reshape(-1, V)
    return x2, x2.shape[0], V


def forward(logits: torch.Tensor, targets: torch.Tensor, n_threads: int = 0):
    """(logprob, entropy, lse) in fp64; shapes of targets (flattened order)."""
    x, N, V = _rows(logits)
    t = targets.detach().to("cpu", torch.int64).contiguous().reshape(-1)
    assert t.numel() == N
    lp, h, l = (np.empty(N, np.float64) for _ in range(3))
    rc = lib().k1o_forward(_ptr(x), _DTYPE[x.dtype], N, V, max(N, 1), V, 0, _ptr(t),
                           _ptr(lp), _ptr(h), _ptr(l), n_threads)
    assert rc == 0
    shape = tuple(targets.shape)
    return lp.reshape(shape), h.reshape(shape), l.reshape(shape)


def backward(logits: torch.Tensor, targets: torch.Tensor, lse, entropy, g_logp=None,
             g_ent=None, g_lse=None, n_threads: int = 0):
    """d_logits in fp64, shape of logits.  lse / entropy: forward values to use."""
    x, N, V = _rows(logits)
    t = targets.detach().to("cpu", torch.int64).contiguous().reshape(-1)

    def f64(a):
        if a is None:
            return None
        if isinstance(a, torch.Tensor):
            a = a.detach().to("cpu", torch.float64).numpy()
        return np.ascontiguousarray(np.asarray(a, np.float64).reshape(-1))

    l, h = f64(lse), f64(entropy)
    gl, ge, gs = f64(g_logp), f64(g_ent), f64(g_lse)
    out = np.empty((N, V), np.float64)
    rc = lib().k1o_backward(_ptr(x), _DTYPE[x.dtype], N, V, max(N, 1), V, 0, _ptr(t),
                            _ptr(l), _ptr(h), None if gl is None else _ptr(gl),
                            None if ge is None else _ptr(ge), None if gs is None else _ptr(gs),
                            _ptr(out), n_threads)
    assert rc == 0
    return out.reshape(tuple(logits.shape))


def shard_partials(logits_shard: torch.Tensor, targets: torch.Tensor, vocab_offset: int,
                   n_threads: int = 0):
    """Per-row (m, z, t, x_t, has_target) of a vocabulary shard, as an [N, 4] float64
    array in the k1_partial word layout (z, t, then m / x_t and has_target packed)."""
    x, N, V = _rows(logits_shard)
    t = targets.detach().to("cpu", torch.int64).contiguous().reshape(-1)
    m, z, tt, xt = (np.empty(N, np.float64) for _ in range(4))
    has = np.empty(N, np.int32)
    rc = lib().k1o_shard_partials(_ptr(x), _DTYPE[x.dtype], N, V, max(N, 1), V, 0,
                                  int(vocab_offset), _ptr(t), _ptr(m), _ptr(z), _ptr(tt),
                                  _ptr(xt), _ptr(has), n_threads)
    assert rc == 0
    return pack_partials(m, z, tt, xt, has)


def pack_partials(m, z, t, xt, has) -> np.ndarray:
    """Arrays -> [N, 4] float64 words with the k1_partial struct layout."""
    N = len(m)
    rec = np.zeros(N, dtype=np.dtype([("z", "<f8"), ("t", "<f8"), ("m", "<f4"),
                                      ("x_t", "<f4"), ("has", "<i4"), ("res", "<i4")]))
    rec["z"], rec["t"], rec["m"], rec["x_t"], rec["has"] = z, t, m, xt, has
    return rec.view(np.float64).reshape(N, 4)


def unpack_partials(words: np.ndarray):
    """[..., N, 4] float64 words -> dict of arrays (m, z, t, x_t, has)."""
    w = np.ascontiguousarray(np.asarray(words, np.float64))
    rec = w.reshape(-1, 4).view(np.dtype([("z", "<f8"), ("t", "<f8"), ("m", "<f4"),
                                           ("x_t", "<f4"), ("has", "<i4"), ("res", "<i4")]))
    rec = rec.reshape(w.shape[:-1])
    return {k: np.ascontiguousarray(rec[k]) for k in ("m", "z", "t", "x_t", "has")}


def combine(gathered_words: np.ndarray):
    """[n_shards, N, 4] partial words -> (logprob, entropy, lse) fp64."""
    u = unpack_partials(gathered_words)
    S, N = u["m"].shape
    m = np.ascontiguousarray(u["m"].astype(np.float64))
    z, t = np.ascontiguousarray(u["z"]), np.ascontiguousarray(u["t"])
    xt = np.ascontiguousarray(u["x_t"].astype(np.float64))
    has = np.ascontiguousarray(u["has"].astype(np.int32))
    lp, h, l = (np.empty(N, np.float64) for _ in range(3))
    rc = lib().k1o_combine(_ptr(m), _ptr(z), _ptr(t), _ptr(xt), _ptr(has), S, N, _ptr(lp),
                           _ptr(h), _ptr(l))
    assert rc == 0
    return lp, h, l

"""Forward with one block per SM (k1_fwd_sm_kernel): a few wide rows per SM, each row cut
into fixed grabs that the block's warps take in turn and merged in grab order.

Launches with at least one row per SM, rows of at least 24 chunks (6144 vectors) and at
most 8192 chunks per SM select it.  Results must meet the oracle's tolerances, repeat bit
for bit (whichever warp took a grab), and handle -inf in some or all grabs of a row (the
clamped re-reduction of a grab), NaN and +inf, targets in the first and last grab, the
ignore index, near-one-hot rows, strided GRPO-window layouts, temperature scaling and
vocabulary-shard partials.
"""
import numpy as np
import pytest
import torch

import kernel_opt
from _gpu import check_forward_outputs, seeded_logits, seeded_targets

pytestmark = pytest.mark.gpu

SHAPES = [
    (148, 152064, torch.bfloat16),   # one row per SM
    (1024, 152064, torch.bfloat16),  # config 2
    (600, 65536, torch.float16),
    (400, 128256, torch.float32),
    (2000, 98304, torch.bfloat16),
]


def _edge_rows(x, t):
    V = x.shape[1]
    t[0], t[1], t[2] = 0, V - 1, -100
    x[3, ::7] = float("-inf")          # -inf in every grab
    x[4, :] = float("-inf")            # nothing but -inf
    x[5, : V - 3] = float("-inf")      # one grab with finite logits
    x[6, V // 2] = float("nan")
    x[7, 11] = float("inf")
    x[8, V - 2] = float("-inf")        # a single -inf in the last grab
    x[9, int(t[9])] += 40.0            # near one-hot
    t[3], t[4], t[5], t[8] = 7, 1, V - 1, V - 2


@pytest.mark.parametrize("rows,vocab,dtype", SHAPES)
def test_sm_forward_matches_oracle_and_repeats(rows, vocab, dtype):
    x = seeded_logits((rows, vocab), torch.float32, 3.0, seed=rows + vocab)
    t = seeded_targets((rows,), vocab, seed=rows)
    _edge_rows(x, t)
    x = x.to(dtype)
    xg, tg = x.cuda(), t.cuda()
    first = kernel_opt.fused_logprob_entropy_forward(xg, tg)
    idx = torch.cat([torch.arange(0, 24), torch.arange(rows // 2, rows // 2 + 8),
                     torch.arange(rows - 24, rows)])
    check_forward_outputs(tuple(o[idx.cuda()] for o in first), x[idx], t[idx],
                          f"sm {rows}x{vocab} {dtype}")
    for _ in range(3):
        again = kernel_opt.fused_logprob_entropy_forward(xg, tg)
        for a, b in zip(first, again):
            torch.testing.assert_close(a, b, rtol=0, atol=0, equal_nan=True)


def test_sm_forward_strided_window_and_temperature():
    """The GRPO window of a [B, L, V] parent (row stride L*V, a batch boundary every L-1
    rows): same bits as the contiguous copy, and the folded temperature gives the same
    bits as dividing first."""
    from kernel_opt import _C, grpo
    B, L, V = 4, 301, 131072
    parent = seeded_logits((B, L, V), torch.bfloat16, 2.5, seed=21).cuda()
    win = parent[:, :-1]
    t = seeded_targets((B, L - 1), V, seed=22).cuda()
    a = kernel_opt.fused_logprob_entropy_forward(win, t)
    b = kernel_opt.fused_logprob_entropy_forward(win.contiguous(), t)
    for u, v in zip(a, b):
        torch.testing.assert_close(u, v, rtol=0, atol=0)
    T = 0.7
    n = B * (L - 1)
    s1 = [torch.empty((B, L - 1), device="cuda") for _ in range(3)]
    s2 = [torch.empty((B, L - 1), device="cuda") for _ in range(3)]
    y = win.contiguous().div_(T)
    _C.fused_logprob_entropy_scaled(win, t, *s1, grpo.temperature_scale(T))
    _C.fused_logprob_entropy_v1(y, t, *s2)
    for u, v in zip(s1, s2):
        torch.testing.assert_close(u, v, rtol=0, atol=0)
    idx = torch.tensor([0, 299, 300, 301, 899, 1199])
    check_forward_outputs(tuple(o.reshape(-1)[idx.cuda()] for o in s1),
                          y.reshape(n, V)[idx.cuda()].cpu(), t.reshape(-1).cpu()[idx],
                          "sm window scaled")


def test_sm_shard_partials():
    from kernel_opt import _C
    from oracle import oracle
    rows, V, off = 600, 98304, 50000
    x = seeded_logits((rows, V), torch.bfloat16, 3.0, seed=31)
    t = seeded_targets((rows,), V + 2 * off, seed=32)   # some targets outside the shard
    t[0], t[1], t[2] = off, off + V - 1, -100
    xg, tg = x.cuda(), t.cuda()
    parts = torch.empty((rows, 4), dtype=torch.float64, device="cuda")
    _C.vocab_shard_partials(xg, tg, off, parts)
    sub = torch.cat([torch.arange(0, 32), torch.arange(rows - 32, rows)])
    want = oracle.unpack_partials(oracle.shard_partials(x[sub], t[sub], off))
    got = oracle.unpack_partials(parts[sub.cuda()].cpu().numpy())
    np.testing.assert_array_equal(got["has"], want["has"])
    np.testing.assert_allclose(got["m"], want["m"], rtol=0, atol=0)
    np.testing.assert_allclose(got["z"], want["z"], rtol=1e-5)
    np.testing.assert_allclose(got["x_t"], want["x_t"], rtol=0, atol=0)


def test_sm_scaled_equals_divided_at_config2():
    """The scaled forward runs with more warps and no prefetch buffer; a grab's arithmetic
    is the same, so it keeps the bits of the unscaled forward on pre-divided logits."""
    from kernel_opt import _C, grpo
    N, V, T = 1024, 152064, 0.85
    x = seeded_logits((N, V), torch.bfloat16, 3.0, seed=41).cuda()
    t = seeded_targets((N,), V, seed=42).cuda()
    a = [torch.empty(N, device="cuda") for _ in range(3)]
    b = [torch.empty(N, device="cuda") for _ in range(3)]
    _C.fused_logprob_entropy_scaled(x, t, *a, grpo.temperature_scale(T))
    _C.fused_logprob_entropy_v1(x.clone().div_(T), t, *b)
    for u, v in zip(a, b):
        torch.testing.assert_close(u, v, rtol=0, atol=0)

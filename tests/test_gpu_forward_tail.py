"""Forward work distribution.  Row groups (k1_fwd_rows_kernel: groups of 1, 2, 4 or 8
warps taking whole rows from an atomic queue) serve launches with enough rows; the block
kernel (rows split between blocks, with a dynamic tail of whole-row chunks from 4 rows per
block) serves the rest and the scalar path.  Results must meet the oracle's tolerances, be
bit-identical from run to run (which group or block takes a row or chunk must not
matter), leave the queue counters zeroed for the next call, and agree between the strided
and contiguous layouts."""
import pytest
import torch

import kernel_opt
from _gpu import check_forward_outputs, seeded_logits, seeded_targets

pytestmark = pytest.mark.gpu

# (rows, vocab, dtype) on 148 SMs: row groups of several sizes, and the scalar path
# (a vocab whose rows are not 16-byte multiples) through the block kernel with its tail
SHAPES = [
    (20000, 256, torch.bfloat16),
    (3000, 4096, torch.float32),
    (2500, 2048, torch.float16),
    (1777, 1003, torch.bfloat16),    # scalar path: block kernel, dynamic tail
    (40000, 3001, torch.float32),    # scalar path: multi-row tail chunks (owner cap)
]


@pytest.mark.parametrize("rows,vocab,dtype", SHAPES)
def test_tail_matches_oracle_and_repeats_bit_for_bit(rows, vocab, dtype):
    x = seeded_logits((rows, vocab), dtype, 3.0, seed=rows)
    t = seeded_targets((rows,), vocab, seed=rows + 1)
    t[5] = -100
    xg, tg = x.cuda(), t.cuda()
    first = kernel_opt.fused_logprob_entropy_forward(xg, tg)
    # oracle on a row subsample that covers the static pieces and the tail
    idx = torch.cat([torch.arange(0, 40), torch.arange(rows // 2, rows // 2 + 40),
                     torch.arange(rows - 200, rows)])
    check_forward_outputs(tuple(o[idx.cuda()] for o in first), x[idx], t[idx],
                          f"tail {rows}x{vocab} {dtype}")
    # a different shape in between, then the same call again: identical bits
    y = seeded_logits((4096, 512), dtype, 3.0, seed=7).cuda()
    kernel_opt.fused_logprob_entropy_forward(y, seeded_targets((4096,), 512, seed=8).cuda())
    for _ in range(3):
        again = kernel_opt.fused_logprob_entropy_forward(xg, tg)
        for a, b in zip(first, again):
            torch.testing.assert_close(a, b, rtol=0, atol=0)


def test_tail_strided_window_equals_contiguous():
    B, L, V = 8, 513, 4096
    parent = seeded_logits((B, L, V), torch.bfloat16, 2.5, seed=3).cuda()
    win = parent[:, :-1]
    t = seeded_targets((B, L - 1), V, seed=4).cuda()
    a = kernel_opt.fused_logprob_entropy_forward(win, t)
    b = kernel_opt.fused_logprob_entropy_forward(win.contiguous(), t)
    for u, v in zip(a, b):
        torch.testing.assert_close(u, v, rtol=0, atol=0)


# Row groups: the smallest group of 1, 2 or 4 warps with >= 3 rows each, else 8-warp
# groups with >= 2 rows each (444 blocks of 8 warps on 148 SMs); these shapes select each.
ROW_GROUP_SHAPES = [
    (60000, 512, torch.bfloat16),   # one-warp groups
    (8000, 1024, torch.float16),    # two-warp groups
    (4000, 4096, torch.float32),    # four-warp groups
    (2000, 2048, torch.bfloat16),   # whole-block groups
    (600, 8192, torch.bfloat16),    # block kernel (too few rows for groups)
]


@pytest.mark.parametrize("rows,vocab,dtype", ROW_GROUP_SHAPES)
def test_row_groups_match_oracle_and_repeat(rows, vocab, dtype):
    x = seeded_logits((rows, vocab), dtype, 3.0, seed=rows + 5)
    t = seeded_targets((rows,), vocab, seed=rows + 6)
    t[7] = -100
    x.view(-1, vocab)[11, ::5] = float("-inf")  # the clamped re-stream inside a group
    xg, tg = x.cuda(), t.cuda()
    first = kernel_opt.fused_logprob_entropy_forward(xg, tg)
    idx = torch.cat([torch.arange(0, 64), torch.arange(rows - 64, rows)])
    check_forward_outputs(tuple(o[idx.cuda()] for o in first), x[idx], t[idx],
                          f"row groups {rows}x{vocab} {dtype}")
    for _ in range(2):
        again = kernel_opt.fused_logprob_entropy_forward(xg, tg)
        for a, b in zip(first, again):
            torch.testing.assert_close(a, b, rtol=0, atol=0)


def test_row_groups_scaled_and_shard():
    from kernel_opt import _C, grpo
    from oracle import oracle
    rows, V = 60000, 512
    x = seeded_logits((rows, V), torch.bfloat16, 3.0, seed=9).cuda()
    t = seeded_targets((rows,), V, seed=10).cuda()
    # temperature folded in == division first (same launch shape, same bits)
    T = 0.85
    a = [torch.empty(rows, device="cuda") for _ in range(3)]
    b = [torch.empty(rows, device="cuda") for _ in range(3)]
    _C.fused_logprob_entropy_scaled(x, t, *a, grpo.temperature_scale(T))
    _C.fused_logprob_entropy_v1(x.clone().div_(T), t, *b)
    for u, v in zip(a, b):
        torch.testing.assert_close(u, v, rtol=0, atol=0)
    # vocabulary shard partials against the oracle's restatement
    off = 1000
    parts = torch.empty((rows, 4), dtype=torch.float64, device="cuda")
    tt = t + off
    _C.vocab_shard_partials(x, tt, off, parts)
    want = oracle.unpack_partials(oracle.shard_partials(x[:256].cpu(), tt[:256].cpu(), off))
    got = oracle.unpack_partials(parts[:256].cpu().numpy())
    import numpy as np
    np.testing.assert_array_equal(got["has"], want["has"])
    np.testing.assert_allclose(got["m"], want["m"], rtol=0, atol=0)
    np.testing.assert_allclose(got["z"], want["z"], rtol=1e-5)
    np.testing.assert_allclose(got["x_t"], want["x_t"], rtol=0, atol=0)


# Vocabularies that are not whole 16-byte vectors (GPT-2's 50257, odd shard widths): rows
# are peeled into single-element head and tail around an aligned vector interior.
PEELED = [
    (12000, 50257, torch.bfloat16),   # row groups, one-warp groups
    (1500, 50257, torch.float16),     # row groups, whole-block groups
    (300, 32001, torch.bfloat16),     # block kernel (rows split between blocks)
    (2000, 12347, torch.float32),
]


@pytest.mark.parametrize("rows,vocab,dtype", PEELED)
def test_peeled_rows_forward_and_backward(rows, vocab, dtype):
    from _gpu import check_grad, grads_like
    from kernel_opt import _C
    x = seeded_logits((rows, vocab), dtype, 3.0, seed=vocab)
    t = seeded_targets((rows,), vocab, seed=vocab + 1)
    t[0], t[1], t[2] = 0, vocab - 1, -100   # targets in the head / tail elements
    x.view(-1, vocab)[3, 1::7] = float("-inf")
    xg, tg = x.cuda(), t.cuda()
    outs = kernel_opt.fused_logprob_entropy_forward(xg, tg)
    idx = torch.cat([torch.arange(0, 48), torch.arange(rows - 48, rows)])
    fwd = check_forward_outputs(tuple(o[idx.cuda()] for o in outs), x[idx], t[idx],
                                f"peeled {rows}x{vocab} {dtype}")
    g = grads_like((rows,), seed=vocab + 2)
    lp, h, l = outs
    d = torch.empty_like(xg)
    _C.fused_logprob_entropy_v1_backward(xg, tg, l, h, *(a.cuda() for a in g), d)
    sub = idx[:16]
    check_grad(d[sub.cuda()], x[sub], t[sub], *(a[sub] for a in g), what="peeled bwd",
               fwd=tuple(a[:16] for a in fwd))
    # in place: same bits as out of place (the backward is elementwise)
    d2 = xg.clone()
    _C.fused_logprob_entropy_v1_backward(d2, tg, l, h, *(a.cuda() for a in g), d2)
    torch.testing.assert_close(d2, d, rtol=0, atol=0)


def test_peeled_backward_gradient_layout_with_other_alignment():
    """A gradient view whose rows are misaligned differently from the logits rows (a
    slice of a wider buffer) takes the single-element path; ring, register and element
    paths compute the same bits."""
    from _gpu import grads_like
    from kernel_opt import _C
    N, V = 3000, 50257
    x = seeded_logits((N, V), torch.bfloat16, 3.0, seed=77).cuda()
    t = seeded_targets((N,), V, seed=78).cuda()
    lp, h, l = kernel_opt.fused_logprob_entropy_forward(x, t)
    g = [a.cuda() for a in grads_like((N,), seed=79)]
    d_same = torch.empty_like(x)                       # congruent: peeled ring
    _C.fused_logprob_entropy_v1_backward(x, t, l, h, *g, d_same)
    wide = torch.empty((N, V + 3), dtype=x.dtype, device="cuda")
    d_other = wide[:, 1:V + 1]                         # rows shifted by 2 bytes and 6 per row
    _C.fused_logprob_entropy_v1_backward(x, t, l, h, *g, d_other)
    torch.testing.assert_close(d_other, d_same, rtol=0, atol=0)


# A row whose first logits are all -inf: in the clamped re-stream they sit at the lowest
# finite value as the running maximum of a lane until a finite logit arrives; the
# rescale then must give exactly 0 for their t terms (not NaN from an overflowing
# (lowest - m) * count product).
CLAMPED_PREFIX = [
    (20000, 4096, torch.bfloat16),    # one-warp row groups
    (2000, 2048, torch.float16),      # whole-block groups
    (600, 8192, torch.bfloat16),      # block kernel
    (300, 32001, torch.bfloat16),     # block kernel, peeled rows
    (12000, 50257, torch.bfloat16),   # row groups, peeled rows
    (1024, 152064, torch.bfloat16),   # one block per SM
    (3000, 4096, torch.float32),
]


@pytest.mark.parametrize("rows,vocab,dtype", CLAMPED_PREFIX)
def test_rows_with_a_long_minus_inf_prefix(rows, vocab, dtype):
    x = seeded_logits((rows, vocab), torch.float32, 3.0, seed=rows + 3)
    t = seeded_targets((rows,), vocab, seed=rows + 4)
    for i, keep in enumerate((96, 3, 1000, 1, vocab // 2, 2100)):
        x[i, : vocab - keep] = float("-inf")
        t[i] = vocab - 1
    x = x.to(dtype)
    outs = kernel_opt.fused_logprob_entropy_forward(x.cuda(), t.cuda())
    idx = torch.cat([torch.arange(0, 8), torch.arange(rows - 8, rows)])
    check_forward_outputs(tuple(o[idx.cuda()] for o in outs), x[idx], t[idx],
                          f"-inf prefix {rows}x{vocab} {dtype}")

"""The forward's dynamic tail (launches with at least 4 rows per block): the last quarter
of the rows goes out as whole-row chunks taken from an atomic counter, several rows per
chunk once the workspace's owner slots would run out.  Results must meet the oracle's
tolerances, be bit-identical from run to run (chunk boundaries are fixed; which block
takes a chunk must not matter), leave the counters zeroed for the next call, and agree
between the strided and contiguous layouts."""
import pytest
import torch

import kernel_opt
from _gpu import check_forward_outputs, seeded_logits, seeded_targets

pytestmark = pytest.mark.gpu

# (rows, vocab, dtype): vector path with one- and multi-row tail chunks, fp32, fp16, and
# the scalar path (a vocab whose rows are not 16-byte multiples)
SHAPES = [
    (20000, 256, torch.bfloat16),    # ~64 rows per block: multi-row chunks (owner cap)
    (3000, 4096, torch.float32),
    (2500, 2048, torch.float16),
    (1777, 1003, torch.bfloat16),    # scalar path
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

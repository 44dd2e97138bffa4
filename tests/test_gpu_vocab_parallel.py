"""Vocab-parallel kernels on one GPU: the shard partial kernel over each column block, the
gathered partials merged by the combine kernel, and per-shard backward must reproduce the
unsharded K1 (and the oracle).  The NCCL exchange itself is covered by the gloo CPU test
and by the multi-GPU run of bench.py."""
import numpy as np
import pytest
import torch

import kernel_opt
from _gpu import check_forward_outputs, check_grad, grads_like, seeded_logits, seeded_targets
from kernel_opt import _C, parallel
from oracle import oracle

pytestmark = pytest.mark.gpu


def shard_forward(x, t, bounds):
    n = t.numel()
    parts = []
    for a, b in zip(bounds, bounds[1:]):
        p = torch.empty((n, 4), dtype=torch.float64, device="cuda")
        _C.vocab_shard_partials(x[..., a:b], t, a, p)
        parts.append(p)
    gathered = torch.stack(parts)
    outs = [torch.empty(t.shape, device="cuda") for _ in range(3)]
    _C.vocab_combine(gathered, len(parts), *outs)
    return outs, gathered


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32, torch.float16])
@pytest.mark.parametrize("world", [2, 3, 8])
def test_sharded_forward_and_backward_equal_full(dtype, world):
    N, V = 64, 32000
    x = seeded_logits((N, V), dtype, 3.0, seed=world)
    t = seeded_targets((N,), V, seed=world + 1)
    t[0], t[1], t[2] = -100, V - 1, 0
    xg, tg = x.cuda(), t.cuda()
    bounds = [parallel.vocab_shard(V, world, r).start for r in range(world)] + [V]
    outs, gathered = shard_forward(xg, tg, bounds)
    check_forward_outputs(outs, x, t, f"vp{world}")
    # partials agree with the oracle's restatement of the same shards
    for k, (a, b) in enumerate(zip(bounds, bounds[1:])):
        want = oracle.unpack_partials(oracle.shard_partials(x[:, a:b], t, a))
        got = oracle.unpack_partials(gathered[k].cpu().numpy())
        np.testing.assert_array_equal(got["has"], want["has"])
        np.testing.assert_allclose(got["m"], want["m"], rtol=0, atol=0)
        np.testing.assert_allclose(got["z"], want["z"], rtol=1e-5)
    # per-shard backward == columns of the full backward
    g = [a.cuda() for a in grads_like((N,), seed=3)]
    lp, h, l = outs
    full = torch.empty_like(xg)
    _C.fused_logprob_entropy_v1_backward(xg, tg, l, h, *g, full)
    for a, b in zip(bounds, bounds[1:]):
        d = torch.empty_like(xg[:, a:b])
        _C.vocab_shard_backward(xg[:, a:b], tg, a, l, h, *g, d)
        # unaligned shards take the scalar path, which evaluates the same expression
        torch.testing.assert_close(d, full[:, a:b], rtol=0, atol=0)
    check_grad(full, x, t, *(a.cpu() for a in g), what=f"vp{world} bwd")


def test_vocab_parallel_autograd_single_rank():
    """The autograd wrapper with a one-rank process group (NCCL) equals plain K1."""
    import os
    import torch.distributed as dist

    if not dist.is_initialized():
        os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
        os.environ.setdefault("MASTER_PORT", "29533")
        dist.init_process_group("nccl", rank=0, world_size=1)
    try:
        x = seeded_logits((2, 8, 4096), torch.bfloat16, 2.0, seed=40).cuda()
        t = seeded_targets((2, 8), 4096).cuda()
        a = x.clone().requires_grad_(True)
        b = x.clone().requires_grad_(True)
        o1 = parallel.vocab_parallel_fused_logprob_entropy(a, t, 0)
        o2 = kernel_opt.fused_logprob_entropy(b, t)
        for u, v in zip(o1, o2):
            torch.testing.assert_close(u, v, rtol=0, atol=2e-6)
        g = grads_like((2, 8), seed=41)
        (o1[0] * g[0].cuda() + o1[1] * g[1].cuda()).sum().backward()
        (o2[0] * g[0].cuda() + o2[1] * g[1].cuda()).sum().backward()
        torch.testing.assert_close(a.grad, b.grad, rtol=1e-2, atol=1e-6)
    finally:
        dist.destroy_process_group()

"""Multi-GPU K1 over NCCL (skipped with fewer than 2 GPUs): one child process per GPU.

* vocab-parallel: each rank holds a contiguous column shard of the same logits; forward
  (shard partials -> one all-gather -> merge) and backward must equal single-GPU K1 on
  the full logits;
* row-sharded: each rank runs K1 on its block of rows with no collective; gathering the
  per-row results afterwards must equal K1 over all rows;
* vocab-parallel LM head: each rank holds a row shard of the head's weight; the fused
  tensor-core head (shard partials -> one all-gather -> merge; backward with one
  all-reduce of the hidden state's gradient) must equal the single-GPU fused head.
"""
import os
import socket
import sys

import pytest
import torch
import torch.multiprocessing as mp

from conftest import PKG_ROOT, REPO

pytestmark = pytest.mark.gpu


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _head_problem(N, V, H=256):
    g = torch.Generator().manual_seed(321)
    hid = (torch.randn(N, H, generator=g) * 0.5).to(torch.bfloat16)
    wt = (torch.randn(V, H, generator=g) * (2.5 / H ** 0.5)).to(torch.bfloat16)
    return hid, wt


def _worker(rank, world, port, out_dir):
    for p in (REPO, PKG_ROOT):
        if p not in sys.path:
            sys.path.insert(0, p)
    import datetime

    import torch.distributed as dist

    import kernel_opt
    from kernel_opt import parallel

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    dev = torch.device("cuda", rank)
    torch.cuda.set_device(dev)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev,
                            timeout=datetime.timedelta(seconds=120))
    try:
        g = torch.Generator().manual_seed(123)
        N, V = 96, 50000
        x = (torch.randn(N, V, generator=g) * 3).to(torch.bfloat16)
        t = torch.randint(0, V, (N,), generator=g)
        t[0], t[1] = -100, V - 1
        gl = torch.randn(N, generator=g)
        ge = torch.randn(N, generator=g) * 0.1

        # vocab-parallel
        cols = parallel.vocab_shard(V, world, rank)
        xs = x[:, cols].contiguous().to(dev).requires_grad_(True)
        lp, h, l = parallel.vocab_parallel_fused_logprob_entropy(xs, t.to(dev), cols.start)
        (d,) = torch.autograd.grad((lp, h), xs, (gl.to(dev), ge.to(dev)))
        # row-sharded
        rows = parallel.row_shard(N, world, rank)
        o_rows = kernel_opt.fused_logprob_entropy_forward(x[rows].to(dev), t[rows].to(dev))
        counts = [parallel.row_shard(N, world, k).stop - parallel.row_shard(N, world, k).start
                  for k in range(world)]
        gathered = []
        for o in o_rows:
            parts = [torch.empty(c, device=dev) for c in counts]
            dist.all_gather(parts, o.contiguous())
            gathered.append(torch.cat(parts))
        # vocab-parallel LM head (bf16, tensor cores)
        hid, wt = _head_problem(N, V)
        hx = hid.to(dev).requires_grad_(True)
        wx = wt[cols].contiguous().to(dev).requires_grad_(True)
        hl = parallel.vocab_parallel_fused_linear_logprob_entropy(hx, wx, t.to(dev), cols.start,
                                                                  0.7, chunk_rows=64)
        dh, dw = torch.autograd.grad(hl[:2], (hx, wx), (gl.to(dev), ge.to(dev)))
        # keep_logits: the same results from the kept logits shard
        hk = parallel.vocab_parallel_fused_linear_logprob_entropy(hx, wx, t.to(dev), cols.start,
                                                                  0.7, keep_logits=True)
        dhk, dwk = torch.autograd.grad(hk[:2], (hx, wx), (gl.to(dev), ge.to(dev)))
        assert all(torch.equal(a, b) for a, b in zip(hk, hl))
        torch.testing.assert_close(dhk.float(), dh.float(), rtol=1e-2,
                                   atol=1e-3 * float(dh.float().abs().max()))
        torch.testing.assert_close(dwk.float(), dw.float(), rtol=1e-2,
                                   atol=1e-3 * float(dw.float().abs().max()))
        torch.save({"lp": lp.cpu(), "h": h.cpu(), "l": l.cpu(), "d": d.cpu(),
                    "cols": torch.tensor([cols.start, cols.stop]),
                    "rows": [a.cpu() for a in gathered],
                    "head": [o.detach().cpu() for o in hl], "dh": dh.cpu(), "dw": dw.cpu()},
                   os.path.join(out_dir, f"rank{rank}.pt"))
    finally:
        dist.destroy_process_group()


def test_vocab_parallel_and_row_sharded_match_single_gpu(tmp_path):
    world = min(torch.cuda.device_count(), 4)
    if world < 2:
        pytest.skip("needs at least 2 GPUs")
    mp.start_processes(_worker, args=(world, _free_port(), str(tmp_path)), nprocs=world,
                       join=True, start_method="spawn")
    import kernel_opt

    g = torch.Generator().manual_seed(123)
    N, V = 96, 50000
    x = (torch.randn(N, V, generator=g) * 3).to(torch.bfloat16)
    t = torch.randint(0, V, (N,), generator=g)
    t[0], t[1] = -100, V - 1
    gl = torch.randn(N, generator=g)
    ge = torch.randn(N, generator=g) * 0.1
    xg = x.cuda().requires_grad_(True)
    lp, h, l = kernel_opt.fused_logprob_entropy(xg, t.cuda())
    (d,) = torch.autograd.grad((lp, h), xg, (gl.cuda(), ge.cuda()))
    for r in range(world):
        res = torch.load(tmp_path / f"rank{r}.pt")
        for a, b in zip((res["lp"], res["h"], res["l"]), (lp, h, l)):
            torch.testing.assert_close(a, b.detach().cpu(), rtol=1e-6, atol=4e-6)
        c0, c1 = (int(v) for v in res["cols"])
        torch.testing.assert_close(res["d"].float(), d[:, c0:c1].float().cpu(), rtol=8e-3,
                                   atol=1e-6 * float(d.float().abs().max()))
        for a, b in zip(res["rows"], (lp, h, l)):
            torch.testing.assert_close(a, b.detach().cpu(), rtol=1e-6, atol=4e-6)

    from kernel_opt import lm_head
    hid, wt = _head_problem(N, V)
    hx, wx = hid.cuda().requires_grad_(True), wt.cuda().requires_grad_(True)
    hl = lm_head.fused_linear_logprob_entropy(hx, wx, t.cuda(), 0.7, chunk_rows=64)
    dh, dw = torch.autograd.grad(hl[:2], (hx, wx), (gl.cuda(), ge.cuda()))
    for r in range(world):
        res = torch.load(tmp_path / f"rank{r}.pt")
        for a, b, rtol in zip(res["head"], hl, (0.0, 1e-4, 0.0)):
            torch.testing.assert_close(a, b.detach().cpu(), rtol=rtol, atol=1e-5)
        torch.testing.assert_close(res["dh"].float(), dh.float().cpu(), rtol=1e-2,
                                   atol=1e-3 * float(dh.float().abs().max()))
        c0, c1 = (int(v) for v in res["cols"])
        torch.testing.assert_close(res["dw"].float(), dw[c0:c1].float().cpu(), rtol=1e-2,
                                   atol=1e-3 * float(dw.float().abs().max()))

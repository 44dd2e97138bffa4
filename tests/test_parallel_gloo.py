"""Vocab-parallel exchange on CPU: two gloo ranks, each holding half of the vocabulary,
compute their shard partials with the oracle, exchange them through the product's
collective step (kernel_opt.parallel.exchange_partials), merge, and must reproduce the
unsharded result.  Also: a rank that fails surfaces as an error on the other rank."""
import os
import socket
import sys

import numpy as np
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from conftest import PKG_ROOT, REPO


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _worker(rank, world, port, result_dir, mode):
    for p in (REPO, PKG_ROOT):
        if p not in sys.path:
            sys.path.insert(0, p)
    import datetime

    from kernel_opt import parallel
    from oracle import oracle

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=20))
    try:
        gen = torch.Generator().manual_seed(11)
        N, V = 12, 1000
        x = (torch.randn(N, V, generator=gen) * 3).to(torch.bfloat16)
        t = torch.randint(-2, V, (N,), generator=gen)  # a few out-of-range ids
        t[0], t[1] = 499, 500  # targets on both sides of the shard boundary
        cols = parallel.vocab_shard(V, world, rank)
        if mode == "fail" and rank == 1:
            raise RuntimeError("injected failure before the exchange")
        words = torch.from_numpy(oracle.shard_partials(x[:, cols], t, cols.start))
        gathered = parallel.exchange_partials(words)
        lp, h, l = oracle.combine(gathered.numpy())
        np.save(os.path.join(result_dir, f"r{rank}.npy"), np.stack([lp, h, l]))
        if rank == 0:
            lp0, h0, l0 = oracle.forward(x, t)
            np.save(os.path.join(result_dir, "full.npy"), np.stack([lp0, h0, l0]))
    finally:
        dist.destroy_process_group()


def test_vocab_parallel_exchange_two_ranks(tmp_path):
    port = _free_port()
    mp.start_processes(_worker, args=(2, port, str(tmp_path), "ok"), nprocs=2, join=True,
                       start_method="spawn")
    full = np.load(tmp_path / "full.npy")
    for r in range(2):
        got = np.load(tmp_path / f"r{r}.npy")
        np.testing.assert_allclose(got, full, rtol=1e-12, atol=1e-12)


def test_failed_rank_is_reported(tmp_path):
    port = _free_port()
    try:
        mp.start_processes(_worker, args=(2, port, str(tmp_path), "fail"), nprocs=2,
                           join=True, start_method="spawn")
    except Exception as e:
        # Either rank 1's own exception is reported first, or rank 0's collective fails
        # (peer gone / timeout) instead of hanging.
        msg = str(e)
        assert "injected failure" in msg or "exchange_partials" in msg, msg
    else:
        raise AssertionError("the injected failure was not reported")

"""kernel_opt imports without a GPU (its native extension and C-ABI library load), keeps
the reference's public surface, and reports bad input the way the reference does."""
import os

import numpy as np
import pytest
import torch

import kernel_opt
from kernel_opt import _C, grpo, parallel


def test_public_surface_matches_reference():
    # reference python/kernel_opt/__init__.py:1-15 and csrc/bindings.cpp:17-26
    for name in ("fused_logprob_entropy", "fused_logprob_entropy_forward",
                 "fused_logprob_entropy_naive"):
        assert callable(getattr(kernel_opt, name))
    for name in ("fused_logprob_entropy_naive", "fused_logprob_entropy_v1",
                 "fused_logprob_entropy_v1_backward"):
        assert callable(getattr(_C, name))
    assert _C.abi_version() == 2


def test_trainer_is_lazy():
    with pytest.raises((ImportError, AttributeError)):
        kernel_opt.KernelOptGRPOTrainer  # trl is not installed here
    with pytest.raises(AttributeError):
        kernel_opt.does_not_exist


def test_native_libraries_are_the_in_tree_builds():
    maps = open("/proc/self/maps").read()
    root = os.path.dirname(kernel_opt.__file__)
    assert os.path.join(root, "lib", "libk1_b200.so") in maps
    assert os.path.dirname(_C.__file__) == root


def test_binding_errors_match_reference_messages():
    x = torch.randn(2, 8)
    t = torch.zeros(2, dtype=torch.int64)
    o = torch.empty(2)
    with pytest.raises(RuntimeError, match="logits must be CUDA"):
        _C.fused_logprob_entropy_v1(x, t, o, o, o)
    with pytest.raises(RuntimeError, match="logits dtype must be bf16, fp16, or fp32"):
        _C.fused_logprob_entropy_v1(x.double(), t, o, o, o)
    with pytest.raises(AssertionError):
        kernel_opt.fused_logprob_entropy(x, t)  # python layer asserts CUDA, as the reference


def test_row_and_vocab_shards_partition():
    for n in (0, 1, 7, 16, 1025):
        for w in (1, 2, 3, 8):
            parts = [parallel.row_shard(n, w, r) for r in range(w)]
            assert parts[0].start == 0 and parts[-1].stop == n
            for a, b in zip(parts, parts[1:]):
                assert a.stop == b.start
            sizes = [s.stop - s.start for s in parts]
            assert max(sizes) - min(sizes) <= 1
    with pytest.raises(ValueError):
        parallel.row_shard(10, 2, 2)
    assert parallel.vocab_shard(256000, 8, 7) == slice(224000, 256000)


def test_completion_window_is_a_strided_view():
    base = torch.randn(3, 11, 5)
    w = grpo.completion_window(base, 6)
    assert w.shape == (3, 6, 5)
    assert w.data_ptr() == base[:, 4:10].data_ptr()
    assert w.stride() == (55, 5, 1) and not w.is_contiguous()
    torch.testing.assert_close(w, base[:, :-1][:, -6:])


def test_temperature_scale_is_the_rounded_double_reciprocal():
    # torch multiplies by (float)(1.0 / T); 1.0f / (float)T differs for T = 0.85
    for T in (0.7, 0.85, 0.9, 1.3, 2.0, 1e-3, 1.0):
        assert grpo.temperature_scale(T) == float(np.float32(1.0 / T))
    assert grpo.temperature_scale(0.85) != float(np.float32(1.0) / np.float32(0.85))
    assert grpo.temperature_scale(1.0) == 1.0
    for bad in (0.0, -1.0, float("inf"), float("nan")):
        with pytest.raises(ValueError):
            grpo.temperature_scale(bad)


def test_custom_op_fake_shapes():
    """The registered op's fake implementation (used by torch.compile tracing)."""
    from kernel_opt import ops
    x = torch.empty(2, 3, 40, device="meta", dtype=torch.bfloat16)
    t = torch.empty(2, 3, device="meta", dtype=torch.int64)
    lp, h, l = ops._fwd_op(x, t)
    assert all(o.shape == (2, 3) and o.dtype == torch.float32 for o in (lp, h, l))
    d = ops._bwd_op(x, t, l, h, lp, None, None)
    assert d.shape == x.shape and d.dtype == x.dtype
    assert hasattr(torch.ops.kernel_opt, "fused_logprob_entropy_fwd")


def test_binding_exports_every_function_the_package_calls():
    """Every `_C.<name>` used by the Python layer exists in the built extension (a stale
    build fails here, not on the GPU box)."""
    import re
    pkg = os.path.dirname(kernel_opt.__file__)
    used = set()
    for f in os.listdir(pkg):
        if f.endswith(".py"):
            used |= set(re.findall(r"\b_C\.(\w+)", open(os.path.join(pkg, f)).read()))
    assert used, "no _C calls found"
    missing = sorted(n for n in used if not hasattr(_C, n))
    assert not missing, f"kernel_opt._C lacks {missing}; rebuild the extension"


def test_lm_head_chunk_rows():
    from kernel_opt import lm_head
    q = lm_head.ROW_QUANTUM
    for N, V, es in ((16384, 151936, 2), (1000, 152064, 2), (8192, 128256, 4), (300, 32000, 2),
                     (50000, 256000, 2)):
        c = lm_head.default_chunk_rows(N, V, es)
        assert c % q == 0 and c >= q
        assert c * V * es <= lm_head.CHUNK_BUDGET_BYTES or c == q
        n_chunks = -(-N // c)
        # fewest chunks that respect the budget, and no chunk much smaller than the others
        assert n_chunks == max(1, -(-N // max(q, lm_head.CHUNK_BUDGET_BYTES // (V * es) // q * q)))
        assert N - (n_chunks - 1) * c > 0
    assert lm_head.default_chunk_rows(16384, 151936, 2) == 3328
    assert lm_head.default_chunk_rows(100, 10 ** 9, 4) == q


def test_fused_head_parts_gates_on_plain_linear_heads():
    import types

    from kernel_opt import lm_head

    class M(torch.nn.Module):
        def __init__(self, bias=False, **cfg):
            super().__init__()
            self.dec = torch.nn.Identity()
            self.head = torch.nn.Linear(4, 10, bias=bias)
            self.config = types.SimpleNamespace(**cfg)

        def get_decoder(self):
            return self.dec

        def get_output_embeddings(self):
            return self.head

    m = M()
    dec, w = lm_head.fused_head_parts(m)
    assert dec is m.dec and w is m.head.weight
    assert lm_head.fused_head_parts(M(bias=True)) is None
    assert lm_head.fused_head_parts(M(final_logit_softcapping=30.0)) is None
    assert lm_head.fused_head_parts(M(logit_scale=0.125)) is None
    assert lm_head.fused_head_parts(M(logit_scale=1.0)) is not None
    assert lm_head.fused_head_parts(torch.nn.Linear(2, 2)) is None


def test_host_chunk_schedule_covers_rows_once_and_ramps():
    from kernel_opt.host import chunk_schedule
    for n, r in ((1024, 110), (5, 110), (300, 110), (110, 110), (1000, 7), (16384, 3328), (1, 1)):
        s = chunk_schedule(n, r)
        assert s[0][0] == 0 and s[-1][1] == n
        assert all(b > a for a, b in s) and all(s[i][1] == s[i + 1][0] for i in range(len(s) - 1))
        assert max(b - a for a, b in s) <= r
    s = chunk_schedule(1024, 110)
    sizes = [b - a for a, b in s]
    assert sizes[:3] == [13, 27, 55] and sizes[-3:] == [55, 27, 13]


class _FakeNvml:
    """NVML stand-in: one GPU whose CPU affinity mask is `masks`."""

    def __init__(self, masks, fail=False):
        self.masks, self.fail, self.bus = masks, fail, None

    def nvmlInit(self):
        if self.fail:
            raise RuntimeError("no NVML")

    def nvmlShutdown(self):
        pass

    def nvmlDeviceGetHandleByPciBusId(self, bus):
        self.bus = bus
        return object()

    def nvmlDeviceGetCpuAffinity(self, handle, n_words):
        return self.masks[:n_words]


def test_gpu_local_cpus_and_binding(monkeypatch):
    import types
    from kernel_opt import host
    props = types.SimpleNamespace(pci_domain_id=0, pci_bus_id=0x18, pci_device_id=0)
    monkeypatch.setattr(host.torch.cuda, "get_device_properties", lambda d: props)
    fake = _FakeNvml([0b1011])
    assert host.gpu_local_cpus("cuda:0", fake) == {0, 1, 3}
    assert fake.bus == "00000000:18:00.0"
    assert host.gpu_local_cpus("cuda:0", _FakeNvml([0], fail=True)) is None
    assert host.gpu_local_cpus("cuda:0", _FakeNvml([0])) is None
    calls = []
    monkeypatch.setattr(host.os, "sched_getaffinity", lambda pid: {1, 2, 3})
    monkeypatch.setattr(host.os, "sched_setaffinity", lambda pid, cpus: calls.append(set(cpus)))
    assert host.bind_to_device_cpus("cuda:0", _FakeNvml([0b1011])) == {1, 3}
    assert calls == [{1, 3}]
    assert host.bind_to_device_cpus("cuda:0", _FakeNvml([0b10000])) is None  # none allowed
    assert calls == [{1, 3}]

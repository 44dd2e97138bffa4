"""K1 forward + backward for logits that live in host memory.

`fused_logprob_entropy_fwd_bwd_host` streams the rows through the GPU in chunks: while
chunk i is reduced and differentiated on the device, chunk i+1 is copied in and chunk
i-1's gradient is copied out, on three CUDA streams with events between them.  The
transfer in and the transfer out then overlap, so a step costs about one direction of
the host link instead of both.  Use it when the [N, V] logits (and their gradient) are
kept in host memory, e.g. offloaded activations; with device-resident logits call
`kernel_opt.fused_logprob_entropy` instead.

Chunks ramp up at the start and down at the end (1/8, 1/4, 1/2 of the full chunk, then
full chunks, then the mirror image): the first chunk's copy in and the last chunk's copy
out are the only transfers that cannot overlap the other direction, so they are kept
small.

The upstream gradients are per row and known before the call (as for a policy-gradient
loss whose per-token weights come from advantages and masks), so each chunk's backward
can run right after its forward.  Rows are independent, so chunking changes no result.
"""
from __future__ import annotations

import os

import torch

from kernel_opt import _C


_STREAMS: dict = {}


def _streams(dev: torch.device):
    # three persistent side streams per device (copy in, compute, copy out)
    if dev not in _STREAMS:
        _STREAMS[dev] = tuple(torch.cuda.Stream(dev) for _ in range(3))
    return _STREAMS[dev]


def gpu_local_cpus(device, nvml=None) -> set[int] | None:
    """The host CPUs that NVML reports as closest to `device` (the cores of the NUMA node
    its PCIe link hangs off), or None when NVML is missing or cannot tell.  `nvml` is the
    NVML module to use (default: pynvml)."""
    if nvml is None:
        try:
            import pynvml as nvml
        except ImportError:
            return None
    props = torch.cuda.get_device_properties(torch.device(device))
    bus = f"{props.pci_domain_id:08x}:{props.pci_bus_id:02x}:{props.pci_device_id:02x}.0"
    n_cpu = os.cpu_count() or 1
    try:
        nvml.nvmlInit()
        try:
            h = nvml.nvmlDeviceGetHandleByPciBusId(bus)
            masks = nvml.nvmlDeviceGetCpuAffinity(h, (n_cpu + 63) // 64)
        finally:
            nvml.nvmlShutdown()
    except Exception:
        return None
    cpus = {64 * i + b for i, m in enumerate(masks) for b in range(64) if (int(m) >> b) & 1}
    return cpus or None


def bind_to_device_cpus(device, nvml=None) -> set[int] | None:
    """Restrict this process to the host CPUs closest to `device` (see gpu_local_cpus),
    within its current affinity, so that host memory it allocates from then on -- pinned
    staging buffers in particular -- is placed on that NUMA node and host<->device copies
    do not cross the socket interconnect.  Meant for one process per GPU; call it before
    allocating host buffers.  Returns the CPUs bound to, or None (nothing changed) when
    the GPU's CPUs are unknown or none of them is allowed."""
    cpus = gpu_local_cpus(device, nvml)
    if not cpus:
        return None
    allowed = cpus & os.sched_getaffinity(0)
    if not allowed:
        return None
    os.sched_setaffinity(0, allowed)
    return allowed


def chunk_schedule(n_rows: int, chunk_rows: int, ramp: int = 3) -> list[tuple[int, int]]:
    """Row ranges [a, b) covering [0, n_rows) in order: `ramp` chunks growing by powers of
    two up to chunk_rows, full chunks, then `ramp` chunks shrinking back."""
    R = max(1, chunk_rows)
    ramp_sizes = [max(1, R >> k) for k in range(ramp, 0, -1)]  # R/8, R/4, R/2
    head = list(ramp_sizes)
    tail = list(reversed(ramp_sizes))
    if sum(head) + sum(tail) >= n_rows:  # too few rows to ramp: uniform chunks
        head, tail = [], []
    sizes = list(head)
    middle = n_rows - sum(head) - sum(tail)
    sizes += [R] * (middle // R)
    if middle % R:
        sizes.append(middle % R)
    sizes += tail
    out, a = [], 0
    for s in sizes:
        out.append((a, a + s))
        a += s
    assert a == n_rows
    return out


def _rows2d(t: torch.Tensor, V: int) -> torch.Tensor:
    if not t.is_contiguous():
        raise ValueError("host logits / gradient buffers must be contiguous")
    return t.view(-1, V)


def fused_logprob_entropy_fwd_bwd_host(logits: torch.Tensor, targets: torch.Tensor,
                                       g_logp: torch.Tensor | None = None,
                                       g_ent: torch.Tensor | None = None,
                                       g_lse: torch.Tensor | None = None,
                                       d_logits: torch.Tensor | None = None,
                                       outputs: tuple | None = None,
                                       chunk_rows: int | None = None,
                                       device: torch.device | int | None = None):
    """Forward and backward of K1 over host-resident logits.

    Args:
        logits:  CPU tensor [..., V] (bf16 / fp16 / fp32), contiguous; pinned memory is
                 needed for the copies to overlap.
        targets: [...] int64 (CPU or CUDA).
        g_logp, g_ent, g_lse: upstream gradients [...] (fp32, CPU or CUDA) or None (zero).
        d_logits: tensor like `logits` for the gradient: a CPU tensor (allocated pinned
                 if None; may be `logits` itself, which is then overwritten chunk by
                 chunk), or a CUDA tensor on `device`, into which each chunk's backward
                 writes directly (the gradient then stays on the device, as it does in a
                 training step, and only the per-row outputs travel back).
        outputs: optional (logprob, entropy, lse) CPU fp32 tensors shaped like targets.
        chunk_rows: rows per chunk (default: about 32 MB of logits per chunk).
        device: CUDA device (default: current).

    Returns (logprob, entropy, lse, d_logits); the outputs are on the host.  The call
    returns when all host buffers hold their results.
    """
    dev = torch.device("cuda", torch.cuda.current_device() if device is None else
                       (device.index if isinstance(device, torch.device) else device))
    if logits.is_cuda:
        raise ValueError("logits must be in host memory (use fused_logprob_entropy on device)")
    V = logits.shape[-1]
    x = _rows2d(logits, V)
    N = x.shape[0]
    if targets.numel() != N:
        raise ValueError("targets numel must match leading dims of logits")
    if d_logits is None:
        d_logits = torch.empty_like(logits, pin_memory=True)
    d = _rows2d(d_logits, V)
    grad_on_device = d_logits.is_cuda
    if grad_on_device and d_logits.device != dev:
        raise ValueError("a device d_logits must be on `device`")
    if d_logits.shape != logits.shape or d_logits.dtype != logits.dtype:
        raise ValueError("d_logits must match logits in shape and dtype")
    if outputs is None:
        outputs = tuple(torch.empty(targets.shape, dtype=torch.float32, pin_memory=True)
                        for _ in range(3))
    outs = [o.view(-1) for o in outputs]
    if N == 0:
        return (*outputs, d_logits)

    esize = x.element_size()
    if chunk_rows is None:
        chunk_rows = max(1, (32 << 20) // (V * esize))
    R = min(chunk_rows, N)
    ranges = chunk_schedule(N, R)
    nchunks = len(ranges)

    # small per-row inputs go to the device once
    t_dev = targets.reshape(-1).to(dev, non_blocking=True)
    grads = [None if g is None else g.reshape(-1).to(dev, torch.float32, non_blocking=True)
             for g in (g_logp, g_ent, g_lse)]
    o_dev = [torch.empty(N, dtype=torch.float32, device=dev) for _ in range(3)]

    main = torch.cuda.current_stream(dev)
    s_in, s_run, s_out = _streams(dev)
    nbuf = 3
    bufs = [torch.empty((R, V), dtype=x.dtype, device=dev) for _ in range(min(nbuf, nchunks))]
    ev_in = [torch.cuda.Event() for _ in bufs]
    ev_run = [torch.cuda.Event() for _ in bufs]
    ev_out = [torch.cuda.Event() for _ in bufs]
    start = torch.cuda.Event()
    start.record(main)
    for s in (s_in, s_run, s_out):
        s.wait_event(start)

    for i, (a, b) in enumerate(ranges):
        k = i % len(bufs)
        buf = bufs[k][: b - a]
        with torch.cuda.stream(s_in):
            if i >= len(bufs):
                s_in.wait_event(ev_out[k])  # the buffer's previous gradient has left
            buf.copy_(x[a:b], non_blocking=True)
            ev_in[k].record(s_in)
        with torch.cuda.stream(s_run):
            s_run.wait_event(ev_in[k])
            lp, h, l = (o[a:b] for o in o_dev)
            tt = t_dev[a:b]
            _C.fused_logprob_entropy_v1(buf, tt, lp, h, l)
            gg = [None if g is None else g[a:b] for g in grads]
            if grad_on_device:
                _C.fused_logprob_entropy_v1_backward(buf, tt, l, h, *gg, d[a:b])
            else:
                _C.fused_logprob_entropy_v1_backward(buf, tt, l, h, *gg, buf)  # in place
            ev_run[k].record(s_run)
        with torch.cuda.stream(s_out):
            s_out.wait_event(ev_run[k])
            if not grad_on_device:
                d[a:b].copy_(buf, non_blocking=True)
            ev_out[k].record(s_out)

    with torch.cuda.stream(s_out):
        s_out.wait_stream(s_run)
        for o, od in zip(outs, o_dev):
            o.copy_(od, non_blocking=True)
    main.wait_stream(s_out)
    main.synchronize()  # host buffers hold the results; device buffers are free again
    return (*outputs, d_logits)

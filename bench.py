#!/usr/bin/env python
"""bench.py -- K1 forward + backward throughput on B200, one process per GPU.

Workload (the metric's single-GPU headline): bf16 logits
[B=8, S=128, V=152064] ~ N(0, 3^2), targets sampled per row from softmax(logits),
upstream gradients g_logp = -1/N, g_entropy = -0.01/N.  A step is one forward and one
backward over that batch through the public API (kernel_opt.fused_logprob_entropy +
torch.autograd.grad), inputs resident in HBM.  `value` times that step captured once as a
CUDA graph and replayed (the same two kernel launches per step without the per-step
Python launch overhead); the eager steps are timed too (`eager`).  With --gpus N under
torchrun every rank processes its own batch (row-sharded, weak scaling, no collective in
the data path).

Also on the line:
  fwd / bwd, roofline.per_kernel -- each launch of the step timed alone on the device: a
      CUDA graph of (L2 flush, launch) replayed between CUDA events, minus a flush-only
      graph;
  c3, c4_bf16, c4_fp16, c4_fp32 (N = 1) -- the same per-launch figures for config 3 (the
      strided GRPO window, 16 384 x 151 936: the north-star shape) and config 4 per dtype;
  vocab_parallel -- config 5 [32768, 256000] over the same N ranks, vocabulary sharded,
      one NCCL all-gather of partials per forward (strong scaling), the all-gather timed
      alone, and a 128-row parity check against an fp64 torch recomputation;
  lmhead_vocab_parallel -- the LM head [3584 -> 151936] fused with K1 on 16 384 rows, its
      weight split over the same N ranks (tensor-parallel head, strong scaling): training
      step (logits recomputed, or kept with keep_logits) and no-grad forward;
  e2e -- the step from pinned host buffers through kernel_opt.host (host<->device copies
      inside the timed region);
  cpu_baseline (N = 1) -- the reference's CPU path on the host cores.

Metric: algorithmic bytes per step / time, fwd = N V s + 20 N, bwd = 2 N V s + 28 N
(s = 2 for bf16), reported in GB/s together with rows/s.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                  [--config c2|c3|c4-bf16|c4-fp16|c4-fp32] [--no-cpu-baseline] [--eager]
                  [--no-extra-configs] [--no-vocab-parallel] [--no-lmhead-tp]
                  [--mode rows|vocab|grpo|lmhead]

--impl reference times the reference's CPU path (TRL-1.4 selective_log_softmax +
entropy_from_logits + autograd, restated in oracle/trl_eager.py since TRL is not
installed) on the host cores, on rank 0 only, with every host thread the process may use.
"""
from __future__ import annotations

import argparse
import datetime
import json
import os
import statistics
import sys
import threading
import time

REPO = os.path.dirname(os.path.abspath(__file__))
PKG_ROOT = os.path.join(REPO, "fused-logprob-entropy-cuda-kernel-for-llm-post-training_b200")
for _p in (REPO, PKG_ROOT):
    if _p not in sys.path:
        sys.path.insert(0, _p)

import torch  # noqa: E402

METRIC = "fwd+bwd HBM GB/s (% of B200 peak) and rows/s, V=152k bf16, 1/2/4/8 GPUs"
UNIT = "GB/s"
L2_BYTES = 126 * 1024 * 1024

CONFIGS = {
    "c2": dict(workload="baseline-config-2: single-GPU headline", B=8, S=128, V=152064,
               dtype=torch.bfloat16, scale=3.0, window=False),
    "c3": dict(workload="baseline-config-3: GRPO window logits[:, :-1] of [16,1025,V]", B=16,
               S=1024, V=151936, dtype=torch.bfloat16, scale=2.5, window=True),
    "c3s": dict(workload="config-3 window, 2 sequences (profiling case: 623 MB parent)", B=2,
                S=1024, V=151936, dtype=torch.bfloat16, scale=2.5, window=True),
    "c4-bf16": dict(workload="baseline-config-4: stress, bf16", B=1, S=8192, V=128256,
                    dtype=torch.bfloat16, scale=2.0, window=False, spikes=True),
    "c4-fp16": dict(workload="baseline-config-4: stress, fp16", B=1, S=8192, V=128256,
                    dtype=torch.float16, scale=2.0, window=False, spikes=True),
    "c4-fp32": dict(workload="baseline-config-4: stress, fp32", B=1, S=8192, V=128256,
                    dtype=torch.float32, scale=2.0, window=False, spikes=True),
    "c5": dict(workload="baseline-config-5: vocab-parallel LM head [32768, 256000]", B=1,
               S=32768, V=256000, dtype=torch.bfloat16, scale=3.0, window=False),
}
DTYPE_NAME = {torch.bfloat16: "bf16", torch.float16: "fp16", torch.float32: "fp32"}


def algorithmic_bytes(n_rows: int, vocab: int, esize: int):
    fwd = n_rows * vocab * esize + n_rows * (8 + 3 * 4)
    bwd = 2 * n_rows * vocab * esize + n_rows * (8 + 2 * 4 + 3 * 4)
    return fwd, bwd


def measured_peak_gbs():
    path = os.path.join(REPO, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            return float(json.load(f)["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


def committed_traffic(config_name: str):
    """Per-launch DRAM bytes of the dominant kernel from the committed ncu summary."""
    path = os.path.join(REPO, "profiles", "traffic.json")
    try:
        with open(path) as f:
            return json.load(f).get(config_name)
    except Exception:
        return None


# ---------------------------------------------------------------------------------------
# Workload
# ---------------------------------------------------------------------------------------
def make_workload(cfg: dict, device, seed: int):
    B, S, V, dt = cfg["B"], cfg["S"], cfg["V"], cfg["dtype"]
    gen = torch.Generator(device=device).manual_seed(seed)
    rows_total = B * (S + 1 if cfg["window"] else S)
    parent = torch.empty((rows_total, V), dtype=dt, device=device)
    chunk = 1024
    for a in range(0, rows_total, chunk):
        b = min(rows_total, a + chunk)
        blk = torch.randn((b - a, V), generator=gen, device=device, dtype=torch.float32)
        blk.mul_(cfg["scale"])
        if cfg.get("spikes"):
            spike = torch.rand((b - a, V), generator=gen, device=device) < 0.01
            blk.add_(spike.float() * 15.0)
            hot = torch.rand((b - a,), generator=gen, device=device) < 0.001
            if hot.any():
                col = torch.randint(0, V, (b - a,), generator=gen, device=device)
                blk[hot, col[hot]] += 40.0
        parent[a:b] = blk.to(dt)
        del blk
    if cfg["window"]:
        logits = parent.view(B, S + 1, V)[:, :-1, :]
    else:
        logits = parent.view(B, S, V)
    N = B * S
    targets = torch.empty((B, S), dtype=torch.int64, device=device)
    for bi in range(B):
        for a in range(0, S, chunk):
            b = min(S, a + chunk)
            if cfg.get("spikes"):
                # config 4: half the rows target their argmax, half a uniform column
                am = logits[bi, a:b].argmax(-1)
                un = torch.randint(0, V, (b - a,), generator=gen, device=device)
                pick = torch.rand((b - a,), generator=gen, device=device) < 0.5
                targets[bi, a:b] = torch.where(pick, am, un)
            else:
                probs = torch.softmax(logits[bi, a:b].float(), dim=-1)
                targets[bi, a:b] = torch.multinomial(probs, 1, generator=gen).view(-1)
                del probs
    if cfg["window"]:
        # config 3: completion mask, ones up to a random length per sequence (mean about
        # 0.7 S), zeros after; the loss averages over the unmasked tokens
        lens = torch.randint(int(0.4 * S), S + 1, (B,), generator=gen, device=device)
        mask = (torch.arange(S, device=device)[None, :] < lens[:, None]).float()
        g_lp = -mask / mask.sum()
        g_h = -0.01 * mask / mask.sum()
    else:
        g_lp = torch.full((B, S), -1.0 / N, device=device)
        g_h = torch.full((B, S), -0.01 / N, device=device)
    return logits, targets, g_lp, g_h


# ---------------------------------------------------------------------------------------
# Clock sampling (NVML, background thread, during the timed region)
# ---------------------------------------------------------------------------------------
class ClockSampler:
    REASONS = {
        "gpu_idle": 0x1, "applications_clocks_setting": 0x2, "sw_power_cap": 0x4,
        "hw_slowdown": 0x8, "sync_boost": 0x10, "sw_thermal_slowdown": 0x20,
        "hw_thermal_slowdown": 0x40, "hw_power_brake_slowdown": 0x80,
    }

    def __init__(self, device, period_s: float = 0.002):
        self.samples, self.power, self.reasons, self.ok = [], [], 0, False
        self.period = period_s
        self._stop = threading.Event()
        try:
            import pynvml
            pynvml.nvmlInit()
            self.nv = pynvml
            props = torch.cuda.get_device_properties(device)
            try:
                bus = "%08x:%02x:%02x.0" % (props.pci_domain_id, props.pci_bus_id,
                                            props.pci_device_id)
                self.h = pynvml.nvmlDeviceGetHandleByPciBusId(bus)
            except Exception:
                self.h = pynvml.nvmlDeviceGetHandleByIndex(device.index)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self.h, pynvml.NVML_CLOCK_SM)
            self._reasons_fn = getattr(pynvml, "nvmlDeviceGetCurrentClocksEventReasons", None) \
                or getattr(pynvml, "nvmlDeviceGetCurrentClocksThrottleReasons")
            self.ok = True
        except Exception:
            self.max_mhz = None

    def _run(self):
        nv = self.nv
        while not self._stop.is_set():
            try:
                self.samples.append(nv.nvmlDeviceGetClockInfo(self.h, nv.NVML_CLOCK_SM))
                self.reasons |= self._reasons_fn(self.h)
                self.power.append(nv.nvmlDeviceGetPowerUsage(self.h) / 1000.0)
            except Exception:
                pass
            time.sleep(self.period)

    def __enter__(self):
        if self.ok:
            self.t = threading.Thread(target=self._run, daemon=True)
            self.t.start()
        return self

    def __exit__(self, *a):
        if self.ok:
            self._stop.set()
            self.t.join()

    def summary(self):
        if not self.ok or not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": self.max_mhz, "reasons": ["unavailable"],
                    "samples": 0}
        names = [k for k, bit in self.REASONS.items() if self.reasons & bit]
        out = {"sm_mhz": statistics.median(self.samples), "sm_max_mhz": self.max_mhz,
               "reasons": names, "samples": len(self.samples)}
        if self.power:
            out["power_w"] = round(statistics.median(self.power), 1)
        return out


# ---------------------------------------------------------------------------------------
# CPU baseline: the reference's CPU path restated (oracle/trl_eager.py)
# ---------------------------------------------------------------------------------------
def cpu_trl_step_fn(logits_cpu, targets_cpu, g_lp_cpu, g_h_cpu):
    from oracle import trl_eager

    def step():
        trl_eager.forward_backward(logits_cpu, targets_cpu, g_lp_cpu, g_h_cpu)
    return step


def host_cores():
    return {"os_cpu_count": os.cpu_count(), "affinity": len(os.sched_getaffinity(0)),
            "torch_threads": torch.get_num_threads()}


def time_oracle_fp64(x, t, a, b, budget_s=4.0):
    """The fp64 C oracle (oracle/k1_oracle.c, OpenMP) on a bounded row sample."""
    from oracle import oracle as k1_oracle
    rows = min(t.numel(), 64)
    xs = x.reshape(-1, x.shape[-1])[:rows].contiguous()
    ts, as_, bs = t.reshape(-1)[:rows], a.reshape(-1)[:rows], b.reshape(-1)[:rows]
    t0 = time.perf_counter()
    n = 0
    while True:
        _lp, h0, l0 = k1_oracle.forward(xs, ts)
        k1_oracle.backward(xs, ts, l0, h0, as_.numpy(), bs.numpy(), None)
        n += 1
        if time.perf_counter() - t0 >= budget_s:
            break
    dt = (time.perf_counter() - t0) / n
    return {"rows_per_s": round(rows / dt, 2),
            "sample": f"first {rows} rows x {x.shape[-1]}, fwd+bwd, {n} repetitions"}


def time_cpu_baseline(logits, targets, g_lp, g_h, esize, budget_s=12.0, max_rows=1024):
    """TRL eager path restated, on the host cores; configs above max_rows rows are
    subsampled to their first 256 rows (full V) and labelled so."""
    N_all = targets.numel()
    V = logits.shape[-1]
    sub = N_all > max_rows
    rows = min(256, N_all) if sub else N_all

    def first_rows(v):
        # the first `rows` rows in order, sequence by sequence (no copy of the whole
        # strided window)
        parts, need = [], rows
        for bi in range(v.shape[0]):
            if need == 0:
                break
            take = v[bi, :need]
            parts.append(take.detach().cpu())
            need -= take.shape[0]
        return torch.cat(parts).unsqueeze(0)

    x, t, a, b = (first_rows(v) for v in (logits, targets, g_lp, g_h))
    step = cpu_trl_step_fn(x, t, a, b)
    step()
    t0 = time.perf_counter()
    n = 0
    while True:
        step()
        n += 1
        if time.perf_counter() - t0 >= budget_s:
            break
    dt = (time.perf_counter() - t0) / n
    N = t.numel()
    fwd, bwd = algorithmic_bytes(N, V, esize)
    what = (f"subsampled: first {N} of {N_all} rows x {V}" if sub
            else f"the full batch ({N} rows x {V})")
    return {"value": round((fwd + bwd) / dt / 1e9, 4), "unit": UNIT,
            "rows_per_s": round(N / dt, 2), "cores": torch.get_num_threads(), "kind": "port",
            "sample": f"{what}, {n} fwd+bwd steps in {n * dt:.1f} s, TRL-1.4 eager path "
                      f"restated (oracle/trl_eager.py)",
            "host_cores": host_cores(),
            "oracle_fp64": time_oracle_fp64(x, t, a, b)}


# ---------------------------------------------------------------------------------------
# Arms
# ---------------------------------------------------------------------------------------
def dist_env():
    return (int(os.environ.get("RANK", "0")), int(os.environ.get("LOCAL_RANK", "0")),
            int(os.environ.get("WORLD_SIZE", "1")))


def reference_arm(args, cfg, rank, world):
    if rank != 0:
        return
    # torchrun sets OMP_NUM_THREADS=1 for every rank; the reference's CPU path gets all
    # the host threads this process may use, at every N
    torch.set_num_threads(len(os.sched_getaffinity(0)))
    from oracle import trl_eager
    V, dt = cfg["V"], cfg["dtype"]
    esize = torch.tensor([], dtype=dt).element_size()
    B, S = cfg["B"], cfg["S"]
    gen = torch.Generator().manual_seed(1234)
    full = (torch.randn(B, S, V, generator=gen) * cfg["scale"]).to(dt)
    targets = torch.randint(0, V, (B, S), generator=gen)
    N = B * S
    g_lp, g_h = torch.full((B, S), -1.0 / N), torch.full((B, S), -0.01 / N)
    probe = time.perf_counter()
    trl_eager.forward_backward(full, targets, g_lp, g_h)
    probe = time.perf_counter() - probe
    # Each step is the full batch unless the whole run would exceed ~3 minutes; then a
    # leading block of batch elements is used.
    budget = 180.0 / max(1, args.steps + args.warmup)
    b_use = B if probe <= budget else max(1, int(B * budget / probe))
    x, t = full[:b_use].contiguous(), targets[:b_use].contiguous()
    gl, gh = g_lp[:b_use].contiguous(), g_h[:b_use].contiguous()
    for _ in range(args.warmup):
        trl_eager.forward_backward(x, t, gl, gh)
    t0 = time.perf_counter()
    for _ in range(args.steps):
        trl_eager.forward_backward(x, t, gl, gh)
    el = time.perf_counter() - t0
    n_rows = b_use * S
    fwd, bwd = algorithmic_bytes(n_rows, V, esize)
    value = (fwd + bwd) * args.steps / el / 1e9
    ref_gpu = time_reference_k1_gpu(cfg)
    out = {
        "metric": METRIC, "value": round(value, 4), "unit": UNIT, "impl": "reference",
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(el / args.steps * 1e3, 3), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": DTYPE_NAME[dt], "data": "synthetic",
        "rows_per_s": round(n_rows * args.steps / el, 2),
        "config": arm_config(cfg, world, esize),
        "cpu_baseline": {"value": round(value, 4), "unit": UNIT, "cores": torch.get_num_threads(),
                         "kind": "port",
                         "sample": f"{b_use}/{B} batch elements ({n_rows} rows x {V}) per step "
                                   "on rank 0's host threads; TRL-1.4 selective_log_softmax + "
                                   "entropy_from_logits + autograd, restated in "
                                   "oracle/trl_eager.py",
                         "host_cores": host_cores()},
        "e2e": {"value": round(value, 4), "unit": UNIT, "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    if ref_gpu is not None:
        out["reference_k1_sm100a"] = ref_gpu
    print(json.dumps(out), flush=True)


def reference_grpo_arm(args, cfg, rank, world):
    """The GRPO loss block of grpo_arm run the reference trainer's way with the reference's
    own K1 kernels (rebuilt for sm_100a by oracle/build_ref.py): slice the completion window,
    divide it in place by the temperature, one K1 call per sequence (trainer.py:96-127,
    through the reference's autograd wrapper, ops.py:49-89), then autograd back to the
    logits.  Same workload, metric and algorithmic bytes as `--mode grpo`."""
    if rank != 0:
        return
    from oracle import reference_k1
    fn = reference_k1.autograd_function() if torch.cuda.is_available() else None
    if fn is None:
        print(json.dumps({"impl": "reference", "unavailable":
                          "reference K1 build (oracle/_ref) or GPU absent"}), flush=True)
        return
    if not cfg["window"]:
        cfg = CONFIGS["c3"]
    device = torch.device("cuda", 0)
    torch.cuda.set_device(device)
    B, S, V, dt = cfg["B"], cfg["S"], cfg["V"], cfg["dtype"]
    T = 0.7
    esize = torch.tensor([], dtype=dt).element_size()
    window, targets, g_lp, g_h = make_workload(cfg, device, seed=4321)
    parent = torch.as_strided(window, (B, S + 1, V), ((S + 1) * V, V, 1), 0)
    N = B * S
    fwd_bytes = N * V * esize + N * 20
    bwd_bytes = N * V * esize + B * (S + 1) * V * esize + N * 16
    stream = torch.cuda.current_stream(device)

    def step(timed_events=None):
        x = parent.detach().requires_grad_(True)
        logits = x.clone()  # the model output the trainer receives
        if timed_events:
            timed_events[0].record(stream)
        w = logits[:, :-1, :][:, -S:, :]
        w.div_(T)
        lps, ents = [], []
        for b in range(B):
            lp, h, _ = fn.apply(w[b].contiguous(), targets[b].contiguous())
            lps.append(lp.unsqueeze(0))
            ents.append(h.unsqueeze(0))
        lp, h = torch.cat(lps), torch.cat(ents)
        if timed_events:
            timed_events[1].record(stream)
        (d,) = torch.autograd.grad((lp, h), x, (g_lp, g_h))
        if timed_events:
            timed_events[2].record(stream)
        return d

    for _ in range(max(3, args.warmup)):
        step()
    torch.cuda.synchronize(device)
    K = args.steps
    ev = [[torch.cuda.Event(enable_timing=True) for _ in range(3)] for _ in range(K)]
    for i in range(K):
        step(ev[i])
    torch.cuda.synchronize(device)
    f_ms = statistics.mean(e[0].elapsed_time(e[1]) for e in ev)
    b_ms = statistics.mean(e[1].elapsed_time(e[2]) for e in ev)
    total = f_ms + b_ms
    value = (fwd_bytes + bwd_bytes) / (total / 1e3) / 1e9
    out = {
        "metric": METRIC, "value": round(value, 2), "unit": UNIT, "impl": "reference",
        "n_gpus": world, "steps": K, "warmup": max(3, args.warmup),
        "ms_per_step": round(total, 4), "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": DTYPE_NAME[dt], "data": "synthetic",
        "rows_per_s": round(N / (total / 1e3), 1),
        "config": {"workload": "GRPO loss block on " + cfg["workload"], "global_batch": B,
                   "seq_len": S, "vocab": V, "temperature": T,
                   "parallelism": "one GPU, the reference trainer's per-sequence loop"},
        "reference_trainer_sm100a": {"fwd_ms": round(f_ms, 4), "bwd_ms": round(b_ms, 4),
                                     "kernel_launches_per_step": 2 * B,
                                     "note": "reference kernels rebuilt for sm_100a "
                                             "(oracle/build_ref.py) in the reference "
                                             "trainer's sequence; CUDA events"},
        "e2e": {"value": round(value, 2), "unit": UNIT, "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    print(json.dumps(out), flush=True)


def time_reference_k1_gpu(cfg, iters=20):
    """The reference's own CUDA K1 (csrc/fused_logprob.cu, rebuilt for sm_100a by
    oracle/build_ref.py) on the same workload shape, timed with CUDA events (median).
    Informational: it is the reference's GPU kernel, not its CPU path."""
    try:
        if not torch.cuda.is_available():
            return None
        from oracle import reference_k1
        if reference_k1.load() is None:
            return {"unavailable": "oracle/_ref build absent"}
    except Exception as e:  # pragma: no cover
        return {"unavailable": f"{type(e).__name__}: {e}"[:200]}
    dev = torch.device("cuda", 0)
    B, S, V, dt = cfg["B"], cfg["S"], cfg["V"], cfg["dtype"]
    N = B * S
    gen = torch.Generator(device=dev).manual_seed(4321)
    x = (torch.randn((N, V), generator=gen, device=dev) * cfg["scale"]).to(dt)
    t = torch.randint(0, V, (N,), generator=gen, device=dev)
    gl = torch.full((N,), -1.0 / N, device=dev)
    gh = torch.full((N,), -0.01 / N, device=dev)
    gz = torch.zeros(N, device=dev)
    lp, h, l = reference_k1.forward(x, t)
    d = reference_k1.backward(x, t, l, h, gl, gh, gz)
    tf, tb = [], []
    for _ in range(iters):
        a, b, c = (torch.cuda.Event(enable_timing=True) for _ in range(3))
        a.record()
        lp, h, l = reference_k1.forward(x, t)
        b.record()
        d = reference_k1.backward(x, t, l, h, gl, gh, gz)
        c.record()
        torch.cuda.synchronize()
        tf.append(a.elapsed_time(b))
        tb.append(b.elapsed_time(c))
    esize = torch.tensor([], dtype=dt).element_size()
    fwd, bwd = algorithmic_bytes(N, V, esize)
    mf, mb = statistics.median(tf), statistics.median(tb)
    del x, d
    return {"fwd_ms": round(mf, 4), "bwd_ms": round(mb, 4),
            "fwd_gbs": round(fwd / (mf / 1e3) / 1e9, 1), "bwd_gbs": round(bwd / (mb / 1e3) / 1e9, 1),
            "fwd_bwd_gbs": round((fwd + bwd) / ((mf + mb) / 1e3) / 1e9, 1),
            "note": "reference csrc/fused_logprob.cu v1 kernels rebuilt for sm_100a "
                    "(oracle/build_ref.py), same shape, CUDA events, median of %d" % iters}


def arm_config(cfg, world, esize):
    """The `config` object both arms print (identical keys and values for one workload and
    GPU count, so the two lines can be matched)."""
    n_rows = cfg["B"] * cfg["S"]
    return {"workload": cfg["workload"], "global_batch": cfg["B"] * world, "seq_len": cfg["S"],
            "vocab": cfg["V"], "rows_per_gpu": n_rows,
            "parallelism": f"row-sharded x{world} (no collective)",
            "l2": (f"inputs larger than L2: {n_rows * cfg['V'] * esize / 2**20:.0f} MiB of "
                   f"logits read and written per step vs {L2_BYTES // 2**20} MiB L2")}


# ---------------------------------------------------------------------------------------
# Device-true kernel timing: one launch per CUDA graph, L2 flushed before it
# ---------------------------------------------------------------------------------------
class GraphTimer:
    """Times single launches on the device.  A launch is captured in a CUDA graph behind a
    write of a buffer twice the size of L2 (so it starts cold, as it would after any other
    large kernel), the graph is replayed K times between two CUDA events on the launching
    stream, and the same measurement of a graph holding the flush alone is subtracted."""

    def __init__(self, device, stream):
        self.device, self.stream = device, stream
        self.flush = torch.empty(2 * L2_BYTES, dtype=torch.uint8, device=device)
        self.graphs = []
        self.g_flush = self.capture(lambda: None)

    def capture(self, fn):
        side = torch.cuda.Stream(self.device)
        side.wait_stream(self.stream)
        with torch.cuda.stream(side):
            for _ in range(3):
                self.flush.zero_()
                fn()
        self.stream.wait_stream(side)
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=side):
            self.flush.zero_()
            fn()
        torch.cuda.synchronize(self.device)
        self.graphs.append(g)
        return g

    def replay_ms(self, g, K):
        for _ in range(3):
            g.replay()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record(self.stream)
        for _ in range(K):
            g.replay()
        b.record(self.stream)
        b.synchronize()
        return a.elapsed_time(b) / K

    def kernel_ms(self, fn, K, reps=3):
        """Median over `reps` of (flush + launch) - (flush), per launch, in ms."""
        g = self.capture(fn)
        vals = sorted(self.replay_ms(g, K) - self.replay_ms(self.g_flush, K) for _ in range(reps))
        return vals[len(vals) // 2]

    def close(self):
        self.graphs.clear()
        del self.flush


def kernel_legs(timer, logits, targets, g_lp, g_h, K, peak):
    """The workload's forward and backward launches (the ones the autograd step makes),
    each timed alone by `timer`, with bytes, GB/s and fraction of the measured peak."""
    from kernel_opt import _C
    N, V = targets.numel(), logits.shape[-1]
    esize = logits.element_size()
    fwd_bytes, bwd_bytes = algorithmic_bytes(N, V, esize)
    tg = targets.contiguous()
    gl, gh = g_lp.contiguous(), g_h.contiguous()
    lp, h, l = (torch.empty(targets.shape, device=logits.device) for _ in range(3))
    d = torch.empty(logits.shape, dtype=logits.dtype, device=logits.device)

    def fwd():
        _C.fused_logprob_entropy_v1(logits, tg, lp, h, l)

    def bwd():
        _C.fused_logprob_entropy_v1_backward(logits, tg, l, h, gl, gh, None, d)

    fwd()
    f_ms = timer.kernel_ms(fwd, K)
    b_ms = timer.kernel_ms(bwd, K)

    def entry(ms, nbytes, what):
        gbs = nbytes / (ms / 1e3) / 1e9
        return {"kernel": what, "ms": round(ms, 5), "algorithmic_bytes": nbytes,
                "gbs": round(gbs, 1), "frac": round(gbs / peak, 4),
                "rows_per_s": round(N / (ms / 1e3), 1)}

    return {"fwd": entry(f_ms, fwd_bytes, "forward launch (kernel chosen by shape)"),
            "bwd": entry(b_ms, bwd_bytes, "backward launch (k1_bwd_ring_kernel on the vector path)")}


def extra_config_legs(device, stream, timer, peak, K, names=("c3", "c4-bf16", "c4-fp16", "c4-fp32")):
    """Forward / backward launches of the other BASELINE shapes on this GPU (N = 1 only):
    config 3 (the GRPO window logits[:, :-1] of [16, 1025, 151936], the north-star
    16 384 x 151 936 shape) and config 4 in each dtype."""
    out = {}
    for name in names:
        cfg = CONFIGS[name]
        logits, targets, g_lp, g_h = make_workload(cfg, device, seed=777)
        legs = kernel_legs(timer, logits, targets, g_lp, g_h, K, peak)
        N = targets.numel()
        esize = logits.element_size()
        fb, bb = algorithmic_bytes(N, cfg["V"], esize)
        step_ms = legs["fwd"]["ms"] + legs["bwd"]["ms"]
        out[name.replace("-", "_")] = {
            "workload": cfg["workload"], "rows": N, "vocab": cfg["V"], "dtype": DTYPE_NAME[cfg["dtype"]],
            "strided_window": bool(cfg["window"]), **legs,
            "fwd_plus_bwd": {"ms": round(step_ms, 5),
                             "gbs": round((fb + bb) / (step_ms / 1e3) / 1e9, 1),
                             "frac": round((fb + bb) / (step_ms / 1e3) / 1e9 / peak, 4)}}
        del logits, targets, g_lp, g_h
        torch.cuda.empty_cache()
    return out


def lmhead_tp_leg(args, rank, world, device, stream, barrier, max_over_ranks):
    """The LM head fused with K1, split over the vocabulary across the ranks (tensor-parallel
    head), strong scaling: hidden [16384, 3584] bf16 and the targets on every rank, rank k
    holding rows vocab_shard(151936, world, k) of one [151936, 3584] weight, T = 0.7.
    Forward = the tensor-core kernel's shard partials + ONE NCCL all-gather + combine;
    backward = the shard's gradient recomputed on the tensor cores + library GEMMs + ONE
    NCCL all-reduce of dL/dhidden.  At one GPU: the same call over the whole weight."""
    from kernel_opt import parallel
    N, H, V, T = 16384, 3584, 151936, 0.7
    cols = parallel.vocab_shard(V, world, rank)
    gen = torch.Generator(device=device).manual_seed(7)
    h = (torch.randn(N, H, generator=gen, device=device) * 0.5).to(torch.bfloat16)
    t = torch.randint(0, V, (N,), generator=gen, device=device)
    w = (torch.randn(V, H, generator=gen, device=device) * (2.5 / H ** 0.5)).to(torch.bfloat16)
    w = w[cols].contiguous()
    torch.cuda.empty_cache()
    g_lp = torch.full((N,), -1.0 / N, device=device)
    g_h = torch.full((N,), -0.01 / N, device=device)

    def step(grad, keep=False):
        hx = h.detach().requires_grad_(grad)
        wx = w.detach().requires_grad_(grad)
        with torch.set_grad_enabled(grad):
            lp, ent, _ = parallel.vocab_parallel_fused_linear_logprob_entropy(
                hx, wx, t, cols.start, T, keep_logits=keep)
            if grad:
                torch.autograd.grad((lp, ent), (hx, wx), (g_lp, g_h))

    K = max(1, min(args.steps, 5))
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    got = {}
    for name, grad, keep in (("train_ms", True, False), ("train_keep_ms", True, True),
                             ("nograd_ms", False, False)):
        for _ in range(2):
            step(grad, keep)
        barrier()
        a.record(stream)
        for _ in range(K):
            step(grad, keep)
        b.record(stream)
        barrier()
        got[name] = max_over_ranks(a.elapsed_time(b)) / K
    del h, w
    torch.cuda.empty_cache()
    useful = 3 * 2.0 * N * H * V  # forward logits, dL/dhidden, dL/dweight
    return {"workload": f"LM head [{H} -> {V}] fused with K1 on {N} rows, vocabulary split "
                        f"over the GPUs ({cols.stop - cols.start} rows of W on rank {rank})",
            "n_gpus": world, "scaling": "strong", "steps": K, "dtype": "bf16", "temperature": T,
            "train_ms": round(got["train_ms"], 3), "nograd_ms": round(got["nograd_ms"], 3),
            "train_keep_ms": round(got["train_keep_ms"], 3),
            "train_useful_tflops_total": round(useful / (got["train_ms"] / 1e3) / 1e12, 1),
            "train_keep_useful_tflops_total": round(useful / (got["train_keep_ms"] / 1e3) / 1e12, 1),
            "collectives": ("forward: one NCCL all-gather of [N, 4] float64 partials; backward: "
                            "one NCCL all-reduce of dL/dhidden [N, H] fp32" if world > 1
                            else "none (one process holds the whole weight)"),
            "note": "max over ranks of CUDA-event time; parity: tests/test_gpu_multi.py, "
                    "tests/test_gpu_lm_head.py"}


def vocab_parallel_leg(args, rank, world, device, stream, barrier, max_over_ranks, peak):
    """Config 5, vocab-parallel (tensor-parallel LM head layout), strong scaling: rank k holds
    columns vocab_shard(256000, world, k) of all 32 768 rows; forward = shard partials, ONE
    NCCL all-gather of [N, 4] float64 partials, merge; backward local.  Also times the
    all-gather alone and checks 128 rows against an fp64 torch recomputation."""
    import torch.distributed as dist

    from kernel_opt import parallel
    cfg = CONFIGS["c5"]
    N, V, dt = cfg["B"] * cfg["S"], cfg["V"], cfg["dtype"]
    esize = torch.tensor([], dtype=dt).element_size()
    cols = parallel.vocab_shard(V, world, rank)
    Vr = cols.stop - cols.start
    gen = torch.Generator(device=device).manual_seed(7000 + rank)
    xs = torch.empty((N, Vr), dtype=dt, device=device)
    for a in range(0, N, 1024):
        b = min(N, a + 1024)
        xs[a:b] = (torch.randn((b - a, Vr), generator=gen, device=device) * cfg["scale"]).to(dt)
    targets = torch.randint(0, V, (N,), generator=torch.Generator(device=device).manual_seed(99),
                            device=device)
    g_lp = torch.full((N,), -1.0 / N, device=device)
    g_h = torch.full((N,), -0.01 / N, device=device)

    def step():
        x = xs.detach().requires_grad_(True)
        lp, h, l = parallel.vocab_parallel_fused_logprob_entropy(x, targets, cols.start)
        (d,) = torch.autograd.grad((lp, h), x, (g_lp, g_h))
        return lp, h, l, d

    for _ in range(3):
        step()
    barrier()
    K = max(1, min(args.steps, 50))
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier()
    a.record(stream)
    for _ in range(K):
        step()
    b.record(stream)
    barrier()
    ms = max_over_ranks(a.elapsed_time(b)) / K

    # the collective alone: the same all-gather of [N, 4] float64 partials, K times
    ag_ms = 0.0
    if world > 1:
        part = torch.zeros((N, parallel.PARTIAL_WORDS), dtype=torch.float64, device=device)
        for _ in range(3):
            parallel.exchange_partials(part)
        barrier()
        a.record(stream)
        for _ in range(K):
            parallel.exchange_partials(part)
        b.record(stream)
        barrier()
        ag_ms = max_over_ranks(a.elapsed_time(b)) / K

    # parity: 128 rows, the full vocabulary gathered from every shard, against fp64 torch
    lp, h, l, d = step()
    idx = torch.linspace(0, N - 1, 128, device=device).round().long()
    sub = xs[idx].contiguous()
    if world > 1:
        parts = [torch.empty_like(sub) for _ in range(world)]
        dist.all_gather(parts, sub)
        full = torch.cat(parts, dim=1)
    else:
        full = sub
    barrier()
    parity = None
    if rank == 0:
        x64 = full.double()
        t = targets[idx]
        logp_all = torch.log_softmax(x64, dim=-1)
        p = logp_all.exp()
        ent0 = -(p * logp_all).sum(-1)
        lse0 = torch.logsumexp(x64, dim=-1)
        lp0 = logp_all.gather(1, t[:, None]).squeeze(1)
        gl, gh = g_lp[idx].double()[:, None], g_h[idx].double()[:, None]
        d0 = -gl * p - gh * p * (logp_all + ent0[:, None])
        d0.scatter_add_(1, t[:, None], gl)
        d0 = d0[:, cols.start:cols.stop]
        dd = d[idx].double()
        floor = 1e-7 * float(d0.abs().max())
        grad_rel = float(((dd - d0).abs() / (d0.abs() + floor)).max())
        parity = {
            "rows_checked": 128, "reference": "fp64 torch log_softmax / logsumexp on the "
                                              "gathered full-vocabulary rows",
            "lse_max_abs_err": float((l[idx].double() - lse0).abs().max()),
            "logp_max_abs_err": float((lp[idx].double() - lp0).abs().max()),
            "entropy_max_rel_err": float(((h[idx].double() - ent0).abs() / ent0.abs()).max()),
            "grad_max_rel_err_rank0_shard": grad_rel,
        }
        parity["within_tolerance"] = bool(parity["lse_max_abs_err"] <= 1e-5
                                          and parity["logp_max_abs_err"] <= 1e-5
                                          and parity["entropy_max_rel_err"] <= 1e-4
                                          and grad_rel <= 1e-2)
    del xs, d
    torch.cuda.empty_cache()
    fwd, bwd = algorithmic_bytes(N, V, esize)
    gbs = (fwd + bwd) / (ms / 1e3) / 1e9
    return {"workload": cfg["workload"], "rows": N, "vocab": V, "vocab_per_gpu": Vr,
            "n_gpus": world, "scaling": "strong", "steps": K,
            "ms_per_step": round(ms, 4), "gbs_total": round(gbs, 1),
            "gbs_per_gpu": round(gbs / world, 1), "pct_of_peak_per_gpu": round(100 * gbs / world / peak, 2),
            "rows_per_s": round(N / (ms / 1e3), 1),
            "collective": ("NCCL all_gather_into_tensor of [N, 4] float64 partials "
                           f"({N * 32} bytes per rank), one per forward" if world > 1
                           else "none (one process holds the whole vocabulary)"),
            "allgather_ms": round(ag_ms, 4),
            "allgather_share_of_step": round(ag_ms / ms, 4) if ms > 0 else None,
            "parity": parity,
            "step": "eager: vocab_parallel_fused_logprob_entropy + torch.autograd.grad"}


def ours_arm(args, cfg, rank, local_rank, world):
    import torch.distributed as dist

    import kernel_opt

    device = torch.device("cuda", local_rank)
    torch.cuda.set_device(device)
    bound = None
    if world > 1:
        # one process per GPU: run on the host cores next to this GPU, so the pinned
        # buffers of the e2e leg sit on its NUMA node (no cross-socket copies)
        from kernel_opt import host as k1_host
        bound = k1_host.bind_to_device_cpus(device)
        dist.init_process_group("nccl", rank=rank, world_size=world, device_id=device,
                                timeout=datetime.timedelta(seconds=300))
    V, dt = cfg["V"], cfg["dtype"]
    esize = torch.tensor([], dtype=dt).element_size()
    logits, targets, g_lp, g_h = make_workload(cfg, device, seed=1234 + rank)
    N = targets.numel()
    fwd_bytes, bwd_bytes = algorithmic_bytes(N, V, esize)
    step_bytes = fwd_bytes + bwd_bytes
    stream = torch.cuda.current_stream(device)
    peak, peak_kind = measured_peak_gbs()

    def step():
        x = logits.detach().requires_grad_(True)
        lp, h, _l = kernel_opt.fused_logprob_entropy(x, targets)
        (d,) = torch.autograd.grad((lp, h), x, (g_lp, g_h))
        return d

    def barrier():
        if world > 1:
            dist.barrier(device_ids=[local_rank])
        torch.cuda.synchronize(device)

    def max_over_ranks(ms):
        t = torch.tensor([ms], device=device, dtype=torch.float64)
        if world > 1:
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    for _ in range(max(3, args.warmup)):
        step()
    barrier()

    # ---- device-resident timing (value) --------------------------------------------
    # Eager steps (one Python call per op), then the same step captured once as a CUDA
    # graph and replayed K times: identical launches and work, without the per-step host
    # launch overhead, which otherwise dominates once several processes share one host.
    K = args.steps
    start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(device) as clocks:
        barrier()
        start.record(stream)
        for i in range(K):
            x = logits.detach().requires_grad_(True)
            lp, h, _l = kernel_opt.fused_logprob_entropy(x, targets)
            (d,) = torch.autograd.grad((lp, h), x, (g_lp, g_h))
            del d, lp, h, _l, x
        stop.record(stream)
        barrier()
        eager_ms = max_over_ranks(start.elapsed_time(stop))
        graph, graph_ms = None, None
        if not args.eager:
            # capture after the eager steps: capturing empties torch's allocator cache
            side = torch.cuda.Stream(device)
            side.wait_stream(stream)
            with torch.cuda.stream(side):
                for _ in range(3):
                    step()
            stream.wait_stream(side)
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph, stream=side):
                step()
            for _ in range(max(3, args.warmup)):
                graph.replay()
            barrier()
            start.record(stream)
            for _ in range(K):
                graph.replay()
            stop.record(stream)
            barrier()
            graph_ms = max_over_ranks(start.elapsed_time(stop))
    max_ms = graph_ms if graph_ms is not None else eager_ms
    del graph

    # ---- each kernel alone, device-true (graph replays, L2 flushed before each) --------
    timer = GraphTimer(device, stream)
    legs = kernel_legs(timer, logits, targets, g_lp, g_h, max(10, min(K, 50)), peak)
    extra = None
    if world == 1 and not args.no_extra_configs:
        extra = extra_config_legs(device, stream, timer, peak, max(5, min(K, 20)))
    timer.close()
    del timer
    torch.cuda.empty_cache()

    # ---- end to end through the public API with host buffers (e2e) ----------------
    pin = dict(pin_memory=True)
    logits_h = torch.empty(logits.shape, dtype=dt, **pin)
    logits_h.copy_(logits)
    targets_h = targets.cpu().pin_memory()
    glp_h, gh_h = g_lp.cpu().pin_memory(), g_h.cpu().pin_memory()
    d_h = torch.empty(logits.shape, dtype=dt, **pin)
    d_dev = torch.empty(logits.shape, dtype=dt, device=device)
    outs_h = [torch.empty(targets.shape, dtype=torch.float32, **pin) for _ in range(3)]
    h2d = logits_h.numel() * esize + targets_h.numel() * 8 + 2 * glp_h.numel() * 4
    d2h_outputs = 3 * outs_h[0].numel() * 4
    d2h_with_grad = d_h.numel() * esize + d2h_outputs

    from kernel_opt import host as k1_host

    def e2e_step(d_logits):
        # public host-buffer API: chunks of rows copied in and reduced + differentiated on
        # overlapping streams; the per-row outputs (and, for a host d_logits, the gradient)
        # are copied out; returns once the host buffers are filled
        k1_host.fused_logprob_entropy_fwd_bwd_host(logits_h, targets_h, glp_h, gh_h, None,
                                                   d_logits=d_logits, outputs=outs_h,
                                                   device=device)

    K2 = max(1, min(K, 20))

    def time_e2e(d_logits):
        for _ in range(2):
            e2e_step(d_logits)
        barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(K2):
            e2e_step(d_logits)
        e1.record(stream)
        barrier()
        return max_over_ranks(e0.elapsed_time(e1))

    # the step's result (per-row log-prob / entropy / lse) comes back to the host; the
    # logits gradient stays in HBM, where a training step's next backward op reads it
    e2e_ms = time_e2e(d_dev)
    # offload variant: the gradient also goes back to host memory
    e2e_host_grad_ms = time_e2e(d_h)
    del logits_h, d_h, d_dev

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        cpu = time_cpu_baseline(logits, targets, g_lp, g_h, esize)

    # ---- config 5, vocab-parallel over the same ranks (one NCCL all-gather) -----------
    vocab = None
    if not args.no_vocab_parallel:
        del logits
        torch.cuda.empty_cache()
        vocab = vocab_parallel_leg(args, rank, world, device, stream, barrier, max_over_ranks,
                                   peak)

    # ---- the tensor-parallel LM head fused with K1 over the same ranks -----------------
    lmh_tp = None
    if not args.no_lmhead_tp:
        lmh_tp = lmhead_tp_leg(args, rank, world, device, stream, barrier, max_over_ranks)

    if world > 1:
        dist.barrier(device_ids=[local_rank])
        dist.destroy_process_group()
    if rank != 0:
        return

    value = step_bytes * K * world / (max_ms / 1e3) / 1e9
    fwd_ms, bwd_ms = legs["fwd"]["ms"], legs["bwd"]["ms"]
    cfg_name = args.config
    out = {
        "metric": METRIC, "value": round(value, 2), "unit": UNIT, "n_gpus": world, "steps": K,
        "warmup": args.warmup, "ms_per_step": round(max_ms / K, 4), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": DTYPE_NAME[dt], "data": "synthetic",
        "rows_per_s": round(N * K * world / (max_ms / 1e3), 1),
        "pct_of_peak": round(100 * value / world / peak, 2),
        "config": arm_config(cfg, world, esize),
        "step": ("one CUDA-graph replay of the captured fwd + bwd step (kernel_opt."
                 "fused_logprob_entropy + torch.autograd.grad), inputs resident in HBM"
                 if graph_ms is not None else "eager fwd + bwd calls"),
        "fwd": legs["fwd"], "bwd": legs["bwd"],
        "kernel_timing": ("each launch alone in a CUDA graph behind a write of "
                          f"{2 * L2_BYTES // 2**20} MiB (L2 flush), replayed between CUDA "
                          "events; the flush-only graph's time subtracted; median of 3"),
        "eager": {"value": round(step_bytes * K * world / (eager_ms / 1e3) / 1e9, 2),
                  "ms_per_step": round(eager_ms / K, 4),
                  "note": "kernel_opt.fused_logprob_entropy + torch.autograd.grad called "
                          "from Python every step"},
        "roofline": {"bound": "hbm", "kernel": "k1_bwd_ring_kernel",
                     "achieved": legs["bwd"]["gbs"], "peak": peak, "unit": "GB/s",
                     "frac": legs["bwd"]["frac"],
                     "peak_source": f"{peak_kind} (MEASURED_PEAKS.json hbm_gbs, copy)",
                     "algorithmic_bytes_per_launch": bwd_bytes,
                     "launch_ms": round(bwd_ms, 5),
                     "traffic": committed_traffic(cfg_name),
                     "per_kernel": [
                         {"kernel": "forward", "achieved": legs["fwd"]["gbs"],
                          "frac": legs["fwd"]["frac"], "launch_ms": round(fwd_ms, 5),
                          "algorithmic_bytes_per_launch": fwd_bytes},
                         {"kernel": "backward (k1_bwd_ring_kernel)", "achieved": legs["bwd"]["gbs"],
                          "frac": legs["bwd"]["frac"], "launch_ms": round(bwd_ms, 5),
                          "algorithmic_bytes_per_launch": bwd_bytes}],
                     "kernels_sum_over_step": round((fwd_ms + bwd_ms) / (max_ms / K), 4)},
        "gpu_launches": 2 * K,
        "e2e": {"value": round(step_bytes * K2 * world / (e2e_ms / 1e3) / 1e9, 3), "unit": UNIT,
                "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h_outputs,
                "ms_per_step": round(e2e_ms / K2, 3), "steps": K2,
                "note": "logits, targets and upstream grads from pinned host memory; "
                        "logprob/entropy/lse read back; the logits gradient stays on the GPU",
                "host_cpus_rank0": (f"bound to the {len(bound)} cores NVML reports next to "
                                    "the GPU" if bound else "process affinity unchanged")},
        "e2e_gradient_to_host": {
            "value": round(step_bytes * K2 * world / (e2e_host_grad_ms / 1e3) / 1e9, 3),
            "unit": UNIT, "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h_with_grad,
            "ms_per_step": round(e2e_host_grad_ms / K2, 3), "steps": K2},
        "clocks": clocks.summary(),
    }
    if extra is not None:
        out.update(extra)
    if vocab is not None:
        out["vocab_parallel"] = vocab
    if lmh_tp is not None:
        out["lmhead_vocab_parallel"] = lmh_tp
    if cpu is not None:
        out["cpu_baseline"] = cpu
    print(json.dumps(out), flush=True)


def grpo_arm(args, cfg, rank, local_rank, world):
    """The GRPO loss block on config 3: model logits [B, L, V] (the parent) -> per-token
    logps / entropies of the completion window at temperature T -> gradient w.r.t. the
    parent.  Two implementations on identical inputs, one GPU each (rows shard by batch
    element, no collective):
      fused   -- kernel_opt.grpo window node: scaled K1 forward on the strided window, one
                 backward launch writing the parent-shaped gradient;
      unfused -- the reference trainer's sequence (trainer.py:96-127): slice, in-place
                 division by T, K1, autograd backward through the division and the slices
                 (our K1 inside, one launch on the window).
    Peak extra device memory of one step is reported for both and for the fused node with
    inplace_backward (which reuses the logits' storage for the gradient)."""
    import torch.distributed as dist

    import kernel_opt
    from kernel_opt import grpo

    device = torch.device("cuda", local_rank)
    torch.cuda.set_device(device)
    if world > 1:
        dist.init_process_group("nccl", rank=rank, world_size=world, device_id=device,
                                timeout=datetime.timedelta(seconds=300))
    if not cfg["window"]:
        cfg = CONFIGS["c3"]
    B, S, V, dt = cfg["B"], cfg["S"], cfg["V"], cfg["dtype"]
    T = 0.7
    esize = torch.tensor([], dtype=dt).element_size()
    window, targets, g_lp, g_h = make_workload(cfg, device, seed=4321 + rank)
    parent = torch.as_strided(window, (B, S + 1, V), ((S + 1) * V, V, 1), 0)
    assert grpo.completion_window(parent, S).data_ptr() == window.data_ptr()
    N = B * S
    scale = grpo.temperature_scale(T)
    stream = torch.cuda.current_stream(device)
    # algorithmic bytes: forward reads the window; backward reads the window and writes
    # the whole parent-shaped gradient (window rows + the zeroed last row per sequence)
    fwd_bytes = N * V * esize + N * 20
    bwd_bytes = N * V * esize + B * (S + 1) * V * esize + N * 16
    step_bytes = fwd_bytes + bwd_bytes

    def fused(x):
        lp, h, _ = grpo._WindowLogprobEntropy.apply(x, targets, S, scale, False)
        return lp, h

    def unfused_fwd(y):
        w = grpo.completion_window(y, S)
        w.div_(T)
        lp, h, _ = kernel_opt.fused_logprob_entropy(w, targets)
        return lp, h

    def barrier():
        if world > 1:
            dist.barrier(device_ids=[local_rank])
        torch.cuda.synchronize(device)

    def run(kind, K, timed):
        ev = [[torch.cuda.Event(enable_timing=True) for _ in range(3)] for _ in range(K)]
        for i in range(K):
            x = parent.detach().requires_grad_(True)
            y = x.clone() if kind == "unfused" else x  # the clone stands in for the model
            ev[i][0].record(stream)                    # output that div_ overwrites
            lp, h = unfused_fwd(y) if kind == "unfused" else fused(y)
            ev[i][1].record(stream)
            (d,) = torch.autograd.grad((lp, h), x, (g_lp, g_h))
            ev[i][2].record(stream)
            del d, lp, h, x, y
        barrier()
        if not timed:
            return None
        f = [e[0].elapsed_time(e[1]) for e in ev]
        b = [e[1].elapsed_time(e[2]) for e in ev]
        return statistics.mean(f), statistics.mean(b)

    def check_equal():
        x = parent.detach().requires_grad_(True)
        a = fused(x)
        (da,) = torch.autograd.grad(a, x, (g_lp, g_h))
        x2 = parent.detach().requires_grad_(True)
        b = unfused_fwd(x2.clone())
        (db,) = torch.autograd.grad(b, x2, (g_lp, g_h))
        same = all(torch.equal(u.detach(), v.detach()) for u, v in zip(a, b)) and torch.equal(da, db)
        del x, x2, a, b, da, db
        return same

    class _ModelOutput(torch.autograd.Function):
        """Stand-in for the LM head: returns a copy of the parent as a non-leaf tensor and
        passes the gradient through without allocating."""

        @staticmethod
        def forward(ctx, src):
            return src.clone()

        @staticmethod
        def backward(ctx, g):
            return g

    def peak_extra(block):
        """Device memory the loss block allocates beyond the model output it consumes,
        forward through backward (peak, bytes)."""
        src = parent.detach().requires_grad_(True)
        y = _ModelOutput.apply(src)
        torch.cuda.synchronize(device)
        torch.cuda.reset_peak_memory_stats(device)
        base = torch.cuda.memory_allocated(device)
        lp, h = block(y)
        d = torch.autograd.grad((lp, h), src, (g_lp, g_h))
        torch.cuda.synchronize(device)
        extra = torch.cuda.max_memory_allocated(device) - base
        del d, lp, h, y, src
        return extra

    def fused_block(inplace):
        def f(y):
            lp, h, _ = grpo._WindowLogprobEntropy.apply(y, targets, S, scale, inplace)
            return lp, h
        return f

    for kind in ("fused", "unfused"):
        run(kind, max(3, args.warmup), False)
    bit_equal = check_equal()
    K = args.steps
    with ClockSampler(device) as clocks:
        barrier()
        t0 = torch.cuda.Event(enable_timing=True)
        t1 = torch.cuda.Event(enable_timing=True)
        t0.record(stream)
        fused_fb = run("fused", K, True)
        t1.record(stream)
        barrier()
    unfused_fb = run("unfused", K, True)
    total = torch.tensor([t0.elapsed_time(t1)], device=device, dtype=torch.float64)
    if world > 1:
        dist.all_reduce(total, op=dist.ReduceOp.MAX)
    max_ms = float(total.item())
    mem = {"fused": peak_extra(fused_block(False)), "fused_inplace": peak_extra(fused_block(True)),
           "unfused": peak_extra(unfused_fwd)}
    if world > 1:
        dist.barrier(device_ids=[local_rank])
        dist.destroy_process_group()
    if rank != 0:
        return
    peak, peak_kind = measured_peak_gbs()
    value = step_bytes * K * world / (max_ms / 1e3) / 1e9
    f_ms, b_ms = fused_fb
    uf_ms, ub_ms = unfused_fb
    out = {
        "metric": METRIC, "value": round(value, 2), "unit": UNIT, "n_gpus": world, "steps": K,
        "warmup": args.warmup, "ms_per_step": round(max_ms / K, 4), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": DTYPE_NAME[dt], "data": "synthetic",
        "rows_per_s": round(N * K * world / (max_ms / 1e3), 1),
        "pct_of_peak": round(100 * value / world / peak, 2),
        "config": {"workload": "GRPO loss block on " + cfg["workload"], "global_batch": B * world,
                   "seq_len": S, "vocab": V, "temperature": T,
                   "parallelism": f"row-sharded x{world} (no collective)",
                   "l2": (f"inputs larger than L2: {parent.numel() * esize / 2**20:.0f} MiB "
                          f"parent logits vs {L2_BYTES // 2**20} MiB L2")},
        "fused": {"fwd_ms": round(f_ms, 4), "bwd_ms": round(b_ms, 4),
                  "fwd_gbs": round(fwd_bytes / (f_ms / 1e3) / 1e9, 1),
                  "bwd_gbs": round(bwd_bytes / (b_ms / 1e3) / 1e9, 1)},
        "unfused_reference_sequence": {"fwd_ms": round(uf_ms, 4), "bwd_ms": round(ub_ms, 4)},
        "speedup_fused_vs_unfused": round((uf_ms + ub_ms) / (f_ms + b_ms), 3),
        "bit_identical": bit_equal,
        "peak_extra_bytes_per_step": mem,
        "peak_source": f"{peak_kind} (MEASURED_PEAKS.json hbm_gbs, copy)",
        "gpu_launches": 2 * K,
        "clocks": clocks.summary(),
    }
    print(json.dumps(out), flush=True)


def lmhead_arm(args, cfg, rank, local_rank, world):
    """LM head fused with K1 (kernel_opt.lm_head) against materialised logits, on config 3's
    rows and vocabulary with a Qwen2.5-7B-sized hidden state (H = 3584), bf16, T = 0.7:
      fused        -- tensor-core kernel: the forward folds each logits tile into K1's
                      statistics in the GEMM epilogue (no [N, V] tensor); the backward
                      recomputes the tiles chunk by chunk and writes K1's gradient, then
                      dh / dW by library GEMMs (4 GEMMs per training step);
      fused_keep   -- the same forward also writing the logits (keep_logits=True); backward
                      = K1's in-place backward + 2 library GEMMs (3 GEMMs, materialised
                      memory);
      materialised -- logits = h W^T (library GEMM), K1 with the temperature folded in,
                      autograd (3 GEMMs).
    Training step (forward + backward to hidden and weight) and no-grad forward (the
    old-policy / reference-policy log-probs of GRPO), peak extra device memory of each, and
    the fused forward kernel's own TFLOP/s against the library GEMM of the same shape.  The
    arms compared with each other take turns step by step (per-step events, medians), so
    they share the power-cap and thermal history."""
    import torch.distributed as dist

    import kernel_opt
    from kernel_opt import _C, lm_head

    device = torch.device("cuda", local_rank)
    torch.cuda.set_device(device)
    if world > 1:
        dist.init_process_group("nccl", rank=rank, world_size=world, device_id=device,
                                timeout=datetime.timedelta(seconds=300))
    B, S, V, H = 16, 1024, 151936, 3584
    N = B * S
    if args.lmh_rows:
        N = args.lmh_rows
    if args.lmh_vocab:
        V = args.lmh_vocab
    dt = torch.bfloat16
    T = 0.7
    gen = torch.Generator(device=device).manual_seed(99 + rank)
    h = (torch.randn(N, H, generator=gen, device=device) * 0.5).to(dt)
    w = (torch.randn(V, H, generator=gen, device=device) * (2.5 / H ** 0.5)).to(dt)
    t = torch.randint(0, V, (N,), generator=gen, device=device)
    g_lp = torch.full((N,), -1.0 / N, device=device)
    g_h = torch.full((N,), -0.01 / N, device=device)
    stream = torch.cuda.current_stream(device)
    gemm_flops = 2.0 * N * H * V
    from kernel_opt import grpo
    scale = grpo.temperature_scale(T)

    def fused_step(grad, keep=False):
        hx = h.detach().requires_grad_(grad)
        wx = w.detach().requires_grad_(grad)
        lp, ent, _ = lm_head.fused_linear_logprob_entropy(hx, wx, t, T, keep_logits=keep)
        if grad:
            torch.autograd.grad((lp, ent), (hx, wx), (g_lp, g_h))

    def fused_keep_step(grad):
        fused_step(grad, keep=True)

    def materialised_step(grad):
        hx = h.detach().requires_grad_(grad)
        wx = w.detach().requires_grad_(grad)
        z = hx @ wx.t()
        lp, ent, _ = kernel_opt.fused_logprob_entropy_scaled(z, t, T)
        if grad:
            torch.autograd.grad((lp, ent), (hx, wx), (g_lp, g_h))

    def timed(fn, grad, K):
        for _ in range(max(3, args.warmup)):
            with torch.set_grad_enabled(grad):
                fn(grad)
        torch.cuda.synchronize(device)
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record(stream)
        for _ in range(K):
            with torch.set_grad_enabled(grad):
                fn(grad)
        b.record(stream)
        torch.cuda.synchronize(device)
        return a.elapsed_time(b) / K

    def peak_extra(fn, grad):
        torch.cuda.synchronize(device)
        torch.cuda.reset_peak_memory_stats(device)
        base = torch.cuda.memory_allocated(device)
        with torch.set_grad_enabled(grad):
            fn(grad)
        torch.cuda.synchronize(device)
        return torch.cuda.max_memory_allocated(device) - base

    # the fused forward kernel alone (statistics only) against the library GEMM alone
    outs = [torch.empty(N, device=device) for _ in range(3)]
    zbuf = torch.empty((N, V), dtype=dt, device=device)

    def kernel_only(_grad):
        _C.lm_head_forward(h, w, t, *outs, scale, None)

    def library_gemm(_grad):
        torch.mm(h, w.t(), out=zbuf)

    def interleaved(arms, grad, K):
        # the arms take turns step by step (each step timed alone, median over K), so all
        # of them run under the same power-cap and thermal history
        for fn in arms.values():
            for _ in range(max(3, args.warmup)):
                with torch.set_grad_enabled(grad):
                    fn(grad)
        torch.cuda.synchronize(device)
        got = {k: [] for k in arms}
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        for _ in range(K):
            for k, fn in arms.items():
                a.record(stream)
                with torch.set_grad_enabled(grad):
                    fn(grad)
                b.record(stream)
                torch.cuda.synchronize(device)
                got[k].append(a.elapsed_time(b))
        return {k: statistics.median(v) for k, v in got.items()}

    K = max(1, min(args.steps, 10))
    with ClockSampler(device) as clocks:
        if world > 1:
            dist.barrier(device_ids=[local_rank])
        res = {}
        res.update(interleaved({"fused_train_ms": fused_step, "fused_keep_train_ms": fused_keep_step,
                                "materialised_train_ms": materialised_step}, True, K))
        res.update(interleaved({"fused_nograd_ms": fused_step,
                                "materialised_nograd_ms": materialised_step}, False, K))
        res.update(interleaved({"fused_forward_kernel_ms": kernel_only,
                                "library_gemm_ms": library_gemm}, False, K))
    def sustained(fn, seconds):
        # back to back for `seconds`, long enough to reach the board's power cap: TFLOP/s
        # with the median SM clock and board power seen meanwhile
        reps = max(5, int(seconds * 1e3 / timed(fn, False, 3)))
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        with ClockSampler(device, period_s=0.02) as cs:
            a.record(stream)
            for _ in range(reps):
                fn(False)
            b.record(stream)
            torch.cuda.synchronize(device)
        c = cs.summary()
        ms = a.elapsed_time(b) / reps
        return {"tflops": round(gemm_flops / (ms / 1e3) / 1e12, 1), "ms": round(ms, 3), "reps": reps,
                "sm_mhz": c["sm_mhz"], "power_w": c.get("power_w"), "reasons": c["reasons"]}

    sus = {}
    if args.lmh_sustained > 0:
        for _ in range(2):  # interleaved, so both see the same thermal history
            for name, fn in (("fused_forward_kernel", kernel_only), ("library_gemm", library_gemm)):
                sus.setdefault(name, []).append(sustained(fn, args.lmh_sustained))
    del zbuf
    torch.cuda.empty_cache()
    mem = {"fused_train": peak_extra(fused_step, True),
           "fused_keep_train": peak_extra(fused_keep_step, True),
           "materialised_train": peak_extra(materialised_step, True),
           "fused_nograd": peak_extra(fused_step, False),
           "materialised_nograd": peak_extra(materialised_step, False)}
    tp_ms = None
    if world > 1:
        # the same full-size head split over the ranks (tensor parallel): rank k holds rows
        # vocab_shard(V, world, k) of one shared weight; hidden and targets are the same on
        # every rank.  Forward: shard partials + one all-gather + combine; backward: shard
        # gradient recomputed + one fp32 all-reduce of dL/dhidden.  Strong scaling.
        from kernel_opt import parallel
        cols = parallel.vocab_shard(V, world, rank)
        g_tp = torch.Generator(device=device).manual_seed(7)
        h_tp = (torch.randn(N, H, generator=g_tp, device=device) * 0.5).to(dt)
        t_tp = torch.randint(0, V, (N,), generator=g_tp, device=device)
        w_tp = ((torch.randn(V, H, generator=g_tp, device=device) * (2.5 / H ** 0.5)).to(dt)
                [cols].contiguous())
        torch.cuda.empty_cache()

        def tp_step(grad, keep=False):
            hx = h_tp.detach().requires_grad_(grad)
            wx = w_tp.detach().requires_grad_(grad)
            lp, ent, _ = parallel.vocab_parallel_fused_linear_logprob_entropy(
                hx, wx, t_tp, cols.start, T, keep_logits=keep)
            if grad:
                torch.autograd.grad((lp, ent), (hx, wx), (g_lp, g_h))

        def tp_keep_step(grad):
            tp_step(grad, keep=True)

        got = []
        for fn, grad in ((tp_step, True), (tp_step, False), (tp_keep_step, True)):
            dist.barrier(device_ids=[local_rank])
            got.append(timed(fn, grad, K))
        tp_ms = torch.tensor(got, device=device, dtype=torch.float64)
        dist.all_reduce(tp_ms, op=dist.ReduceOp.MAX)
        del h_tp, w_tp
    tt = torch.tensor([res["fused_keep_train_ms"]], device=device, dtype=torch.float64)
    if world > 1:
        dist.all_reduce(tt, op=dist.ReduceOp.MAX)
        dist.barrier(device_ids=[local_rank])
        dist.destroy_process_group()
    if rank != 0:
        return
    max_ms = float(tt.item())
    peaks = {}
    try:
        with open(os.path.join(REPO, "MEASURED_PEAKS.json")) as f:
            peaks = json.load(f)
    except Exception:
        pass
    tc_peak = float(peaks.get("bf16_tflops") or 1590.0)
    kern_tf = gemm_flops / (res["fused_forward_kernel_ms"] / 1e3) / 1e12
    useful = 3 * gemm_flops  # forward logits, dh, dW
    out = {
        "metric": "LM head + K1 fwd+bwd, useful GEMM TFLOP/s (3 GEMMs per step)",
        "value": round(useful * world / (max_ms / 1e3) / 1e12, 1), "unit": "TFLOP/s",
        "n_gpus": world, "steps": K, "warmup": max(3, args.warmup), "ms_per_step": round(max_ms, 3),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic",
        "config": {"workload": (f"LM head [{H} -> {V}] + K1 on {N} rows" if (args.lmh_rows or args.lmh_vocab)
                                else "LM head [3584 -> 151936] + K1 on config 3's 16 x 1024 rows"),
                   "rows": N, "hidden": H, "vocab": V, "temperature": T,
                   "step": "fused_keep (keep_logits=True) training step",
                   "parallelism": f"row-sharded x{world} (no collective)"},
        "times_ms": {k: round(v, 3) for k, v in res.items()},
        "speedup_train_keep_vs_materialised": round(res["materialised_train_ms"] / res["fused_keep_train_ms"], 3),
        "speedup_train_fused_vs_materialised": round(res["materialised_train_ms"] / res["fused_train_ms"], 3),
        "speedup_nograd": round(res["materialised_nograd_ms"] / res["fused_nograd_ms"], 3),
        "peak_extra_bytes": mem,
        "roofline": {"bound": "tensor", "kernel": "k1_lmhead_kernel (statistics only)",
                     "achieved": round(kern_tf, 1), "peak": tc_peak, "unit": "TFLOP/s",
                     "frac": round(kern_tf / tc_peak, 4),
                     "library_gemm_tflops": round(gemm_flops / (res["library_gemm_ms"] / 1e3) / 1e12, 1),
                     "note": "2 N H V flops per launch; peak = MEASURED_PEAKS.json bf16 "
                             "(burst, cuBLAS 8192^3)"},
        "gpu_launches": 2 * K,
        "clocks": clocks.summary(),
    }
    if tp_ms is not None:
        tr, tn, tk = float(tp_ms[0]), float(tp_ms[1]), float(tp_ms[2])
        out["vocab_parallel"] = {
            "workload": f"the same head split over {world} GPUs: {V} vocabulary rows of W, "
                        f"{V // world}-{-(-V // world)} per GPU; hidden and targets on every GPU",
            "scaling": "strong",
            "train_ms": round(tr, 3), "nograd_ms": round(tn, 3), "train_keep_ms": round(tk, 3),
            "speedup_train_keep_vs_one_gpu_keep": round(res["fused_keep_train_ms"] / tk, 3),
            "train_useful_tflops_total": round(useful / (tr / 1e3) / 1e12, 1),
            "speedup_train_vs_one_gpu_fused": round(res["fused_train_ms"] / tr, 3),
            "speedup_nograd_vs_one_gpu_fused": round(res["fused_nograd_ms"] / tn, 3),
            "collectives": "forward: one NCCL all-gather of [N, 4] float64 partials; backward: "
                           "one NCCL all-reduce of dL/dhidden [N, H] fp32",
            "note": "max over ranks of CUDA-event step times; one-GPU figures are this run's "
                    "fused (memory-light) arms",
        }
    if sus:
        out["sustained"] = dict(sus, note=f"each kernel back to back for ~{args.lmh_sustained:g} s "
                                          "(at the power cap), the two interleaved, 2 rounds")
    print(json.dumps(out), flush=True)


def vocab_arm(args, cfg, rank, local_rank, world):
    """Vocab-parallel K1 (tensor-parallel LM head layout): rank k holds columns
    vocab_shard(V, world, k) of every row; forward = shard partials + one all-gather + merge,
    backward local.  The total problem is fixed (strong scaling)."""
    import torch.distributed as dist

    from kernel_opt import parallel

    device = torch.device("cuda", local_rank)
    torch.cuda.set_device(device)
    os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
    os.environ.setdefault("MASTER_PORT", "29561")
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=device,
                            timeout=datetime.timedelta(seconds=300))
    N, V, dt = cfg["B"] * cfg["S"], cfg["V"], cfg["dtype"]
    esize = torch.tensor([], dtype=dt).element_size()
    cols = parallel.vocab_shard(V, world, rank)
    Vr = cols.stop - cols.start
    gen = torch.Generator(device=device).manual_seed(7000 + rank)
    xs = torch.empty((N, Vr), dtype=dt, device=device)
    for a in range(0, N, 1024):
        b = min(N, a + 1024)
        xs[a:b] = (torch.randn((b - a, Vr), generator=gen, device=device) * cfg["scale"]).to(dt)
    tg = torch.Generator(device=device).manual_seed(99)
    targets = torch.randint(0, V, (N,), generator=tg, device=device)
    g_lp = torch.full((N,), -1.0 / N, device=device)
    g_h = torch.full((N,), -0.01 / N, device=device)
    stream = torch.cuda.current_stream(device)

    def step():
        x = xs.detach().requires_grad_(True)
        lp, h, _l = parallel.vocab_parallel_fused_logprob_entropy(x, targets, cols.start)
        (d,) = torch.autograd.grad((lp, h), x, (g_lp, g_h))
        return d

    def barrier():
        dist.barrier(device_ids=[local_rank])
        torch.cuda.synchronize(device)

    for _ in range(max(3, args.warmup)):
        step()
    barrier()
    K = args.steps
    start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(device) as clocks:
        barrier()
        start.record(stream)
        for _ in range(K):
            step()
        stop.record(stream)
        barrier()
    t = torch.tensor([start.elapsed_time(stop)], device=device, dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    max_ms = float(t.item())
    barrier()
    dist.destroy_process_group()
    if rank != 0:
        return
    fwd, bwd = algorithmic_bytes(N, V, esize)
    value = (fwd + bwd) * K / (max_ms / 1e3) / 1e9
    peak, peak_kind = measured_peak_gbs()
    out = {
        "metric": METRIC, "value": round(value, 2), "unit": UNIT, "n_gpus": world, "steps": K,
        "warmup": args.warmup, "ms_per_step": round(max_ms / K, 4), "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": DTYPE_NAME[dt], "data": "synthetic",
        "rows_per_s": round(N * K / (max_ms / 1e3), 1),
        "pct_of_peak_per_gpu": round(100 * value / world / peak, 2),
        "config": {"workload": cfg["workload"], "rows": N, "vocab": V, "vocab_per_gpu": Vr,
                   "parallelism": f"vocab-parallel x{world}: one all-gather of [N,4] float64 "
                                  "per forward, local backward"},
        "peak_source": f"{peak_kind} (MEASURED_PEAKS.json hbm_gbs, copy)",
        "gpu_launches": 4 * K,
        "clocks": clocks.summary(),
    }
    print(json.dumps(out), flush=True)


def main():
    ap = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=100)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--config", choices=sorted(CONFIGS), default="c2")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-extra-configs", action="store_true",
                    help="skip the config 3 / config 4 kernel legs of the N = 1 line")
    ap.add_argument("--no-lmhead-tp", action="store_true",
                    help="skip the tensor-parallel LM head record (lmhead_vocab_parallel)")
    ap.add_argument("--no-vocab-parallel", action="store_true",
                    help="skip the config 5 vocab-parallel sub-record")
    ap.add_argument("--lmh-rows", type=int, default=0,
                    help="--mode lmhead: rows (default 16384; smaller for profiling)")
    ap.add_argument("--lmh-sustained", type=float, default=2.0,
                    help="--mode lmhead: seconds per sustained (power-capped) run of the fused "
                         "forward kernel and of the library GEMM; 0 skips them")
    ap.add_argument("--lmh-vocab", type=int, default=0,
                    help="--mode lmhead: vocabulary (default 151936; smaller for profiling)")
    ap.add_argument("--eager", action="store_true",
                    help="time eager steps only (no CUDA-graph replay of the step)")
    ap.add_argument("--mode", choices=["rows", "vocab", "grpo", "lmhead"], default="rows",
                    help="rows: row-sharded (default); vocab: vocab-parallel (config c5); "
                         "grpo: the GRPO loss block on config c3, fused vs unfused; "
                         "lmhead: LM head fused with K1 vs materialised logits")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    rank, local_rank, world = dist_env()
    cfg = CONFIGS[args.config]
    if args.impl == "reference":
        if args.mode == "grpo":
            reference_grpo_arm(args, cfg, rank, world)
        else:
            reference_arm(args, cfg, rank, world)
    elif args.mode == "grpo":
        grpo_arm(args, cfg, rank, local_rank, world)
    elif args.mode == "lmhead":
        lmhead_arm(args, cfg, rank, local_rank, world)
    elif args.mode == "vocab":
        vocab_arm(args, CONFIGS["c5"] if args.config == "c2" else cfg, rank, local_rank, world)
    else:
        ours_arm(args, cfg, rank, local_rank, world)


if __name__ == "__main__":
    main()

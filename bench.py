#!/usr/bin/env python
"""Benchmark of the hot path on B200: one JSON line on rank 0.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--workload NAME]

Workloads (synthetic, seeded inputs with the documented shapes/distributions):

  tv_iso_l1   (default) tv_loss_iso_3d (eps 1e-8) and tv_loss_l1_3d forward +
              gradient on fp32 [4, 256, 256, 256], uniform[0, 1) with 1% of
              voxels set to their +W neighbour, seed 1. A step runs both
              single-sweep ops on the volume. At N GPUs the volume is
              [4, 256*N, 256, 256], split along D (one 256-plane slab per rank,
              halo exchange and rank-ordered loss sum each step): weak scaling.
  tv_sq_128   tv_loss_sq_3d forward + gradient on [128, 128, 128], seed 0.
  kplanes     kplanes_tilted_fuse forward + backward (autograd ops), N = 2^20
              points uniform in [-1, 1]^3, 4 rotations from normalised N(0, 1)
              quaternions, C = 32, 256x256 planes uniform[0.1, 0.5], upstream
              N(0, 1), seed 2. At N GPUs each rank holds its own 2^20 points
              and the plane/rotation gradients are all-reduced: weak scaling.
  tv_1024     tv_loss_sq_3d + tv_loss_iso_3d forward + gradient on [1024]^3,
              sum of 64 Gaussian blobs (sigma 8..64) + N(0, 0.01) noise, seed 4.

The default line (tv_iso_l1) also carries a `kplanes` object: the kplanes
workload measured in the same run, with the same keys, so that one run
reports both halves of the metric.

`value` is whole-job throughput with inputs resident in HBM; `e2e` is the same
metric through the public API from pinned host buffers: the host->device copy
of the step's inputs and the device->host copy of everything the step
produces (losses and gradients; for K-Planes the output and all gradients)
inside the timed region (`e2e.losses_only` leaves the TV gradients on the
device). `roofline` reports the dominant kernel's algorithmic bytes per launch
over its CUDA-event duration against the measured HBM copy bandwidth.
`ref_cuda` times the reference's own sm_100a kernels (its `_core` built from
its sources into oracle/_ref/) on the same GPU, driven with the calls its op
layer makes. `cpu_baseline` is the C oracle (OpenMP, all host threads) and
`cpu_baseline_torch` the reference's pure-torch test definitions on the host
cores, each on a bounded sample. At N > 1 `breakdown` splits a step into the
local work and the exposed cross-rank exchange.
`--impl reference` times the reference computation on the host cores (the
CPU oracle, a restatement of the reference's kernels: the reference itself
has no CPU implementation), on a bounded sample of the same workload.
"""

from __future__ import annotations

import argparse
import datetime
import json
import math
import os
import statistics
import sys
import time
from pathlib import Path

REPO = Path(__file__).resolve().parent
sys.path.insert(0, str(REPO / "quantem-cuda_b200"))
sys.path.insert(0, str(REPO))

import numpy as np  # noqa: E402
import torch  # noqa: E402
import torch.distributed as dist  # noqa: E402

FALLBACK_HBM_GBS = 6650.0


# ── environment ─────────────────────────────────────────────────────────────


def measured_hbm_peak() -> tuple[float, str]:
    p = REPO / "MEASURED_PEAKS.json"
    try:
        return float(json.loads(p.read_text())["hbm_gbs"]), "measured"
    except Exception:
        return FALLBACK_HBM_GBS, "fallback"


def ncu_traffic(workload: str) -> dict | None:
    """Per-launch DRAM traffic of the dominant kernel from a committed ncu
    summary (profiles/*.md lines 'traffic <workload> <bytes_per_unit> <unit>')."""
    for f in sorted((REPO / "profiles").glob("*.md")):
        for line in f.read_text().splitlines():
            parts = line.strip().strip("`").split()
            if len(parts) >= 4 and parts[0] == "traffic" and parts[1] == workload:
                try:
                    return {"bytes_per_unit": float(parts[2]), "unit": parts[3], "source": f.name}
                except ValueError:
                    pass
    return None


# The NVML poller runs in a process of its own: in a thread of this process it
# would wait for the GIL, which the loop issuing the timed steps holds for
# most of a region a few milliseconds long. It keeps (monotonic time, SM MHz,
# reasons, power W) samples until told the region's bounds on stdin, answers
# with the samples inside them as one JSON line and exits; it also exits when
# its stdin closes (this process gone).
_POLLER = r"""
import json, select, sys, time
import pynvml as nv
nv.nvmlInit()
key, period = sys.argv[1], float(sys.argv[2])
h = nv.nvmlDeviceGetHandleByUUID(key[5:]) if key.startswith("uuid:") else nv.nvmlDeviceGetHandleByIndex(int(key[6:]))
out, k, power = [], 0, float("nan")
print("ready", flush=True)
while True:
    if select.select([sys.stdin], [], [], 0)[0]:
        line = sys.stdin.readline()
        if line:
            t0, t1 = map(float, line.split())
            print(json.dumps([s for s in out if t0 <= s[0] <= t1]), flush=True)
        break
    try:
        mhz = nv.nvmlDeviceGetClockInfo(h, nv.NVML_CLOCK_SM)
        reasons = nv.nvmlDeviceGetCurrentClocksEventReasons(h)
        if k % 8 == 0:
            power = nv.nvmlDeviceGetPowerUsage(h) / 1000.0
        k += 1
        out.append((time.monotonic(), mhz, reasons, power))
    except Exception:
        pass
    time.sleep(period)
"""


class ClockSampler:
    """Samples SM clock, power and throttle reasons through NVML while the
    timed region runs (reads only; changes no setting), from a poller process
    started with the sampler (before the warm-up)."""

    REASONS = {
        0x1: "gpu_idle",
        0x2: "applications_clocks_setting",
        0x4: "sw_power_cap",
        0x8: "hw_slowdown",
        0x20: "sync_boost",
        0x40: "sw_thermal_slowdown",
        0x80: "hw_thermal_slowdown",
        0x100: "hw_power_brake_slowdown",
        0x200: "display_clock_setting",
    }

    def __init__(self, device_index: int, period_s: float = 0.0005, ready_timeout_s: float = 30.0):
        import subprocess

        self.samples: list[tuple[int, int, float]] = []
        self.max_mhz = None
        self.handle = None
        self._proc = None
        self._t0 = self._t1 = None
        try:
            import pynvml

            pynvml.nvmlInit()
            key = None
            try:
                key = "uuid:GPU-" + str(torch.cuda.get_device_properties(device_index).uuid)
                self.handle = pynvml.nvmlDeviceGetHandleByUUID(key[5:])
            except Exception:
                self.handle = None
            if self.handle is None:
                vis = os.environ.get("CUDA_VISIBLE_DEVICES")
                idx = int(vis.split(",")[device_index]) if vis and vis.split(",")[0].isdigit() else device_index
                key = f"index:{idx}"
                self.handle = pynvml.nvmlDeviceGetHandleByIndex(idx)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self.handle, pynvml.NVML_CLOCK_SM)
        except Exception:
            self.handle = None
            return
        try:
            self._proc = subprocess.Popen([sys.executable, "-c", _POLLER, key, str(period_s)],
                                          stdin=subprocess.PIPE, stdout=subprocess.PIPE,
                                          stderr=subprocess.DEVNULL, text=True)
            if self._readline(ready_timeout_s) != "ready":
                self._close()
        except Exception:
            self._close()

    def _readline(self, timeout_s: float) -> str | None:
        import select

        if select.select([self._proc.stdout], [], [], timeout_s)[0]:
            return self._proc.stdout.readline().strip()
        return None

    def _close(self):
        if self._proc is not None:
            try:
                self._proc.kill()
                self._proc.wait(timeout=10)
            except Exception:
                pass
        self._proc = None

    def _collect(self):
        if self._proc is None:
            return
        try:
            if self._t0 is not None and self._t1 is not None:
                self._proc.stdin.write(f"{self._t0!r} {self._t1!r}\n")
                self._proc.stdin.flush()
                line = self._readline(30.0)
                if line:
                    self.samples = [(int(m), int(r), float(p)) for _, m, r, p in json.loads(line)]
            self._proc.stdin.close()
            self._proc.wait(timeout=10)
        except Exception:
            pass
        self._close()

    def __enter__(self):
        self._t0 = time.monotonic()
        return self

    def __exit__(self, *exc):
        self._t1 = time.monotonic()

    def __del__(self):
        self._close()

    def summary(self) -> dict:
        self._collect()
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": self.max_mhz, "reasons": [], "samples": 0}
        mhz = [s[0] for s in self.samples]
        bits = 0
        for s in self.samples:
            bits |= s[1]
        reasons = [name for bit, name in self.REASONS.items() if bits & bit and name != "gpu_idle"]
        return {
            "sm_mhz": statistics.median(mhz),
            "sm_max_mhz": self.max_mhz,
            "reasons": reasons,
            "samples": len(self.samples),
            "power_w_max": max((s[2] for s in self.samples if s[2] == s[2]), default=None),
        }


# ── workload inputs ─────────────────────────────────────────────────────────


def tv_iso_l1_volume(seed: int, d: int = 256) -> torch.Tensor:
    gen = torch.Generator().manual_seed(seed)
    vol = torch.rand((4, d, 256, 256), generator=gen)
    flat = vol.view(-1, 256)
    rows = torch.randint(0, flat.shape[0], (vol.numel() // 100,), generator=gen)
    cols = torch.randint(0, 255, rows.shape, generator=gen)
    flat[rows, cols] = flat[rows, cols + 1]  # dw == 0 exactly: sign(0) = 0
    return vol


def blob_volume(n: int, seed: int, device, z0: int = 0, z1: int | None = None) -> torch.Tensor:
    """Planes [z0, z1) of an [n, n, n] volume: sum of 64 Gaussian blobs
    (centres U[0, n)^3, sigma U[8, 64], amplitude 1) + N(0, 0.01) noise, built
    on the device plane by plane (each plane's noise seeded by its index, so a
    D-slab of the volume does not depend on how the volume is split)."""
    z1 = n if z1 is None else z1
    gen = torch.Generator().manual_seed(seed)
    centres = torch.rand((64, 3), generator=gen) * n
    sigmas = 8 + torch.rand(64, generator=gen) * 56
    vol = torch.empty((z1 - z0, n, n), device=device)
    ax = torch.arange(n, device=device, dtype=torch.float32)
    for z in range(z0, z1):
        plane = torch.zeros((n, n), device=device)
        for (cz, cy, cx), s in zip(centres.tolist(), sigmas.tolist()):
            wz = math.exp(-((z - cz) ** 2) / (2 * s * s))
            if wz < 1e-6:
                continue
            gy = torch.exp(-((ax - cy) ** 2) / (2 * s * s))
            gx = torch.exp(-((ax - cx) ** 2) / (2 * s * s))
            plane += wz * gy[:, None] * gx[None, :]
        gd = torch.Generator(device=device).manual_seed(seed * 1_000_003 + z)
        vol[z - z0] = plane + 0.01 * torch.randn((n, n), device=device, generator=gd)
    return vol


def quaternion_rotations(T: int, gen: torch.Generator) -> torch.Tensor:
    q = torch.randn((T, 4), generator=gen)
    q = q / q.norm(dim=1, keepdim=True)
    w, x, y, z = q.unbind(1)
    return torch.stack(
        [
            1 - 2 * (y * y + z * z), 2 * (x * y - z * w), 2 * (x * z + y * w),
            2 * (x * y + z * w), 1 - 2 * (x * x + z * z), 2 * (y * z - x * w),
            2 * (x * z - y * w), 2 * (y * z + x * w), 1 - 2 * (x * x + y * y),
        ],
        dim=1,
    ).reshape(T, 3, 3)


def kplanes_inputs(seed: int, N: int = 1 << 20, T: int = 4, C: int = 32, res: int = 256):
    gen = torch.Generator().manual_seed(seed)
    pts = torch.empty((N, 3)).uniform_(-1.0, 1.0, generator=gen)
    rot = quaternion_rotations(T, gen)
    plane = torch.empty((3 * T, C, res, res)).uniform_(0.1, 0.5, generator=gen)
    up = torch.randn((N, T * C), generator=gen)
    return pts, rot, plane, up


# ── timing helpers ──────────────────────────────────────────────────────────


class Ctx:
    def __init__(self, args):
        self.args = args
        self.world = int(os.environ.get("WORLD_SIZE", "1"))
        self.rank = int(os.environ.get("RANK", "0"))
        self.local_rank = int(os.environ.get("LOCAL_RANK", "0"))
        self.device = None

    def barrier(self):
        if self.world > 1:
            dist.barrier(device_ids=[self.local_rank]) if self.device is not None else dist.barrier()

    def max_over_ranks(self, x: float) -> float:
        if self.world == 1:
            return x
        t = torch.tensor([x], dtype=torch.float64, device=self.device)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())


def time_steps(ctx: Ctx, step, steps: int, warmup: int, sampler: ClockSampler | None = None):
    for _ in range(warmup):
        step()
    torch.cuda.synchronize()
    ctx.barrier()
    torch.cuda.synchronize()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    if sampler is not None:
        sampler.__enter__()
    start.record()
    for _ in range(steps):
        step()
    end.record()
    torch.cuda.synchronize()
    if sampler is not None:
        sampler.__exit__(None, None, None)
    ctx.barrier()
    ms = start.elapsed_time(end)
    return ctx.max_over_ranks(ms)


def time_with_op_events(ctx: Ctx, step, steps: int, warmup: int, timers, sampler=None) -> float:
    """The timed pass (K steps, no events between the ops; its duration is
    returned), then a second pass of K steps with each timer's events around
    its op, which is where the per-op durations of the line come from."""
    for t in timers:
        t.enabled = False
    ms = time_steps(ctx, step, steps, warmup, sampler)
    for t in timers:
        t.enabled = True
    time_steps(ctx, step, steps, 0)
    return ms


def time_pipelined(ctx: Ctx, step, steps: int, warmup: int, side_streams) -> float:
    """time_steps for steps whose copies run on side streams: the end event
    is recorded once the compute stream has waited for every side stream, so
    the timed region holds all K steps' copies and kernels."""
    for _ in range(warmup):
        step()
    torch.cuda.synchronize()
    ctx.barrier()
    torch.cuda.synchronize()
    cur = torch.cuda.current_stream()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record(cur)
    for _ in range(steps):
        step()
    for s_ in side_streams:
        cur.wait_stream(s_)
    end.record(cur)
    torch.cuda.synchronize()
    ctx.barrier()
    return ctx.max_over_ranks(start.elapsed_time(end))


class KernelTimer:
    """CUDA-event durations of one launch site (an op) of the step. Disabled
    timers call straight through: events recorded between two ops would
    separate a sweep from the kernel before it, which costs it the
    programmatic-dependent-launch overlap, so the timed pass runs without them
    and time_with_op_events() measures the ops in a second pass."""

    def __init__(self):
        self.pairs = []
        self.enabled = True

    def wrap(self, fn):
        def run(*a, **k):
            if not self.enabled:
                return fn(*a, **k)
            s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            s.record()
            r = fn(*a, **k)
            e.record()
            self.pairs.append((s, e))
            return r

        return run

    def mean_ms(self, last: int) -> float:
        sel = self.pairs[-last:]
        return sum(s.elapsed_time(e) for s, e in sel) / max(1, len(sel))


# ── CPU baselines: the C oracle (OpenMP) and the pure-torch definitions ─────


def cpu_oracle():
    from oracle import oracle

    oracle.build()
    n = oracle.available_cores()
    oracle.set_threads(n)
    return oracle, oracle.threads()


def _time_cpu(step, min_seconds: float, reps: int | None, warmup: int) -> tuple[float, int]:
    """Runs `step` `warmup` times, then `reps` times (or until `min_seconds`
    have passed); returns (elapsed seconds, steps timed)."""
    for _ in range(warmup):
        step()
    t0 = time.perf_counter()
    k = 0
    while True:
        step()
        k += 1
        el = time.perf_counter() - t0
        if (reps is not None and k >= reps) or (reps is None and el >= min_seconds):
            return el, k


def _torch_threads() -> int:
    try:
        n = len(os.sched_getaffinity(0))
    except AttributeError:  # pragma: no cover
        n = os.cpu_count() or 1
    torch.set_num_threads(n)
    return torch.get_num_threads()


def cpu_tv_iso_l1(sample_d: int = 32, min_seconds: float = 10.0, reps: int | None = None, warmup: int = 1):
    oracle, threads = cpu_oracle()
    x = tv_iso_l1_volume(1, d=sample_d).numpy()
    b, d, h, w = x.shape
    n = b * (d - 1) * (h - 1) * (w - 1)

    def step():
        oracle.tv_iso_sum(x, 1e-8)
        oracle.tv_iso_grad(x, 1.0 / n, 1e-8)
        oracle.tv_l1_loss(x)
        oracle.tv_l1_grad(x, [1.0, 1.0, 1.0])

    el, k = _time_cpu(step, min_seconds, reps, warmup)
    return {
        "value": x.size / (el / k),
        "unit": "voxels/s",
        "cores": threads,
        "kind": "port",
        "sample": f"[4, {sample_d}, 256, 256] slab of the workload volume (1/{256 // sample_d} of it): "
        f"iso loss + iso grad + L1 sums + L1 grad with the C oracle (OpenMP), {k} reps, {el:.3f} s",
    }, el / k


def torch_cpu_tv_iso_l1(sample_d: int = 16, min_seconds: float = 10.0, reps: int | None = None, warmup: int = 1):
    """The reference's pure-torch definitions (its tests' tv_iso_ref and
    tv_l1_ref, restated in oracle/torch_ref.py) with autograd gradients."""
    from oracle import torch_ref

    threads = _torch_threads()
    vol = tv_iso_l1_volume(1, d=sample_d)
    ones = torch.ones(3)

    def step():
        v = vol.clone().requires_grad_(True)
        torch_ref.tv_iso(v, 1e-8).backward()
        v2 = vol.clone().requires_grad_(True)
        torch_ref.tv_l1(v2).backward(ones)

    el, k = _time_cpu(step, min_seconds, reps, warmup)
    return {
        "value": vol.numel() / (el / k),
        "unit": "voxels/s",
        "cores": threads,
        "kind": "port (pure torch, the reference's test definitions)",
        "sample": f"[4, {sample_d}, 256, 256] slab of the workload volume: iso loss + L1 sums with torch "
        f"autograd gradients, {k} reps, {el:.3f} s",
    }, el / k


def cpu_tv_sq_128(min_seconds: float = 10.0, reps: int | None = None, warmup: int = 1):
    oracle, threads = cpu_oracle()
    x = torch.rand((128, 128, 128), generator=torch.Generator().manual_seed(0)).numpy()

    def step():
        oracle.tv_sq_loss(x)
        oracle.tv_sq_grad(x, 1.0)

    el, k = _time_cpu(step, min_seconds, reps, warmup)
    return {
        "value": x.size / (el / k),
        "unit": "voxels/s",
        "cores": threads,
        "kind": "port",
        "sample": f"the whole [128, 128, 128] volume: sq loss + grad with the C oracle (OpenMP), "
        f"{k} reps, {el:.3f} s",
    }, el / k


def torch_cpu_tv_sq_128(min_seconds: float = 10.0, reps: int | None = None, warmup: int = 1):
    from oracle import torch_ref

    threads = _torch_threads()
    vol = torch.rand((128, 128, 128), generator=torch.Generator().manual_seed(0))

    def step():
        v = vol.clone().requires_grad_(True)
        torch_ref.tv_sq(v).backward()

    el, k = _time_cpu(step, min_seconds, reps, warmup)
    return {
        "value": vol.numel() / (el / k),
        "unit": "voxels/s",
        "cores": threads,
        "kind": "port (pure torch, the reference's test definitions)",
        "sample": f"the whole [128, 128, 128] volume: sq loss with a torch autograd gradient, {k} reps, "
        f"{el:.3f} s",
    }, el / k


def cpu_kplanes(sample_n: int = 1 << 14, min_seconds: float = 10.0, reps: int | None = None, warmup: int = 1):
    oracle, threads = cpu_oracle()
    pts, rot, plane, up = kplanes_inputs(2)
    p, r, g, u = pts[:sample_n].numpy(), rot.numpy(), plane.numpy(), up[:sample_n].numpy()

    def step():
        oracle.kplanes_fwd(p, r, g)
        oracle.kplanes_bwd(p, r, g, u)

    el, k = _time_cpu(step, min_seconds, reps, warmup)
    return {
        "value": sample_n / (el / k),
        "unit": "points/s",
        "cores": threads,
        "kind": "port",
        "sample": f"first {sample_n} of the 2^20 points, forward + backward with the C oracle "
        f"(OpenMP), {k} reps, {el:.3f} s",
    }, el / k


def torch_cpu_kplanes(sample_n: int = 1 << 15, min_seconds: float = 10.0, reps: int | None = None,
                      warmup: int = 1):
    """The reference's pure-torch definition (its test's grid_sample
    `reference`, restated in oracle/torch_ref.py) with autograd gradients."""
    from oracle import torch_ref

    threads = _torch_threads()
    pts, rot, plane, up = kplanes_inputs(2)
    p, u = pts[:sample_n].clone(), up[:sample_n].clone()

    def step():
        inp = [t.clone().requires_grad_(True) for t in (p, rot, plane)]
        torch_ref.kplanes_tilted(*inp).backward(u)

    el, k = _time_cpu(step, min_seconds, reps, warmup)
    return {
        "value": sample_n / (el / k),
        "unit": "points/s",
        "cores": threads,
        "kind": "port (pure torch, the reference's test definition)",
        "sample": f"first {sample_n} of the 2^20 points, forward + autograd backward (grid_sample), "
        f"{k} reps, {el:.3f} s",
    }, el / k


def cpu_tv_1024(sample_d: int = 4, min_seconds: float = 10.0, reps: int | None = None, warmup: int = 1):
    oracle, threads = cpu_oracle()
    x = blob_volume(1024, 4, "cpu", 510, 510 + sample_d).numpy()

    def step():
        oracle.tv_sq_loss(x)
        oracle.tv_sq_grad(x, 1.0)
        oracle.tv_iso_sum(x, 1e-8)
        oracle.tv_iso_grad(x, 1.0, 1e-8)

    el, k = _time_cpu(step, min_seconds, reps, warmup)
    return {
        "value": x.size / (el / k),
        "unit": "voxels/s",
        "cores": threads,
        "kind": "port",
        "sample": f"[{sample_d}, 1024, 1024] slab (planes 510..) of the volume: sq loss + grad and iso "
        f"loss + grad with the C oracle (OpenMP), {k} reps, {el:.3f} s",
    }, el / k


def cpu_kplanes_ms(sample_n: int = 2048, min_seconds: float = 10.0, reps: int | None = None, warmup: int = 1):
    oracle, threads = cpu_oracle()
    gen = torch.Generator().manual_seed(3)
    pts = torch.empty((sample_n, 3)).uniform_(-1.0, 1.0, generator=gen).numpy()
    rot = quaternion_rotations(8, gen).numpy()
    planes = [torch.empty((24, 32, r, r)).uniform_(0.1, 0.5, generator=gen).numpy() for r in (64, 128, 256, 512)]
    up = torch.randn((sample_n, 256), generator=gen).numpy()

    def step():
        for g in planes:
            oracle.kplanes_fwd(pts, rot, g)
            oracle.kplanes_bwd(pts, rot, g, up)

    el, k = _time_cpu(step, min_seconds, reps, warmup)
    return {
        "value": sample_n / (el / k),
        "unit": "points/s",
        "cores": threads,
        "kind": "port",
        "sample": f"{sample_n} points through all four levels (T=8, C=32), forward + backward with the "
        f"C oracle (OpenMP), {k} reps, {el:.3f} s",
    }, el / k


CPU_BASELINES = {
    "tv_iso_l1": cpu_tv_iso_l1,
    "reference_suite": cpu_tv_iso_l1,
    "tv_multi": cpu_tv_iso_l1,
    "tv_sq_128": cpu_tv_sq_128,
    "tv_1024": cpu_tv_1024,
    "kplanes": cpu_kplanes,
    "kplanes_ms": cpu_kplanes_ms,
}

TORCH_CPU_BASELINES = {
    "tv_iso_l1": torch_cpu_tv_iso_l1,
    "tv_multi": torch_cpu_tv_iso_l1,
    "tv_sq_128": torch_cpu_tv_sq_128,
    "kplanes": torch_cpu_kplanes,
}


# ── the reference's own CUDA kernels on this GPU ────────────────────────────


def reference_core():
    """(the reference's `_core` built from its sources into oracle/_ref/, or
    None, and the reason when it is missing)."""
    try:
        from oracle import oracle
    except Exception as e:  # pragma: no cover
        return None, f"oracle package not importable: {e}"
    core = oracle.ref_core()
    if core is None:
        return None, "the reference's _core was not built into oracle/_ref"
    return core, None


def ref_cuda_tv_iso_l1(ctx: Ctx, vol: torch.Tensor, steps: int, warmup: int) -> dict:
    """The reference's TV kernels driven as its op layer drives them
    (src/quantem/cuda/core/_ops.py:39-92, :187-228): per step the isotropic
    loss (zeroed accumulator, loss kernel, division by the corner count) and
    its gradient (upstream / corner count, zero-filled gradient, gradient
    kernel), then the L1 sums and their gradient."""
    core, why = reference_core()
    if core is None:
        return {"unavailable": why}
    b, d, h, w = vol.shape
    n = float(max(1, b * (d - 1) * (h - 1) * (w - 1)))
    dev = vol.device
    g1 = torch.ones(1, device=dev)
    g3 = torch.ones(3, device=dev)

    def step():
        st = torch.cuda.current_stream(dev).cuda_stream
        acc = torch.zeros(1, dtype=torch.float32, device=dev)
        core.tv_loss_iso_3d_cuda(vol.data_ptr(), acc.data_ptr(), b, d, h, w, 1e-8, st)
        _ = acc.squeeze(0) / n
        g_scaled = (g1.reshape(1) / n).contiguous()
        grad = torch.zeros_like(vol)
        core.tv_loss_iso_3d_grad_cuda(vol.data_ptr(), g_scaled.data_ptr(), grad.data_ptr(), b, d, h, w, 1e-8, st)
        acc3 = torch.zeros(3, dtype=torch.float32, device=dev)
        core.tv_loss_l1_3d_cuda(vol.data_ptr(), acc3.data_ptr(), b, d, h, w, st)
        grad3 = torch.empty_like(vol)
        core.tv_loss_l1_3d_grad_cuda(vol.data_ptr(), g3.data_ptr(), grad3.data_ptr(), b, d, h, w, st)

    ms = time_steps(ctx, step, steps, warmup)
    return {"value": vol.numel() / (ms / steps / 1e3), "unit": "voxels/s", "ms_per_step": ms / steps,
            "what": "the reference's sm_100a kernels (oracle/_ref/_core, built from its sources) through its "
                    "op layer's calls: iso loss + iso gradient + L1 sums + L1 gradient, 4 sweeps"}


def ref_cuda_kplanes(ctx: Ctx, p, r, g, u, steps: int, warmup: int) -> dict:
    """The reference's K-Planes kernels driven as its op layer drives them
    (src/quantem/cuda/core/ml/_ops.py:21-82): forward (channels-last copy of
    the planes, output, kernel) and backward (channels-last copy, zero-filled
    point, rotation and plane gradients, kernel, plane gradient permuted back
    to the parameter layout)."""
    core, why = reference_core()
    if core is None:
        return {"unavailable": why}
    N, T = p.shape[0], r.shape[0]
    C, H, W = g.shape[1:]
    dev = p.device

    def step():
        st = torch.cuda.current_stream(dev).cuda_stream
        gc = g.permute(0, 2, 3, 1).contiguous()
        out = torch.empty((N, T * C), dtype=torch.float32, device=dev)
        core.kplanes_tilted_fuse_cuda(p.data_ptr(), r.data_ptr(), gc.data_ptr(), out.data_ptr(), N, T, C, H, W, st)
        gc = g.permute(0, 2, 3, 1).contiguous()
        g_pts, g_r, g_cl = torch.zeros_like(p), torch.zeros_like(r), torch.zeros_like(gc)
        core.kplanes_tilted_fuse_grad_cuda(p.data_ptr(), r.data_ptr(), gc.data_ptr(), u.data_ptr(), g_cl.data_ptr(),
                                           g_r.data_ptr(), g_pts.data_ptr(), N, T, C, H, W, st)
        _ = g_cl.permute(0, 3, 1, 2).contiguous()

    ms = time_steps(ctx, step, steps, warmup)
    return {"value": N / (ms / steps / 1e3), "unit": "points/s", "ms_per_step": ms / steps,
            "what": "the reference's sm_100a kernels (oracle/_ref/_core, built from its sources) through its "
                    "op layer's calls: forward op + backward op"}


# ── workloads (ours) ────────────────────────────────────────────────────────


def run_tv_iso_l1(ctx: Ctx, steps: int, warmup: int) -> dict:
    from quantem.cuda import _core, sharded
    from quantem.cuda.core import tv_loss_iso_3d_fwd_grad, tv_loss_l1_3d_fwd_grad

    dev = ctx.device
    D_LOCAL = 256
    vol_cpu = tv_iso_l1_volume(1 + 1000 * ctx.rank, d=D_LOCAL)
    voxels_local = vol_cpu.numel()
    g1 = torch.ones(1, device=dev)
    g3 = torch.ones(3, device=dev)
    t_iso, t_l1 = KernelTimer(), KernelTimer()
    launches_per_step = 4  # two sweeps + two fixed-order finalize kernels

    if ctx.world == 1:
        vol = vol_cpu.to(dev)
        iso = t_iso.wrap(lambda v: tv_loss_iso_3d_fwd_grad(v, g1, eps=1e-8))
        l1 = t_l1.wrap(lambda v: tv_loss_l1_3d_fwd_grad(v, g3))

        def step():
            iso(vol)
            l1(vol)

    elif ctx.args.tv_transport == "peer":
        # halos and loss sums over peer memory: kernels only, no collective
        global_d = D_LOCAL * ctx.world
        ps = sharded.PeerSlab(4, global_d, 256, 256, device=dev)
        ps.owned.copy_(vol_cpu.to(dev))
        slab = ps.slab
        grads = [torch.empty_like(slab), torch.empty_like(slab)]
        # the iso sweep exchanges the halos itself, the L1 sweep reuses them,
        # and one finalize kernel sums both losses over the ranks
        terms = [(sharded.ISO, g1, 1e-8), (sharded.L1, g3, 0.0)]
        both = t_iso.wrap(lambda: ps.fwd_grad_many(terms, exchange=True, grads=grads))
        launches_per_step = 3  # two sweeps, one cross-rank finalize kernel

        def step():
            both()

    else:
        global_d = D_LOCAL * ctx.world
        slab = torch.zeros((4, D_LOCAL + 2, 256, 256), device=dev)
        slab[:, 1 : D_LOCAL + 1] = vol_cpu.to(dev)
        iso = t_iso.wrap(lambda: sharded.tv_loss_slab_fwd_grad(sharded.ISO, slab, g1, global_d, 1e-8, exchange=False))
        l1 = t_l1.wrap(lambda: sharded.tv_loss_slab_fwd_grad(sharded.L1, slab, g3, global_d, exchange=False))

        sharded.exchange_halos(slab)  # the neighbours' shapes are checked once, before the loop

        def step():
            sharded.exchange_halos(slab, check_shapes=False)
            iso()
            l1()

    sampler = ClockSampler(ctx.local_rank)
    ms = time_with_op_events(ctx, step, steps, warmup, (t_iso, t_l1), sampler)
    ms_step = ms / steps
    iso_ms = t_iso.mean_ms(steps)
    l1_ms = t_l1.mean_ms(steps) if t_l1.pairs else None
    if l1_ms is None:
        # both sweeps and their finalize in one timed call: report them per sweep
        dom_ms = iso_ms / 2
        dom = "tv iso + L1 sweeps with one cross-rank finalize (per sweep, per rank)"
    else:
        dom_ms = max(iso_ms, l1_ms)
        dom = "tv iso single sweep" if iso_ms >= l1_ms else "tv L1 single sweep"

    # Cross-rank pieces at N > 1: the same sweeps on this rank's slab with no
    # halo exchange and only a local finalize, timed alone; the difference to
    # the step is the exposed halo exchange + cross-rank finalize wait.
    breakdown = None
    if ctx.world > 1:
        from quantem.cuda._common import _workspace

        dp = slab.shape[1]
        has_prev, has_next = int(ctx.rank > 0), int(ctx.rank < ctx.world - 1)
        loc_grads = [torch.empty_like(slab), torch.empty_like(slab)]
        loc_acc = [torch.empty(1, device=dev), torch.empty(3, device=dev)]
        loc_ws = _workspace(dev)
        iso_scale = 1.0 / (4 * (global_d - 1) * 255 * 255)
        flags = sharded._LOSS | sharded._GRAD | sharded._OVERWRITE

        def local_step():
            st = torch.cuda.current_stream(dev).cuda_stream
            for (variant, g, eps, scale), acc, grad in zip(((sharded.ISO, g1, 1e-8, iso_scale), (sharded.L1, g3, 0.0, 1.0)),
                                                          loc_acc, loc_grads):
                _core.tv_loss_3d_slab_cuda(variant, flags, slab.data_ptr(), g.data_ptr(), acc.data_ptr(),
                                           grad.data_ptr(), 4, dp, 256, 256, 1, dp - 1, has_prev, has_next,
                                           eps, scale, loc_ws.data_ptr(), loc_ws.numel(), st)

        local_ms = time_steps(ctx, local_step, steps, min(warmup, 3)) / steps
        breakdown = {"step_ms": ms_step, "local_sweeps_ms": local_ms,
                     "exposed_halo_and_cross_rank_sum_ms": ms_step - local_ms,
                     "what": "local_sweeps_ms: both sweeps with a local finalize, no halo exchange and no "
                             "cross-rank wait (max over ranks)"}

    # end to end: the public API from pinned host memory. Each step copies its
    # volume (slab) in and reads both losses and both gradients back into
    # pinned host buffers, as the CPU computation leaves them in host memory.
    host = vol_cpu.pin_memory()
    res_host = torch.empty(4, pin_memory=True)
    grad_host = [torch.empty(vol_cpu.shape, pin_memory=True) for _ in range(2)]
    owned = (slice(None), slice(1, D_LOCAL + 1))

    def read_back(li, ls, gi, gl, sl=None):
        res_host[:1].copy_(li.reshape(1), non_blocking=True)
        res_host[1:].copy_(ls, non_blocking=True)
        grad_host[0].copy_(gi if sl is None else gi[sl], non_blocking=True)
        grad_host[1].copy_(gl if sl is None else gl[sl], non_blocking=True)

    if ctx.world == 1:
        def e2e_step(with_grads=True):
            v = host.to(dev, non_blocking=True)
            li, gi = tv_loss_iso_3d_fwd_grad(v, g1, eps=1e-8)
            ls, gl = tv_loss_l1_3d_fwd_grad(v, g3)
            if with_grads:
                read_back(li, ls, gi, gl)
            else:
                res_host[:1].copy_(li.reshape(1), non_blocking=True)
                res_host[1:].copy_(ls, non_blocking=True)
            torch.cuda.current_stream().synchronize()
    elif ctx.args.tv_transport == "peer":
        def e2e_step(with_grads=True):
            ps.owned.copy_(host, non_blocking=True)
            (li, gi), (ls, gl) = ps.fwd_grad_many(terms, exchange=True, grads=grads)
            if with_grads:
                read_back(li, ls, gi, gl, owned)
            else:
                res_host[:1].copy_(li.reshape(1), non_blocking=True)
                res_host[1:].copy_(ls, non_blocking=True)
            torch.cuda.current_stream().synchronize()
    else:
        def e2e_step(with_grads=True):
            slab[:, 1 : D_LOCAL + 1].copy_(host, non_blocking=True)
            sharded.exchange_halos(slab, check_shapes=False)
            li, gi = sharded.tv_loss_slab_fwd_grad(sharded.ISO, slab, g1, global_d, 1e-8, exchange=False)
            ls, gl = sharded.tv_loss_slab_fwd_grad(sharded.L1, slab, g3, global_d, exchange=False)
            if with_grads:
                read_back(li, ls, gi, gl, owned)
            else:
                res_host[:1].copy_(li.reshape(1), non_blocking=True)
                res_host[1:].copy_(ls, non_blocking=True)
            torch.cuda.current_stream().synchronize()

    e2e_ms = time_steps(ctx, e2e_step, steps, min(warmup, 3))
    e2e_losses_ms = time_steps(ctx, lambda: e2e_step(False), steps, min(warmup, 3))
    piped = None
    if ctx.world == 1:
        # The same public ops with the steps pipelined the way a caller that
        # streams volumes through the GPU would run them: step k+1's volume
        # comes in on one copy stream and step k's gradients go out on another
        # while step k computes (two device slots; every copy of every step is
        # still inside the timed region).
        s_in, s_out = torch.cuda.Stream(dev), torch.cuda.Stream(dev)
        comp = torch.cuda.current_stream(dev)
        slots = [torch.empty_like(vol) for _ in range(2)]
        ev_in = [torch.cuda.Event() for _ in range(2)]
        ev_comp = [torch.cuda.Event() for _ in range(2)]
        ev_out = [torch.cuda.Event() for _ in range(2)]
        out_host = [[torch.empty(4, pin_memory=True)] + [torch.empty(vol_cpu.shape, pin_memory=True)
                                                         for _ in range(2)] for _ in range(2)]
        used = [False, False]
        k_ = [0]

        def piped_step():
            i = k_[0] % 2
            if used[i]:
                s_in.wait_event(ev_comp[i])  # the slot's previous volume has been read
            with torch.cuda.stream(s_in):
                slots[i].copy_(host, non_blocking=True)
                ev_in[i].record(s_in)
            comp.wait_event(ev_in[i])
            if used[i]:
                comp.wait_event(ev_out[i])  # the slot's previous results have left
            li, gi = tv_loss_iso_3d_fwd_grad(slots[i], g1, eps=1e-8)
            ls, gl = tv_loss_l1_3d_fwd_grad(slots[i], g3)
            ev_comp[i].record(comp)
            s_out.wait_event(ev_comp[i])
            with torch.cuda.stream(s_out):
                res, hg_i, hg_l = out_host[i]
                res[:1].copy_(li.reshape(1), non_blocking=True)
                res[1:].copy_(ls, non_blocking=True)
                hg_i.copy_(gi, non_blocking=True)
                hg_l.copy_(gl, non_blocking=True)
                ev_out[i].record(s_out)
            for t_ in (li, ls, gi, gl):
                t_.record_stream(s_out)
            used[i] = True
            k_[0] += 1

        piped_ms = time_pipelined(ctx, piped_step, steps, min(warmup, 3), (s_in, s_out))
        piped = {"value": voxels_local / (piped_ms / steps / 1e3), "ms_per_step": piped_ms / steps,
                 "what": "the same copies and public ops, step k+1's volume in and step k's losses and "
                         "gradients out on two copy streams while step k computes"}
    ref_cuda = None
    one_sweep = None
    if ctx.world == 1:
        ref_cuda = ref_cuda_tv_iso_l1(ctx, vol, steps, warmup)
        # the same two losses and their summed gradient from one sweep
        # (tv_loss_multi_3d_fwd_grad), timed on its own: not the headline step
        from quantem.cuda.core import tv_loss_multi_3d_fwd_grad

        t_one = KernelTimer()
        both = t_one.wrap(lambda: tv_loss_multi_3d_fwd_grad(vol, iso=g1, l1=g3, eps=1e-8))
        one_ms = time_with_op_events(ctx, both, steps, warmup, (t_one,)) / steps
        peak_, _ = measured_hbm_peak()
        one_sweep = {"value": voxels_local / (one_ms / 1e3), "unit": "voxels/s", "ms_per_step": one_ms,
                     "op_ms": t_one.mean_ms(steps),
                     "roofline_frac": 8.0 * voxels_local / (t_one.mean_ms(steps) / 1e3) / 1e9 / peak_,
                     "what": "iso + L1 losses and their summed gradient in one sweep "
                             "(tv_loss_multi_3d_fwd_grad; 8 B/voxel for both terms)"}
    if ctx.world > 1 and ctx.args.tv_transport == "peer":
        ps.close()
    e2e = {
        "value": voxels_local * ctx.world / (e2e_ms / steps / 1e3),
        "unit": "voxels/s",
        "h2d_bytes_per_step": host.numel() * 4 * ctx.world,
        "d2h_bytes_per_step": (16 + 2 * host.numel() * 4) * ctx.world,
        "what": "volume copied in, both losses and both gradients copied back to pinned host memory, "
                "one step after the other",
        "losses_only": {"value": voxels_local * ctx.world / (e2e_losses_ms / steps / 1e3),
                        "d2h_bytes_per_step": 16 * ctx.world,
                        "what": "gradients left on the device, losses read back"},
        "pipelined": piped,
    }

    peak, peak_kind = measured_hbm_peak()
    algo_bytes = 8.0 * voxels_local  # single sweep: read 4 B + write 4 B per voxel
    achieved = algo_bytes / (dom_ms / 1e3) / 1e9
    tr = ncu_traffic("tv_iso_l1")
    return {
        "metric": "TV fwd+grad voxels/sec",
        "value": voxels_local * ctx.world / (ms_step / 1e3),
        "unit": "voxels/s",
        "ms_per_step": ms_step,
        "gpu_launches": launches_per_step * steps,
        "config": {
            "workload": DESCRIPTIONS["tv_iso_l1"],
            "shape_per_gpu": [4, D_LOCAL, 256, 256],
            "global_shape": [4, D_LOCAL * ctx.world, 256, 256],
            "parallelism": f"d-slab{ctx.world} ({ctx.args.tv_transport})" if ctx.world > 1 else "single GPU",
            "l2": "inputs larger than L2 (268 MB volume per GPU, 2 x 268 MB of gradients written per step)",
            "per_loss_ms": {"iso": iso_ms, "l1": l1_ms} if l1_ms is not None else {"iso_plus_l1": iso_ms},
            "per_loss_ms_how": "CUDA events around each op in a second pass of the K steps (events between "
                               "the ops of the timed pass would cost each sweep its overlap with the kernel "
                               "before it)",
        },
        "roofline": {
            "bound": "hbm",
            "kernel": dom,
            "achieved": achieved,
            "peak": peak,
            "peak_kind": f"{peak_kind} HBM copy bandwidth",
            "unit": "GB/s",
            "frac": achieved / peak,
            "traffic": None if tr is None else tr["bytes_per_unit"] * voxels_local,
            "algorithmic_bytes": algo_bytes,
        },
        "clocks": sampler.summary(),
        "e2e": e2e,
        "ref_cuda": ref_cuda,
        "one_sweep": one_sweep,
        "breakdown": breakdown,
        "dtype": "f32",
    }


def run_tv_multi(ctx: Ctx, steps: int, warmup: int) -> dict:
    """The tv_iso_l1 volume with both losses and their summed gradient from
    one sweep (tv_loss_multi_3d_fwd_grad): one GPU, one JSON line."""
    from quantem.cuda.core import tv_loss_multi_3d_fwd_grad

    if ctx.world > 1:
        raise SystemExit("tv_multi runs on one GPU")
    dev = ctx.device
    vol_cpu = tv_iso_l1_volume(1)
    vol = vol_cpu.to(dev)
    g1 = torch.ones(1, device=dev)
    g3 = torch.ones(3, device=dev)
    t = KernelTimer()
    both = t.wrap(lambda: tv_loss_multi_3d_fwd_grad(vol, iso=g1, l1=g3, eps=1e-8))
    sampler = ClockSampler(ctx.local_rank)
    ms = time_steps(ctx, both, steps, warmup, sampler)
    op_ms = t.mean_ms(steps)
    algo = 8.0 * vol.numel()
    peak, peak_kind = measured_hbm_peak()
    return {
        "metric": "TV fwd+grad voxels/sec",
        "value": vol.numel() / (ms / steps / 1e3),
        "unit": "voxels/s",
        "ms_per_step": ms / steps,
        "gpu_launches": 2 * steps,
        "config": {"workload": DESCRIPTIONS["tv_multi"], "shape_per_gpu": list(vol.shape),
                   "l2": "inputs larger than L2 (268 MB volume, 268 MB gradient per step)"},
        "roofline": {"bound": "hbm", "kernel": "tv iso + L1 mixed sweep (with its finalize)",
                     "achieved": algo / (op_ms / 1e3) / 1e9, "peak": peak,
                     "peak_kind": f"{peak_kind} HBM copy bandwidth", "unit": "GB/s",
                     "frac": algo / (op_ms / 1e3) / 1e9 / peak, "traffic": None, "algorithmic_bytes": algo},
        "clocks": sampler.summary(),
        "e2e": None,
        "dtype": "f32",
    }


def run_tv_sq_128(ctx: Ctx, steps: int, warmup: int) -> dict:
    from quantem.cuda.core import tv_loss_sq_3d_fwd_grad

    gen = torch.Generator().manual_seed(0)
    vol_cpu = torch.rand((128, 128, 128), generator=gen)
    vol = vol_cpu.to(ctx.device)
    g1 = torch.ones(1, device=ctx.device)
    flush = torch.empty(192 << 20, dtype=torch.uint8, device=ctx.device)  # > L2
    # The volume is 8 MiB: one call is a few microseconds of GPU work, less
    # than the host takes to dispatch the op, so the op is captured once in a
    # CUDA graph (sweep + finalize kernels) and replayed.
    for _ in range(3):
        tv_loss_sq_3d_fwd_grad(vol, g1)
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        loss_g, grad_g = tv_loss_sq_3d_fwd_grad(vol, g1)
    t = KernelTimer()
    sq = t.wrap(graph.replay)

    def step():
        flush.zero_()
        sq()

    sampler = ClockSampler(ctx.local_rank)
    ms = time_steps(ctx, step, steps, warmup, sampler)
    k_ms = t.mean_ms(steps)
    peak, peak_kind = measured_hbm_peak()
    algo = 8.0 * vol.numel()
    return {
        "metric": "TV fwd+grad voxels/sec",
        "value": vol.numel() * ctx.world / (k_ms / 1e3),
        "unit": "voxels/s",
        "ms_per_step": k_ms,
        "gpu_launches": 2 * steps,
        "config": {"workload": DESCRIPTIONS["tv_sq_128"],
                   "l2": "L2 flushed (192 MB write) between steps; value uses the op's event time",
                   "launch": "the op captured in a CUDA graph and replayed",
                   "step_ms_with_flush": ms / steps},
        "roofline": {"bound": "hbm", "kernel": "tv sq single sweep", "achieved": algo / (k_ms / 1e3) / 1e9,
                     "peak": peak, "peak_kind": f"{peak_kind} HBM copy bandwidth", "unit": "GB/s",
                     "frac": algo / (k_ms / 1e3) / 1e9 / peak, "traffic": None, "algorithmic_bytes": algo},
        "clocks": sampler.summary(),
        "e2e": None,
        "dtype": "f32",
    }


def run_tv_1024(ctx: Ctx, steps: int, warmup: int) -> dict:
    """The tomography-scale volume [1024, 1024, 1024]: sq + iso single-sweep
    fwd+grad. On N GPUs the volume is split along D into N slabs (strong
    scaling: the job's volume is fixed), halos and the two loss sums over
    peer memory."""
    from quantem.cuda import sharded
    from quantem.cuda.core import tv_loss_iso_3d_fwd_grad, tv_loss_sq_3d_fwd_grad

    n = 1024
    dev = ctx.device
    g1 = torch.ones(1, device=dev)
    t_sq, t_iso = KernelTimer(), KernelTimer()
    if ctx.world == 1:
        vol = blob_volume(n, 4, dev)
        sq = t_sq.wrap(lambda: tv_loss_sq_3d_fwd_grad(vol, g1))
        iso = t_iso.wrap(lambda: tv_loss_iso_3d_fwd_grad(vol, g1, eps=1e-8))

        def step():
            sq()
            iso()

        local_voxels = vol.numel()
        launches = 4
    else:
        ps = sharded.PeerSlab(1, n, n, n, device=dev)
        ps.owned.copy_(blob_volume(n, 4, dev, ps.d_lo, ps.d_hi).unsqueeze(0))
        grads = [torch.empty_like(ps.slab), torch.empty_like(ps.slab)]
        terms = [(sharded.SQ, g1, 0.0), (sharded.ISO, g1, 1e-8)]
        both = t_sq.wrap(lambda: ps.fwd_grad_many(terms, exchange=True, grads=grads))

        def step():
            both()

        local_voxels = (ps.d_hi - ps.d_lo) * n * n
        launches = 3
    sampler = ClockSampler(ctx.local_rank)
    ms = time_with_op_events(ctx, step, steps, warmup, (t_sq, t_iso), sampler)
    ms_step = ms / steps
    peak, peak_kind = measured_hbm_peak()
    one_sweep = None
    if ctx.world == 1:
        per_loss = {"sq": t_sq.mean_ms(steps), "iso": t_iso.mean_ms(steps)}
        dom_ms = max(per_loss.values())
        kernel = "tv single sweep (the slower of sq and iso)"
        # both terms and their summed gradient from one sweep
        from quantem.cuda.core import tv_loss_multi_3d_fwd_grad

        one_ms = time_steps(ctx, lambda: tv_loss_multi_3d_fwd_grad(vol, sq=g1, iso=g1, eps=1e-8), steps,
                            min(warmup, 3)) / steps
        one_sweep = {"value": n ** 3 / (one_ms / 1e3), "unit": "voxels/s", "ms_per_step": one_ms,
                     "roofline_frac": 8.0 * local_voxels / (one_ms / 1e3) / 1e9 / peak,
                     "what": "sq + iso losses and their summed gradient in one sweep (tv_loss_multi_3d_fwd_grad)"}
    else:
        per_loss = {"sq_plus_iso": t_sq.mean_ms(steps)}
        dom_ms = per_loss["sq_plus_iso"] / 2
        kernel = "tv sq + iso sweeps with one cross-rank finalize (per sweep, per rank)"
        ps.close()
    algo = 8.0 * local_voxels
    return {
        "metric": "TV fwd+grad voxels/sec",
        "value": n ** 3 / (ms_step / 1e3),
        "unit": "voxels/s",
        "ms_per_step": ms_step,
        "scaling": "strong" if ctx.world > 1 else "weak",
        "gpu_launches": launches * steps,
        "config": {"workload": DESCRIPTIONS["tv_1024"],
                   "global_shape": [n, n, n],
                   "parallelism": f"d-slab{ctx.world} (peer)" if ctx.world > 1 else "single GPU",
                   "l2": "inputs larger than L2 (4 GiB volume)",
                   "per_loss_ms": per_loss,
                   "one_sweep": one_sweep},
        "roofline": {"bound": "hbm", "kernel": kernel, "achieved": algo / (dom_ms / 1e3) / 1e9,
                     "peak": peak, "peak_kind": f"{peak_kind} HBM copy bandwidth", "unit": "GB/s",
                     "frac": algo / (dom_ms / 1e3) / 1e9 / peak, "traffic": None, "algorithmic_bytes": algo},
        "clocks": sampler.summary(),
        "e2e": None,
        "dtype": "f32",
    }


def kplanes_ms_inputs(world: int, rank: int, device):
    """The multiscale configuration: 4 levels at 64/128/256/512, N = 2^24
    points U[-1, 1]^3 (this rank's contiguous share), R = 8 rotations from
    normalised N(0,1) quaternions, C = 32, planes U[0.1, 0.5], upstream
    gradient N(0, 1) per level (drawn on the device from a seeded generator:
    17 GB per level at one GPU)."""
    from quantem.cuda import sharded

    n_total, T, C = 1 << 24, 8, 32
    gen = torch.Generator().manual_seed(3)
    pts = torch.empty((n_total, 3)).uniform_(-1.0, 1.0, generator=gen)
    rot = quaternion_rotations(T, gen)
    planes = [torch.empty((3 * T, C, r, r)).uniform_(0.1, 0.5, generator=gen) for r in (64, 128, 256, 512)]
    lo, hi = sharded.slab_bounds(n_total, rank, world)
    p = pts[lo:hi].to(device)
    gd = torch.Generator(device=device).manual_seed(3 + rank)
    ups = [torch.randn((hi - lo, T * C), device=device, generator=gd) for _ in planes]
    return p, rot.to(device), [g.to(device) for g in planes], ups, n_total


def run_kplanes_ms(ctx: Ctx, steps: int, warmup: int) -> dict:
    """Multiscale K-Planes fwd+bwd over 4 levels, N = 2^24 points split over
    the ranks (strong scaling), plane and rotation gradients of each level
    summed over the ranks over peer memory right after its backward."""
    from quantem.cuda import sharded

    dev = ctx.device
    p, r, planes, ups, n_total = kplanes_ms_inputs(ctx.world, ctx.rank, dev)
    T, C = r.shape[0], planes[0].shape[1]
    reducers = [sharded.kplanes_gradient_reducer(g, r) for g in planes] if ctx.world > 1 else None
    timers = [KernelTimer() for _ in planes]

    def level(k):
        if ctx.world > 1:
            return sharded.kplanes_fwd_bwd_sharded(p, r, planes[k], ups[k], reducer=reducers[k])
        out = torch.ops.quantem_cuda.kplanes_tilted_fuse(p, r, planes[k])
        grads = torch.ops.quantem_cuda.kplanes_tilted_fuse_bwd(p, r, planes[k], ups[k])
        return out, grads

    runs = [t.wrap(lambda k=k: level(k)) for k, t in enumerate(timers)]

    def step():
        for run in runs:
            run()  # each level's output and gradients are released before the next

    sampler = ClockSampler(ctx.local_rank)
    ms = time_with_op_events(ctx, step, steps, warmup, timers, sampler)
    ms_step = ms / steps
    if reducers is not None:
        for red in reducers:
            red.close()
    one_launch = None
    if ctx.world == 1:
        # all four levels in one launch per pass (kplanes_tilted_fuse_levels),
        # the same work as the per-level loop above
        torch.cuda.empty_cache()

        def levels_step():
            outs = torch.ops.quantem_cuda.kplanes_tilted_fuse_levels(p, r, planes)
            grads = torch.ops.quantem_cuda.kplanes_tilted_fuse_levels_bwd(p, r, planes, ups)
            return outs, grads

        try:
            lv_ms = time_steps(ctx, lambda: levels_step() and None, steps, min(warmup, 3)) / steps
            one_launch = {"value": n_total / (lv_ms / 1e3), "ms_per_step": lv_ms,
                          "what": "kplanes_tilted_fuse_levels forward + backward: all four levels in one launch "
                                  "per pass (all four outputs alive at once)"}
        except torch.OutOfMemoryError as e:  # four 17 GB outputs at once
            one_launch = {"unavailable": f"out of device memory: {str(e).splitlines()[0]}"}
        torch.cuda.empty_cache()
    n_local = p.shape[0]
    P = [g.numel() * 4 for g in planes]
    # per rank: out + upstream (2·4·N·R·C) + points (12 N fwd, 12 N bwd, 12 N gpts)
    # per level, plus plane, plane gradient read-modify-write (3 P) per level
    algo = sum(2 * 4 * n_local * T * C + 36 * n_local + 3 * pl for pl in P)
    peak, peak_kind = measured_hbm_peak()
    lvl_ms = [t.mean_ms(steps) for t in timers]
    return {
        "metric": "K-Planes fwd+bwd points/sec",
        "value": n_total / (ms_step / 1e3),
        "unit": "points/s",
        "ms_per_step": ms_step,
        "scaling": "strong" if ctx.world > 1 else "weak",
        "gpu_launches": (5 if ctx.world == 1 else 6) * len(planes) * steps,
        "config": {"workload": DESCRIPTIONS["kplanes_ms"],
                   "points_per_gpu": n_local,
                   "parallelism": f"points{ctx.world} (gradient sum: peer)" if ctx.world > 1 else "single GPU",
                   "l2": "inputs larger than L2 (17 GB output + 17 GB upstream gradient per level at 1 GPU)",
                   "level_ms": dict(zip(("64", "128", "256", "512"), lvl_ms)),
                   "one_launch_all_levels": one_launch},
        "roofline": {"bound": "hbm", "kernel": "all four levels' fwd+bwd (per rank, step)",
                     "achieved": algo / (ms_step / 1e3) / 1e9, "peak": peak,
                     "peak_kind": f"{peak_kind} HBM copy bandwidth", "unit": "GB/s",
                     "frac": algo / (ms_step / 1e3) / 1e9 / peak, "traffic": None,
                     "algorithmic_bytes": algo},
        "clocks": sampler.summary(),
        "e2e": None,
        "dtype": "f32",
    }


def run_kplanes(ctx: Ctx, steps: int, warmup: int) -> dict:
    from quantem.cuda import sharded
    from quantem.cuda.core.ml import kplanes_tilted_fuse

    pts, rot, plane, up = kplanes_inputs(2 + 1000 * ctx.rank)
    dev = ctx.device
    N, T, C = pts.shape[0], rot.shape[0], plane.shape[1]
    p, r, g, u = pts.to(dev), rot.to(dev), plane.to(dev), up.to(dev)
    t_f, t_b = KernelTimer(), KernelTimer()
    fwd = t_f.wrap(lambda: torch.ops.quantem_cuda.kplanes_tilted_fuse(p, r, g))
    bwd = t_b.wrap(lambda: torch.ops.quantem_cuda.kplanes_tilted_fuse_bwd(p, r, g, u))

    if ctx.world == 1:
        def step():
            fwd()
            bwd()
    else:
        # one channels-last copy of the planes for both passes, one backward
        # launch, then the plane- and rotation-gradient sum over the ranks:
        # by default one kernel over peer memory (deterministic, rank order);
        # --kp-reduce nccl uses NCCL all_reduce; --kp-buckets > 1 overlaps
        # each bucket's gradient sum (peer kernel of at most --kp-reduce-ctas
        # CTAs on a second stream, or NCCL) with the next bucket's backward
        if ctx.args.kp_reduce == "peer":
            reducer = sharded.kplanes_gradient_reducer(g, r)
            fb = t_b.wrap(lambda: sharded.kplanes_fwd_bwd_sharded(p, r, g, u, reducer=reducer,
                                                                  buckets=ctx.args.kp_buckets,
                                                                  reduce_ctas=ctx.args.kp_reduce_ctas))
        else:
            fb = t_b.wrap(lambda: sharded.kplanes_fwd_bwd_sharded(p, r, g, u, buckets=ctx.args.kp_buckets))

        def step():
            fb()

    sampler = ClockSampler(ctx.local_rank)
    ms = time_with_op_events(ctx, step, steps, warmup, (t_f, t_b), sampler)
    ms_step = ms / steps
    f_ms, b_ms = t_f.mean_ms(steps), t_b.mean_ms(steps)
    if ctx.world > 1:
        f_ms = None  # b_ms covers the whole sharded forward + backward
    P = 3 * T * C * plane.shape[2] * plane.shape[3] * 4
    fwd_bytes = 12 * N + P + 4 * N * T * C
    bwd_bytes = 12 * N + 4 * N * T * C + P + P + 12 * N
    peak, peak_kind = measured_hbm_peak()
    roof_bytes = bwd_bytes if ctx.world == 1 else fwd_bytes + bwd_bytes
    tr = ncu_traffic("kplanes")
    kp_traffic = None if tr is None else tr["bytes_per_unit"] * N

    # Cross-rank piece at N > 1: this rank's forward and backward ops with no
    # gradient sum, timed alone; the difference to the step is the exposed
    # sum of the plane and rotation gradients over the ranks.
    breakdown = None
    if ctx.world > 1:
        def local_step():
            torch.ops.quantem_cuda.kplanes_tilted_fuse(p, r, g)
            torch.ops.quantem_cuda.kplanes_tilted_fuse_bwd(p, r, g, u)

        local_ms = time_steps(ctx, local_step, steps, min(warmup, 3)) / steps
        breakdown = {"step_ms": ms_step, "local_fwd_bwd_ms": local_ms,
                     "exposed_gradient_sum_ms": ms_step - local_ms,
                     "what": "local_fwd_bwd_ms: forward + backward ops on this rank's points with no gradient "
                             "sum (max over ranks)"}

    # End to end through the public API from pinned host memory: each step
    # copies its inputs in and reads the output and every gradient back into
    # pinned host buffers, as the CPU computation leaves them in host memory.
    e2e = None
    ref_cuda = None
    l2_ceiling = None
    if ctx.world == 1:
        hp, hr, hg, hu = (t.pin_memory() for t in (pts, rot, plane, up))
        out_host = torch.empty((N, T * C), pin_memory=True)
        gh = [torch.empty(t.shape, pin_memory=True) for t in (pts, rot, plane)]

        def e2e_step():
            pp = hp.to(dev, non_blocking=True).requires_grad_(True)
            rr = hr.to(dev, non_blocking=True).requires_grad_(True)
            gg = hg.to(dev, non_blocking=True).requires_grad_(True)
            uu = hu.to(dev, non_blocking=True)
            out = kplanes_tilted_fuse(pp, rr, gg)
            out.backward(uu)
            out_host.copy_(out.detach(), non_blocking=True)
            for h_, t_ in zip(gh, (pp, rr, gg)):
                h_.copy_(t_.grad, non_blocking=True)
            torch.cuda.current_stream().synchronize()

        e2e_ms = time_steps(ctx, e2e_step, steps, min(warmup, 3))

        # the same steps pipelined: step k+1's inputs in on one copy stream and
        # step k's output and gradients out on another while step k computes
        s_in, s_out = torch.cuda.Stream(dev), torch.cuda.Stream(dev)
        comp = torch.cuda.current_stream(dev)
        slots = [[torch.empty(t.shape, device=dev) for t in (pts, rot, plane, up)] for _ in range(2)]
        hosts = [[torch.empty((N, T * C), pin_memory=True)] + [torch.empty(t.shape, pin_memory=True)
                                                              for t in (pts, rot, plane)] for _ in range(2)]
        ev_in = [torch.cuda.Event() for _ in range(2)]
        ev_comp = [torch.cuda.Event() for _ in range(2)]
        ev_out = [torch.cuda.Event() for _ in range(2)]
        used = [False, False]
        k_ = [0]

        def piped_step():
            i = k_[0] % 2
            if used[i]:
                s_in.wait_event(ev_comp[i])
            with torch.cuda.stream(s_in):
                for d_, h_ in zip(slots[i], (hp, hr, hg, hu)):
                    d_.copy_(h_, non_blocking=True)
                ev_in[i].record(s_in)
            comp.wait_event(ev_in[i])
            if used[i]:
                comp.wait_event(ev_out[i])
            pp, rr, gg = (t.detach().requires_grad_(True) for t in slots[i][:3])
            out = kplanes_tilted_fuse(pp, rr, gg)
            out.backward(slots[i][3])
            ev_comp[i].record(comp)
            s_out.wait_event(ev_comp[i])
            results = (out.detach(), pp.grad, rr.grad, gg.grad)
            with torch.cuda.stream(s_out):
                for h_, t_ in zip(hosts[i], results):
                    h_.copy_(t_, non_blocking=True)
                ev_out[i].record(s_out)
            for t_ in results:
                t_.record_stream(s_out)
            used[i] = True
            k_[0] += 1

        piped_ms = time_pipelined(ctx, piped_step, steps, min(warmup, 3), (s_in, s_out))
        e2e = {"value": N / (e2e_ms / steps / 1e3), "unit": "points/s",
               "h2d_bytes_per_step": sum(t.numel() * 4 for t in (hp, hr, hg, hu)),
               "d2h_bytes_per_step": (out_host.numel() + sum(t.numel() for t in gh)) * 4,
               "what": "points, rotations, planes and upstream gradient copied in; output and the point, "
                       "rotation and plane gradients copied back to pinned host memory, one step after "
                       "the other",
               "pipelined": {"value": N / (piped_ms / steps / 1e3), "ms_per_step": piped_ms / steps,
                             "what": "the same copies and public ops, step k+1's inputs in and step k's "
                                     "results out on two copy streams while step k computes"}}
        ref_cuda = ref_cuda_kplanes(ctx, p, r, g, u, steps, warmup)
        l2_ceiling = kplanes_l2_ceiling(p, r, g, u)
    else:
        # each rank brings its points and upstream gradient in from pinned host
        # memory (planes and rotations are parameters resident on the device)
        # and reads its output, its point gradient and the summed rotation and
        # plane gradients back
        hp, hu = pts.pin_memory(), up.pin_memory()
        out_host = torch.empty((N, T * C), pin_memory=True)
        gp_host = torch.empty((N, 3), pin_memory=True)
        gr_host = torch.empty(T * 9, pin_memory=True)
        gg_host = torch.empty(plane.shape, pin_memory=True)

        def e2e_step():
            pp = hp.to(dev, non_blocking=True)
            uu = hu.to(dev, non_blocking=True)
            if ctx.args.kp_reduce == "peer":
                out, g_pts, g_rot, g_plane, _ = sharded.kplanes_fwd_bwd_sharded(
                    pp, r, g, uu, reducer=reducer, buckets=ctx.args.kp_buckets,
                    reduce_ctas=ctx.args.kp_reduce_ctas)
            else:
                out, g_pts, g_rot, g_plane, _ = sharded.kplanes_fwd_bwd_sharded(pp, r, g, uu,
                                                                              buckets=ctx.args.kp_buckets)
            out_host.copy_(out, non_blocking=True)
            gp_host.copy_(g_pts, non_blocking=True)
            gr_host.copy_(g_rot.reshape(-1), non_blocking=True)
            gg_host.copy_(g_plane, non_blocking=True)
            torch.cuda.current_stream().synchronize()

        e2e_ms = time_steps(ctx, e2e_step, steps, min(warmup, 3))
        e2e = {"value": N * ctx.world / (e2e_ms / steps / 1e3), "unit": "points/s",
               "h2d_bytes_per_step": (hp.numel() + hu.numel()) * 4 * ctx.world,
               "d2h_bytes_per_step": (out_host.numel() + gp_host.numel() + gr_host.numel() + gg_host.numel())
               * 4 * ctx.world,
               "what": "each rank's points and upstream gradient copied in; its output, point gradient and the "
                       "summed rotation and plane gradients copied back to pinned host memory"}
    if ctx.world > 1 and ctx.args.kp_reduce == "peer":
        reducer.close()

    return {
        "metric": "K-Planes fwd+bwd points/sec",
        "value": N * ctx.world / (ms_step / 1e3),
        "unit": "points/s",
        "ms_per_step": ms_step,
        "gpu_launches": (5 if ctx.world == 1 else
                         (3 if ctx.args.kp_reduce == "peer" else 2) + 2 * min(max(ctx.args.kp_buckets, 1), T)) * steps,
        "config": {"workload": DESCRIPTIONS["kplanes"],
                   "points_per_gpu": N,
                   "parallelism": (f"points{ctx.world} (gradient sum: {ctx.args.kp_reduce}"
                                   + f", buckets {ctx.args.kp_buckets}"
                                   + (f", reduce CTAs {ctx.args.kp_reduce_ctas})"
                                      if ctx.args.kp_reduce == "peer" and ctx.args.kp_buckets > 1 else ")"))
                   if ctx.world > 1 else "single GPU",
                   "l2": "inputs larger than L2 (512 MiB output + 512 MiB upstream gradient per step)",
                   "fwd_op_ms": f_ms, "bwd_op_ms": b_ms},
        "roofline": {"bound": "hbm",
                     "kernel": "kplanes backward op" if ctx.world == 1 else "kplanes sharded fwd+bwd (per rank)",
                     "achieved": roof_bytes / (b_ms / 1e3) / 1e9, "peak": peak,
                     "peak_kind": f"{peak_kind} HBM copy bandwidth", "unit": "GB/s",
                     "frac": roof_bytes / (b_ms / 1e3) / 1e9 / peak,
                     "traffic": kp_traffic if ctx.world == 1 else None,
                     "algorithmic_bytes": roof_bytes, "step_algorithmic_bytes": fwd_bytes + bwd_bytes,
                     "step_frac": (fwd_bytes + bwd_bytes) / (ms_step / 1e3) / 1e9 / peak},
        "clocks": sampler.summary(),
        "e2e": e2e,
        "ref_cuda": ref_cuda,
        "l2_ceiling": l2_ceiling,
        "breakdown": breakdown,
        "dtype": "f32",
    }


def kplanes_l2_ceiling(p, r, g, u, reps: int = 10) -> dict:
    """The forward and backward kernels (C ABI, no op-layer work) against
    kplanes_l2_probe_cuda, which replays their memory traffic at C = 32
    without arithmetic: 12 corner rows of 128 B gathered per (point,
    rotation), plus a vector reduction per corner in the backward. The
    probe's time is the L2-side ceiling of the access pattern."""
    from quantem.cuda import _core

    N, T = p.shape[0], r.shape[0]
    C, H, W = g.shape[1:]
    if C != 32:
        return {"unavailable": "the probe replays C = 32"}
    dev = p.device
    st = torch.cuda.current_stream(dev).cuda_stream
    pairs = N * T
    planes = torch.rand((3, H, W, C), device=dev)
    pgrad = torch.zeros_like(planes)
    out = torch.empty((N, T * C), device=dev)
    gpts = torch.zeros((N, 3), device=dev)
    sink = torch.empty(int(_core.kplanes_l2_probe_sink_floats()), device=dev)
    grid_cl = g.permute(0, 2, 3, 1).contiguous()
    gg, gr = torch.zeros_like(grid_cl), torch.zeros_like(r)

    def timed(fn) -> float:
        for _ in range(3):
            fn()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        torch.cuda.synchronize()
        a.record()
        for _ in range(reps):
            fn()
        b.record()
        torch.cuda.synchronize()
        return a.elapsed_time(b) / reps

    def probe(mode):
        return lambda: _core.kplanes_l2_probe_cuda(mode, planes.data_ptr(), pgrad.data_ptr(), u.data_ptr(),
                                                   out.data_ptr(), gpts.data_ptr(), sink.data_ptr(), pairs, N,
                                                   H, W, st)

    res = {m: timed(probe(getattr(_core, f"KP_PROBE_{m.upper()}"))) for m in ("gather", "reduce", "backward",
                                                                             "forward")}
    fwd_ms = timed(lambda: _core.kplanes_tilted_fuse_cuda(p.data_ptr(), r.data_ptr(), grid_cl.data_ptr(),
                                                          out.data_ptr(), N, T, C, H, W, st))
    bwd_ms = timed(lambda: _core.kplanes_tilted_fuse_grad_cuda(p.data_ptr(), r.data_ptr(), grid_cl.data_ptr(),
                                                               u.data_ptr(), gg.data_ptr(), gr.data_ptr(),
                                                               gpts.data_ptr(), N, T, C, H, W, st))
    lines = 12.0 * pairs * 128
    return {
        "what": "kernels (C ABI) against kplanes_l2_probe_cuda, their memory traffic without arithmetic "
                "(hashed cells, 8 lanes x float4 per pair); traffic_ms / kernel_ms = fraction of the ceiling",
        "fwd_kernel_ms": fwd_ms, "fwd_traffic_ms": res["forward"], "fwd_frac": res["forward"] / fwd_ms,
        "bwd_kernel_ms": bwd_ms, "bwd_traffic_ms": res["backward"], "bwd_frac": res["backward"] / bwd_ms,
        "gather_only_ms": res["gather"], "reduce_only_ms": res["reduce"],
        "l2_gather_GBps": lines / (res["gather"] / 1e3) / 1e9,
        "l2_reduce_GBps": lines / (res["reduce"] / 1e3) / 1e9,
    }


# ── the reference's own benchmark configurations ──────────────────────────


def _ref_suite_time(fn, iters: int, warmup: int) -> float:
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    for _ in range(iters):
        fn()
    b.record()
    torch.cuda.synchronize()
    return a.elapsed_time(b) / iters


def _ray_points(n: int, dev, gen, samples_per_ray: int = 200) -> torch.Tensor:
    """Points laid out like a tomography ray sampler: consecutive entries are
    consecutive samples along one ray (a random (x, y), z from -1 to 1)."""
    n_rays = n // samples_per_ray
    xy = (torch.rand((n_rays, 1, 2), generator=gen) * 2 - 1).to(dev)
    z = torch.linspace(-1, 1, samples_per_ray, device=dev).view(1, -1, 1)
    return torch.cat([xy.expand(-1, samples_per_ray, -1), z.expand(n_rays, -1, -1)], dim=-1).reshape(-1, 3)


def run_reference_suite(ctx: Ctx, steps: int, warmup: int) -> dict:
    """The configurations of the reference's own benchmarks
    (benchmarks/core/bench_tv_loss.py: 4 shapes x iso/sq/L1 x fwd, fwd+bwd
    through the public ops and autograd; benchmarks/core/ml/bench_kplanes_tilted.py:
    3 point sets, two of them ray-structured, x fwd, fwd+bwd), timed for this
    build's public ops, for the reference's own sm_100a kernels driven with its
    op layer's calls (no autograd around them), and for the pure-torch chains
    the reference benchmarks compare against. Seeded synthetic inputs."""
    from quantem.cuda.core import tv_loss_iso_3d, tv_loss_l1_3d, tv_loss_sq_3d
    from quantem.cuda.core.ml import kplanes_tilted_fuse
    from oracle import torch_ref

    if ctx.world > 1:
        raise SystemExit("reference_suite runs on one GPU")
    dev = ctx.device
    core, why = reference_core()
    iters = max(steps, 5)
    gen = torch.Generator().manual_seed(5)
    rows = []

    def l1_mean(sums, shape):
        d, h, w = shape[-3:]
        n = int(np.prod(shape)) // (d * h * w)
        counts = sums.new_tensor([n * (d - 1) * h * w, n * d * (h - 1) * w, n * d * h * (w - 1)])
        return (sums / counts).sum() / 3

    def torch_l1(v):
        v4 = v.reshape(-1, *v.shape[-3:])
        return sum(torch.mean(torch.abs(v4.diff(dim=d))) for d in (1, 2, 3)) / 3

    for shape in ((16, 1024, 1024), (256, 256, 256), (4, 256, 256, 256), (512, 512, 512)):
        vol = torch.rand(shape, generator=gen).to(dev)
        v4 = vol.reshape(-1, *shape[-3:])
        b, d, h, w = v4.shape
        n_iso = float(max(1, b * (d - 1) * (h - 1) * (w - 1)))
        ours = {"iso": lambda v: tv_loss_iso_3d(v, 1e-8), "squared": tv_loss_sq_3d,
                "L1": lambda v: l1_mean(tv_loss_l1_3d(v), shape)}
        torchs = {"iso": lambda v: torch_ref.tv_iso(v, 1e-8), "squared": torch_ref.tv_sq, "L1": torch_l1}
        for name in ("iso", "squared", "L1"):
            for backward in (False, True):
                def mk(fn):
                    def run():
                        v = vol.detach().requires_grad_(backward)
                        loss = fn(v)
                        if backward:
                            loss.backward()
                    return run

                t_ours = _ref_suite_time(mk(ours[name]), iters, warmup)
                t_torch = _ref_suite_time(mk(torchs[name]), iters, warmup)
                t_ref = None
                if core is not None:
                    st = torch.cuda.current_stream(dev).cuda_stream

                    def ref_run():
                        if name == "iso":
                            acc = torch.zeros(1, device=dev)
                            core.tv_loss_iso_3d_cuda(v4.data_ptr(), acc.data_ptr(), b, d, h, w, 1e-8, st)
                            _ = acc.squeeze(0) / n_iso
                            if backward:
                                g = (torch.ones(1, device=dev) / n_iso).contiguous()
                                gv = torch.zeros_like(v4)
                                core.tv_loss_iso_3d_grad_cuda(v4.data_ptr(), g.data_ptr(), gv.data_ptr(), b, d, h, w,
                                                              1e-8, st)
                        elif name == "squared":
                            acc = torch.zeros(1, device=dev)
                            core.tv_loss_sq_3d_cuda(v4.data_ptr(), acc.data_ptr(), b, d, h, w, st)
                            if backward:
                                g = torch.ones(1, device=dev)
                                gv = torch.empty_like(v4)
                                core.tv_loss_sq_3d_grad_cuda(v4.data_ptr(), g.data_ptr(), gv.data_ptr(), b, d, h, w,
                                                             st)
                        else:
                            acc = torch.zeros(3, device=dev)
                            core.tv_loss_l1_3d_cuda(v4.data_ptr(), acc.data_ptr(), b, d, h, w, st)
                            _ = l1_mean(acc, shape)
                            if backward:
                                g = torch.ones(3, device=dev)
                                gv = torch.empty_like(v4)
                                core.tv_loss_l1_3d_grad_cuda(v4.data_ptr(), g.data_ptr(), gv.data_ptr(), b, d, h, w,
                                                             st)

                    t_ref = _ref_suite_time(ref_run, iters, warmup)
                rows.append({"bench": "tv", "config": str(shape), "op": name,
                             "pass": "fwd+bwd" if backward else "fwd", "ours_ms": t_ours,
                             "reference_kernels_ms": t_ref, "torch_ms": t_torch})
        del vol, v4

    kp_configs = (("light (8192x200 rays, T=4, C=8, 200^2)", 8192 * 200, 4, 8, 200, True),
                  ("heavy (8192x200 rays, T=8, C=32, 200^2)", 8192 * 200, 8, 32, 200, True),
                  ("decode (5*200^2 pts, T=4, C=8, 200^2)", 5 * 200 * 200, 4, 8, 200, False))
    for label, n, t, c, res, rays in kp_configs:
        pts = _ray_points(n, dev, gen) if rays else (torch.rand((n, 3), generator=gen) * 2 - 1).to(dev)
        rot = torch.randn((t, 3, 3), generator=gen).to(dev)
        plane = torch.empty((3 * t, c, res, res)).uniform_(0.1, 0.5, generator=gen).to(dev)
        up = torch.randn((n, t * c), generator=gen).to(dev)
        leaves = [x.detach().requires_grad_(True) for x in (pts, rot, plane)]
        for backward in (False, True):
            def mk(fn):
                def run():
                    out = fn(*leaves)
                    if backward:
                        (out * up).sum().backward()
                        for x in leaves:
                            x.grad = None
                return run

            t_ours = _ref_suite_time(mk(kplanes_tilted_fuse), iters, warmup)
            t_torch = _ref_suite_time(mk(torch_ref.kplanes_tilted), max(3, iters // 4), 2)
            t_ref = None
            if core is not None:
                st = torch.cuda.current_stream(dev).cuda_stream

                def ref_run():
                    gc = plane.permute(0, 2, 3, 1).contiguous()
                    out = torch.empty((n, t * c), device=dev)
                    core.kplanes_tilted_fuse_cuda(pts.data_ptr(), rot.data_ptr(), gc.data_ptr(), out.data_ptr(),
                                                  n, t, c, res, res, st)
                    if backward:
                        # the benchmark's loss (out * upstream).sum() and the
                        # gradient autograd hands the op's backward
                        _ = (out * up).sum()
                        gout = (up * 1.0).contiguous()
                        gc2 = plane.permute(0, 2, 3, 1).contiguous()
                        gp, gr, gg = torch.zeros_like(pts), torch.zeros_like(rot), torch.zeros_like(gc2)
                        core.kplanes_tilted_fuse_grad_cuda(pts.data_ptr(), rot.data_ptr(), gc2.data_ptr(),
                                                           gout.data_ptr(), gg.data_ptr(), gr.data_ptr(),
                                                           gp.data_ptr(), n, t, c, res, res, st)
                        _ = gg.permute(0, 3, 1, 2).contiguous()

                t_ref = _ref_suite_time(ref_run, iters, warmup)
            rows.append({"bench": "kplanes", "config": label, "op": "kplanes_tilted_fuse",
                         "pass": "fwd+bwd" if backward else "fwd", "ours_ms": t_ours,
                         "reference_kernels_ms": t_ref, "torch_ms": t_torch})

    def gmean(xs):
        xs = [x for x in xs if x]
        return float(np.exp(np.mean(np.log(xs)))) if xs else None

    for r in rows:
        r["ours_over_reference"] = None if r["reference_kernels_ms"] is None else r["reference_kernels_ms"] / r["ours_ms"]
        r["ours_over_torch"] = r["torch_ms"] / r["ours_ms"]
    vs_ref = gmean([r["ours_over_reference"] for r in rows])
    return {
        "metric": "speed-up over the reference's own kernels on its benchmark configurations (geometric mean)",
        "value": vs_ref,
        "unit": "x",
        "ms_per_step": sum(r["ours_ms"] for r in rows),
        "gpu_launches": None,
        "config": {"workload": DESCRIPTIONS["reference_suite"],
                   "reference_kernels": "oracle/_ref/_core" if core is not None else why,
                   "geomean_over_torch": gmean([r["ours_over_torch"] for r in rows]),
                   "geomean_over_reference_tv": gmean([r["ours_over_reference"] for r in rows if r["bench"] == "tv"]),
                   "geomean_over_reference_kplanes": gmean([r["ours_over_reference"] for r in rows
                                                            if r["bench"] == "kplanes"])},
        "rows": rows,
        "roofline": None,
        "clocks": None,
        "e2e": None,
        "dtype": "f32",
    }


DESCRIPTIONS = {
    "tv_iso_l1": "tv_iso_l1: tv_loss_iso_3d (eps 1e-8) + tv_loss_l1_3d single-sweep fwd+grad",
    "tv_sq_128": "tv_sq_128: tv_loss_sq_3d single-sweep fwd+grad on [128,128,128]",
    "reference_suite": "reference_suite: the reference's benchmark configurations (bench_tv_loss.py, "
                       "bench_kplanes_tilted.py) for this build, the reference's kernels and pure torch",
    "tv_multi": "tv_multi: tv_loss_iso_3d (eps 1e-8) + tv_loss_l1_3d losses and summed gradient in one sweep "
                "(tv_loss_multi_3d_fwd_grad) on the tv_iso_l1 volume",
    "tv_1024": "tv_1024: tv_loss_sq_3d + tv_loss_iso_3d single-sweep fwd+grad on [1024]^3 blobs",
    "kplanes": "kplanes: kplanes_tilted_fuse fwd + bwd ops, N=2^20, T=4, C=32, 256^2",
    "kplanes_ms": "kplanes_ms: multiscale kplanes_tilted_fuse fwd + bwd, 4 levels 64/128/256/512, N=2^24, T=8, C=32",
}

WORKLOADS = {
    "tv_iso_l1": run_tv_iso_l1,
    "tv_sq_128": run_tv_sq_128,
    "tv_multi": run_tv_multi,
    "reference_suite": run_reference_suite,
    "tv_1024": run_tv_1024,
    "kplanes": run_kplanes,
    "kplanes_ms": run_kplanes_ms,
}


# ── reference arm: the reference computation on the host cores ──────────────


def run_reference(ctx: Ctx, args) -> dict | None:
    if ctx.rank != 0:
        return None
    warmup = max(args.warmup, 3)
    cb, per_step = CPU_BASELINES[args.workload](reps=args.steps, warmup=warmup)
    metric = "K-Planes fwd+bwd points/sec" if args.workload.startswith("kplanes") else "TV fwd+grad voxels/sec"
    res = {
        "metric": metric,
        "value": cb["value"],
        "unit": cb["unit"],
        "impl": "reference",
        "ms_per_step": per_step * 1e3,
        "config": {"workload": DESCRIPTIONS[args.workload], "sample": cb["sample"]},
        "cpu_baseline": cb,
        "e2e": {"value": cb["value"], "unit": cb["unit"], "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "dtype": "f32",
    }
    if args.workload == "tv_iso_l1" and not args.no_kplanes:
        # the other half of the metric, as in our arm's line
        kb, kstep = cpu_kplanes(reps=max(1, args.steps // 4), warmup=1)
        res["kplanes"] = {"metric": "K-Planes fwd+bwd points/sec", "value": kb["value"], "unit": kb["unit"],
                          "ms_per_step": kstep * 1e3, "config": {"workload": DESCRIPTIONS["kplanes"],
                                                                 "sample": kb["sample"]},
                          "cpu_baseline": kb}
    return res


def _emit(line: str) -> None:
    os.write(_JSON_FD, (line + "\n").encode())


_JSON_FD = 1


def main() -> None:
    global _JSON_FD
    # Keep stdout for the one JSON line: anything else written to file
    # descriptor 1 while the benchmark runs (library banners such as NCCL's
    # version line, warnings) goes to stderr instead.
    sys.stdout.flush()
    _JSON_FD = os.dup(1)
    os.dup2(2, 1)
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=("ours", "reference"), default="ours")
    ap.add_argument("--workload", choices=sorted(WORKLOADS), default="tv_iso_l1")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-kplanes", action="store_true",
                    help="default workload only: leave out the K-Planes half of the line")
    ap.add_argument("--kp-reduce", choices=("peer", "nccl"), default="peer",
                    help="multi-GPU K-Planes: gradient sum over peer memory or with NCCL all_reduce")
    ap.add_argument("--kp-buckets", type=int, default=None,
                    help="multi-GPU K-Planes: backward launches whose gradient sum overlaps the next "
                         "(default 4 with the peer sum, 1 with NCCL)")
    ap.add_argument("--kp-reduce-ctas", type=int, default=32,
                    help="multi-GPU K-Planes, peer sum with --kp-buckets > 1: CTAs of an overlapped sum")
    ap.add_argument("--tv-transport", choices=("peer", "nccl"), default="peer",
                    help="multi-GPU TV: halos and loss sums over peer memory, or NCCL send/recv + all_gather")
    args = ap.parse_args()
    if args.kp_buckets is None:
        args.kp_buckets = 4 if args.kp_reduce == "peer" else 1
    ctx = Ctx(args)
    warmup = max(args.warmup, 3)

    if args.impl == "reference":
        res = run_reference(ctx, args)
        if res is not None:
            res.update({"n_gpus": args.gpus, "steps": args.steps, "warmup": warmup,
                        "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
                        "data": "synthetic"})
            _emit(json.dumps(res))
        return

    if ctx.world > 1:
        # NCCL's communicator set-up log on stderr (the JSON line keeps stdout):
        # it names every rank and its GPU, although the data plane of the
        # default transports is peer memory
        if os.environ.get("NCCL_DEBUG", "").upper() not in ("INFO", "TRACE"):
            os.environ["NCCL_DEBUG"] = "INFO"
            os.environ["NCCL_DEBUG_SUBSYS"] = "INIT"
        torch.cuda.set_device(ctx.local_rank)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", ctx.local_rank))
    ctx.device = torch.device("cuda", ctx.local_rank)
    torch.cuda.set_device(ctx.device)

    res = WORKLOADS[args.workload](ctx, args.steps, warmup)
    kp = None
    if args.workload == "tv_iso_l1" and not args.no_kplanes:
        # the default line carries both halves of the metric: TV (headline)
        # and K-Planes, each timed in its own region of this run
        kp = run_kplanes(ctx, args.steps, warmup)

    if ctx.rank == 0 and ctx.world == 1 and not args.no_cpu_baseline:
        res["cpu_baseline"], _ = CPU_BASELINES[args.workload]()
        if args.workload in TORCH_CPU_BASELINES:
            res["cpu_baseline_torch"], _ = TORCH_CPU_BASELINES[args.workload]()
        if kp is not None:
            kp["cpu_baseline"], _ = cpu_kplanes()
            kp["cpu_baseline_torch"], _ = torch_cpu_kplanes()
    for r_ in (res, kp):
        if r_ is not None and isinstance(r_.get("ref_cuda"), dict) and "value" in r_["ref_cuda"]:
            r_["ref_cuda"]["ours_over_reference"] = r_["value"] / r_["ref_cuda"]["value"]
    if kp is not None:
        kp.pop("dtype", None)
        res["kplanes"] = kp

    if ctx.world > 1:
        dist.barrier(device_ids=[ctx.local_rank])
        dist.destroy_process_group()
    if ctx.rank == 0:
        out = {
            "metric": res.pop("metric"),
            "value": res.pop("value"),
            "unit": res.pop("unit"),
            "n_gpus": ctx.world,
            "steps": args.steps,
            "warmup": warmup,
            "ms_per_step": res.pop("ms_per_step"),
            "higher_is_better": True,
            "scaling": res.pop("scaling", "weak"),
            "vs_baseline": None,
            "dtype": res.pop("dtype"),
            "data": "synthetic",
        }
        out.update(res)
        _emit(json.dumps(out))


if __name__ == "__main__":
    main()

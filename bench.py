#!/usr/bin/env python
"""Benchmark of the B200 tensor-core GEMM library (one JSON line on rank 0).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--workload f16|fp8|mxfp4|fp4] [--shape MxNxK] [--no-extra] [--no-compare]
                    [--no-cpu] [--multicast]

A step is one GEMM over one batch of synthetic inputs already resident in HBM:
  N = 1: C = A x B at M = N = K = 8192 (FP16 in, FP32 accumulate,
         FP32 out, uniform[-1, 1] seeded inputs rounded to FP16).
  N > 1: one process per GPU; rank r computes the column shard C[:, r*8192:(r+1)*8192] =
         A x B[:, shard r] of an 8192 x (8192 N) x 8192 GEMM (weak scaling; no collective in
         the timed region).
`value` is whole-job TFLOP/s = (all ranks' FLOPs) / (max over ranks of the device time of
K steps). A (128 MiB) + B (128 MiB) exceed the 126 MB L2, so no flush is needed between steps.

Sub-records of the same line:
  e2e        the same GEMM through the public C ABI from FP32 host buffers (what the
             reference's launch_* surface takes): per step FP32 A, B host -> device, the FP16
             cast (bw_quantize_f16) and the GEMM, FP32 C device -> host; pipelined over two
             buffer sets exactly like the reference arm's e2e leg.
  sustained  back-to-back GEMMs for >= 2.5 s with the clock record of that window, against the
             measured sustained bf16 peak, plus FLOP per SM per clock.
  precisions (N = 1) FP8 E4M3 amax/448 -> BF16, MXFP4 block32 -> BF16, FP4 per-tensor -> BF16 at
             8192^3, and the skinny 128 x 65536 x 8192 in FP16 and FP8: time, roofline, library
             row timed interleaved, max_abs_err against an FP64 GEMM of the dequantised inputs.
  sharded    (every N) BASELINE configs[4]: 16384 x 65536 x 8192 split column-wise over the N
             ranks (strong scaling), FP16 -> FP32 and FP8 -> BF16: GEMM alone, and for N > 1
             GEMM + fused all-gather (one kernel) and GEMM + NCCL all-gather + unshard (with
             --multicast also the fused gather through NVSwitch multicast); plus the skinny
             128 x 65536 x 8192 on the same sharding.

--impl reference runs the reference's own stock launcher (launch_mma_warptile, its headline
FP16 kernel, built from its sources for sm_100a by oracle/build_ref.sh) through its launch_*
API on the same workload, on every rank for that rank's shard, with the same e2e pipeline.
"""
from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import sys
import threading
import time

REPO = os.path.dirname(os.path.abspath(__file__))
PKG = os.path.join(REPO, "blackwell-tensorcore-kernels_b200")
ORACLE = os.path.join(REPO, "oracle")
for _p in (PKG, ORACLE):
    if _p not in sys.path:
        sys.path.insert(0, _p)

METRIC = "TFLOP/s & % of B200 dense peak (FP16/FP8/MXFP4 8192^3); box TFLOP/s @1/2/4/8"
FALLBACK_PEAKS = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}
DIM = 8192
SHAPE = [DIM, DIM, DIM]  # M, N (per GPU), K; --shape overrides (e.g. the skinny 128x65536x8192)
SHARDED = (16384, 65536, 8192)  # M, N_total, K
SKINNY = (128, 65536, 8192)
NUM_SMS = 148
_MULTICAST_BUFFERS = []  # symmetric-memory buffers bound to a multicast object (see multicast_gather)


def load_peaks():
    path = os.path.join(REPO, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            d = json.load(f)
        return d, "measured"
    except (OSError, ValueError):
        return dict(FALLBACK_PEAKS), "fallback"


def profile_traffic(name: str, key: str = "traffic_bytes_per_launch"):
    """DRAM bytes per launch recorded from an ncu capture in profiles/<name>.md
    (line `<key>: <int>`), or None."""
    path = os.path.join(REPO, "profiles", name + ".md")
    try:
        for line in open(path):
            if line.strip().startswith(key + ":"):
                return int(float(line.split(":", 1)[1]))
    except OSError:
        pass
    return None


def nvml_handle_for_cuda_device(nv, cuda_index: int):
    """The NVML handle of CUDA device `cuda_index`. NVML enumerates every GPU of the machine
    while CUDA sees only the visible ones (CUDA_VISIBLE_DEVICES), so an NVML index can name
    another job's GPU; the UUID identifies the same device in both."""
    import torch

    uuid = str(torch.cuda.get_device_properties(cuda_index).uuid)
    if not uuid.startswith("GPU-"):
        uuid = "GPU-" + uuid
    return nv.nvmlDeviceGetHandleByUUID(uuid)


class ClockSampler:
    """SM clock, clock-event (throttle) reasons and board power polled through NVML every 10 ms.

    NVML's clock and power telemetry trails the GPU by roughly 0.1-0.15 s (measured here: a
    GEMM loop started at t = 0 shows its power-capped clock from t = 0.15 s on), so the samples
    that describe a timed region are those taken LAG_S later: window() waits until the end of
    the region + LAG_S and reports [start + LAG_S, end + LAG_S]; stop() does the same and ends
    the polling."""

    REASONS = {"gpu_idle": 0x1, "applications_clocks_setting": 0x2, "sw_power_cap": 0x4, "hw_slowdown": 0x8,
               "sync_boost": 0x10, "sw_thermal_slowdown": 0x20, "hw_thermal_slowdown": 0x40,
               "hw_power_brake_slowdown": 0x80, "display_clock_setting": 0x100}
    LAG_S = 0.15

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index  # CUDA device ordinal (NVML numbers GPUs differently: matched by UUID)
        self.samples: list[tuple[float, float, int, float]] = []  # (time, SM MHz, reason bits, board W)
        self.smax = 0.0
        self._stop = threading.Event()
        self.t = None
        self.ok = False

    def start(self):
        try:
            import pynvml as nv

            nv.nvmlInit()
            h = nvml_handle_for_cuda_device(nv, self.gpu)
            self.smax = float(nv.nvmlDeviceGetMaxClockInfo(h, nv.NVML_CLOCK_SM))
        except Exception:
            return
        self.ok = True

        def poll():
            while not self._stop.is_set():
                try:
                    clk = float(nv.nvmlDeviceGetClockInfo(h, nv.NVML_CLOCK_SM))
                    rs = int(nv.nvmlDeviceGetCurrentClocksEventReasons(h))
                    pw = nv.nvmlDeviceGetPowerUsage(h) / 1000.0
                    self.samples.append((time.monotonic(), clk, rs, pw))
                except Exception:
                    pass
                self._stop.wait(0.01)

        self.t = threading.Thread(target=poll, daemon=True)
        self.t.start()

    def mark(self) -> float:
        """Start of a timed region (call right before it)."""
        return time.monotonic()

    def _summary(self, since: float, end: float):
        window = [x for x in self.samples if since + self.LAG_S <= x[0] <= end + self.LAG_S]
        if len(window) < 3:  # a region shorter than a few polls: take everything it may cover
            window = [x for x in self.samples if since <= x[0] <= end + self.LAG_S]
        if not window:
            return None
        reasons = sorted({n for _, _, r, _ in window for n, bit in self.REASONS.items() if r & bit})
        return {"sm_mhz": statistics.median(c for _, c, _, _ in window), "sm_max_mhz": self.smax,
                "reasons": reasons, "power_w": round(statistics.median(w for _, _, _, w in window), 1),
                "samples": len(window), "region_s": round(end - since, 3),
                "source": f"NVML (device matched by UUID), 10 ms polls shifted by the {self.LAG_S} s telemetry lag"}

    def window(self, since: float):
        """End of a timed region, polling continues: the lag-shifted window's summary."""
        if not self.ok:
            return None
        end = time.monotonic()
        time.sleep(self.LAG_S + 0.03)
        return self._summary(since, end)

    def stop(self, since: float):
        """End of the last timed region: its summary, and the polling stops."""
        if not self.ok:
            return None
        end = time.monotonic()
        time.sleep(self.LAG_S + 0.03)
        self._stop.set()
        self.t.join(timeout=2)
        return self._summary(since, end)


def dist_setup(args):
    import torch
    import torch.distributed as dist

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", device_id=torch.device("cuda", local))
    else:
        torch.cuda.set_device(0)
    return world, rank, local


def barrier(world):
    if world > 1:
        import torch.distributed as dist

        dist.barrier()


def max_over_ranks(x: float, world: int) -> float:
    if world == 1:
        return x
    import torch
    import torch.distributed as dist

    t = torch.tensor([x], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def timed_steps(step, K: int, W: int, world: int, stream):
    """W warm-up steps, then K steps bracketed by barrier + synchronize; returns device ms
    per step (CUDA events on the launching stream), max over ranks."""
    import torch

    for _ in range(W):
        step()
    torch.cuda.synchronize()
    barrier(world)
    torch.cuda.synchronize()
    s = torch.cuda.Event(enable_timing=True)
    e = torch.cuda.Event(enable_timing=True)
    s.record(stream)
    for _ in range(K):
        step()
    e.record(stream)
    torch.cuda.synchronize()
    barrier(world)
    ms = s.elapsed_time(e) / K
    return max_over_ranks(ms, world)


def tflops(flops: float, ms: float) -> float:
    return flops / (ms * 1e-3) / 1e12


def config_dict(wl: str, M: int, N: int, K: int, world: int) -> dict:
    """The workload description, identical on both arms (the driver compares them)."""
    return {"workload": f"{wl}_gemm_{M}x{N}x{K}_per_gpu", "M": M, "N_per_gpu": N, "K": K, "N_total": N * world,
            "parallelism": f"column shards x{world} (no collective in the timed region)",
            "l2": "inputs larger than L2 (A and B 8192x8192 each)" if M * K + K * N >= 2 * DIM * DIM
            else "inputs smaller than L2", "accumulate": "fp32", "out": "fp32" if wl == "f16" else "bf16",
            "e2e_inputs": "fp32 host A and B (the launch_* operator surface), fp32 C back to the host"}


class E2EPipeline:
    """End-to-end GEMM with host buffers: each step copies its FP32 A and B from pinned host
    memory, runs `gemm(dA, dB, dC)` on the compute stream and copies FP32 C back to pinned host
    memory. Two device buffer sets and separate H2D / compute / D2H streams let step i+1's
    upload and step i-1's download run while step i multiplies (the copy engines of the two
    directions work in parallel); events keep every buffer's reuse in order. The two buffer
    sets alternate, so a launcher that caches its staging by input pointer re-stages every
    step."""

    def __init__(self, hA, hB, c_shape, dev, compute_stream, gemm):
        import torch

        self.hA, self.hB = hA, hB
        self.cs = compute_stream
        self.gemm = gemm
        self.h2d = torch.cuda.Stream(dev)
        self.d2h = torch.cuda.Stream(dev)
        self.dA = [torch.empty(hA.shape, dtype=hA.dtype, device=dev) for _ in range(2)]
        self.dB = [torch.empty(hB.shape, dtype=hB.dtype, device=dev) for _ in range(2)]
        self.dC = [torch.empty(c_shape, dtype=torch.float32, device=dev) for _ in range(2)]
        self.hC = [torch.empty(c_shape, dtype=torch.float32, pin_memory=True) for _ in range(2)]
        self.ev_in = [torch.cuda.Event() for _ in range(2)]
        self.ev_mm = [torch.cuda.Event() for _ in range(2)]
        self.ev_out = [torch.cuda.Event() for _ in range(2)]
        self.i = 0

    def step(self):
        import torch

        b = self.i & 1
        self.i += 1
        if self.i > 2:
            self.h2d.wait_event(self.ev_mm[b])  # the GEMM two steps back has read dA/dB[b]
        with torch.cuda.stream(self.h2d):
            self.dA[b].copy_(self.hA, non_blocking=True)
            self.dB[b].copy_(self.hB, non_blocking=True)
        self.ev_in[b].record(self.h2d)
        self.cs.wait_event(self.ev_in[b])
        if self.i > 2:
            self.cs.wait_event(self.ev_out[b])  # dC[b] has been downloaded
        self.gemm(self.dA[b], self.dB[b], self.dC[b])
        self.ev_mm[b].record(self.cs)
        self.d2h.wait_event(self.ev_mm[b])
        with torch.cuda.stream(self.d2h):
            self.hC[b].copy_(self.dC[b], non_blocking=True)
        self.ev_out[b].record(self.d2h)

    def timed(self, K: int, W: int, world: int) -> float:
        """W warm-up steps, then K steps from one event on the compute stream (both copy
        streams wait on it) to one recorded after joining both copy streams; ms per step,
        max over ranks."""
        import torch

        for _ in range(W):
            self.step()
        torch.cuda.synchronize()
        barrier(world)
        torch.cuda.synchronize()
        s = torch.cuda.Event(enable_timing=True)
        e = torch.cuda.Event(enable_timing=True)
        s.record(self.cs)
        self.h2d.wait_event(s)
        self.d2h.wait_event(s)
        for _ in range(K):
            self.step()
        self.cs.wait_stream(self.h2d)
        self.cs.wait_stream(self.d2h)
        e.record(self.cs)
        torch.cuda.synchronize()
        barrier(world)
        return max_over_ranks(s.elapsed_time(e) / K, world)

    def bytes(self):
        return (int(self.hA.numel() * self.hA.element_size() + self.hB.numel() * self.hB.element_size()),
                int(self.hC[0].numel() * 4))


def run_e2e(hA32, hB32, M, N, K, dev, stream, gemm, steps, world, flops):
    """The e2e record of one arm: pipelined FP32-host GEMM steps; the result that came back
    is spot-checked on 4 rows against the FP16-rounded host product."""
    import torch

    pipe = E2EPipeline(hA32, hB32, (M, N), dev, stream, gemm)
    e_steps = max(4, min(steps, 12))
    ems = pipe.timed(e_steps, 2, world)
    bi, bo = pipe.bytes()
    rows = [0, 1, M // 2, M - 1]
    ref = hA32[rows].half().float() @ hB32.half().float()
    ok = all(bool(torch.allclose(hC[rows], ref, atol=2 ** -10 * (K ** 0.5), rtol=0)) for hC in pipe.hC)
    del pipe
    if not ok:
        raise SystemExit("e2e result mismatch")
    return {"value": round(world * tflops(flops, ems), 2), "unit": "TFLOP/s", "h2d_bytes_per_step": bi,
            "d2h_bytes_per_step": bo, "ms_per_step": round(ems, 4), "steps": e_steps,
            "pipelining": "two buffer sets: H2D of step i+1 and D2H of step i-1 overlap the GEMM of step i",
            "checked": "4 rows of every returned C against the host product"}


def make_inputs(workload: str, rank: int, dev, shape=None):  # noqa: C901
    """Seeded synthetic inputs of the BASELINE shapes (per rank: its own column shard)."""
    import torch

    # A is the same on every rank (replicated); B is this rank's column shard of the full B.
    ga = torch.Generator(device=dev)
    ga.manual_seed(1234)
    gb = torch.Generator(device=dev)
    gb.manual_seed(4321 + 17 * rank)
    M, N, K = shape or SHAPE
    if workload == "f16":
        A = (torch.rand((M, K), generator=ga, device=dev) * 2 - 1).half()
        B = (torch.rand((K, N), generator=gb, device=dev) * 2 - 1).half()
        return {"A": A, "B": B}
    A32 = torch.randn((M, K), generator=ga, device=dev)
    B32 = torch.randn((K, N), generator=gb, device=dev)
    return {"A32": A32, "B32": B32}


def cpu_model() -> str:
    """The host CPU's model name (first /proc/cpuinfo entry) and its logical CPU count."""
    name = "unknown CPU"
    try:
        with open("/proc/cpuinfo") as f:
            for line in f:
                if line.startswith("model name"):
                    name = line.split(":", 1)[1].strip()
                    break
    except OSError:
        pass
    return f"{name}, {os.cpu_count()} logical CPUs"


def cpu_baseline(threads: int, budget_s: float = 12.0):
    """FP64 oracle GEMM (oracle/bw_oracle.c) on host cores over a bounded row sample of the
    8192^3 FP16 workload; returns TFLOP/s and the sample description."""
    import numpy as np

    import oracle as o

    K = N = DIM
    rng = np.random.default_rng(5)
    B = o.f16_to_f32(o.f32_to_f16(rng.uniform(-1, 1, size=(K, N)).astype(np.float32)))
    # double the row sample until one run takes at least budget_s / 2 (capped at all rows)
    rows = 64
    while True:
        A = o.f16_to_f32(o.f32_to_f16(rng.uniform(-1, 1, size=(rows, K)).astype(np.float32)))
        t0 = time.perf_counter()
        o.gemm_f64(A, B, threads=threads)
        dt = time.perf_counter() - t0
        if dt >= budget_s / 2 or rows >= DIM:
            break
        rows = min(DIM, rows * max(2, int(budget_s / 2 / max(dt, 1e-3))))
    flops = 2.0 * rows * N * K
    return flops / dt / 1e12, f"{rows} x {N} x {K} rows of the 8192^3 fp16 GEMM, FP64 oracle, {dt:.1f} s"


def cpu_full_1024(threads: int):
    """The whole 1024^3 FP16 GEMM (the host-computable anchor) through the
    FP64 oracle on host cores: TFLOP/s and seconds."""
    import numpy as np

    import oracle as o

    rng = np.random.default_rng(6)
    A = o.f16_to_f32(o.f32_to_f16(rng.uniform(-1, 1, size=(1024, 1024)).astype(np.float32)))
    B = o.f16_to_f32(o.f32_to_f16(rng.uniform(-1, 1, size=(1024, 1024)).astype(np.float32)))
    t0 = time.perf_counter()
    o.gemm_f64(A, B, threads=threads)
    dt = time.perf_counter() - t0
    return 2.0 * 1024 ** 3 / dt / 1e12, dt


# ---------------------------------------------------------------------------------------
# dequantisation on the device (FP64) for the max_abs_err of the precision records
E2M1 = [0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0, -0.0, -0.5, -1.0, -1.5, -2.0, -3.0, -4.0, -6.0]


def deq_e2m1_packed(q, K):
    """Packed E2M1 (outer x K/2 bytes, even k in the low nibble) -> outer x K float64."""
    import torch

    lut = torch.tensor(E2M1, dtype=torch.float64, device=q.device)
    q = q.long()
    out = torch.stack([lut[q & 15], lut[q >> 4]], dim=-1)
    return out.reshape(q.shape[0], K)


def deq_ue8m0_tiled(sf, outer, K):
    """The tiled UE8M0 layout (128-row x 4-block atoms of 512 B, K-group fastest; inside an atom
    row r, block j at (r % 32) * 16 + (r / 32) * 4 + j) -> outer x K/32 float64 factors."""
    import torch

    nkb = K // 32
    kg = (nkb + 3) // 4
    r = torch.arange(outer, device=sf.device).view(-1, 1)
    j = torch.arange(nkb, device=sf.device).view(1, -1)
    off = ((r >> 7) * kg + (j >> 2)) * 512 + (r & 31) * 16 + ((r >> 5) & 3) * 4 + (j & 3)
    e = sf.long()[off] - 127
    return torch.pow(torch.tensor(2.0, dtype=torch.float64, device=sf.device), e.double())


def max_abs_err(C, dA_rows, dBt, rows, scale=1.0):
    """max |C[rows] - FP64(dA_rows x dBt^T) * scale|."""
    R = (dA_rows @ dBt.t()) * scale
    return float((C[rows].double() - R).abs().max())


def sample_rows(M, n=64):
    import torch

    g = torch.Generator()
    g.manual_seed(99)
    idx = torch.randperm(M, generator=g)[: min(n, M)]
    return torch.unique(torch.cat([idx, torch.tensor([0, M - 1])]))


def interleaved(fa, fb, block, stream, flops, rounds=4):
    """Median TFLOP/s of fa and fb timed in alternating blocks of equal length, so both see
    the same power / clock state."""
    ra, rb = [], []
    for _ in range(rounds):
        ra.append(tflops(flops, timed_steps(fa, block, 2, 1, stream)))
        if fb is not None:
            rb.append(tflops(flops, timed_steps(fb, block, 2, 1, stream)))
    return round(statistics.median(ra), 1), (round(statistics.median(rb), 1) if rb else None)


# ---------------------------------------------------------------------------------------
def run_precisions(args, dev, stream, peaks, peak_src):
    """Per-precision records at N = 1 (the reference's bench.csv reports every precision as a
    row of its own): FP8, MXFP4, plain FP4 at 8192^3 and the skinny shape in FP16 and FP8."""
    import torch
    import torch.nn.functional as F

    import bwgemm

    out = {}
    block = max(10, min(args.steps, 50))
    bf16 = float(peaks.get("bf16_tflops", FALLBACK_PEAKS["bf16_tflops"]))
    hbm = float(peaks.get("hbm_gbs", FALLBACK_PEAKS["hbm_gbs"]))
    M = N = K = DIM
    flops = 2.0 * M * N * K
    inp = make_inputs("fp8", 0, dev, (M, N, K))
    A32, B32 = inp["A32"], inp["B32"]
    rows = sample_rows(M).to(dev)

    def record(name, ours, lib, lib_name, mult, traffic_name, err, tol, kind):
        ms = timed_steps(ours, args.steps, args.warmup, 1, stream)
        a, b = interleaved(ours, lib, block, stream, flops)
        peak = mult * bf16
        ach = tflops(flops, ms)
        rec = {"workload": f"{name}_gemm_{M}x{N}x{K}", "quantisation": kind, "ms_per_step": round(ms, 4),
               "tflops": round(ach, 2),
               "roofline": {"bound": "tensor", "achieved": round(ach, 2), "peak": round(peak, 1), "unit": "TFLOP/s",
                            "frac": round(ach / peak, 4), "traffic": profile_traffic(traffic_name),
                            "peak_source": f"{peak_src}: {mult:.0f} x bf16_tflops (burst; nominal dense-rate ratio)"},
               "vs_nominal_dense_peak": round(ach / (2250.0 * mult), 4),
               "interleaved": {"ours_tflops": a, "library_tflops": b, "library": lib_name, "block_steps": block},
               "max_abs_err": err, "tolerance": tol, "within_tolerance": err <= tol}
        out[name] = rec

    # FP8 E4M3, per-tensor amax/448, BF16 out; the library row is cuBLASLt through torch._scaled_mm
    qa, sa = bwgemm.quantize_fp8(A32, False, bwgemm.SCALE_AMAX)
    qb, sb = bwgemm.quantize_fp8(B32, True, bwgemm.SCALE_AMAX)
    C8 = torch.empty((M, N), dtype=torch.bfloat16, device=dev)
    bwgemm.gemm_fp8(qa, qb, sa, sb, C8, stream=stream)
    dA = qa.view(torch.float8_e4m3fn).double()
    dB = qb.view(torch.float8_e4m3fn).double()
    s = float(sa.item()) * float(sb.item())
    err = max_abs_err(C8, dA[rows], dB, rows, s)
    ma, mb = float(dA.abs().max()) * float(sa.item()), float(dB.abs().max()) * float(sb.item())
    tol = 1e-5 * K * ma * mb + 2 ** -8 * float(C8.float().abs().max())
    a8, b8 = qa.view(torch.float8_e4m3fn), qb.view(torch.float8_e4m3fn).t()
    record("fp8", lambda: bwgemm.gemm_fp8(qa, qb, sa, sb, C8, stream=stream),
           lambda: torch._scaled_mm(a8, b8, scale_a=sa, scale_b=sb, out_dtype=torch.bfloat16),
           "cuBLASLt FP8 (torch._scaled_mm, tensor-wise scales, BF16 out)", 2.0, "bw_tc_gemm_pair_fp8_8192",
           err, tol, "E4M3, per-tensor scale amax/448, BF16 C")
    del dA, dB, qa, qb

    # MXFP4: E2M1 + UE8M0 per 32 K, BF16 out; library row: the CUTLASS kernel torch's scaled_mm runs
    q4a, sfa = bwgemm.quantize_mxfp4(A32, False, bwgemm.MX_BLOCK32)
    q4b, sfb = bwgemm.quantize_mxfp4(B32, True, bwgemm.MX_BLOCK32)
    bwgemm.gemm_mxfp4(q4a, q4b, sfa, sfb, K, C=C8, stream=stream)
    dA = deq_e2m1_packed(q4a, K) * deq_ue8m0_tiled(sfa, M, K).repeat_interleave(32, dim=1)
    dB = deq_e2m1_packed(q4b, K) * deq_ue8m0_tiled(sfb, N, K).repeat_interleave(32, dim=1)
    err = max_abs_err(C8, dA[rows], dB, rows)
    tol = 1e-5 * K * float(dA.abs().max()) * float(dB.abs().max()) + 2 ** -8 * float(C8.float().abs().max())
    del dA, dB
    a4, b4 = q4a.view(torch.float4_e2m1fn_x2), q4b.view(torch.float4_e2m1fn_x2).t()
    e8a, e8b = sfa.view(torch.float8_e8m0fnu), sfb.view(torch.float8_e8m0fnu)
    record("mxfp4", lambda: bwgemm.gemm_mxfp4(q4a, q4b, sfa, sfb, K, C=C8, stream=stream),
           lambda: F.scaled_mm(a4, b4, e8a, F.ScalingType.BlockWise1x32, e8b, F.ScalingType.BlockWise1x32,
                               swizzle_a=F.SwizzleType.SWIZZLE_32_4_4, swizzle_b=F.SwizzleType.SWIZZLE_32_4_4,
                               output_dtype=torch.bfloat16),
           "torch scaled_mm MXFP4 (a CUTLASS kernel; cuBLASLt 12.9 has no E2M1/VEC32_UE8M0/BF16 path)", 4.0,
           "bw_tc_gemm_pair_mxfp4_8192", err, tol, "E2M1, UE8M0 per 32 K (floor(log2 amax) - 2), BF16 C")
    del q4a, q4b

    # plain FP4: E2M1 with a per-tensor scale amax/6, BF16 out (no library kernel takes this form)
    p4a, pa = bwgemm.quantize_fp4(A32, False, bwgemm.SCALE_AMAX, bwgemm.FP4_PACKED)
    p4b, pb = bwgemm.quantize_fp4(B32, True, bwgemm.SCALE_AMAX, bwgemm.FP4_PACKED)
    bwgemm.gemm_fp4(p4a, p4b, K, pa, pb, C=C8, stream=stream)
    dA, dB = deq_e2m1_packed(p4a, K), deq_e2m1_packed(p4b, K)
    s = float(pa.item()) * float(pb.item())
    err = max_abs_err(C8, dA[rows], dB, rows, s)
    tol = 1e-5 * K * 36.0 * s + 2 ** -8 * float(C8.float().abs().max())
    del dA, dB
    record("fp4", lambda: bwgemm.gemm_fp4(p4a, p4b, K, pa, pb, C=C8, stream=stream), None,
           "none (no library kernel takes E2M1 with per-tensor scales)", 4.0, "bw_tc_gemm_pair_fp4_8192",
           err, tol, "E2M1, per-tensor scale amax/6, BF16 C")
    del p4a, p4b, A32, B32, C8, inp

    # skinny decode-style shape: HBM-bound (B is read once)
    Ms, Ns, Ks = SKINNY
    sflops = 2.0 * Ms * Ns * Ks
    srows = sample_rows(Ms, 32).to(dev)
    fin = make_inputs("f16", 0, dev, SKINNY)
    A, B = fin["A"], fin["B"]
    Cf = torch.empty((Ms, Ns), dtype=torch.float32, device=dev)
    bwgemm.gemm_f16(A, B, Cf, stream=stream)
    err = max_abs_err(Cf, A.double()[srows], B.double().t(), srows)
    tol = 2 ** -10 * math.sqrt(Ks)
    del fin
    n_in = {"f16": Ms * Ks * 2 + Ks * Ns * 2 + Ms * Ns * 4, "fp8": Ms * Ks + Ks * Ns + Ms * Ns * 2}

    def skinny_record(name, ours, lib, lib_name, nbytes, err, tol, kind, traffic):
        ms = timed_steps(ours, args.steps, args.warmup, 1, stream)
        a, b = interleaved(ours, lib, block, stream, sflops)
        gbs = nbytes / (ms * 1e-3) / 1e9
        out[name] = {"workload": f"{name.split('_')[1]}_gemm_{Ms}x{Ns}x{Ks}", "quantisation": kind,
                     "ms_per_step": round(ms, 4), "tflops": round(tflops(sflops, ms), 2),
                     "roofline": {"bound": "hbm", "achieved": round(gbs, 1), "peak": round(hbm, 1), "unit": "GB/s",
                                  "frac": round(gbs / hbm, 4), "traffic": traffic,
                                  "algorithmic_bytes_per_launch": nbytes, "peak_source": f"{peak_src}: hbm_gbs"},
                     "interleaved": {"ours_tflops": a, "library_tflops": b, "library": lib_name, "block_steps": block},
                     "max_abs_err": err, "tolerance": tol, "within_tolerance": err <= tol}

    skinny_record("skinny_f16", lambda: bwgemm.gemm_f16(A, B, Cf, stream=stream),
                  lambda: torch.mm(A, B, out_dtype=torch.float32), "cuBLAS (torch.mm fp16 -> fp32)", n_in["f16"],
                  err, tol, "FP16 uniform[-1, 1], FP32 C (column-panel kernel, one 128 x 448 unit per SM)",
                  profile_traffic("bw_tc_gemm_panel_128x65536x8192", "traffic_bytes_per_launch_f16"))
    del A, B, Cf
    sin = make_inputs("fp8", 0, dev, SKINNY)
    qa, sa = bwgemm.quantize_fp8(sin["A32"], False, bwgemm.SCALE_AMAX)
    qb, sb = bwgemm.quantize_fp8(sin["B32"], True, bwgemm.SCALE_AMAX)
    del sin
    Cb = torch.empty((Ms, Ns), dtype=torch.bfloat16, device=dev)
    bwgemm.gemm_fp8(qa, qb, sa, sb, Cb, stream=stream)
    dA = qa.view(torch.float8_e4m3fn).double()
    dB = qb.view(torch.float8_e4m3fn).double()
    s = float(sa.item()) * float(sb.item())
    err = max_abs_err(Cb, dA[srows], dB, srows, s)
    tol = 1e-5 * Ks * float(dA.abs().max()) * float(dB.abs().max()) * s + 2 ** -8 * float(Cb.float().abs().max())
    del dA, dB
    a8, b8 = qa.view(torch.float8_e4m3fn), qb.view(torch.float8_e4m3fn).t()
    skinny_record("skinny_fp8", lambda: bwgemm.gemm_fp8(qa, qb, sa, sb, Cb, stream=stream),
                  lambda: torch._scaled_mm(a8, b8, scale_a=sa, scale_b=sb, out_dtype=torch.bfloat16),
                  "cuBLASLt FP8 (torch._scaled_mm, BF16 out)", n_in["fp8"], err, tol,
                  "E4M3 amax/448, BF16 C (column-panel kernel, one 128 x 448 unit per SM)",
                  profile_traffic("bw_tc_gemm_panel_128x65536x8192"))
    return out


def run_sharded(args, world, rank, dev, stream):
    """BASELINE configs[4] strong scaling: 16384 x 65536 x 8192 split column-wise over the
    world, FP16 -> FP32 and FP8 -> BF16; GEMM alone (max over ranks), and for world > 1 the
    GEMM + fused all-gather and GEMM + NCCL all-gather + unshard, whose gathered C must be
    bit-identical on every rank; the skinny 128 x 65536 x 8192 on the same sharding."""
    import torch

    import bwgemm
    import sharding

    M, Nt, K = SHARDED
    if Nt % world:
        return {"error": f"N = {Nt} does not split over {world} ranks"}
    Ns = Nt // world
    steps = max(5, min(args.steps, 20))
    total_flops = 2.0 * M * Nt * K
    out = {"workload": f"{M}x{Nt}x{K} split column-wise x{world} ({M}x{Ns}x{K} per GPU)", "scaling": "strong"}
    for wl in ("f16", "fp8"):
        inp = make_inputs(wl, rank, dev, (M, Ns, K))
        if wl == "f16":
            A, B = inp["A"], inp["B"]
            C = torch.empty((M, Ns), dtype=torch.float32, device=dev)
            step = lambda: bwgemm.gemm_f16(A, B, C, stream=stream)  # noqa: E731
            operands = (A, B)
        else:
            qa, sa = bwgemm.quantize_fp8(inp["A32"], False, bwgemm.SCALE_AMAX)
            qb, sb = bwgemm.quantize_fp8(inp["B32"], True, bwgemm.SCALE_AMAX)
            del inp
            C = torch.empty((M, Ns), dtype=torch.bfloat16, device=dev)
            step = lambda: bwgemm.gemm_fp8(qa, qb, sa, sb, C, stream=stream)  # noqa: E731
            operands = (qa, qb, sa, sb)
        ms = timed_steps(step, steps, 3, world, stream)
        rec = {"gemm_ms": round(ms, 4), "gemm_tflops_all_gpus": round(tflops(total_flops, ms), 2), "steps": steps,
               "out": "fp32" if wl == "f16" else "bf16"}
        if world > 1:
            # NCCL all-gather of the shards + unshard into row-major M x N_total
            sharding.gather_columns(C, world)  # warm-up: communicator and buffers
            torch.cuda.synchronize()
            reps = 3
            g_ms = timed_steps(lambda: sharding.gather_columns(C, world), reps, 0, world, stream)
            full = sharding.gather_columns(C, world)
            torch.cuda.synchronize()
            rec["nccl_gather"] = {"gather_ms": round(g_ms, 4), "gemm_plus_gather_ms": round(ms + g_ms, 4),
                                  "tflops_all_gpus": round(tflops(total_flops, ms + g_ms), 2),
                                  "bytes_sent_per_rank": int(C.numel() * C.element_size() * (world - 1)),
                                  "how": "torch.distributed.all_gather_into_tensor (NCCL) + bw_unshard_columns"}
            rec["fused_gather"] = fused_gather(args, wl, operands, C, full, world, rank, dev, stream, steps)
            rec["fused_gather"]["tflops_all_gpus"] = round(tflops(total_flops, rec["fused_gather"]["ms_per_step"]), 2)
            link = 770.0  # GB/s per direction, measured peer copy on this pool
            sent = rec["fused_gather"]["bytes_sent_per_rank"]
            floor_ms = max(ms, sent / (link * 1e9) * 1e3)
            rec["fused_gather"]["roofline"] = {
                "target_ms": round(floor_ms, 4), "frac": round(floor_ms / rec["fused_gather"]["ms_per_step"], 4),
                "how": "max(GEMM time, bytes sent per rank / 770 GB/s measured peer-copy rate)",
                "limiter": "NVLink egress of the gathered C" if sent / (link * 1e9) * 1e3 > ms else "GEMM"}
            if args.multicast:
                mc = multicast_gather(wl, operands, C, full, world, rank, dev, stream, steps)
                if mc.get("ms_per_step"):
                    mc["tflops_all_gpus"] = round(tflops(total_flops, mc["ms_per_step"]), 2)
                    sent_mc = int(C.numel() * C.element_size())
                    floor_mc = max(ms, sent_mc / (link * 1e9) * 1e3)
                    mc["roofline"] = {"target_ms": round(floor_mc, 4), "frac": round(floor_mc / mc["ms_per_step"], 4),
                                      "how": "max(GEMM time, shard bytes leaving each GPU once / 770 GB/s)"}
                rec["fused_gather_multicast"] = mc
            del full
        out[wl] = rec
        del C
        torch.cuda.empty_cache()
    # skinny on the same sharding (GEMM only: HBM-bound per GPU)
    Ms, Nst, Ks = SKINNY
    Nss = Nst // world
    fin = make_inputs("f16", rank, dev, (Ms, Nss, Ks))
    Cs = torch.empty((Ms, Nss), dtype=torch.float32, device=dev)
    ms = timed_steps(lambda: bwgemm.gemm_f16(fin["A"], fin["B"], Cs, stream=stream), steps * 5, 3, world, stream)
    out["skinny_f16"] = {"workload": f"{Ms}x{Nst}x{Ks} split x{world}", "gemm_ms": round(ms, 4),
                         "gemm_tflops_all_gpus": round(tflops(2.0 * Ms * Nst * Ks, ms), 2)}
    del fin, Cs
    sin = make_inputs("fp8", rank, dev, (Ms, Nss, Ks))
    qa, sa = bwgemm.quantize_fp8(sin["A32"], False, bwgemm.SCALE_AMAX)
    qb, sb = bwgemm.quantize_fp8(sin["B32"], True, bwgemm.SCALE_AMAX)
    del sin
    Cb = torch.empty((Ms, Nss), dtype=torch.bfloat16, device=dev)
    ms = timed_steps(lambda: bwgemm.gemm_fp8(qa, qb, sa, sb, Cb, stream=stream), steps * 5, 3, world, stream)
    out["skinny_fp8"] = {"workload": f"{Ms}x{Nst}x{Ks} split x{world}", "gemm_ms": round(ms, 4),
                         "gemm_tflops_all_gpus": round(tflops(2.0 * Ms * Nst * Ks, ms), 2)}
    torch.cuda.empty_cache()
    return out


def fused_gather(args, wl, operands, C, full, world, rank, dev, stream, steps):
    """GEMM and all-gather in one kernel: every rank's epilogue stores its columns into its own
    and every peer's IPC-mapped row-major C (bw_gemm_*_allgather). Timed like the GEMM (device
    events, max over ranks, after a barrier); checked bit-for-bit against the NCCL gather."""
    import torch

    import bwgemm
    import sharding

    M, N = C.shape
    sym = sharding.SymmetricC(M, N * world, C.dtype, dev, world, rank)
    if wl == "f16":
        A, B = operands
        step = lambda: bwgemm.gemm_f16_allgather(A, B, sym.C, sym.peers, rank, stream=stream)  # noqa: E731
    else:
        qa, qb, sa, sb = operands
        step = lambda: bwgemm.gemm_fp8_allgather(qa, qb, sa, sb, sym.C, sym.peers, rank, stream=stream)  # noqa: E731
    ms = timed_steps(step, steps, 3, world, stream)
    torch.cuda.synchronize()
    barrier(world)
    same = bool(torch.equal(sym.C, full))
    same_all = max_over_ranks(0.0 if same else 1.0, world) == 0.0
    barrier(world)
    sym.close()
    return {"ms_per_step": round(ms, 4), "bytes_sent_per_rank": int(C.numel() * C.element_size() * (world - 1)),
            "matches_nccl_gather_on_all_ranks": same_all,
            "how": "one kernel: each staged 32-row chunk is TMA-stored to the local C and to every peer's C over NVLink"}


def multicast_gather(wl, operands, C, full, world, rank, dev, stream, steps):
    """GEMM and all-gather in one kernel through NVSwitch multicast: every rank binds its C_full
    to one NVLink multicast object (torch symmetric memory) and the epilogue writes each staged
    chunk once with multimem.st, which the switch replicates into every rank's C_full. Timed
    like the GEMM; checked bit-for-bit against the NCCL gather on every rank."""
    import torch

    import bwgemm
    import sharding

    M, N = C.shape
    try:
        mcC = sharding.MulticastC(M, N * world, C.dtype, dev)
    except Exception as ex:  # no symmetric-memory multicast on this platform
        return {"unavailable": f"{type(ex).__name__}: {ex}"[:200]}
    # kept until the process ends: no rank unbinds its memory from the multicast object while
    # another rank may still use it
    _MULTICAST_BUFFERS.append(mcC)
    if not mcC.available:
        return {"unavailable": "symmetric memory reports no multicast address (no NVLS on this platform)"}
    if wl == "f16":
        A, B = operands
        step = lambda: bwgemm.gemm_f16_allgather_multicast(A, B, mcC.mc, world, rank, N * world, stream=stream)  # noqa: E731
    else:
        qa, qb, sa, sb = operands
        step = lambda: bwgemm.gemm_fp8_allgather_multicast(qa, qb, sa, sb, mcC.mc, world, rank, N * world,  # noqa: E731
                                                           stream=stream)
    ms = timed_steps(step, steps, 3, world, stream)
    torch.cuda.synchronize()
    barrier(world)
    same = bool(torch.equal(mcC.C, full))
    same_all = max_over_ranks(0.0 if same else 1.0, world) == 0.0
    barrier(world)
    return {"ms_per_step": round(ms, 4), "bytes_leaving_each_gpu": int(C.numel() * C.element_size()),
            "matches_nccl_gather_on_all_ranks": same_all,
            "how": "one kernel: each staged 32-row chunk is written once with multimem.st to the multicast "
                   "address; NVSwitch replicates it into every rank's C"}


def run_sustained(step, flops, ms_hint, stream, clocks, peaks, peak_src, seconds=2.5):
    """Back-to-back steps for `seconds`, with the clock record of that window."""
    n = max(20, int(seconds / (ms_hint * 1e-3)))
    mark = clocks.mark()
    ms = timed_steps(step, n, 0, 1, stream)
    clk = clocks.window(mark)
    ach = tflops(flops, ms)
    sus = float(peaks.get("bf16_tflops_sustained", FALLBACK_PEAKS["bf16_tflops_sustained"]))
    rec = {"steps": n, "ms_per_step": round(ms, 4), "tflops": round(ach, 2), "region_s": round(n * ms * 1e-3, 3),
           "vs_bf16_tflops_sustained": round(ach / sus, 4), "peak_source": f"{peak_src}: bf16_tflops_sustained",
           "clocks": clk}
    if clk and clk.get("sm_mhz"):
        rec["flop_per_sm_per_clk"] = round(ach * 1e12 / (NUM_SMS * clk["sm_mhz"] * 1e6), 1)
    return rec


def run_ours(args, world, rank, local):
    import torch

    import bwgemm

    dev = torch.device("cuda", local)
    bwgemm.init(local)
    stream = torch.cuda.current_stream()
    M, N, K = SHAPE
    flops = 2.0 * M * N * K
    clocks = ClockSampler(local)
    clocks.start()
    inp = make_inputs(args.workload, rank, dev)
    wl = args.workload
    if wl == "f16":
        A, B = inp["A"], inp["B"]
        C = torch.empty((M, N), dtype=torch.float32, device=dev)
        step = lambda: bwgemm.gemm_f16(A, B, C, stream=stream)  # noqa: E731
        dtype = "f16"
    elif wl == "fp8":
        qa, sa = bwgemm.quantize_fp8(inp["A32"], False, bwgemm.SCALE_AMAX)
        qb, sb = bwgemm.quantize_fp8(inp["B32"], True, bwgemm.SCALE_AMAX)
        C = torch.empty((M, N), dtype=torch.bfloat16, device=dev)
        step = lambda: bwgemm.gemm_fp8(qa, qb, sa, sb, C, stream=stream)  # noqa: E731
        dtype = "e4m3"
    elif wl in ("mxfp4", "fp4"):
        if wl == "mxfp4":
            qa, sfa = bwgemm.quantize_mxfp4(inp["A32"], False, bwgemm.MX_BLOCK32)
            qb, sfb = bwgemm.quantize_mxfp4(inp["B32"], True, bwgemm.MX_BLOCK32)
            C = torch.empty((M, N), dtype=torch.bfloat16, device=dev)
            step = lambda: bwgemm.gemm_mxfp4(qa, qb, sfa, sfb, K, C=C, stream=stream)  # noqa: E731
        else:
            qa, sa = bwgemm.quantize_fp4(inp["A32"], False, bwgemm.SCALE_AMAX, bwgemm.FP4_PACKED)
            qb, sb = bwgemm.quantize_fp4(inp["B32"], True, bwgemm.SCALE_AMAX, bwgemm.FP4_PACKED)
            C = torch.empty((M, N), dtype=torch.bfloat16, device=dev)
            step = lambda: bwgemm.gemm_fp4(qa, qb, K, sa, sb, C=C, stream=stream)  # noqa: E731
        dtype = "e2m1"
    else:
        raise SystemExit(f"unknown workload {wl}")

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    mark = clocks.mark()
    ms = timed_steps(step, args.steps, 0, world, stream)
    clk = clocks.window(mark)
    status = bwgemm.device_status()
    if status != 0:
        raise SystemExit(f"kernel reported status {status}")
    value = world * tflops(flops, ms)
    peaks, peak_src = load_peaks()

    sustained = None
    if world == 1 and not args.no_extra:
        sustained = run_sustained(step, flops, ms, stream, clocks, peaks, peak_src)

    # ---- e2e: FP32 host inputs -> device, FP16 cast + GEMM through the C ABI, C -> host
    e2e = None
    if wl == "f16":
        hA = torch.empty((M, K), dtype=torch.float32, pin_memory=True)
        hB = torch.empty((K, N), dtype=torch.float32, pin_memory=True)
        hA.copy_(A.float().cpu())
        hB.copy_(B.float().cpu())
        a16 = torch.empty((M, K), dtype=torch.float16, device=dev)
        b16 = torch.empty((K, N), dtype=torch.float16, device=dev)

        def gemm(dA, dB, dC):
            bwgemm.quantize_f16(dA, a16, stream=stream)
            bwgemm.quantize_f16(dB, b16, stream=stream)
            bwgemm.gemm_f16(a16, b16, dC, stream=stream)

        e2e = run_e2e(hA, hB, M, N, K, dev, stream, gemm, args.steps, world, flops)
        e2e["path"] = "bw_quantize_f16 (A, B) + bw_gemm_f16 per step, the work launch_tc_f16 does for new inputs"
        del hA, hB, a16, b16

    if wl == "f16":
        peak = float(peaks.get("bf16_tflops", FALLBACK_PEAKS["bf16_tflops"]))
        peak_name = "bf16_tflops (burst, cuBLAS bf16 8192^3)"
    else:
        # no measured FP8/FP4 library peak in MEASURED_PEAKS.json: scale the measured bf16
        # figure by the nominal dense-rate ratio (2x FP8, 4x FP4)
        mult = 2.0 if wl == "fp8" else 4.0
        peak = mult * float(peaks.get("bf16_tflops", FALLBACK_PEAKS["bf16_tflops"]))
        peak_name = f"{mult:.0f} x bf16_tflops (burst)"
    achieved = tflops(flops, ms)
    traffic = profile_traffic({"f16": "bw_tc_gemm_pair_f16_8192", "fp8": "bw_tc_gemm_pair_fp8_8192",
                               "mxfp4": "bw_tc_gemm_pair_mxfp4_8192", "fp4": "bw_tc_gemm_pair_fp4_8192"}[wl])
    roofline = {"bound": "tensor", "achieved": round(achieved, 2), "peak": round(peak, 1), "unit": "TFLOP/s",
                "frac": round(achieved / peak, 4), "traffic": traffic,
                "peak_source": f"{peak_src}: {peak_name}",
                "algorithmic_flops_per_launch": flops}

    comparisons = {}
    if not args.no_compare and rank == 0 and world == 1 and wl == "f16":
        block = max(10, min(args.steps, 50))
        try:
            a, b = interleaved(step, lambda: torch.mm(A, B, out_dtype=torch.float32), block, stream, flops)
            comparisons = {"ours_f16_f32out_tflops": a, "cublas_f16_f32out_tflops": b, "block_steps": block}
        except Exception as ex:  # a missing library path must not hide the headline number
            comparisons = {"error": f"{type(ex).__name__}: {ex}"[:200]}
    del inp, C
    torch.cuda.empty_cache()

    precisions = None
    if world == 1 and wl == "f16" and not args.no_extra:
        precisions = run_precisions(args, dev, stream, peaks, peak_src)
        torch.cuda.empty_cache()
    sharded = None
    if not args.no_extra:
        sharded = run_sharded(args, world, rank, dev, stream)
    clocks.stop(time.monotonic())

    line = {
        "metric": METRIC,
        "value": round(value, 2), "unit": "TFLOP/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(ms, 4), "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": dtype, "data": "synthetic (seeded uniform[-1,1] rounded to FP16)" if wl == "f16"
        else "synthetic (seeded N(0,1), quantised on device)",
        "config": config_dict(wl, M, N, K, world),
        "e2e": e2e,
        "roofline": roofline,
        "gpu_launches": args.steps,
        "clocks": clk,
        "impl": "ours",
    }
    if sustained:
        line["sustained"] = sustained
    if comparisons:
        line["comparisons"] = comparisons
    if precisions:
        line["precisions"] = precisions
    if sharded:
        line["sharded"] = sharded
    if rank == 0 and world == 1 and not args.no_cpu:
        threads = os.cpu_count() or 1
        v, sample = cpu_baseline(threads)
        v1, t1 = cpu_full_1024(threads)
        line["cpu_baseline"] = {"value": round(v, 5), "unit": "TFLOP/s", "cores": threads, "kind": "port",
                                "sample": sample, "cpu": cpu_model(),
                                "full_1024": {"tflops": round(v1, 5), "seconds": round(t1, 3),
                                              "what": "the whole 1024^3 FP16 GEMM (configs[0]), FP64 oracle"}}
    return line


# ---------------------------------------------------------------------------------------
def run_reference(args, world, rank, local):
    """The reference's stock FP16 launcher (launch_mma_warptile) on the same workload, on every
    rank for its own shard (max over ranks), with the same e2e pipeline as our arm."""
    import ctypes

    import torch

    lib_path = os.path.join(ORACLE, "_ref", "libref_kernels.so")
    base = {"impl": "reference", "metric": METRIC}
    if not os.path.exists(lib_path):
        base["unavailable"] = "oracle/_ref/libref_kernels.so was not built (oracle/build_ref.sh needs the reference sources)"
        return base
    L = ctypes.CDLL(lib_path)
    L.ref_launch.argtypes = [ctypes.c_char_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int,
                             ctypes.c_int, ctypes.c_int]
    L.ref_launch.restype = ctypes.c_int
    dev = torch.device("cuda", local)
    # The reference's launchers run on the legacy default stream (src/main.cu:91-92).
    stream = torch.cuda.default_stream(dev)
    M, N, K = SHAPE
    flops = 2.0 * M * N * K
    name = b"mma_warptile"
    inp = make_inputs("f16", rank, dev)
    A = inp["A"].float().contiguous()
    B = inp["B"].float().contiguous()
    C = torch.empty((M, N), dtype=torch.float32, device=dev)

    def launch(a, b, c):
        rc = L.ref_launch(name, a.data_ptr(), b.data_ptr(), c.data_ptr(), M, N, K)
        if rc != 0:
            raise RuntimeError(f"reference launch failed: {rc}")

    with torch.cuda.stream(stream):
        clocks = ClockSampler(local)
        clocks.start()
        step = lambda: launch(A, B, C)  # noqa: E731
        for _ in range(args.warmup):
            step()
        torch.cuda.synchronize()
        mark = clocks.mark()
        ms = timed_steps(step, args.steps, 0, world, stream)
        clk = clocks.stop(mark)
        value = world * tflops(flops, ms)
        # e2e through the reference's API: FP32 host inputs -> device, launch (the two
        # alternating device buffer pairs make it re-stage FP16 every step), FP32 C -> host
        hA = torch.empty((M, K), dtype=torch.float32, pin_memory=True)
        hB = torch.empty((K, N), dtype=torch.float32, pin_memory=True)
        hA.copy_(A.cpu())
        hB.copy_(B.cpu())
        e2e = run_e2e(hA, hB, M, N, K, dev, stream, launch, args.steps, world, flops)
        e2e["path"] = "launch_mma_warptile per step (pointer-keyed staging re-casts: alternating buffers)"
    line = dict(base)
    line.update({
        "value": round(value, 2), "unit": "TFLOP/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(ms, 4), "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "f16", "data": "synthetic (seeded uniform[-1,1] rounded to FP16)",
        "config": config_dict("f16", M, N, K, world),
        "kernel": "reference launch_mma_warptile (mma.sync m16n8k16, built for sm_100a from its sources)",
        "reference_kind": "the reference has no CPU GEMM; its own implementation of the path is this GPU launcher",
        "e2e": e2e,
        "clocks": clk,
    })
    return line


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--workload", choices=["f16", "fp8", "mxfp4", "fp4"], default="f16")
    ap.add_argument("--shape", default=None, help="MxNxK per GPU (default 8192x8192x8192, BASELINE configs[1])")
    ap.add_argument("--no-extra", action="store_true", help="headline, e2e and comparisons only")
    ap.add_argument("--no-compare", action="store_true")
    ap.add_argument("--multicast", action="store_true",
                    help="also time the fused gather through NVSwitch multicast (multimem.st)")
    ap.add_argument("--no-cpu", action="store_true")
    args = ap.parse_args()
    if args.shape:
        SHAPE[:] = [int(x) for x in args.shape.lower().split("x")]
        args.no_cpu = True  # the CPU baseline is defined on the headline workload
        args.no_extra = True
    if args.warmup < 3:
        args.warmup = 3
    world, rank, local = dist_setup(args)
    if args.impl == "reference":
        line = run_reference(args, world, rank, local)
    else:
        line = run_ours(args, world, rank, local)
    if rank == 0:
        print(json.dumps(line), flush=True)
    if world > 1:
        import torch.distributed as dist

        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()

#!/usr/bin/env python3
"""Benchmark of the npu-ai offload hot path on B200: bf16 GEMM + fused attention TFLOP/s, and SD1.5 UNet steps/s.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
    python -m torch.distributed.run --nnodes=1 --nproc-per-node N --master-addr 127.0.0.1 --master-port P \
        bench.py --gpus N --steps K --warmup W

One step = one pass of the hot path over the SD1.5 workload the reference quotes its GEMM and attention numbers
on (synthetic, seeded inputs of those shapes and distributions; the reference publishes no dataset for it):
  * the fused attention blocks: self-attention (2, 8, 4096, 4096, 40), (2, 8, 1024, 1024, 80),
    (2, 8, 256, 256, 160) and cross-attention (2, 8, 4096, 77, 40) as (B, H, Sq, Skv, d), q/k/v ~ N(0,1),
    scale d^-0.5, all batch x head pairs in one launch each (4 launches);
  * the shape-agnostic GEMM sweep: M in {77, 154, 256, 1024, 4096, 8192} x 11 SD1.5 (K, N) Linear shapes,
    x ~ N(0,1), W ~ N(0, 0.02^2), b ~ N(0, 0.01^2), bf16 operands, f32 accumulation, bf16 out (66 launches).
Metric: total algorithmic FLOPs (2MKN per GEMM, 4 B H Sq Skv d per attention block, the reference's own counts)
per second, whole job. Multi-GPU (torchrun, one rank per GPU): weak scaling. The GEMMs do not shard (a single
Linear is microseconds; every rank runs its own replica of the sweep); the attention blocks shard over batch x
head pairs: rank r owns batches [2r, 2r+2) of a (2N, ...) block and the outputs are all-gathered over NCCL on a
communication stream while the GEMM sweep runs.

Reported in the same JSON line:
  * roofline: the dominant kernel (GEMM) against the measured burst bf16 peak, per sweep M group, config 1
    (4096x320x320 with bias, bf16 out) as a standalone launch sequence over rotating buffers larger than L2
    against its HBM roofline, and every attention block with its exponential-unit floor;
  * e2e: the same step end to end through the public API (NpuGemm with pinned host buffers, host<->device copies
    of inputs, biases and results inside the timed region);
  * unet: SD1.5-architecture UNet (random init) Euler CFG denoise steps at batch 16 (8 prompts x CFG) on 64x64
    and 128x128 latents, the batch sharded over the N ranks with latents all-gathered every step; at N = 1 also
    batch 2 (one prompt, 4 Euler steps per image) and the host CPU's batch-2 UNet call;
  * cpu_baseline: the reference's CPU fallback (F.linear / SDPA in f32 on bf16-rounded inputs) on a bounded
    sample of the step, on the host cores;
  * clocks: SM clock, power and throttle reasons sampled through NVML every ~1 ms during the timed region.
`--impl reference` times that CPU path alone on the whole 70-op step, with all host threads.

Other modes (not the driver's line):
  --workload unet [--batch B --latent L [--kernel-times]]  only the UNet leg, on one configuration; --kernel-times
      prints the step's device time per kernel kind to stderr.
  --case KIND:dims  one kernel on one shape (gemm, attn, geglu, conv, gn, ln, up, cat), the small cases the ncu
      summaries use.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time

import torch

ROOT = os.path.dirname(os.path.abspath(__file__))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

METRIC = "bf16 GEMM & fused-attn TFLOP/s"
WORKLOAD = "sd15-linear-sweep+attention-blocks"
SD15_M = [77, 154, 256, 1024, 4096, 8192]
SD15_KN = [(320, 320), (320, 2560), (1280, 320), (768, 320), (640, 640), (640, 5120), (2560, 640), (1280, 1280),
           (1280, 10240), (5120, 1280), (768, 1280)]
ATTN_BLOCKS = [(2, 8, 4096, 4096, 40), (2, 8, 1024, 1024, 80), (2, 8, 256, 256, 160), (2, 8, 4096, 77, 40)]
CONFIG1 = (4096, 320, 320)  # single SD1.5 to_q Linear at the 64x64 latent
L2_BYTES = 126 * 2**20
SMS = 148
EX2_PER_CLK_PER_SM = 16  # MUFU exponentials per clock per SM (measured with a probe kernel)

# DRAM traffic per launch of the dominant kernel (GEMM, mean over the 66 sweep launches of one step) from the ncu
# capture summarised in profiles/gemm_sweep_dram.md; null when that capture predates the current GEMM kernel.
GEMM_DRAM_BYTES_PER_LAUNCH = 14441336


def _peaks() -> dict:
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return {"hbm_gbs": float(p["hbm_gbs"]), "bf16_tflops": float(p["bf16_tflops"]),
                "bf16_tflops_sustained": float(p.get("bf16_tflops_sustained", p["bf16_tflops"])),
                "sm_max_mhz": float(p.get("sm_max_mhz", 1965.0)), "source": "measured"}
    except (OSError, KeyError, ValueError):
        return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0, "sm_max_mhz": 1965.0,
                "source": "fallback"}


def hotpath_config(world: int) -> dict:
    """The `config` of the hot-path line; the reference arm prints the same object."""
    step_bytes = sum(2 * (M * K + N * K + N + M * N) for M, K, N in gemm_shapes()) + \
        sum(2 * B * H * D * (2 * Sq + 2 * Skv) for B, H, Sq, Skv, D in ATTN_BLOCKS)
    return {"workload": WORKLOAD,
            "gemm_shapes": "M{77,154,256,1024,4096,8192} x 11 SD1.5 (K,N), bf16 out, bias",
            "attention_blocks": ATTN_BLOCKS, "per_rank_attention_batch": 2,
            "parallelism": f"replicas(gemm)+pairs-sharded(attention) x{world}",
            "l2": f"inputs larger than L2: {step_bytes / 2**20:.0f} MiB touched once per step vs "
                  f"{L2_BYTES / 2**20:.0f} MiB L2"}


# ----------------------------------------------------------------------------------------------------------------
# distributed plumbing
# ----------------------------------------------------------------------------------------------------------------
class Dist:
    def __init__(self, use_cuda: bool):
        self.world = int(os.environ.get("WORLD_SIZE", "1"))
        self.rank = int(os.environ.get("RANK", "0"))
        self.local_rank = int(os.environ.get("LOCAL_RANK", "0"))
        self.pg = None
        if self.world > 1:
            import datetime
            import torch.distributed as dist
            if use_cuda:
                torch.cuda.set_device(self.local_rank)
            dist.init_process_group("nccl" if use_cuda else "gloo", timeout=datetime.timedelta(seconds=120),
                                    device_id=torch.device("cuda", self.local_rank) if use_cuda else None)
            self.pg = dist

    def barrier(self):
        if self.pg is not None:
            self.pg.barrier()

    def max(self, x: float, device) -> float:
        if self.pg is None:
            return x
        t = torch.tensor([x], dtype=torch.float64, device=device)
        self.pg.all_reduce(t, op=self.pg.ReduceOp.MAX)
        return float(t.item())

    def close(self):
        if self.pg is not None:
            self.pg.barrier()
            self.pg.destroy_process_group()


# ----------------------------------------------------------------------------------------------------------------
# clocks
# ----------------------------------------------------------------------------------------------------------------
class ClockSampler:
    """SM clock, power and throttle-reason samples of this rank's GPU, read (never set) through NVML every ~1 ms
    on a background thread, so even a timed region of a few tens of milliseconds holds 20+ samples; falls back to
    `nvidia-smi -lms 200` where NVML is unavailable. Windows are marked on the host clock."""
    NAMES = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")
    FIELDS = ("uuid,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.hw_slowdown,"
              "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
              "clocks_event_reasons.sw_power_cap")

    def __init__(self, uuid: str, period_s: float = 0.001):
        self.uuid = uuid
        self.period_s = period_s
        self.samples: list[tuple] = []   # (host time, sm MHz, max sm MHz, power W, {reason names})
        self.source = None
        self._stop = threading.Event()
        self.proc = None
        self.thread = None

    def _start_nvml(self) -> bool:
        try:
            import pynvml
            pynvml.nvmlInit()
            h = pynvml.nvmlDeviceGetHandleByUUID(self.uuid)
            max_sm = float(pynvml.nvmlDeviceGetMaxClockInfo(h, pynvml.NVML_CLOCK_SM))
        except Exception:  # noqa: BLE001 - any NVML failure selects the nvidia-smi sampler
            return False
        bits = {"hw_slowdown": pynvml.nvmlClocksThrottleReasonHwSlowdown,
                "hw_thermal_slowdown": pynvml.nvmlClocksThrottleReasonHwThermalSlowdown,
                "sw_thermal_slowdown": pynvml.nvmlClocksThrottleReasonSwThermalSlowdown,
                "sw_power_cap": pynvml.nvmlClocksThrottleReasonSwPowerCap}

        def loop():
            while not self._stop.is_set():
                try:
                    sm = float(pynvml.nvmlDeviceGetClockInfo(h, pynvml.NVML_CLOCK_SM))
                    pw = pynvml.nvmlDeviceGetPowerUsage(h) / 1000.0
                    rs = pynvml.nvmlDeviceGetCurrentClocksThrottleReasons(h)
                except Exception:  # noqa: BLE001
                    break
                self.samples.append((time.perf_counter(), sm, max_sm, pw, {n for n, b in bits.items() if rs & b}))
                time.sleep(self.period_s)
        self.source = f"NVML every {self.period_s * 1e3:.0f} ms"
        self.thread = threading.Thread(target=loop, daemon=True)
        self.thread.start()
        return True

    def start(self):
        if self._start_nvml():
            return
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                                          "-lms", "200"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None
            return
        want = self.uuid.lower().replace("gpu-", "")
        num = lambda v: float(v) if v.replace(".", "", 1).isdigit() else float("nan")  # noqa: E731

        def reader():
            for line in self.proc.stdout:
                p = [x.strip() for x in line.split(",")]
                if len(p) == 8 and p[0].lower().replace("gpu-", "") == want:
                    self.samples.append((time.perf_counter(), num(p[1]), num(p[2]), num(p[3]),
                                         {n for n, v in zip(self.NAMES, p[4:]) if v.lower() == "active"}))
        self.source = "nvidia-smi -lms 200"
        self.thread = threading.Thread(target=reader, daemon=True)
        self.thread.start()

    def stop(self) -> None:
        self._stop.set()
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
        if self.thread is not None:
            self.thread.join(timeout=2)

    def summary(self, t_begin: float, t_end: float, window: str) -> dict:
        if self.source is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["clock sampling unavailable"], "samples": 0}
        mine = [s for s in list(self.samples) if t_begin <= s[0] <= t_end]
        sm = [s[1] for s in mine if s[1] == s[1]]
        pw = [s[3] for s in mine if s[3] == s[3]]
        return {"sm_mhz": statistics.median(sm) if sm else None,
                "sm_max_mhz": max(s[2] for s in mine) if mine else None,
                "reasons": sorted(set().union(*[s[4] for s in mine])) if mine else [],
                "samples": len(mine), "power_w_median": statistics.median(pw) if pw else None,
                "window": window, "source": self.source}


def _gpu_uuid(dev: int) -> str:
    try:
        return "GPU-" + str(torch.cuda.get_device_properties(dev).uuid)
    except Exception:
        return ""


# ----------------------------------------------------------------------------------------------------------------
# workload
# ----------------------------------------------------------------------------------------------------------------
def gemm_shapes():
    return [(M, K, N) for M in SD15_M for (K, N) in SD15_KN]


def step_flops() -> tuple[float, float]:
    """(GEMM, attention) algorithmic FLOPs of one rank's step."""
    g = sum(2.0 * M * K * N for M, K, N in gemm_shapes())
    a = sum(4.0 * B * H * Sq * Skv * D for B, H, Sq, Skv, D in ATTN_BLOCKS)
    return g, a


def _seeded(shape, std, seed, device, dtype=torch.bfloat16):
    g = torch.Generator(device="cpu").manual_seed(seed)
    t = torch.randn(*shape, generator=g) * std
    return t.to(device=device, dtype=dtype)


def _gemm_seed(rank: int, i: int) -> int:
    return 1000 * rank + 3 * i


def _attn_seed(rank: int, j: int) -> int:
    return 500000 + 1000 * rank + 7 * j


class GpuWorkload:
    def __init__(self, device: torch.device, rank: int, world: int):
        from npu_ai_b200 import kernels
        self.k = kernels
        self.device = device
        self.world = world
        self.gemms = []
        for i, (M, K, N) in enumerate(gemm_shapes()):
            s = _gemm_seed(rank, i)
            x = _seeded((M, K), 1.0, s, device)
            w = _seeded((N, K), 0.02, s + 1, device)
            b = _seeded((N,), 0.01, s + 2, device)
            out = torch.empty((M, N), dtype=torch.bfloat16, device=device)
            h = kernels.register_weight(w)
            self.gemms.append((x, w, b, out, h, 2.0 * M * K * N, 2 * (M * K + N * K + N + M * N)))
        self.attn = []
        # The attention outputs are views of one flat buffer, so with N > 1 ranks one all-gather per step (after the
        # last block) moves them all: rank r's outputs land at [r * n, (r + 1) * n) of `attn_full`.
        sizes = [B * Sq * H * D for (B, H, Sq, Skv, D) in ATTN_BLOCKS]
        self.attn_out = torch.empty(sum(sizes), dtype=torch.bfloat16, device=device)
        self.attn_full = torch.empty(world * sum(sizes), dtype=torch.bfloat16, device=device) if world > 1 else None
        off = 0
        for j, (B, H, Sq, Skv, D) in enumerate(ATTN_BLOCKS):
            s = _attn_seed(rank, j)
            q = _seeded((B, Sq, H * D), 1.0, s, device)
            kk = _seeded((B, Skv, H * D), 1.0, s + 1, device)
            v = _seeded((B, Skv, H * D), 1.0, s + 2, device)
            out = self.attn_out[off:off + sizes[j]].view(B, Sq, H * D)
            off += sizes[j]
            self.attn.append((q, kk, v, out, H, 4.0 * B * H * Sq * Skv * D))
        self.comm = torch.cuda.Stream(device) if world > 1 else None

    def step(self, dist, events=None):
        """One pass: the attention blocks, then the GEMM sweep in M order. With N > 1 ranks the attention outputs are
        all-gathered (one NCCL call for all four) on the communication stream while the sweep runs; the step joins
        it at the end.

        `events` (see make_events) marks the start of every attention block, the start of every M group of the
        sweep and the end of the step. Only boundaries carry an event, so launches inside an M group keep their
        programmatic-dependent-launch overlap."""
        k = self.k
        main = torch.cuda.current_stream(self.device)
        ei = 0
        for (q, kk, v, out, H, _) in self.attn:
            if events is not None:
                events[ei].record()
                ei += 1
            k.attention(q, kk, v, H, out=out)
        if self.attn_full is not None:
            self.comm.wait_stream(main)
            with torch.cuda.stream(self.comm):
                dist.pg.all_gather_into_tensor(self.attn_full, self.attn_out)
        group = None
        for (x, w, b, out, h, _, _) in self.gemms:
            if events is not None and x.shape[0] != group:
                group = x.shape[0]
                events[ei].record()
                ei += 1
            k.gemm(x, w, b, out=out, handle=h)
        if self.comm is not None:
            main.wait_stream(self.comm)
        if events is not None:
            events[ei].record()

    def m_groups(self) -> list[int]:
        return list(dict.fromkeys(g[0].shape[0] for g in self.gemms))

    def make_events(self) -> list:
        """[start of attention block 0..3, start of M group 0..5, end of step]"""
        return [torch.cuda.Event(enable_timing=True, external=True)
                for _ in range(len(self.attn) + len(self.m_groups()) + 1)]

    def capture(self, dist, events=None) -> torch.cuda.CUDAGraph:
        """One step captured as a CUDA graph (kernels launched back to back by the GPU, no host in the loop). The
        capture stream runs one eager step first so its per-stream workspace exists before capture."""
        if not hasattr(self, "_capture_stream"):
            self._capture_stream = torch.cuda.Stream(self.device)
            self._capture_stream.wait_stream(torch.cuda.current_stream(self.device))
            with torch.cuda.stream(self._capture_stream):
                self.step(dist)
            torch.cuda.current_stream(self.device).wait_stream(self._capture_stream)
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=self._capture_stream):
            self.step(dist, events)
        return g

    def launches_per_step(self) -> int:
        return len(self.gemms) + len(self.attn)

    def release(self):
        for g in self.gemms:
            self.k.release_weight(g[4])


class E2EWorkload:
    """The same step through the public API (NpuGemm) with pinned host inputs, biases and outputs."""

    def __init__(self, device: torch.device, rank: int, world: int):
        from npu_ai_b200.runner import NpuGemm
        self.rt = NpuGemm(device=device, verbose=False, out_dtype=torch.bfloat16)
        self.device = device
        self.world = world
        self.gemms = []
        self.h2d = 0
        self.d2h = 0
        for i, (M, K, N) in enumerate(gemm_shapes()):
            s = _gemm_seed(rank, i)
            x = _seeded((M, K), 1.0, s, "cpu").pin_memory()
            w = self.rt.upload_weight(_seeded((N, K), 0.02, s + 1, "cpu"), layout="nk")
            b = _seeded((N,), 0.01, s + 2, "cpu").pin_memory()
            y = torch.empty((M, N), dtype=torch.bfloat16).pin_memory()
            self.gemms.append((x, w, b, y))
            self.h2d += (x.numel() + b.numel()) * 2
            self.d2h += y.numel() * 2
        self.attn = []
        for j, (B, H, Sq, Skv, D) in enumerate(ATTN_BLOCKS):
            s = _attn_seed(rank, j)
            q, kk, v = (_seeded((B, S, H * D), 1.0, s + t, "cpu").pin_memory()
                        for t, S in ((0, Sq), (1, Skv), (2, Skv)))
            y = torch.empty((B * world, Sq, H * D), dtype=torch.bfloat16).pin_memory()
            full = torch.empty((B * world, Sq, H * D), dtype=torch.bfloat16, device=device) if world > 1 else None
            self.attn.append((q, kk, v, H, y, full))
            self.h2d += (q.numel() + kk.numel() + v.numel()) * 2
            self.d2h += y.numel() * 2

    def _out(self, o, y):
        """Result o (on the current stream) back to pinned host y on the copy-out stream, so the device-to-host
        transfer overlaps the next ops' host-to-device copies and kernels (PCIe is full duplex)."""
        ev = torch.cuda.Event()
        ev.record(torch.cuda.current_stream(self.device))
        self.d2h_stream.wait_event(ev)
        with torch.cuda.stream(self.d2h_stream):
            y.copy_(o, non_blocking=True)
        o.record_stream(self.d2h_stream)

    def step(self, dist):
        rt = self.rt
        if not hasattr(self, "d2h_stream"):
            self.d2h_stream = torch.cuda.Stream(self.device)
        for (q, kk, v, H, y, full) in self.attn:
            o = rt.attention(q, kk, v, H)
            if full is not None:
                dist.pg.all_gather_into_tensor(full, o)
                o = full
            self._out(o, y)
        for (x, w, b, y) in self.gemms:
            self._out(rt.linear(x, w, b), y)  # host x and bias -> device, and the GEMM, on the current stream
        # The step ends when the last result is in host memory.
        torch.cuda.current_stream(self.device).wait_stream(self.d2h_stream)


# ----------------------------------------------------------------------------------------------------------------
# CPU path (the reference's CPU fallback semantics, via the oracle)
# ----------------------------------------------------------------------------------------------------------------
def _cpu_ops():
    """The step's 70 ops in a fixed interleaved order (large and small alternate, so a prefix is representative).
    Each op carries the seed its GPU counterpart uses on rank 0."""
    ops = [("gemm", s, _gemm_seed(0, i)) for i, s in enumerate(gemm_shapes())] + \
        [("attn", a, _attn_seed(0, j)) for j, a in enumerate(ATTN_BLOCKS)]
    ops.sort(key=lambda o: (o[1][0] * o[1][1] * o[1][2]) if o[0] == "gemm" else o[1][2] * o[1][3] * o[1][4] * 16)
    inter = []
    lo, hi = 0, len(ops) - 1
    while lo <= hi:
        inter.append(ops[hi])
        if lo != hi:
            inter.append(ops[lo])
        lo, hi = lo + 1, hi - 1
    return inter


def _cpu_inputs(op):
    kind, shp, seed = op
    if kind == "gemm":
        M, K, N = shp
        return (_seeded((M, K), 1.0, seed, "cpu"), _seeded((N, K), 0.02, seed + 1, "cpu"),
                _seeded((N,), 0.01, seed + 2, "cpu"))
    B, H, Sq, Skv, D = shp
    return (_seeded((B, Sq, H * D), 1.0, seed, "cpu"), _seeded((B, Skv, H * D), 1.0, seed + 1, "cpu"),
            _seeded((B, Skv, H * D), 1.0, seed + 2, "cpu"))


def _cpu_run(op, inputs) -> tuple[float, float]:
    """Run one op of the step on the host cores: (seconds, algorithmic FLOPs)."""
    from oracle import attention_ref, linear_ref
    kind, shp, _ = op
    t0 = time.perf_counter()
    if kind == "gemm":
        linear_ref(*inputs)
        M, K, N = shp
        return time.perf_counter() - t0, 2.0 * M * K * N
    B, H, Sq, Skv, D = shp
    attention_ref(*inputs, H)
    return time.perf_counter() - t0, 4.0 * B * H * Sq * Skv * D


def cpu_baseline(budget_s: float = 20.0) -> dict:
    """One pass over the step's ops on the host cores (stops early past the time budget)."""
    torch.set_num_threads(os.cpu_count() or 1)
    warm = ("gemm", (64, 64, 64), 1)
    _cpu_run(warm, _cpu_inputs(warm))
    tot_t = tot_f = 0.0
    n = 0
    ops = _cpu_ops()
    for op in ops:
        dt, fl = _cpu_run(op, _cpu_inputs(op))
        tot_t += dt
        tot_f += fl
        n += 1
        if tot_t > budget_s:
            break
    return {"value": round(tot_f / tot_t / 1e12, 4), "unit": "TFLOP/s", "cores": torch.get_num_threads(),
            "kind": "port",
            "sample": f"{n} of the step's {len(ops)} ops (interleaved large/small), torch CPU F.linear / SDPA in f32 "
                      f"on bf16-rounded inputs (the reference's CPU fallback), {tot_f / 1e9:.0f} GFLOP in {tot_t:.1f} s"}


def run_reference(args) -> None:
    """--impl reference: the reference's CPU path (the oracle port: F.linear / SDPA in f32 on bf16-rounded inputs,
    the reference's CPU fallback) on the host cores. Each bench step is the whole 70-op hot-path step on the same
    seeded inputs as the GPU arm's rank 0; inputs are generated once, outside the timed region."""
    torch.set_num_threads(os.cpu_count() or 1)
    ops = _cpu_ops()
    inputs = [_cpu_inputs(op) for op in ops]
    warm = ("gemm", (64, 64, 64), 1)
    _cpu_run(warm, _cpu_inputs(warm))
    for _ in range(args.warmup):
        for op, inp in zip(ops, inputs):
            _cpu_run(op, inp)
    tot_t = tot_f = 0.0
    for _ in range(args.steps):
        for op, inp in zip(ops, inputs):
            dt, fl = _cpu_run(op, inp)
            tot_t += dt
            tot_f += fl
    value = tot_f / tot_t / 1e12
    n = args.steps
    sample = (f"the whole {len(ops)}-op step ({tot_f / n / 1e9:.0f} GFLOP) per bench step: torch CPU F.linear / SDPA "
              "in f32 on bf16-rounded inputs, the reference's CPU fallback (comfyui node :151, "
              "scripts/11-attn-fused-test.py:115-119)")
    line = {"metric": METRIC, "value": round(value, 4), "unit": "TFLOP/s", "n_gpus": args.gpus, "steps": n,
            "warmup": args.warmup, "ms_per_step": round(tot_t / n * 1e3, 3), "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "f32 (bf16-rounded inputs)", "data": "synthetic",
            "impl": "reference", "config": hotpath_config(args.gpus),
            "cpu_baseline": {"value": round(value, 4), "unit": "TFLOP/s", "cores": torch.get_num_threads(),
                             "kind": "port", "sample": sample},
            "e2e": {"value": round(value, 4), "unit": "TFLOP/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


# ----------------------------------------------------------------------------------------------------------------
# our arm
# ----------------------------------------------------------------------------------------------------------------
def _time_graph(g: torch.cuda.CUDAGraph, replays: int) -> float:
    """ms per replay of a graph, CUDA events on the current stream."""
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(replays):
        g.replay()
    e1.record()
    torch.cuda.synchronize()
    return e0.elapsed_time(e1) / replays


def config1_roofline(device, peaks) -> dict:
    """Config 1 (x [4096x320] . W[320x320]^T + b, bf16 out) as a standalone sequence: 48 launches over rotating x
    and out buffers (252 MB, twice the L2) with one resident weight, captured as a CUDA graph (PDL between the
    launches, as in a model's chain of Linears)."""
    from npu_ai_b200 import kernels
    M, K, N = CONFIG1
    copies = 48
    xs = [_seeded((M, K), 1.0, 77 + i, device) for i in range(copies)]
    outs = [torch.empty((M, N), dtype=torch.bfloat16, device=device) for _ in range(copies)]
    w = _seeded((N, K), 0.02, 7, device)
    b = _seeded((N,), 0.01, 8, device)
    h = kernels.register_weight(w)
    s = torch.cuda.Stream(device)
    s.wait_stream(torch.cuda.current_stream(device))
    with torch.cuda.stream(s):
        for x, o in zip(xs, outs):
            kernels.gemm(x, w, b, out=o, handle=h)
    torch.cuda.current_stream(device).wait_stream(s)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=s):
        for x, o in zip(xs, outs):
            kernels.gemm(x, w, b, out=o, handle=h)
    for _ in range(3):
        g.replay()
    us = _time_graph(g, 10) * 1e3 / copies
    kernels.check_status(device)
    del g
    kernels.release_weight(h)
    flops = 2.0 * M * K * N
    nbytes = 2 * (M * K + N * K + N + M * N)
    ideal_us = nbytes / (peaks["hbm_gbs"] * 1e3)
    return {"shape": "4096x320x320 + bias, bf16 out", "us": round(us, 3), "tflops": round(flops / us / 1e6, 1),
            "gbs": round(nbytes / us / 1e3, 1), "hbm_roofline_us": round(ideal_us, 3),
            "frac_of_roofline": round(ideal_us / us, 4), "bound": "hbm",
            "timing": f"CUDA graph of {copies} launches over rotating buffers ({copies * 2 * M * K * 2 / 2**20:.0f} MiB "
                      "of x and out, larger than L2), 10 replays, CUDA events"}


def run_ours(args, dist) -> None:
    from npu_ai_b200 import kernels
    device = torch.device("cuda", dist.local_rank)
    torch.cuda.set_device(device)
    peaks = _peaks()
    wl = GpuWorkload(device, dist.rank, dist.world)
    for _ in range(max(3, args.warmup)):
        wl.step(dist)
    torch.cuda.synchronize()
    kernels.check_status(device)

    sampler = ClockSampler(_gpu_uuid(dist.local_rank)) if dist.rank == 0 else None
    if sampler is not None:
        sampler.start()
    # The step runs as a CUDA graph. A twin graph carries timing events at the attention-block and GEMM M-group
    # boundaries; it runs as the last step of the timed region.
    graph = wl.capture(dist)
    events = wl.make_events()
    graph_ev = wl.capture(dist, events)
    for _ in range(2):
        graph.replay()
    graph_ev.replay()
    torch.cuda.synchronize()
    kernels.check_status(device)
    # Optional soak (--soak-s, default none): step replays right before the timed region, e.g. to time the step in
    # the GPU's power-capped steady state (every rank replays the same count: the graphs hold collectives).
    soak = 0
    if args.soak_s > 0:
        one = _time_graph(graph, 3)
        soak = int(dist.max(float(min(20000, max(10, round(args.soak_s * 1e3 / max(one, 1e-3))))), device))
    dist.barrier()
    torch.cuda.synchronize()
    for _ in range(soak):
        graph.replay()
    t_begin = time.perf_counter()
    t0 = torch.cuda.Event(enable_timing=True)
    t1 = torch.cuda.Event(enable_timing=True)
    t0.record()
    for _ in range(args.steps - 1):
        graph.replay()
    graph_ev.replay()
    t1.record()
    torch.cuda.synchronize()
    t_end = time.perf_counter()
    dist.barrier()
    clocks = sampler.summary(t_begin, t_end, "the timed region" + (f", after a soak of {soak} step replays"
                                                                  if soak else "")) if sampler is not None else None
    kernels.check_status(device)
    ms_local = t0.elapsed_time(t1) / args.steps
    ms = dist.max(ms_local, device)
    gflops, aflops = step_flops()
    total = (gflops + aflops) * dist.world
    value = total / (ms / 1e3) / 1e12

    na = len(wl.attn)
    groups = wl.m_groups()
    seg = [events[i].elapsed_time(events[i + 1]) for i in range(len(events) - 1)]
    attn_ms = sum(seg[:na])
    gemm_ms = sum(seg[na:])
    peak = peaks["bf16_tflops"]
    hbm = peaks["hbm_gbs"]
    by_m = {}
    for gi, M in enumerate(groups):
        g_ms = seg[na + gi]
        mine = [g for g in wl.gemms if g[0].shape[0] == M]
        g_fl = sum(g[5] for g in mine)
        ideal_ms = sum(max(g[5] / (peak * 1e12), g[6] / (hbm * 1e9)) for g in mine) * 1e3
        by_m[str(M)] = {"us": round(g_ms * 1e3, 1), "tflops": round(g_fl / (g_ms / 1e3) / 1e12, 1),
                        "frac": round(g_fl / (g_ms / 1e3) / 1e12 / peak, 4),
                        "frac_of_roofline": round(ideal_ms / g_ms, 4),
                        "roofline_bound": "tensor" if all(g[5] / peak / 1e3 >= g[6] / hbm for g in mine) else
                        ("hbm" if all(g[5] / peak / 1e3 < g[6] / hbm for g in mine) else "mixed")}
    attn_blocks = {}
    for j, (B, H, Sq, Skv, D) in enumerate(ATTN_BLOCKS):
        a_ms = seg[j]
        fl = 4.0 * B * H * Sq * Skv * D
        mufu_us = B * H * Sq * Skv / (SMS * EX2_PER_CLK_PER_SM * peaks["sm_max_mhz"] * 1e6) * 1e6
        attn_blocks[f"{B}x{H}x{Sq}x{Skv}x{D}"] = {
            "us": round(a_ms * 1e3, 1), "tflops": round(fl / (a_ms / 1e3) / 1e12, 1),
            "frac": round(fl / (a_ms / 1e3) / 1e12 / peak, 4), "mufu_floor_us": round(mufu_us, 1),
            "bytes": 2 * B * H * D * (2 * Sq + 2 * Skv)}

    gemm_bytes = sum(g[6] for g in wl.gemms)
    achieved = gflops / (gemm_ms / 1e3) / 1e12
    roofline = {"bound": "tensor", "achieved": round(achieved, 1), "peak": peak, "unit": "TFLOP/s",
                "frac": round(achieved / peak, 4),
                "peak_kind": f"{peaks['source']} burst bf16 (cuBLAS 8192^3, best of 10): the timed region is "
                             f"{args.steps} steps of about {ms:.2f} ms" + (" after a soak" if soak else ""),
                "frac_of_sustained": round(achieved / peaks["bf16_tflops_sustained"], 4),
                "kernel": "gemm_bf16_tcgen05_kernel (66 sweep launches per step)",
                "algorithmic_bytes_per_launch": int(gemm_bytes / len(wl.gemms)),
                "traffic": GEMM_DRAM_BYTES_PER_LAUNCH,
                "traffic_source": "ncu dram__bytes_read.sum + dram__bytes_write.sum, mean per sweep launch "
                                  "(profiles/gemm_sweep_dram.md)",
                "gemm_launch_us": round(gemm_ms * 1e3 / len(wl.gemms), 3),
                "gemm_ms_per_step": round(gemm_ms, 4),
                "attention_ms_per_step": round(attn_ms, 4),
                "gemm_by_m": by_m,
                "gemm_tflops": round(achieved, 1),
                "attention_tflops": round(aflops / (attn_ms / 1e3) / 1e12, 1),
                "attention_blocks": attn_blocks,
                "config1": config1_roofline(device, peaks),
                "timing": "CUDA events at the attention-block and GEMM M-group boundaries of the timed region's "
                          "last step (graph replay); average launch duration = segment time / launches"}

    e2e = None if args.no_e2e else run_e2e(args, dist, device, total)
    roofline["attention_sharded"] = sharded_attention_leg(dist, device)
    kernels.check_status(device)
    del graph, graph_ev  # graphs holding NCCL calls go before the process group
    wl.release()
    del wl
    torch.cuda.empty_cache()

    unet = None if args.no_unet else unet_leg(args, dist, device, sampler)
    if sampler is not None:
        sampler.stop()

    cpu = cpu_baseline() if (dist.rank == 0 and dist.world == 1 and not args.no_cpu) else None
    if dist.rank == 0:
        line = {"metric": METRIC, "value": round(value, 2), "unit": "TFLOP/s", "n_gpus": dist.world,
                "steps": args.steps, "warmup": max(3, args.warmup), "ms_per_step": round(ms, 4),
                "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
                "data": "synthetic", "config": hotpath_config(dist.world),
                "gpu_launches": (len(ATTN_BLOCKS) + len(gemm_shapes())) * args.steps,
                "execution": "CUDA graph of the step (PDL between kernels), replayed per step",
                "roofline": roofline, "e2e": e2e, "cpu_baseline": cpu, "clocks": clocks, "unet": unet}
        print(json.dumps(line), flush=True)


def sharded_attention_leg(dist, device, reps: int = 10) -> dict:
    """One fixed attention block (the 64x64-latent self-attention, (2, 8, 4096, 4096, 40)) split over the ranks
    by (batch, head) pairs (npu_ai_b200.sharding): every rank holds the whole block, runs the fused kernel on its
    contiguous pair range, and one NCCL all-gather assembles the (B, Sq, H*d) result on every rank. Strong
    scaling of one block; the all-gather and the head-major -> (B, Sq, H*d) relayout are reported apart from the
    kernel time, against the unsharded launch on one GPU. Device times (CUDA events), median over `reps` calls,
    max over ranks. Each timed call is queued behind a ~100 us spin on the stream, so the host's launch work
    (argument checks, tensor maps, the NCCL call) is done before the GPU reaches the first event: the events bracket
    device time only."""
    from npu_ai_b200 import kernels
    from npu_ai_b200.sharding import attention_sharded, pair_width, resolve_timings
    B, H, Sq, Skv, D = ATTN_BLOCKS[0]
    q, k, v = (_seeded((B, S, H * D), 1.0, 900 + i, device) for i, S in ((0, Sq), (1, Skv), (2, Skv)))
    out = torch.empty((B, Sq, H * D), dtype=torch.bfloat16, device=device)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    one = []
    for i in range(reps + 3):
        torch.cuda._sleep(200_000)
        e0.record()
        kernels.attention(q, k, v, H, out=out)
        e1.record()
        torch.cuda.synchronize()
        if i >= 3:
            one.append(e0.elapsed_time(e1))
    res = {"block": [B, H, Sq, Skv, D], "ranks": dist.world, "unsharded_us": round(statistics.median(one) * 1e3, 1)}
    if dist.world == 1:
        return res
    parts = []
    for i in range(reps + 3):
        tm = {}
        torch.cuda._sleep(200_000)
        attention_sharded(q, k, v, H, timings=tm, out_dtype=torch.bfloat16)
        r = resolve_timings(tm)
        if i >= 3:
            parts.append(r)
    kern = dist.max(statistics.median(p["kernel_ms"] for p in parts), device)
    gath = dist.max(statistics.median(p["gather_ms"] for p in parts), device)
    rel = dist.max(statistics.median(p["relayout_ms"] for p in parts), device)
    total = kern + gath + rel
    res.update({"pairs_per_rank": pair_width(B * H, dist.world), "kernel_us": round(kern * 1e3, 1),
                "gather_us": round(gath * 1e3, 1), "relayout_us": round(rel * 1e3, 1),
                "total_us": round(total * 1e3, 1), "speedup_vs_unsharded": round(statistics.median(one) / total, 3),
                "gather_bytes_per_rank": parts[0]["gather_bytes_per_rank"],
                "note": "the scatter is free (inputs resident on every rank); the gather moves (N-1)/N of the output"})
    return res


def run_e2e(args, dist, device, total_flops) -> dict:
    e2e_wl = E2EWorkload(device, dist.rank, dist.world)
    e2e_steps = max(2, min(args.steps, 5))
    e2e_wl.step(dist)
    torch.cuda.synchronize()
    dist.barrier()
    torch.cuda.synchronize()
    s0 = torch.cuda.Event(enable_timing=True)
    s1 = torch.cuda.Event(enable_timing=True)
    s0.record()
    for _ in range(e2e_steps):
        e2e_wl.step(dist)
    s1.record()
    torch.cuda.synchronize()
    dist.barrier()
    e2e_ms = dist.max(s0.elapsed_time(s1) / e2e_steps, device)
    return {"value": round(total_flops / (e2e_ms / 1e3) / 1e12, 3), "unit": "TFLOP/s",
            "h2d_bytes_per_step": int(e2e_wl.h2d), "d2h_bytes_per_step": int(e2e_wl.d2h),
            "ms_per_step": round(e2e_ms, 3), "steps": e2e_steps,
            "api": "npu_ai_b200.runner.NpuGemm.linear / .attention",
            "copies": "host inputs and biases copied by the API on the compute stream; results copied out on a second "
                      "stream, overlapping the next ops"}


# ----------------------------------------------------------------------------------------------------------------
# UNet: SD1.5-architecture UNet denoise steps (batch 16 sharded over the ranks; batch 2 with 4 Euler steps)
# ----------------------------------------------------------------------------------------------------------------
def _kernel_kind(name: str) -> str:
    if "attention_fwd" in name:
        return "attention"
    if "gemm_bf16_tcgen05" in name:
        mode = name.split("gemm_bf16_tcgen05_kernel<", 1)[-1].split(",")
        return {"1": "GEGLU GEMM", "2": "3x3 convolution"}.get(mode[2].strip() if len(mode) > 2 else "", "GEMM")
    for key, kind in (("gn_", "GroupNorm"), ("layer_norm", "LayerNorm"), ("concat_channels", "NHWC copy"),
                      ("upsample_nearest2x", "NHWC copy"), ("repack_rows", "GEMM operand repack")):
        if key in name:
            return kind
    if "conv" in name or "cutlass" in name:
        return "torch convolution (cuDNN)"
    if "nvjet" in name or "gemm" in name.lower():
        return "torch GEMM (cuBLAS)"
    return "torch elementwise / copies"


def kernel_times(replay, steps: int = 3) -> str:
    """Device time of one replay per kernel kind (torch profiler over `steps` replays). Kernels launched with
    programmatic dependent launch start early and wait, so their own durations overlap; each kernel is charged the
    part of the replay's busy span it adds past the ends of the kernels before it."""
    from torch.profiler import ProfilerActivity, profile
    with profile(activities=[ProfilerActivity.CUDA]) as prof:
        for _ in range(steps):
            replay()
        torch.cuda.synchronize()
    evs = sorted((e for e in prof.events() if e.device_type == torch.autograd.DeviceType.CUDA
                  and e.time_range.end > e.time_range.start), key=lambda e: e.time_range.start)
    charged: dict[str, list] = {}
    frontier = None
    for e in evs:
        s0, s1 = e.time_range.start, e.time_range.end
        add = (s1 - s0) if frontier is None or s0 >= frontier else max(0.0, s1 - frontier)
        frontier = s1 if frontier is None else max(frontier, s1)
        c = charged.setdefault(_kernel_kind(e.name), [0, 0.0])
        c[0] += 1
        c[1] += add
    total = sum(t for _, t in charged.values())
    lines = [f"{'kernel kind':28s} {'launches':>9s} {'us/step':>9s} {'share':>6s}"]
    for kind, (n, t) in sorted(charged.items(), key=lambda kv: -kv[1][1]):
        lines.append(f"{kind:28s} {n / steps:9.1f} {t / steps:9.1f} {100 * t / total:5.1f}%")
    lines.append(f"{'busy span':28s} {len(evs) / steps:9.1f} {total / steps:9.1f}")
    return "\n".join(lines)


class UNetBench:
    """Euler CFG denoise steps of a random-init SD1.5-architecture UNet with every Linear, attention, convolution
    and normalisation the node takes over on the B200 kernels (through the ComfyUI node runtime). The batch
    (prompts x CFG pair) is sharded over the ranks with each prompt's pair local; latents are all-gathered over NCCL
    every step. One step = one UNet call on the rank's batch plus the guidance combine and the Euler update,
    captured as a CUDA graph. Strong scaling: the total batch is fixed as GPUs are added."""

    def __init__(self, dist, device):
        from npu_ai_b200 import comfy_nodes as cn
        from npu_ai_b200.sd15_unet import build_unet
        self.dist, self.device = dist, device
        self.model = build_unet(seed=0, device=device, dtype=torch.bfloat16)
        # Channels-last activations: the convolution kernels take NHWC directly, and the transformer blocks'
        # (b, c, h, w) -> (b, hw, c) reshapes become views.
        self.model.to(memory_format=torch.channels_last)
        self.rt = cn._get_runtime(device)
        self.rt.min_tokens = 64
        self.rt.take_over(self.model, 320, ("time_embed", "label_emb", "emb_layers"))
        self.rt.attn.mode = "gpu"
        self.rt.enabled = True
        self.to = {"optimized_attention_override": cn._gpu_attention_override}

    def measure(self, batch: int, latent: int, steps: int, warmup: int, unet_steps: int = 4,
                sampler: ClockSampler | None = None, kernel_times_out: bool = False) -> dict:
        from npu_ai_b200 import kernels
        from npu_ai_b200.sd15_unet import karras_sigmas, prompt_shard, seeded_prompts, sigma_to_t
        dist, device = self.dist, self.device
        P = batch // 2
        lo, hi = prompt_shard(P, dist.world, dist.rank)
        if hi - lo < 1:
            raise SystemExit("need at least one prompt (two images: uncond + cond) per rank")
        lat, ctx, unc = seeded_prompts(P, latent, seed=1, device=device, dtype=torch.bfloat16)
        lat, ctx, unc = lat[lo:hi].contiguous(), ctx[lo:hi].contiguous(), unc[lo:hi].contiguous()
        cond = torch.cat([unc, ctx])
        sigmas = karras_sigmas(unet_steps).to(device)
        sig = torch.zeros(2, device=device)  # [sigma, sigma_next] of the step being replayed
        x = (lat.float() * sigmas[0]).contiguous()
        # uneven shards are padded to the largest one for a single all-gather
        width = -(-P // dist.world)
        pad = torch.zeros((width, *lat.shape[1:]), dtype=torch.float32, device=device) if dist.world > 1 else None
        full = torch.empty((width * dist.world, *lat.shape[1:]), dtype=torch.float32, device=device) \
            if dist.world > 1 else None
        model, to = self.model, self.to

        def step():
            s, s_next = sig[0], sig[1]
            x_in = (torch.cat([x, x]) / torch.sqrt(s * s + 1.0)).to(torch.bfloat16).contiguous(
                memory_format=torch.channels_last)
            t = sigma_to_t(s).expand(x_in.shape[0])
            eps = model(x_in, t, cond, to).float()
            eu, ec = eps.chunk(2)
            x.add_((s_next - s) * (eu + 7.5 * (ec - eu)))
            if full is not None:
                pad[: hi - lo].copy_(x)
                dist.pg.all_gather_into_tensor(full, pad)

        def set_step(i):
            i %= unet_steps
            sig.copy_(torch.stack([sigmas[i], sigmas[i + 1]]))

        with torch.no_grad():
            for i in range(max(3, warmup)):
                set_step(i)
                step()
            torch.cuda.synchronize()
            cs = torch.cuda.Stream(device)
            cs.wait_stream(torch.cuda.current_stream(device))
            with torch.cuda.stream(cs):
                step()
            torch.cuda.current_stream(device).wait_stream(cs)
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, stream=cs):
                step()
            torch.cuda.synchronize()
            kernels.check_status(device)
            for i in range(3):
                set_step(i)
                g.replay()
            dist.barrier()
            torch.cuda.synchronize()
            tb = time.perf_counter()
            t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            t0.record()
            for i in range(steps):
                set_step(i)
                g.replay()
            t1.record()
            torch.cuda.synchronize()
            te = time.perf_counter()
            dist.barrier()
            kernels.check_status(device)
            kt = kernel_times(g.replay) if (kernel_times_out and dist.world == 1) else None
        ms = dist.max(t0.elapsed_time(t1) / steps, device)
        del g
        torch.cuda.empty_cache()
        out = {"batch": batch, "latent": latent, "per_rank_batch": 2 * (hi - lo), "ms_per_step": round(ms, 3),
               "steps_per_s": round(1e3 / ms, 3), "s_per_image": round(ms * unet_steps / 1e3 / P, 5),
               "euler_steps_per_image": unet_steps, "steps": steps}
        if sampler is not None:
            out["clocks"] = sampler.summary(tb, te, "the timed region")
        if kt is not None:
            out["kernel_times"] = kt
        return out

    def cpu_baseline(self, latent: int) -> dict:
        """One batch-2 (one prompt x CFG) UNet call of the same architecture in f32 on the host cores with torch's
        CPU F.linear / SDPA / conv (the reference's CPU fallback)."""
        from npu_ai_b200.sd15_unet import build_unet, seeded_prompts
        torch.set_num_threads(os.cpu_count() or 1)
        cpu_model = build_unet(seed=0, device="cpu", dtype=torch.bfloat16).float()
        lat, ctx, unc = seeded_prompts(1, latent, seed=1)
        xc = torch.cat([lat, lat]).bfloat16().float()
        cond = torch.cat([unc, ctx]).bfloat16().float()
        tc = torch.full((2,), 500.0)
        with torch.no_grad():
            cpu_model(xc[:, :, :8, :8], tc, cond)
            c0 = time.perf_counter()
            cpu_model(xc, tc, cond)
            cdt = time.perf_counter() - c0
        return {"value": round(1.0 / cdt, 4), "unit": "steps/s (batch 2)", "cores": torch.get_num_threads(),
                "kind": "port", "ms_per_step_batch2": round(cdt * 1e3, 1),
                "s_per_image": round(cdt * 4 / 1, 3),
                "sample": f"one batch-2 UNet call ({latent}x{latent} latent) in f32 on the host with torch's CPU "
                          f"F.linear / SDPA / conv (the reference's CPU fallback): {cdt:.2f} s; the batch-16 step "
                          f"is 8 such calls ({8 * cdt:.1f} s, extrapolated per prompt)"}


def unet_leg(args, dist, device, sampler) -> dict:
    """The UNet object of the driver's line: batch 16 on every latent of --unet-latents, sharded over the ranks;
    at N = 1 also batch 2 (config 4: one prompt, 4 Euler steps) and the CPU's batch-2 UNet call."""
    ub = UNetBench(dist, device)
    res = {"metric": "SD1.5 UNet denoise steps/s", "unit": "steps/s", "scaling": "strong",
           "parallelism": f"batch-sharded x{dist.world} (prompts with both CFG halves local), latents all-gathered "
                          "over NCCL every step",
           "execution": "CUDA graph of one denoise step (channels-last activations); device time, max over ranks",
           "model": "SD1.5-architecture UNet, random init (seeded), bf16",
           "linear_layers_on_gemm_kernel": len(ub.rt.weights)}
    for L in args.unet_latents:
        res[f"batch16_{L}"] = ub.measure(16, L, args.steps, args.warmup, sampler=sampler)
    if dist.world == 1:
        res["batch2_64"] = ub.measure(2, 64, args.steps, args.warmup, sampler=sampler)
        if dist.rank == 0 and not args.no_cpu:
            res["cpu_baseline"] = ub.cpu_baseline(64)
    return res


def run_unet(args, dist) -> None:
    """--workload unet: the UNet leg alone on one configuration, its own JSON line."""
    device = torch.device("cuda", dist.local_rank)
    torch.cuda.set_device(device)
    sampler = ClockSampler(_gpu_uuid(dist.local_rank)) if dist.rank == 0 else None
    if sampler is not None:
        sampler.start()
    ub = UNetBench(dist, device)
    r = ub.measure(args.batch, args.latent, args.steps, args.warmup, args.unet_steps, sampler=sampler,
                   kernel_times_out=args.kernel_times)
    if sampler is not None:
        sampler.stop()
    kt = r.pop("kernel_times", None)
    if kt is not None:
        print(kt, file=sys.stderr, flush=True)
    cpu = ub.cpu_baseline(args.latent) if (dist.rank == 0 and dist.world == 1 and not args.no_cpu) else None
    if dist.rank == 0:
        P = args.batch // 2
        line = {"metric": "SD1.5 UNet denoise steps/s", "value": r["steps_per_s"], "unit": "steps/s",
                "n_gpus": dist.world, "steps": args.steps, "warmup": max(3, args.warmup),
                "ms_per_step": r["ms_per_step"], "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
                "dtype": "bf16", "data": "synthetic",
                "config": {"workload": f"sd15-unet-random-init batch {args.batch} ({P} prompts x CFG) "
                                       f"{args.latent}x{args.latent} latent, {args.unet_steps} Euler steps per image",
                           "parallelism": f"batch-sharded x{dist.world}, latents all-gathered per step",
                           "s_per_image": r["s_per_image"],
                           "linear_layers_on_gemm_kernel": len(ub.rt.weights)},
                "execution": "CUDA graph of one denoise step (channels-last activations)",
                "cpu_baseline": cpu, "clocks": r.get("clocks")}
        print(json.dumps(line), flush=True)


def run_case(args) -> None:
    """--case: one kernel on one shape, `warmup` + `steps` launches (the small cases the ncu summaries use)."""
    from npu_ai_b200 import kernels
    device = torch.device("cuda", 0)
    kind, dims = args.case.split(":")
    d = [int(t) for t in dims.split(",")]
    gn_bytes = 0.0
    if kind == "gemm":
        M, K, N = d
        x, w, b = _seeded((M, K), 1.0, 1, device), _seeded((N, K), 0.02, 2, device), _seeded((N,), 0.01, 3, device)
        out = torch.empty((M, N), dtype=torch.bfloat16, device=device)
        fn, flops = (lambda: kernels.gemm(x, w, b, out=out)), 2.0 * M * K * N
    elif kind == "attn":
        B, H, Sq, Skv, D = d
        q, k, v = (_seeded((B, S, H * D), 1.0, i, device) for i, S in ((1, Sq), (2, Skv), (3, Skv)))
        out = torch.empty((B, Sq, H * D), dtype=torch.bfloat16, device=device)
        fn, flops = (lambda: kernels.attention(q, k, v, H, out=out)), 4.0 * B * H * Sq * Skv * D
    elif kind == "geglu":
        M, K, n = d
        x, w, b = _seeded((M, K), 1.0, 1, device), _seeded((2 * n, K), 0.05, 2, device), _seeded((2 * n,), 0.1, 3, device)
        out = torch.empty((M, n), dtype=torch.bfloat16, device=device)
        fn, flops = (lambda: kernels.gemm_geglu(x, w, b, out=out)), 2.0 * M * K * 2 * n
    elif kind == "conv":
        n, h, w_, cin, cout = d
        x = _seeded((n, h, w_, cin), 1.0, 1, device)
        wp = kernels.pack_conv3x3_weight(_seeded((cout, cin, 3, 3), (9 * cin) ** -0.5, 2, device))
        b = _seeded((cout,), 0.1, 3, device).float()
        out = torch.empty((n, h, w_, cout), dtype=torch.bfloat16, device=device)
        fn, flops = (lambda: kernels.conv3x3(x, wp, b, out=out)), 2.0 * n * h * w_ * cout * 9 * cin
    elif kind == "gn":
        n, h, w_, c = d
        x = _seeded((n, h, w_, c), 1.0, 1, device)
        g, bb = torch.ones(c, device=device), torch.zeros(c, device=device)
        out = torch.empty_like(x)
        # bytes, not FLOPs: one read for the statistics, one read and one write for the apply pass
        fn, flops = (lambda: kernels.group_norm(x, 32, g, bb, silu=True, out=out)), 0.0
        gn_bytes = 3.0 * x.numel() * 2
    elif kind == "ln":
        rows, c = d
        x = _seeded((rows, c), 1.0, 1, device)
        g, bb = torch.ones(c, device=device), torch.zeros(c, device=device)
        out = torch.empty_like(x)
        # bytes: one read and one write of the tensor
        fn, flops = (lambda: kernels.layer_norm(x, g, bb, out=out)), 0.0
        gn_bytes = 2.0 * x.numel() * 2
    elif kind == "up":
        n, c, h, w_ = d
        x = _seeded((n, c, h, w_), 1.0, 1, device).contiguous(memory_format=torch.channels_last)
        out = torch.empty((n, c, 2 * h, 2 * w_), dtype=torch.bfloat16, device=device, memory_format=torch.channels_last)
        # bytes: one read of the input, one write of the 4x output
        fn, flops = (lambda: kernels.upsample_nearest2x(x, out=out)), 0.0
        gn_bytes = 5.0 * x.numel() * 2
    elif kind == "cat":
        n, ca, cb, h, w_ = d
        a = _seeded((n, ca, h, w_), 1.0, 1, device).contiguous(memory_format=torch.channels_last)
        b = _seeded((n, cb, h, w_), 1.0, 2, device).contiguous(memory_format=torch.channels_last)
        out = torch.empty((n, ca + cb, h, w_), dtype=torch.bfloat16, device=device, memory_format=torch.channels_last)
        # bytes: one read of both sources, one write of the output
        fn, flops = (lambda: kernels.concat_channels(a, b, out=out)), 0.0
        gn_bytes = 2.0 * out.numel() * 2
    else:
        raise SystemExit(f"unknown case kind {kind!r} (gemm:M,K,N, attn:B,H,Sq,Skv,D, geglu:M,K,n, "
                         "conv:n,h,w,cin,cout, gn:n,h,w,c, ln:rows,c, up:n,c,h,w or cat:n,ca,cb,h,w)")
    for _ in range(args.warmup):
        fn()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(args.steps):
        fn()
    e1.record()
    torch.cuda.synchronize()
    kernels.check_status(device)
    ms = e0.elapsed_time(e1) / args.steps
    print(json.dumps({"case": args.case, "us_per_launch": round(ms * 1e3, 2),
                      "tflops": round(flops / ms / 1e9, 1),
                      **({"gbs": round(gn_bytes / ms / 1e6, 1)} if gn_bytes else {})}), flush=True)


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--no-cpu", action="store_true", help="skip the CPU baseline legs")
    ap.add_argument("--no-e2e", action="store_true", help="skip the host-buffer end-to-end leg")
    ap.add_argument("--no-unet", action="store_true", help="skip the UNet leg of the default run")
    ap.add_argument("--unet-latents", default="64,128",
                    help="latent sizes of the default run's batch-16 UNet leg (comma-separated)")
    ap.add_argument("--soak-s", type=float, default=0.0,
                    help="seconds of step replays right before the timed region (default none)")
    ap.add_argument("--case", default=None, help="time one kernel: gemm:M,K,N, attn:B,H,Sq,Skv,D, geglu:M,K,n, "
                                                   "conv:n,h,w,cin,cout, gn:n,h,w,c, ln:rows,c, up:n,c,h,w or "
                                                   "cat:n,ca,cb,h,w")
    ap.add_argument("--workload", choices=["hotpath", "unet"], default="hotpath",
                    help="hotpath: the driver's line (GEMM sweep + attention blocks, with the UNet leg); unet: only "
                         "the UNet on one configuration")
    ap.add_argument("--batch", type=int, default=2, help="unet: images per step, both CFG halves (2 = 1 prompt)")
    ap.add_argument("--latent", type=int, default=64, help="unet: latent height/width")
    ap.add_argument("--unet-steps", type=int, default=4, help="unet: Euler steps per image")
    ap.add_argument("--kernel-times", action="store_true",
                    help="unet: after the timed region, print the step's device time per kernel kind to stderr "
                         "(torch profiler over three extra graph replays; the JSON line is unaffected)")
    args = ap.parse_args(argv)
    args.warmup = max(3, args.warmup)
    args.unet_latents = [int(v) for v in str(args.unet_latents).split(",") if v.strip()]
    if args.case:
        run_case(args)
        return 0
    if args.impl == "reference":
        # The CPU path runs on rank 0 alone; other ranks exit at once, no process group is formed.
        if int(os.environ.get("RANK", "0")) == 0:
            run_reference(args)
        return 0
    dist = Dist(use_cuda=True)
    try:
        if args.workload == "unet":
            run_unet(args, dist)
        else:
            run_ours(args, dist)
    finally:
        dist.close()
    return 0


if __name__ == "__main__":
    sys.exit(main())

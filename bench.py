#!/usr/bin/env python
"""Benchmark of the B200-native low-precision path (one JSON line on rank 0).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--workload NAME] [--impl kab|reference]

Workloads (synthetic, seeded; BASELINE.json's configurations):
  w4a4     config 4: NVFP4 W4A4 linear with bias, X [8192, 8192] x W [28672, 8192]^T: the
           per-token NVFP4 producer of X plus the block-scaled tcgen05 GEMM with its fused
           dequant / bias epilogue (default once the GEMM is built). At N > 1 the GEMM is
           column-sharded over the ranks and the bf16 output all-gathered over NVLink.
  nvfp4_producer  config 4's activation producer alone (HBM-bound).
  mxfp8_producer  config 3's fused SiLU(gate) * up -> MXFP8 producer (HBM-bound).
  compare  the comparator on a config-4-sized bf16 output pair (HBM-bound).
  fp8_blockwise  config 2: 1x128 FP8 producer + blockwise-scaled tcgen05 GEMM (M = 2048).
  fp8_attention  config 5: per-head e4m3 quantisation + causal tcgen05 FP8 attention.
  w8a8_decode    decode-size INT8 W8A8 linear (M = 16): per-token producer + skinny GEMM.
  rmsnorm_fp8    fused RMSNorm -> FP8 per token (x [16384, 4096] bf16, one pass).
  rmsnorm_fp4    fused RMSNorm -> NVFP4 per token (x [16384, 4096] bf16, one pass).
  kv_decode      FP8 KV-cache decode attention (16 / 2 heads, head_dim 128, batch 4, 4096
                 cached tokens): split-KV tcgen05 attention over e4m3 K / V.

``value`` is the whole-job throughput with inputs resident in HBM, timed with CUDA events
over exactly K steps between barriers, the max over ranks; ``e2e`` is the same metric through
the public Python API with host buffers (pinned host -> device copies of the step's inputs
and a device -> host read of its result inside the timed region). ``roofline`` covers the
dominant kernel (its launches timed with events on the launching stream); ``cpu_baseline``
the CPU oracle on a bounded sample on this host's cores. ``--impl reference`` times the
reference's CPU path (the oracle port: the reference is Python and does not travel) on the
host cores for the same workload and prints its own line.
"""

from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import time
from datetime import timedelta
from pathlib import Path

ROOT = Path(__file__).resolve().parent
for _p in (str(ROOT), str(ROOT / "kernel-agent_b200")):
    if _p not in sys.path:
        sys.path.insert(0, _p)

METRIC = "scaled-GEMM TFLOPS & % block-scaled tensor peak; quantize GB/s & % HBM"
PEAKS_FILE = ROOT / "MEASURED_PEAKS.json"
TRAFFIC_FILE = ROOT / "profiles" / "traffic.json"
SHAPE: tuple[int, int, int] | None = None  # (M, K, N) override of the w4a4 workload
ASSEMBLE = "peer"  # w4a4 at N > 1: "peer" (GEMM epilogue stores into every rank's output) or "nccl"
FALLBACK_PEAKS = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}


def peaks() -> tuple[dict, str]:
    if PEAKS_FILE.exists():
        return json.loads(PEAKS_FILE.read_text()), "measured"
    return dict(FALLBACK_PEAKS), "fallback"


# ------------------------------------------------------------------ distributed plumbing


class Dist:
    def __init__(self) -> None:
        import torch

        self.world = int(os.environ.get("WORLD_SIZE", "1"))
        self.rank = int(os.environ.get("RANK", "0"))
        self.local = int(os.environ.get("LOCAL_RANK", "0"))
        self.torch = torch
        if self.world > 1:
            import torch.distributed as dist

            torch.cuda.set_device(self.local)
            dist.init_process_group("nccl", timeout=timedelta(seconds=300),
                                    device_id=torch.device("cuda", self.local))
            self.dist = dist
        else:
            self.dist = None

    def barrier(self) -> None:
        if self.dist is not None:
            self.dist.barrier()

    def max(self, v: float) -> float:
        if self.dist is None:
            return v
        t = self.torch.tensor([v], dtype=self.torch.float64, device="cuda")
        self.dist.all_reduce(t, op=self.dist.ReduceOp.MAX)
        return float(t.item())

    def close(self) -> None:
        if self.dist is not None:
            self.dist.destroy_process_group()


# ------------------------------------------------------------------ clocks


class Clocks:
    """nvidia-smi samples of the SM clock and throttle reasons during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int) -> None:
        self.gpu = gpu_index
        self.proc = None

    def start(self) -> None:
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "100", "-i", str(self.gpu)],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None

    def stop(self) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            out, _ = self.proc.communicate(timeout=10)
        except subprocess.TimeoutExpired:
            self.proc.kill()
            out, _ = self.proc.communicate()
        rows = [r.split(",") for r in out.strip().splitlines() if r.strip()]
        sm, mx, reasons, power = [], [], set(), []
        names = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")
        for r in rows:
            try:
                sm.append(float(r[1]))
                mx.append(float(r[2]))
                power.append(float(r[3]))
                for name, val in zip(names, r[5:9]):
                    if val.strip().lower() == "active":
                        reasons.add(name)
            except (ValueError, IndexError):
                continue
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no samples"]}
        loaded = [s for s, p in zip(sm, power) if p > 0.5 * max(power)] or sm
        return {"sm_mhz": statistics.median(loaded), "sm_max_mhz": max(mx),
                "reasons": sorted(reasons), "samples": len(sm)}


# ------------------------------------------------------------------ CPU baselines (oracle)


def _cpu_worker(args):
    """One chunk of the CPU oracle's work (runs in a spawned process)."""
    kind, payload = args
    import numpy as np  # noqa: F401

    sys.path.insert(0, str(ROOT))
    from oracle import quant as oq

    t0 = time.perf_counter()
    if kind == "nvfp4":
        oq.quantize_fp4_activations(payload, "nvfp4", "token")
    elif kind == "mxfp8_silu":
        g, u = payload
        oq.quantize_mxfp8(oq.silu_mul(g, u))
    elif kind == "w4a4":
        x, codes, scales, ts, bias = payload
        oq.fp4_w4a4_linear(x, codes, scales, ts, bias)
    elif kind == "w8a8":
        x, q, sc, bias = payload
        oq.int8_w8a8_linear(x, q, sc, bias)
    elif kind == "rmsnorm_fp8":
        x, w = payload
        oq.quantize_fp8_activations(oq.rmsnorm(x, w, 1e-6, "bf16"))
    elif kind == "rmsnorm_fp4":
        x, w = payload
        oq.quantize_fp4_activations(oq.rmsnorm(x, w, 1e-6, "bf16"), "nvfp4", "token")
    elif kind == "kv":
        from oracle import kv_quant as okv

        okv.fp8_kv_attention(*payload)
    elif kind == "compare":
        from oracle import compare as ocmp

        a, b = payload
        ocmp.compare_tensors("y", a, b, "bf16", tier="near-lossless-fp4a")
    return time.perf_counter() - t0


def cpu_rate(kind: str, chunks: list, units: float, budget_s: float, processes: int) -> tuple[float, int]:
    """Throughput (units per second) of the oracle over ``chunks`` (each worth units /
    len(chunks)), repeated until ``budget_s`` of wall time, on ``processes`` spawned workers."""
    import multiprocessing as mp

    ctx = mp.get_context("spawn")
    done = 0.0
    t0 = time.perf_counter()
    with ctx.Pool(processes) as pool:
        pool.map(_cpu_worker, [(kind, chunks[0])] * processes)  # warm the workers' imports
        t0 = time.perf_counter()
        while True:
            pool.map(_cpu_worker, [(kind, c) for c in chunks])
            done += units
            if time.perf_counter() - t0 >= budget_s:
                break
    return done / (time.perf_counter() - t0), processes


# ------------------------------------------------------------------ workloads


class Workload:
    name = ""
    unit = ""
    dtype = ""
    scaling = "weak"
    config: dict = {}

    def setup(self, dev, world, rank):
        raise NotImplementedError

    def step(self):
        """One pass of the hot path on device-resident inputs; returns the number of this
        library's kernel launches."""
        raise NotImplementedError

    def e2e_step(self):
        """One pass through the public API with host buffers (copies included)."""
        raise NotImplementedError


class Nvfp4Producer(Workload):
    name = "nvfp4_producer"
    unit = "GB/s"
    dtype = "bf16->nvfp4"

    def setup(self, dev, world, rank):
        import torch

        from kernel_agent_b200 import workloads
        from kernel_agent_b200.kernels import producers

        self.torch, self.producers = torch, producers
        self.m, self.k = 8192, 8192
        x, _, _ = workloads.config4(seed=0, device="cuda", n=128)
        self.x = x.to(dev)
        self.bytes = self.m * self.k * 2 + self.m * self.k // 2 + self.m * self.k // 16 + 4 * self.m
        self.units = self.bytes / 1e9  # GB per step
        self.kernel = "quant_fp4_fast_kernel"
        self.kernel_bytes = self.bytes
        self.x_host = self.x.cpu().pin_memory()
        self.h2d = self.x.numel() * 2
        self.d2h = self.m * self.k // 2 + self.m * self.k // 16 + 4 * self.m
        q, s, o = producers.quantize_rows_fp4(self.x, swizzle=True)
        self.out_host = [t.cpu().pin_memory() for t in (q, s.view(torch.uint8), o)]
        self.config = {"workload": "config 4 NVFP4 activation producer (per-token outer, swizzled scales)",
                       "rows": self.m, "k": self.k, "l2": "inputs larger than L2 (134 MB per step)"}

    def step(self):
        self.producers.quantize_rows_fp4(self.x, swizzle=True)
        return 1

    def e2e_step(self):
        x = self.x_host.to(self.x.device, non_blocking=True)
        q, s, o = self.producers.quantize_rows_fp4(x, swizzle=True)
        for host, t in zip(self.out_host, (q, s.view(self.torch.uint8), o)):
            host.copy_(t, non_blocking=True)
        return 1

    def cpu_baseline(self):
        import numpy as np

        rows = 64
        x = self.x[:rows].float().cpu().numpy()
        chunks = [x]
        gb = rows * self.k * (2 + 0.5 + 1 / 16) / 1e9
        rate, cores = cpu_rate("nvfp4", chunks, gb, 10.0, 1)
        return {"value": rate, "unit": "GB/s", "cores": cores, "kind": "port",
                "sample": f"oracle quantize_fp4_activations on {rows} x {self.k} rows, repeated ~10 s"}

    def reference(self, steps, warmup):
        rows = 256
        x = self.x[:rows].float().cpu().numpy()
        procs = os.cpu_count() or 1
        chunks = [x[i::procs] for i in range(procs)]
        gb = rows * self.k * (2 + 0.5 + 1 / 16) / 1e9
        rate, cores = cpu_rate("nvfp4", chunks, gb, 2.0 * max(steps, 1), procs)
        return rate, cores, f"oracle NVFP4 producer on {rows} x {self.k} rows per step, {procs} processes"


class Mxfp8Producer(Workload):
    name = "mxfp8_producer"
    unit = "GB/s"
    dtype = "bf16->mxfp8"

    def setup(self, dev, world, rank):
        import torch

        from kernel_agent_b200 import workloads
        from kernel_agent_b200.kernels import producers

        self.torch, self.producers = torch, producers
        g, u, _ = workloads.config3(seed=0, device="cuda", h=128)
        self.g, self.u = g.to(dev), u.to(dev)
        m, f = g.shape
        self.m, self.f = m, f
        self.bytes = 2 * m * f * 2 + m * f + m * f // 32
        self.units = self.bytes / 1e9
        self.kernel = "quant_mxfp8_kernel"
        self.kernel_bytes = self.bytes
        self.h2d = 2 * m * f * 2
        self.d2h = m * f + m * f // 32
        self.g_host, self.u_host = self.g.cpu().pin_memory(), self.u.cpu().pin_memory()
        self.out_host = [torch.empty(m * f, dtype=torch.uint8).pin_memory(),
                         torch.empty(m * f // 32, dtype=torch.uint8).pin_memory()]
        self.config = {"workload": "config 3 fused SiLU(gate)*up -> MXFP8 producer (swizzled scales)",
                       "rows": m, "k": f, "l2": "inputs larger than L2 (235 MB per step)"}

    def step(self):
        self.producers.silu_mul_fp8(self.g, self.u, mx=True, blocked=True)
        return 1

    def e2e_step(self):
        g = self.g_host.to(self.g.device, non_blocking=True)
        u = self.u_host.to(self.g.device, non_blocking=True)
        q, s = self.producers.silu_mul_fp8(g, u, mx=True, blocked=True)
        self.out_host[0].copy_(q.view(self.torch.uint8).reshape(-1), non_blocking=True)
        self.out_host[1].copy_(s.reshape(-1), non_blocking=True)
        return 1

    def cpu_baseline(self):
        rows = 16
        g = self.g[:rows].float().cpu().numpy()
        u = self.u[:rows].float().cpu().numpy()
        gb = rows * self.f * (4 + 1 + 1 / 32) / 1e9
        rate, cores = cpu_rate("mxfp8_silu", [(g, u)], gb, 10.0, 1)
        return {"value": rate, "unit": "GB/s", "cores": cores, "kind": "port",
                "sample": f"oracle silu_mul + quantize_mxfp8 on {rows} x {self.f}, repeated ~10 s"}

    def reference(self, steps, warmup):
        rows = 64
        procs = os.cpu_count() or 1
        g = self.g[:rows].float().cpu().numpy()
        u = self.u[:rows].float().cpu().numpy()
        chunks = [(g[i::procs], u[i::procs]) for i in range(procs)]
        gb = rows * self.f * (4 + 1 + 1 / 32) / 1e9
        rate, cores = cpu_rate("mxfp8_silu", chunks, gb, 2.0 * max(steps, 1), procs)
        return rate, cores, f"oracle SiLU*up + MXFP8 on {rows} x {self.f} per step, {procs} processes"


class W8a8Decode(Workload):
    """Decode-size W8A8: y = int8_w8a8_linear(x, W) at M = 16 tokens, X [16, 4096],
    W [14336, 4096] int8 (58.7 MB, per-channel scales), bf16 out: the per-token producer and
    the skinny GEMM (the weight streams through the tensor core). Four weight copies rotate so
    every step reads its weight from HBM (4 x 58.7 MB > L2)."""

    name = "w8a8_decode"
    unit = "GB/s"
    dtype = "int8 x int8 -> int32 -> bf16"
    graph = True  # a step is microseconds: the K timed steps run as one CUDA graph

    def setup(self, dev, world, rank):
        import torch

        from kernel_agent_b200.kernels import gemm, quant

        self.torch, self.quant, self.gemm = torch, quant, gemm
        self.m, self.k, self.n = 16, 4096, 14336
        g = torch.Generator(device="cuda").manual_seed(0)
        self.x = torch.randn(self.m, self.k, device=dev, generator=g).to(torch.bfloat16)
        w = (torch.randn(self.n, self.k, device=dev, generator=g) * 0.02).to(torch.bfloat16)
        q, s = quant.quantize_int8(w)
        del w
        self.copies = [(q.clone(), s.clone()) for _ in range(4)]
        self.bias = (torch.randn(self.n, device=dev, generator=g) * 0.1).to(torch.bfloat16)
        self.i = 0
        wbytes = self.n * self.k + 4 * self.n
        self.bytes = wbytes + self.m * self.k * 2 + self.m * self.n * 2
        self.units = self.bytes / 1e9
        self.kernel = "gemm_skinny_kernel<KIND=0 int8>"
        self.kernel_bytes = wbytes + self.m * self.k + self.m * self.n * 2
        self.x_host = self.x.cpu().pin_memory()
        self.y_host = torch.empty(self.m, self.n, dtype=torch.bfloat16).pin_memory()
        self.h2d = self.m * self.k * 2
        self.d2h = self.m * self.n * 2
        self.config = {"workload": "decode-size W8A8 INT8 linear, X [16, 4096] x W [14336, 4096]^T -> bf16",
                       "m": self.m, "k": self.k, "n": self.n,
                       "l2": "4 rotating weight copies (235 MB) larger than L2",
                       "launch": "the K timed steps are one CUDA graph (2 kernels per step)"}

    def _next(self):
        q, s = self.copies[self.i % len(self.copies)]
        self.i += 1
        return q, s

    def step_at(self, i):
        q, s = self.copies[i % len(self.copies)]
        self.quant.int8_w8a8_linear(self.x, q, s, self.bias)
        return 2

    def dominant_at(self, i):
        if not hasattr(self, "_xq"):
            self._xq = self.quant.quantize_int8_activations(self.x)
        q, s = self.copies[i % len(self.copies)]
        xq, xs = self._xq
        self.gemm.int8(xq, q, xs, s, self.bias, out_dtype=self.torch.bfloat16)
        return 1

    def step(self):
        return self.step_at(0)

    def e2e_step(self):
        x = self.x_host.to(self.x.device, non_blocking=True)
        q, s = self._next()
        y = self.quant.int8_w8a8_linear(x, q, s, self.bias)
        self.y_host.copy_(y, non_blocking=True)
        return 2

    def library_bar(self):
        """cuBLASLt's int8 GEMM (torch._int_mm, M padded to 32) on the same codes: GB/s of
        weight streamed."""
        torch = self.torch
        try:
            xq, _ = self.quant.quantize_int8_activations(self.x)
            xp = torch.zeros(32, self.k, dtype=torch.int8, device=self.x.device)
            xp[: self.m] = xq
            qs = [c[0] for c in self.copies]
            for i in range(3):
                torch._int_mm(xp, qs[i % 4].t())
            torch.cuda.synchronize()
            run = as_graph(lambda: [torch._int_mm(xp, qs[i % 4].t()) for i in range(20)], torch)
            run()
            torch.cuda.synchronize()
            a, b = torch.cuda.Event(True), torch.cuda.Event(True)
            a.record()
            run()
            b.record()
            torch.cuda.synchronize()
            ms = a.elapsed_time(b) / 20
            return {"cublaslt_int8_gbs": (self.n * self.k) / (ms / 1e3) / 1e9,
                    "what": "torch._int_mm int8 (M padded to 32), weight bytes per second, no epilogue, "
                            "20 calls in one CUDA graph"}
        except Exception as e:  # noqa: BLE001 - the bar is informational
            return {"unavailable": f"{type(e).__name__}: {e}"[:200]}

    def cpu_baseline(self):
        return self._cpu(10.0, 1)

    def _cpu(self, budget, procs):
        import numpy as np

        q, s = self.copies[0]
        cols = 1024
        chunks = [(self.x.float().cpu().numpy(), q[:cols].cpu().numpy().view(np.int8), s[:cols].cpu().numpy(),
                   self.bias[:cols].float().cpu().numpy())]
        gb = (cols * self.k + self.m * self.k * 2 + self.m * cols * 2) / 1e9
        rate, cores = cpu_rate("w8a8", chunks * procs, gb * procs, budget, procs)
        return {"value": rate, "unit": "GB/s", "cores": cores, "kind": "port",
                "sample": f"oracle int8_w8a8_linear on X [16, 4096] x {cols} weight rows, repeated ~{budget:.0f} s"}

    def reference(self, steps, warmup):
        procs = os.cpu_count() or 1
        r = self._cpu(2.0 * max(steps, 1), procs)
        return r["value"], r["cores"], r["sample"] + f", {procs} processes"


class RmsnormFp8(Workload):
    """The fused RMSNorm -> FP8 producer (triton_fp8_producers.py:191-202, per-token e4m3):
    x [16384, 4096] bf16, one pass over x (the norm kept in registers, then the codes)."""

    name = "rmsnorm_fp8"
    unit = "GB/s"
    dtype = "bf16->e4m3"

    def setup(self, dev, world, rank):
        import torch

        from kernel_agent_b200.kernels import producers

        self.torch, self.producers = torch, producers
        self.m, self.k = 16384, 4096
        g = torch.Generator(device="cuda").manual_seed(0)
        self.x = (torch.randn(self.m, self.k, device=dev, generator=g) * 3).to(torch.bfloat16)
        self.w = (1.0 + 0.1 * torch.randn(self.k, device=dev, generator=g)).to(torch.bfloat16)
        self.bytes = self.m * self.k * 2 + self.k * 2 + self.m * self.k + 4 * self.m
        self.units = self.bytes / 1e9
        self.kernel = "rmsnorm_quant_fp8_packed_kernel"
        self.kernel_bytes = self.bytes
        self.x_host = self.x.cpu().pin_memory()
        self.h2d = self.x.numel() * 2
        self.d2h = self.m * self.k + 4 * self.m
        self.out_host = [torch.empty(self.m, self.k, dtype=torch.uint8).pin_memory(),
                         torch.empty(self.m, dtype=torch.float32).pin_memory()]
        self.config = {"workload": "RMSNorm -> FP8 per token, x [16384, 4096] bf16, one pass",
                       "rows": self.m, "k": self.k, "l2": "inputs larger than L2 (134 MB read, 67 MB written "
                       "per step)"}

    def step(self):
        self.producers.rmsnorm_fp8(self.x, self.w, 1e-6)
        return 1

    def e2e_step(self):
        x = self.x_host.to(self.x.device, non_blocking=True)
        q, s = self.producers.rmsnorm_fp8(x, self.w, 1e-6)
        self.out_host[0].copy_(q.view(self.torch.uint8), non_blocking=True)
        self.out_host[1].copy_(s, non_blocking=True)
        return 1

    def library_bar(self):
        """The same result in two passes (kab_rmsnorm into h, then the row quantiser)."""
        torch = self.torch
        try:
            f = lambda: self.producers.quantize_rows(self.producers._rmsnorm(self.x, self.w, 1e-6, None))  # noqa: E731
            for _ in range(3):
                f()
            torch.cuda.synchronize()
            a, b = torch.cuda.Event(True), torch.cuda.Event(True)
            a.record()
            for _ in range(10):
                f()
            b.record()
            torch.cuda.synchronize()
            ms = a.elapsed_time(b) / 10
            return {"two_pass_gbs": self.bytes / (ms / 1e3) / 1e9, "two_pass_ms": ms,
                    "what": "kab_rmsnorm then kab_quant_rows_fp8, the same algorithmic bytes"}
        except Exception as e:  # noqa: BLE001 - the bar is informational
            return {"unavailable": f"{type(e).__name__}: {e}"[:200]}

    def cpu_baseline(self):
        return self._cpu(10.0, 1)

    def _cpu(self, budget, procs):
        rows = 64
        chunk = (self.x[:rows].float().cpu().numpy(), self.w.float().cpu().numpy())
        gb = rows * (self.k * 3 + 4) / 1e9
        rate, cores = cpu_rate("rmsnorm_fp8", [chunk] * procs, gb * procs, budget, procs)
        return {"value": rate, "unit": "GB/s", "cores": cores, "kind": "port",
                "sample": f"oracle rmsnorm + quantize_fp8_activations on {rows} rows, repeated ~{budget:.0f} s"}

    def reference(self, steps, warmup):
        procs = os.cpu_count() or 1
        r = self._cpu(2.0 * max(steps, 1), procs)
        return r["value"], r["cores"], r["sample"] + f", {procs} processes"


class RmsnormFp4(RmsnormFp8):
    """The fused RMSNorm -> NVFP4 producer (triton_fp4_producers.py:384-405, per-token outer
    scale): x [16384, 4096] bf16, one pass over x (the norm kept in registers, then the codes,
    block scales and outer scales)."""

    name = "rmsnorm_fp4"
    dtype = "bf16->e2m1"

    def setup(self, dev, world, rank):
        super().setup(dev, world, rank)
        m, k = self.m, self.k
        self.bytes = m * k * 2 + k * 2 + m * k // 2 + m * k // 16 + 4 * m
        self.units = self.bytes / 1e9
        self.kernel = "quant_fp4_fast_kernel<NORM>"
        self.kernel_bytes = self.bytes
        self.d2h = m * k // 2 + m * k // 16 + 4 * m
        torch = self.torch
        self.out_host = [torch.empty(m, k // 2, dtype=torch.uint8).pin_memory(),
                         torch.empty(m, k // 16, dtype=torch.uint8).pin_memory(),
                         torch.empty(m, dtype=torch.float32).pin_memory()]
        self.config = {"workload": "RMSNorm -> NVFP4 per token, x [16384, 4096] bf16, one pass",
                       "rows": m, "k": k, "l2": "inputs larger than L2 (134 MB read, 38 MB written per step)"}

    def step(self):
        self.producers.rmsnorm_fp4(self.x, self.w, 1e-6)
        return 1

    def e2e_step(self):
        x = self.x_host.to(self.x.device, non_blocking=True)
        for dst, src in zip(self.out_host, self.producers.rmsnorm_fp4(x, self.w, 1e-6)):
            dst.copy_(src.view(self.torch.uint8) if src.dtype != self.torch.float32 else src, non_blocking=True)
        return 1

    def library_bar(self):
        """The same result in two passes (kab_rmsnorm into h, then the NVFP4 producer)."""
        torch = self.torch
        try:
            f = lambda: self.producers.quantize_rows_fp4(self.producers._rmsnorm(self.x, self.w, 1e-6, None))  # noqa: E731
            for _ in range(3):
                f()
            torch.cuda.synchronize()
            a, b = torch.cuda.Event(True), torch.cuda.Event(True)
            a.record()
            for _ in range(10):
                f()
            b.record()
            torch.cuda.synchronize()
            ms = a.elapsed_time(b) / 10
            return {"two_pass_gbs": self.bytes / (ms / 1e3) / 1e9, "two_pass_ms": ms,
                    "what": "kab_rmsnorm then kab_quant_fp4, the same algorithmic bytes"}
        except Exception as e:  # noqa: BLE001 - the bar is informational
            return {"unavailable": f"{type(e).__name__}: {e}"[:200]}

    def _cpu(self, budget, procs):
        rows = 64
        chunk = (self.x[:rows].float().cpu().numpy(), self.w.float().cpu().numpy())
        gb = rows * (self.k * 2 + self.k // 2 + self.k // 16 + 4) / 1e9
        rate, cores = cpu_rate("rmsnorm_fp4", [chunk] * procs, gb * procs, budget, procs)
        return {"value": rate, "unit": "GB/s", "cores": cores, "kind": "port",
                "sample": f"oracle rmsnorm + quantize_fp4_activations on {rows} rows, repeated ~{budget:.0f} s"}


class KvDecode(Workload):
    """FP8 KV-cache decode (kv_quant.py, triton_fp8_kv_decode.py): one query token per sequence,
    16 query / 2 KV heads, head_dim 128, batch 4, 4096 cached tokens (the reference selftest's
    long-cache call, selftest.py:749), e4m3 K / V with one fp32 scale per (token, head). A step
    is one fp8_kv_decode call: one kernel (split-KV, the splits merged in the same launch).
    24 cache copies rotate so that every step reads its cache from HBM (24 x 8.65 MB > L2)."""

    name = "kv_decode"
    unit = "GB/s"
    dtype = "e4m3 K / V, bf16 q -> fp32 -> bf16"
    graph = True

    def setup(self, dev, world, rank):
        import torch

        from kernel_agent_b200.kernels import kv_quant

        self.torch, self.kv = torch, kv_quant
        self.b, self.hq, self.hkv, self.l, self.d = 4, 16, 2, 4096, 128
        g = torch.Generator(device="cuda").manual_seed(0)
        self.q = torch.randn(self.b, self.hq, self.d, device=dev, generator=g).to(torch.bfloat16)
        self.copies, self.bf16_kv = [], []
        for i in range(24):
            k = torch.randn(self.b, self.hkv, self.l, self.d, device=dev, generator=g).to(torch.bfloat16)
            v = torch.randn(self.b, self.hkv, self.l, self.d, device=dev, generator=g).to(torch.bfloat16)
            self.copies.append((*kv_quant.quantize_kv(k), *kv_quant.quantize_kv(v)))
            if i < 12:  # the bf16 cache of the library bar, rotated the same way (201 MB > L2)
                self.bf16_kv.append((k, v))
        rows = self.b * self.hkv * self.l
        qo = 2 * self.b * self.hq * self.d * 2
        self.bytes = 2 * rows * self.d + 2 * rows * 4 + qo
        self.units = self.bytes / 1e9
        self.kernel = "kv_decode_kernel<128, 8, bf16>"
        self.kernel_bytes = self.bytes
        self.q_host = self.q.cpu().pin_memory()
        self.y_host = torch.empty(self.b, self.hq, self.d, dtype=torch.bfloat16).pin_memory()
        self.h2d = self.b * self.hq * self.d * 2
        self.d2h = self.h2d
        self.config = {"workload": "FP8 KV-cache decode, q [4, 16, 128] over e4m3 K / V [4, 2, 4096, 128]",
                       "batch": self.b, "heads_q": self.hq, "heads_kv": self.hkv, "tokens": self.l,
                       "head_dim": self.d,
                       "l2": "24 rotating cache copies (208 MB) larger than L2",
                       "launch": "the K timed steps are one CUDA graph (1 kernel per step)"}

    def step_at(self, i):
        kc, ks, vc, vs = self.copies[i % len(self.copies)]
        self.kv.fp8_kv_decode(self.q, kc, ks, vc, vs)
        return 1

    def dominant_at(self, i):
        return self.step_at(i)

    def step(self):
        return self.step_at(0)

    def e2e_step(self):
        q = self.q_host.to(self.q.device, non_blocking=True)
        self.i = getattr(self, "i", 0) + 1
        kc, ks, vc, vs = self.copies[self.i % len(self.copies)]
        y = self.kv.fp8_kv_decode(q, kc, ks, vc, vs)
        self.y_host.copy_(y, non_blocking=True)
        return 1

    def library_bar(self):
        """torch SDPA (bf16, GQA) on the unquantised bf16 cache: the decode the e4m3 cache
        replaces (half the cache bytes)."""
        torch = self.torch
        try:
            q4 = self.q[:, :, None]
            kvs = self.bf16_kv
            f = lambda i: torch.nn.functional.scaled_dot_product_attention(  # noqa: E731
                q4, kvs[i % len(kvs)][0], kvs[i % len(kvs)][1], enable_gqa=True)
            for i in range(3):
                f(i)
            torch.cuda.synchronize()
            run = as_graph(lambda: [f(i) for i in range(24)], torch)
            run()
            torch.cuda.synchronize()
            a, b = torch.cuda.Event(True), torch.cuda.Event(True)
            a.record()
            run()
            b.record()
            torch.cuda.synchronize()
            us = a.elapsed_time(b) / 24 * 1e3
            return {"sdpa_bf16_us": us, "sdpa_bf16_gbs": (2 * kvs[0][0].numel() * 2) / (us / 1e6) / 1e9,
                    "what": "torch SDPA bf16 GQA decode on the unquantised bf16 cache, 12 rotating copies "
                            "(201 MB, larger than L2), 24 calls in one CUDA graph"}
        except Exception as e:  # noqa: BLE001 - the bar is informational
            return {"unavailable": f"{type(e).__name__}: {e}"[:200]}

    def cpu_baseline(self):
        return self._cpu(10.0, 1)

    def _cpu(self, budget, procs):
        import numpy as np

        kc, ks, vc, vs = self.copies[0]
        q = self.q[:1, :, None].float().cpu().numpy()  # one sequence of the batch
        u8 = lambda t: t[:1].cpu().view(self.torch.uint8).numpy()  # noqa: E731
        chunk = (q, u8(kc), ks[:1].cpu().numpy(), u8(vc), vs[:1].cpu().numpy())
        gb = self.bytes / self.b / 1e9
        rate, cores = cpu_rate("kv", [chunk] * procs, gb * procs, budget, procs)
        return {"value": rate, "unit": "GB/s", "cores": cores, "kind": "port",
                "sample": "oracle fp8_kv_attention (float64) on one sequence of the batch, repeated "
                          f"~{budget:.0f} s"}

    def reference(self, steps, warmup):
        procs = os.cpu_count() or 1
        r = self._cpu(2.0 * max(steps, 1), procs)
        return r["value"], r["cores"], r["sample"] + f", {procs} processes"


class Compare(Workload):
    name = "compare"
    unit = "GB/s"
    dtype = "bf16"

    def setup(self, dev, world, rank):
        import torch

        from kernel_agent_b200.kernels import compare

        self.torch, self.compare = torch, compare
        g = torch.Generator(device="cuda").manual_seed(0)
        shape = (8192, 28672)
        self.ref = torch.randn(*shape, generator=g, device="cuda").to(torch.bfloat16).to(dev)
        self.new = (self.ref.float() * (1 + 0.01 * torch.randn(*shape, generator=g, device="cuda"))).to(torch.bfloat16)
        n = self.ref.numel()
        self.bytes = 2 * n * 2  # one read of each (exact tier)
        self.units = self.bytes / 1e9
        self.kernel = "compare_kernel"
        self.kernel_bytes = self.bytes
        self.ref_host, self.new_host = self.ref.cpu().pin_memory(), self.new.cpu().pin_memory()
        self.h2d = 2 * n * 2
        self.d2h = 152  # the verdict's sums, counts and maxima (KabCompareResult)
        self.config = {"workload": "comparator, exact tier, bf16 [8192, 28672] pair (config-4 output)",
                       "l2": "inputs larger than L2 (940 MB per step)"}

    def step(self):
        self.compare.compare_tensors("y", self.ref, self.new)
        return 2

    def e2e_step(self):
        ref = self.ref_host.to(self.ref.device, non_blocking=True)
        new = self.new_host.to(self.ref.device, non_blocking=True)
        self.compare.compare_tensors("y", ref, new)  # its verdict is read back to the host
        return 2

    def cpu_baseline(self):
        a = self.ref[:256].float().cpu().numpy()
        b = self.new[:256].float().cpu().numpy()
        gb = a.size * 4 / 1e9
        rate, cores = cpu_rate("compare", [(a, b)], gb, 10.0, 1)
        return {"value": rate, "unit": "GB/s", "cores": cores, "kind": "port",
                "sample": "oracle compare_tensors on 256 rows of the pair, repeated ~10 s"}

    def reference(self, steps, warmup):
        procs = os.cpu_count() or 1
        a = self.ref[:1024].float().cpu().numpy()
        b = self.new[:1024].float().cpu().numpy()
        chunks = [(a[i::procs], b[i::procs]) for i in range(procs)]
        gb = a.size * 4 / 1e9
        rate, cores = cpu_rate("compare", chunks, gb, 2.0 * max(steps, 1), procs)
        return rate, cores, f"oracle compare_tensors on 1024 rows per step, {procs} processes"


class W4A4Linear(Workload):
    """Config 4: y = fp4_w4a4_linear(x, W) with bias, W [28672, 8192] NVFP4 (tensor scale from
    the whole weight), X [8192, 8192] quantised per token on every step. At N ranks each rank
    holds N / world output channels of W; the GEMM epilogue writes each tile into every rank's
    [M, N] output over NVLink (CUDA IPC peer stores, ``--assemble peer``, the default), or the
    shards are all-gathered by NCCL and reordered (``--assemble nccl``)."""

    name = "w4a4"
    unit = "TFLOP/s"
    dtype = "nvfp4 (e2m1 x e2m1, e4m3 / fp32 scales) -> bf16"
    scaling = "strong"

    def setup(self, dev, world, rank):
        import torch

        from kernel_agent_b200 import workloads
        from kernel_agent_b200.kernels import gemm, producers, quant, sharded

        self.torch, self.gemm, self.producers, self.quant, self.sharded = torch, gemm, producers, quant, sharded
        m, k, n = SHAPE or (8192, 8192, 28672)
        self.m, self.k, self.n, self.world, self.rank = m, k, n, world, rank
        x, w, b = workloads.config4(seed=0, device="cuda", m=m, k=k, n=n)  # the same on every rank
        self.x, self.bias_full = x.to(dev), b.to(dev)
        cols = sharded.shard_columns(n, world, rank)
        ns = cols.stop - cols.start
        # build time: this rank's rows of W, with the whole weight's tensor scale (all-reduced amax)
        codes, scales, ts = sharded.quantize_fp4_weight_shard(w[cols].to(dev))
        del w
        self.ns = ns
        self.wq = codes
        self.ws = quant.swizzle_fp4_scales(scales).view(torch.uint8)
        self.ts = ts
        self.bias = self.bias_full[cols].contiguous()
        self.w_unswizzled = (codes, scales)
        self.peers = None
        if world > 1 and ASSEMBLE == "peer":
            self.peers = sharded.PeerOutput(m, n, torch.bfloat16, device=dev)
            self.col0 = cols.start
            self.out_local = self.peers.buffer[:, cols]
            self.peer_ptrs = self.peers.peer_ptrs(cols.start)
            self.out, self.gathered = self.peers.buffer, None
        else:
            self.peer_ptrs = None
            self.out_local = torch.empty(m, ns, dtype=torch.bfloat16, device=dev)
            self.out = torch.empty(m, n, dtype=torch.bfloat16, device=dev) if world > 1 else self.out_local
            self.gathered = torch.empty(world, m, ns, dtype=torch.bfloat16, device=dev) if world > 1 else None
        self.flops = 2.0 * m * n * k
        self.units = self.flops / 1e12
        self.kernel = "gemm_kernel<KIND=3 nvf4>"
        self.kernel_flops = 2.0 * m * ns * k
        self.h2d = m * k * 2
        self.d2h = m * n * 2
        self.x_host = self.x.cpu().pin_memory()
        self.y_host = torch.empty(m, n, dtype=torch.bfloat16).pin_memory()
        self.config = {
            "workload": "config 4: W4A4 NVFP4 linear with bias, X [8192, 8192] x W [28672, 8192]^T -> bf16",
            "m": m, "k": k, "n": n, "step": "NVFP4 activation producer + tcgen05 mxf4nvf4 GEMM with fused epilogue"
            + ("" if world == 1 else " storing every tile into all ranks' outputs over NVLink (CUDA IPC),"
               " ordered by two 1-element NCCL all-reduces" if self.peers is not None
               else " + NCCL all-gather of the column shards and a reordering copy"),
            "parallelism": f"column-sharded over {world} GPU(s)" if world > 1 else "1 GPU",
            "l2": "inputs larger than L2 (W codes 117 MB, X 134 MB, output 470 MB per step)",
        }

    def _gemm(self, xq, xs, outer):
        return self.gemm.nvf4(xq, xs.view(self.torch.uint8), outer, self.wq, self.ws, self.ts, self.bias,
                              out=self.out_local, peer_out=self.peer_ptrs)

    def step(self):
        xq, xs, outer = self.producers.quantize_rows_fp4(self.x, swizzle=True)
        if self.peers is not None:
            self.peers.barrier()  # every rank has finished reading the previous step's output
            self._gemm(xq, xs, outer)
            self.peers.barrier()  # every rank's tiles have landed in every output
        else:
            self._gemm(xq, xs, outer)
            if self.world > 1:
                self.sharded.gather_columns(self.out_local, out=self.out, staging=self.gathered)
        return 2

    def dominant(self):
        if not hasattr(self, "_xq"):
            self._xq = self.producers.quantize_rows_fp4(self.x, swizzle=True)
        self._gemm(*self._xq)
        return 1

    def e2e_step(self):
        x = self.x_host.to(self.x.device, non_blocking=True)
        if self.world == 1:
            y = self.quant.fp4_w4a4_linear(x, self.wq, self.ws, self.ts, self.bias)
        else:
            y = self.sharded.fp4_w4a4_linear_sharded(x, self.wq, self.ws, self.ts, self.bias,
                                                     out_local=self.out_local, out=self.out, staging=self.gathered,
                                                     peers=self.peers)
        self.y_host.copy_(y, non_blocking=True)
        return 2

    def close(self):
        if self.peers is not None:
            self.peers.barrier()  # no rank unmaps while another may still store into it
            self.torch.cuda.synchronize()
            self.peers.close()

    def tensor_peak(self, pk, pk_kind):
        """The dense NVFP4 tensor peak as 4 x the measured bf16 GEMM burst (B200: 9 vs 2.25
        PFLOP/s nominal dense)."""
        return 4.0 * pk["bf16_tflops"], f"4 x {pk_kind} bf16 burst ({pk['bf16_tflops']:.0f} TFLOP/s): NVFP4 dense"

    def library_bar(self):
        """cuBLASLt's NVFP4 GEMM (torch F.scaled_mm, BlockWise1x16) on the same codes: TFLOP/s."""
        torch = self.torch
        import torch.nn.functional as F

        try:
            xq, xs, outer = self.producers.quantize_rows_fp4(self.x, swizzle=True)
            a = xq.view(torch.float4_e2m1fn_x2)
            b = self.wq.view(torch.float4_e2m1fn_x2).t()
            kw = dict(scale_a=xs, scale_recipe_a=F.ScalingType.BlockWise1x16,
                      scale_b=self.ws.view(torch.float8_e4m3fn), scale_recipe_b=F.ScalingType.BlockWise1x16,
                      swizzle_a=F.SwizzleType.SWIZZLE_32_4_4, swizzle_b=F.SwizzleType.SWIZZLE_32_4_4,
                      output_dtype=torch.float32)
            for _ in range(3):
                F.scaled_mm(a, b, **kw)
            ms, _ = timed(lambda: (F.scaled_mm(a, b, **kw), 1)[1], 10, torch)
            return {"cublaslt_nvfp4_tflops": 2.0 * self.m * self.ns * self.k / (ms / 10 / 1e3) / 1e12,
                    "what": "F.scaled_mm BlockWise1x16 NVFP4, fp32 out, same codes (no epilogue)"}
        except Exception as exc:  # a torch without the NVFP4 path
            return {"unavailable": f"{type(exc).__name__}: {exc}"[:200]}

    def _cpu_sample(self, rows: int, cols: int):
        import numpy as np

        codes, scales = self.w_unswizzled
        x = self.x[:rows].float().cpu().numpy()
        wq = codes[:cols].cpu().numpy()
        ws = scales[:cols].view(self.torch.uint8).cpu().numpy()
        b = self.bias_full[:cols].float().cpu().numpy()
        return x, wq, ws, float(self.ts), b

    def cpu_baseline(self):
        import time as _t

        sys.path.insert(0, str(ROOT))
        from oracle import quant as oq

        rows, cols = 32, 4096
        x, wq, ws, ts, b = self._cpu_sample(rows, cols)
        flops = 2.0 * rows * cols * self.k
        t0 = _t.perf_counter()
        reps = 0
        while _t.perf_counter() - t0 < 10.0:
            oq.fp4_w4a4_linear(x, wq, ws, ts, b)
            reps += 1
        rate = flops * reps / (_t.perf_counter() - t0) / 1e12
        return {"value": rate, "unit": "TFLOP/s", "cores": os.cpu_count() or 1, "kind": "port",
                "sample": f"oracle fp4_w4a4_linear (float64 BLAS matmul, all threads) on {rows} rows x "
                          f"{cols} output channels x K {self.k}, repeated ~10 s"}

    def reference(self, steps, warmup):
        import time as _t

        sys.path.insert(0, str(ROOT))
        from oracle import quant as oq

        rows, cols = 64, 4096
        x, wq, ws, ts, b = self._cpu_sample(rows, cols)
        flops = 2.0 * rows * cols * self.k
        for _ in range(max(1, warmup // 3)):
            oq.fp4_w4a4_linear(x, wq, ws, ts, b)
        t0 = _t.perf_counter()
        for _ in range(steps):
            oq.fp4_w4a4_linear(x, wq, ws, ts, b)
        rate = flops * steps / (_t.perf_counter() - t0) / 1e12
        return rate, os.cpu_count() or 1, f"oracle fp4_w4a4_linear on {rows} rows x {cols} output channels per step"


class Fp8Blockwise(Workload):
    """Config 2: y = fp8_blockwise_linear(x, W): x [M, 1024] quantised per 1 x 128 group on
    every step, W [3072, 1024] with 128 x 128 block scales (build time), promoted per
    128-wide K step; bf16 out. M = 2048 (the tensor-bound case) unless --shape says otherwise.
    The step is a few microseconds, so the K timed steps run as one CUDA graph, step i on
    input copy i % copies: the copies together are larger than L2, so each step reads HBM."""

    name = "fp8_blockwise"
    graph = True
    unit = "TFLOP/s"
    dtype = "e4m3 x e4m3 (fp32 1x128 / 128x128 scales) -> bf16"
    scaling = "weak"

    def setup(self, dev, world, rank):
        import torch

        from kernel_agent_b200 import workloads
        from kernel_agent_b200.kernels import blockwise, gemm

        self.torch, self.blockwise, self.gemm = torch, blockwise, gemm
        m, k, n = SHAPE or (2048, 1024, 3072)
        self.m, self.k, self.n = m, k, n
        x, w = workloads.config2(m, seed=0, device="cuda", k=k, n=n)
        self.x = x.to(dev)
        self.wq, self.ws = blockwise.quantize_fp8_blocks(w.to(dev))
        per_step = m * k * 2 + m * k + n * k + m * n * 2  # x, its codes, W codes, y
        self.copies = max(2, -(-(256 << 20) // per_step))
        self.xs_ = [self.x.clone() for _ in range(self.copies)]
        self.ws_ = [(self.wq.clone(), self.ws.clone()) for _ in range(self.copies)]
        self.xq_ = [blockwise.quantize_fp8_groups(t) for t in self.xs_]
        self.flops = 2.0 * m * n * k
        self.units = self.flops / 1e12
        self.kernel = "gemm_blockwise_kernel"
        self.kernel_flops = self.flops
        self.h2d = m * k * 2
        self.d2h = m * n * 2
        self.x_host = self.x.cpu().pin_memory()
        self.y_host = torch.empty(m, n, dtype=torch.bfloat16).pin_memory()
        self.config = {
            "workload": f"config 2: blockwise FP8 linear, X [{m}, {k}] x W [{n}, {k}]^T -> bf16",
            "m": m, "k": k, "n": n,
            "step": "1x128 FP8 activation producer + tcgen05 f8f6f4 GEMM with per-128-K fp32 promotion",
            "parallelism": "replicas",
            "l2": f"inputs larger than L2: step i uses copy i % {self.copies} of X and W ({self.copies} x "
                  f"{per_step / 2**20:.1f} MB)",
            "launch": "the K timed steps are one CUDA graph (2 kernels per step)",
        }

    def step_at(self, i):
        j = i % self.copies
        xq, xs = self.blockwise.quantize_fp8_groups(self.xs_[j])
        wq, ws = self.ws_[j]
        self.gemm.fp8_blockwise(xq, xs, wq, ws)
        return 2

    def dominant_at(self, i):
        j = i % self.copies
        xq, xs = self.xq_[j]
        wq, ws = self.ws_[j]
        self.gemm.fp8_blockwise(xq, xs, wq, ws)
        return 1

    def step(self):
        return self.step_at(0)

    def e2e_step(self):
        x = self.x_host.to(self.x.device, non_blocking=True)
        y = self.blockwise.fp8_blockwise_linear(x, self.wq, self.ws)
        self.y_host.copy_(y, non_blocking=True)
        return 2

    def tensor_peak(self, pk, pk_kind):
        return 2.0 * pk["bf16_tflops"], f"2 x {pk_kind} bf16 burst ({pk['bf16_tflops']:.0f} TFLOP/s): FP8 dense"

    def library_bar(self):
        """cuBLASLt's blockwise FP8 GEMM (F.scaled_mm BlockWise1x128 x BlockWise128x128)."""
        torch = self.torch
        import torch.nn.functional as F

        xq, xs = self.blockwise.quantize_fp8_groups(self.x)
        b = self.wq.t()
        errors = []
        # the scale layouts torch may ask for: row-major, or outer-dim-major (transposed)
        for sa, sb in ((xs.t().contiguous().t(), self.ws), (xs, self.ws), (xs.t().contiguous().t(), self.ws.t()),
                       (xs, self.ws.t())):
            kw = dict(scale_a=sa, scale_recipe_a=F.ScalingType.BlockWise1x128, scale_b=sb,
                      scale_recipe_b=F.ScalingType.BlockWise128x128, output_dtype=torch.bfloat16)
            try:
                for _ in range(3):
                    F.scaled_mm(xq, b, **kw)
                ms, _ = timed(lambda: (F.scaled_mm(xq, b, **kw), 1)[1], 20, torch)
            except Exception as exc:
                errors.append(f"{type(exc).__name__}: {exc}"[:120])
                continue
            return {"cublaslt_blockwise_tflops": self.flops / (ms / 20 / 1e3) / 1e12,
                    "what": "F.scaled_mm BlockWise1x128 x BlockWise128x128, bf16 out, same codes, L2 warm"}
        return {"unavailable": " | ".join(errors)[:400]}

    def _cpu_case(self, rows):
        import numpy as np

        sys.path.insert(0, str(ROOT))
        from oracle import fp8lib

        x = self.x[:rows].float().cpu().numpy()
        wq = self.wq.view(self.torch.uint8).cpu().numpy()
        ws = self.ws.cpu().numpy()
        return fp8lib, x, wq, ws

    def cpu_baseline(self):
        import time as _t

        rows = 64
        fp8lib, x, wq, ws = self._cpu_case(rows)
        t0 = _t.perf_counter()
        reps = 0
        while _t.perf_counter() - t0 < 10.0:
            xq, xs = fp8lib.quantize_fp8_groups(x, 128)
            fp8lib.fp8_blockwise_gemm(xq, xs, wq, ws)
            reps += 1
        rate = 2.0 * rows * self.n * self.k * reps / (_t.perf_counter() - t0) / 1e12
        return {"value": rate, "unit": "TFLOP/s", "cores": os.cpu_count() or 1, "kind": "port",
                "sample": f"oracle fq_groups + blockwise GEMM (float64 BLAS per K step, all threads) on "
                          f"{rows} rows x {self.n} x K {self.k}, repeated ~10 s"}

    def reference(self, steps, warmup):
        import time as _t

        rows = 128
        fp8lib, x, wq, ws = self._cpu_case(rows)
        for _ in range(max(1, warmup // 3)):
            fp8lib.fp8_blockwise_gemm(*fp8lib.quantize_fp8_groups(x, 128), wq, ws)
        t0 = _t.perf_counter()
        for _ in range(steps):
            fp8lib.fp8_blockwise_gemm(*fp8lib.quantize_fp8_groups(x, 128), wq, ws)
        rate = 2.0 * rows * self.n * self.k * steps / (_t.perf_counter() - t0) / 1e12
        return rate, os.cpu_count() or 1, f"oracle blockwise FP8 linear on {rows} rows per step"


class Fp8Attention(Workload):
    """Config 5: causal FP8 attention prefill, B 4, Hq 32, Hkv 8, S 4096, D 128: the per-head
    e4m3 quantisation of Q, K, V plus the tcgen05 attention kernel; bf16 out."""

    name = "fp8_attention"
    unit = "TFLOP/s"
    dtype = "e4m3 Q K^T and P V (fp32 softmax) -> bf16"
    scaling = "weak"

    def setup(self, dev, world, rank):
        import torch

        from kernel_agent_b200 import workloads
        from kernel_agent_b200.kernels import attention

        self.torch, self.attention = torch, attention
        self.q, self.k, self.v = (t.to(dev) for t in workloads.config5(seed=0, device="cuda"))
        b, hq, s, d = self.q.shape
        self.b, self.hq, self.s, self.d = b, hq, s, d
        # causal: sum over query tiles of the keys up to the diagonal, both products
        self.flops = 4.0 * b * hq * d * (s * (s + 1) / 2)
        self.units = self.flops / 1e12
        self.kernel = "attention_fp8_kernel"
        self.kernel_flops = self.flops
        self.h2d = (self.q.numel() + self.k.numel() + self.v.numel()) * 2
        self.d2h = self.q.numel() * 2
        self.hosts = [t.cpu().pin_memory() for t in (self.q, self.k, self.v)]
        self.y_host = torch.empty(self.q.shape, dtype=torch.bfloat16).pin_memory()
        self.config = {
            "workload": "config 5: causal FP8 attention prefill, Q [4, 32, 4096, 128], K/V [4, 8, 4096, 128] -> bf16",
            "batch": b, "heads_q": hq, "heads_kv": self.k.shape[1], "seq": s, "head_dim": d,
            "step": "per-head e4m3 quantisation of Q, K, V + tcgen05 attention (S = QK^T, online softmax, PV)",
            "parallelism": "replicas", "l2": "inputs larger than L2 (Q, K, V, out 402 MB bf16)",
        }

    def step(self):
        self.attention.attention_fp8(self.q, self.k, self.v, is_causal=True, enable_gqa=True)
        return 7

    def dominant(self):
        if not hasattr(self, "_codes"):
            a = self.attention
            self._codes = (a.quantize_fp8_heads(self.q), a.quantize_fp8_heads(self.k),
                           a.quantize_fp8_heads(self.v, transpose=True))
            self._out = self.torch.empty(self.q.shape, dtype=self.torch.bfloat16, device=self.q.device)
        from kernel_agent_b200 import _native as nat

        (qc, qs), (kc, ks), (vt, vs) = self._codes
        nat.call("kab_attention_fp8", qc.data_ptr(), qs.data_ptr(), kc.data_ptr(), ks.data_ptr(), vt.data_ptr(),
                 vs.data_ptr(), self.b, self.hq, self.k.shape[1], self.s, self.d, 1, self.d ** -0.5,
                 self._out.data_ptr(), nat.stream_of(self.q))
        return 1

    def e2e_step(self):
        q, k, v = (h.to(self.q.device, non_blocking=True) for h in self.hosts)
        y = self.attention.attention_fp8(q, k, v, is_causal=True, enable_gqa=True)
        self.y_host.copy_(y, non_blocking=True)
        return 7

    def tensor_peak(self, pk, pk_kind):
        return 2.0 * pk["bf16_tflops"], f"2 x {pk_kind} bf16 burst ({pk['bf16_tflops']:.0f} TFLOP/s): FP8 dense"

    def library_bar(self):
        """torch's bf16 flash attention (F.scaled_dot_product_attention, causal, GQA) on the
        same inputs: TFLOP/s."""
        torch = self.torch
        import torch.nn.functional as F

        try:
            fn = lambda: F.scaled_dot_product_attention(self.q, self.k, self.v, is_causal=True, enable_gqa=True)  # noqa: E731
            for _ in range(2):
                fn()
            ms, _ = timed(lambda: (fn(), 1)[1], 5, torch)
            return {"sdpa_bf16_tflops": self.flops / (ms / 5 / 1e3) / 1e12,
                    "what": "F.scaled_dot_product_attention bf16, causal, enable_gqa (not FP8)"}
        except Exception as exc:
            return {"unavailable": f"{type(exc).__name__}: {exc}"[:200]}

    def _head(self, b, h):
        hk = h // (self.hq // self.k.shape[1])
        return tuple(t.float().cpu().numpy() for t in (self.q[b, h], self.k[b, hk], self.v[b, hk]))

    def cpu_baseline(self):
        import time as _t

        sys.path.insert(0, str(ROOT))
        from oracle import fp8lib

        q, k, v = self._head(0, 0)
        flops_head = 4.0 * self.d * (self.s * (self.s + 1) / 2)
        t0 = _t.perf_counter()
        reps = 0
        while _t.perf_counter() - t0 < 10.0:
            fp8lib.attention_fp8_head(q, k, v, causal=True)
            reps += 1
        rate = flops_head * reps / (_t.perf_counter() - t0) / 1e12
        return {"value": rate, "unit": "TFLOP/s", "cores": os.cpu_count() or 1, "kind": "port",
                "sample": "oracle emulated_sdpa (qkpv) of one (batch, head) [4096 x 4096], float64 BLAS, "
                          "repeated ~10 s"}

    def reference(self, steps, warmup):
        import time as _t

        sys.path.insert(0, str(ROOT))
        from oracle import fp8lib

        q, k, v = self._head(0, 0)
        flops_head = 4.0 * self.d * (self.s * (self.s + 1) / 2)
        t0 = _t.perf_counter()
        for _ in range(steps):
            fp8lib.attention_fp8_head(q, k, v, causal=True)
        rate = flops_head * steps / (_t.perf_counter() - t0) / 1e12
        return rate, os.cpu_count() or 1, "oracle qkpv attention of one (batch, head) per step"


WORKLOADS = {w.name: w for w in (W4A4Linear, Nvfp4Producer, Mxfp8Producer, Compare, Fp8Blockwise, Fp8Attention,
                                  W8a8Decode, KvDecode, RmsnormFp8, RmsnormFp4)}
DEFAULT = "w4a4"


# ------------------------------------------------------------------ timing


def timed(fn, steps: int, torch):
    """(total ms of `steps` calls on the current stream, launches) with CUDA events."""
    launches = 0
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    start.record()
    for _ in range(steps):
        launches += fn()
    end.record()
    torch.cuda.synchronize()
    return start.elapsed_time(end), launches


def as_graph(fn, torch):
    """`fn` captured once into a CUDA graph; the returned callable replays it and returns the
    launch count the captured call reported."""
    stream = torch.cuda.Stream()
    stream.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(stream):
        fn()  # first call outside capture (lazy set-up)
    torch.cuda.current_stream().wait_stream(stream)
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        launches = fn()

    def replay():
        graph.replay()
        return launches

    replay.graph = graph
    return replay


def kernel_ms(fn, steps: int, torch) -> float:
    """Average device time of one call of `fn` (one dominant launch), events around each."""
    evs = []
    for _ in range(steps):
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        fn()
        b.record()
        evs.append((a, b))
    torch.cuda.synchronize()
    return sum(a.elapsed_time(b) for a, b in evs) / steps


def main() -> int:
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=("kab", "reference"), default="kab")
    ap.add_argument("--workload", default=None)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--assemble", choices=("peer", "nccl"), default="peer",
                    help="w4a4 at N > 1: GEMM epilogue peer stores (CUDA IPC) or an NCCL all-gather")
    ap.add_argument("--shape", default=None,
                    help="M,N,K of the w4a4 / fp8_blockwise workload (default: the config's shape)")
    args = ap.parse_args()
    global SHAPE, ASSEMBLE
    ASSEMBLE = args.assemble
    if args.shape:
        m_, n_, k_ = (int(v) for v in args.shape.split(","))
        SHAPE = (m_, k_, n_)
    args.warmup = max(args.warmup, 3)

    workloads = dict(WORKLOADS)
    name = args.workload or DEFAULT
    if name not in workloads:
        print(json.dumps({"error": f"unknown workload {name}", "known": sorted(workloads)}))
        return 2

    dist = Dist()
    torch = dist.torch
    dev = torch.device("cuda", dist.local)
    torch.cuda.set_device(dev)
    wl = workloads[name]()

    if args.impl == "reference":
        if dist.rank != 0:
            dist.close()
            return 0
        wl.setup(dev, 1, 0)
        t0 = time.perf_counter()
        rate, cores, sample = wl.reference(args.steps, args.warmup)
        line = {
            "impl": "reference", "metric": METRIC, "value": rate, "unit": wl.unit,
            "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": None, "higher_is_better": True, "scaling": wl.scaling,
            "vs_baseline": None, "dtype": wl.dtype, "data": "synthetic (seeded)",
            "config": wl.config,
            "cpu_baseline": {"value": rate, "unit": wl.unit, "cores": cores, "kind": "port", "sample": sample},
            "e2e": {"value": rate, "unit": wl.unit, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
            "wall_s": round(time.perf_counter() - t0, 1),
        }
        print(json.dumps(line))
        dist.close()
        return 0

    wl.setup(dev, dist.world, dist.rank)
    for _ in range(args.warmup):
        wl.step()
    torch.cuda.synchronize()
    graphed = getattr(wl, "graph", False)
    if graphed:
        # launch-bound steps: the K timed steps (and K dominant launches) are one CUDA graph,
        # each step on its own copy of the inputs (the copies together exceed L2)
        k_steps = args.steps
        steps_graph = as_graph(lambda: sum(wl.step_at(i) for i in range(k_steps)), torch)
        dom_graph = as_graph(lambda: sum(wl.dominant_at(i) for i in range(k_steps)), torch)
        steps_graph()
        torch.cuda.synchronize()
    dist.barrier()
    clocks = Clocks(dist.local)
    clocks.start()
    time.sleep(0.3)
    dist.barrier()
    if graphed:
        total_ms, launches = timed(steps_graph, 1, torch)
        dist.barrier()
        k_ms = kernel_ms(dom_graph, 1, torch) / args.steps
    else:
        total_ms, launches = timed(wl.step, args.steps, torch)
        dist.barrier()
        k_ms = kernel_ms(getattr(wl, "dominant", wl.step), args.steps, torch)
    clk = clocks.stop()
    total_ms = dist.max(total_ms)
    k_ms = dist.max(k_ms)
    ms_per_step = total_ms / args.steps
    value = wl.units * dist.world / (ms_per_step / 1e3) if wl.scaling == "weak" else wl.units / (ms_per_step / 1e3)

    # end to end through the public API with host buffers
    for _ in range(2):
        wl.e2e_step()
    torch.cuda.synchronize()
    dist.barrier()
    e2e_ms, _ = timed(wl.e2e_step, max(3, args.steps // 2), torch)
    e2e_ms = dist.max(e2e_ms) / max(3, args.steps // 2)
    e2e_value = wl.units * dist.world / (e2e_ms / 1e3) if wl.scaling == "weak" else wl.units / (e2e_ms / 1e3)

    pk, pk_kind = peaks()
    if wl.unit == "GB/s":
        achieved = wl.kernel_bytes / (k_ms / 1e3) / 1e9
        peak = pk["hbm_gbs"]
        roof = {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                "frac": achieved / peak, "peak_kind": f"{pk_kind} copy bandwidth"}
    else:
        achieved = wl.kernel_flops / (k_ms / 1e3) / 1e12
        peak, peak_kind = wl.tensor_peak(pk, pk_kind)
        roof = {"bound": "tensor", "achieved": achieved, "peak": peak, "unit": "TFLOP/s",
                "frac": achieved / peak, "peak_kind": peak_kind}
    roof["kernel"] = wl.kernel
    roof["kernel_ms"] = k_ms
    traffic = None
    if TRAFFIC_FILE.exists():
        traffic = json.loads(TRAFFIC_FILE.read_text()).get(f"{wl.kernel} {wl.name}")
    roof["traffic"] = traffic

    library = wl.library_bar() if hasattr(wl, "library_bar") else None
    cpu = None
    if dist.rank == 0 and dist.world == 1 and not args.no_cpu_baseline:
        cpu = wl.cpu_baseline()
    line = {
        "metric": METRIC, "value": value, "unit": wl.unit, "n_gpus": dist.world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms_per_step,
        "higher_is_better": True, "scaling": wl.scaling, "vs_baseline": None,
        "dtype": wl.dtype, "data": "synthetic (seeded)", "config": wl.config,
        "roofline": roof, "cpu_baseline": cpu,
        "e2e": {"value": e2e_value, "unit": wl.unit, "h2d_bytes_per_step": wl.h2d,
                "d2h_bytes_per_step": wl.d2h},
        "gpu_launches": launches, "clocks": clk,
    }
    if library is not None:
        line["library_bar"] = library
    if dist.rank == 0:
        print(json.dumps(line))
    closer = getattr(wl, "close", None)
    if closer is not None:
        closer()
    dist.close()
    return 0


if __name__ == "__main__":
    sys.exit(main())

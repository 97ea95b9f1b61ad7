#!/usr/bin/env python
"""Benchmark of the B200-native low-precision path (one JSON line on rank 0).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--workload NAME] [--impl kab|reference]

The default line is config 4 (BASELINE.json's headline GEMM: the NVFP4 W4A4 linear with bias,
X [8192, 8192] x W [28672, 8192]^T -> bf16, column-sharded over the ranks at N > 1). At one GPU
it also carries ``sub_results``: the rest of the metric ("quantize GB/s & % HBM") and every
other configuration, each with its own roofline fraction and CPU baseline: the config-4 NVFP4
producer, config 1 (W8A8 INT8 [128, 1024] x [1024, 1024]), config 2 (blockwise FP8 at
M = 1, 16 and 2048), config 3 (SiLU(gate) * up -> MXFP8 producer + the down-projection GEMM),
the comparator on a config-4-sized output pair and config 5 (FP8 attention prefill).

Workloads (``--workload``; synthetic, seeded, BASELINE.json's shapes and distributions):
  w4a4            config 4 (default)
  nvfp4_producer  config 4's activation producer alone (HBM-bound)
  w8a8_config1    config 1: per-token INT8 producer + int8 GEMM + epilogue (latency-bound)
  fp8_blockwise   config 2 at M = 2048; fp8_blockwise_m16 / fp8_blockwise_m1 (weight-streaming)
  mxfp8_mlp       config 3: fused SiLU * up -> MXFP8 producer + down-projection GEMM
  mxfp8_producer  config 3's fused producer alone (HBM-bound)
  fp8_attention   config 5: per-head e4m3 quantisation + causal tcgen05 FP8 attention
  compare         the comparator on a config-4-sized bf16 output pair (HBM-bound)
  w8a8_decode, kv_decode, rmsnorm_fp8, rmsnorm_fp4   the next-step rows (decode GEMM, FP8 KV
                  decode, fused RMSNorm producers)

``value`` is the whole-job throughput with inputs resident in HBM, timed with CUDA events
over exactly K steps between barriers, the max over ranks; ``e2e`` is the same metric through
the public Python API with host buffers (pinned host -> device copies of the step's inputs and
a device -> host read of its result inside the timed region). ``roofline`` covers the dominant
kernel (its launches timed with events on the launching stream). The CPU legs time the
reference's CPU execution path (``oracle/cpu_path.py``: the oracle's quantisers and the
reference's fp32 BLAS GEMMs) on one bounded sample per workload, built with torch and the
oracle only (the product library is not loaded by ``--impl reference``): ``cpu_baseline`` in the
GPU arm and the ``--impl reference`` arm use the same sample.
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


# ------------------------------------------------------------------ CPU legs


def _cpu_worker(args):
    """One chunk of a CPU leg (in this process or a spawned one): the reference's CPU
    execution path (``oracle.cpu_path``) or the oracle's quantisers on one payload."""
    kind, payload = args
    sys.path.insert(0, str(ROOT))
    from oracle import compare as ocmp
    from oracle import cpu_path as cp
    from oracle import kv_quant as okv
    from oracle import quant as oq

    t0 = time.perf_counter()
    if kind == "nvfp4":
        oq.quantize_fp4_activations(payload, "nvfp4", "token")
    elif kind == "mxfp8_silu":
        cp.silu_mul_mxfp8(*payload)
    elif kind == "w4a4":
        cp.fp4_w4a4_linear(*payload)
    elif kind == "w8a8":
        cp.int8_w8a8_linear(*payload)
    elif kind == "mxfp8_mlp":
        g, u, wq, ws = payload
        cp.mxfp8_linear_codes(*cp.silu_mul_mxfp8(g, u), wq, ws)
    elif kind == "blockwise":
        cp.fp8_blockwise_linear(*payload)
    elif kind == "attention":
        cp.attention_fp8_head(*payload, causal=True)
    elif kind == "rmsnorm_fp8":
        x, w = payload
        oq.quantize_fp8_activations(oq.rmsnorm(x, w, 1e-6, "bf16"))
    elif kind == "rmsnorm_fp4":
        x, w = payload
        oq.quantize_fp4_activations(oq.rmsnorm(x, w, 1e-6, "bf16"), "nvfp4", "token")
    elif kind == "kv":
        okv.fp8_kv_attention(*payload)
    elif kind == "compare":
        a, b = payload
        ocmp.compare_tensors("y", a, b, "bf16")
    else:
        raise ValueError(f"unknown CPU leg {kind}")
    return time.perf_counter() - t0


class CpuCase:
    """One bounded sample of a workload for the CPU legs: ``chunks`` run together make one
    round worth ``units`` of the workload's metric. One chunk runs in this process (its GEMMs on
    torch's BLAS threads); several run in as many spawned processes (numpy element-wise work
    is single-threaded)."""

    def __init__(self, kind: str, chunks: list, units: float, sample: str):
        self.kind, self.chunks, self.units, self.sample = kind, chunks, units, sample

    def run(self, *, budget_s: float | None = None, rounds: int | None = None, warmup: int = 1) -> tuple[float, int]:
        """(units per second, host threads used) over ``rounds`` rounds after ``warmup``, or
        as many rounds as fit ``budget_s`` seconds."""
        import multiprocessing as mp

        if len(self.chunks) == 1:
            import torch

            cores = torch.get_num_threads()
            run_round = lambda: _cpu_worker((self.kind, self.chunks[0]))  # noqa: E731
            pool = None
        else:
            cores = len(self.chunks)
            pool = mp.get_context("spawn").Pool(cores)
            pool.map(_cpu_worker, [(self.kind, c) for c in self.chunks])  # warm the workers' imports
            run_round = lambda: pool.map(_cpu_worker, [(self.kind, c) for c in self.chunks])  # noqa: E731
        try:
            for _ in range(max(warmup, 0)):
                run_round()
            done = 0
            t0 = time.perf_counter()
            while True:
                run_round()
                done += 1
                if rounds is not None and done >= rounds:
                    break
                if rounds is None and time.perf_counter() - t0 >= (budget_s or 0.0):
                    break
            return done * self.units / (time.perf_counter() - t0), cores
        finally:
            if pool is not None:
                pool.close()
                pool.join()


def _host(t) -> "np.ndarray":  # noqa: F821
    """fp32 numpy values of a torch tensor (bf16 values are exact in fp32)."""
    return t.detach().float().cpu().numpy()


def _split(rows, procs: int) -> list:
    """Row chunks of an array (or of each array of a tuple) for ``procs`` processes."""
    n = max(1, min(procs, (rows[0] if isinstance(rows, tuple) else rows).shape[0]))
    if isinstance(rows, tuple):
        return [tuple(r[i::n] for r in rows) for i in range(n)]
    return [rows[i::n] for i in range(n)]


def host_procs() -> int:
    return len(os.sched_getaffinity(0)) if hasattr(os, "sched_getaffinity") else (os.cpu_count() or 1)


# ------------------------------------------------------------------ workloads


class Workload:
    """One benchmarked pass of the hot path. A subclass sets ``name``, ``unit``, ``dtype``,
    ``scaling`` and, in ``setup``, ``units`` (metric units per step), ``kernel`` (the dominant
    kernel), ``kernel_units`` (its algorithmic bytes or FLOPs per launch), ``bound`` ("hbm" or
    "tensor"), ``h2d`` / ``d2h`` and ``config``; ``step()`` runs one step on device-resident
    inputs and returns the number of this library's kernel launches; ``e2e_step()`` one step
    through the public API from host buffers; ``dominant()`` one launch of the dominant
    kernel (default: the step); ``cpu_case(dev)`` the CPU legs' sample, built with torch and
    the oracle only. ``graph`` workloads (microsecond steps) run their K timed steps as one
    CUDA graph over ``step_at(i)`` / ``dominant_at(i)``, each step on its own input copy."""

    name = ""
    unit = ""
    dtype = ""
    scaling = "weak"
    graph = False
    bound = "hbm"
    config: dict = {}

    def setup(self, dev, world, rank):
        raise NotImplementedError

    def step(self):
        raise NotImplementedError

    def e2e_step(self):
        raise NotImplementedError

    def pipelined_e2e(self, hosts, run, out_host):
        """One end-to-end step through the public API, pipelined as a serving loop runs it:
        this step's input copies (pinned `hosts` -> device, on their own stream) and the
        previous step's output copy (device -> pinned host, on another stream) overlap this
        step's kernels. Every step still copies all of its own inputs and its whole output:
        two device input slots and two pinned output buffers alternate. `run(*device_inputs)`
        returns the step's output tensor."""
        torch = self.torch
        if not hasattr(self, "_pipe"):
            dev = torch.device("cuda", torch.cuda.current_device())
            self._pipe = {
                "in": torch.cuda.Stream(), "out": torch.cuda.Stream(), "i": 0,
                "dev": [[torch.empty(h.shape, dtype=h.dtype, device=dev) for h in hosts] for _ in range(2)],
                "host": [out_host, torch.empty_like(out_host).pin_memory()],
                "ev_in": [torch.cuda.Event() for _ in range(2)], "ev_done": [None, None], "ev_out": [None, None],
                "y": [None, None],
            }
        p = self._pipe
        slot = p["i"] % 2
        cur = torch.cuda.current_stream()
        if p["ev_done"][slot] is not None:
            p["in"].wait_event(p["ev_done"][slot])  # step i - 2's kernels have read this input slot
        with torch.cuda.stream(p["in"]):
            for d, h in zip(p["dev"][slot], hosts):
                d.copy_(h, non_blocking=True)
        p["ev_in"][slot].record(p["in"])
        cur.wait_event(p["ev_in"][slot])
        if p["ev_out"][slot] is not None:
            cur.wait_event(p["ev_out"][slot])  # step i - 2's output copy has read its slot
        y = run(*p["dev"][slot])
        done = torch.cuda.Event()
        done.record(cur)
        p["ev_done"][slot] = done
        p["out"].wait_event(done)
        with torch.cuda.stream(p["out"]):
            p["host"][slot].copy_(y, non_blocking=True)
        ev_out = torch.cuda.Event()
        ev_out.record(p["out"])
        p["ev_out"][slot] = ev_out
        p["y"][slot] = y  # alive until its copy is done: step i + 2 waits for ev_out first
        p["i"] += 1

    def e2e_drain(self):
        """Makes the current stream wait for the output copies a pipelined e2e step left."""
        if hasattr(self, "_pipe"):
            for ev in self._pipe["ev_out"]:
                if ev is not None:
                    self.torch.cuda.current_stream().wait_event(ev)

    def cpu_case(self, dev) -> CpuCase:
        raise NotImplementedError

    def tensor_peak(self, pk, pk_kind):
        """The dense 8-bit tensor peak as 2 x the measured bf16 GEMM burst."""
        return 2.0 * pk["bf16_tflops"], f"2 x {pk_kind} bf16 burst ({pk['bf16_tflops']:.0f} TFLOP/s): 8-bit dense"

    def close(self):
        pass


def _rotating_copies(per_step_bytes: int, floor: int = 2) -> int:
    """Input copies whose total exceeds the 126 MB L2 twice over (each step reads HBM)."""
    return max(floor, -(-(256 << 20) // max(per_step_bytes, 1)))


class W4A4Linear(Workload):
    """Config 4: y = fp4_w4a4_linear(x, W) with bias, W [28672, 8192] NVFP4 (tensor scale from
    the whole weight), X [8192, 8192] quantised per token on every step. At N ranks each rank
    holds N / world output channels of W; the GEMM epilogue writes each tile into every rank's
    [M, N] output over NVLink (CUDA IPC peer stores, ``--assemble peer``, the default), or the
    shards are all-gathered by NCCL and reordered (``--assemble nccl``)."""

    name = "w4a4"
    title = "config 4: W4A4 NVFP4 linear with bias, X [8192, 8192] x W [28672, 8192]^T -> bf16"
    unit = "TFLOP/s"
    dtype = "nvfp4 (e2m1 x e2m1, e4m3 / fp32 scales) -> bf16"
    scaling = "strong"
    bound = "tensor"

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
        self.peers = None
        if world > 1 and ASSEMBLE == "peer":
            self.peers = sharded.PeerOutput(m, n, torch.bfloat16, device=dev)
            self.out_local = self.peers.buffer[:, cols]
            self.peer_ptrs = self.peers.peer_ptrs(cols.start)
            self.out, self.gathered = self.peers.buffer, None
        else:
            self.peer_ptrs = None
            self.out_local = torch.empty(m, ns, dtype=torch.bfloat16, device=dev)
            self.out = torch.empty(m, n, dtype=torch.bfloat16, device=dev) if world > 1 else self.out_local
            self.gathered = torch.empty(world, m, ns, dtype=torch.bfloat16, device=dev) if world > 1 else None
        self.units = 2.0 * m * n * k / 1e12
        self.kernel = "gemm_pair_kernel<KIND=3 nvf4, bf16>"
        self.kernel_units = 2.0 * m * ns * k
        self.h2d = m * k * 2
        self.d2h = m * n * 2
        self.x_host = self.x.cpu().pin_memory()
        self.y_host = torch.empty(m, n, dtype=torch.bfloat16).pin_memory()
        self.config = {
            "workload": self.title,
            "m": m, "k": k, "n": n, "step": "NVFP4 activation producer + tcgen05 mxf4nvf4 GEMM (CTA-pair "
            "256 x 256 tiles) with fused epilogue"
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

    def gemm_only_ms(self, steps):
        """The GEMM launches alone (no producer, no barrier or gather), device time per launch."""
        return kernel_ms(self.dominant, steps, self.torch)

    def e2e_step(self):
        """One step through the public API with host buffers: on one GPU pipelined over three
        streams (`pipelined_e2e`), every step copying its own 134 MB in and 470 MB out."""
        if self.world > 1:
            x = self.x_host.to(self.x.device, non_blocking=True)
            y = self.sharded.fp4_w4a4_linear_sharded(x, self.wq, self.ws, self.ts, self.bias,
                                                     out_local=self.out_local, out=self.out, staging=self.gathered,
                                                     peers=self.peers)
            self.y_host.copy_(y, non_blocking=True)
            return 2
        self.pipelined_e2e([self.x_host], lambda x: self.quant.fp4_w4a4_linear(x, self.wq, self.ws, self.ts, self.bias),
                           self.y_host)
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
        """cuBLASLt's NVFP4 GEMM (torch F.scaled_mm, BlockWise1x16) on the same codes, with bf16
        out (the output this GEMM writes) and fp32 out: TFLOP/s."""
        torch = self.torch
        import torch.nn.functional as F

        try:
            xq, xs, outer = self.producers.quantize_rows_fp4(self.x, swizzle=True)
            a = xq.view(torch.float4_e2m1fn_x2)
            b = self.wq.view(torch.float4_e2m1fn_x2).t()
            bar = {}
            for name, odt in (("cublaslt_nvfp4_bf16_tflops", torch.bfloat16), ("cublaslt_nvfp4_tflops", torch.float32)):
                kw = dict(scale_a=xs, scale_recipe_a=F.ScalingType.BlockWise1x16,
                          scale_b=self.ws.view(torch.float8_e4m3fn), scale_recipe_b=F.ScalingType.BlockWise1x16,
                          swizzle_a=F.SwizzleType.SWIZZLE_32_4_4, swizzle_b=F.SwizzleType.SWIZZLE_32_4_4,
                          output_dtype=odt)
                for _ in range(3):
                    F.scaled_mm(a, b, **kw)
                ms, _ = timed(lambda: (F.scaled_mm(a, b, **kw), 1)[1], 10, torch)
                bar[name] = 2.0 * self.m * self.ns * self.k / (ms / 10 / 1e3) / 1e12
            bar["what"] = "F.scaled_mm BlockWise1x16 NVFP4 on the same codes, bf16 and fp32 out (no bias)"
            return bar
        except Exception as exc:  # a torch without the NVFP4 path
            return {"unavailable": f"{type(exc).__name__}: {exc}"[:200]}

    def cpu_case(self, dev):
        import torch

        sys.path.insert(0, str(ROOT))
        from kernel_agent_b200 import workloads
        from oracle import quant as oq

        rows, cols = 64, 4096
        m, k, n = SHAPE or (8192, 8192, 28672)
        x, w, b = workloads.config4(seed=0, device="cuda", m=m, k=k, n=n)
        amax = float(w.float().abs().amax())  # the whole weight's tensor scale (quant.py:253-254)
        codes, scales, ts = oq.quantize_fp4(_host(w[:cols]), amax=amax)
        payload = (_host(x[:rows]), codes, scales, float(ts), _host(b[:cols]))
        del x, w, b
        torch.cuda.empty_cache()
        return CpuCase("w4a4", [payload], 2.0 * rows * cols * k / 1e12,
                       f"the reference's CPU fp4_w4a4_linear (quant.py:1233-1257: NVFP4 activation quantiser, "
                       f"fp32 BLAS matmul of the block-scaled values, epilogue) on {rows} rows x {cols} output "
                       f"channels x K {k} of config 4")


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
        nbytes = self.m * self.k * 2 + self.m * self.k // 2 + self.m * self.k // 16 + 4 * self.m
        self.units = nbytes / 1e9  # GB per step
        self.kernel = "quant_fp4_fast_kernel"
        self.kernel_units = nbytes
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

    def cpu_case(self, dev):
        from kernel_agent_b200 import workloads

        rows, k = 256, 8192
        x, _, _ = workloads.config4(seed=0, device="cuda", n=128)
        gb = rows * k * (2 + 0.5 + 1 / 16) / 1e9
        return CpuCase("nvfp4", _split(_host(x[:rows]), host_procs()), gb,
                       f"oracle quantize_fp4_activations (NVFP4 per token) on {rows} x {k} rows of config 4")


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
        nbytes = 2 * m * f * 2 + m * f + m * f // 32
        self.units = nbytes / 1e9
        self.kernel = "quant_mxfp8_kernel"
        self.kernel_units = nbytes
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

    def cpu_case(self, dev):
        from kernel_agent_b200 import workloads

        rows = 64
        g, u, _ = workloads.config3(seed=0, device="cuda", h=128)
        f = g.shape[1]
        gb = rows * f * (4 + 1 + 1 / 32) / 1e9
        return CpuCase("mxfp8_silu", _split((_host(g[:rows]), _host(u[:rows])), host_procs()), gb,
                       f"oracle SiLU(gate) * up (bf16 roundings) + quantize_mxfp8 on {rows} x {f} rows of config 3")


class Mxfp8Mlp(Workload):
    """Config 3: the MXFP8 MLP block at 8B-class shapes: the fused SiLU(gate) * up -> MXFP8
    producer on gate, up [4096, 14336] (scales written swizzled) and the down-projection GEMM
    against W_down [4096, 14336] (tcgen05 kind::mxf8f6f4, e8m0 per 32 on both operands),
    bf16 out. ``value``: the GEMM's FLOPs per step time (producer included); the producer's
    own GB/s is reported beside it."""

    name = "mxfp8_mlp"
    unit = "TFLOP/s"
    dtype = "mxfp8 (e4m3 x e4m3, e8m0 per 32) -> bf16"
    bound = "tensor"

    def setup(self, dev, world, rank):
        import torch

        from kernel_agent_b200 import workloads
        from kernel_agent_b200.kernels import gemm, producers, quant

        self.torch, self.gemm, self.producers, self.quant = torch, gemm, producers, quant
        g, u, w = workloads.config3(seed=0, device="cuda")
        self.g, self.u = g.to(dev), u.to(dev)
        self.m, self.f = g.shape
        self.h = w.shape[0]
        wq, ws = quant.quantize_mxfp8(w.to(dev))
        del w
        self.wq, self.ws = wq, quant.swizzle_mx_scales(ws).view(torch.uint8)
        self.units = 2.0 * self.m * self.h * self.f / 1e12
        self.kernel = "gemm_pair_kernel<KIND=2 mxf8, bf16>"
        self.kernel_units = 2.0 * self.m * self.h * self.f
        self.producer_bytes = 2 * self.m * self.f * 2 + self.m * self.f + self.m * self.f // 32
        self.out = torch.empty(self.m, self.h, dtype=torch.bfloat16, device=dev)
        self.h2d = 2 * self.m * self.f * 2
        self.d2h = self.m * self.h * 2
        self.g_host, self.u_host = self.g.cpu().pin_memory(), self.u.cpu().pin_memory()
        self.y_host = torch.empty(self.m, self.h, dtype=torch.bfloat16).pin_memory()
        self.config = {"workload": "config 3: MXFP8 MLP block, SiLU(gate [4096, 14336]) * up -> MXFP8, "
                                   "down-projection x W_down [4096, 14336]^T -> bf16",
                       "m": self.m, "f": self.f, "h": self.h,
                       "step": "fused SiLU * up -> MXFP8 producer + tcgen05 mxf8f6f4 GEMM",
                       "l2": "inputs larger than L2 (gate + up 235 MB, W codes 59 MB)"}

    def _gemm(self, xq, xs):
        return self.gemm.mxf8(xq, xs.view(self.torch.uint8), self.wq, self.ws, None, out_dtype=self.torch.bfloat16)

    def step(self):
        xq, xs = self.producers.silu_mul_fp8(self.g, self.u, mx=True, blocked=True)
        self._gemm(xq, xs)
        return 2

    def dominant(self):
        if not hasattr(self, "_x"):
            self._x = self.producers.silu_mul_fp8(self.g, self.u, mx=True, blocked=True)
        self._gemm(*self._x)
        return 1

    def extra(self, steps):
        """The producer kernel alone: device time and GB/s."""
        ms = kernel_ms(lambda: self.producers.silu_mul_fp8(self.g, self.u, mx=True, blocked=True), steps, self.torch)
        return {"producer_kernel_ms": ms, "producer_gbs": self.producer_bytes / (ms / 1e3) / 1e9}

    def e2e_step(self):
        def run(g, u):
            xq, xs = self.producers.silu_mul_fp8(g, u, mx=True, blocked=True)
            return self._gemm(xq, xs)

        self.pipelined_e2e([self.g_host, self.u_host], run, self.y_host)
        return 2

    def library_bar(self):
        """cuBLASLt's MXFP8 GEMM (F.scaled_mm BlockWise1x32, SWIZZLE_32_4_4) on the same codes, bf16 out."""
        torch = self.torch
        import torch.nn.functional as F

        try:
            xq, xs = self.producers.silu_mul_fp8(self.g, self.u, mx=True, blocked=True)
            kw = dict(scale_a=xs.view(torch.float8_e8m0fnu), scale_recipe_a=F.ScalingType.BlockWise1x32,
                      scale_b=self.ws.view(torch.float8_e8m0fnu), scale_recipe_b=F.ScalingType.BlockWise1x32,
                      swizzle_a=F.SwizzleType.SWIZZLE_32_4_4, swizzle_b=F.SwizzleType.SWIZZLE_32_4_4,
                      output_dtype=torch.bfloat16)
            fn = lambda: F.scaled_mm(xq, self.wq.t(), **kw)  # noqa: E731
            for _ in range(3):
                fn()
            ms, _ = timed(lambda: (fn(), 1)[1], 10, torch)
            return {"cublaslt_mxfp8_tflops": self.kernel_units / (ms / 10 / 1e3) / 1e12,
                    "what": "F.scaled_mm BlockWise1x32 MXFP8 on the same codes, bf16 out"}
        except Exception as exc:
            return {"unavailable": f"{type(exc).__name__}: {exc}"[:200]}

    def cpu_case(self, dev):
        sys.path.insert(0, str(ROOT))
        from kernel_agent_b200 import workloads
        from oracle import quant as oq

        rows, cols = 64, 1024
        g, u, w = workloads.config3(seed=0, device="cuda")
        f = g.shape[1]
        wq, ws = oq.quantize_mxfp8(_host(w[:cols]))
        payload = (_host(g[:rows]), _host(u[:rows]), wq, ws)
        return CpuCase("mxfp8_mlp", [payload], 2.0 * rows * cols * f / 1e12,
                       f"the reference's CPU path on {rows} rows x {cols} output channels x K {f} of config 3: "
                       "SiLU * up (bf16), quantize_mxfp8, then mxfp8_linear's fp32 BLAS matmul of the "
                       "dequantised operands (quant.py:615-617)")


class W8a8Config1(Workload):
    """Config 1, the reference's CPU-runnable case: y = int8_w8a8_linear(x, W, bias), X [128,
    1024] bf16 (0.5 % of columns x 20), W [1024, 1024] int8 per channel, bf16 out: the per-token
    producer, the exact int8 GEMM and the fp32 epilogue. A step is microseconds, so the K timed
    steps run as one CUDA graph, step i on input copy i % copies (together larger than L2)."""

    name = "w8a8_config1"
    unit = "TFLOP/s"
    dtype = "int8 x int8 -> int32 -> bf16"
    graph = True
    bound = "tensor"

    def setup(self, dev, world, rank):
        import torch

        from kernel_agent_b200 import workloads
        from kernel_agent_b200.kernels import gemm, quant

        self.torch, self.quant, self.gemm = torch, quant, gemm
        x, w, b = workloads.config1(seed=0, device="cuda")
        self.m, self.k = x.shape
        self.n = w.shape[0]
        q, s = quant.quantize_int8(w.to(dev))
        per_step = self.m * self.k * 2 + self.n * self.k + self.m * self.n * 2
        self.copies = _rotating_copies(per_step)
        self.xs_ = [x.to(dev).clone() for _ in range(self.copies)]
        self.ws_ = [(q.clone(), s.clone()) for _ in range(self.copies)]
        self.bias = b.to(dev)
        self.xq_ = [quant.quantize_int8_activations(t) for t in self.xs_]
        self.units = 2.0 * self.m * self.n * self.k / 1e12
        self.kernel = "gemm_kernel<KIND=0 int8, bf16>"
        self.kernel_units = 2.0 * self.m * self.n * self.k
        self.kernel_bytes = self.m * self.k + self.n * self.k + 4 * (self.m + self.n) + self.m * self.n * 2
        self.h2d = self.m * self.k * 2
        self.d2h = self.m * self.n * 2
        self.x_host = self.xs_[0].cpu().pin_memory()
        self.y_host = torch.empty(self.m, self.n, dtype=torch.bfloat16).pin_memory()
        self.config = {"workload": "config 1: W8A8 INT8 linear with bias, X [128, 1024] x W [1024, 1024]^T -> bf16",
                       "m": self.m, "k": self.k, "n": self.n,
                       "step": "per-token INT8 producer + tcgen05 kind::i8 GEMM with fused dequant / bias epilogue",
                       "l2": f"step i uses copy i % {self.copies} of X and W ({self.copies} x "
                             f"{per_step / 2**20:.2f} MB, larger than L2)",
                       "launch": "the K timed steps are one CUDA graph (2 kernels per step)",
                       "note": "latency-bound (4 output tiles): the roofline gives both the tensor and HBM fractions"}

    def step_at(self, i):
        j = i % self.copies
        q, s = self.ws_[j]
        self.quant.int8_w8a8_linear(self.xs_[j], q, s, self.bias)
        return 2

    def dominant_at(self, i):
        j = i % self.copies
        xq, xs = self.xq_[j]
        q, s = self.ws_[j]
        self.gemm.int8(xq, q, xs, s, self.bias, out_dtype=self.torch.bfloat16)
        return 1

    def step(self):
        return self.step_at(0)

    def e2e_step(self):
        x = self.x_host.to(self.xs_[0].device, non_blocking=True)
        q, s = self.ws_[0]
        self.y_host.copy_(self.quant.int8_w8a8_linear(x, q, s, self.bias), non_blocking=True)
        return 2

    def cpu_case(self, dev):
        sys.path.insert(0, str(ROOT))
        from kernel_agent_b200 import workloads
        from oracle import quant as oq

        x, w, b = workloads.config1(seed=0, device="cuda")
        q, s = oq.quantize_int8(_host(w))
        m, k = x.shape
        return CpuCase("w8a8", [(_host(x), q, s, _host(b))], 2.0 * m * w.shape[0] * k / 1e12,
                       "the reference's CPU int8_w8a8_linear on the whole of config 1 (quant.py:901-923: "
                       "per-token quantiser, int8 product as fp32 BLAS over K = 1024, fp32 epilogue)")


class Fp8Blockwise(Workload):
    """Config 2: y = fp8_blockwise_linear(x, W): x [M, 1024] quantised per 1 x 128 group on
    every step, W [3072, 1024] with 128 x 128 block scales (build time), promoted per
    128-wide K step; bf16 out. M = 2048 (the tensor-bound case; ``fp8_blockwise``), 16 and 1
    (weight-streaming: ``fp8_blockwise_m16``, ``fp8_blockwise_m1``). The step is a few
    microseconds, so the K timed steps run as one CUDA graph, step i on input copy
    i % copies: the copies together are larger than L2, so each step reads HBM."""

    name = "fp8_blockwise"
    graph = True
    unit = "TFLOP/s"
    dtype = "e4m3 x e4m3 (fp32 1x128 / 128x128 scales) -> bf16"
    M = 2048

    def setup(self, dev, world, rank):
        import torch

        from kernel_agent_b200 import workloads
        from kernel_agent_b200.kernels import blockwise, gemm

        self.torch, self.blockwise, self.gemm = torch, blockwise, gemm
        m, k, n = SHAPE or (self.M, 1024, 3072)
        self.m, self.k, self.n = m, k, n
        self.bound = "hbm" if m <= 16 else "tensor"
        x, w = workloads.config2(m, seed=0, device="cuda", k=k, n=n)
        self.x = x.to(dev)
        self.wq, self.ws = blockwise.quantize_fp8_blocks(w.to(dev))
        per_step = m * k * 2 + m * k + n * k + m * n * 2  # x, its codes, W codes, y
        self.copies = _rotating_copies(per_step)
        self.xs_ = [self.x.clone() for _ in range(self.copies)]
        self.ws_ = [(self.wq.clone(), self.ws.clone()) for _ in range(self.copies)]
        self.xq_ = [blockwise.quantize_fp8_groups(t) for t in self.xs_]
        self.units = 2.0 * m * n * k / 1e12
        self.kernel = "gemm_blockwise_kernel" if m > 32 else "gemm_blockwise_skinny_kernel (cluster split-K)"
        self.kernel_bytes = m * k + 4 * m * (k // 128) + n * k + 4 * (n // 128) * (k // 128) + m * n * 2
        self.kernel_units = self.kernel_bytes if self.bound == "hbm" else 2.0 * m * n * k
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
            return {"cublaslt_blockwise_tflops": 2.0 * self.m * self.n * self.k / (ms / 20 / 1e3) / 1e12,
                    "what": "F.scaled_mm BlockWise1x128 x BlockWise128x128, bf16 out, same codes, L2 warm"}
        return {"unavailable": " | ".join(errors)[:400]}

    def cpu_case(self, dev):
        sys.path.insert(0, str(ROOT))
        from kernel_agent_b200 import workloads
        from oracle import fp8lib

        m, k, n = SHAPE or (self.M, 1024, 3072)
        rows = min(m, 64)
        x, w = workloads.config2(m, seed=0, device="cuda", k=k, n=n)
        wq, ws = fp8lib.quantize_fp8_blocks(_host(w))
        return CpuCase("blockwise", [(_host(x[:rows]), wq, ws)], 2.0 * rows * n * k / 1e12,
                       f"the research script's blockwise FP8 linear on the CPU (fp8lib.py:22-40: fake-quantised "
                       f"operands, fp32 BLAS matmul) on {rows} rows x {n} x K {k} of config 2 (M = {m})")


class Fp8BlockwiseM16(Fp8Blockwise):
    name = "fp8_blockwise_m16"
    M = 16


class Fp8BlockwiseM1(Fp8Blockwise):
    name = "fp8_blockwise_m1"
    M = 1


class Fp8Attention(Workload):
    """Config 5: causal FP8 attention prefill, B 4, Hq 32, Hkv 8, S 4096, D 128: the per-head
    e4m3 quantisation of Q, K, V plus the tcgen05 attention kernel; bf16 out."""

    name = "fp8_attention"
    unit = "TFLOP/s"
    dtype = "e4m3 Q K^T and P V (fp32 softmax) -> bf16"
    bound = "tensor"

    def setup(self, dev, world, rank):
        import torch

        from kernel_agent_b200 import workloads
        from kernel_agent_b200.kernels import attention

        self.torch, self.attention = torch, attention
        self.q, self.k, self.v = (t.to(dev) for t in workloads.config5(seed=0, device="cuda"))
        b, hq, s, d = self.q.shape
        self.b, self.hq, self.s, self.d = b, hq, s, d
        # causal: sum over query tiles of the keys up to the diagonal, both products
        flops = 4.0 * b * hq * d * (s * (s + 1) / 2)
        self.units = flops / 1e12
        self.kernel = "attention_fp8_kernel"
        self.kernel_units = flops
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
        self.pipelined_e2e(list(self.hosts),
                           lambda q, k, v: self.attention.attention_fp8(q, k, v, is_causal=True, enable_gqa=True),
                           self.y_host)
        return 7

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
            return {"sdpa_bf16_tflops": self.kernel_units / (ms / 5 / 1e3) / 1e12,
                    "what": "F.scaled_dot_product_attention bf16, causal, enable_gqa (not FP8)"}
        except Exception as exc:
            return {"unavailable": f"{type(exc).__name__}: {exc}"[:200]}

    def cpu_case(self, dev):
        from kernel_agent_b200 import workloads

        q, k, v = workloads.config5(seed=0, device="cuda")
        s, d = q.shape[2], q.shape[3]
        return CpuCase("attention", [(_host(q[0, 0]), _host(k[0, 0]), _host(v[0, 0]))], 4.0 * d * (s * (s + 1) / 2) / 1e12,
                       "the research script's emulated_sdpa (qkpv, fp8lib.py:184-215: fake-quantised Q, K, V, fp32 "
                       f"BLAS scores and P V) of one (batch, head) [{s} x {s}] of config 5")


class Compare(Workload):
    name = "compare"
    unit = "GB/s"
    dtype = "bf16"

    def setup(self, dev, world, rank):
        import torch

        from kernel_agent_b200.kernels import compare

        self.torch, self.compare = torch, compare
        self.ref, self.new = _compare_pair(dev)
        n = self.ref.numel()
        self.units = 2 * n * 2 / 1e9  # one read of each (exact tier)
        self.kernel = "compare_kernel"
        self.kernel_units = 2 * n * 2
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

    def cpu_case(self, dev):
        rows = 1024
        ref, new = _compare_pair(dev, rows)
        return CpuCase("compare", _split((_host(ref), _host(new)), host_procs()), rows * 28672 * 2 * 2 / 1e9,
                       f"oracle compare_tensors (exact tier) on {rows} rows of the config-4-sized bf16 pair")


def _compare_pair(dev, rows: int | None = None):
    """The comparator's bf16 [8192, 28672] pair (a config-4-sized output and a 1 % perturbation),
    drawn on the GPU; its first ``rows`` rows when given."""
    import torch

    g = torch.Generator(device="cuda").manual_seed(0)
    shape = (8192, 28672)
    ref = torch.randn(*shape, generator=g, device="cuda").to(torch.bfloat16)
    new = (ref.float() * (1 + 0.01 * torch.randn(*shape, generator=g, device="cuda"))).to(torch.bfloat16)
    if rows is not None:
        ref, new = ref[:rows].clone(), new[:rows].clone()
    return ref.to(dev), new.to(dev)


class W8a8Decode(Workload):
    """Decode-size W8A8: y = int8_w8a8_linear(x, W) at M = 16 tokens, X [16, 4096],
    W [14336, 4096] int8 (58.7 MB, per-channel scales), bf16 out: the per-token producer and
    the skinny GEMM (the weight streams through the tensor core). Four weight copies rotate so
    every step reads its weight from HBM (4 x 58.7 MB > L2)."""

    name = "w8a8_decode"
    unit = "GB/s"
    dtype = "int8 x int8 -> int32 -> bf16"
    graph = True

    def _inputs(self, dev):
        import torch

        g = torch.Generator(device="cuda").manual_seed(0)
        x = torch.randn(16, 4096, device="cuda", generator=g).to(torch.bfloat16)
        w = (torch.randn(14336, 4096, device="cuda", generator=g) * 0.02).to(torch.bfloat16)
        bias = (torch.randn(14336, device="cuda", generator=g) * 0.1).to(torch.bfloat16)
        return x.to(dev), w.to(dev), bias.to(dev)

    def setup(self, dev, world, rank):
        import torch

        from kernel_agent_b200.kernels import gemm, quant

        self.torch, self.quant, self.gemm = torch, quant, gemm
        self.x, w, self.bias = self._inputs(dev)
        self.m, self.k = self.x.shape
        self.n = w.shape[0]
        q, s = quant.quantize_int8(w)
        del w
        self.copies = [(q.clone(), s.clone()) for _ in range(4)]
        self.i = 0
        wbytes = self.n * self.k + 4 * self.n
        self.units = (wbytes + self.m * self.k * 2 + self.m * self.n * 2) / 1e9
        self.kernel = "gemm_skinny_kernel<KIND=0 int8>"
        self.kernel_units = wbytes + self.m * self.k + self.m * self.n * 2
        self.x_host = self.x.cpu().pin_memory()
        self.y_host = torch.empty(self.m, self.n, dtype=torch.bfloat16).pin_memory()
        self.h2d = self.m * self.k * 2
        self.d2h = self.m * self.n * 2
        self.config = {"workload": "decode-size W8A8 INT8 linear, X [16, 4096] x W [14336, 4096]^T -> bf16",
                       "m": self.m, "k": self.k, "n": self.n,
                       "l2": "4 rotating weight copies (235 MB) larger than L2",
                       "launch": "the K timed steps are one CUDA graph (2 kernels per step)"}

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
        self.i += 1
        q, s = self.copies[self.i % len(self.copies)]
        self.y_host.copy_(self.quant.int8_w8a8_linear(x, q, s, self.bias), non_blocking=True)
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

    def cpu_case(self, dev):
        sys.path.insert(0, str(ROOT))
        from oracle import quant as oq

        cols = 1024
        x, w, bias = self._inputs(dev)
        q, s = oq.quantize_int8(_host(w[:cols]))
        gb = (cols * 4096 + 16 * 4096 * 2 + 16 * cols * 2) / 1e9
        return CpuCase("w8a8", [(_host(x), q, s, _host(bias[:cols]))], gb,
                       f"the reference's CPU int8_w8a8_linear on X [16, 4096] x {cols} weight rows")


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

    def _draw(self, dev, copies):
        import torch

        g = torch.Generator(device="cuda").manual_seed(0)
        q = torch.randn(4, 16, 128, device="cuda", generator=g).to(torch.bfloat16)
        kvs = []
        for _ in range(copies):
            k = torch.randn(4, 2, 4096, 128, device="cuda", generator=g).to(torch.bfloat16)
            v = torch.randn(4, 2, 4096, 128, device="cuda", generator=g).to(torch.bfloat16)
            kvs.append((k.to(dev), v.to(dev)))
        return q.to(dev), kvs

    def setup(self, dev, world, rank):
        import torch

        from kernel_agent_b200.kernels import kv_quant

        self.torch, self.kv = torch, kv_quant
        self.b, self.hq, self.hkv, self.l, self.d = 4, 16, 2, 4096, 128
        self.q, kvs = self._draw(dev, 24)
        self.copies = [(*kv_quant.quantize_kv(k), *kv_quant.quantize_kv(v)) for k, v in kvs]
        self.bf16_kv = kvs[:12]  # the bf16 cache of the library bar, rotated the same way (201 MB > L2)
        rows = self.b * self.hkv * self.l
        qo = 2 * self.b * self.hq * self.d * 2
        nbytes = 2 * rows * self.d + 2 * rows * 4 + qo
        self.units = nbytes / 1e9
        self.kernel = "kv_decode_kernel<128, 8, bf16>"
        self.kernel_units = nbytes
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
        self.y_host.copy_(self.kv.fp8_kv_decode(q, kc, ks, vc, vs), non_blocking=True)
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

    def cpu_case(self, dev):
        sys.path.insert(0, str(ROOT))
        from oracle import kv_quant as okv

        q, kvs = self._draw(dev, 1)
        k, v = kvs[0]
        kc, ks = okv.quantize_fp8_kv(_host(k[:1]))
        vc, vs = okv.quantize_fp8_kv(_host(v[:1]))
        gb = (2 * 2 * 4096 * 128 + 2 * 2 * 4096 * 4 + 2 * 16 * 128 * 2) / 1e9
        return CpuCase("kv", [(_host(q[:1, :, None]), kc, ks, vc, vs)], gb,
                       "oracle fp8_kv_attention (kv_quant.py:56-83) on one sequence of the batch")


class RmsnormFp8(Workload):
    """The fused RMSNorm -> FP8 producer (triton_fp8_producers.py:191-202, per-token e4m3):
    x [16384, 4096] bf16, one pass over x (the norm kept in registers, then the codes)."""

    name = "rmsnorm_fp8"
    unit = "GB/s"
    dtype = "bf16->e4m3"

    def _inputs(self, dev):
        import torch

        g = torch.Generator(device="cuda").manual_seed(0)
        x = (torch.randn(16384, 4096, device="cuda", generator=g) * 3).to(torch.bfloat16)
        w = (1.0 + 0.1 * torch.randn(4096, device="cuda", generator=g)).to(torch.bfloat16)
        return x.to(dev), w.to(dev)

    def setup(self, dev, world, rank):
        import torch

        from kernel_agent_b200.kernels import producers

        self.torch, self.producers = torch, producers
        self.x, self.w = self._inputs(dev)
        self.m, self.k = self.x.shape
        nbytes = self.m * self.k * 2 + self.k * 2 + self.m * self.k + 4 * self.m
        self.units = nbytes / 1e9
        self.kernel = "rmsnorm_quant_fp8_packed_kernel"
        self.kernel_units = nbytes
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

    def _two_pass(self):
        return self.producers.quantize_rows(self.producers._rmsnorm(self.x, self.w, 1e-6, None))

    def library_bar(self):
        """The same result in two passes (kab_rmsnorm into h, then the quantiser)."""
        torch = self.torch
        try:
            for _ in range(3):
                self._two_pass()
            ms, _ = timed(lambda: (self._two_pass(), 1)[1], 10, torch)
            return {"two_pass_gbs": self.kernel_units / (ms / 10 / 1e3) / 1e9, "two_pass_ms": ms / 10,
                    "what": "kab_rmsnorm then the quantiser, the same algorithmic bytes"}
        except Exception as e:  # noqa: BLE001 - the bar is informational
            return {"unavailable": f"{type(e).__name__}: {e}"[:200]}

    def cpu_case(self, dev):
        rows = 256
        x, w = self._inputs(dev)
        k = x.shape[1]
        per_row = k * 2 + k + 4 if self.name == "rmsnorm_fp8" else k * 2 + k // 2 + k // 16 + 4
        procs = host_procs()
        xs = _host(x[:rows])
        chunks = [(c, _host(w)) for c in _split(xs, procs)]
        return CpuCase(self.name, chunks, rows * per_row / 1e9,
                       f"oracle rmsnorm + the {'FP8' if self.name == 'rmsnorm_fp8' else 'NVFP4'} per-token "
                       f"quantiser on {rows} rows x {k}")


class RmsnormFp4(RmsnormFp8):
    """The fused RMSNorm -> NVFP4 producer (triton_fp4_producers.py:384-405, per-token outer
    scale): x [16384, 4096] bf16, one pass over x (the norm kept in registers, then the codes,
    block scales and outer scales)."""

    name = "rmsnorm_fp4"
    dtype = "bf16->e2m1"

    def setup(self, dev, world, rank):
        super().setup(dev, world, rank)
        m, k = self.m, self.k
        nbytes = m * k * 2 + k * 2 + m * k // 2 + m * k // 16 + 4 * m
        self.units = nbytes / 1e9
        self.kernel = "quant_fp4_fast_kernel<NORM>"
        self.kernel_units = nbytes
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

    def _two_pass(self):
        return self.producers.quantize_rows_fp4(self.producers._rmsnorm(self.x, self.w, 1e-6, None))


WORKLOADS = {w.name: w for w in (W4A4Linear, Nvfp4Producer, W8a8Config1, Fp8Blockwise, Fp8BlockwiseM16,
                                  Fp8BlockwiseM1, Mxfp8Mlp, Mxfp8Producer, Fp8Attention, Compare, W8a8Decode,
                                  KvDecode, RmsnormFp8, RmsnormFp4)}
DEFAULT = "w4a4"
# the rest of the metric and the other configurations, measured beside the default line at one GPU
SUB_RESULTS = ("nvfp4_producer", "w8a8_config1", "fp8_blockwise_m1", "fp8_blockwise_m16", "fp8_blockwise",
               "mxfp8_mlp", "compare", "fp8_attention")


# ------------------------------------------------------------------ timing


def timed(fn, steps: int, torch, drain=None):
    """(total ms of `steps` calls on the current stream, launches) with CUDA events. `drain`,
    if given, runs before the end event (it makes the current stream wait for work that `fn`
    left on other streams)."""
    launches = 0
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    start.record()
    for _ in range(steps):
        launches += fn()
    if drain is not None:
        drain()
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


def roofline(wl, k_ms: float) -> dict:
    """The dominant kernel against the measured peak of its bound."""
    pk, pk_kind = peaks()
    if wl.bound == "hbm":
        achieved = wl.kernel_units / (k_ms / 1e3) / 1e9
        peak = pk["hbm_gbs"]
        roof = {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s", "frac": achieved / peak,
                "peak_kind": f"{pk_kind} copy bandwidth"}
    else:
        achieved = wl.kernel_units / (k_ms / 1e3) / 1e12
        peak, peak_kind = wl.tensor_peak(pk, pk_kind)
        roof = {"bound": "tensor", "achieved": achieved, "peak": peak, "unit": "TFLOP/s", "frac": achieved / peak,
                "peak_kind": peak_kind}
        if hasattr(wl, "kernel_bytes"):  # latency-bound shapes: the HBM side too
            gbs = wl.kernel_bytes / (k_ms / 1e3) / 1e9
            roof["hbm_gbs"], roof["hbm_frac"] = gbs, gbs / pk["hbm_gbs"]
    roof["kernel"] = wl.kernel
    roof["kernel_ms"] = k_ms
    traffic = None
    if TRAFFIC_FILE.exists():
        traffic = json.loads(TRAFFIC_FILE.read_text()).get(f"{wl.kernel} {wl.name}")
    roof["traffic"] = traffic
    return roof


def measure(wl, dist, torch, steps: int, warmup: int) -> dict:
    """Warm-up, then exactly `steps` timed steps between barriers (max over ranks), the dominant
    kernel's device time, and the public-API end-to-end time with host buffers."""
    for _ in range(warmup):
        wl.step()
    torch.cuda.synchronize()
    if wl.graph:
        # launch-bound steps: the K timed steps (and K dominant launches) are one CUDA graph,
        # each step on its own copy of the inputs (the copies together exceed L2)
        steps_graph = as_graph(lambda: sum(wl.step_at(i) for i in range(steps)), torch)
        dom_graph = as_graph(lambda: sum(wl.dominant_at(i) for i in range(steps)), torch)
        steps_graph()
        torch.cuda.synchronize()
    dist.barrier()
    clocks = Clocks(dist.local)
    clocks.start()
    time.sleep(0.3)
    dist.barrier()
    if wl.graph:
        total_ms, launches = timed(steps_graph, 1, torch)
        dist.barrier()
        k_ms = kernel_ms(dom_graph, 1, torch) / steps
    else:
        total_ms, launches = timed(wl.step, steps, torch)
        dist.barrier()
        k_ms = kernel_ms(getattr(wl, "dominant", wl.step), steps, torch)
    clk = clocks.stop()
    total_ms = dist.max(total_ms)
    k_ms = dist.max(k_ms)
    ms_per_step = total_ms / steps
    value = wl.units * dist.world / (ms_per_step / 1e3) if wl.scaling == "weak" else wl.units / (ms_per_step / 1e3)
    for _ in range(2):
        wl.e2e_step()
    torch.cuda.synchronize()
    dist.barrier()
    e2e_steps = max(3, steps // 2)
    e2e_ms, _ = timed(wl.e2e_step, e2e_steps, torch, getattr(wl, "e2e_drain", None))
    e2e_ms = dist.max(e2e_ms) / e2e_steps
    e2e_value = wl.units * dist.world / (e2e_ms / 1e3) if wl.scaling == "weak" else wl.units / (e2e_ms / 1e3)
    out = {"value": value, "unit": wl.unit, "ms_per_step": ms_per_step, "roofline": roofline(wl, k_ms),
           "e2e": {"value": e2e_value, "unit": wl.unit, "h2d_bytes_per_step": wl.h2d, "d2h_bytes_per_step": wl.d2h},
           "gpu_launches": launches, "clocks": clk}
    if hasattr(wl, "extra"):
        out.update(wl.extra(steps))
    return out


def cpu_leg(wl, dev, budget_s: float) -> dict:
    case = wl.cpu_case(dev)
    rate, cores = case.run(budget_s=budget_s)
    return {"value": rate, "unit": wl.unit, "cores": cores, "kind": "port", "sample": case.sample}


def sub_result(name: str, dev, dist, torch, steps: int, warmup: int) -> dict:
    """One other configuration measured beside the default line: its value, roofline, library
    bar and CPU baseline (a shorter CPU budget than the main line's)."""
    wl = WORKLOADS[name]()
    try:
        wl.setup(dev, 1, 0)
        res = {"metric_unit": wl.unit, "config": wl.config, "dtype": wl.dtype}
        res.update(measure(wl, dist, torch, steps, warmup))
        bar = getattr(wl, "library_bar", None)
        if bar is not None:
            res["library_bar"] = bar()
        res["cpu_baseline"] = cpu_leg(wl, dev, 3.0)
        res.pop("clocks", None)
        return res
    except Exception as exc:  # noqa: BLE001 - one sub-result failing keeps the line
        return {"error": f"{type(exc).__name__}: {exc}"[:300]}
    finally:
        wl.close()
        del wl
        torch.cuda.synchronize()
        torch.cuda.empty_cache()


def main() -> int:
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=("kab", "reference"), default="kab")
    ap.add_argument("--workload", default=None)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-sub-results", action="store_true", help="the default line without the other configurations")
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

    name = args.workload or DEFAULT
    if name not in WORKLOADS:
        print(json.dumps({"error": f"unknown workload {name}", "known": sorted(WORKLOADS)}))
        return 2

    dist = Dist()
    torch = dist.torch
    dev = torch.device("cuda", dist.local)
    torch.cuda.set_device(dev)
    wl = WORKLOADS[name]()

    if args.impl == "reference":
        # the reference's CPU execution path on this host's cores, on the sample the GPU arm's
        # cpu_baseline uses; its inputs come from torch and the oracle (libkab is not loaded)
        if dist.rank != 0:
            dist.close()
            return 0
        t0 = time.perf_counter()
        case = wl.cpu_case(dev)
        rate, cores = case.run(rounds=args.steps, warmup=min(args.warmup, 3))
        line = {
            "impl": "reference", "metric": METRIC, "value": rate, "unit": wl.unit,
            "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": None, "higher_is_better": True, "scaling": wl.scaling,
            "vs_baseline": None, "dtype": wl.dtype, "data": "synthetic (seeded)",
            "config": {"workload": getattr(wl, "title", name)},
            "cpu_baseline": {"value": rate, "unit": wl.unit, "cores": cores, "kind": "port", "sample": case.sample},
            "e2e": {"value": rate, "unit": wl.unit, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
            "wall_s": round(time.perf_counter() - t0, 1),
        }
        print(json.dumps(line))
        dist.close()
        return 0

    wl.setup(dev, dist.world, dist.rank)
    res = measure(wl, dist, torch, args.steps, args.warmup)
    extra = {}
    if name == "w4a4":
        extra["gemm_only_ms"] = dist.max(wl.gemm_only_ms(args.steps))
    library = wl.library_bar() if hasattr(wl, "library_bar") else None
    cpu = None
    if dist.rank == 0 and dist.world == 1 and not args.no_cpu_baseline:
        cpu = cpu_leg(wl, dev, 10.0)
    line = {
        "metric": METRIC, "value": res["value"], "unit": wl.unit, "n_gpus": dist.world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": res["ms_per_step"],
        "higher_is_better": True, "scaling": wl.scaling, "vs_baseline": None,
        "dtype": wl.dtype, "data": "synthetic (seeded)", "config": wl.config,
        "roofline": res["roofline"], "cpu_baseline": cpu, "e2e": res["e2e"],
        "gpu_launches": res["gpu_launches"], "clocks": res["clocks"],
    }
    line.update(extra)
    for key in ("producer_kernel_ms", "producer_gbs"):
        if key in res:
            line[key] = res[key]
    if library is not None:
        line["library_bar"] = library
    closer = getattr(wl, "close", None)
    if closer is not None:
        closer()
    if name == DEFAULT and dist.world == 1 and not args.no_sub_results and SHAPE is None:
        del wl
        torch.cuda.empty_cache()
        line["sub_results"] = {sub: sub_result(sub, dev, dist, torch, args.steps, args.warmup) for sub in SUB_RESULTS}
    if dist.rank == 0:
        print(json.dumps(line))
    dist.close()
    return 0


if __name__ == "__main__":
    sys.exit(main())

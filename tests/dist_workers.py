"""Worker bodies for the multi-process tests (run under ``torch.multiprocessing`` with the
``spawn`` start method; each returns its result through a queue)."""

from __future__ import annotations

import os
import sys
import traceback
from pathlib import Path

ROOT = Path(__file__).resolve().parents[1]


def _init(rank: int, world: int, port: int, backend: str) -> None:
    for p in (str(ROOT), str(ROOT / "kernel-agent_b200")):
        if p not in sys.path:
            sys.path.insert(0, p)
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    import datetime

    import torch.distributed as dist

    dist.init_process_group(backend, rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))


def run(rank: int, world: int, port: int, backend: str, body: str, queue) -> None:
    import torch.distributed as dist

    try:
        _init(rank, world, port, backend)
        result = globals()[body](rank, world)
        queue.put((rank, "ok", result))
    except BaseException:  # reported to the parent, which fails the test
        queue.put((rank, "error", traceback.format_exc()))
    finally:
        if dist.is_initialized():
            dist.destroy_process_group()


# ------------------------------------------------------------------ bodies (CPU, gloo)


def gather_body(rank: int, world: int):
    import torch

    from kernel_agent_b200.kernels import sharded

    m, ns = 5, 3
    local = torch.arange(m * ns, dtype=torch.float32).reshape(m, ns) + 1000.0 * rank
    full = sharded.gather_columns(local)
    return full.tolist()


def amax_body(rank: int, world: int):
    import torch

    from kernel_agent_b200.kernels import sharded

    plain = sharded.global_amax(torch.tensor(0.5 + rank, dtype=torch.float32))
    nan_in = torch.tensor(float("nan") if rank == world - 1 else 2.0, dtype=torch.float32)
    with_nan = sharded.global_amax(nan_in)
    return [float(plain), float(with_nan)]


# ------------------------------------------------------------------ bodies (GPUs, NCCL)


def w4a4_body(rank: int, world: int):
    import torch

    from kernel_agent_b200 import workloads
    from kernel_agent_b200.kernels import quant, sharded

    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    m, k, n = 256, 1024, 1024
    x, w, b = workloads.config4(seed=3, device="cpu", m=m, k=k, n=n)
    cols = sharded.shard_columns(n, world, rank)
    codes, scales, ts = sharded.quantize_fp4_weight_shard(w[cols].to(dev))
    fc, fs, fts = quant.quantize_fp4(w.to(dev))  # the unsharded quantisation, for comparison
    same_codes = bool(torch.equal(codes, fc[cols]) and torch.equal(scales.view(torch.uint8),
                                                                   fs[cols].view(torch.uint8)))
    same_ts = bool(torch.equal(ts, fts))
    y = sharded.fp4_w4a4_linear_sharded(x.to(dev), codes, scales, ts, b[cols].to(dev))
    y_full = quant.fp4_w4a4_linear(x.to(dev), fc, fs, fts, b.to(dev))
    return [same_codes, same_ts, bool(torch.equal(y, y_full)), float((y.float() - y_full.float()).abs().max())]


def w4a4_fused_body(rank: int, world: int):
    """The fused path: each rank's GEMM epilogue writes its column shard into every rank's
    output (CUDA IPC). Two calls on one buffer (the second after the output changed), with M
    not a multiple of the 128-row tile; each must equal the one-GPU linear bit for bit."""
    import torch

    from kernel_agent_b200 import workloads
    from kernel_agent_b200.kernels import quant, sharded

    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    m, k, n = 200, 1024, 1536
    x, w, b = workloads.config4(seed=5, device="cpu", m=m, k=k, n=n)
    cols = sharded.shard_columns(n, world, rank)
    codes, scales, ts = sharded.quantize_fp4_weight_shard(w[cols].to(dev))
    fc, fs, fts = quant.quantize_fp4(w.to(dev))
    peers = sharded.PeerOutput(m, n, torch.bfloat16, device=dev)
    results = []
    try:
        for scale in (1.0, -0.5):
            xs = (x * scale).to(dev)
            y = sharded.fp4_w4a4_linear_sharded(xs, codes, scales, ts, b[cols].to(dev), peers=peers)
            y_full = quant.fp4_w4a4_linear(xs, fc, fs, fts, b.to(dev))
            torch.cuda.synchronize()
            results.append(bool(torch.equal(y, y_full)))
            results.append(float((y.float() - y_full.float()).abs().max()))
        peers.barrier()  # nobody unmaps while another rank may still write
        torch.cuda.synchronize()
    finally:
        peers.close()
    return results

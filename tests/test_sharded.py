"""Host logic of the column-sharded W4A4 linear with two gloo ranks on the CPU: the shard
partition, the all-reduced tensor-scale amax (NaN-keeping) and the all-gather + reordering
of column shards. The same code over NCCL on two GPUs is ``test_gpu_sharded.py``."""

from __future__ import annotations

import socket

import pytest
import torch.multiprocessing as mp

import dist_workers


def free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def run_ranks(body: str, world: int = 2, backend: str = "gloo", timeout: float = 120.0):
    ctx = mp.get_context("spawn")
    queue = ctx.Queue()
    port = free_port()
    procs = [ctx.Process(target=dist_workers.run, args=(r, world, port, backend, body, queue)) for r in range(world)]
    for p in procs:
        p.start()
    results = {}
    try:
        for _ in range(world):
            rank, status, value = queue.get(timeout=timeout)
            assert status == "ok", f"rank {rank} failed:\n{value}"
            results[rank] = value
    finally:
        for p in procs:
            p.join(timeout=30)
            if p.is_alive():
                p.kill()
    return [results[r] for r in range(world)]


def test_shard_columns_partition():
    from kernel_agent_b200.kernels import sharded

    for world in (1, 2, 4, 8):
        shards = [sharded.shard_columns(28672, world, r) for r in range(world)]
        assert shards[0].start == 0 and shards[-1].stop == 28672
        assert all(a.stop == b.start for a, b in zip(shards, shards[1:]))
        assert all((s.stop - s.start) % 128 == 0 for s in shards)
    with pytest.raises(ValueError):
        sharded.shard_columns(28672 + 64, 2, 0)
    with pytest.raises(ValueError):
        sharded.shard_columns(1024, 2, 2)


def test_gather_columns_two_ranks():
    outs = run_ranks("gather_body")
    m, ns, world = 5, 3, 2
    want = [[float(i * ns + j) + 1000.0 * r for r in range(world) for j in range(ns)] for i in range(m)]
    for out in outs:
        assert out == want


def test_global_amax_two_ranks():
    outs = run_ranks("amax_body")
    for plain, with_nan in outs:
        assert plain == 1.5
        assert with_nan != with_nan  # NaN on one rank is NaN everywhere

"""The column-sharded W4A4 linear over NCCL on two GPUs: each rank's shard quantised with the
all-reduced tensor scale equals the slice of the unsharded quantisation bit for bit, and the
gathered output equals the one-GPU linear. Skipped with fewer than two GPUs."""

from __future__ import annotations

import pytest
import torch

from test_sharded import run_ranks

pytestmark = pytest.mark.gpu


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_w4a4_sharded_matches_one_gpu():
    for same_codes, same_ts, same_y, max_diff in run_ranks("w4a4_body", world=2, backend="nccl", timeout=300):
        assert same_codes and same_ts
        assert same_y, max_diff


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_w4a4_fused_peer_stores_match_one_gpu():
    """The GEMM epilogue writes every rank's shard straight into every rank's output (CUDA IPC
    over NVLink): the full output equals the one-GPU linear, on two successive calls."""
    for eq1, d1, eq2, d2 in run_ranks("w4a4_fused_body", world=2, backend="nccl", timeout=300):
        assert eq1, d1
        assert eq2, d2


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_w4a4_fused_peer_stores_with_the_pair_kernel(monkeypatch):
    """The same with the CTA-pair GEMM forced on (the kernel the large shapes take): its
    epilogue's TMA stores into the peer's IPC mapping, M = 200 inside one 256-row pair tile."""
    monkeypatch.setenv("KAB_GEMM_PAIR", "1")  # the spawned ranks inherit it
    for eq1, d1, eq2, d2 in run_ranks("w4a4_fused_body", world=2, backend="nccl", timeout=300):
        assert eq1, d1
        assert eq2, d2

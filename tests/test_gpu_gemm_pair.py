"""Both tile kernels on every GEMM parity case. The library picks the CTA-pair kernel (two SMs
per 256 x 256 tile, tcgen05.mma.cta_group::2) for large shapes and the one-CTA kernel for the
rest; KAB_GEMM_PAIR (read once per process) forces one of them. So the GEMM parity tests run
again in child processes: with the pair kernel forced on, every shape with M > 128 and
N >= 256 goes through it, and with it forced off the full-size configuration tests go
through the one-CTA kernel."""

from __future__ import annotations

import os
import subprocess
import sys
from pathlib import Path

import pytest
import torch

pytestmark = pytest.mark.gpu

HERE = Path(__file__).resolve().parent


def run_with(mode: str, *files: str) -> None:
    env = dict(os.environ, KAB_GEMM_PAIR=mode)
    r = subprocess.run([sys.executable, "-m", "pytest", *(str(HERE / f) for f in files), "-q", "-x", "-m", "gpu",
                        "-p", "no:cacheprovider"], env=env, capture_output=True, text=True, timeout=900, cwd=HERE.parent)
    assert r.returncode == 0, r.stdout[-4000:] + r.stderr[-2000:]


@pytest.mark.skipif(not torch.cuda.is_available(), reason="needs a GPU")
def test_gemm_parity_with_pair_kernel_forced():
    run_with("1", "test_gpu_gemm.py", "test_gpu_fp4_options.py")


@pytest.mark.skipif(not torch.cuda.is_available(), reason="needs a GPU")
def test_full_configs_with_one_cta_kernel_forced():
    run_with("0", "test_gpu_full_configs.py")

"""The CTA-pair GEMM kernel (two SMs per 256 x 256 tile, tcgen05.mma.cta_group::2) is opt-in
(KAB_GEMM_PAIR=1, read once per process): the GEMM parity tests run again in a child process
with it on, so every shape with M > 128 and N >= 256 goes through it."""

from __future__ import annotations

import os
import subprocess
import sys
from pathlib import Path

import pytest
import torch

pytestmark = pytest.mark.gpu

HERE = Path(__file__).resolve().parent


@pytest.mark.skipif(not torch.cuda.is_available(), reason="needs a GPU")
def test_gemm_parity_with_pair_kernel():
    env = dict(os.environ, KAB_GEMM_PAIR="1")
    r = subprocess.run([sys.executable, "-m", "pytest", str(HERE / "test_gpu_gemm.py"), "-q", "-x", "-m", "gpu",
                        "-p", "no:cacheprovider"], env=env, capture_output=True, text=True, timeout=900, cwd=HERE.parent)
    assert r.returncode == 0, r.stdout[-4000:] + r.stderr[-2000:]

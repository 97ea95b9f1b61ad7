"""FP8 attention prefill on the GPU: the per-head quantiser bit for bit against the oracle
(fp8lib.py:173-176), and the tcgen05 attention against fp32 attention by relative L2 and
cosine next to the reference emulation's own error (fp8lib.py:184-215, mode "qkpv"), on the
golden case and at configuration 5's shapes on sampled heads."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from helpers import np_bytes, np_values
from oracle import fp8lib as ofp8
from oracle.formats import bf16_to_f32

pytestmark = pytest.mark.gpu
DEV = "cuda"


@pytest.fixture(scope="module")
def ka():
    from kernel_agent_b200.kernels import attention

    return attention


def rel_cos(got: np.ndarray, want: np.ndarray) -> tuple[float, float]:
    a, b = got.astype(np.float64).ravel(), want.astype(np.float64).ravel()
    return float(np.linalg.norm(a - b) / np.linalg.norm(b)), float(a @ b / (np.linalg.norm(a) * np.linalg.norm(b)))


def bf(g, key):
    return torch.from_numpy(g[key].view(np.int16)).view(torch.bfloat16)


@pytest.mark.parametrize("shape", [(2, 3, 256, 128), (1, 1, 128, 64), (4, 2, 192, 128), (1, 2, 100, 128),
                                   (2, 2, 37, 64)])
@pytest.mark.parametrize("transpose", [False, True])
def test_quantize_heads_bit_exact(ka, shape, transpose):
    g = torch.Generator().manual_seed(sum(shape))
    x = (torch.randn(*shape, generator=g) * torch.logspace(-3, 3, shape[1])[None, :, None, None]).to(torch.bfloat16)
    x[0, 0, 5, 7] = 0.0
    if shape[1] > 1:
        x[-1, 1] = 0.0  # a zero head: scale 1
    codes, scales = ka.quantize_fp8_heads(x.to(DEV), transpose=transpose)
    rc, rs = ofp8.quantize_head(np_values(x))
    assert np.array_equal(scales.cpu().numpy(), rs)
    got = np_bytes(codes)
    if transpose:
        got = np.swapaxes(got, -1, -2)
    assert np.array_equal(got, rc)


def test_attention_golden(ka, golden):
    """The reference emulation's output (att2: B 1, Hq 4, Hkv 2, S 256, D 128): ours is as close
    to fp32 attention as the emulation is, and close to the emulation itself."""
    g = golden
    q, k, v = bf(g, "att2_q").to(DEV), bf(g, "att2_k").to(DEV), bf(g, "att2_v").to(DEV)
    fp32 = g["att2_y_fp32"]
    for key, causal in (("att2_y", True), ("att2_y_nc", False)):
        y = ka.attention_fp8(q, k, v, is_causal=causal, enable_gqa=True)
        assert y.dtype == torch.bfloat16 and y.shape == q.shape
        got = np_values(y.cpu())
        emu = bf16_to_f32(g[key])
        rel_e, cos_e = rel_cos(got, emu)
        assert rel_e < 0.03 and cos_e > 0.9995, (key, rel_e, cos_e)
        if causal:
            rel, cos = rel_cos(got, fp32)
            rel_ref, _ = rel_cos(emu, fp32)
            assert rel < max(0.05, 1.25 * rel_ref) and cos > 0.998, (rel, rel_ref, cos)


def test_attention_config5_heads(ka):
    """Configuration 5 (B 4, Hq 32, Hkv 8, S 4096, D 128, causal): the whole call on the GPU,
    sampled heads against the oracle's fp32 attention and the qkpv emulation."""
    from kernel_agent_b200 import workloads

    q, k, v = workloads.config5(seed=0, device="cuda")
    y = ka.attention_fp8(q, k, v, is_causal=True, enable_gqa=True)
    assert torch.isfinite(y.float()).all()
    for b, h in ((0, 0), (3, 31), (1, 13)):
        hk = h // 4
        qh, kh, vh = (t.float().cpu().numpy() for t in (q[b, h], k[b, hk], v[b, hk]))
        got = y[b, h].float().cpu().numpy()
        emu = ofp8.attention_fp8_head(qh, kh, vh, causal=True)
        ref = ofp8.sdpa_fp32(qh[None, None], kh[None, None], vh[None, None], causal=True)[0, 0]
        rel, cos = rel_cos(got, ref)
        rel_emu, _ = rel_cos(emu, ref)
        assert rel < max(0.05, 1.25 * rel_emu) and cos > 0.998, ((b, h), rel, rel_emu, cos)


@pytest.mark.parametrize("b,hq,hkv,s,d", [(1, 2, 2, 100, 128), (2, 4, 2, 300, 128), (1, 2, 1, 17, 128),
                                          (1, 1, 1, 129, 128), (1, 2, 2, 256, 64), (2, 4, 2, 300, 64),
                                          (1, 3, 1, 70, 64)])
@pytest.mark.parametrize("causal", [True, False])
def test_attention_ragged_sequences(ka, b, hq, hkv, s, d, causal):
    """Sequences that are not a multiple of the 128-row tile, and head_dim 64: the keys past S
    in the last tile are masked and its rows past S are not stored (they would land on the
    next head's first rows); every head against the qkpv emulation and fp32 attention."""
    g = torch.Generator().manual_seed(b * 1000 + s + d)
    q, k, v = (torch.randn(b, h, s, d, generator=g).to(torch.bfloat16) for h in (hq, hkv, hkv))
    y = ka.attention_fp8(q.to(DEV), k.to(DEV), v.to(DEV), is_causal=causal, enable_gqa=hq != hkv)
    assert y.shape == q.shape
    got_all = y.float().cpu().numpy()
    for bi in range(b):
        for h in range(hq):
            hk = h // (hq // hkv)
            qh, kh, vh = (t.float().numpy() for t in (q[bi, h], k[bi, hk], v[bi, hk]))
            emu = ofp8.attention_fp8_head(qh, kh, vh, causal=causal)
            ref = ofp8.sdpa_fp32(qh[None, None], kh[None, None], vh[None, None], causal=causal)[0, 0]
            got = got_all[bi, h]
            rel, cos = rel_cos(got, ref)
            rel_emu, _ = rel_cos(emu, ref)
            assert rel < max(0.05, 1.25 * rel_emu) and cos > 0.998, ((bi, h), rel, rel_emu, cos)


def test_attention_rejects_bad_shapes(ka):
    q = torch.zeros(1, 2, 128, 96, device=DEV, dtype=torch.bfloat16)
    with pytest.raises(ValueError, match="head_dim"):
        ka.attention_fp8(q, q, q)
    q = torch.zeros(1, 4, 128, 128, device=DEV, dtype=torch.bfloat16)
    kv = torch.zeros(1, 2, 128, 128, device=DEV, dtype=torch.bfloat16)
    with pytest.raises(ValueError, match="enable_gqa"):
        ka.attention_fp8(q, kv, kv)
    with pytest.raises(NotImplementedError):
        ka.emulated_sdpa(q, q, q, mode="qk")


def test_attention_status_clean():
    from kernel_agent_b200 import _native

    assert _native.device_status() == 0

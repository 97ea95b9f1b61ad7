"""FP8 KV cache on the GPU (kv_quant.py, triton_fp8_kv_decode.py): the quantiser and the
cache's append bit for bit against the oracle and the reference's golden vectors; the tcgen05
decode attention against the oracle's float64 attention over the same codes, on the
reference test's shapes (tests/test_fp8_toolkit.py:496-514: batch 4, 16 / 2 heads, 4096
tokens, head_dim 128; batch 3, 8 / 8 heads, 77 tokens, head_dim 64, lengths 77 / 1 / 40; splits
0, 1, 3) and on grouped-query, multi-query, strided and ragged cases.

The reference test bounds the relative L2 error by 1e-2; the kernel's error is the bf16
rounding of its output plus the two-term e4m3 rounding of P (about as fine as the reference
kernel's bf16 P), so the bound here is 4e-3.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from conftest import GOLDEN
from helpers import np_bytes, np_values
from oracle import kv_quant as okv

pytestmark = pytest.mark.gpu
DEV = "cuda"
TOL = 4e-3


@pytest.fixture(scope="module")
def kv():
    from kernel_agent_b200.kernels import kv_quant

    return kv_quant


@pytest.fixture(scope="module")
def kvg():
    with np.load(GOLDEN / "kv_golden.npz") as z:
        return {k: z[k] for k in z.files}


def rel(got, want) -> float:
    a, b = np.asarray(got, np.float64).ravel(), np.asarray(want, np.float64).ravel()
    return float(np.linalg.norm(a - b) / np.linalg.norm(b))


def same_codes(got: np.ndarray, want: np.ndarray) -> bool:
    """e4m3 bytes equal, NaN codes compared as NaN: for an invalid quotient (inf / inf, 0 / 0)
    the reference's CPU run stores x86's default NaN (sign set, 0xFF) where CUDA, and the
    reference on a GPU, store the canonical 0x7F; both are NaN in e4m3fn."""
    nan = ((got & 0x7F) == 0x7F) & ((want & 0x7F) == 0x7F)
    return bool(np.all((got == want) | nan))


def status_clean():
    from kernel_agent_b200 import _native as nat

    assert nat.device_status() == 0


# ------------------------------------------------------------------ quantiser and cache


@pytest.mark.parametrize("case,dtype", [("q_bf16", torch.bfloat16), ("q_f32", torch.float32),
                                        ("q_f16", torch.float16)])
def test_quantize_golden(kv, kvg, case, dtype):
    raw = kvg[f"{case}_x"]
    x = torch.from_numpy(raw.view(np.int16)).view(dtype) if dtype != torch.float32 else torch.from_numpy(raw)
    codes, scales = kv.quantize_fp8_kv(x.to(DEV))
    assert np.array_equal(scales.cpu().numpy().view(np.uint32), kvg[f"{case}_scales"].view(np.uint32))
    assert same_codes(np_bytes(codes), kvg[f"{case}_codes"])
    status_clean()


@pytest.mark.parametrize("d", [16, 32, 64, 128, 256])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_quantize_shapes(kv, d, dtype):
    g = torch.Generator().manual_seed(d)
    x = (torch.randn(3, 5, 33, d, generator=g) * torch.logspace(-4, 4, 33)[:, None]).to(dtype)
    x[1, 2, 7] = 0.0
    codes, scales = kv.quantize_fp8_kv(x.to(DEV))
    rc, rs = okv.quantize_fp8_kv(np_values(x))
    assert np.array_equal(scales.cpu().numpy(), rs)
    assert np.array_equal(np_bytes(codes), rc)


def test_cache_append_equals_whole(kv):
    g = torch.Generator().manual_seed(3)
    k = torch.randn(2, 3, 176, 128, generator=g).to(torch.bfloat16).to(DEV)
    v = torch.randn(2, 3, 176, 128, generator=g).to(torch.bfloat16).to(DEV)
    cache = kv.Fp8KVCache(2, 3, 200, 128, device=DEV)
    cache.append(k[:, :, :130], v[:, :, :130])
    for t in range(130, 136):  # decode: one token per step
        cache.append(k[:, :, t:t + 1], v[:, :, t:t + 1])
    kc, ks, vc, vs = cache.append(k[:, :, 136:], v[:, :, 136:])
    assert cache.length == 176 and kc.shape == (2, 3, 176, 128) and vs.shape == (2, 3, 176)
    rk, rks = okv.quantize_fp8_kv(np_values(k))
    rv, rvs = okv.quantize_fp8_kv(np_values(v))
    assert np.array_equal(np_bytes(kc), rk) and np.array_equal(ks.cpu().numpy(), rks)
    assert np.array_equal(np_bytes(vc), rv) and np.array_equal(vs.cpu().numpy(), rvs)
    assert not np_bytes(cache.k[:, :, 176:]).any()  # slots past the length untouched
    with pytest.raises(ValueError, match="cache full"):
        cache.append(k[:, :, :30], v[:, :, :30])


# ------------------------------------------------------------------ decode attention


def _case(b, hq, hkv, length, d, seed, dtype=torch.bfloat16):
    g = torch.Generator().manual_seed(seed)
    q = torch.randn(b, hq, 1, d, generator=g).to(dtype)
    k = torch.randn(b, hkv, length, d, generator=g).to(torch.bfloat16)
    v = torch.randn(b, hkv, length, d, generator=g).to(torch.bfloat16)
    return q, k, v


def _oracle(q, kc, ks, vc, vs, scale=None, lengths=None):
    return okv.fp8_kv_attention(np_values(q), np_bytes(kc), ks.cpu().numpy(), np_bytes(vc), vs.cpu().numpy(),
                                scale=scale, lengths=None if lengths is None else lengths.cpu().numpy())


@pytest.mark.parametrize("shape", [(4, 16, 2, 4096, 128, None), (3, 8, 8, 77, 64, [77, 1, 40])])
@pytest.mark.parametrize("splits", [0, 1, 3])
def test_decode_reference_shapes(kv, shape, splits):
    b, hq, hkv, length, d, lengths = shape
    q, k, v = _case(b, hq, hkv, length, d, seed=length + splits)
    kc, ks = kv.quantize_kv(k.to(DEV))
    vc, vs = kv.quantize_kv(v.to(DEV))
    lens = torch.tensor(lengths, device=DEV) if lengths else None
    out = kv.fp8_kv_decode(q.to(DEV), kc, ks, vc, vs, lengths=lens, splits=splits)
    assert out.shape == q.shape and out.dtype == torch.bfloat16
    want = _oracle(q, kc, ks, vc, vs, lengths=lens)
    r = rel(np_values(out), want)
    assert np.isfinite(r) and r < TOL, (splits, r)
    status_clean()


@pytest.mark.parametrize("hq,hkv", [(1, 1), (4, 1), (10, 2), (12, 1), (16, 1), (32, 1), (24, 3)])
@pytest.mark.parametrize("d", [64, 128])
def test_decode_groups_and_lengths(kv, hq, hkv, d):
    b, length = 3, 700
    q, k, v = _case(b, hq, hkv, length, d, seed=hq * 7 + d)
    kc, ks = kv.quantize_kv(k.to(DEV))
    vc, vs = kv.quantize_kv(v.to(DEV))
    lens = torch.tensor([700, 129, 3], device=DEV)
    for splits in (0, 2, 9):
        out = kv.fp8_kv_decode(q.to(DEV), kc, ks, vc, vs, scale=0.07, lengths=lens, splits=splits)
        r = rel(np_values(out), _oracle(q, kc, ks, vc, vs, scale=0.07, lengths=lens))
        assert r < TOL, (splits, r)
    status_clean()


@pytest.mark.parametrize("dtype", [torch.float16, torch.float32])
def test_decode_query_dtypes(kv, dtype):
    q, k, v = _case(2, 8, 2, 300, 128, seed=11, dtype=dtype)
    kc, ks = kv.quantize_kv(k.to(DEV))
    vc, vs = kv.quantize_kv(v.to(DEV))
    out = kv.fp8_kv_decode(q.to(DEV), kc, ks, vc, vs)
    assert rel(np_values(out), _oracle(q, kc, ks, vc, vs)) < TOL


def test_decode_scaled_queries(kv):
    """Query rows of very different magnitudes: each row's two e4m3 terms get their own
    power-of-two scale."""
    q, k, v = _case(2, 8, 2, 256, 128, seed=12)
    q = q * torch.logspace(-6, 3, 8)[None, :, None, None].to(q.dtype)
    kc, ks = kv.quantize_kv(k.to(DEV))
    vc, vs = kv.quantize_kv(v.to(DEV))
    out = kv.fp8_kv_decode(q.to(DEV), kc, ks, vc, vs)
    want = _oracle(q, kc, ks, vc, vs)
    for h in range(8):  # every head on its own (their softmaxes differ in sharpness)
        assert rel(np_values(out)[:, h], want[:, h]) < TOL, h


def test_several_queries_golden(kv, kvg):
    """fp8_kv_attention with three query tokens per sequence against the reference's output."""
    g = kvg
    q = torch.from_numpy(g["att2_q"].view(np.int16)).view(torch.bfloat16).to(DEV)
    kc = torch.from_numpy(g["att2_kc"]).view(torch.float8_e4m3fn).to(DEV)
    vc = torch.from_numpy(g["att2_vc"]).view(torch.float8_e4m3fn).to(DEV)
    ks, vs = torch.from_numpy(g["att2_ks"]).to(DEV), torch.from_numpy(g["att2_vs"]).to(DEV)
    out = kv.fp8_kv_attention(q, kc, ks, vc, vs)
    ref = np_values(torch.from_numpy(g["att2_out"].view(np.int16)).view(torch.bfloat16))
    assert out.shape == q.shape and rel(np_values(out), ref) < TOL
    # the small golden case: 40 tokens, lengths and scale 0.1, fp32 q
    q1 = torch.from_numpy(g["att_q"]).to(DEV)
    args = [torch.from_numpy(g[n]).to(DEV) for n in ("att_kc", "att_ks", "att_vc", "att_vs")]
    args[0], args[2] = args[0].view(torch.float8_e4m3fn), args[2].view(torch.float8_e4m3fn)
    lens = torch.from_numpy(g["att_lengths"]).to(DEV)
    out1 = kv.fp8_kv_attention(q1, *args, scale=0.1, lengths=lens)
    assert out1.dtype == torch.float32 and rel(out1.cpu().numpy(), g["att_masked"]) < TOL


def test_decode_ignores_tokens_past_lengths(kv):
    """Codes past a sequence's length (NaN codes here) do not reach its output: the result is
    bit-identical to the one over zeroed codes."""
    q, k, v = _case(3, 8, 2, 400, 128, seed=13)
    kc, ks = kv.quantize_kv(k.to(DEV))
    vc, vs = kv.quantize_kv(v.to(DEV))
    lens = torch.tensor([400, 200, 77], device=DEV)
    clean_k, clean_v = kc.clone(), vc.clone()
    for i, n in enumerate(lens.tolist()):
        clean_k[i, :, n:] = 0
        clean_v[i, :, n:] = 0
        kc.view(torch.uint8)[i, :, n:] = 0x7F
        vc.view(torch.uint8)[i, :, n:] = 0x7F
    for splits in (0, 1, 3):
        dirty = kv.fp8_kv_decode(q.to(DEV), kc, ks, vc, vs, lengths=lens, splits=splits)
        clean = kv.fp8_kv_decode(q.to(DEV), clean_k, ks, clean_v, vs, lengths=lens, splits=splits)
        assert torch.isfinite(dirty.float()).all() and torch.equal(dirty, clean), splits


def test_decode_cache_views_and_determinism(kv):
    """The cache's strided views (max_tokens > length) give the same bits as contiguous
    copies, and two runs give the same bits."""
    g = torch.Generator().manual_seed(14)
    k = torch.randn(2, 2, 333, 128, generator=g).to(torch.bfloat16).to(DEV)
    v = torch.randn(2, 2, 333, 128, generator=g).to(torch.bfloat16).to(DEV)
    q = torch.randn(2, 16, 128, generator=g).to(torch.bfloat16).to(DEV)
    cache = kv.Fp8KVCache(2, 2, 1024, 128, device=DEV)
    kc, ks, vc, vs = cache.append(k, v)
    a = kv.fp8_kv_decode(q, kc, ks, vc, vs)
    b = kv.fp8_kv_decode(q, kc.contiguous(), ks.contiguous(), vc.contiguous(), vs.contiguous())
    c = kv.fp8_kv_decode(q, kc, ks, vc, vs)
    assert a.shape == q.shape and torch.equal(a, b) and torch.equal(a, c)
    assert rel(np_values(a), _oracle(q[:, :, None], kc, ks, vc, vs)[:, :, 0]) < TOL
    status_clean()


def test_decode_split_edges(kv):
    """More splits than tiles (clamped) and splits past a short sequence's end (empty)."""
    q, k, v = _case(2, 4, 1, 300, 128, seed=15)
    kc, ks = kv.quantize_kv(k.to(DEV))
    vc, vs = kv.quantize_kv(v.to(DEV))
    lens = torch.tensor([1, 300], device=DEV)
    want = _oracle(q, kc, ks, vc, vs, lengths=lens)
    for splits in (1, 3, 64):
        out = kv.fp8_kv_decode(q.to(DEV), kc, ks, vc, vs, lengths=lens, splits=splits)
        assert rel(np_values(out), want) < TOL, splits
    status_clean()


@pytest.mark.parametrize("splits", [4, 16, 32])
def test_decode_split_merges(kv, splits):
    """The splits' merge both ways: up to 16 splits of a (sequence, KV head) form one
    thread-block cluster and merge through distributed shared memory; 32 go through the global
    workspace and the last CTA. Each run twice (the workspace's counters return to zero)."""
    q, k, v = _case(2, 8, 2, 4096, 128, seed=17)
    kc, ks = kv.quantize_kv(k.to(DEV))
    vc, vs = kv.quantize_kv(v.to(DEV))
    lens = torch.tensor([4096, 1500], device=DEV)
    want = _oracle(q, kc, ks, vc, vs, lengths=lens)
    a = kv.fp8_kv_decode(q.to(DEV), kc, ks, vc, vs, lengths=lens, splits=splits)
    b = kv.fp8_kv_decode(q.to(DEV), kc, ks, vc, vs, lengths=lens, splits=splits)
    assert rel(np_values(a), want) < TOL and torch.equal(a, b)
    status_clean()


def test_module_against_sdpa(kv):
    """Fp8KVDecodeAttention (quantising K and V per call) against SDPA on the unquantised
    K / V: the quantisation error the reference test allows (kv_quant's < 0.04)."""
    q, k, v = _case(2, 16, 2, 512, 128, seed=16)
    q, k, v = q.to(DEV), k.to(DEV), v.to(DEV)

    class Ref(torch.nn.Module):
        def forward(self, q, k, v):
            return torch.nn.functional.scaled_dot_product_attention(q, k, v, enable_gqa=True)

    mod = kv.build(Ref())
    out = mod(q, k, v)
    ref = Ref()(q.float(), k.float(), v.float())
    assert out.shape == q.shape and rel(np_values(out), np_values(ref)) < 0.04
    with pytest.raises(NotImplementedError):
        mod(q[..., :96], k[..., :96], v[..., :96])


def test_error_report_golden(kv, kvg):
    """fp8_kv_error (one GPU pass of row sums per tensor) against the reference's report."""
    import json

    want = json.loads((GOLDEN / "kv_golden.json").read_text())["error"]
    k = torch.from_numpy(kvg["err_k"].view(np.int16)).view(torch.bfloat16).to(DEV)
    got = kv.fp8_kv_error(k, k * 0.5)
    assert got["bytes"] == want["bytes"] and got["format"] == want["format"]
    for key in ("k_rel_l2", "k_worst_row_rel_l2", "v_rel_l2", "v_worst_row_rel_l2"):
        assert got[key] == pytest.approx(want[key], abs=2e-5), key

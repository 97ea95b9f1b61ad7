"""Generate the golden vectors that pin the FP8 KV-cache oracle (``oracle/kv_quant.py``).

Run in a container where the reference sources are present (they are not on the GPU box):

    python tests/golden/make_golden_kv.py /path/to/kernel-agent/src

It imports the reference's own ``kernel_agent.kernels.kv_quant``, runs it on seeded inputs
and writes ``kv_golden.npz`` (inputs and outputs as raw arrays: bf16 as uint16 bits, e4m3 as
uint8 bytes) and ``kv_golden.json`` (``fp8_kv_error`` and ``kv_cache_share`` results). The
fixtures are committed; the tests only read them.
"""

from __future__ import annotations

import json
import sys
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent


def bits(t: torch.Tensor) -> np.ndarray:
    t = t.detach().contiguous().cpu()
    if t.dtype in (torch.bfloat16, torch.float16):
        return t.view(torch.int16).numpy().view(np.uint16)
    if t.dtype == torch.float8_e4m3fn:
        return t.view(torch.uint8).numpy()
    return t.numpy()


def main(src: str) -> None:
    sys.path.insert(0, src)
    from kernel_agent.kernels import kv_quant  # noqa: E402  (the reference)

    out: dict[str, np.ndarray] = {}
    meta: dict[str, object] = {}
    bf = torch.bfloat16

    # ---------------------------------------------------------------- quantiser (bf16, D 64)
    g = torch.Generator().manual_seed(10)
    k = (torch.randn(2, 3, 17, 64, generator=g) * torch.logspace(-2, 2, 17)[:, None]).to(bf)
    k[0, 1, 5] = 0  # a token of zeros: scale 1
    k[1, 2, 3, 7] = 50.0  # an outlier: only its own row's scale moves
    k[1, 0, 2, 3] = float("nan")  # NaN: amax NaN -> scale 1, the rest saturates
    k[1, 1, 4, 9] = float("inf")  # inf: scale inf -> codes 0 and NaN
    k[0, 2, 9] = k[0, 2, 9] * 1e-30  # tiny values
    c, s = kv_quant.quantize_fp8_kv(k)
    out.update(q_bf16_x=bits(k), q_bf16_codes=bits(c), q_bf16_scales=s.numpy())

    # ---------------------------------------------------------------- quantiser (f32, D 128 / 16)
    x = torch.randn(3, 5, 128, generator=g) * 3.0
    x[0, 1] = 1e-44  # amax / 448 underflows to 0: the reference keeps the zero scale
    x[0, 1, 5] = 0.0
    x[2, 2] = 0.0
    c, s = kv_quant.quantize_fp8_kv(x)
    out.update(q_f32_x=x.numpy(), q_f32_codes=bits(c), q_f32_scales=s.numpy())
    y = (torch.randn(4, 7, 16, generator=g) * 0.01).to(torch.float16)
    c, s = kv_quant.quantize_fp8_kv(y)
    out.update(q_f16_x=bits(y), q_f16_codes=bits(c), q_f16_scales=s.numpy())

    # ---------------------------------------------------------------- attention
    q = torch.randn(3, 8, 1, 64, generator=g)
    kk = torch.randn(3, 2, 40, 64, generator=g)
    vv = torch.randn(3, 2, 40, 64, generator=g)
    kc, ks = kv_quant.quantize_fp8_kv(kk)
    vc, vs = kv_quant.quantize_fp8_kv(vv)
    plain = kv_quant.fp8_kv_attention(q, kc, ks, vc, vs)
    lengths = torch.tensor([40, 1, 17])
    masked = kv_quant.fp8_kv_attention(q, kc, ks, vc, vs, scale=0.1, lengths=lengths)
    out.update(att_q=q.numpy(), att_kc=bits(kc), att_ks=ks.numpy(), att_vc=bits(vc), att_vs=vs.numpy(),
               att_out=plain.numpy(), att_lengths=lengths.numpy(), att_masked=masked.numpy())
    # several query tokens per sequence, bf16 q, D 128
    q2 = torch.randn(2, 4, 3, 128, generator=g).to(bf)
    k2 = torch.randn(2, 2, 150, 128, generator=g).to(bf)
    v2 = torch.randn(2, 2, 150, 128, generator=g).to(bf)
    kc2, ks2 = kv_quant.quantize_fp8_kv(k2)
    vc2, vs2 = kv_quant.quantize_fp8_kv(v2)
    o2 = kv_quant.fp8_kv_attention(q2, kc2, ks2, vc2, vs2)
    out.update(att2_q=bits(q2), att2_kc=bits(kc2), att2_ks=ks2.numpy(), att2_vc=bits(vc2),
               att2_vs=vs2.numpy(), att2_out=bits(o2))

    # ---------------------------------------------------------------- reports
    clean = torch.randn(2, 3, 17, 64, generator=g).to(bf)
    meta["error"] = kv_quant.fp8_kv_error(clean, clean * 0.5)
    out["err_k"] = bits(clean)
    meta["share"] = kv_quant.kv_cache_share(
        batch=8, tokens=8192, layers=28, kv_heads=8, head_dim=128, other_bytes=16e9
    )
    meta["share_small"] = kv_quant.kv_cache_share(
        batch=1, tokens=77, layers=2, kv_heads=2, head_dim=64, other_bytes=0.0, elem_bytes=4.0
    )

    np.savez_compressed(HERE / "kv_golden.npz", **out)
    (HERE / "kv_golden.json").write_text(json.dumps(meta, indent=1, sort_keys=True) + "\n")
    print(f"wrote {len(out)} arrays, {len(meta)} reports")


if __name__ == "__main__":
    if len(sys.argv) != 2:
        sys.exit(f"usage: python {sys.argv[0]} <path to the reference's src directory>")
    main(sys.argv[1])

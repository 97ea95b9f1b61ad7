"""Generate the golden vectors that pin the CPU oracle (``oracle/``) to the reference.

Run in a container where the reference sources are present (they are not on the GPU box):

    python tests/golden/make_golden.py /path/to/kernel-agent/src

It imports the reference's own ``kernel_agent.kernels.quant`` / ``compare`` and
``docs/research-scripts/fp8-sm120/fp8lib.py``, runs them on seeded inputs and writes
``golden.npz`` (inputs and outputs as raw arrays: bf16 as uint16 bits, fp8 / e8m0 as uint8
bytes) and ``golden.json`` (the comparator's and the scale checks' result dicts). The
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
    """Raw bits of a tensor as a numpy array (bf16/f16 -> uint16, fp8/e8m0 -> uint8)."""
    t = t.detach().contiguous().cpu()
    if t.dtype in (torch.bfloat16, torch.float16):
        return t.view(torch.int16).numpy().view(np.uint16)
    if t.dtype in (torch.float8_e4m3fn, torch.float8_e8m0fnu, torch.float8_e5m2):
        return t.view(torch.uint8).numpy()
    return t.numpy()


def main(src: str) -> None:
    sys.path.insert(0, src)
    from kernel_agent.kernels import compare, quant  # noqa: E402  (the reference)

    research = Path(src).parent / "docs" / "research-scripts" / "fp8-sm120"
    sys.path.insert(0, str(research))
    import fp8lib  # noqa: E402  (the reference's research math)

    out: dict[str, np.ndarray] = {}
    meta: dict[str, object] = {}
    bf = torch.bfloat16

    # ---------------------------------------------------------------- INT8
    g = torch.Generator().manual_seed(0)
    x = (torch.randn(64, 256, generator=g) * torch.logspace(-3, 3, 64)[:, None]).to(bf)
    x[1] = 0  # a zero row
    x[2, 7] = 300.0  # an outlier row
    x[3, :4] = torch.tensor([127.0, 2.5, 3.5, -2.5])  # ties: 2.5 and 3.5 steps
    x[3, 4:] = 0
    q, s = quant.quantize_int8_activations(x)
    out.update(int8_x=bits(x), int8_xq=q.numpy(), int8_xs=s.numpy())
    w = (torch.randn(48, 256, generator=g) * 0.05).to(bf)
    w[5] = 0
    w[6, 3] = 4.0
    wq, ws = quant.quantize_int8(w)
    bias = (torch.randn(48, generator=g) * 0.1).to(bf)
    y = quant.int8_w8a8_linear(x, wq, ws, bias)
    out.update(int8_w=bits(w), int8_wq=wq.numpy(), int8_ws=ws.numpy(), int8_bias=bits(bias),
               int8_y=bits(y))
    sm = torch.rand(256, generator=g) + 0.5
    qs, ss = quant.quantize_int8_activations(x, sm)
    out.update(int8_smooth=sm.numpy(), int8_xq_smooth=qs.numpy(), int8_xs_smooth=ss.numpy())

    # ---------------------------------------------------------------- FP8 per token / channel
    xf = (torch.randn(40, 320, generator=g) * torch.logspace(-4, 4, 40)[:, None]).to(bf)
    xf[0] = 0
    xf[5, 9] = -5000.0
    fq, fs = quant.quantize_fp8_activations(xf)
    wf = (torch.randn(24, 320, generator=g) * 0.02).to(bf)
    wfq, wfs = quant.quantize_fp8(wf)
    fb = (torch.randn(24, generator=g) * 0.1).to(bf)
    fy = quant.fp8_w8a8_linear(xf[1:], wfq, wfs, fb)
    out.update(fp8_x=bits(xf), fp8_xq=bits(fq), fp8_xs=fs.numpy(), fp8_w=bits(wf),
               fp8_wq=bits(wfq), fp8_ws=wfs.numpy(), fp8_bias=bits(fb), fp8_y=bits(fy))

    # ---------------------------------------------------------------- MXFP8
    amax = torch.cat([
        torch.tensor([0.0, 1e-40, 1.0, 224.0, 448.0, 449.0, 15.2, 3.0e38, 1e-45, 6e-43, 7e-43]),
        torch.rand(20000, generator=g) * torch.logspace(-40, 38, 20000),
        448.0 * torch.pow(2.0, torch.arange(-120, 110).float()),
        torch.nextafter(448.0 * torch.pow(2.0, torch.arange(-120, 110).float()), torch.tensor(1e38)),
    ])
    out.update(mx_amax=amax.numpy(), mx_e_ceil=quant.mx_scale_exponents(amax, "ceil").numpy(),
               mx_e_floor=quant.mx_scale_exponents(amax, "floor").numpy())
    xm = (torch.randn(48, 256, generator=g) * torch.logspace(-30, 30, 48)[:, None]).to(bf)
    xm[0, :32] = 0
    xm[1, 5] = 3000.0
    xm[2, 32:64] = 1e-39  # a subnormal block maximum
    mq, ms = quant.quantize_mxfp8(xm)
    out.update(mx_x=bits(xm), mx_q=bits(mq), mx_s=bits(ms))
    mqf, msf = quant.quantize_mxfp8(xm, "floor")
    out.update(mx_q_floor=bits(mqf), mx_s_floor=bits(msf))
    for rows, cols in ((352, 32), (22, 8), (200, 12), (128, 4)):
        sc = torch.randint(1, 255, (rows, cols), generator=g, dtype=torch.uint8)
        out[f"swz_in_{rows}_{cols}"] = sc.numpy()
        out[f"swz_out_{rows}_{cols}"] = bits(quant.swizzle_mx_scales(sc.view(torch.float8_e8m0fnu)))
    wm = (torch.randn(64, 256, generator=g) * 256**-0.5).to(bf)
    wmq, wms = quant.quantize_mxfp8(wm)
    mb = torch.randn(64, generator=g).to(bf)
    xl = torch.randn(44, 256, generator=g).to(bf)
    my = quant.mxfp8_linear(xl, wmq, wms, mb)
    out.update(mxl_x=bits(xl), mxl_w=bits(wm), mxl_wq=bits(wmq), mxl_ws=bits(wms),
               mxl_bias=bits(mb), mxl_y=bits(my))
    # SiLU * up in bf16 (eager), then MXFP8: the fused producer's math
    gt = (torch.randn(32, 256, generator=g) * 3).to(bf)
    up = torch.randn(32, 256, generator=g).to(bf)
    h = torch.nn.functional.silu(gt) * up
    hq, hs = quant.quantize_mxfp8(h)
    out.update(silu_g=bits(gt), silu_u=bits(up), silu_h=bits(h), silu_hq=bits(hq), silu_hs=bits(hs))

    # ---------------------------------------------------------------- NVFP4 / MXFP4
    ga = torch.Generator().manual_seed(7)
    xa = torch.randn(256, 64, generator=ga) * torch.logspace(-4, 4, 256)[:, None]
    xa[1] = torch.randn(64, generator=ga) * 4e-3
    xa[1, 5] = 1e3
    xa[1, 48:64] = torch.randn(16, generator=ga) * 1e-5
    xa[2, 16:32] = 0
    xa[3] = 0
    xa = xa.to(bf)
    out["fp4_x"] = bits(xa)
    for gran in ("token", "tensor"):
        c, sc, o = quant.quantize_fp4_activations(xa, "nvfp4", gran)
        out.update({f"nvfp4_{gran}_q": c.numpy(), f"nvfp4_{gran}_s": bits(sc),
                    f"nvfp4_{gran}_o": o.numpy()})
    xa2 = xa[:64].reshape(64, 64).repeat(1, 2)
    c, sc, o = quant.quantize_fp4_activations(xa2, "mxfp4")
    out.update(mxfp4_x=bits(xa2), mxfp4_q=c.numpy(), mxfp4_s=bits(sc))
    for fmt in ("nvfp4", "mxfp4"):
        c, sc, ts = quant.quantize_fp4(xa2, fmt)
        out.update({f"w{fmt}_q": c.numpy(), f"w{fmt}_s": bits(sc), f"w{fmt}_ts": ts.numpy()})
    gl = torch.Generator().manual_seed(0)
    w4 = (torch.randn(128, 256, generator=gl) * 256**-0.5).to(bf)
    x4 = torch.randn(48, 256, generator=gl).to(bf)
    b4 = torch.randn(128, generator=gl).to(bf)
    c4, s4, t4 = quant.quantize_fp4(w4)
    y4 = quant.fp4_w4a4_linear(x4, c4, s4, t4, b4)
    out.update(w4a4_x=bits(x4), w4a4_w=bits(w4), w4a4_bias=bits(b4), w4a4_q=c4.numpy(),
               w4a4_s=bits(s4), w4a4_ts=t4.numpy(), w4a4_y=bits(y4))
    # rotation and the opt-in bias correction (W4A4 options of fp4_w4a4_linear / quantize_fp4)
    gr = torch.Generator().manual_seed(11)
    xr = torch.randn(24, 256, generator=gr).to(bf)
    xr[3, 17] = 40.0
    wr = (torch.randn(160, 256, generator=gr) * 0.02).to(bf)
    br = (torch.randn(160, generator=gr) * 0.05).to(bf)
    out.update(rot_x=bits(xr), rot_w=bits(wr), rot_b=bits(br),
               rot_x16=quant.hadamard_rotate(xr, 16).numpy(), rot_x128=quant.hadamard_rotate(xr, 128).numpy())
    for fmt in ("nvfp4", "mxfp4"):
        cx, sx, ox = quant.quantize_fp4_activations(xr, fmt)
        out[f"bc_{fmt}_x"] = quant.fp4_bias_correction(xr, cx, sx, ox).numpy()
        cu, su, tu = quant.quantize_fp4(wr, fmt, unbiased=True)
        out.update({f"ub_{fmt}_q": cu.numpy(), f"ub_{fmt}_s": bits(su), f"ub_{fmt}_ts": tu.numpy()})
        out[f"ub_{fmt}_y"] = bits(quant.fp4_w4a4_linear(xr, cu, su, tu, br, fmt=fmt, unbiased=True))
        wrot = quant.hadamard_rotate(wr, 16).to(bf)
        cr, sr, tr = quant.quantize_fp4(wrot, fmt)
        out.update({f"rot_{fmt}_wq": cr.numpy(), f"rot_{fmt}_ws": bits(sr), f"rot_{fmt}_ts": tr.numpy()})
        out[f"rot_{fmt}_y"] = bits(quant.fp4_w4a4_linear(xr, cr, sr, tr, br, fmt=fmt, rotate=16))

    # e2m1 ties: the hardware's directions
    ties = torch.tensor([0.25, 0.75, 1.25, 1.75, 2.5, 3.5, 5.0, -0.25, -5.0])
    out.update(e2m1_ties=ties.numpy(), e2m1_ties_codes=quant._round_e2m1(ties).numpy())

    # ---------------------------------------------------------------- blockwise FP8 (research math)
    gb = torch.Generator().manual_seed(3)
    xb = torch.randn(24, 512, generator=gb).to(bf)
    xb[2, 128:256] = 0
    wb = (torch.randn(256, 512, generator=gb) * 0.02).to(bf)
    out.update(bw_x=bits(xb), bw_w=bits(wb),
               bw_x_fq=fp8lib.fq_groups(xb.float(), 128).numpy(),
               bw_w_fq=fp8lib.fq_block(wb.float(), 128).numpy())

    # ---------------------------------------------------------------- FP8 attention (qkpv)
    gq = torch.Generator().manual_seed(5)
    qa = torch.randn(1, 4, 64, 64, generator=gq).to(bf)
    ka = torch.randn(1, 2, 64, 64, generator=gq).to(bf)
    va = torch.randn(1, 2, 64, 64, generator=gq).to(bf)
    ya = fp8lib.emulated_sdpa(qa, ka, va, is_causal=True, enable_gqa=True, mode="qkpv")
    out.update(att_q=bits(qa), att_k=bits(ka), att_v=bits(va), att_y=bits(ya))
    # the GPU kernel's shape class (head_dim 128, whole 128-token tiles), causal and not, with
    # the emulation's own fp32 attention for the error ratios
    qb = torch.randn(1, 4, 256, 128, generator=gq).to(bf)
    kb = torch.randn(1, 2, 256, 128, generator=gq).to(bf)
    vb = torch.randn(1, 2, 256, 128, generator=gq).to(bf)
    yb = fp8lib.emulated_sdpa(qb, kb, vb, is_causal=True, enable_gqa=True, mode="qkpv")
    yb_nc = fp8lib.emulated_sdpa(qb, kb, vb, is_causal=False, enable_gqa=True, mode="qkpv")
    yb_ref = fp8lib.emulated_sdpa(qb.float(), kb.float(), vb.float(), is_causal=True, enable_gqa=True, mode="none")
    out.update(att2_q=bits(qb), att2_k=bits(kb), att2_v=bits(vb), att2_y=bits(yb), att2_y_nc=bits(yb_nc),
               att2_y_fp32=yb_ref.numpy())

    # ---------------------------------------------------------------- comparator
    cases = []

    stored: dict[bytes, str] = {}

    def keep(t: torch.Tensor) -> str:
        """Store a tensor once (by content) and return its key."""
        arr = bits(t)
        tag = arr.tobytes() + str(arr.dtype).encode() + str(arr.shape).encode()
        if tag not in stored:
            stored[tag] = f"cmpt{len(stored)}"
            out[stored[tag]] = arr
        return stored[tag]

    def case(name: str, ref: torch.Tensor, new: torch.Tensor, **kw) -> None:
        res = compare.compare_tensors(name, ref, new, **kw)
        rer = kw.pop("rerounded", None)
        cases.append({"ref": keep(ref), "new": keep(new),
                      "rer": None if rer is None else keep(rer),
                      "dtype": str(ref.dtype).removeprefix("torch."), "kw": kw, "result": res})

    gc = torch.Generator().manual_seed(11)
    a = torch.randn(4096, generator=gc).to(bf)
    case("same", a, a.clone())
    b = a.clone()
    b[:5] += 10
    case("five_off", a, b)
    case("noisy", a, (a.float() * (1 + 1e-3)).to(bf))
    one = a.clone()
    one[7] = 1e4
    case("one_outlier", a, one)
    small = (a.float() * 0.1).to(bf)
    case("biased_small", small, small + 0.01)
    nf = a.clone()
    nf[3], nf[9], nf[11] = float("nan"), float("inf"), float("-inf")
    nf2 = nf.clone()
    nf2[20] += 0.5
    case("nonfinite_same_positions", nf, nf2)
    nf3 = nf.clone()
    nf3[3] = 1.0
    case("nan_moved", nf, nf3)
    case("f32", a.float(), a.float() * (1 + 3e-5))
    case("f32_off", a.float(), a.float() + 1e-3)
    case("ints", torch.arange(16), torch.arange(16) + (torch.arange(16) == 3))
    # config 1 of the build (seed 0): W8A8 INT8 output against the fp32 matmul
    gw = torch.Generator().manual_seed(0)
    x1 = torch.randn(128, 1024, generator=gw)
    cols = torch.randperm(1024, generator=gw)[:5]
    x1[:, cols] *= 20
    x1 = x1.to(bf)
    w1 = (torch.randn(1024, 1024, generator=gw) * 0.02).to(bf)
    b1 = (torch.randn(1024, generator=gw) * 0.1).to(bf)
    q1, s1 = quant.quantize_int8(w1)
    y1 = quant.int8_w8a8_linear(x1, q1, s1, b1)
    r1 = (x1.float() @ w1.float().T + b1.float()).to(bf)
    for tier in ("exact", "near-lossless", "relaxed"):
        case(f"config1_{tier}", r1, y1, tier=tier)
    # reduced tiers with and without signal, perturbed bounds, the channel RMS, rerounded
    y2 = (r1.float() * 1.03).to(bf)
    case("config1_norm_off", r1, y2, tier="near-lossless")
    rr = (r1.float() + torch.randn(r1.shape, generator=gw) * 0.003).to(bf)
    case("perturbed_near", r1, y1, tier="near-lossless", perturbed=True)
    case("perturbed_relaxed_fp4a", r1, y1, tier="relaxed-fp4a", perturbed=True)
    case("rerounded_exact", r1, y1, rerounded=rr)
    case("rerounded_small_noise", r1, rr, rerounded=(r1.float() - (rr.float() - r1.float())).to(bf))
    case("input_scale_3", r1, y1, input_scale=3.0)
    case("input_scale_001", (r1.float() * 0.01).to(bf), (y1.float() * 0.01).to(bf), input_scale=0.01)
    tiny = torch.full((4096,), 1e-3, dtype=bf)
    case("no_signal", tiny, tiny * 1.5)
    case("no_signal_perturbed", tiny, tiny * 1.5, tier="near-lossless", perturbed=True)
    meta["compare"] = cases

    # ---------------------------------------------------------------- scale checks
    checks = []
    sx = quant.mxfp8_stress_input((64, 256), seed=3)
    out["stress_mx"] = bits(sx)
    for rule in ("ceil", "floor"):
        _, scl = quant.quantize_mxfp8(sx, rule)
        checks.append({"kind": "mxfp8", "input": "stress_mx", "rule": rule,
                       "result": quant.mxfp8_saturation(sx, scl)})
    sf = quant.fp4_stress_input((64, 256), "nvfp4", seed=4)
    out["stress_fp4"] = bits(sf)
    _, scl, o = quant.quantize_fp4_activations(sf, "nvfp4")
    checks.append({"kind": "fp4", "input": "stress_fp4", "fmt": "nvfp4", "variant": "reference",
                   "result": quant.fp4_scale_check(sf, scl, o)})
    trunc = torch.floor(scl.float() * 8) / 8  # a rule that rounds down (caught)
    out["stress_fp4_trunc_scales"] = bits(trunc.to(torch.float8_e4m3fn))
    checks.append({"kind": "fp4", "input": "stress_fp4", "fmt": "nvfp4", "variant": "trunc",
                   "result": quant.fp4_scale_check(sf, trunc.to(torch.float8_e4m3fn), o)})
    out.update(stress_fp4_s=bits(scl), stress_fp4_o=o.numpy())
    sm4 = quant.fp4_stress_input((64, 256), "mxfp4", seed=5)
    out["stress_mx4"] = bits(sm4)
    _, scl4, o4 = quant.quantize_fp4_activations(sm4, "mxfp4")
    checks.append({"kind": "fp4", "input": "stress_mx4", "fmt": "mxfp4", "variant": "reference",
                   "result": quant.fp4_scale_check(sm4, scl4, o4)})
    meta["checks"] = checks

    np.savez_compressed(HERE / "golden.npz", **out)
    (HERE / "golden.json").write_text(json.dumps(meta, indent=1, default=float) + "\n")
    size = (HERE / "golden.npz").stat().st_size
    print(f"wrote {len(out)} arrays ({size / 1e6:.2f} MB) and {len(cases)} comparator cases")


if __name__ == "__main__":
    if len(sys.argv) != 2:
        sys.exit(f"usage: python {sys.argv[0]} <path to the reference's src directory>")
    main(sys.argv[1])

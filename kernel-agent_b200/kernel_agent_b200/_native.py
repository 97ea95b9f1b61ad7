"""The C ABI of ``libkab.so`` (``include/kab.h``) through ctypes.

The library is loaded on first use; when it is missing (not built) or no sm_100 GPU is
present the call raises, loudly: the package has no CPU fallback. ``call(name, *args)``
runs one entry point and maps a non-zero status to an exception (``KAB_EINVAL`` ->
``ValueError``, anything else -> ``RuntimeError``) carrying ``kab_last_error()``.
"""

from __future__ import annotations

import ctypes
import os
from ctypes import POINTER, c_float, c_int, c_int64, c_size_t, c_uint, c_void_p
from pathlib import Path

import torch

LIB_PATH = Path(os.environ.get("KAB_LIBRARY", Path(__file__).resolve().parent / "_native" / "libkab.so"))

KAB_OK, KAB_EINVAL, KAB_EUNSUPPORTED, KAB_ECUDA, KAB_ETIMEOUT = range(5)
KAB_F32, KAB_BF16, KAB_F16 = 0, 1, 2
KAB_NVFP4, KAB_MXFP4 = 0, 1
KAB_FP4_TOKEN, KAB_FP4_TENSOR, KAB_FP4_WEIGHT = 0, 1, 2
CMP_NCOUNT, CMP_NSUM, CMP_NMAX = 11, 6, 3

DTYPES = {torch.float32: KAB_F32, torch.bfloat16: KAB_BF16, torch.float16: KAB_F16}


class KabCompareResult(ctypes.Structure):
    _fields_ = [
        ("count", ctypes.c_longlong * CMP_NCOUNT),
        ("sum", ctypes.c_double * CMP_NSUM),
        ("max", ctypes.c_float * CMP_NMAX),
        ("pad_", ctypes.c_float),
    ]


class KabScaleCheck(ctypes.Structure):
    _fields_ = [
        ("saturated", ctypes.c_ulonglong),
        ("underflow", ctypes.c_ulonglong),
        ("nonfinite", ctypes.c_ulonglong),
        ("not_representable", ctypes.c_ulonglong),
        ("coarser", ctypes.c_ulonglong),
        ("not_pow2", ctypes.c_ulonglong),
        ("worst_ratio_bits", ctypes.c_uint),
        ("pad_", ctypes.c_uint),
        ("saturated_plain", ctypes.c_ulonglong),
    ]


class KabCompareParams(ctypes.Structure):
    _fields_ = [
        ("ref", c_void_p), ("new_", c_void_p), ("rerounded", c_void_p),
        ("n", c_int64), ("channels", c_int64),
        ("dtype", c_int), ("has_rerounded", c_int), ("vector", c_int), ("alt_bound", c_int),
        ("atol", c_float), ("rtol", c_float), ("alt_atol", c_float), ("alt_rtol", c_float),
        ("widen_mode", c_int), ("widen_scalar", c_float), ("widen_channel", c_void_p),
        ("element_mode", c_int), ("element_first", c_float), ("element_atol", c_float),
        ("element_rtol", c_float), ("element_scale", c_void_p),
    ]


KAB_DIFF_MAXDIM = 8
KAB_DIFF_F64 = 3  # the difference census also reads float64 tensors
KAB_DIFF_BITS = {1: 4, 2: 5, 4: 6, 8: 7}  # ... and compares integer / boolean tensors by their bits


class KabDiffParams(ctypes.Structure):
    _fields_ = [
        ("a", c_void_p), ("b", c_void_p), ("base", c_void_p),
        ("dtype", c_int), ("nan_equal", c_int),
        ("outer", c_int64), ("len", c_int64), ("inner", c_int64),
        ("a_dim", c_int64), ("a_off", c_int64), ("base_dim", c_int64), ("base_off", c_int64),
        ("ndim", c_int), ("shape", c_int64 * KAB_DIFF_MAXDIM),
        ("hits", c_void_p), ("box", c_void_p), ("mask", c_void_p),
    ]


class KabKvDecodeParams(ctypes.Structure):
    _fields_ = [
        ("q", c_void_p), ("q_dtype", c_int), ("q_stride_b", c_int64), ("q_stride_row", c_int64),
        ("k_codes", c_void_p), ("k_scales", c_void_p), ("v_codes", c_void_p), ("v_scales", c_void_p),
        ("kc_stride_b", c_int64), ("kc_stride_h", c_int64), ("kc_stride_l", c_int64),
        ("vc_stride_b", c_int64), ("vc_stride_h", c_int64), ("vc_stride_l", c_int64),
        ("ks_stride_b", c_int64), ("ks_stride_h", c_int64),
        ("vs_stride_b", c_int64), ("vs_stride_h", c_int64),
        ("lengths", c_void_p),
        ("batch", c_int64), ("heads_q", c_int64), ("heads_kv", c_int64), ("q_len", c_int64),
        ("length", c_int64), ("head_dim", c_int64),
        ("sm_scale", c_float), ("splits", c_int), ("out", c_void_p),
    ]


# name -> argument types (the return type is int unless listed in _RESTYPES)
_SIGNATURES: dict[str, list] = {
    "kab_last_error": [],
    "kab_abi_version": [],
    "kab_device_check": [c_int],
    "kab_device_status": [POINTER(c_uint), c_int, c_void_p],
    "kab_quant_rows_int8": [c_void_p, c_int, c_int64, c_int64, c_int64, c_void_p, c_int, c_void_p,
                            c_void_p, c_void_p],
    "kab_quant_rows_fp8": [c_void_p, c_int, c_int64, c_int64, c_int64, c_void_p, c_int64, c_void_p,
                           c_void_p, c_void_p, c_void_p],
    "kab_quant_groups_fp8": [c_void_p, c_int, c_int64, c_int64, c_int64, c_int, c_void_p, c_void_p,
                             c_void_p],
    "kab_quant_blocks_fp8": [c_void_p, c_int, c_int64, c_int64, c_int64, c_void_p, c_void_p, c_void_p],
    "kab_quant_mxfp8": [c_void_p, c_int, c_int64, c_int64, c_int64, c_void_p, c_int64, c_int, c_void_p,
                        c_void_p, c_int, c_void_p, c_void_p],
    "kab_quant_fp4": [c_void_p, c_int, c_int64, c_int64, c_int64, c_void_p, c_int64, c_int, c_int,
                      c_void_p, c_void_p, c_void_p, c_void_p, c_int, c_void_p, c_void_p, c_void_p],
    "kab_amax": [c_void_p, c_int, c_int64, c_int64, c_int64, c_void_p, c_void_p],
    "kab_fp4_tensor_scale": [c_void_p, c_void_p, c_void_p],
    "kab_mx_exponents": [c_void_p, c_int64, c_int, c_void_p, c_void_p],
    "kab_swizzle_scales": [c_void_p, c_int64, c_int64, c_void_p, c_void_p],
    "kab_fp4_values": [c_void_p, c_void_p, c_int64, c_int64, c_int, c_void_p, c_void_p],
    "kab_gemm_i8": [c_void_p, c_void_p, c_int64, c_int64, c_int64, c_void_p, c_void_p, c_void_p, c_int,
                    c_void_p, c_int, c_int64, c_void_p, c_void_p],
    "kab_gemm_f8": [c_void_p, c_void_p, c_int64, c_int64, c_int64, c_void_p, c_void_p, c_void_p, c_int,
                    c_void_p, c_int, c_int64, c_void_p],
    "kab_gemm_mxf8": [c_void_p, c_void_p, c_void_p, c_void_p, c_int64, c_int64, c_int64, c_void_p, c_int,
                      c_void_p, c_int, c_int64, c_void_p],
    "kab_gemm_nvf4": [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_int, c_int64, c_int64,
                      c_int64, c_void_p, c_int, c_void_p, c_int, c_int64, c_void_p],
    "kab_gemm_nvf4_scatter": [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_int, c_int64, c_int64,
                              c_int64, c_void_p, c_int, c_void_p, c_int, c_int64, c_void_p, c_int, c_void_p],
    "kab_ipc_handle": [c_void_p, c_void_p, POINTER(c_int64)],
    "kab_ipc_open": [c_void_p, POINTER(c_void_p)],
    "kab_ipc_close": [c_void_p],
    "kab_gemm_mxf4": [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_int, c_int64, c_int64,
                      c_int64, c_void_p, c_int, c_void_p, c_int, c_int64, c_void_p],
    "kab_hadamard_rotate": [c_void_p, c_int, c_int64, c_int64, c_int64, c_int, c_void_p, c_void_p],
    "kab_rmsnorm": [c_void_p, c_int, c_int64, c_int64, c_int64, c_void_p, c_float, c_void_p, c_void_p],
    "kab_rmsnorm_quant_fp8": [c_void_p, c_int, c_int64, c_int64, c_int64, c_void_p, c_float, c_int, c_int, c_void_p,
                              c_void_p, c_void_p, c_void_p],
    "kab_rmsnorm_quant_fp4": [c_void_p, c_int, c_int64, c_int64, c_int64, c_void_p, c_float, c_int, c_int, c_void_p,
                              c_void_p, c_void_p, c_void_p, c_void_p],
    "kab_fp4_bias_correction": [c_void_p, c_int, c_int64, c_int64, c_int64, c_void_p, c_void_p, c_int, c_int,
                                c_void_p, c_int, c_void_p, c_void_p],
    "kab_gemm_f8_blockwise": [c_void_p, c_void_p, c_void_p, c_void_p, c_int64, c_int64, c_int64, c_void_p,
                              c_int, c_void_p, c_int, c_int64, c_void_p],
    "kab_quant_heads_fp8": [c_void_p, c_int, c_int64, c_int64, c_int64, c_int, c_void_p, c_void_p, c_void_p,
                            c_void_p],
    "kab_attention_fp8": [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_int64, c_int64, c_int64,
                          c_int64, c_int64, c_int, ctypes.c_float, c_void_p, c_void_p],
    "kab_diff_census": [c_void_p, c_void_p, c_void_p],
    "kab_outlier_stats": [c_void_p, c_int, c_int64, c_int64, c_int64, c_void_p, c_void_p, c_void_p, c_void_p],
    "kab_row_pair_stats": [c_void_p, c_int, c_int64, c_void_p, c_int, c_int64, c_int64, c_int64, c_void_p,
                           c_void_p],
    "kab_quant_kv_fp8": [c_void_p, c_int, c_int64, c_int64, c_int64, c_int64, c_int64, c_void_p, c_int64, c_int64,
                         c_void_p, c_int64, c_int64, c_void_p],
    "kab_kv_decode_workspace": [POINTER(KabKvDecodeParams), POINTER(c_int), POINTER(c_size_t)],
    "kab_kv_decode_fp8": [POINTER(KabKvDecodeParams), c_void_p, c_size_t, c_void_p],
    "kab_mxfp8_saturation": [c_void_p, c_int, c_int64, c_int64, c_int64, c_void_p, c_void_p, c_void_p],
    "kab_fp4_scale_check": [c_void_p, c_int, c_int64, c_int64, c_int64, c_int, c_void_p, c_void_p, c_int, c_void_p,
                            c_void_p],
    "kab_compare_scratch_bytes": [c_int64],
    "kab_compare": [POINTER(KabCompareParams), c_void_p, c_size_t, c_void_p, c_void_p],
    "kab_compare_noalloc": [POINTER(KabCompareParams), c_void_p, c_void_p],
    "kab_channel_rms_scratch_bytes": [c_int64, c_int64],
    "kab_channel_rms": [c_void_p, c_void_p, c_int, c_int64, c_int64, c_void_p, c_void_p, c_size_t,
                        c_void_p],
}
_RESTYPES = {
    "kab_last_error": ctypes.c_char_p,
    "kab_compare_scratch_bytes": c_size_t,
    "kab_channel_rms_scratch_bytes": c_size_t,
}

_lib: ctypes.CDLL | None = None
_checked_devices: set[int] = set()


def load(path: Path | str | None = None) -> ctypes.CDLL:
    """The loaded library (raises RuntimeError when it was not built)."""
    global _lib
    if _lib is not None:
        return _lib
    p = Path(path) if path is not None else LIB_PATH
    if not p.exists():
        raise RuntimeError(
            f"{p} is missing: build the CUDA library first (python kernel-agent_b200/build.py); "
            "kernel_agent_b200 has no CPU fallback"
        )
    lib = ctypes.CDLL(str(p))
    for name, args in _SIGNATURES.items():
        fn = getattr(lib, name)
        fn.argtypes = args
        fn.restype = _RESTYPES.get(name, c_int)
    _lib = lib
    return lib


def last_error() -> str:
    return (load().kab_last_error() or b"").decode()


def call(name: str, *args) -> None:
    """Run entry point ``name``; a non-zero status raises with the library's message."""
    status = getattr(load(), name)(*args)
    if status != KAB_OK:
        msg = f"{name}: {last_error()}"
        if status == KAB_EINVAL:
            raise ValueError(msg)
        raise RuntimeError(msg)


def query(name: str, *args):
    """Run an entry point that returns a value (not a status)."""
    return getattr(load(), name)(*args)


def ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


def stream_of(t: torch.Tensor) -> int:
    """The current CUDA stream of ``t``'s device, as the void* the ABI takes."""
    return torch.cuda.current_stream(t.device).cuda_stream


def require_cuda(*tensors: torch.Tensor | None) -> torch.device:
    """The device of the given tensors: CUDA, one device, an sm_100 GPU. CPU tensors raise
    ``ValueError("CUDA tensor required")`` (there is no CPU fallback)."""
    dev = None
    for t in tensors:
        if t is None:
            continue
        if not isinstance(t, torch.Tensor) or not t.is_cuda:
            raise ValueError("CUDA tensor required (kernel_agent_b200 runs on the GPU only)")
        if dev is None:
            dev = t.device
        elif t.device != dev:
            raise ValueError(f"tensors on different devices: {dev} and {t.device}")
    if dev is None:
        raise ValueError("CUDA tensor required (kernel_agent_b200 runs on the GPU only)")
    index = dev.index if dev.index is not None else torch.cuda.current_device()
    if index not in _checked_devices:
        call("kab_device_check", index)
        _checked_devices.add(index)
    return dev


def dtype_code(t: torch.Tensor) -> int:
    if t.dtype not in DTYPES:
        raise ValueError(f"unsupported dtype {t.dtype} (float32, bfloat16 or float16)")
    return DTYPES[t.dtype]


def device_status(device: torch.device | None = None, clear: bool = True) -> int:
    """Error bits kernels raised on the device (1: a wait timed out, 2: a bounds check);
    synchronises the current stream."""
    bits = c_uint(0)
    with torch.cuda.device(device):
        call("kab_device_status", ctypes.byref(bits), int(clear), torch.cuda.current_stream().cuda_stream)
    return int(bits.value)

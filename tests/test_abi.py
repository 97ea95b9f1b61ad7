"""The C-ABI library loads and exports every entry point ``include/kab.h`` declares (no GPU:
nothing is called that touches a device)."""

from __future__ import annotations

import ctypes
import re
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
HEADERS = sorted((ROOT / "include").glob("*.h"))
LIB = ROOT / "kernel-agent_b200" / "kernel_agent_b200" / "_native" / "libkab.so"


def declared() -> list[str]:
    names = []
    for h in HEADERS:
        text = re.sub(r"/\*.*?\*/", "", h.read_text(), flags=re.S)
        names += re.findall(r"^\s*(?:const\s+)?[\w]+\s*\*?\s*(kab_\w+)\s*\(", text, flags=re.M)
    return sorted(set(names))


@pytest.fixture(scope="module")
def lib():
    if not LIB.exists():
        from kernel_agent_b200 import __name__ as _  # noqa: F401

        import subprocess
        import sys

        subprocess.run([sys.executable, str(ROOT / "kernel-agent_b200" / "build.py")], check=True)
    return ctypes.CDLL(str(LIB))


def test_header_declares_entry_points():
    names = declared()
    assert "kab_quant_fp4" in names and "kab_compare" in names and len(names) >= 15


def test_library_exports_every_declared_symbol(lib):
    missing = [n for n in declared() if not hasattr(lib, n)]
    assert not missing, f"declared in include/*.h but not exported: {missing}"


def test_no_gpu_calls_needed_for_metadata(lib):
    lib.kab_abi_version.restype = ctypes.c_int
    assert lib.kab_abi_version() == 1
    lib.kab_last_error.restype = ctypes.c_char_p
    assert lib.kab_last_error() == b""
    lib.kab_compare_scratch_bytes.restype = ctypes.c_size_t
    lib.kab_compare_scratch_bytes.argtypes = [ctypes.c_int64]


def test_argument_checks_fail_before_any_launch(lib):
    """Bad arguments return KAB_EINVAL with a message and launch nothing (no device needed)."""
    f = lib.kab_quant_rows_fp8
    f.restype = ctypes.c_int
    f.argtypes = [ctypes.c_void_p, ctypes.c_int, ctypes.c_int64, ctypes.c_int64, ctypes.c_int64,
                  ctypes.c_void_p, ctypes.c_int64, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p,
                  ctypes.c_void_p]
    assert f(16, 1, 4, 12, 16, None, 0, None, None, None, None) == 1  # K not a multiple of 8
    lib.kab_last_error.restype = ctypes.c_char_p
    assert b"multiple of 8" in lib.kab_last_error()
    assert f(16, 7, 4, 16, 16, None, 0, None, None, None, None) == 1  # unknown dtype
    assert b"dtype" in lib.kab_last_error()

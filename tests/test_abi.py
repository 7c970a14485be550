"""The C-ABI library builds for sm_100a, loads, and exports every symbol that
include/*.h declares.  No compute calls (CPU only)."""
import ctypes
import re
from pathlib import Path

import pytest

import fp4x

REPO = Path(__file__).resolve().parent.parent


def declared_symbols():
    names = []
    for h in sorted((REPO / "include").glob("*.h")):
        text = h.read_text()
        names += re.findall(r"^FP4X_API\s+[\w\s\*]+?\b(\w+)\s*\(", text, flags=re.M)
    return names


def test_header_declares_symbols():
    names = declared_symbols()
    assert "fp4_gemv" in names and "llama_attn_decode" in names and "llama_rmsnorm" in names
    assert len(names) == len(set(names))


def test_library_exports_every_declared_symbol():
    lib = fp4x.lib()
    missing = [n for n in declared_symbols() if not hasattr(lib, n)]
    assert not missing, f"declared but not exported: {missing}"


def test_python_mirror_covers_the_header():
    names = set(declared_symbols())
    assert names <= set(fp4x.SIGNATURES) | set(getattr(fp4x, "EXTRA_SIGNATURES", {})), \
        sorted(names - set(fp4x.SIGNATURES))


def test_only_c_abi_is_exported():
    # the library hides everything but the FP4X_API entry points
    import subprocess
    out = subprocess.run(["nm", "-D", "--defined-only", str(fp4x._build.LIB)], capture_output=True, text=True).stdout
    exported = {line.split()[-1] for line in out.splitlines() if " T " in line}
    ours = {n for n in exported if n.startswith(("fp4", "llama"))}
    assert ours == set(declared_symbols()), (ours ^ set(declared_symbols()))


def test_version_and_error_string_without_gpu():
    lib = fp4x.lib()
    assert b"sm_100a" in lib.fp4x_version()
    assert lib.fp4x_last_error() is not None


def test_invalid_arguments_rejected_before_launch():
    # argument validation happens on the host and never reaches the device
    lib = fp4x.lib()
    st = lib.fp4_gemv(None, 16, 33, None, None, None, None)  # null pointers, k % 32 != 0
    assert st == 1
    assert b"null" in lib.fp4x_last_error() or b"k=" in lib.fp4x_last_error()
    st = lib.fp4_gemv(None, 16, 48, ctypes.c_void_p(16), ctypes.c_void_p(16), ctypes.c_void_p(16),
                      ctypes.c_void_p(16))
    assert st == 1 and b"multiple of 32" in lib.fp4x_last_error()
    st = lib.llama_attn_decode_hd(None, 32, 5, 96, 10, ctypes.c_void_p(16), ctypes.c_void_p(16),
                                  ctypes.c_void_p(16), ctypes.c_void_p(16), None, 0)
    assert st == 1

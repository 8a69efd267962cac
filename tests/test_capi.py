"""The C-ABI library: it loads, exports every symbol the public headers declare, and its
host-only logic (type sizes, argument checks) behaves like the reference (CPU only; no
call here reaches a CUDA kernel)."""
from __future__ import annotations

import ctypes as C
import re
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent


def declared_symbols() -> set[str]:
    names = set()
    for h in (ROOT / "include").glob("*.h"):
        text = re.sub(r"/\*.*?\*/", "", h.read_text(), flags=re.S)
        names |= set(re.findall(r"\b(efg_[a-z0-9_]+)\s*\(", text))
    return names


def test_library_exports_every_declared_symbol(efg_lib):
    lib = C.CDLL(str(efg_lib.LIB_PATH))
    names = declared_symbols()
    assert len(names) >= 20
    missing = [n for n in sorted(names) if not hasattr(lib, n)]
    assert not missing, missing


def test_python_binding_covers_the_header(efg_lib):
    from edgeforge_b200._lib import SIGNATURES

    assert declared_symbols() == set(SIGNATURES)


def test_row_bytes_like_the_reference(efg_lib):
    # quant.cpp:136-149 / test_quant.cpp:126-130
    assert efg_lib.row_bytes(efg_lib.QType.Q4_0, 2048) == 1152
    assert efg_lib.row_bytes(efg_lib.QType.Q8_0, 2048) == 2176
    assert efg_lib.row_bytes(efg_lib.QType.BF16, 2048) == 4096
    assert efg_lib.row_bytes(efg_lib.QType.F32, 7) == 28
    assert efg_lib.row_bytes(efg_lib.QType.Q4_0, 131072) == 131072 // 32 * 18
    with pytest.raises(efg_lib.EdgeForgeError, match="needs a row length divisible by 32, got 30"):
        efg_lib.row_bytes(efg_lib.QType.Q4_0, 30)


def test_status_strings_and_abi(efg_lib):
    lib = efg_lib.load()
    assert lib.efg_abi_version() == 1
    assert lib.efg_status_string(0) == b"EFG_OK"
    assert lib.efg_status_string(4) == b"EFG_ETIMEOUT"
    assert lib.efg_status_string(99) == b"EFG_UNKNOWN"


def test_argument_errors_before_any_device_work(efg_lib):
    """Bad arguments are rejected on the host with the reference's wording and codes."""
    lib = efg_lib.load()
    # cols % 32 != 0 -> EFG_EINVAL before a device is touched
    assert lib.efg_matvec_q4_0(None, None, None, 4, 30, None) == 1
    assert b"divisible by 32, got 30" in lib.efg_last_error()
    assert lib.efg_quantize_rows(4, None, 2, 33, None, 1, None) == 1
    assert lib.efg_matvec(7, None, None, None, 1, 32, None) == 1  # no such storage type
    assert b"unknown type" in lib.efg_last_error()
    assert lib.efg_matvec(0, None, None, None, 1, 32, None) == 1  # F32 rows need W, x and y
    assert b"null pointer" in lib.efg_last_error()
    assert lib.efg_host_matvec(4, None, None, None, 1, 40) == 1
    assert lib.efg_host_quantize_row(2, None, 32, None, 1) == 1


def test_reference_names_are_mirrored(efg_lib):
    for name in ("matvec_q4_0", "matvec_q8_0", "matvec", "matvec_jobs", "dot_q4_0", "dot_q8_0", "quantize_row",
                 "dequantize_row", "row_f32", "row_bytes"):
        assert callable(getattr(efg_lib, name))


def test_reference_api_shim_compiles(efg_lib, tmp_path):
    """include/efg_ref_shim.hpp gives the reference's C++ signatures; reference-style test
    code (tests/shim/shim_test.cpp) compiles and links against it and libefg.so."""
    import subprocess

    exe = tmp_path / "shim_test"
    r = subprocess.run(["g++", "-std=c++20", "-O1", "-Wall", "-Werror", "-I", str(ROOT / "include"),
                        str(ROOT / "tests" / "shim" / "shim_test.cpp"), "-L", str(ROOT / "edgeforge_b200"), "-lefg",
                        "-o", str(exe)], capture_output=True, text=True)
    assert r.returncode == 0, r.stderr

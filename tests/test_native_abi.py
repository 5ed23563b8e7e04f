"""The C-ABI library: it loads, exports every symbol include/nv4.h declares, and
rejects bad arguments before touching the GPU (no compute calls here)."""
import ctypes
import os
import re

import pytest

from nanovllm import _native

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared_symbols():
    with open(os.path.join(ROOT, "include", "nv4.h")) as f:
        text = f.read()
    return sorted(set(re.findall(r"\b(nv4_[a-z0-9_]+)\s*\(", text)))


def test_library_exports_every_declared_symbol():
    lib = _native.load()
    names = declared_symbols()
    assert len(names) >= 11
    for name in names:
        assert hasattr(lib, name), name
    assert set(names) == set(_native.EXPORTS)


def test_version_and_status_strings():
    lib = _native.load()
    assert lib.nv4_version() >= 100
    for status in (0, -1, -2, -3, -4, -5):
        assert lib.nv4_status_string(status).decode()
    assert lib.nv4_status_string(123).decode() == "unknown status"


def test_library_is_sm100a_and_self_contained():
    path = _native.LIB_PATH
    with open(path, "rb") as f:
        head = f.read(4)
    assert head == b"\x7fELF"
    # The CUDA runtime is linked statically: no libcudart dependency to resolve.
    import subprocess
    out = subprocess.run(["ldd", path], capture_output=True, text=True).stdout
    assert "libcudart" not in out


V = ctypes.c_void_p


@pytest.mark.parametrize("args,expected", [
    ((None, V(16), V(16), V(16), 1, 4096, 0, -8, None), _native.ERR_INVALID_ARGUMENT),   # null x
    ((V(16), V(16), V(16), V(16), 0, 4096, 0, -8, None), _native.ERR_INVALID_ARGUMENT),  # m = 0
    ((V(16), V(16), V(16), V(16), 1, 4000, 0, -8, None), _native.ERR_INVALID_ARGUMENT),  # k % 128
    ((V(16), V(16), V(16), V(16), 1, 8192, 1, -8, None), _native.ERR_INVALID_ARGUMENT),  # row_DH k
    ((V(16), V(16), V(16), V(16), 1, 4096, 2, -8, None), _native.ERR_INVALID_ARGUMENT),  # layout
    ((V(16), V(16), V(16), V(16), 1, 4096, 0, -6, None), _native.ERR_INVALID_ARGUMENT),  # clamp
    ((V(24), V(16), V(16), V(16), 1, 4096, 0, -8, None), _native.ERR_ALIGNMENT),         # x not 16B
    ((V(16), V(12), V(16), V(16), 1, 4096, 0, -8, None), _native.ERR_ALIGNMENT),         # signs not 8B
])
def test_rht_argument_checks(args, expected):
    assert _native.load().nv4_rht_quant_pack(*args) == expected


@pytest.mark.parametrize("mnk,flags,ptrs,expected", [
    ((1, 8, 100), 1, (16, 16, 16, 16, 16), _native.ERR_INVALID_ARGUMENT),   # k % 128
    ((1, 12, 128), 1, (16, 16, 16, 16, 16), _native.ERR_INVALID_ARGUMENT),  # n % 8
    ((0, 8, 128), 1, (16, 16, 16, 16, 16), _native.ERR_INVALID_ARGUMENT),   # m < 1
    ((1, 8, 128), 64, (16, 16, 16, 16, 16), _native.ERR_INVALID_ARGUMENT),  # unknown flag
    ((1, 8, 128), 1, (8, 16, 16, 16, 16), _native.ERR_ALIGNMENT),           # a_packed not 16B
    ((1, 8, 128), 3, (16, 16, 16, 16, 18), _native.ERR_ALIGNMENT),          # fp32 out not 4B
])
def test_gemm_argument_checks(mnk, flags, ptrs, expected):
    m, n, k = mnk
    p = [V(x) for x in ptrs]
    assert _native.load().nv4_w4a4_grouped_gemm(*p, m, n, k, flags, None) == expected


def test_w4a16_argument_checks():
    lib = _native.load()
    p = [V(16)] * 5
    assert lib.nv4_w4a16_gemm(*p, 1, 64, 128, 64, None, 0, None) == _native.ERR_UNSUPPORTED   # group 64
    assert lib.nv4_w4a16_gemm(*p, 1, 96, 128, 128, None, 0, None) == _native.ERR_INVALID_ARGUMENT  # n % 64
    assert lib.nv4_w4a16_gemm(V(8), *p[1:], 1, 64, 128, 128, None, 0, None) == _native.ERR_ALIGNMENT


def test_python_status_mapping():
    with pytest.raises(ValueError):
        _native.check(_native.ERR_INVALID_ARGUMENT, "x")
    with pytest.raises(ValueError):
        _native.check(_native.ERR_ALIGNMENT, "x")
    with pytest.raises(_native.NativeCallError):
        _native.check(_native.ERR_DEVICE, "x")
    _native.check(_native.OK, "x")


def test_missing_library_fails_loudly(tmp_path):
    with pytest.raises(_native.NativeLibraryError):
        _native.load(str(tmp_path / "libnv4.so"))

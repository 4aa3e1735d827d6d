"""C-ABI checks that need no GPU: the library loads, exports every symbol that
include/yufb200.h declares, and rejects bad arguments on the host before any
CUDA call (the reference op validates in Python, cuda_ops.py:200-209; here the
ABI itself validates so every caller gets the same errors)."""

import ctypes
import re
from pathlib import Path

import pytest

from yufmusicgen_b200 import _lib

HEADER = Path(__file__).resolve().parent.parent / "include" / "yufb200.h"


def declared_functions():
    text = HEADER.read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(yuf_[a-z0-9_]+)\s*\(", text)))


def test_library_exports_every_declared_symbol():
    lib = _lib.load()
    names = declared_functions()
    assert "yuf_wkv7_forward" in names and "yuf_rosa_forward" in names
    missing = [n for n in names if not hasattr(lib, n)]
    assert not missing, f"declared but not exported: {missing}"


def test_python_signatures_cover_header():
    names = set(declared_functions())
    assert set(_lib.SIGNATURES) <= names


def test_status_strings_and_version():
    lib = _lib.load()
    assert _lib.status_name(0) == "YUF_OK"
    assert _lib.status_name(1) == "YUF_ERR_INVALID_ARGUMENT"
    assert lib.yuf_abi_version() >= 1


def _wkv(lib, N=40, B=1, T=4, H=1, ptrs=None, s0=None, compat=False):
    p = ptrs or [16] * 7  # fake but aligned, never dereferenced: validation fails first
    if compat:
        return lib.yuf_wkv7_forward_compat(*p[:7], 16, 16, B, T, H, N, None)
    return lib.yuf_wkv7_forward(*p[:6], s0, p[6], None, B, T, H, N, None)


def test_wkv_rejects_bad_sizes_on_host():
    lib = _lib.load()
    assert _wkv(lib, N=0) == 1
    assert _wkv(lib, B=-1) == 1
    assert "negative" in lib.yuf_last_error().decode()


def test_wkv_rejects_null_and_misaligned():
    lib = _lib.load()
    assert _wkv(lib, ptrs=[16, 16, None, 16, 16, 16, 16]) == 1
    assert "NULL" in lib.yuf_last_error().decode()
    assert _wkv(lib, ptrs=[16, 16, 20, 16, 16, 16, 16]) == 1
    assert "aligned" in lib.yuf_last_error().decode()
    assert _wkv(lib, s0=4) == 1


def test_wkv_compat_requires_padded_T():
    lib = _lib.load()
    assert _wkv(lib, T=17, compat=True) == 1
    assert "multiple of 16" in lib.yuf_last_error().decode()


def test_wkv_unsupported_head_size_is_reported_before_launch():
    # N=24 passes validation but has no kernel: UNSUPPORTED, not a launch.
    lib = _lib.load()
    st = _wkv(lib, N=24)
    assert st == 2, lib.yuf_last_error()
    assert "N=24" in lib.yuf_last_error().decode()


def test_rosa_rejects_bad_args_on_host():
    lib = _lib.load()
    f = lib.yuf_rosa_forward
    assert f(16, 16, 16, 16, 16, 16, 16, 16, 1, 4, 0, 1, None) == 1      # R = 0
    assert f(16, 16, 16, 16, 16, 16, 16, 16, 1, 4, 2000, 1, None) == 1   # R too large
    assert f(16, 16, None, 16, 16, 16, 16, 16, 1, 4, 32, 1, None) == 1   # gated without gate
    g = lib.yuf_rosa_forward_compat
    assert g(*([16] * 14), 1, 4, 48, None) == 1                            # D not in the set
    assert "16, 32, 64, 128, 256" in lib.yuf_last_error().decode()


def test_empty_batch_is_a_noop_without_gpu():
    lib = _lib.load()
    assert _wkv(lib, B=0) == 0
    assert lib.yuf_rosa_forward(None, None, None, 16, 16, 16, None, None, 0, 4, 32, 1, None) == 0


def test_backward_ops_validate_on_host():
    lib = _lib.load()
    wb = lib.yuf_wkv7_backward
    assert wb(*([16] * 15), 1, 17, 1, 40, None) == 1                      # T not a multiple of 16
    assert "multiple of 16" in lib.yuf_last_error().decode()
    assert wb(*([16] * 6), None, *([16] * 8), 1, 16, 1, 40, None) == 1   # dy NULL
    assert wb(*([16] * 15), 1, 16, 1, 24, None) == 2                      # no kernel for N=24
    assert "N=24" in lib.yuf_last_error().decode()
    assert wb(*([16] * 15), 0, 16, 1, 40, None) == 0                      # empty batch
    rb = lib.yuf_rosa_backward
    assert rb(*([16] * 16), 1, 4, 0, None) == 1                           # R = 0
    assert rb(*([16] * 16), 1, 4, 2000, None) == 1                        # R too large
    assert rb(*([16] * 8), None, *([16] * 7), 1, 4, 32, None) == 1       # d_read NULL
    assert rb(*([None] * 16), 0, 4, 32, None) == 0                        # empty batch


def test_generate_params_layout_and_host_validation():
    """yuf_generate_params matches the C layout, and yuf_generate rejects a
    missing model or params before any CUDA call."""
    import ctypes as ct

    assert ct.sizeof(_lib.GenerateParamsC) == 40
    assert _lib.GenerateParamsC.seed.offset == 16
    lib = _lib.load()
    p = _lib.GenerateParamsC(1.0, 32, 1.0, 0, 0, 0, -1, 16)
    assert lib.yuf_generate(None, 16, 1, 1, 0, 1, ct.byref(p), 16, 16, None) == 1
    assert "null model" in lib.yuf_last_error().decode()


def test_python_algorithm_constants_match_the_header():
    """cuda_ops.ALGO_* carry the values of the header's YUF_WKV_* enum."""
    from yufmusicgen_b200 import cuda_ops

    text = HEADER.read_text()
    enum = dict((m.group(1), int(m.group(2))) for m in re.finditer(r"YUF_WKV_([A-Z_]+) = (\d+)", text))
    assert enum == {"AUTO": 0, "SEQUENTIAL": 1, "CHUNKED": 2, "PARALLEL": 3, "PARALLEL_TC": 4, "ROWS": 5,
                    "CHUNKED_TC": 6}
    for name, value in enum.items():
        assert getattr(cuda_ops, f"ALGO_{name}") == value

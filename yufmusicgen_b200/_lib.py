"""ctypes binding of ``libyufb200.so`` (the C ABI in ``include/yufb200.h``).

The library is built in-tree by ``yufmusicgen_b200.build``.  There is no CPU
fallback: if the library is missing or a call fails, the error is raised.
"""

from __future__ import annotations

import ctypes
import threading
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "libyufb200.so"

_lock = threading.Lock()
_lib = None

P = ctypes.c_void_p
I = ctypes.c_int

# name -> argtypes (restype is always int: yuf_status_t)
SIGNATURES = {
    "yuf_wkv7_forward": [P] * 9 + [I] * 4 + [P],
    "yuf_wkv7_forward_ex": [P] * 9 + [I] * 5 + [P],
    "yuf_wkv7_forward_compat": [P] * 9 + [I] * 4 + [P],
    "yuf_rosa_forward": [P] * 8 + [I] * 4 + [P],
    "yuf_rosa_forward_compat": [P] * 14 + [I] * 3 + [P],
    "yuf_wkv7_backward": [P] * 15 + [I] * 4 + [P],
    "yuf_rosa_backward": [P] * 16 + [I] * 3 + [P],
    "yuf_model_create": [P, I, I, I, P, P, P, P],
    "yuf_model_create_from_yuf": [ctypes.c_char_p, I, I, P],
    "yuf_model_destroy": [P],
    "yuf_model_get_config": [P, P],
    "yuf_state_alloc": [P, I],
    "yuf_state_reset": [P, I, I, P],
    "yuf_state_export": [P, I, I, I, P, P, P, P],
    "yuf_state_import": [P, I, I, I, P, P, P, P],
    "yuf_prefill": [P, P, I, I, I, P, P, P],
    "yuf_step": [P, P, I, I, P, P],
    "yuf_step_static": [P, P, I, I, P, P],
    "yuf_model_set_decode_graphs": [P, I],
    "yuf_sample": [P, I, I, ctypes.c_float, I, ctypes.c_float, ctypes.c_uint64, ctypes.c_uint64, I, I,
                   I, I, P, P, P],
    "yuf_philox_uniform": [ctypes.c_uint64, ctypes.c_uint64, I, I, P, P],
    "yuf_generate": [P, P, I, I, I, I, P, P, P, P],
    "yuf_remi_create": [P, I, P],
    "yuf_remi_destroy": [P],
    "yuf_remi_token_id": [P, ctypes.c_char_p],
    "yuf_remi_encode": [P, I, P, I, P, ctypes.c_int64, P],
    "yuf_remi_decode": [P, P, ctypes.c_int64, P, I, P, P, P, ctypes.c_int64, P],
    "yuf_midi_render": [I, P, I, P, ctypes.c_int64, P],
    "yuf_midi_parse": [P, ctypes.c_int64, P, P, P, I, P, P, P, ctypes.c_int64, P],
    "yuf_model_sync_check": [P, P],
    "yuf_sync_check": [P],
    "yuf_debug_wait_selftest": [ctypes.c_ulonglong, P],
    "yuf_model_set_debug": [P, I],
    "yuf_gemm_tf32x3": [P, ctypes.c_longlong, ctypes.c_longlong, P, P, ctypes.c_longlong, P, ctypes.c_longlong,
                        ctypes.c_longlong, I, I, I, I, I, I, I, P],
    "yuf_tf32_split": [P, ctypes.c_size_t, P, P],
    "yuf_mt19937_create": [ctypes.c_uint64, P],
    "yuf_mt19937_destroy": [P],
    "yuf_mt19937_next": [P, P, ctypes.c_int64],
    "yuf_mt19937_exponential": [P, P, ctypes.c_int64],
    "yuf_sample_host": [P, I, I, ctypes.c_float, ctypes.c_float, P, P],
    "yuf_gemm_bf16": [P, ctypes.c_longlong, ctypes.c_longlong, P, ctypes.c_longlong, P, ctypes.c_longlong,
                      ctypes.c_longlong, I, I, I, I, I, I, I, P],
    "yuf_model_set_debug_filter": [P, ctypes.c_char_p, P, I],
    "yuf_debug_dump": [P, ctypes.c_char_p, I, P, ctypes.c_size_t, P],
}


class ModelConfigC(ctypes.Structure):
    """``yuf_model_config`` of include/yufb200.h."""

    _fields_ = [(n, ctypes.c_int) for n in ("vocab_size", "d_model", "n_layers", "n_heads",
                                             "head_size", "rosa_size", "low_rank")]


class GenerateParamsC(ctypes.Structure):
    """``yuf_generate_params`` of include/yufb200.h."""

    _fields_ = [("temperature", ctypes.c_float), ("top_k", ctypes.c_int), ("top_p", ctypes.c_float),
                ("seed", ctypes.c_uint64), ("seq0", ctypes.c_int), ("mask_below", ctypes.c_int),
                ("eos_id", ctypes.c_int), ("min_tokens_before_eos", ctypes.c_int)]


class YufError(RuntimeError):
    """A C-ABI call returned a non-OK status."""

    def __init__(self, func: str, status: int, message: str):
        self.status = status
        super().__init__(f"{func} failed with {status_name(status)}: {message}")


def load():
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is not None:
            return _lib
        if not LIB_PATH.exists():
            raise RuntimeError(
                f"{LIB_PATH} is missing: build it with `python -m yufmusicgen_b200.build` "
                "(this package has no CPU fallback)"
            )
        lib = ctypes.CDLL(str(LIB_PATH))
        lib.yuf_status_string.restype = ctypes.c_char_p
        lib.yuf_status_string.argtypes = [I]
        lib.yuf_last_error.restype = ctypes.c_char_p
        lib.yuf_last_error.argtypes = []
        lib.yuf_abi_version.restype = I
        lib.yuf_wait_timeouts.restype = ctypes.c_uint
        lib.yuf_wait_timeouts.argtypes = []
        for name, args in SIGNATURES.items():
            fn = getattr(lib, name)
            fn.argtypes = args
            fn.restype = I
        _lib = lib
        return lib


def status_name(status: int) -> str:
    return load().yuf_status_string(status).decode()


def call(name: str, *args) -> None:
    lib = load()
    st = getattr(lib, name)(*args)
    if st != 0:
        raise YufError(name, st, lib.yuf_last_error().decode())


def wait_timeouts() -> int:
    """Bounded device waits that expired since the last call (0 when healthy)."""
    return int(load().yuf_wait_timeouts())


def ptr(t) -> int | None:
    """Device pointer of a torch tensor (None for None)."""
    if t is None:
        return None
    return t.data_ptr()

"""Loads libtempo_b200.so (building it in-tree first if it is missing or stale) and declares its C ABI.

There is no fallback: if the library cannot be built or loaded, :func:`load` raises, and every op that needs it
raises with it. Status codes map to the exceptions the reference runtime raises in the same situations
(ValueError, MemoryError, KeyError, RuntimeError, TimeoutError).
"""

from __future__ import annotations

import ctypes
import pathlib
import threading

from tempo_compiler_b200 import build as _build

LIBRARY_PATH: pathlib.Path = _build.LIBRARY

OK, ERR_VALUE, ERR_MEMORY, ERR_KEY, ERR_RUNTIME, ERR_TIMEOUT, ERR_STATE = range(7)

KIND = {"gemm": 1, "gemm_bias": 2, "add": 3, "add_bias": 4, "layernorm": 5, "attention": 6, "decode_attention": 7,
        "copy": 8, "halt": 9}
IMAGE_MAGIC = 0x49324254
IMAGE_BYTES = 64
GEMM_GELU = 1
GEMM_ARGMAX = 2
GEMM_LN = 4

_EXCEPTIONS = {ERR_VALUE: ValueError, ERR_MEMORY: MemoryError, ERR_KEY: KeyError, ERR_RUNTIME: RuntimeError,
               ERR_TIMEOUT: TimeoutError, ERR_STATE: RuntimeError}

_lock = threading.Lock()
_lib: ctypes.CDLL | None = None

_u32, _u64, _i32, _i64, _f32, _f64 = (ctypes.c_uint32, ctypes.c_uint64, ctypes.c_int32, ctypes.c_int64,
                                       ctypes.c_float, ctypes.c_double)
_vp = ctypes.c_void_p


class DecodeLayer(ctypes.Structure):
    """tempo_decode_layer (include/tempo_b200.h): one block's device operands for the persistent decode step."""

    _fields_ = [(name, ctypes.c_void_p) for name in (
        "ln1_gamma", "ln1_beta", "w_qkv", "b_qkv", "w_proj", "b_proj", "ln2_gamma", "ln2_beta", "w_fc", "b_fc",
        "w_out", "b_out", "k_cache", "v_cache")]


class DecodeStepArgs(ctypes.Structure):
    """tempo_decode_step_args (include/tempo_b200.h)."""

    _fields_ = [("layers", ctypes.c_uint32), ("rows", ctypes.c_uint32), ("width", ctypes.c_uint32),
                ("heads", ctypes.c_uint32), ("vocab", ctypes.c_uint32), ("max_positions", ctypes.c_uint32),
                ("capacity", ctypes.c_uint32), ("epsilon", ctypes.c_float), ("layer", ctypes.POINTER(DecodeLayer)),
                ("wte", ctypes.c_void_p), ("wpe", ctypes.c_void_p), ("lnf_gamma", ctypes.c_void_p),
                ("lnf_beta", ctypes.c_void_p), ("ids", ctypes.c_void_p), ("positions", ctypes.c_void_p),
                ("tokens_out", ctypes.c_void_p), ("out_stride", ctypes.c_uint32), ("index_offset", ctypes.c_int32),
                ("workspace", ctypes.c_void_p), ("workspace_bytes", ctypes.c_uint64)]


_SIGNATURES = {
    "tempo_open": [ctypes.c_int, _u64],
    "tempo_close": [],
    "tempo_address_space": [ctypes.POINTER(_u32), ctypes.POINTER(_u64), ctypes.POINTER(_u32)],
    "tempo_malloc": [ctypes.POINTER(_u32), _u64],
    "tempo_free": [_u32],
    "tempo_device_reset": [],
    "tempo_memcpy_h2d": [_u32, _vp, _u64],
    "tempo_memcpy_d2h": [_vp, _u32, _u64],
    "tempo_launch": [_u64, _u64, ctypes.POINTER(_i64), _u32, _f64],
    "tempo_sync": [_f64],
    "tempo_host_alloc": [ctypes.POINTER(_vp), _u64],
    "tempo_host_free": [_vp],
    "tempo_last_error": [ctypes.c_char_p, _u64],
    "tempo_stats": [ctypes.POINTER(_u64), ctypes.POINTER(_u64)],
    "tempo_watchdog": [ctypes.POINTER(_i32)],
    "tempo_wait_probe": [_u32, _u64, _vp],
    "tempo_block_gemm": [_vp, _vp, _vp, _vp, _u32, _u32, _u32, _vp],
    "tempo_block_add": [_vp, _vp, _vp, _u32, _u32, _vp],
    "tempo_block_layernorm": [_vp, _vp, _vp, _u32, _vp],
    "tempo_block_attention": [_vp, _vp, _u32, _u32, _u32, _vp],
    "tempo_block_decode_attention": [_vp, _vp, _vp, _u32, _u32, _u32, _u32, _vp],
    "tempo_block_copy": [_vp, _vp, _u32, _u32, _vp],
    "tempo_gemm": [_vp, _u32, _vp, _u32, _vp, _vp, _u32, _vp, _u32, _u32, _u32, _u32, _u32, _vp, _vp, _vp],
    "tempo_gemm_qkv": [_vp, _u32, _vp, _u32, _vp, _vp, _u32, _u32, _u32, _vp, _vp, _u32, _u32, _u32, _u32, _u32, _vp,
                       _vp],
    "tempo_gemm_ln": [_vp, _u32, _vp, _u32, _vp, _vp, _f32, _vp, _u32, _u32, _u32, _u32, _u32, _vp, _vp, _u32, _u32,
                      _u32, _u32, _vp, _vp],
    "tempo_gemm_rowstats": [_vp, _u32, _vp, _u32, _vp, _vp, _u32, _vp, _u32, _u32, _u32, _u32, _u32, _vp, _vp],
    "tempo_gemm_ln_rowstats": [_vp, _u32, _vp, _u32, _vp, _vp, _f32, _vp, _vp, _u32, _u32, _u32, _u32, _u32, _vp, _vp,
                               _u32, _u32, _u32, _u32, _vp, _vp],
    "tempo_row_stats": [_vp, _u32, _u32, _u32, _vp, _vp],
    "tempo_layernorm": [_vp, _u32, _vp, _vp, _vp, _u32, _u32, _f32, _vp],
    "tempo_embed": [_vp, _vp, _vp, _vp, _vp, _u32, _u32, _u32, _u32, _vp],
    "tempo_attention_prefill": [_vp, _vp, _u32, _u32, _u32, _u32, _vp],
    "tempo_kv_store": [_vp, _vp, _vp, _vp, _vp, _u32, _u32, _u32, _u32, _u32, _vp],
    "tempo_decode_attention": [_vp, _vp, _vp, _vp, _i32, _vp, _u32, _u32, _u32, _u32, _vp],
    "tempo_argmax_finish": [_vp, _vp, _u32, _u32, _vp, _vp, _u32, _vp, _i32, _i32, _vp],
    "tempo_lm_head_argmax_noalloc": [_vp, _u32, _vp, _u32, _u32, _u32, _u32, _vp, _vp],
    "tempo_gemm_norm": [_vp, _u32, _vp, _vp, _f32, _vp, _u32, _vp, _vp, _u32, _u32, _u32, _u32, _u32, _vp, _vp, _vp,
                        _vp, _u32, _u32, _u32, _vp, _vp],
    "tempo_decode_step_workspace": [_u32, _u32, _u32, _u32, ctypes.POINTER(_u64)],
    "tempo_decode_step": [ctypes.POINTER(DecodeStepArgs), _vp],
    "tempo_stream_read_threads": [ctypes.POINTER(_u32)],
    "tempo_stream_read": [_vp, _u64, _vp, _vp],
}

EXPORTED = tuple(_SIGNATURES)
"""Every symbol include/tempo_b200.h declares."""


def load(*, build: bool = True) -> ctypes.CDLL:
    """Returns the loaded library, building it first when missing or stale. Raises if it cannot be had."""
    global _lib
    with _lock:
        if _lib is not None:
            return _lib
        if build:
            _build.build()
        if not LIBRARY_PATH.exists():
            raise ImportError(f"{LIBRARY_PATH} is missing and was not built; the B200 kernels are unavailable")
        lib = ctypes.CDLL(str(LIBRARY_PATH), mode=ctypes.RTLD_GLOBAL)
        for name, argtypes in _SIGNATURES.items():
            fn = getattr(lib, name)
            fn.argtypes = argtypes
            fn.restype = ctypes.c_int32
        _lib = lib
        return lib


def last_error() -> str:
    buffer = ctypes.create_string_buffer(1024)
    load().tempo_last_error(buffer, len(buffer))
    return buffer.value.decode(errors="replace")


def check(status: int) -> None:
    """Raises the exception the reference raises for this status, with the library's message."""
    if status == OK:
        return
    raise _EXCEPTIONS.get(status, RuntimeError)(last_error())


def call(name: str, *args) -> None:
    """Calls one entry point and raises on a non-zero status."""
    check(getattr(load(), name)(*args))

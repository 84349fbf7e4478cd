"""ctypes binding of ``libhayate_b200.so`` (the C ABI in ``include/hayate_b200.h``).

The library is loaded lazily and there is no fallback: if it is missing or does
not export a symbol, every op raises instead of computing on the CPU.
"""

from __future__ import annotations

import ctypes
import os
import threading

from ._build import LIB_PATH

HYT_OK = 0
HYT_ERR_INVALID, HYT_ERR_UNSUPPORTED, HYT_ERR_CUDA, HYT_ERR_WORKSPACE = -1, -2, -3, -4
# size of the static scratch array of hyt_decode_attention_noalloc (include/hayate_b200.h)
HYT_NOALLOC_SCRATCH_BYTES = 8 << 20
HYT_DTYPE_BF16, HYT_DTYPE_F16, HYT_DTYPE_F32 = 0, 1, 2
DEVICE_ERRORS = {
    1: "page id outside the pool",
    2: "kv length needs more pages than the page table row holds",
    4: "kv length beyond the max_kv_len the launch was sized for",
    8: "a bounded pipeline wait gave up",
    16: "tensor-core ops issued on other than exactly one lane (work skipped)",
    32: "packed batch metadata (q_start / q_len / request id) out of range",
    64: "prefill plan item out of range",
}

_c_i32, _c_i64, _c_f32, _c_size, _c_p = (ctypes.c_int32, ctypes.c_int64, ctypes.c_float,
                                         ctypes.c_size_t, ctypes.c_void_p)
_ATTENTION_ARGS = [_c_p, _c_p, _c_p, _c_p, _c_i32, _c_i32, _c_i64, _c_p, _c_i32, _c_p, _c_p, _c_p,
                   _c_i32, _c_i32, _c_i32, _c_i32, _c_i32, _c_i32, _c_i32, _c_f32]

# name -> (restype, argtypes); the list every test checks the library against.
SIGNATURES = {
    "hyt_last_error": (ctypes.c_char_p, []),
    "hyt_version": (ctypes.c_int, []),
    "hyt_kv_scatter": (ctypes.c_int, [_c_p, _c_p, _c_p, _c_p, _c_p, _c_i32, _c_i32, _c_i64, _c_p,
                                      _c_i32, _c_p, _c_i32, _c_i32, _c_i32, _c_i32, _c_i32, _c_i32,
                                      _c_p, _c_p]),
    "hyt_paged_attention": (ctypes.c_int, _ATTENTION_ARGS + [_c_i32, _c_i32, _c_p, _c_size, _c_p, _c_p]),
    "hyt_paged_attention_scatter": (ctypes.c_int, [_c_p, _c_p, _c_p, _c_p, _c_p, _c_p, _c_p, _c_i32,
                                                   _c_i32, _c_i64, _c_p, _c_i32, _c_p, _c_p, _c_p,
                                                   _c_i32, _c_i32, _c_i32, _c_i32, _c_i32, _c_i32,
                                                   _c_i32, _c_f32, _c_i32, _c_i32, _c_p, _c_size,
                                                   _c_p, _c_p]),
    "hyt_decode_attention": (ctypes.c_int, _ATTENTION_ARGS + [_c_i32, _c_i32, _c_p, _c_size, _c_p, _c_p]),
    "hyt_decode_attention_noalloc": (ctypes.c_int, _ATTENTION_ARGS + [_c_i32, _c_i32, _c_p, _c_p]),
    "hyt_prefill_attention": (ctypes.c_int, _ATTENTION_ARGS + [_c_i32, _c_p, _c_p]),
    "hyt_generic_attention": (ctypes.c_int, _ATTENTION_ARGS + [_c_p, _c_p]),
    "hyt_norm_rope_scatter": (ctypes.c_int, [_c_p, _c_p, _c_p, _c_p, _c_p, _c_p, _c_f32, _c_p, _c_p,
                                             _c_i32, _c_p, _c_p, _c_p, _c_p, _c_i32, _c_i32, _c_i64,
                                             _c_p, _c_i32, _c_p, _c_i32, _c_i32, _c_i32, _c_i32,
                                             _c_i32, _c_i32, _c_i32, _c_p, _c_p]),
    # packed (mixed prefill + decode) batches
    "hyt_kv_scatter_packed": (ctypes.c_int, [_c_p, _c_p, _c_p, _c_p, _c_p, _c_i32, _c_i32, _c_i64,
                                             _c_p, _c_i32, _c_p, _c_p, _c_p, _c_i32, _c_i32, _c_i32,
                                             _c_i32, _c_i32, _c_i32, _c_p, _c_p]),
    "hyt_norm_rope_scatter_packed": (ctypes.c_int, [_c_p, _c_p, _c_p, _c_p, _c_p, _c_p, _c_f32, _c_p,
                                                    _c_p, _c_i32, _c_p, _c_p, _c_p, _c_p, _c_i32,
                                                    _c_i32, _c_i64, _c_p, _c_i32, _c_p, _c_p, _c_p,
                                                    _c_i32, _c_i32, _c_i32, _c_i32, _c_i32, _c_i32,
                                                    _c_i32, _c_p, _c_p]),
    "hyt_paged_attention_packed": (ctypes.c_int, [_c_p, _c_p, _c_p, _c_p, _c_i32, _c_i32, _c_i64, _c_p,
                                                  _c_i32, _c_p, _c_p, _c_p, _c_p, _c_p, _c_i32, _c_i32,
                                                  _c_i32, _c_i32, _c_i32, _c_i32, _c_i32, _c_f32, _c_p,
                                                  _c_i32, _c_p, _c_i32, _c_i32, _c_i32, _c_i32, _c_p,
                                                  _c_size, _c_p, _c_p]),
    "hyt_prefill_plan": (_c_i32, [_c_p, _c_p, _c_i32, _c_i32, _c_i32, _c_i32, _c_i32, _c_f32, _c_f32,
                                  _c_p, _c_i32, _c_p]),
    "hyt_prefill_workspace_bytes": (_c_size, [_c_i32]),
    "hyt_prefill_attention_planned": (ctypes.c_int, _ATTENTION_ARGS + [_c_p, _c_i32, _c_i32, _c_p, _c_size,
                                                                       _c_p, _c_p]),
    "hyt_paged_attention_packed_planned": (ctypes.c_int, [_c_p, _c_p, _c_p, _c_p, _c_i32, _c_i32, _c_i64,
                                                          _c_p, _c_i32, _c_p, _c_p, _c_p, _c_p, _c_p,
                                                          _c_i32, _c_i32, _c_i32, _c_i32, _c_i32,
                                                          _c_i32, _c_i32, _c_f32, _c_p, _c_i32, _c_p,
                                                          _c_i32, _c_i32, _c_i32, _c_i32, _c_p, _c_size,
                                                          _c_p, _c_i32, _c_i32, _c_p, _c_size, _c_p,
                                                          _c_p]),
    "hyt_attention_workspace_bytes": (_c_size, [_c_i32] * 8),
    "hyt_workspace_init": (ctypes.c_int, [_c_p, _c_size, _c_p]),
    "hyt_wait_self_test": (ctypes.c_int, [_c_p, _c_p, _c_p]),
    "hyt_read_probe": (ctypes.c_int, [_c_p, _c_size, _c_p, _c_i32, _c_p]),
}

_lock = threading.Lock()
_lib = None


def library_path() -> str:
    return os.environ.get("HAYATE_B200_LIB", LIB_PATH)


def lib() -> ctypes.CDLL:
    """Load and type the native library (raises if it is not built)."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            path = library_path()
            if not os.path.exists(path):
                raise RuntimeError(
                    f"hayate_b200 native library not found at {path}; build it with "
                    "`python -m hayate_b200._build` (there is no CPU fallback)")
            handle = ctypes.CDLL(path)
            for name, (restype, argtypes) in SIGNATURES.items():
                fn = getattr(handle, name)
                fn.restype = restype
                fn.argtypes = argtypes
            _lib = handle
    return _lib


def check(rc: int, what: str) -> None:
    if rc != HYT_OK:
        message = lib().hyt_last_error().decode(errors="replace")
        raise RuntimeError(f"{what} failed ({rc}): {message}")


_int64_arrays: dict = {}


def int64_array(values) -> ctypes.Array:
    """A ctypes int64 array of ``values`` (the C side only reads it: equal tuples share one,
    so per-call stride arrays cost a dictionary lookup)."""
    key = tuple(int(v) for v in values)
    arr = _int64_arrays.get(key)
    if arr is None:
        if len(_int64_arrays) > 4096:
            _int64_arrays.clear()
        arr = (ctypes.c_int64 * len(key))(*key)
        _int64_arrays[key] = arr
    return arr

"""Loads libq38.so (the C ABI of include/q38.h) with ctypes and checks every call's status.

There is no fallback: if the library is missing or a call fails, this raises. Build it with
`python -m` on the package's build.py, or `__graft_entry__.build()`.
"""

from __future__ import annotations

import ctypes
from ctypes import c_float, c_int, c_int64, c_size_t, c_void_p
from pathlib import Path

LIBRARY = Path(__file__).resolve().parent / "libq38.so"

Q38_OK = 0
ERRORS = {-1: "bad argument", -2: "CUDA error", -3: "device wait timed out", -4: "unsupported", -5: "device error"}

# name -> (restype, argtypes), one entry per function of include/q38.h
SIGNATURES = {
    "q38_abi_version": (c_int, []),
    "q38_last_error": (c_int, [ctypes.c_char_p, c_size_t]),
    "q38_set_pdl": (c_int, [c_int]),
    "q38_device_status": (c_int, [c_int]),
    "q38_fp8_gemm_workspace_bytes": (c_size_t, [c_int64, c_int64, c_int]),
    "q38_fp8_gemm": (
        c_int,
        [c_void_p, c_int64, c_int64, c_void_p, c_void_p, c_int64, c_int, c_void_p, c_int64, c_void_p, c_int64, c_int,
         c_void_p, c_size_t, c_void_p],
    ),
    "q38_fp8_gemm_streamk_workspace_bytes": (c_size_t, [c_int64, c_int64, c_int64]),
    "q38_fp8_gemm_streamk": (
        c_int,
        [c_void_p, c_int64, c_int64, c_void_p, c_void_p, c_int64, c_int, c_void_p, c_int64, c_void_p, c_int64, c_void_p,
         c_size_t, c_void_p],
    ),
    "q38_fp8_gemm_static_scratch": (
        c_int,
        [c_void_p, c_int64, c_int64, c_void_p, c_void_p, c_int64, c_int, c_void_p, c_int64, c_void_p, c_int64, c_int,
         c_void_p],
    ),
    "q38_sf_tile_bytes": (c_size_t, [c_int64, c_int64]),
    "q38_rmsnorm_quant": (
        c_int, [c_void_p, c_int64, c_void_p, c_int64, c_int64, c_float, c_void_p, c_int64, c_void_p, c_int64, c_void_p]
    ),
    "q38_rmsnorm_divide": (
        c_int, [c_void_p, c_int64, c_void_p, c_void_p, c_int64, c_int64, c_float, c_void_p, c_int64, c_void_p]
    ),
    "q38_silu_mul_quant": (c_int, [c_void_p, c_int64, c_int64, c_int64, c_void_p, c_int64, c_void_p]),
    "q38_weight_tile_bytes": (c_size_t, [c_int64, c_int64]),
    "q38_bf16_linear": (
        c_int,
        [c_void_p, c_int64, c_int64, c_int64, c_void_p, c_int64, c_void_p, c_int64, c_int, c_void_p, c_size_t, c_void_p],
    ),
    "q38_gdn_decode_workspace_bytes": (c_size_t, [c_int64, c_int, c_int]),
    "q38_gdn_decode": (
        c_int,
        [c_void_p, c_int64, c_void_p, c_int64, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p,
         c_void_p, c_void_p, c_int64, c_int64, c_int, c_int, c_int, c_int, c_int, c_float, c_void_p, c_size_t,
         c_void_p],
    ),
    "q38_attn_decode": (
        c_int,
        [c_void_p, c_int64, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_int64, c_void_p, c_void_p,
         c_void_p, c_int64, c_int64, c_int, c_int, c_int, c_int, c_float, c_void_p, c_void_p],
    ),
    "q38_attn_row_order": (c_int, [c_void_p, c_void_p, c_int64, c_int64, c_void_p, c_void_p]),
    "q38_gdn_prefill_workspace_bytes": (c_size_t, [c_int64, c_int, c_int, c_int, c_int]),
    "q38_gdn_prefill_chunk": (
        c_int,
        [c_void_p, c_int64, c_void_p, c_int64, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_int64,
         c_int64, c_int64, c_int64, c_int64, c_void_p, c_int64, c_int, c_int, c_int, c_int, c_int, c_float, c_void_p,
         c_size_t, c_void_p],
    ),
    "q38_attn_prefill_workspace_bytes": (c_size_t, [c_int64, c_int, c_int]),
    "q38_attn_prefill": (
        c_int,
        [c_void_p, c_int64, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_int64, c_int64, c_int64,
         c_int64, c_int64, c_void_p, c_int64, c_int, c_int, c_int, c_int, c_float, c_void_p, c_size_t, c_void_p],
    ),
    "q38_attn_prefill_e4m3": (
        c_int,
        [c_void_p, c_int64, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_float, c_float, c_int64,
         c_int64, c_int64, c_int64, c_int64, c_void_p, c_int64, c_int, c_int, c_int, c_int, c_float, c_void_p, c_size_t,
         c_void_p],
    ),
    "q38_gdn_verify_workspace_bytes": (c_size_t, [c_int64, c_int, c_int, c_int]),
    "q38_gdn_verify_commit": (
        c_int,
        [c_void_p, c_int64, c_void_p, c_int64, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p,
         c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_int64, c_int64, c_int, c_int, c_int,
         c_int, c_int, c_int, c_float, c_void_p, c_size_t, c_void_p],
    ),
    "q38_attn_verify": (
        c_int,
        [c_void_p, c_int64, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_int64, c_void_p, c_void_p,
         c_void_p, c_int64, c_int64, c_int, c_int, c_int, c_int, c_int, c_float, c_void_p],
    ),
    "q38_comm_init": (c_int, [c_int, c_int, c_int64, c_int64, ctypes.POINTER(c_void_p)]),
    "q38_comm_ipc_handle_bytes": (c_size_t, []),
    "q38_comm_ipc_handle": (c_int, [c_void_p, c_void_p, c_size_t]),
    "q38_comm_connect": (c_int, [c_void_p, c_void_p]),
    "q38_comm_residual": (c_void_p, [c_void_p]),
    "q38_comm_destroy": (c_int, [c_void_p]),
    "q38_fp8_gemm_allreduce": (c_int, [c_void_p, c_int64, c_int64, c_void_p, c_void_p, c_int64, c_int, c_void_p, c_void_p]),
    "q38_fp8_gemm_silu": (c_int, [c_void_p, c_int64, c_int64, c_void_p, c_void_p, c_int64, c_void_p, c_int64, c_void_p]),
    "q38_lm_head_groupmax": (
        c_int, [c_void_p, c_int64, c_int64, c_void_p, c_int64, c_int, c_void_p, c_int64, c_void_p]
    ),    "q38_attn_split_workspace_bytes": (c_size_t, [c_int64, c_int, c_int, c_int, c_int64, c_int]),
    "q38_attn_split": (
        c_int,
        [c_void_p, c_int64, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_int, c_float, c_float,
         c_int64, c_void_p, c_void_p, c_void_p, c_int64, c_int64, c_int, c_int, c_int, c_int, c_int, c_float, c_void_p,
         c_size_t, c_void_p],
    ),
    "q38_lm_head_recheck": (
        c_int,
        [c_void_p, c_int64, c_void_p, c_float, c_void_p, c_int64, c_int64, c_void_p, c_int64, c_int64, c_int64, c_int,
         c_int, c_int64, c_void_p, c_void_p, c_void_p, c_void_p],
    ),
    "q38_embed_rows": (c_int, [c_void_p, c_int64, c_int64, c_void_p, c_int64, c_void_p, c_int64, c_void_p]),
    "q38_lm_head_pick": (c_int, [c_void_p, c_void_p, c_int, c_int64, c_void_p, c_void_p]),
    "q38_copy_state_rows": (
        c_int, [ctypes.POINTER(c_void_p), ctypes.POINTER(c_int64), ctypes.POINTER(c_int64), c_int, c_int64, c_int64,
                c_void_p]
    ),
}

_lib = None


class Q38Error(RuntimeError):
    pass


def load() -> ctypes.CDLL:
    """The loaded library (loaded once). Raises ImportError if it has not been built."""
    global _lib
    if _lib is None:
        if not LIBRARY.exists():
            raise ImportError(f"{LIBRARY} is not built; run the package's build.py (or __graft_entry__.build())")
        lib = ctypes.CDLL(str(LIBRARY))
        for name, (restype, argtypes) in SIGNATURES.items():
            fn = getattr(lib, name)
            fn.restype = restype
            fn.argtypes = argtypes
        _lib = lib
    return _lib


def last_error() -> str:
    buf = ctypes.create_string_buffer(512)
    load().q38_last_error(buf, 512)
    return buf.value.decode(errors="replace")


def check(status: int, what: str) -> None:
    if status != Q38_OK:
        raise Q38Error(f"{what} failed: {ERRORS.get(status, status)}: {last_error()}")


def call(name: str, *args) -> None:
    check(getattr(load(), name)(*args), name)

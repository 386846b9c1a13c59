"""The C-ABI library loads without a GPU and exports every function include/q38.h declares."""

import re
from pathlib import Path

HEADER = Path(__file__).resolve().parent.parent / "include" / "q38.h"


def declared_functions() -> set[str]:
    text = HEADER.read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return set(re.findall(r"^\s*(?:int|size_t)\s+(q38_\w+)\s*\(", text, flags=re.M))


def test_header_declares_the_hot_path():
    names = declared_functions()
    for required in ("q38_fp8_gemm", "q38_gdn_decode", "q38_attn_decode", "q38_lm_head_groupmax", "q38_rmsnorm_quant"):
        assert required in names


def test_library_exports_every_declared_symbol(pkg):
    lib_mod = __import__(pkg.__name__ + "._lib", fromlist=["_lib"])
    lib = lib_mod.load()
    names = declared_functions()
    missing = [n for n in names if not hasattr(lib, n)]
    assert not missing, missing
    assert set(names) <= set(lib_mod.SIGNATURES), set(names) - set(lib_mod.SIGNATURES)
    assert lib.q38_abi_version() >= 1


def test_host_side_argument_checks_need_no_gpu(pkg):
    """Bad arguments are refused on the host, before any CUDA call."""
    lib_mod = __import__(pkg.__name__ + "._lib", fromlist=["_lib"])
    lib = lib_mod.load()
    assert lib.q38_fp8_gemm(None, 1, 128, None, None, 128, 0, None, 128, None, 0, 1, None, 0, None) == -1
    assert "null pointer" in lib_mod.last_error()
    assert lib.q38_sf_tile_bytes(5120, 17408) == 40 * 136 * 512
    assert lib.q38_fp8_gemm_workspace_bytes(256, 5120, 1) == 0
    assert lib.q38_fp8_gemm_workspace_bytes(256, 5120, 3) == 256 + 3 * 40 * 128 * 256 * 4


def test_static_scratch_gemm_checks_arguments_before_any_device_call(pkg):
    """q38_fp8_gemm_static_scratch refuses bad sizes, null pointers and oversized shapes on the host,
    before it looks up or clears its fixed scratch array (no GPU here, so any CUDA call would fail)."""
    import ctypes

    lib_mod = __import__(pkg.__name__ + "._lib", fromlist=["_lib"])
    lib = lib_mod.load()
    dummy = ctypes.c_void_p(16)
    for tokens, features in ((0, 1024), (-5, 1024), (64, 0), (64, -128)):
        status = lib.q38_fp8_gemm_static_scratch(dummy, tokens, 4096, dummy, dummy, features, 0, dummy, 1024, None, 0,
                                                 12, None)
        assert status == -1 and "bad sizes" in lib_mod.last_error(), (tokens, features, lib_mod.last_error())
    assert lib.q38_fp8_gemm_static_scratch(dummy, 64, 4096, dummy, dummy, 1024, 0, None, 1024, None, 0, 12, None) == -1
    assert "null pointer" in lib_mod.last_error()
    assert lib.q38_fp8_gemm_static_scratch(dummy, 64, 4096, dummy, dummy, 1024, 1, dummy, 1024, None, 0, 12, None) == -1
    assert "residual" in lib_mod.last_error()
    status = lib.q38_fp8_gemm_static_scratch(dummy, 4096, 4096, dummy, dummy, 32768, 0, dummy, 32768, None, 0, 12, None)
    assert status == -1 and "scratch" in lib_mod.last_error()


def test_streamk_gemm_checks_arguments_on_the_host(pkg):
    """q38_fp8_gemm_streamk refuses bad sizes, null pointers and a missing residual before any device call,
    and its workspace query answers 0 for a bad shape."""
    import ctypes

    lib_mod = __import__(pkg.__name__ + "._lib", fromlist=["_lib"])
    lib = lib_mod.load()
    dummy = ctypes.c_void_p(16)
    for tokens, features in ((0, 1024), (64, -128)):
        status = lib.q38_fp8_gemm_streamk(dummy, tokens, 4096, dummy, dummy, features, 0, dummy, 1024, None, 0, dummy,
                                          1 << 20, None)
        assert status == -1 and "bad sizes" in lib_mod.last_error(), (tokens, features, lib_mod.last_error())
    assert lib.q38_fp8_gemm_streamk(dummy, 64, 4096, dummy, dummy, 1024, 0, None, 1024, None, 0, dummy, 1 << 20, None) == -1
    assert "null pointer" in lib_mod.last_error()
    assert lib.q38_fp8_gemm_streamk(dummy, 64, 4096, dummy, dummy, 1024, 1, dummy, 1024, None, 0, dummy, 1 << 20, None) == -1
    assert "residual" in lib_mod.last_error()
    assert lib.q38_fp8_gemm_streamk_workspace_bytes(0, 5120, 17408) == 0
    assert lib.q38_fp8_gemm_streamk_workspace_bytes(256, 5120, -1) == 0


def test_copy_state_rows_checks_rows_on_the_host(pkg):
    """Rows outside a buffer, null buffers and empty rows are refused before any CUDA call."""
    import ctypes

    lib_mod = __import__(pkg.__name__ + "._lib", fromlist=["_lib"])
    lib = lib_mod.load()
    ptrs = (ctypes.c_void_p * 2)(16, 32)
    row_bytes = (ctypes.c_int64 * 2)(64, 128)
    rows = (ctypes.c_int64 * 2)(4, 2)
    assert lib.q38_copy_state_rows(ptrs, row_bytes, rows, 2, 0, 3, None) == -1  # row 3 of a 2-row buffer
    assert "outside" in lib_mod.last_error()
    assert lib.q38_copy_state_rows(ptrs, row_bytes, rows, 2, -1, 0, None) == -1
    assert lib.q38_copy_state_rows((ctypes.c_void_p * 2)(16, None), row_bytes, rows, 2, 0, 1, None) == -1
    assert lib.q38_copy_state_rows(ptrs, row_bytes, rows, 2, 1, 1, None) == 0  # same row: nothing to do
    assert lib.q38_copy_state_rows(None, None, None, 0, 0, 1, None) == 0

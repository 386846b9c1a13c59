"""q38_fp8_gemm_static_scratch: the split-K GEMM for callers that cannot allocate device memory.

Callers such as a host whose device memory belongs to a framework pool, a plugin that must not
synchronise the device (cudaMalloc and cudaFree do), or a thin FFI binding that carries only input and
output pointers cannot hand the GEMM a workspace. This entry point keeps the split-K partial sums in a
fixed array inside the library instead. The test calls it through the C ABI, twice in a row (the array
keeps the last call's contents, so the second call checks that nothing stale leaks in), and compares
each result with q38_fp8_gemm given a caller workspace: same kernel, same split order, so bit-equal.
This file sorts last so that a run stopping at the first failure has run everything else first.
"""

import ctypes

import pytest
import torch

pytestmark = pytest.mark.gpu
DEV = "cuda"


@pytest.fixture(scope="module")
def mods(pkg):
    lib_mod = __import__(pkg.__name__ + "._lib", fromlist=["_lib"])
    ops = __import__(pkg.__name__ + ".ops", fromlist=["ops"])
    return lib_mod, ops


# (tokens, k, features, splits, row padding of the output). Padding of 4 bf16 makes the output's row
# stride no multiple of 16 bytes, so it cannot be tensor-mapped and the partial sums go through the
# scratch array even with few splits; more than 8 splits always use it. The other shapes take the
# cluster epilogue, which needs no scratch: the entry point must give the same bits there too.
CASES = [(256, 17408, 5120, 3, 0), (8, 6144, 5120, 3, 0), (37, 512, 384, 2, 0), (256, 17408, 1024, 12, 0),
         (64, 4096, 1024, 4, 4), (200, 3072, 640, 2, 4)]


@pytest.mark.parametrize("tokens,k,features,splits,pad", CASES)
def test_static_scratch_gemm_matches_workspace_gemm_twice(pkg, mods, tokens, k, features, splits, pad):
    lib_mod, ops = mods
    lib = lib_mod.load()
    gen = torch.Generator().manual_seed(tokens + k)
    lin = ops.DeviceLinear(pkg.weights.FP8Weight.from_float(torch.randn(features, k, generator=gen) * 0.02), DEV)
    stream = torch.cuda.current_stream().cuda_stream
    for call in range(2):
        x = pkg.codec.to_e5m2_bytes(torch.randn(tokens, k, generator=gen).to(torch.bfloat16)).to(DEV)
        res = torch.randn(tokens, features + pad, generator=gen).to(torch.bfloat16).to(DEV)
        want = res.clone()
        ws = torch.zeros(max(256, ops.gemm_workspace_bytes(tokens, features, splits)), dtype=torch.uint8, device=DEV)
        ops.fp8_gemm(x, lin, want, residual=want, splits=splits, workspace=ws)
        got = res.clone()
        status = lib.q38_fp8_gemm_static_scratch(x.data_ptr(), tokens, k, lin.q.data_ptr(), lin.sf.data_ptr(), features,
                                                 1, got.data_ptr(), got.stride(0), got.data_ptr(), got.stride(0), splits,
                                                 stream)
        assert status == 0, lib_mod.last_error()
        torch.cuda.synchronize()
        assert torch.equal(got, want), f"call {call}: static-scratch result differs from the workspace result"


def test_static_scratch_refuses_shapes_beyond_its_size(pkg, mods):
    lib_mod, _ = mods
    lib = lib_mod.load()
    tokens, features, splits = 4096, 32768, 12  # more than 8 splits: the scratch path
    assert lib.q38_fp8_gemm_workspace_bytes(tokens, features, splits) > 16 * 1024 * 1024
    dummy = ctypes.c_void_p(16)
    status = lib.q38_fp8_gemm_static_scratch(dummy, tokens, 4096, dummy, dummy, features, 0, dummy, features, None, 0,
                                             splits, None)
    assert status == -1 and "scratch" in lib_mod.last_error()

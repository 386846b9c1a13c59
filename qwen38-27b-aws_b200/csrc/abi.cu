// Host-side plumbing of the C ABI: error messages, the device error word, tensor-map encoding.
#include <atomic>
#include <cstdarg>
#include <cstdlib>
#include <cstdio>
#include <cstring>

#include "q38_common.cuh"

namespace q38 {
__device__ int g_device_error = 0;
}

namespace {
thread_local char g_last_error[512] = {0};

using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  if (!fn) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  }
  return fn;
}
}  // namespace

namespace q38host {

namespace {
std::atomic<int> g_pdl{-1};  // -1: not decided yet (environment), 0 off, 1 on
}

bool pdl_enabled() {
  int v = g_pdl.load(std::memory_order_relaxed);
  if (v < 0) {
    const char* env = std::getenv("Q38_PDL");
    v = (env && env[0] == '0') ? 0 : 1;
    g_pdl.store(v, std::memory_order_relaxed);
  }
  return v != 0;
}

void set_error(const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_last_error, sizeof(g_last_error), fmt, ap);
  va_end(ap);
}

int cuda_status(cudaError_t e, const char* what) {
  if (e == cudaSuccess) return Q38_OK;
  set_error("%s: %s", what, cudaGetErrorString(e));
  return Q38_ERR_CUDA;
}

int encode_tmap_2d(CUtensorMap* map, const void* base, uint64_t rows, uint64_t cols, uint32_t elem_bytes,
                   uint32_t box_rows, uint32_t box_cols, bool swizzle128, uint64_t ld) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return set_error("cuTensorMapEncodeTiled is not available from the driver"), Q38_ERR_CUDA;
  if (ld == 0) ld = cols;
  if ((reinterpret_cast<uintptr_t>(base) & 15u) != 0 || (ld * elem_bytes) % 16 != 0)
    return set_error("tensor map: base must be 16-byte aligned and rows a multiple of 16 bytes apart"), Q38_ERR_ARG;
  const CUtensorMapDataType dt = elem_bytes == 1 ? CU_TENSOR_MAP_DATA_TYPE_UINT8 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
  cuuint64_t dims[2] = {cols, rows};
  cuuint64_t strides[1] = {ld * elem_bytes};
  cuuint32_t box[2] = {box_cols, box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(map, dt, 2, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                  swizzle128 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    return set_error("cuTensorMapEncodeTiled failed (%d) rows=%llu cols=%llu box=%ux%u", static_cast<int>(r),
                     static_cast<unsigned long long>(rows), static_cast<unsigned long long>(cols), box_rows, box_cols),
           Q38_ERR_CUDA;
  return Q38_OK;
}

}  // namespace q38host

extern "C" int q38_abi_version(void) { return 1; }

extern "C" int q38_set_pdl(int enable) {
  q38host::g_pdl.store(enable ? 1 : 0, std::memory_order_relaxed);
  return Q38_OK;
}

extern "C" int q38_last_error(char* buf, size_t n) {
  const size_t len = strlen(g_last_error);
  if (buf && n > 0) {
    const size_t c = len < n - 1 ? len : n - 1;
    memcpy(buf, g_last_error, c);
    buf[c] = '\0';
  }
  return static_cast<int>(len);
}

extern "C" int q38_device_status(int reset) {
  cudaError_t e = cudaDeviceSynchronize();
  if (e != cudaSuccess) return q38host::cuda_status(e, "cudaDeviceSynchronize");
  int code = 0;
  e = cudaMemcpyFromSymbol(&code, q38::g_device_error, sizeof(int));
  if (e != cudaSuccess) return q38host::cuda_status(e, "read device error word");
  if (reset && code != 0) {
    const int zero = 0;
    e = cudaMemcpyToSymbol(q38::g_device_error, &zero, sizeof(int));
    if (e != cudaSuccess) return q38host::cuda_status(e, "clear device error word");
  }
  if (code != 0) q38host::set_error("a kernel recorded device error %d", code);
  return code;
}

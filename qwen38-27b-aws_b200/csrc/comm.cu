// The tensor-parallel communicator: one exchange region per rank, mapped into every peer through CUDA
// IPC, for the fused GEMM + all-reduce (q38_fp8_gemm_allreduce). Replaces the reference's NxD
// all-reduce plumbing (qwen38_inf2/neuron.py:9, the all_reduce injection model.py:44-45) with peer
// memory: the host passes the IPC handles between ranks (torch.distributed in this package), the
// kernels do the exchange.
#include <cstring>

#include "comm_internal.cuh"
#include "q38_common.cuh"

namespace {

size_t align256(size_t x) { return (x + 255) & ~size_t(255); }

}  // namespace

extern "C" int q38_comm_init(int rank, int world, int64_t max_tokens, int64_t hidden, void** comm) {
  using namespace q38host;
  if (!comm) return set_error("q38_comm_init: null output"), Q38_ERR_ARG;
  *comm = nullptr;
  if (world < 1 || world > q38::kMaxRanks || rank < 0 || rank >= world)
    return set_error("q38_comm_init: rank %d of world %d (1..%d ranks built)", rank, world, q38::kMaxRanks), Q38_ERR_ARG;
  if (max_tokens <= 0 || max_tokens > 65536 || hidden <= 0 || hidden % 128 != 0)
    return set_error("q38_comm_init: max_tokens %lld, hidden %lld (a multiple of 128)", static_cast<long long>(max_tokens),
                     static_cast<long long>(hidden)),
           Q38_ERR_ARG;
  Comm* c = new Comm();
  c->rank = rank;
  c->world = world;
  c->tmax = max_tokens;
  c->hidden = hidden;
  cudaError_t e = cudaGetDevice(&c->device);
  if (e != cudaSuccess) {
    delete c;
    return cuda_status(e, "cudaGetDevice");
  }
  const size_t slab = 2 * static_cast<size_t>(max_tokens) * hidden;  // bytes of one [tokens][hidden] bf16 slab
  size_t off = 0;
  c->off_x = off;
  off = align256(off + slab);
  c->off_part = off;
  off = align256(off + 2 * static_cast<size_t>(world) * slab);
  c->off_pflag = off;
  off = align256(off + sizeof(uint32_t) * world * q38::kMaxCtas);
  c->off_rflag = off;
  off = align256(off + sizeof(uint32_t) * world * q38::kMaxCtas);
  c->off_epoch = off;
  c->off_done = off + sizeof(uint32_t);
  c->bytes = align256(off + 2 * sizeof(uint32_t));
  e = cudaMalloc(&c->base, c->bytes);
  if (e != cudaSuccess) {
    delete c;
    return cuda_status(e, "cudaMalloc(comm region)");
  }
  e = cudaMemset(c->base, 0, c->bytes);
  const uint32_t one = 1;  // epochs start at 1: the zeroed flags hold epoch 0
  if (e == cudaSuccess) e = cudaMemcpy(c->base + c->off_epoch, &one, sizeof(one), cudaMemcpyHostToDevice);
  if (e != cudaSuccess) {
    cudaFree(c->base);
    delete c;
    return cuda_status(e, "initialise comm region");
  }
  c->peer[rank] = c->base;
  *comm = c;
  return Q38_OK;
}

extern "C" int q38_comm_ipc_handle(void* comm, void* handle, size_t handle_bytes) {
  using namespace q38host;
  Comm* c = static_cast<Comm*>(comm);
  if (!c || !handle || handle_bytes < sizeof(cudaIpcMemHandle_t))
    return set_error("q38_comm_ipc_handle: needs a communicator and %zu bytes", sizeof(cudaIpcMemHandle_t)), Q38_ERR_ARG;
  cudaIpcMemHandle_t h;
  cudaError_t e = cudaIpcGetMemHandle(&h, c->base);
  if (e != cudaSuccess) return cuda_status(e, "cudaIpcGetMemHandle");
  std::memcpy(handle, &h, sizeof(h));
  return Q38_OK;
}

extern "C" size_t q38_comm_ipc_handle_bytes(void) { return sizeof(cudaIpcMemHandle_t); }

extern "C" int q38_comm_connect(void* comm, const void* handles) {
  using namespace q38host;
  Comm* c = static_cast<Comm*>(comm);
  if (!c || !handles) return set_error("q38_comm_connect: null argument"), Q38_ERR_ARG;
  if (c->connected) return Q38_OK;
  const uint8_t* hs = static_cast<const uint8_t*>(handles);
  for (int r = 0; r < c->world; ++r) {
    if (r == c->rank) continue;
    cudaIpcMemHandle_t h;
    std::memcpy(&h, hs + r * sizeof(cudaIpcMemHandle_t), sizeof(h));
    void* p = nullptr;
    cudaError_t e = cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess);
    if (e != cudaSuccess) {
      for (int q = 0; q < r; ++q)
        if (q != c->rank && c->peer[q]) {
          cudaIpcCloseMemHandle(c->peer[q]);
          c->peer[q] = nullptr;
        }
      return cuda_status(e, "cudaIpcOpenMemHandle (peer access over NVLink)");
    }
    c->peer[r] = static_cast<uint8_t*>(p);
  }
  c->connected = true;
  return Q38_OK;
}

extern "C" void* q38_comm_residual(void* comm) {
  q38host::Comm* c = static_cast<q38host::Comm*>(comm);
  return c ? c->base + c->off_x : nullptr;
}

extern "C" int q38_comm_destroy(void* comm) {
  using namespace q38host;
  Comm* c = static_cast<Comm*>(comm);
  if (!c) return Q38_OK;
  cudaError_t first = cudaSuccess;
  for (int r = 0; r < c->world; ++r)
    if (r != c->rank && c->peer[r]) {
      cudaError_t e = cudaIpcCloseMemHandle(c->peer[r]);
      if (first == cudaSuccess) first = e;
    }
  cudaError_t e = cudaFree(c->base);
  if (first == cudaSuccess) first = e;
  delete c;
  return cuda_status(first, "q38_comm_destroy");
}

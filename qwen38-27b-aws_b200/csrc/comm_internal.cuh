// The tensor-parallel exchange region shared by the fused GEMM + all-reduce (fp8_gemm.cu) and the
// communicator's C ABI (comm.cu).
//
// Each rank allocates one region with cudaMalloc and maps every peer's region through CUDA IPC (over
// NVLink peer access), so a kernel can store straight into a peer's HBM. Everything that crosses
// NVLink travels as 64-bit words {two bf16 values, the call's epoch}: an aligned 64-bit store arrives
// whole, so a receiver polling its own memory sees data and "ready" together, with no fence and no
// separate flag (a system-scope fence costs ~10 us on B200; this is the low-latency form of NCCL's LL
// protocol). Layout (same offsets on every rank), by epoch parity so a rank one call ahead never
// overwrites words still being read:
//   x       bf16 [max_tokens][hidden]                 the residual stream, replicated on every rank
//   part    u64  [2][world][max_tokens][hidden / 2]   partials pushed to this rank (the owner) by each source
//   result  u64  [2][max_tokens][hidden / 2]          reduced rows pushed to this rank by their owners
//   epoch   u32                                       the call counter, advanced by the last CTA of a call
//   done    u32                                       CTAs finished in the current call
#pragma once

#include <stdint.h>

#include <cuda_bf16.h>

namespace q38 {

constexpr int kMaxRanks = 8;

struct ArArgs {
  int rank, world;
  int ftiles;  // 128-feature tiles of hidden
  int64_t tmax, hidden;
  __nv_bfloat16* x[kMaxRanks];
  unsigned long long* part[kMaxRanks];
  unsigned long long* result[kMaxRanks];
  uint32_t* epoch;  // this rank's
  uint32_t* done;   // this rank's
};

}  // namespace q38

namespace q38host {

struct Comm {
  int rank = 0, world = 0, device = 0;
  int64_t tmax = 0, hidden = 0;
  size_t off_x = 0, off_part = 0, off_result = 0, off_epoch = 0, off_done = 0, bytes = 0;
  uint8_t* base = nullptr;                     // this rank's region
  uint8_t* peer[q38::kMaxRanks] = {nullptr};  // every rank's region as mapped here (peer[rank] == base)
  bool connected = false;
};

// Fills the device view of a connected communicator.
inline q38::ArArgs ar_args(const Comm& c) {
  q38::ArArgs a{};
  a.rank = c.rank;
  a.world = c.world;
  a.ftiles = static_cast<int>((c.hidden + 127) / 128);
  a.tmax = c.tmax;
  a.hidden = c.hidden;
  for (int r = 0; r < c.world; ++r) {
    a.x[r] = reinterpret_cast<__nv_bfloat16*>(c.peer[r] + c.off_x);
    a.part[r] = reinterpret_cast<unsigned long long*>(c.peer[r] + c.off_part);
    a.result[r] = reinterpret_cast<unsigned long long*>(c.peer[r] + c.off_result);
  }
  a.epoch = reinterpret_cast<uint32_t*>(c.base + c.off_epoch);
  a.done = reinterpret_cast<uint32_t*>(c.base + c.off_done);
  return a;
}

}  // namespace q38host

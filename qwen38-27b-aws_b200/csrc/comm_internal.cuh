// The tensor-parallel exchange region shared by the fused GEMM + all-reduce (fp8_gemm.cu) and the
// communicator's C ABI (comm.cu).
//
// Each rank allocates one region with cudaMalloc and maps every peer's region through CUDA IPC (over
// NVLink peer access), so a kernel can store straight into a peer's HBM. Layout (same offsets on every
// rank):
//   x       bf16 [max_tokens][hidden]      the residual stream, replicated on every rank
//   recv    bf16 [2][world][max_tokens][hidden]   partial tiles pushed by each source rank, by epoch parity
//   flags   u32  [2][world][slots]          "source's partial of this slot has arrived" (= epoch)
//   gflags  u32  [2][slots]                 "the owner's reduced tile of this slot has arrived" (= epoch)
//   epoch   u32                             the call counter, advanced by the last CTA of each call
//   done    u32                             CTAs finished in the current call
// A slot is one 32-token x 128-feature block of the output: slot = (token / 32) * feature_tiles + tile.
#pragma once

#include <stdint.h>

#include <cuda_bf16.h>

namespace q38 {

constexpr int kMaxRanks = 8;

struct ArArgs {
  int rank, world;
  int ftiles;  // 128-feature tiles of hidden
  int slots;   // per parity and source
  int64_t tmax, hidden;
  __nv_bfloat16* x[kMaxRanks];
  __nv_bfloat16* recv[kMaxRanks];
  uint32_t* flags[kMaxRanks];
  uint32_t* gflags[kMaxRanks];
  uint32_t* epoch;  // this rank's
  uint32_t* done;   // this rank's
};

}  // namespace q38

namespace q38host {

struct Comm {
  int rank = 0, world = 0, device = 0;
  int64_t tmax = 0, hidden = 0;
  int slots = 0;
  size_t off_x = 0, off_recv = 0, off_flags = 0, off_gflags = 0, off_epoch = 0, off_done = 0, bytes = 0;
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
  a.slots = c.slots;
  a.tmax = c.tmax;
  a.hidden = c.hidden;
  for (int r = 0; r < c.world; ++r) {
    a.x[r] = reinterpret_cast<__nv_bfloat16*>(c.peer[r] + c.off_x);
    a.recv[r] = reinterpret_cast<__nv_bfloat16*>(c.peer[r] + c.off_recv);
    a.flags[r] = reinterpret_cast<uint32_t*>(c.peer[r] + c.off_flags);
    a.gflags[r] = reinterpret_cast<uint32_t*>(c.peer[r] + c.off_gflags);
  }
  a.epoch = reinterpret_cast<uint32_t*>(c.base + c.off_epoch);
  a.done = reinterpret_cast<uint32_t*>(c.base + c.off_done);
  return a;
}

}  // namespace q38host

// The tensor-parallel exchange region shared by the fused GEMM + all-reduce (fp8_gemm.cu) and the
// communicator's C ABI (comm.cu).
//
// Each rank allocates one region with cudaMalloc and maps every peer's region through CUDA IPC (over
// NVLink peer access), so a kernel can store straight into a peer's HBM. Data crosses NVLink as plain
// bf16 rows (16-byte stores); each CTA that has pushed rows to a rank then publishes the call's epoch in
// a flag of its own there (a system-scope release after its stores), and the receiving CTA (the same
// grid position on that rank) acquires it before reading. Layout (same offsets on every rank):
//   x       bf16 [max_tokens][hidden]               the residual stream; owners write their reduced rows
//                                                   straight into every rank's x
//   part    bf16 [2][world][max_tokens][hidden]     partials pushed to this rank by each source, by the
//                                                   call's parity (a rank runs at most one call ahead)
//   pflag   u32  [world][kMaxCtas]                  per source rank and CTA: the last call whose partials
//                                                   it has pushed here
//   rflag   u32  [world][kMaxCtas]                  per owner rank and CTA: the last call whose reduced
//                                                   rows it has written into this rank's x
//   epoch   u32                                     the call counter, advanced by the last CTA of a call
//   done    u32                                     CTAs finished in the current call
#pragma once

#include <stdint.h>

#include <cuda_bf16.h>

namespace q38 {

constexpr int kMaxRanks = 8;
constexpr int kMaxCtas = 16384;  // CTAs of one fused GEMM + all-reduce launch

struct ArArgs {
  int rank, world;
  int ftiles;  // 128-feature tiles of hidden
  int64_t tmax, hidden;
  __nv_bfloat16* x[kMaxRanks];
  __nv_bfloat16* part[kMaxRanks];
  uint32_t* pflag[kMaxRanks];
  uint32_t* rflag[kMaxRanks];
  uint32_t* epoch;  // this rank's
  uint32_t* done;   // this rank's
};

}  // namespace q38

namespace q38host {

struct Comm {
  int rank = 0, world = 0, device = 0;
  int64_t tmax = 0, hidden = 0;
  size_t off_x = 0, off_part = 0, off_pflag = 0, off_rflag = 0, off_epoch = 0, off_done = 0, bytes = 0;
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
    a.part[r] = reinterpret_cast<__nv_bfloat16*>(c.peer[r] + c.off_part);
    a.pflag[r] = reinterpret_cast<uint32_t*>(c.peer[r] + c.off_pflag);
    a.rflag[r] = reinterpret_cast<uint32_t*>(c.peer[r] + c.off_rflag);
  }
  a.epoch = reinterpret_cast<uint32_t*>(c.base + c.off_epoch);
  a.done = reinterpret_cast<uint32_t*>(c.base + c.off_done);
  return a;
}

}  // namespace q38host

// Tensor-core GEMMs for sm_100a: the FP8 linear layers (and their fused epilogues) and the BF16 linear.
//
// Layout ("swap AB"): the weight matrix W [features, K] is the MMA's A operand (M = 128 features
// per tile) and the activations X [tokens, K] are its B operand (N = 128 or 256 tokens per tile),
// so a decode batch of 8..256 rows fills the MMA's N side and every weight byte is read once per
// token tile. D[feature, token] accumulates in TMEM (lane = feature, column = token).
//
// Weights arrive pre-tiled (codec.tile_weight): 128 rows x 128 bytes of K per 16 KB tile, tiles of
// one row block consecutive along K, each already 128-byte swizzled. A stage's W tile is therefore
// one contiguous bulk copy, and a CTA streams one long contiguous run of HBM.
//
// Roles in one CTA of 192 threads:
//   warp 0      producer: W tile (bulk copy of 16 KB), X tile [NTOK x 128 B] (TMA, 128-byte
//               swizzle) and, for FP8, the 512-byte scale block of the W tile, into a STAGES-deep ring.
//   warp 1      MMA issuer: one thread copies the W scales to TMEM (tcgen05.cp) and issues the
//               4 MMAs of each stage (K = 32 bytes each), then commits the stage back to warp 0.
//   warps 2..5  epilogue: tcgen05.ld of their 32-lane quarter, then the epilogue below.
//
// FP8 path: tcgen05.mma kind::mxf8f6f4.block_scale, A = e4m3 weights with UE8M0 scales per 32 K
// (exact dequantisation: the reference's weights are e4m3 * 2^s), B = e5m2 activations with scale
// 1.0. BF16 path (in_proj_b/a): kind::f16 with BF16 A and B. The lm_head has its own kernel (lm_head.cu).
//
// Split K: up to 8 K splits of a tile form one thread-block cluster; each split sends the 32-token
// blocks of its fp32 partial that other splits own to them by bulk shared-memory copies, and each
// owner sums its blocks in split order 0..S-1 (the own partial straight from TMEM) and applies the
// epilogue. With more splits (or an output that cannot be tensor-mapped) each CTA stores its partial
// in a workspace and the last CTA of a tile (by an atomic counter) sums them in split order, then
// resets the counter. Either way results do not depend on which CTA finishes last.
//
// Epilogues: bf16, bf16 + residual, SiLU(gate) * up to e5m2 (persistent kernel), and the fused
// tensor-parallel all-reduce (EPI_ALLREDUCE: rows to their owner ranks over NVLink, see below). The
// persistent kernel also runs stream-K (q38_fp8_gemm_streamk).
#include <algorithm>
#include <cmath>
#include <cstdio>

#include "comm_internal.cuh"
#include "q38_common.cuh"

namespace {

using namespace q38;

constexpr int BM = 128;          // features per tile (MMA M)
constexpr int BK_BYTES = 128;    // K bytes per pipeline stage (one 128-byte swizzle row)
constexpr int SF_BLOCK = 512;    // scale bytes per (128 rows, 128 K) block

enum : int { EPI_BF16 = 0, EPI_RESIDUAL = 1, EPI_ALLREDUCE = 3, EPI_SILU = 4 };

// PAIR: the 2-SM form. A cluster pair of CTAs computes 256 weight rows x NTOK tokens with
// tcgen05.mma.cta_group::2 issued by the even CTA; each CTA loads its own 128 weight rows and half of
// the tokens, so per SM a stage moves 16 KB of activations instead of 32 KB and six stages fit.
template <int NTOK, bool MX, bool PAIR = false>
struct Cfg {
  static constexpr int A_BYTES = BM * BK_BYTES;
  static constexpr int B_ROWS = PAIR ? NTOK / 2 : NTOK;
  static constexpr int B_BYTES = B_ROWS * BK_BYTES;
  static constexpr int SF_BYTES = MX ? SF_BLOCK : 0;
  static constexpr int STAGES = (PAIR || NTOK != 256) ? 6 : 4;
  static constexpr int TMEM_COLS = NTOK == 256 ? 512 : 256;
  static constexpr int SFA_COL = NTOK;       // 4 columns per stage
  static constexpr int SFB_COL = NTOK + 32;  // 8 columns of 1.0 scales for the activations
  static constexpr size_t PIPE = STAGES * (A_BYTES + B_BYTES + SF_BYTES);
  static constexpr size_t SMEM = 1024 + PIPE + 256;
  static_assert(NTOK * BM * 4 + NTOK * BM * 2 <= PIPE, "epilogue staging must fit in the pipeline buffers");
};

struct GemmArgs {
  const uint8_t* w;   // pre-tiled W (16 KB tiles, [row tile][K tile])
  const uint8_t* sf;  // pre-tiled W scales (FP8 path)
  int T, F, nkc;      // tokens, features, K stages
  int splits, kc_per_split;
  int epilogue;
  __nv_bfloat16* y;
  int64_t ldy;
  const __nv_bfloat16* res;
  int64_t ldr;
  float* ws;              // split partials (workspace mode)
  unsigned int* counters; // one per output tile (workspace mode)
  int cluster;            // > 0: epilogue through shared memory, the `cluster` K splits of a tile
                          // forming one thread-block cluster; 0: workspace mode
  ArArgs ar;              // EPI_ALLREDUCE: the ranks' exchange regions
  uint8_t* yq;            // EPI_SILU: e5m2 [T, ldq] of SiLU(gate) * up
  int64_t ldq;
  // Stream-K (persistent kernel, sk_groups > 0): group g of sk_groups owns the linear K steps
  // [g W / G, (g + 1) W / G) of W = tiles x nkc; a tile split between groups sums its fp32 partials
  // from ws ([128-row tile][sk_max_seg slots][128 x NTOK]) in K order, by the last group to finish.
  int sk_groups;
  int sk_max_seg;
};

// Epilogue staging (cluster mode), reusing the pipeline buffers once the accumulator is final: bf16
// [NTOK][128] for the residual in and the output out (the same bytes: each element is read before it
// is overwritten by its own thread), at NTOK * 128 * 4 with one split, over the send buffers below with
// split K.
constexpr int TOK_BLOCK = 32;  // tokens per TMA box of the residual / output
constexpr int BLOCK_F32_BYTES = TOK_BLOCK * BM * 4;  // one token block of a split's fp32 partial: 16 KB

// Split reduction through the cluster (c K splits of one output tile, one CTA each): token block b of
// the tile belongs to the split CTA whose slice [s nb / c, (s + 1) nb / c) holds it. Shared memory,
// reusing the pipeline buffers once the mainloops are done: the receive buffer [c - 1 sources][slice
// tokens][128 rows] fp32 at 0, then this CTA's fp32 partials of the blocks it sends (compact, in block
// order), over which the bf16 output staging [NTOK][128] later lies.
template <int NTOK>
__host__ __device__ constexpr int split_slice_tokens(int c) {
  return (NTOK / TOK_BLOCK + c - 1) / c * TOK_BLOCK;
}
template <int NTOK>
__host__ __device__ constexpr size_t split_send_offset(int c) {
  return c > 1 ? static_cast<size_t>(c - 1) * split_slice_tokens<NTOK>(c) * BM * 4 : 0;
}
template <int NTOK>
__host__ __device__ constexpr size_t split_smem_bytes(int c) {
  // The fewest blocks a split owns is nb / c (rounded down), so it sends at most nb - nb / c.
  return split_send_offset<NTOK>(c) +
         (static_cast<size_t>(NTOK / TOK_BLOCK - NTOK / TOK_BLOCK / c) * BLOCK_F32_BYTES > static_cast<size_t>(NTOK) * BM * 2
              ? static_cast<size_t>(NTOK / TOK_BLOCK - NTOK / TOK_BLOCK / c) * BLOCK_F32_BYTES
              : static_cast<size_t>(NTOK) * BM * 2);
}

__device__ __forceinline__ void epi_bar() { asm volatile("bar.sync 1, 128;" ::: "memory"); }
// The epilogue warps' barrier that also returns, to every one of them, whether any passed `pred`.
__device__ __forceinline__ bool epi_bar_or(bool pred) {
  uint32_t r;
  asm volatile(
      "{\n .reg .pred p, q;\n setp.ne.u32 p, %1, 0;\n bar.red.or.pred q, 1, 128, p;\n selp.u32 %0, 1, 0, q;\n}"
      : "=r"(r)
      : "r"(static_cast<uint32_t>(pred))
      : "memory");
  return r != 0;
}

// Peer-memory exchange of the fused all-reduce: rows go across NVLink as bulk copies (shared memory ->
// the peer's HBM, moved by the SM's TMA unit, off its load/store path). A CTA publishes "my rows for
// call `epoch` are there" by storing the epoch into a flag at the receiving rank once every one of its
// copies is complete: each thread waits for its own bulk group (cp.async.bulk.wait_group 0: the writes
// are performed at their destination, the peer's memory), then a barrier, then the flag store. Nothing
// is left in flight for the flag to overtake, so the store is relaxed; a release store would add a
// system-scope fence, measured at ~3 us per call here. The receiver acquires the flag before it reads.
// Epochs only grow (a rank runs at most one call ahead), so a flag is ready once it is at least the
// call's epoch.
__device__ __forceinline__ void st_flag_sys(uint32_t* p, uint32_t v) {
  asm volatile("st.relaxed.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
// Waits until *flag has reached `epoch`; false if that takes longer than the wait limit (recorded in the
// device error word).
__device__ __forceinline__ bool wait_flag(const uint32_t* flag, uint32_t epoch) {
  if (static_cast<int32_t>(ld_acquire_sys(flag) - epoch) >= 0) return true;
  const unsigned long long t0 = global_ns();
  for (;;) {
    __nanosleep(64);
    if (static_cast<int32_t>(ld_acquire_sys(flag) - epoch) >= 0) return true;
    if (global_ns() - t0 > kWaitLimitNs) {
      record_error(Q38_ERR_TIMEOUT);
      return false;
    }
  }
}
template <int W>
__device__ __forceinline__ uint4 add_rows_bf16(const uint4 (&v)[W], const uint4 xr) {
  // bf16(x + bf16(sum of the W partials in rank order, fp32)) for 8 values
  float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
#pragma unroll
  for (int src = 0; src < W; ++src) {
    const __nv_bfloat16* h = reinterpret_cast<const __nv_bfloat16*>(&v[src]);
#pragma unroll
    for (int e = 0; e < 8; ++e) acc[e] = __fadd_rn(acc[e], __bfloat162float(h[e]));
  }
  const __nv_bfloat16* xh = reinterpret_cast<const __nv_bfloat16*>(&xr);
  uint4 o;
  __nv_bfloat16* oh = reinterpret_cast<__nv_bfloat16*>(&o);
#pragma unroll
  for (int e = 0; e < 8; ++e) oh[e] = __float2bfloat16_rn(__fadd_rn(__bfloat162float(xh[e]), bf16r(acc[e])));
  return o;
}

// Sends this rank's staged bf16 partial of token row t (the tile's 128 features, 256 bytes of shared
// memory) to every other rank that owns the row (with two ranks: the other one), into its receive
// slot for this rank at the call's epoch parity, by a bulk copy: the TMA unit moves it over NVLink
// while the threads go on. The issuing thread completes its copies with bulk_commit + bulk_wait0.
__device__ __forceinline__ void push_row(const ArArgs& r, int64_t par, int t, int m0, const __nv_bfloat16* row) {
  for (int dq = 0; dq < r.world; ++dq)
    if (dq != r.rank && (r.world == 2 || t % r.world == dq))
      bulk_store(r.part[dq] + ((par * r.world + r.rank) * r.tmax + t) * r.hidden + m0, row, BM * 2);
}

// Phase 2 of the fused all-reduce for one thread: the rows of [t_begin, t1) that this rank owns (every
// row with two ranks, t % W == rank above), spread over the 8 row lanes of the 128 threads (this
// thread: owned rows row_lane, row_lane + 8, ...), features f .. f + 7. Every source's partial (this
// rank's from the staging tile `sbase`, the others' from this rank's receive slots) is summed in rank
// order, added to the residual, and written to this rank's x and, above two ranks, back into the
// staging tile (over this rank's partial of the row), from where bulk copies take it to every peer's
// x. The loads of U rows are all issued before the first sum: the step is latency-bound otherwise.
template <int W>
__device__ __forceinline__ void reduce_owned_rows(const ArArgs& r, __nv_bfloat16* sbase, int n0, int m0, int f,
                                                  int t_begin, int row_lane, int t1, int64_t par) {
  constexpr int U = W >= 8 ? 2 : (W >= 4 ? 4 : 8);
  const int64_t H = r.hidden;
  const bool one_shot = W == 2;
  const int stride = one_shot ? 1 : W;                                          // between owned rows
  const int base = one_shot ? t_begin : t_begin + ((r.rank - t_begin % W) + W) % W;  // first owned row
  const int t0 = base + row_lane * stride;
  const int tstep = 8 * stride;
  for (int tb = t0; tb < t1; tb += U * tstep) {
    uint4 v[U][W];
    uint4 xr[U];
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int t = tb + u * tstep;
      if (t < t1) {
#pragma unroll
        for (int src = 0; src < W; ++src)
          v[u][src] = src == r.rank ? *reinterpret_cast<const uint4*>(sbase + (t - n0) * BM + (f - m0))
                                    : __ldcg(reinterpret_cast<const uint4*>(
                                          r.part[r.rank] + ((par * W + src) * r.tmax + t) * H + f));
        xr[u] = *reinterpret_cast<const uint4*>(r.x[r.rank] + static_cast<int64_t>(t) * H + f);
      }
    }
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int t = tb + u * tstep;
      if (t >= t1) break;
      const uint4 o = add_rows_bf16<W>(v[u], xr[u]);
      const int64_t at = static_cast<int64_t>(t) * H + f;
      *reinterpret_cast<uint4*>(r.x[r.rank] + at) = o;
      if (!one_shot) *reinterpret_cast<uint4*>(sbase + (t - n0) * BM + (f - m0)) = o;
    }
  }
}

// Applies the bf16 (or bf16 + residual) epilogue to 16 consecutive tokens of one feature row.
// v[j] = sum over slots s < n of p[s * stride + j], j < 16, in slot order from zero (the split-K and
// stream-K partial sums, fp32): the loads of four slots are in flight before the first add, so a chunk
// costs one memory round trip per four slots instead of one per slot.
__device__ __forceinline__ void sum_slots16(const float* p, size_t stride, int n, float (&v)[16]) {
#pragma unroll
  for (int j = 0; j < 16; ++j) v[j] = 0.f;
  for (int s0 = 0; s0 < n; s0 += 4) {
    float4 q[4][4];
#pragma unroll
    for (int u = 0; u < 4; ++u)
      if (s0 + u < n)
#pragma unroll
        for (int j = 0; j < 4; ++j) q[u][j] = __ldcg(reinterpret_cast<const float4*>(p + (s0 + u) * stride) + j);
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      if (s0 + u >= n) break;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        v[4 * j] += q[u][j].x;
        v[4 * j + 1] += q[u][j].y;
        v[4 * j + 2] += q[u][j].z;
        v[4 * j + 3] += q[u][j].w;
      }
    }
  }
}

// The residual rows are all loaded before the first store: y and the residual may be the same buffer
// (the residual stream updated in place), so a load after a store could not be moved ahead of it and
// each token would cost a dependent round trip to memory.
__device__ __forceinline__ void epilogue16(const GemmArgs& a, int row, int t0, const float (&v)[16], int lane) {
  if (row >= a.F) return;
  float res[16];
#pragma unroll
  for (int j = 0; j < 16; ++j)
    res[j] = (a.epilogue == EPI_RESIDUAL && t0 + j < a.T) ? __bfloat162float(a.res[static_cast<int64_t>(t0 + j) * a.ldr + row])
                                                           : 0.f;
#pragma unroll
  for (int j = 0; j < 16; ++j) {
    const int t = t0 + j;
    if (t < a.T) {
      float out = bf16r(v[j]);
      if (a.epilogue == EPI_RESIDUAL) out = res[j] + out;
      a.y[static_cast<int64_t>(t) * a.ldy + row] = __float2bfloat16_rn(out);
    }
  }
}

template <int NTOK, bool MX, bool PAIR>
__global__ void __launch_bounds__(192, 1)
    gemm_kernel(const __grid_constant__ CUtensorMap tmap_x, const __grid_constant__ CUtensorMap tmap_y,
                const __grid_constant__ CUtensorMap tmap_r, const __grid_constant__ CUtensorMap tmap_w,
                const __grid_constant__ CUtensorMap tmap_sf, GemmArgs a) {
  using C = Cfg<NTOK, MX, PAIR>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = smem;
  uint8_t* sB = sA + C::STAGES * C::A_BYTES;
  uint8_t* sSF = sB + C::STAGES * C::B_BYTES;
  uint64_t* full = reinterpret_cast<uint64_t*>(sSF + C::STAGES * C::SF_BYTES);
  uint64_t* empty = full + C::STAGES;
  uint64_t* accf = empty + C::STAGES;
  uint64_t* resbar = accf + 1;
  uint64_t* redbar = resbar + 1;  // split reduction: the other splits' blocks of this CTA's slice
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(redbar + 1);
  volatile int* flags = reinterpret_cast<volatile int*>(tmem_holder + 1);  // [0] abort, [1] last CTA

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int mt = blockIdx.x, nt = blockIdx.y, split = blockIdx.z;
  const uint32_t crank = (a.cluster > 1 || PAIR) ? cluster_rank() : 0u;
  const int prank = PAIR ? static_cast<int>(crank & 1u) : 0;           // 0: the pair's MMA leader
  const int srank = PAIR ? static_cast<int>(crank >> 1) : static_cast<int>(crank);  // K split within the cluster
  const uint16_t pair_mask = static_cast<uint16_t>(3u << (crank & ~1u));
  const int m0 = mt * BM, n0 = nt * NTOK;
  const int kc0 = split * a.kc_per_split;
  const int kc1 = min(a.nkc, kc0 + a.kc_per_split);
  const int nk = kc1 - kc0;

  if (threadIdx.x == 0) {
    for (int s = 0; s < C::STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(accf, 1);
    mbar_init(resbar, 1);
    mbar_init(redbar, 1);
    flags[0] = 0;
    flags[1] = 0;
    fence_mbar_init();
  }
  if (warp == 1) {
    if constexpr (PAIR) {
      tmem_alloc_pair(tmem_holder, C::TMEM_COLS);
      tmem_relinquish_pair();
    } else {
      tmem_alloc(tmem_holder, C::TMEM_COLS);
      tmem_relinquish();
    }
  }
  tc_fence_before();
  if constexpr (PAIR) cluster_sync();  // the peer's copies signal the leader's barriers: all initialised
  else __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_holder;
  if (MX && warp >= 2) {
    // Activation scales are all 1.0 (UE8M0 127) in every lane quarter.
    const int q = warp & 3;
    tmem_st8_fill(tmem + (static_cast<uint32_t>(q * 32) << 16) + C::SFB_COL, 0x7f7f7f7fu);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();

  if (warp == 0) {
    if (lane == 0) {
      prefetch_tmap(&tmap_x);
      // Stage i's weight tile and scales (constant: they may load before the programmatic-launch
      // wait) and its activation tile (after it). Both CTAs of a pair count on the leader's barrier.
      auto load_w = [&](int i) {
        const int s = i % C::STAGES;
        const int tile_id = mt * a.nkc + kc0 + i;
        if constexpr (PAIR) {
          if (prank == 0) mbar_arrive_expect_tx(&full[s], 2 * (C::A_BYTES + C::B_BYTES + C::SF_BYTES));
          tma_load_2d_pair(sA + s * C::A_BYTES, &tmap_w, &full[s], 0, tile_id * BM);
          tma_load_2d_pair(sSF + s * SF_BLOCK, &tmap_sf, &full[s], 0, tile_id * 32);
        } else {
          mbar_arrive_expect_tx(&full[s], C::A_BYTES + C::B_BYTES + C::SF_BYTES);
          bulk_load(sA + s * C::A_BYTES, a.w + static_cast<size_t>(tile_id) * C::A_BYTES, C::A_BYTES, &full[s]);
          if (MX) bulk_load(sSF + s * SF_BLOCK, a.sf + static_cast<size_t>(tile_id) * SF_BLOCK, SF_BLOCK, &full[s]);
        }
      };
      auto load_x = [&](int i) {
        const int s = i % C::STAGES;
        const int kx = (kc0 + i) * (MX ? BK_BYTES : BK_BYTES / 2);  // element coordinate along K
        if constexpr (PAIR) tma_load_2d_pair(sB + s * C::B_BYTES, &tmap_x, &full[s], kx, n0 + prank * C::B_ROWS);
        else tma_load_2d(sB + s * C::B_BYTES, &tmap_x, &full[s], kx, n0);
      };
      // The ring's first pass needs no slot to drain: its weights start before the wait.
      const int pre = min(nk, C::STAGES);
      for (int i = 0; i < pre; ++i) load_w(i);
      pdl_wait();
      for (int i = 0; i < pre; ++i) load_x(i);
      int issued = pre;
      for (int i = pre; i < nk; ++i) {
        const int s = i % C::STAGES;
        const uint32_t ph = (i / C::STAGES) & 1;
        if (flags[0] || !mbar_wait(&empty[s], ph ^ 1)) {
          flags[0] = 1;
          break;
        }
        load_w(i);
        load_x(i);
        issued = i + 1;
      }
      // Never leave with copies in flight: wait (bounded) for the last load of every stage. (A pair's
      // loads are counted on the leader's barriers, which the leader's MMA waits on before it ends.)
      if (!PAIR || prank == 0)
        for (int i = max(0, issued - C::STAGES); i < issued; ++i) mbar_wait(&full[i % C::STAGES], (i / C::STAGES) & 1);
    }
  } else if (warp == 1) {
    if (lane == 0 && (!PAIR || prank == 0)) {
      uint32_t idesc;
      if (MX) {
        idesc = (0u << 7)                                  // A: E4M3
                | (1u << 10)                               // B: E5M2
                | (static_cast<uint32_t>(NTOK >> 3) << 17)  // N
                | (1u << 23)                               // scales UE8M0
                | (static_cast<uint32_t>((PAIR ? 2 * BM : BM) >> 4) << 24);  // M
      } else {
        idesc = (1u << 4)                                  // D: F32
                | (1u << 7) | (1u << 10)                   // A, B: BF16
                | (static_cast<uint32_t>(NTOK >> 3) << 17) | (static_cast<uint32_t>(BM >> 4) << 24);
      }
      for (int i = 0; i < nk; ++i) {
        const int s = i % C::STAGES;
        const uint32_t ph = (i / C::STAGES) & 1;
        if (flags[0] || !mbar_wait(&full[s], ph)) {
          flags[0] = 1;
          break;
        }
        tc_fence_after();
        const uint32_t a_addr = smem_u32(sA + s * C::A_BYTES);
        const uint32_t b_addr = smem_u32(sB + s * C::B_BYTES);
        if constexpr (PAIR) {
          const uint32_t sfa = tmem + C::SFA_COL + 4 * s;
          tmem_cp_32x128b_x4_pair(sfa, sdesc_rows16(smem_u32(sSF + s * SF_BLOCK)));
#pragma unroll
          for (int kk = 0; kk < 4; ++kk) {
            const uint32_t id = idesc | (static_cast<uint32_t>(kk) << 29) | (static_cast<uint32_t>(kk) << 4);
            mma_mxf8_pair(tmem, sdesc_sw128(a_addr + kk * 32), sdesc_sw128(b_addr + kk * 32), id,
                          sfa | (static_cast<uint32_t>(kk) << 30), (tmem + C::SFB_COL) | (static_cast<uint32_t>(kk) << 30),
                          (i | kk) != 0);
          }
        } else if (MX) {
          const uint32_t sfa = tmem + C::SFA_COL + 4 * s;
          tmem_cp_32x128b_x4(sfa, sdesc_rows16(smem_u32(sSF + s * SF_BLOCK)));
#pragma unroll
          for (int kk = 0; kk < 4; ++kk) {
            const uint32_t id = idesc | (static_cast<uint32_t>(kk) << 29) | (static_cast<uint32_t>(kk) << 4);
            mma_mxf8(tmem, sdesc_sw128(a_addr + kk * 32), sdesc_sw128(b_addr + kk * 32), id,
                     sfa | (static_cast<uint32_t>(kk) << 30), (tmem + C::SFB_COL) | (static_cast<uint32_t>(kk) << 30),
                     (i | kk) != 0);
          }
        } else {
#pragma unroll
          for (int kk = 0; kk < 4; ++kk)
            mma_f16(tmem, sdesc_sw128(a_addr + kk * 32), sdesc_sw128(b_addr + kk * 32), idesc, (i | kk) != 0);
        }
        if constexpr (PAIR) tc_commit_pair(&empty[s], pair_mask);
        else tc_commit(&empty[s]);
      }
      if constexpr (PAIR) tc_commit_pair(accf, pair_mask);
      else tc_commit(accf);
    }
    __syncwarp();
  } else if (a.cluster > 0) {
    // Epilogue part 1. With one split the accumulator goes straight to its bf16 staging (the residual
    // tile loading by TMA meanwhile); with a cluster of splits this CTA arms its reduction barrier for
    // the blocks of its slice and drains the blocks it sends to their owners, fp32 [token][row], for
    // part 2.
    const int q = warp & 3;
    const uint32_t taddr = tmem + (static_cast<uint32_t>(q * 32) << 16);
    pdl_wait();
    const bool ok = mbar_wait(accf, 0);
    // The mainloop is done: the next kernel may launch its prologue. Never from the all-reduce, whose
    // CTAs must all find room on the GPU while peers wait on them.
    if (a.epilogue != EPI_ALLREDUCE) pdl_trigger();
    tc_fence_after();
    if (!ok || flags[0]) {
      flags[0] = 1;
    } else {
      fence_proxy_async_shared();
      uint8_t* stage = smem + NTOK * BM * 4;
      if (a.epilogue == EPI_RESIDUAL && a.cluster == 1 && warp == 2 && lane == 0 && m0 < a.F) {
        const int nb = NTOK / TOK_BLOCK;
        const int b0 = 0, b1 = nb;
        int issued = 0;
        for (int b = b0; b < b1; ++b) issued += n0 + b * TOK_BLOCK < a.T;
        mbar_arrive_expect_tx(resbar, issued * TOK_BLOCK * BM * 2);
        for (int b = b0; b < b1; ++b)
          if (n0 + b * TOK_BLOCK < a.T) tma_load_2d(stage + b * TOK_BLOCK * BM * 2, &tmap_r, resbar, m0, n0 + b * TOK_BLOCK);
      }
      const int r = q * 32 + lane;
      if (a.cluster > 1) {
        if (m0 < a.F) {
          const int c = a.cluster, nb = NTOK / TOK_BLOCK;
          const int b0 = srank * nb / c, b1 = (srank + 1) * nb / c;
          if (warp == 2 && lane == 0) {
            int mine = 0;
            for (int b = b0; b < b1; ++b) mine += n0 + b * TOK_BLOCK < a.T;
            if (mine > 0) mbar_arrive_expect_tx(redbar, static_cast<uint32_t>((c - 1) * mine * BLOCK_F32_BYTES));
          }
          float* send = reinterpret_cast<float*>(smem + split_send_offset<NTOK>(c));
          for (int b = 0; b < nb; ++b) {
            if (n0 + b * TOK_BLOCK >= a.T) break;
            if (b >= b0 && b < b1) continue;
            float v[32];
            tmem_ld32(taddr + b * TOK_BLOCK, v);
            float* blk = send + (b < b0 ? b : b - (b1 - b0)) * TOK_BLOCK * BM;
#pragma unroll
            for (int e = 0; e < 32; ++e) blk[e * BM + r] = v[e];
          }
          fence_proxy_async_shared();  // the drained blocks, for the bulk copies
        }
      } else if (m0 < a.F) {
        // Lanes are consecutive rows: a warp's stores of one token fill 64 contiguous bytes.
        if (a.epilogue == EPI_RESIDUAL && !mbar_wait(resbar, 0)) flags[0] = 1;
        __nv_bfloat16* st = reinterpret_cast<__nv_bfloat16*>(stage);
        for (int c = 0; c < NTOK; c += 64) {
          if (n0 + c >= a.T) break;
          float v[64];
          tmem_ld64(taddr + c, v);
#pragma unroll
          for (int j = 0; j < 64; ++j) {
            const int idx = (c + j) * BM + r;
            float out = bf16r(v[j]);
            if (a.epilogue == EPI_RESIDUAL) out = __bfloat162float(st[idx]) + out;
            st[idx] = __float2bfloat16_rn(out);
          }
        }
      }
    }
  } else {
    // Epilogue: warp w reads TMEM lanes 32*(w%4) .. +31 (its hardware lane quarter).
    pdl_wait();
    const int q = warp & 3;
    const int row = m0 + q * 32 + lane;
    const uint32_t taddr = tmem + (static_cast<uint32_t>(q * 32) << 16);
    const bool ok = mbar_wait(accf, 0);
    pdl_trigger();
    tc_fence_after();
    if (!ok || flags[0]) {
      flags[0] = 1;
    } else if (a.splits == 1) {
      for (int c = 0; c < NTOK; c += 64) {
        if (n0 + c >= a.T) break;
        float v[64];
        tmem_ld64(taddr + c, v);
#pragma unroll
        for (int k = 0; k < 64; k += 16) {
          float w[16];
#pragma unroll
          for (int j = 0; j < 16; ++j) w[j] = v[k + j];
          epilogue16(a, row, n0 + c + k, w, lane);
        }
      }
    } else {
      const int tiles = gridDim.x * gridDim.y;
      const int tile = nt * gridDim.x + mt;
      // Partial tile layout [16-token chunk][128 rows][16 tokens]: a warp's 32 rows of one chunk are
      // 2 KB contiguous.
      float* part = a.ws + (static_cast<size_t>(split) * tiles + tile) * BM * NTOK + static_cast<size_t>(q * 32 + lane) * 16;
      for (int c = 0; c < NTOK; c += 64) {
        if (n0 + c >= a.T) break;
        float v[64];
        tmem_ld64(taddr + c, v);
#pragma unroll
        for (int k = 0; k < 64; k += 16) {
          if (n0 + c + k >= a.T) break;
          float* dst = part + static_cast<size_t>((c + k) / 16) * BM * 16;
#pragma unroll
          for (int j = 0; j < 16; j += 4)
            __stcg(reinterpret_cast<float4*>(dst + j), make_float4(v[k + j], v[k + j + 1], v[k + j + 2], v[k + j + 3]));
        }
      }
      __threadfence();
      epi_bar();
      if (warp == 2 && lane == 0) {
        const unsigned prev = atomicAdd(&a.counters[tile], 1u);
        flags[1] = prev == static_cast<unsigned>(a.splits - 1);
      }
      epi_bar();
      if (flags[1]) {
        __threadfence();
        const float* base = a.ws + static_cast<size_t>(tile) * BM * NTOK + static_cast<size_t>(q * 32 + lane) * 16;
        const size_t split_stride = static_cast<size_t>(tiles) * BM * NTOK;
        for (int c = 0; c < NTOK; c += 16) {
          if (n0 + c >= a.T) break;
          float v[16];
          sum_slots16(base + static_cast<size_t>(c / 16) * BM * 16, split_stride, a.splits, v);
          epilogue16(a, row, n0 + c, v, lane);
        }
        if (warp == 2 && lane == 0) a.counters[tile] = 0u;
      }
    }
  }

  __syncwarp();  // the producer and MMA warps reconverge before any aligned barrier
  if (a.cluster > 0) {
    const int nb = NTOK / TOK_BLOCK;
    const int b0 = srank * nb / a.cluster, b1 = (srank + 1) * nb / a.cluster;
    const bool live = m0 < a.F;  // the odd CTA of the last pair may lie past the last row
    uint8_t* stage = smem + (a.cluster > 1 ? split_send_offset<NTOK>(a.cluster) : static_cast<size_t>(NTOK) * BM * 4);
    if (a.cluster > 1) {
      const int c = a.cluster;
      int mine = 0;  // blocks of this CTA's slice that hold tokens
      for (int b = b0; b < b1; ++b) mine += n0 + b * TOK_BLOCK < a.T;
      // Every CTA of the cluster is past its mainloop (its receive buffer is free), has armed its
      // reduction barrier and has drained the blocks it sends.
      cluster_sync();
      // Part 2a: the blocks go to their owners by bulk copies, shared memory to the owner's shared
      // memory, each completing on the owner's reduction barrier (lane b of warp 2 sends block b).
      if (warp == 2 && live && !flags[0]) {
        const int b = lane;
        if (b < nb && !(b >= b0 && b < b1) && n0 + b * TOK_BLOCK < a.T) {
          int o = 0;
          while (b >= (o + 1) * nb / c) ++o;  // the split CTA whose slice holds block b
          const int j = srank < o ? srank : srank - 1;  // this CTA's place among o's sources
          const int ob0 = o * nb / c;
          const uint32_t peer = PAIR ? static_cast<uint32_t>(prank + 2 * o) : static_cast<uint32_t>(o);
          const uint8_t* src = smem + split_send_offset<NTOK>(c) + (b < b0 ? b : b - (b1 - b0)) * BLOCK_F32_BYTES;
          const uint32_t dst = cluster_map(
              smem_u32(smem + (static_cast<size_t>(j) * split_slice_tokens<NTOK>(c) + (b - ob0) * TOK_BLOCK) * BM * 4), peer);
          bulk_copy_cluster(dst, src, BLOCK_F32_BYTES, cluster_map(smem_u32(redbar), peer));
        }
      }
      // Part 2b: the other splits' partials of this CTA's blocks have arrived.
      if (warp >= 2 && live && !flags[0] && mine > 0 && !mbar_wait(redbar, 0)) flags[0] = 1;
      // Every copy out of this CTA has landed at its owner: its send buffers may take the staging.
      cluster_sync();
      // Part 2c: this CTA's slice, summed in split order (its own partial from TMEM), then the epilogue;
      // thread = row, 32 tokens per step. The residual slice loads by TMA meanwhile.
      if (warp >= 2 && !flags[0] && live && mine > 0) {
        if (a.epilogue == EPI_RESIDUAL && warp == 2 && lane == 0) {
          mbar_arrive_expect_tx(resbar, static_cast<uint32_t>(mine * TOK_BLOCK * BM * 2));
          for (int b = b0; b < b1; ++b)
            if (n0 + b * TOK_BLOCK < a.T) tma_load_2d(stage + b * TOK_BLOCK * BM * 2, &tmap_r, resbar, m0, n0 + b * TOK_BLOCK);
        }
        const int q = warp & 3, r = q * 32 + lane;
        const uint32_t taddr = tmem + (static_cast<uint32_t>(q * 32) << 16);
        const float* recv = reinterpret_cast<const float*>(smem);
        const int slice = split_slice_tokens<NTOK>(c);
        __nv_bfloat16* st = reinterpret_cast<__nv_bfloat16*>(stage);
        bool res_ready = a.epilogue != EPI_RESIDUAL;
        for (int b = b0; b < b1; ++b) {
          if (n0 + b * TOK_BLOCK >= a.T) break;
          float acc[32];
#pragma unroll
          for (int e = 0; e < 32; ++e) acc[e] = 0.f;
          for (int src = 0; src < c; ++src) {
            float v[32];
            if (src == srank) {
              tmem_ld32(taddr + b * TOK_BLOCK, v);
            } else {
              const float* p = recv + (static_cast<size_t>(src < srank ? src : src - 1) * slice + (b - b0) * TOK_BLOCK) * BM + r;
#pragma unroll
              for (int e = 0; e < 32; ++e) v[e] = p[e * BM];
            }
#pragma unroll
            for (int e = 0; e < 32; ++e) acc[e] += v[e];
          }
          if (!res_ready) {
            if (!mbar_wait(resbar, 0)) {
              flags[0] = 1;
              break;
            }
            res_ready = true;
          }
#pragma unroll
          for (int e = 0; e < 32; ++e) {
            const int idx = (b * TOK_BLOCK + e) * BM + r;
            float out = bf16r(acc[e]);
            if (a.epilogue == EPI_RESIDUAL) out = __bfloat162float(st[idx]) + out;
            st[idx] = __float2bfloat16_rn(out);
          }
        }
      }
    }
    // The staged bf16 slice goes out by TMA (boxes past the last token or feature are clipped).
    if (warp >= 2 && a.epilogue != EPI_ALLREDUCE) {
      fence_proxy_async_shared();
      epi_bar();
      if (warp == 2 && lane == 0 && !flags[0] && live) {
        for (int b = b0; b < b1; ++b)
          if (n0 + b * TOK_BLOCK < a.T) tma_store_2d(&tmap_y, stage + b * TOK_BLOCK * BM * 2, m0, n0 + b * TOK_BLOCK);
        bulk_commit();
        bulk_wait_read0();
      }
    }
    // Fused all-reduce of the staged bf16 partial, over this CTA's slice of rows [tb0, tb1) x its 128
    // features. Every row has an owner rank that sums every rank's partial of it in rank order (fp32, one
    // bf16 rounding), adds the residual and writes the new row into every rank's residual stream. With two
    // ranks every rank owns every row ("one shot": each pushes its whole partial to the other and both
    // reduce, one crossing of NVLink, no result traffic); with more, row t is owned by rank t % world (each
    // rank pushes (world - 1) / world of its partial and writes 1 / world of the results to each peer: a
    // quarter of the one-shot bytes at 8 ranks). Thread i of the 128 takes the 16-byte pieces
    // (row i / 16 + 8 j, features 8 (i % 16) ..), so a row's 256 bytes go out as one contiguous run.
    if (warp >= 2 && a.epilogue == EPI_ALLREDUCE) {
      const bool failed = epi_bar_or(flags[0] != 0);  // also: the staged partial is complete
      const ArArgs& r = a.ar;
      const int te = threadIdx.x - 64;
      const uint32_t ep = *reinterpret_cast<volatile uint32_t*>(r.epoch);
      const int64_t par = static_cast<int64_t>(ep & 1u);
      const int cta = static_cast<int>(blockIdx.x + gridDim.x * (blockIdx.y + gridDim.y * blockIdx.z));
      const bool one_shot = r.world == 2;
      __nv_bfloat16* sbase = reinterpret_cast<__nv_bfloat16*>(stage);
      const int tb0 = n0 + b0 * TOK_BLOCK;            // first token of the slice
      const int tb1 = min(a.T, n0 + b1 * TOK_BLOCK);  // one past the last
      const int f = m0 + (te & 15) * 8;               // this thread's eight features in phase 2
      const bool mine_f = live && f < a.F;
      bool bad = failed || !live;
      // 1. This rank's partial of every row another rank owns, to that rank: bulk copies of the staged
      //    rows, all complete before the flags go out.
      if (!bad) fence_proxy_async_shared();
      bad = epi_bar_or(bad);
      if (!bad && warp == 2)
        for (int t = tb0 + lane; t < tb1; t += 32) push_row(r, par, t, m0, sbase + (t - n0) * BM);
      bulk_commit();
      bulk_wait0();
      bad = epi_bar_or(bad);
      if (!bad && te < r.world && te != r.rank) st_flag_sys(r.pflag[te] + r.rank * kMaxCtas + cta, ep);
      // 2. The rows this rank owns: every source's partial (acquired through its flag), summed in rank
      //    order, plus the residual; into this rank's x and, for rows others do not own, into theirs.
      if (!bad && te < r.world && te != r.rank) bad = !wait_flag(r.pflag[r.rank] + te * kMaxCtas + cta, ep);
      bad = epi_bar_or(bad);
      if (!bad && mine_f) {
        switch (r.world) {
          case 1: reduce_owned_rows<1>(r, sbase, n0, m0, f, tb0, te >> 4, tb1, par); break;
          case 2: reduce_owned_rows<2>(r, sbase, n0, m0, f, tb0, te >> 4, tb1, par); break;
          case 3: reduce_owned_rows<3>(r, sbase, n0, m0, f, tb0, te >> 4, tb1, par); break;
          case 4: reduce_owned_rows<4>(r, sbase, n0, m0, f, tb0, te >> 4, tb1, par); break;
          case 5: reduce_owned_rows<5>(r, sbase, n0, m0, f, tb0, te >> 4, tb1, par); break;
          case 6: reduce_owned_rows<6>(r, sbase, n0, m0, f, tb0, te >> 4, tb1, par); break;
          case 7: reduce_owned_rows<7>(r, sbase, n0, m0, f, tb0, te >> 4, tb1, par); break;
          default: reduce_owned_rows<8>(r, sbase, n0, m0, f, tb0, te >> 4, tb1, par); break;
        }
      }
      if (!one_shot) {
        // 3. This rank's reduced rows of the slice (now in the staging tile) to every other rank's x by
        //    bulk copies; the other owners' rows have arrived in this rank's x once their flags have.
        if (!bad) fence_proxy_async_shared();
        bad = epi_bar_or(bad);
        if (!bad && warp == 2) {
          const int W = r.world;
          const int base = tb0 + ((r.rank - tb0 % W) + W) % W;  // the slice's first row this rank owns
          for (int t = base + lane * W; t < tb1; t += 32 * W)
            for (int dq = 0; dq < W; ++dq)
              if (dq != r.rank) bulk_store(r.x[dq] + static_cast<int64_t>(t) * r.hidden + m0, sbase + (t - n0) * BM, BM * 2);
        }
        bulk_commit();
        bulk_wait0();
        bad = epi_bar_or(bad);
        if (!bad && te < r.world && te != r.rank) st_flag_sys(r.rflag[te] + r.rank * kMaxCtas + cta, ep);
        if (!bad && te < r.world && te != r.rank) bad = !wait_flag(r.rflag[r.rank] + te * kMaxCtas + cta, ep);
      }
      epi_bar_or(bad);
    }
    // A pair frees its tensor memory together (after the split reduction's second barrier no CTA
    // touches another's shared memory).
    if (PAIR) cluster_sync();
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    if constexpr (PAIR) tmem_dealloc_pair(tmem, C::TMEM_COLS);
    else tmem_dealloc(tmem, C::TMEM_COLS);
  }
  // The last CTA of a fused all-reduce call advances the epoch for the next call (every CTA has read it).
  if (a.epilogue == EPI_ALLREDUCE && threadIdx.x == 0) {
    __threadfence();
    const unsigned total = gridDim.x * gridDim.y * gridDim.z;
    if (atomicAdd(a.ar.done, 1u) == total - 1) {
      *a.ar.done = 0u;
      atomicAdd(a.ar.epoch, 1u);
    }
  }
}

// The group holding linear K step i of W over G groups (group g holds [floor(g W / G), floor((g+1) W / G))).
__host__ __device__ __forceinline__ int sk_group_of(long long i, long long W, int G) {
  return static_cast<int>(((i + 1) * G + W - 1) / W) - 1;
}
// Segment `idx` of group `group`'s work: tile u, K steps [k0, k1). Without stream-K a segment is a whole
// tile (u = group + idx x ngroups); with it, the group's contiguous range cut at tile boundaries.
__device__ __forceinline__ bool seg_at(const GemmArgs& a, int group, int ngroups, int units, int nk, int idx, int& u,
                                       int& k0, int& k1) {
  if (a.sk_groups == 0) {
    u = group + idx * ngroups;
    k0 = 0;
    k1 = nk;
    return u < units;
  }
  const long long W = static_cast<long long>(units) * nk;
  long long i = group * W / a.sk_groups;
  const long long i1 = (group + 1) * W / a.sk_groups;
  for (int s = 0; i < i1; ++s) {
    u = static_cast<int>(i / nk);
    k0 = static_cast<int>(i % nk);
    k1 = static_cast<int>(k0 + (i1 - i < nk - k0 ? i1 - i : nk - k0));
    if (s == idx) return true;
    i += k1 - k0;
  }
  return false;
}
// The groups sharing tile u under stream-K: the first one, and how many (1: the tile is whole).
__device__ __forceinline__ int sk_tile_split(const GemmArgs& a, int u, int units, int nk, int& first) {
  if (a.sk_groups == 0) {
    first = 0;
    return 1;
  }
  const long long W = static_cast<long long>(units) * nk;
  first = sk_group_of(static_cast<long long>(u) * nk, W, a.sk_groups);
  return sk_group_of(static_cast<long long>(u + 1) * nk - 1, W, a.sk_groups) - first + 1;
}

// ---------------------------------------------------------------------------------------------
// Persistent form for unsplit GEMMs (EPI_BF16, EPI_SILU): each CTA (or 2-SM pair) walks output
// tiles, unit u = (weight rows u / n_tiles, token tile u % n_tiles): the token tiles of one weight tile
// go to neighbouring groups at the same time, so the weight tile comes from HBM once and from L2 for
// the others. The producer's stage ring runs on across tiles; the MMA warp waits for "TMEM empty" before a
// tile's first MMA; the epilogue warps drain the accumulator into their own staging buffer, release
// TMEM at once, and store while the next tile's mainloop runs. Per-CTA setup and the pipeline fill
// are paid once per CTA instead of once per tile, and a grid that would take 1.8 waves becomes one
// pass over the tiles.
// ---------------------------------------------------------------------------------------------
template <int NTOK, bool MX, bool PAIR>
struct PCfg {
  static constexpr int A_BYTES = BM * BK_BYTES;
  static constexpr int B_ROWS = PAIR ? NTOK / 2 : NTOK;
  static constexpr int B_BYTES = B_ROWS * BK_BYTES;
  static constexpr int SF_BYTES = MX ? SF_BLOCK : 0;
  static constexpr int STAGES = PAIR ? 4 : 3;  // leaves room for the output staging tile
  static constexpr int TMEM_COLS = NTOK == 256 ? 512 : 256;
  static constexpr int SFA_COL = NTOK;
  static constexpr int SFB_COL = NTOK + 32;
  static constexpr size_t PIPE = STAGES * (A_BYTES + B_BYTES + SF_BYTES);
  // Output staging: bf16 [NTOK tokens][128 rows] (EPI_BF16, stored by TMA), or bf16 [128 rows][SROW
  // tokens] (EPI_SILU: gate rows then up rows, each row padded by 16 bytes so that a warp's 16-byte
  // accesses of 32 rows fall in distinct bank groups).
  static constexpr int SROW = NTOK + 8;
  static constexpr size_t OUT = static_cast<size_t>(BM) * SROW * 2;
  static constexpr size_t SMEM = 1024 + PIPE + OUT + 256;
  static_assert(SFA_COL + 4 * STAGES <= SFB_COL && SFB_COL + 8 <= TMEM_COLS, "TMEM columns");
};

template <int NTOK, bool MX, bool PAIR>
__global__ void __launch_bounds__(192, 1)
    gemm_persistent_kernel(const __grid_constant__ CUtensorMap tmap_x, const __grid_constant__ CUtensorMap tmap_y,
                           const __grid_constant__ CUtensorMap tmap_w, const __grid_constant__ CUtensorMap tmap_sf,
                           GemmArgs a) {
  using C = PCfg<NTOK, MX, PAIR>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = smem;
  uint8_t* sB = sA + C::STAGES * C::A_BYTES;
  uint8_t* sSF = sB + C::STAGES * C::B_BYTES;
  uint8_t* sOut = smem + C::PIPE;
  uint64_t* full = reinterpret_cast<uint64_t*>(sOut + C::OUT);
  uint64_t* empty = full + C::STAGES;
  uint64_t* accf = empty + C::STAGES;
  uint64_t* tmem_empty = accf + 1;
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(tmem_empty + 1);
  volatile int* flags = reinterpret_cast<volatile int*>(tmem_holder + 1);  // [0] abort, [1] last group (stream-K)

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t crank = PAIR ? cluster_rank() : 0u;
  const int prank = PAIR ? static_cast<int>(crank & 1u) : 0;
  const uint16_t pair_mask = static_cast<uint16_t>(3u << (crank & ~1u));
  const int group = PAIR ? static_cast<int>(blockIdx.x >> 1) : static_cast<int>(blockIdx.x);
  const int ngroups = PAIR ? static_cast<int>(gridDim.x >> 1) : static_cast<int>(gridDim.x);
  const int rows_per_unit = PAIR ? 2 * BM : BM;
  const int m_units = (a.F + rows_per_unit - 1) / rows_per_unit;
  const int n_tiles = (a.T + NTOK - 1) / NTOK;
  const int units = m_units * n_tiles;
  const int nk = a.nkc;

  if (threadIdx.x == 0) {
    for (int s = 0; s < C::STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(accf, 1);
    mbar_init(tmem_empty, PAIR ? 2 : 1);
    flags[0] = 0;
    fence_mbar_init();
  }
  if (warp == 1) {
    if constexpr (PAIR) {
      tmem_alloc_pair(tmem_holder, C::TMEM_COLS);
      tmem_relinquish_pair();
    } else {
      tmem_alloc(tmem_holder, C::TMEM_COLS);
      tmem_relinquish();
    }
  }
  tc_fence_before();
  if constexpr (PAIR) cluster_sync();
  else __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_holder;
  if (MX && warp >= 2) tmem_st8_fill(tmem + (static_cast<uint32_t>((warp & 3) * 32) << 16) + C::SFB_COL, 0x7f7f7f7fu);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();

  if (warp == 0) {
    if (lane == 0) {
      prefetch_tmap(&tmap_x);
      // Ring slot `it` for K step i of weight tile mt: the weight tile and scales (constant, so they
      // may load before the programmatic-launch wait), then the activation tile.
      auto load_w = [&](int it, int mt, int i) {
        const int s = it % C::STAGES;
        const int tile_id = mt * a.nkc + i;
        if constexpr (PAIR) {
          if (prank == 0) mbar_arrive_expect_tx(&full[s], 2 * (C::A_BYTES + C::B_BYTES + C::SF_BYTES));
          tma_load_2d_pair(sA + s * C::A_BYTES, &tmap_w, &full[s], 0, tile_id * BM);
          tma_load_2d_pair(sSF + s * SF_BLOCK, &tmap_sf, &full[s], 0, tile_id * 32);
        } else {
          mbar_arrive_expect_tx(&full[s], C::A_BYTES + C::B_BYTES + C::SF_BYTES);
          bulk_load(sA + s * C::A_BYTES, a.w + static_cast<size_t>(tile_id) * C::A_BYTES, C::A_BYTES, &full[s]);
          if (MX) bulk_load(sSF + s * SF_BLOCK, a.sf + static_cast<size_t>(tile_id) * SF_BLOCK, SF_BLOCK, &full[s]);
        }
      };
      auto load_x = [&](int it, int n0, int i) {
        const int s = it % C::STAGES;
        const int kx = i * (MX ? BK_BYTES : BK_BYTES / 2);
        if constexpr (PAIR) tma_load_2d_pair(sB + s * C::B_BYTES, &tmap_x, &full[s], kx, n0 + prank * C::B_ROWS);
        else tma_load_2d(sB + s * C::B_BYTES, &tmap_x, &full[s], kx, n0);
      };
      // The first pass over the ring needs no slot to drain: the first segment's weights go first.
      int pre = 0;
      {
        int u, k0, k1;
        if (seg_at(a, group, ngroups, units, nk, 0, u, k0, k1)) {
          const int mt = PAIR ? 2 * (u / n_tiles) + prank : u / n_tiles;
          pre = min(k1 - k0, C::STAGES);
          for (int i = 0; i < pre; ++i) load_w(i, mt, k0 + i);
        }
      }
      pdl_wait();
      int it = 0;
      int u, k0, k1;
      for (int si = 0; !flags[0] && seg_at(a, group, ngroups, units, nk, si, u, k0, k1); ++si) {
        const int mp = u / n_tiles, nt = u % n_tiles;
        const int mt = PAIR ? 2 * mp + prank : mp;
        const int n0 = nt * NTOK;
        for (int i = k0; i < k1; ++i, ++it) {
          if (it < pre) {
            load_x(it, n0, i);
            continue;
          }
          const int s = it % C::STAGES;
          const uint32_t ph = (it / C::STAGES) & 1;
          if (flags[0] || !mbar_wait(&empty[s], ph ^ 1)) {
            flags[0] = 1;
            break;
          }
          load_w(it, mt, i);
          load_x(it, n0, i);
        }
      }
      // Never leave with copies in flight: wait (bounded) for the last load of every stage.
      if (!PAIR || prank == 0)
        for (int j = max(0, it - C::STAGES); j < it; ++j) mbar_wait(&full[j % C::STAGES], (j / C::STAGES) & 1);
    }
  } else if (warp == 1) {
    if (lane == 0 && (!PAIR || prank == 0)) {
      uint32_t idesc;
      if (MX) {
        idesc = (0u << 7) | (1u << 10) | (static_cast<uint32_t>(NTOK >> 3) << 17) | (1u << 23) |
                (static_cast<uint32_t>((PAIR ? 2 * BM : BM) >> 4) << 24);
      } else {
        idesc = (1u << 4) | (1u << 7) | (1u << 10) | (static_cast<uint32_t>(NTOK >> 3) << 17) |
                (static_cast<uint32_t>(BM >> 4) << 24);
      }
      int it = 0, tc = 0;
      int u, k0, k1;
      for (int si = 0; !flags[0] && seg_at(a, group, ngroups, units, nk, si, u, k0, k1); ++si, ++tc) {
        // The epilogue has drained the previous segment's accumulator.
        if (!mbar_wait(tmem_empty, (tc & 1) ^ 1)) {
          flags[0] = 1;
          break;
        }
        tc_fence_after();
        for (int i = k0; i < k1; ++i, ++it) {
          const int s = it % C::STAGES;
          const uint32_t ph = (it / C::STAGES) & 1;
          if (flags[0] || !mbar_wait(&full[s], ph)) {
            flags[0] = 1;
            break;
          }
          tc_fence_after();
          const uint32_t a_addr = smem_u32(sA + s * C::A_BYTES);
          const uint32_t b_addr = smem_u32(sB + s * C::B_BYTES);
          if constexpr (PAIR) {
            const uint32_t sfa = tmem + C::SFA_COL + 4 * s;
            tmem_cp_32x128b_x4_pair(sfa, sdesc_rows16(smem_u32(sSF + s * SF_BLOCK)));
#pragma unroll
            for (int kk = 0; kk < 4; ++kk) {
              const uint32_t id = idesc | (static_cast<uint32_t>(kk) << 29) | (static_cast<uint32_t>(kk) << 4);
              mma_mxf8_pair(tmem, sdesc_sw128(a_addr + kk * 32), sdesc_sw128(b_addr + kk * 32), id,
                            sfa | (static_cast<uint32_t>(kk) << 30), (tmem + C::SFB_COL) | (static_cast<uint32_t>(kk) << 30),
                            ((i - k0) | kk) != 0);
            }
            tc_commit_pair(&empty[s], pair_mask);
          } else if (MX) {
            const uint32_t sfa = tmem + C::SFA_COL + 4 * s;
            tmem_cp_32x128b_x4(sfa, sdesc_rows16(smem_u32(sSF + s * SF_BLOCK)));
#pragma unroll
            for (int kk = 0; kk < 4; ++kk) {
              const uint32_t id = idesc | (static_cast<uint32_t>(kk) << 29) | (static_cast<uint32_t>(kk) << 4);
              mma_mxf8(tmem, sdesc_sw128(a_addr + kk * 32), sdesc_sw128(b_addr + kk * 32), id,
                       sfa | (static_cast<uint32_t>(kk) << 30), (tmem + C::SFB_COL) | (static_cast<uint32_t>(kk) << 30),
                       ((i - k0) | kk) != 0);
            }
            tc_commit(&empty[s]);
          } else {
#pragma unroll
            for (int kk = 0; kk < 4; ++kk)
              mma_f16(tmem, sdesc_sw128(a_addr + kk * 32), sdesc_sw128(b_addr + kk * 32), idesc, ((i - k0) | kk) != 0);
            tc_commit(&empty[s]);
          }
        }
        if (flags[0]) break;
        if constexpr (PAIR) tc_commit_pair(accf, pair_mask);
        else tc_commit(accf);
      }
    }
    __syncwarp();
  } else {
    // Epilogue: warp w reads TMEM lanes 32*(w%4) .. +31; lane = output row.
    const int q = warp & 3;
    const int r = q * 32 + lane;
    const uint32_t taddr = tmem + (static_cast<uint32_t>(q * 32) << 16);
    __nv_bfloat16* st = reinterpret_cast<__nv_bfloat16*>(sOut);
    pdl_wait();
    int tc = 0;
    int u, k0, k1;
    for (int si = 0; seg_at(a, group, ngroups, units, nk, si, u, k0, k1); ++si, ++tc) {
      const int mp = u / n_tiles, nt = u % n_tiles;
      const int mt = PAIR ? 2 * mp + prank : mp;
      const int m0 = mt * BM, n0 = nt * NTOK;
      const bool ok = !epi_bar_or(!mbar_wait(accf, tc & 1));
      if (!ok) {
        if (threadIdx.x == 64) flags[0] = 1;
        break;
      }
      {
        int nu, nk0, nk1;
        if (!seg_at(a, group, ngroups, units, nk, si + 1, nu, nk0, nk1)) pdl_trigger();  // this CTA's last mainloop
      }
      tc_fence_after();
      if (a.sk_groups > 0) {
        // Stream-K: a whole tile takes its epilogue straight from TMEM; a tile split between groups
        // leaves this group's fp32 partial in its slot of the workspace ([16-token chunk][128 rows][16]:
        // a warp's 32 rows of one chunk are 2 KB contiguous), and the last group to finish the tile sums
        // every slot in K order and applies the epilogue.
        int first;
        const int nseg = sk_tile_split(a, u, units, nk, first);
        const int ctile = nt * (PAIR ? 2 * m_units : m_units) + mt;
        const size_t tile_f = static_cast<size_t>(BM) * NTOK;
        if (nseg == 1) {
          for (int c = 0; c < NTOK; c += 64) {
            if (n0 + c >= a.T) break;
            float v[64];
            tmem_ld64(taddr + c, v);
#pragma unroll
            for (int k = 0; k < 64; k += 16) {
              float w[16];
#pragma unroll
              for (int j = 0; j < 16; ++j) w[j] = v[k + j];
              epilogue16(a, m0 + r, n0 + c + k, w, lane);
            }
          }
          tc_fence_before();
          epi_bar();
          if (threadIdx.x == 64) {
            if constexpr (PAIR) mbar_arrive_cluster(tmem_empty, crank & ~1u);
            else mbar_arrive(tmem_empty);
          }
          continue;
        }
        float* part = a.ws + (static_cast<size_t>(ctile) * a.sk_max_seg + (group - first)) * tile_f + static_cast<size_t>(r) * 16;
        for (int c = 0; c < NTOK; c += 64) {
          if (n0 + c >= a.T) break;
          float v[64];
          tmem_ld64(taddr + c, v);
#pragma unroll
          for (int k = 0; k < 64; k += 16) {
            if (n0 + c + k >= a.T) break;
            float* dst = part + static_cast<size_t>((c + k) / 16) * BM * 16;
#pragma unroll
            for (int j = 0; j < 16; j += 4)
              __stcg(reinterpret_cast<float4*>(dst + j), make_float4(v[k + j], v[k + j + 1], v[k + j + 2], v[k + j + 3]));
          }
        }
        // TMEM back to the MMA warp at once; the partial is published, then counted.
        tc_fence_before();
        epi_bar();
        if (threadIdx.x == 64) {
          if constexpr (PAIR) mbar_arrive_cluster(tmem_empty, crank & ~1u);
          else mbar_arrive(tmem_empty);
        }
        __threadfence();
        epi_bar();
        if (threadIdx.x == 64) {
          const unsigned prev = atomicAdd(&a.counters[ctile], 1u);
          flags[1] = prev == static_cast<unsigned>(nseg - 1);
        }
        epi_bar();
        if (flags[1]) {
          __threadfence();
          const float* base = a.ws + static_cast<size_t>(ctile) * a.sk_max_seg * tile_f + static_cast<size_t>(r) * 16;
          for (int c = 0; c < NTOK; c += 16) {
            if (n0 + c >= a.T) break;
            float v[16];
            sum_slots16(base + static_cast<size_t>(c / 16) * BM * 16, tile_f, nseg, v);
            epilogue16(a, m0 + r, n0 + c, v, lane);
          }
          if (threadIdx.x == 64) a.counters[ctile] = 0u;
        }
        continue;
      }
      // The previous tile's store has finished reading the staging buffer.
      if (threadIdx.x == 64) bulk_wait_read0();
      epi_bar();
      if (a.epilogue == EPI_SILU) {
        // Rows 0..63 of the tile are gate rows, 64..127 the matching up rows (features mt*64 ..): both go
        // to shared memory as bf16 (the reference's gate_proj / up_proj outputs; row r of the tile is
        // row r of the staging, 8 tokens per 16-byte store), TMEM is handed back, then
        // h = bf16(bf16(g * bf16(sigmoid(g))) * u) goes out as e5m2 (down_proj's input rounding). The
        // epilogue is bound by the conversion unit, so bf16 roundings go two per conversion.
        constexpr int SROW = C::SROW;
        uint4* srow = reinterpret_cast<uint4*>(st + r * SROW);
        for (int c = 0; c < NTOK; c += 64) {
          if (n0 + c >= a.T) break;
          float v[64];
          tmem_ld64(taddr + c, v);
#pragma unroll
          for (int j = 0; j < 64; j += 8)
            srow[(c + j) / 8] = make_uint4(pack_bf16x2(v[j], v[j + 1]), pack_bf16x2(v[j + 2], v[j + 3]),
                                           pack_bf16x2(v[j + 4], v[j + 5]), pack_bf16x2(v[j + 6], v[j + 7]));
        }
        tc_fence_before();
        epi_bar();
        if (threadIdx.x == 64) {
          if constexpr (PAIR) mbar_arrive_cluster(tmem_empty, crank & ~1u);
          else mbar_arrive(tmem_empty);
        }
        const int ntv = min(NTOK, a.T - n0);
        const int f0 = mt * 64;
        if (m0 < a.F) {
          // One feature and 8 tokens per thread and step (consecutive lanes, consecutive features: their
          // e5m2 bytes of one token are 32 contiguous bytes); 8 independent chains per thread.
          const int items = (ntv + 7) / 8 * 64;
          for (int idx = threadIdx.x - 64; idx < items; idx += 128) {
            const int f = idx & 63, t0 = (idx >> 6) * 8;
            const uint4 gw = *reinterpret_cast<const uint4*>(st + f * SROW + t0);
            const uint4 uw = *reinterpret_cast<const uint4*>(st + (64 + f) * SROW + t0);
            const uint32_t gp[4] = {gw.x, gw.y, gw.z, gw.w}, up[4] = {uw.x, uw.y, uw.z, uw.w};
            uint8_t* dst = a.yq + static_cast<int64_t>(n0 + t0) * a.ldq + f0 + f;
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              const float2 h = silu_mul_bf16x2(unpack_bf16x2(gp[e]), unpack_bf16x2(up[e]));
              const uint32_t q = __nv_cvt_float2_to_fp8x2(h, __NV_SATFINITE, __NV_E5M2);
              if (t0 + 2 * e < ntv) dst[static_cast<int64_t>(2 * e) * a.ldq] = static_cast<uint8_t>(q & 0xffu);
              if (t0 + 2 * e + 1 < ntv) dst[static_cast<int64_t>(2 * e + 1) * a.ldq] = static_cast<uint8_t>(q >> 8);
            }
          }
        }
        continue;
      }
      for (int c = 0; c < NTOK; c += 64) {
        if (n0 + c >= a.T) break;
        float v[64];
        tmem_ld64(taddr + c, v);
#pragma unroll
        for (int j = 0; j < 64; ++j) st[(c + j) * BM + r] = __float2bfloat16_rn(v[j]);
      }
      // Every TMEM read of this tile is complete: hand the accumulator back to the MMA warp.
      tc_fence_before();
      epi_bar();
      if (threadIdx.x == 64) {
        if constexpr (PAIR) mbar_arrive_cluster(tmem_empty, crank & ~1u);
        else mbar_arrive(tmem_empty);
      }
      fence_proxy_async_shared();
      epi_bar();
      if (threadIdx.x == 64 && m0 < a.F) {
        for (int b = 0; b < NTOK / TOK_BLOCK; ++b)
          if (n0 + b * TOK_BLOCK < a.T) tma_store_2d(&tmap_y, sOut + b * TOK_BLOCK * BM * 2, m0, n0 + b * TOK_BLOCK);
        bulk_commit();
      }
    }
    if (threadIdx.x == 64) bulk_wait_read0();
  }

  __syncwarp();
  tc_fence_before();
  if constexpr (PAIR) cluster_sync();  // the pair frees its tensor memory together
  else __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    if constexpr (PAIR) tmem_dealloc_pair(tmem, C::TMEM_COLS);
    else tmem_dealloc(tmem, C::TMEM_COLS);
  }
}

template <int NTOK, bool MX, bool PAIR>
int launch_persistent(const CUtensorMap& tx, const CUtensorMap& ty, const CUtensorMap& tw, const CUtensorMap& tsf,
                      const GemmArgs& a, cudaStream_t stream) {
  using C = PCfg<NTOK, MX, PAIR>;
  static unsigned long long done_mask = 0;
  static int sms[64] = {0};
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return q38host::cuda_status(e, "cudaGetDevice");
  if (dev >= 64) return q38host::set_error("device ordinal %d too large", dev), Q38_ERR_UNSUPPORTED;
  if (!(done_mask & (1ull << dev))) {
    e = cudaFuncSetAttribute(gemm_persistent_kernel<NTOK, MX, PAIR>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             static_cast<int>(C::SMEM));
    if (e == cudaSuccess) e = cudaDeviceGetAttribute(&sms[dev], cudaDevAttrMultiProcessorCount, dev);
    if (e != cudaSuccess) return q38host::cuda_status(e, "persistent gemm setup");
    done_mask |= 1ull << dev;
  }
  const int rows_per_unit = PAIR ? 2 * BM : BM;
  const int units = static_cast<int>(((a.F + rows_per_unit - 1) / rows_per_unit) * ((a.T + NTOK - 1) / NTOK));
  const int groups = a.sk_groups > 0 ? a.sk_groups : std::min(units, PAIR ? sms[dev] / 2 : sms[dev]);
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(static_cast<unsigned>(PAIR ? 2 * groups : groups), 1, 1);
  cfg.blockDim = dim3(192, 1, 1);
  cfg.dynamicSmemBytes = C::SMEM;
  cfg.stream = stream;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = PAIR ? 2u : 1u;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = q38host::add_pdl(attr, 1);
  e = cudaLaunchKernelEx(&cfg, gemm_persistent_kernel<NTOK, MX, PAIR>, tx, ty, tw, tsf, a);
  return q38host::cuda_status(e != cudaSuccess ? e : cudaGetLastError(), "persistent gemm launch");
}

// `pair_place` (workspace mode, grid.z even): the K splits launch as 2-CTA clusters, which only
// places each pair on the two SMs of one TPC; the kernel uses no cluster feature then.
template <int NTOK, bool MX, bool PAIR = false>
int launch_gemm(const CUtensorMap& tx, const CUtensorMap& ty, const CUtensorMap& tr, const GemmArgs& a, dim3 grid,
                cudaStream_t stream, const CUtensorMap* tw = nullptr, const CUtensorMap* tsf = nullptr,
                bool resident = false, bool pair_place = false) {
  using C = Cfg<NTOK, MX, PAIR>;
  // The split reduction's buffers live in the pipeline buffers.
  if (a.cluster > 1 && split_smem_bytes<NTOK>(a.cluster) > C::PIPE)
    return q38host::set_error("fp8 gemm: the %d-split reduction of %d-token tiles does not fit shared memory", a.cluster, NTOK),
           Q38_ERR_UNSUPPORTED;
  // The shared-memory opt-in is per device; remember which devices have it.
  static unsigned long long done_mask = 0;
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return q38host::cuda_status(e, "cudaGetDevice");
  if (dev < 64 && !(done_mask & (1ull << dev))) {
    e = cudaFuncSetAttribute(gemm_kernel<NTOK, MX, PAIR>, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(C::SMEM));
    if (e != cudaSuccess) return q38host::cuda_status(e, "cudaFuncSetAttribute(gemm)");
    done_mask |= 1ull << dev;
  }
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = grid;
  cfg.blockDim = dim3(192, 1, 1);
  cfg.dynamicSmemBytes = C::SMEM;
  cfg.stream = stream;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = PAIR ? 2u : 1u;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = a.cluster > 1 ? static_cast<unsigned>(a.cluster) : (pair_place && grid.z % 2 == 0 ? 2u : 1u);
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  if (resident) {
    // CTAs that wait on other GPUs must all be running at once: the whole grid has to fit.
    int clusters = 0;
    e = cudaOccupancyMaxActiveClusters(&clusters, gemm_kernel<NTOK, MX, PAIR>, &cfg);
    if (e != cudaSuccess) return q38host::cuda_status(e, "cudaOccupancyMaxActiveClusters");
    const unsigned csize = attr[0].val.clusterDim.x * attr[0].val.clusterDim.z;
    const unsigned need = grid.x * grid.y * grid.z / csize;
    if (static_cast<unsigned>(clusters) < need)
      return q38host::set_error("fused all-reduce: %u clusters of %u CTAs must be resident, the device holds %d", need,
                                csize, clusters),
             Q38_ERR_UNSUPPORTED;
  }
  cfg.numAttrs = q38host::add_pdl(attr, 1);
  e = cudaLaunchKernelEx(&cfg, gemm_kernel<NTOK, MX, PAIR>, tx, ty, tr, tw ? *tw : tx, tsf ? *tsf : tx, a);
  return q38host::cuda_status(e != cudaSuccess ? e : cudaGetLastError(), "gemm launch");
}

int token_tile(int64_t tokens) { return tokens > 128 ? 256 : 128; }

// The token tile for a split reduction over `cluster` K splits in the 1-SM form: a 256-token tile keeps
// its receive and send buffers inside the pipeline buffers only up to 4 splits; above, 128 tokens.
template <bool MX>
int cluster_token_tile(int ntok, int cluster) {
  if (ntok != 256 || cluster <= 1) return ntok;
  return split_smem_bytes<256>(cluster) <= Cfg<256, MX, false>::PIPE ? 256 : 128;
}

int64_t cdiv(int64_t a, int64_t b) { return (a + b - 1) / b; }

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

constexpr int kMaxClusterSplits = 8;  // portable cluster size

// Picks the epilogue: through shared memory and a cluster of the K splits (no workspace) when the
// splits fit a portable cluster and y / residual can be tensor-mapped; else the workspace path.
// Fills the output and residual tensor maps for the cluster path.
// The split-K workspace starts with one counter per output tile, padded to 256 bytes; the fp32
// partials follow.
size_t split_counter_bytes(int64_t tokens, int64_t features) {
  const int64_t tiles = cdiv(features, BM) * cdiv(tokens, token_tile(tokens));
  return static_cast<size_t>((tiles * 4 + 255) / 256 * 256);
}

// The K splits a launch really runs: K stages are dealt out evenly, so asking for more splits than
// ceil(stages / ceil(stages / splits)) gives that many.
int effective_splits(int64_t k, int splits, int k_stage_bytes = BK_BYTES) {
  const int nkc = static_cast<int>(cdiv(k, k_stage_bytes));
  const int kc_per = static_cast<int>(cdiv(nkc, std::min(splits, nkc)));
  return static_cast<int>(cdiv(nkc, kc_per));
}

// Whether y (and the residual, when the epilogue reads one) can be tensor-mapped for the cluster
// epilogue.
bool epilogue_mappable(const void* y, int64_t ldy, const void* residual, int64_t ldr) {
  return aligned16(y) && ldy % 8 == 0 && (!residual || (aligned16(residual) && ldr % 8 == 0));
}

int setup_epilogue(GemmArgs& a, int splits, int64_t tokens, int64_t features, void* y, int64_t ldy,
                   const void* residual, int64_t ldr, void* workspace, size_t workspace_bytes, CUtensorMap* ty,
                   CUtensorMap* tr, const char* who, bool allow_cluster = true) {
  using namespace q38host;
  const bool mappable = epilogue_mappable(y, ldy, residual, ldr);
  if (allow_cluster && splits <= kMaxClusterSplits && mappable) {
    a.cluster = splits;
    int st = encode_tmap_2d(ty, y, tokens, features, 2, TOK_BLOCK, BM, false, ldy);
    if (st != Q38_OK) return st;
    if (residual) {
      st = encode_tmap_2d(tr, residual, tokens, features, 2, TOK_BLOCK, BM, false, ldr);
      if (st != Q38_OK) return st;
    } else {
      *tr = *ty;
    }
    return Q38_OK;
  }
  a.cluster = 0;
  if (splits > 1) {
    const size_t need = q38_fp8_gemm_workspace_bytes(tokens, features, splits);
    if (!workspace || workspace_bytes < need || !aligned16(workspace))
      return set_error("%s: %d K splits need a 16-byte aligned workspace of %zu bytes", who, splits, need), Q38_ERR_ARG;
    a.counters = static_cast<unsigned int*>(workspace);
    a.ws = reinterpret_cast<float*>(static_cast<uint8_t*>(workspace) + split_counter_bytes(tokens, features));
  }
  return Q38_OK;
}

}  // namespace

extern "C" size_t q38_sf_tile_bytes(int64_t features, int64_t k) {
  if (features <= 0 || k <= 0) return 0;
  return static_cast<size_t>(cdiv(features, BM) * cdiv(k, BK_BYTES)) * SF_BLOCK;
}

extern "C" size_t q38_weight_tile_bytes(int64_t features, int64_t row_bytes) {
  if (features <= 0 || row_bytes <= 0) return 0;
  return static_cast<size_t>(cdiv(features, BM) * cdiv(row_bytes, BK_BYTES)) * BM * BK_BYTES;
}

extern "C" size_t q38_fp8_gemm_workspace_bytes(int64_t tokens, int64_t features, int splits) {
  if (tokens <= 0 || features <= 0 || splits <= 1) return 0;
  const int ntok = token_tile(tokens);
  const int64_t tiles = cdiv(features, BM) * cdiv(tokens, ntok);
  return split_counter_bytes(tokens, features) + static_cast<size_t>(splits) * tiles * BM * ntok * sizeof(float);
}

namespace {

// The FP8 GEMM for every epilogue; `ar` (EPI_ALLREDUCE) carries the communicator's device view.
int gemm_fp8(const void* x, int64_t tokens, int64_t k, const void* w, const void* w_sf, int64_t features, int epilogue,
             void* y, int64_t ldy, const void* residual, int64_t ldr, int splits, void* workspace,
             size_t workspace_bytes, const ArArgs* ar, cudaStream_t s, const char* who) {
  using namespace q38host;
  int ntok = token_tile(tokens);
  const int nkc = static_cast<int>(cdiv(k, BK_BYTES));
  splits = effective_splits(k, splits);
  GemmArgs a{};
  a.w = static_cast<const uint8_t*>(w);
  a.sf = static_cast<const uint8_t*>(w_sf);
  a.T = static_cast<int>(tokens);
  a.F = static_cast<int>(features);
  a.nkc = nkc;
  a.splits = splits;
  a.kc_per_split = static_cast<int>(cdiv(nkc, splits));
  a.epilogue = epilogue;
  a.y = static_cast<__nv_bfloat16*>(y);
  a.ldy = ldy;
  a.res = static_cast<const __nv_bfloat16*>(residual);
  a.ldr = ldr;
  if (ar) a.ar = *ar;
  CUtensorMap tx, ty, tr;
  int st = setup_epilogue(a, splits, tokens, features, y, ldy, epilogue == Q38_EPI_RESIDUAL ? residual : nullptr, ldr,
                          workspace, workspace_bytes, &ty, &tr, who);
  if (st != Q38_OK) return st;
  if (ar && a.cluster == 0)
    return set_error("%s: the fused all-reduce takes at most %d K splits", who, kMaxClusterSplits), Q38_ERR_UNSUPPORTED;
  if (!(ntok == 256 && 2 * a.cluster <= kMaxClusterSplits && features > BM)) ntok = cluster_token_tile<true>(ntok, a.cluster);
  st = encode_tmap_2d(&tx, x, tokens, k, 1, ntok, BK_BYTES);
  if (st != Q38_OK) return st;
  if (a.cluster == 0) ty = tr = tx;
  const bool resident = ar != nullptr;
  // The exchange's flags hold one slot per CTA of the launch (the 2-SM form rounds the tiles up to pairs).
  if (ar && 2 * cdiv(features, 2 * BM) * cdiv(tokens, ntok) * splits > kMaxCtas)
    return set_error("%s: %lld tokens x %lld features x %d splits need more than %d CTAs", who, (long long)tokens,
                     (long long)features, splits, kMaxCtas),
           Q38_ERR_UNSUPPORTED;
  // Unsplit bf16 outputs take the persistent tile loop.
  const bool persistent = ar == nullptr && epilogue == Q38_EPI_BF16 && a.cluster == 1;
  // The 2-SM form for full 256-token tiles whose cluster (2 x splits) stays portable.
  if (ntok == 256 && a.cluster > 0 && 2 * a.cluster <= kMaxClusterSplits && features > BM) {
    // Each CTA of a pair loads half of the 256-token tile: the activation box is 128 rows.
    st = encode_tmap_2d(&tx, x, tokens, k, 1, Cfg<256, true, true>::B_ROWS, BK_BYTES);
    if (st != Q38_OK) return st;
    CUtensorMap tw, tsf;
    const int64_t tiles = cdiv(features, BM) * nkc;
    st = encode_tmap_2d(&tw, w, tiles * BM, BK_BYTES, 1, BM, BK_BYTES, false);
    if (st != Q38_OK) return st;
    st = encode_tmap_2d(&tsf, w_sf, tiles * 32, 16, 1, 32, 16, false);
    if (st != Q38_OK) return st;
    if (persistent) return launch_persistent<256, true, true>(tx, ty, tw, tsf, a, s);
    dim3 grid(static_cast<unsigned>(2 * cdiv(features, 2 * BM)), static_cast<unsigned>(cdiv(tokens, ntok)),
              static_cast<unsigned>(splits));
    return launch_gemm<256, true, true>(tx, ty, tr, a, grid, s, &tw, &tsf, resident);
  }
  if (persistent)
    return ntok == 256 ? launch_persistent<256, true, false>(tx, ty, tx, tx, a, s)
                       : launch_persistent<128, true, false>(tx, ty, tx, tx, a, s);
  dim3 grid(static_cast<unsigned>(cdiv(features, BM)), static_cast<unsigned>(cdiv(tokens, ntok)), static_cast<unsigned>(splits));
  return ntok == 256 ? launch_gemm<256, true>(tx, ty, tr, a, grid, s, nullptr, nullptr, resident)
                     : launch_gemm<128, true>(tx, ty, tr, a, grid, s, nullptr, nullptr, resident);
}

int check_gemm_args(const void* x, int64_t tokens, int64_t k, const void* w, const void* w_sf, int64_t features,
                    int splits, const char* who) {
  using namespace q38host;
  if (!x || !w || !w_sf) return set_error("%s: null pointer", who), Q38_ERR_ARG;
  if (tokens <= 0 || k <= 0 || features <= 0 || tokens > (1 << 24) || features > (1 << 30) || k > (1 << 30))
    return set_error("%s: bad sizes tokens=%lld k=%lld features=%lld", who, (long long)tokens, (long long)k,
                     (long long)features),
           Q38_ERR_ARG;
  if (k % 16 != 0 || !aligned16(x) || !aligned16(w) || !aligned16(w_sf))
    return set_error("%s: k must be a multiple of 16 and x, w, w_sf 16-byte aligned", who), Q38_ERR_ARG;
  if (splits < 1) return set_error("%s: splits must be >= 1", who), Q38_ERR_ARG;
  return Q38_OK;
}

// Every check of q38_fp8_gemm's arguments that needs no workspace.
int check_fp8_gemm_call(const void* x, int64_t tokens, int64_t k, const void* w, const void* w_sf, int64_t features,
                        int epilogue, const void* y, int64_t ldy, const void* residual, int64_t ldr, int splits,
                        const char* who) {
  using namespace q38host;
  int st = check_gemm_args(x, tokens, k, w, w_sf, features, splits, who);
  if (st != Q38_OK) return st;
  if (!y) return set_error("%s: null pointer", who), Q38_ERR_ARG;
  if (epilogue != Q38_EPI_BF16 && epilogue != Q38_EPI_RESIDUAL)
    return set_error("%s: unknown epilogue %d", who, epilogue), Q38_ERR_ARG;
  if (epilogue == Q38_EPI_RESIDUAL && !residual) return set_error("%s: residual epilogue needs residual", who), Q38_ERR_ARG;
  if (ldy < features || (residual && ldr < features)) return set_error("%s: leading dimension too small", who), Q38_ERR_ARG;
  return Q38_OK;
}

}  // namespace

extern "C" int q38_fp8_gemm(const void* x, int64_t tokens, int64_t k, const void* w, const void* w_sf,
                            int64_t features, int epilogue, void* y, int64_t ldy, const void* residual, int64_t ldr,
                            int splits, void* workspace, size_t workspace_bytes, q38_stream_t stream) {
  using namespace q38host;
  const int st = check_fp8_gemm_call(x, tokens, k, w, w_sf, features, epilogue, y, ldy, residual, ldr, splits,
                                     "q38_fp8_gemm");
  if (st != Q38_OK) return st;
  return gemm_fp8(x, tokens, k, w, w_sf, features, epilogue, y, ldy, residual, ldr, splits, workspace, workspace_bytes,
                  nullptr, static_cast<cudaStream_t>(stream), "q38_fp8_gemm");
}

extern "C" int q38_fp8_gemm_allreduce(const void* x, int64_t tokens, int64_t k, const void* w, const void* w_sf,
                                      int64_t features, int splits, void* comm, q38_stream_t stream) {
  using namespace q38host;
  int st = check_gemm_args(x, tokens, k, w, w_sf, features, splits, "q38_fp8_gemm_allreduce");
  if (st != Q38_OK) return st;
  const Comm* c = static_cast<const Comm*>(comm);
  if (!c || !c->connected) return set_error("q38_fp8_gemm_allreduce: communicator not connected"), Q38_ERR_ARG;
  if (features != c->hidden || tokens > c->tmax)
    return set_error("q38_fp8_gemm_allreduce: output [%lld, %lld] does not fit the communicator's [%lld, %lld]",
                     (long long)tokens, (long long)features, (long long)c->tmax, (long long)c->hidden),
           Q38_ERR_ARG;
  const ArArgs ar = ar_args(*c);
  void* y = c->base + c->off_x;
  return gemm_fp8(x, tokens, k, w, w_sf, features, EPI_ALLREDUCE, y, c->hidden, nullptr, 0, splits, nullptr, 0, &ar,
                  static_cast<cudaStream_t>(stream), "q38_fp8_gemm_allreduce");
}

extern "C" int q38_fp8_gemm_silu(const void* x, int64_t tokens, int64_t k, const void* w, const void* w_sf,
                                 int64_t features, void* y, int64_t ldy, q38_stream_t stream) {
  using namespace q38host;
  int st = check_gemm_args(x, tokens, k, w, w_sf, features, 1, "q38_fp8_gemm_silu");
  if (st != Q38_OK) return st;
  if (!y) return set_error("q38_fp8_gemm_silu: null output"), Q38_ERR_ARG;
  if (features % BM != 0 || ldy < features / 2 || ldy % 8 != 0 || (reinterpret_cast<uintptr_t>(y) & 7u) != 0)
    return set_error("q38_fp8_gemm_silu: rows must be a multiple of 128 (64 gate + 64 up per tile), ldy >= rows / 2 "
                     "and a multiple of 8, y 8-byte aligned"),
           Q38_ERR_ARG;
  const int ntok = token_tile(tokens);
  GemmArgs a{};
  a.w = static_cast<const uint8_t*>(w);
  a.sf = static_cast<const uint8_t*>(w_sf);
  a.T = static_cast<int>(tokens);
  a.F = static_cast<int>(features);
  a.nkc = static_cast<int>(cdiv(k, BK_BYTES));
  a.splits = 1;
  a.kc_per_split = a.nkc;
  a.epilogue = EPI_SILU;
  a.cluster = 1;
  a.yq = static_cast<uint8_t*>(y);
  a.ldq = ldy;
  CUtensorMap tx;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (ntok == 256 && features > BM) {
    st = encode_tmap_2d(&tx, x, tokens, k, 1, Cfg<256, true, true>::B_ROWS, BK_BYTES);
    if (st != Q38_OK) return st;
    CUtensorMap tw, tsf;
    const int64_t tiles = cdiv(features, BM) * a.nkc;
    st = encode_tmap_2d(&tw, w, tiles * BM, BK_BYTES, 1, BM, BK_BYTES, false);
    if (st != Q38_OK) return st;
    st = encode_tmap_2d(&tsf, w_sf, tiles * 32, 16, 1, 32, 16, false);
    if (st != Q38_OK) return st;
    return launch_persistent<256, true, true>(tx, tx, tw, tsf, a, s);
  }
  st = encode_tmap_2d(&tx, x, tokens, k, 1, ntok, BK_BYTES);
  if (st != Q38_OK) return st;
  return ntok == 256 ? launch_persistent<256, true, false>(tx, tx, tx, tx, a, s)
                     : launch_persistent<128, true, false>(tx, tx, tx, tx, a, s);
}

extern "C" int q38_bf16_linear(const void* x, int64_t ldx, int64_t rows, int64_t k, const void* w, int64_t n_out,
                               void* y, int64_t ldy, int splits, void* workspace, size_t workspace_bytes,
                               q38_stream_t stream) {
  using namespace q38host;
  if (!x || !w || !y) return set_error("q38_bf16_linear: null pointer"), Q38_ERR_ARG;
  if (rows <= 0 || k <= 0 || n_out <= 0 || k % 8 || ldx != k || ldy < n_out || rows > (1 << 24) || n_out > (1 << 30))
    return set_error("q38_bf16_linear: bad sizes (x must be contiguous [rows, k], k %% 8 == 0)"), Q38_ERR_ARG;
  if (!aligned16(x) || !aligned16(w) || splits < 1)
    return set_error("q38_bf16_linear: x and w must be 16-byte aligned, splits >= 1"), Q38_ERR_ARG;
  // A thin output (one 128-row tile, e.g. in_proj_b/a's 96) gets 128-token tiles: twice the CTAs,
  // each streaming half the activations.
  int ntok = n_out <= BM ? 128 : token_tile(rows);
  const int nkc = static_cast<int>(cdiv(k, BK_BYTES / 2));
  const int kc_per = static_cast<int>(cdiv(nkc, std::min(splits, nkc)));
  splits = static_cast<int>(cdiv(nkc, kc_per));
  GemmArgs a{};
  a.w = static_cast<const uint8_t*>(w);
  a.T = static_cast<int>(rows);
  a.F = static_cast<int>(n_out);
  a.nkc = nkc;
  a.splits = splits;
  a.kc_per_split = kc_per;
  a.epilogue = EPI_BF16;
  a.y = static_cast<__nv_bfloat16*>(y);
  a.ldy = ldy;
  // Given a workspace, the split partials go through it: the CTAs need no K-split cluster and run on
  // whichever SMs are free (beside another kernel on a second stream, say), launched in 2-CTA
  // clusters so each pair takes a whole TPC and leaves whole TPCs to 2-SM kernels. Without one, the
  // splits of a tile form a cluster and sum through shared memory. Both sum the fp32 partials in
  // split order 0..S-1 from zero: the same bits either way.
  const bool via_workspace = splits > 1 && workspace != nullptr;
  CUtensorMap tx, ty, tr;
  int st = setup_epilogue(a, splits, rows, n_out, y, ldy, nullptr, 0, workspace, workspace_bytes, &ty, &tr,
                          "q38_bf16_linear", !via_workspace);
  if (st != Q38_OK) return st;
  ntok = cluster_token_tile<false>(ntok, a.cluster);
  st = encode_tmap_2d(&tx, x, rows, k, 2, ntok, BK_BYTES / 2);
  if (st != Q38_OK) return st;
  if (a.cluster == 0) ty = tr = tx;
  dim3 grid(static_cast<unsigned>(cdiv(n_out, BM)), static_cast<unsigned>(cdiv(rows, ntok)), static_cast<unsigned>(splits));
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  return ntok == 256 ? launch_gemm<256, false>(tx, ty, tr, a, grid, s, nullptr, nullptr, false, via_workspace)
                     : launch_gemm<128, false>(tx, ty, tr, a, grid, s, nullptr, nullptr, false, via_workspace);
}

// ------------------------------------------------------------------------------------------------
// q38_fp8_gemm_streamk: the persistent kernel with stream-K work division.
// ------------------------------------------------------------------------------------------------
namespace {

struct StreamKPlan {
  int ntok = 0;
  bool pair = false;
  int units = 0, nk = 0, groups = 0, ctiles = 0, max_seg = 0;
  size_t counter_bytes = 0, bytes = 0;
};

// The same plan for the size query and the launch: tiles of 128 (256 as a 2-SM pair) weight rows x
// 128 or 256 tokens, the K steps of all tiles divided evenly over one group per SM (pair); `max_seg`
// is the most groups any tile is split between, the workspace's slots per 128-row tile.
int streamk_plan(int64_t tokens, int64_t features, int64_t k, StreamKPlan* p) {
  using namespace q38host;
  int dev = 0, sms = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e == cudaSuccess) e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  if (e != cudaSuccess) return cuda_status(e, "stream-K plan: SM count");
  p->ntok = token_tile(tokens);
  p->pair = p->ntok == 256 && features > BM;
  const int64_t rows = p->pair ? 2 * BM : BM;
  const int64_t m_units = cdiv(features, rows), n_tiles = cdiv(tokens, p->ntok);
  p->units = static_cast<int>(m_units * n_tiles);
  p->nk = static_cast<int>(cdiv(k, BK_BYTES));
  const long long W = static_cast<long long>(p->units) * p->nk;
  p->groups = static_cast<int>(std::min<long long>(W, p->pair ? sms / 2 : sms));
  p->ctiles = static_cast<int>((p->pair ? 2 * m_units : m_units) * n_tiles);
  p->max_seg = 1;
  for (int u = 0; u < p->units; ++u) {
    const int first = sk_group_of(static_cast<long long>(u) * p->nk, W, p->groups);
    const int last = sk_group_of(static_cast<long long>(u + 1) * p->nk - 1, W, p->groups);
    p->max_seg = std::max(p->max_seg, last - first + 1);
  }
  p->counter_bytes = (static_cast<size_t>(p->ctiles) * 4 + 255) / 256 * 256;
  p->bytes = p->counter_bytes + static_cast<size_t>(p->ctiles) * p->max_seg * BM * p->ntok * sizeof(float);
  return Q38_OK;
}

}  // namespace

extern "C" size_t q38_fp8_gemm_streamk_workspace_bytes(int64_t tokens, int64_t features, int64_t k) {
  if (tokens <= 0 || features <= 0 || k <= 0 || tokens > (1 << 24) || features > (1 << 30) || k > (1 << 30)) return 0;
  StreamKPlan p;
  return streamk_plan(tokens, features, k, &p) == Q38_OK ? p.bytes : 0;
}

extern "C" int q38_fp8_gemm_streamk(const void* x, int64_t tokens, int64_t k, const void* w, const void* w_sf,
                                    int64_t features, int epilogue, void* y, int64_t ldy, const void* residual,
                                    int64_t ldr, void* workspace, size_t workspace_bytes, q38_stream_t stream) {
  using namespace q38host;
  const char* who = "q38_fp8_gemm_streamk";
  int st = check_fp8_gemm_call(x, tokens, k, w, w_sf, features, epilogue, y, ldy, residual, ldr, 1, who);
  if (st != Q38_OK) return st;
  StreamKPlan p;
  st = streamk_plan(tokens, features, k, &p);
  if (st != Q38_OK) return st;
  if (!workspace || workspace_bytes < p.bytes || !aligned16(workspace))
    return set_error("%s: needs a 16-byte aligned, zero-initialised workspace of %zu bytes", who, p.bytes), Q38_ERR_ARG;
  GemmArgs a{};
  a.w = static_cast<const uint8_t*>(w);
  a.sf = static_cast<const uint8_t*>(w_sf);
  a.T = static_cast<int>(tokens);
  a.F = static_cast<int>(features);
  a.nkc = p.nk;
  a.splits = 1;
  a.kc_per_split = p.nk;
  a.epilogue = epilogue;
  a.y = static_cast<__nv_bfloat16*>(y);
  a.ldy = ldy;
  a.res = static_cast<const __nv_bfloat16*>(residual);
  a.ldr = ldr;
  a.cluster = 1;
  a.counters = static_cast<unsigned int*>(workspace);
  a.ws = reinterpret_cast<float*>(static_cast<uint8_t*>(workspace) + p.counter_bytes);
  a.sk_groups = p.groups;
  a.sk_max_seg = p.max_seg;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  CUtensorMap tx;
  if (p.pair) {
    st = encode_tmap_2d(&tx, x, tokens, k, 1, PCfg<256, true, true>::B_ROWS, BK_BYTES);
    if (st != Q38_OK) return st;
    CUtensorMap tw, tsf;
    const int64_t tiles = cdiv(features, BM) * a.nkc;
    st = encode_tmap_2d(&tw, w, tiles * BM, BK_BYTES, 1, BM, BK_BYTES, false);
    if (st != Q38_OK) return st;
    st = encode_tmap_2d(&tsf, w_sf, tiles * 32, 16, 1, 32, 16, false);
    if (st != Q38_OK) return st;
    return launch_persistent<256, true, true>(tx, tx, tw, tsf, a, s);
  }
  st = encode_tmap_2d(&tx, x, tokens, k, 1, p.ntok, BK_BYTES);
  if (st != Q38_OK) return st;
  return p.ntok == 256 ? launch_persistent<256, true, false>(tx, tx, tx, tx, a, s)
                       : launch_persistent<128, true, false>(tx, tx, tx, tx, a, s);
}

// ------------------------------------------------------------------------------------------------
// q38_fp8_gemm_static_scratch: the same GEMM for callers that cannot allocate device memory.
//
// Some callers cannot hand this library a workspace: a host whose device memory belongs to a
// framework pool that allows no allocations of its own, a plugin that must not synchronise the
// device (cudaMalloc and cudaFree do), or a thin binding (ctypes, cgo, JNI) that carries device
// pointers for inputs and outputs but has no allocator. For them the split-K partial sums live in a
// fixed array compiled into the library, Q38_STATIC_SCRATCH_BYTES per GPU, which every GPU that
// loads the library keeps until the process exits.
// ------------------------------------------------------------------------------------------------
#include <mutex>

namespace {

static __device__ __align__(256) uint8_t g_static_scratch[Q38_STATIC_SCRATCH_BYTES];

std::mutex g_static_scratch_mutex;
void* g_static_scratch_ptr[64] = {nullptr};

// The array's device address on the current device, looked up once per device. In host code the
// array's name is only a host-side stand-in, so the address must come from cudaGetSymbolAddress.
int static_scratch_address(void** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return q38host::cuda_status(e, "cudaGetDevice");
  if (dev < 0 || dev >= 64) return q38host::set_error("device %d out of range", dev), Q38_ERR_ARG;
  std::lock_guard<std::mutex> lock(g_static_scratch_mutex);
  if (!g_static_scratch_ptr[dev]) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_static_scratch);
    if (e != cudaSuccess) return q38host::cuda_status(e, "cudaGetSymbolAddress(static scratch)");
    g_static_scratch_ptr[dev] = p;
  }
  *out = g_static_scratch_ptr[dev];
  return Q38_OK;
}

}  // namespace

extern "C" int q38_fp8_gemm_static_scratch(const void* x, int64_t tokens, int64_t k, const void* w, const void* w_sf,
                                           int64_t features, int epilogue, void* y, int64_t ldy, const void* residual,
                                           int64_t ldr, int splits, q38_stream_t stream) {
  using namespace q38host;
  const char* who = "q38_fp8_gemm_static_scratch";
  // Every argument is checked before the fixed array is touched.
  int st = check_fp8_gemm_call(x, tokens, k, w, w_sf, features, epilogue, y, ldy, residual, ldr, splits, who);
  if (st != Q38_OK) return st;
  // Only the workspace epilogue (more than 8 K splits, or an output or residual that cannot be
  // tensor-mapped) uses scratch; every other call runs exactly as q38_fp8_gemm without one.
  const int runs = effective_splits(k, splits);
  const void* res = epilogue == Q38_EPI_RESIDUAL ? residual : nullptr;
  if (runs == 1 || (runs <= kMaxClusterSplits && epilogue_mappable(y, ldy, res, ldr)))
    return q38_fp8_gemm(x, tokens, k, w, w_sf, features, epilogue, y, ldy, residual, ldr, splits, nullptr, 0, stream);
  const size_t need = q38_fp8_gemm_workspace_bytes(tokens, features, runs);
  if (need > static_cast<size_t>(Q38_STATIC_SCRATCH_BYTES))
    return set_error("%s: %lld tokens x %lld features with %d splits need %zu bytes of scratch, more than the "
                     "library's fixed %d; use fewer splits or q38_fp8_gemm with a workspace",
                     who, (long long)tokens, (long long)features, runs, need, Q38_STATIC_SCRATCH_BYTES),
           Q38_ERR_ARG;
  void* scratch = nullptr;
  st = static_scratch_address(&scratch);
  if (st != Q38_OK) return st;
  // The split counters must start at zero. A completed call leaves them at zero, but a call that
  // gave up part-way would not, so clear them (a memset node, no allocation) before every call.
  cudaError_t e = cudaMemsetAsync(scratch, 0, split_counter_bytes(tokens, features), static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_status(e, "clear static scratch counters");
  return q38_fp8_gemm(x, tokens, k, w, w_sf, features, epilogue, y, ldy, residual, ldr, runs, scratch,
                      static_cast<size_t>(Q38_STATIC_SCRATCH_BYTES), stream);
}

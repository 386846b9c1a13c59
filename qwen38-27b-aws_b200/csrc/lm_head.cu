// The lm_head's candidate search: logits = x @ W^T over one rank's vocabulary slice and the largest
// logit of every group of 32 vocabulary rows, for every batch row (qwen38_inf2/model.py:890-900, the
// NKI lm_head_group_maxima kernels.py:126-172). The logits never leave the chip: each group's maximum
// is reduced straight out of tensor memory.
//
// At decode batch sizes this is the step's largest single weight stream (vocab x hidden BF16, 2.5 GB
// for the full model) and, at 256 rows, also a dense BF16 contraction of the same duration, so the
// kernel is built to keep both the copy engines and the tensor cores busy:
//   * persistent CTA pairs (cta_group::2): one MMA covers 256 vocabulary rows x NTOK batch rows, each
//     SM of the pair loading its own 128 weight rows and half of the batch rows, so the activations
//     are read once per 256 vocabulary rows instead of once per 128;
//   * 6-10 pipeline stages (no output staging tile is needed), enough bytes in flight to cover HBM
//     latency at full bandwidth;
//   * two TMEM accumulators: the group-max epilogue of one tile runs while the MMAs of the next tile
//     accumulate into the other;
//   * the 32-row maximum as a transpose-reduce across the warp (31 shuffles per 32 columns), whose
//     lane j ends with column j's maximum and stores it.
// Weights are the BF16 linear's pre-tiled 16 KB swizzled tiles (codec.tile_weight): tile (mt, kc)
// holds rows mt*128.. and K elements kc*64...
#include <algorithm>

#include "q38_common.cuh"

namespace {

using namespace q38;

constexpr int BM = 128;           // vocabulary rows per CTA (the pair covers 256)
constexpr int BK_BYTES = 128;     // one 128-byte swizzle row: 64 BF16 values of K per stage
constexpr int KSTEP = BK_BYTES / 2;

template <int NTOK>
struct HCfg {
  static constexpr int A_BYTES = BM * BK_BYTES;
  static constexpr int B_ROWS = NTOK / 2;  // batch rows loaded by each CTA of the pair
  static constexpr int B_BYTES = B_ROWS * BK_BYTES;
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
  static constexpr int STAGES = std::min(10, (200 * 1024) / STAGE_BYTES);
  static constexpr int TMEM_COLS = 2 * NTOK;  // two fp32 accumulators of NTOK columns
  static constexpr size_t SMEM = 1024 + static_cast<size_t>(STAGES) * STAGE_BYTES + 256;
  static_assert(TMEM_COLS >= 32 && TMEM_COLS <= 512 && (TMEM_COLS & (TMEM_COLS - 1)) == 0, "TMEM columns");
  static_assert(B_ROWS % 8 == 0, "swizzle atoms are 8 rows");
};

struct HeadArgs {
  int T;        // batch rows
  int F;        // vocabulary rows (a multiple of 32)
  int nkc;      // K steps of 64
  int tiles;    // 128-row weight tiles
  float* maxima;
  int64_t ldm;
};

__device__ __forceinline__ void mma_f16_pair(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                             uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// v[c] is lane i's value of column c (i = a vocabulary row of the group, c = a batch row). Returns,
// in lane j, the maximum over all 32 lanes of column j: each halving step trades the half of the
// columns this lane gives up for its partner's copy of the half it keeps (16 + 8 + 4 + 2 + 1 shuffles).
__device__ __forceinline__ float transpose_max32(float (&v)[32], int lane) {
#pragma unroll
  for (int w = 16; w >= 1; w >>= 1) {
    const bool hi = (lane & w) != 0;
#pragma unroll
    for (int k = 0; k < w; ++k) {
      const float give = hi ? v[k] : v[k + w];
      const float keep = hi ? v[k + w] : v[k];
      v[k] = fmaxf(keep, __shfl_xor_sync(0xffffffffu, give, w));
    }
  }
  return v[0];
}

template <int NTOK>
__global__ void __launch_bounds__(192, 1)
    lm_head_kernel(const __grid_constant__ CUtensorMap tmap_x, const __grid_constant__ CUtensorMap tmap_w,
                   HeadArgs a) {
  using C = HCfg<NTOK>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = smem;
  uint8_t* sB = sA + C::STAGES * C::A_BYTES;
  uint64_t* full = reinterpret_cast<uint64_t*>(sB + C::STAGES * C::B_BYTES);
  uint64_t* empty = full + C::STAGES;
  uint64_t* accf = empty + C::STAGES;  // [2] accumulator b is complete
  uint64_t* tmem_empty = accf + 2;     // [2] accumulator b has been read by all 8 epilogue warps of the pair
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(tmem_empty + 2);
  volatile int* flags = reinterpret_cast<volatile int*>(tmem_holder + 1);  // [0] abort

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t crank = cluster_rank();
  const int prank = static_cast<int>(crank & 1u);
  const uint16_t pair_mask = static_cast<uint16_t>(3u << (crank & ~1u));
  const int group = static_cast<int>(blockIdx.x >> 1);
  const int ngroups = static_cast<int>(gridDim.x >> 1);
  const int m_units = (a.tiles + 1) / 2;
  const int n_tiles = (a.T + NTOK - 1) / NTOK;
  const int units = m_units * n_tiles;  // unit u: weight pair u / n_tiles, batch tile u % n_tiles
  const int nk = a.nkc;

  if (threadIdx.x == 0) {
    for (int s = 0; s < C::STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&accf[b], 1);
      mbar_init(&tmem_empty[b], 8);
    }
    flags[0] = 0;
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc_pair(tmem_holder, C::TMEM_COLS);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  cluster_sync();
  tc_fence_after();
  const uint32_t tmem = *tmem_holder;

  if (warp == 0) {
    if (lane == 0) {
      prefetch_tmap(&tmap_x);
      prefetch_tmap(&tmap_w);
      // Both CTAs' bytes land on the leader's barrier. A weight tile past the vocabulary (odd tile
      // count) reads as zeros and its groups are never stored. The first unit's first ring pass of
      // weights (constant) starts before the programmatic-launch wait; activations follow it.
      auto load_w = [&](int it, int mt, int i) {
        const int s = it % C::STAGES;
        if (prank == 0) mbar_arrive_expect_tx(&full[s], 2 * C::STAGE_BYTES);
        tma_load_2d_pair(sA + s * C::A_BYTES, &tmap_w, &full[s], 0, (mt * nk + i) * BM);
      };
      auto load_x = [&](int it, int n0, int i) {
        const int s = it % C::STAGES;
        tma_load_2d_pair(sB + s * C::B_BYTES, &tmap_x, &full[s], i * KSTEP, n0 + prank * C::B_ROWS);
      };
      int pre = 0;
      if (group < units) {
        pre = min(nk, C::STAGES);
        for (int i = 0; i < pre; ++i) load_w(i, 2 * (group / n_tiles) + prank, i);
      }
      pdl_wait();
      int it = 0;
      for (int u = group; u < units && !flags[0]; u += ngroups) {
        const int mt = 2 * (u / n_tiles) + prank;
        const int n0 = (u % n_tiles) * NTOK;
        for (int i = 0; i < nk; ++i, ++it) {
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
      if (prank == 0)
        for (int j = max(0, it - C::STAGES); j < it; ++j) mbar_wait(&full[j % C::STAGES], (j / C::STAGES) & 1);
    }
  } else if (warp == 1) {
    if (lane == 0 && prank == 0) {
      // kind::f16, BF16 A and B, fp32 D, K-major both, N = NTOK, M = 256.
      const uint32_t idesc = (1u << 4) | (1u << 7) | (1u << 10) | (static_cast<uint32_t>(NTOK >> 3) << 17) |
                             (static_cast<uint32_t>((2 * BM) >> 4) << 24);
      int it = 0, tc = 0;
      for (int u = group; u < units && !flags[0]; u += ngroups, ++tc) {
        const int b = tc & 1;
        // The epilogue has drained this accumulator's previous tile.
        if (!mbar_wait(&tmem_empty[b], ((tc >> 1) & 1) ^ 1)) {
          flags[0] = 1;
          break;
        }
        tc_fence_after();
        const uint32_t d = tmem + static_cast<uint32_t>(b * NTOK);
        for (int i = 0; i < nk; ++i, ++it) {
          const int s = it % C::STAGES;
          const uint32_t ph = (it / C::STAGES) & 1;
          if (flags[0] || !mbar_wait(&full[s], ph)) {
            flags[0] = 1;
            break;
          }
          tc_fence_after();
          const uint32_t a_addr = smem_u32(sA + s * C::A_BYTES);
          const uint32_t b_addr = smem_u32(sB + s * C::B_BYTES);
#pragma unroll
          for (int kk = 0; kk < 4; ++kk)
            mma_f16_pair(d, sdesc_sw128(a_addr + kk * 32), sdesc_sw128(b_addr + kk * 32), idesc, (i | kk) != 0);
          tc_commit_pair(&empty[s], pair_mask);
        }
        if (flags[0]) break;
        tc_commit_pair(&accf[b], pair_mask);
      }
    }
    __syncwarp();
  } else {
    // Epilogue: warp w reads TMEM lanes 32*(w%4) .. +31, i.e. vocabulary group mt*4 + w%4.
    const int q = warp & 3;
    pdl_wait();
    int tc = 0;
    for (int u = group; u < units; u += ngroups, ++tc) {
      const int b = tc & 1;
      const int mt = 2 * (u / n_tiles) + prank;
      const int n0 = (u % n_tiles) * NTOK;
      if (!mbar_wait(&accf[b], (tc >> 1) & 1)) {
        flags[0] = 1;
        break;
      }
      if (u + ngroups >= units) pdl_trigger();  // this CTA's last mainloop is done
      tc_fence_after();
      const int g = mt * 4 + q;
      if (g * 32 < a.F) {
        const uint32_t taddr = tmem + (static_cast<uint32_t>(q * 32) << 16) + static_cast<uint32_t>(b * NTOK);
#pragma unroll 1
        for (int c = 0; c < NTOK && n0 + c < a.T; c += 64) {
          float v[64];
          tmem_ld64(taddr + c, v);  // one TMEM round trip per 64 columns
#pragma unroll
          for (int half = 0; half < 2; ++half) {
            float w[32];
#pragma unroll
            for (int j = 0; j < 32; ++j) w[j] = v[half * 32 + j];
            const float m = transpose_max32(w, lane);
            const int t = n0 + c + half * 32 + lane;
            if (t < a.T) a.maxima[static_cast<int64_t>(t) * a.ldm + g] = m;
          }
        }
      }
      // This warp's reads of the accumulator are complete: one arrival per warp on the leader's barrier.
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_cluster(&tmem_empty[b], crank & ~1u);
    }
  }

  __syncwarp();
  tc_fence_before();
  cluster_sync();  // the pair frees its tensor memory together
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc_pair(tmem, C::TMEM_COLS);
  }
}

template <int NTOK>
int launch_head(const CUtensorMap& tx, const CUtensorMap& tw, const HeadArgs& a, cudaStream_t stream) {
  using C = HCfg<NTOK>;
  static unsigned long long done_mask = 0;
  static int sms[64] = {0};
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return q38host::cuda_status(e, "cudaGetDevice");
  if (dev >= 64) return q38host::set_error("device ordinal %d too large", dev), Q38_ERR_UNSUPPORTED;
  if (!(done_mask & (1ull << dev))) {
    e = cudaFuncSetAttribute(lm_head_kernel<NTOK>, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(C::SMEM));
    if (e == cudaSuccess) e = cudaDeviceGetAttribute(&sms[dev], cudaDevAttrMultiProcessorCount, dev);
    if (e != cudaSuccess) return q38host::cuda_status(e, "lm_head setup");
    done_mask |= 1ull << dev;
  }
  const int units = ((a.tiles + 1) / 2) * ((a.T + NTOK - 1) / NTOK);
  const int pairs = std::max(1, std::min(units, sms[dev] / 2));
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(2 * pairs));
  cfg.blockDim = dim3(192);
  cfg.dynamicSmemBytes = C::SMEM;
  cfg.stream = stream;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = q38host::add_pdl(attr, 1);
  e = cudaLaunchKernelEx(&cfg, lm_head_kernel<NTOK>, tx, tw, a);
  return q38host::cuda_status(e != cudaSuccess ? e : cudaGetLastError(), "lm_head launch");
}

}  // namespace

extern "C" int q38_lm_head_groupmax(const void* x, int64_t rows, int64_t k, const void* w, int64_t vocab, int group,
                                    float* maxima, int64_t ld_max, q38_stream_t stream) {
  using namespace q38host;
  if (!x || !w || !maxima) return set_error("q38_lm_head_groupmax: null pointer"), Q38_ERR_ARG;
  if (group != 32) return set_error("q38_lm_head_groupmax: group must be 32, got %d", group), Q38_ERR_ARG;
  if (rows <= 0 || k <= 0 || vocab <= 0 || vocab % 32 != 0 || k % KSTEP != 0 || rows > (1 << 24) || vocab > (1 << 28))
    return set_error("q38_lm_head_groupmax: bad sizes rows=%lld k=%lld (a multiple of 64) vocab=%lld (a multiple of 32)",
                     (long long)rows, (long long)k, (long long)vocab),
           Q38_ERR_ARG;
  if ((reinterpret_cast<uintptr_t>(x) & 15u) || (reinterpret_cast<uintptr_t>(w) & 15u))
    return set_error("q38_lm_head_groupmax: x and w must be 16-byte aligned"), Q38_ERR_ARG;
  if (ld_max < vocab / 32) return set_error("q38_lm_head_groupmax: ld_max too small"), Q38_ERR_ARG;
  HeadArgs a{};
  a.T = static_cast<int>(rows);
  a.F = static_cast<int>(vocab);
  a.nkc = static_cast<int>(k / KSTEP);
  a.tiles = static_cast<int>((vocab + BM - 1) / BM);
  a.maxima = maxima;
  a.ldm = ld_max;
  const int ntok = rows <= 64 ? 64 : rows <= 128 ? 128 : 256;
  CUtensorMap tx, tw;
  int st = encode_tmap_2d(&tx, x, rows, k, 2, ntok / 2, KSTEP);
  if (st != Q38_OK) return st;
  // The pre-tiled weights as rows of 128 bytes, one 128-row box per tile and K step.
  st = encode_tmap_2d(&tw, w, static_cast<uint64_t>(a.tiles) * a.nkc * BM, BK_BYTES, 1, BM, BK_BYTES, false);
  if (st != Q38_OK) return st;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  return ntok == 64 ? launch_head<64>(tx, tw, a, s) : ntok == 128 ? launch_head<128>(tx, tw, a, s)
                                                                   : launch_head<256>(tx, tw, a, s);
}

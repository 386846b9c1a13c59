// Gated delta rule over a prefill chunk of one row: GatedDeltaNetStep.prefill
// (qwen38_inf2/model.py:476-521) with the chunked rule of model.py:90-128.
//
// Four launches per call, all on the caller's stream:
//   prep   one CTA per (32-token tile, key head): the causal conv over [history * keep, chunk] with
//          the CPU branch's rounding (bf16 products summed left to right in bf16, model.py:513),
//          bf16 SiLU, fp32 L2 norms of q (then / sqrt(dk)) and k, and the gates beta, log decay
//          (masked to the valid tokens). q and k are written transposed, [key head][dk][tokens], so
//          the delta kernel's loads of a sub-chunk are contiguous runs of 256 bytes.
//   chunk  (delta, phase A) one CTA per (value head, sub-chunk of 64 tokens), all at once: the
//          state-free matrices of each sub-chunk, Aqk = (q k^T) * decay (lower), and the reference's
//          u = A (v beta), w = A (k beta e^g) with A = (I + N)^-1, N = strictly_lower(beta (k k^T) *
//          decay) (blocked solve), plus q e^g and k e^{g_last - g}, into the workspace.
//   state  (delta, phase B) one CTA per (value head, slice of up to 44 state columns). The state's value
//          columns evolve independently given phase A's matrices, so the slices need no exchange; each
//          CTA keeps its fp32 slice in shared memory across the chunk and walks the
//          sub-chunks:  v' = u - w S,  o = (q e^g) S + Aqk v',  S = e^{g_last} S + (k e^{g_last - g})^T v'
//          (model.py:110-128). The sub-chunk length is 64 instead of the CPU branch's 128 (model.py:34):
//          the rule is exact for any split.
//   norm   one CTA per token: the gated RMS norm of each value head (model.py:339-344), times SiLU(z),
//          e5m2 for out_proj; one more CTA carries the last conv_kernel-1 valid inputs into the conv
//          state (model.py:490-492) after the prep CTAs have read the old history.
#include "q38_common.cuh"

namespace {

using namespace q38;

constexpr int KCONV = 4;
constexpr int PREP_TOK = 32;  // tokens per prep CTA
constexpr int SUB = 64;       // tokens per sub-chunk of the delta rule
constexpr int SUBP = SUB + 4; // padded row of the transposed [dk][SUB] tiles (keeps float4 alignment)
constexpr int SDV = 44;       // state columns per state-walk CTA at most (128 columns: slices of 44, 44, 40)
constexpr int STH = SDV / 4 * 16;  // its threads: 11 column groups of 4 x 16 row groups

struct PrefillArgs {
  const __nv_bfloat16* qkvz;  // [tokens, ld_qkvz]: q | k | v | z
  int64_t ld_qkvz;
  const __nv_bfloat16* ab;  // [tokens, ld_ab]: b | a
  int64_t ld_ab;
  __nv_bfloat16* conv_state;  // this slot's row [conv_dim][KCONV - 1]
  const __nv_bfloat16* conv_w;
  const __nv_bfloat16* a_log;
  const __nv_bfloat16* dt_bias;
  const __nv_bfloat16* norm_w;
  __nv_bfloat16* state;  // this slot's row [num_v_heads][dk][dv]
  int tokens, n_valid;
  float keep;  // 1 when start > 0, else the history and state are zero
  uint8_t* out;
  int64_t ld_out;
  int num_k_heads, num_v_heads;
  float eps;
  // workspace
  float* qT;    // [num_k_heads][dk][tokens]
  float* kT;    // [num_k_heads][dk][tokens]
  float* v;     // [num_v_heads][tokens][dv]
  float* beta;  // [num_v_heads][tokens]
  float* g;     // [num_v_heads][tokens]
  __nv_bfloat16* o;  // [tokens][num_v_heads * dv]
  float* chunks;     // [num_v_heads][sub-chunks] phase A's per-sub-chunk matrices (ChunkWs)
};

// ---------------------------------------------------------------------------------------------
// prep
// ---------------------------------------------------------------------------------------------
// Threads of a prep CTA: two channels each (of 2 dk + R dv), so no thread waits on another's third.
template <int DK, int DV, int R>
constexpr int prep_threads() {
  return ((2 * DK + R * DV + 1) / 2 + 31) / 32 * 32;
}
constexpr int PREP_MAX_THREADS = 320;

template <int DK, int DV, int R>
__global__ void __launch_bounds__(PREP_MAX_THREADS, 2) gdn_prefill_prep_kernel(PrefillArgs a) {
  constexpr int CH = 2 * DK + R * DV;
  extern __shared__ __align__(16) uint8_t smem[];
  float* xs = reinterpret_cast<float*>(smem);  // [CH][PREP_TOK + 1]
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int kh = blockIdx.y;
  const int t0 = blockIdx.x * PREP_TOK;
  const int key_dim = a.num_k_heads * DK;
  const int h0 = kh * R;

  for (int i = tid; i < CH; i += blockDim.x) {
    int c;
    if (i < DK) c = kh * DK + i;
    else if (i < 2 * DK) c = key_dim + kh * DK + (i - DK);
    else c = 2 * key_dim + h0 * DV + (i - 2 * DK);
    float w[KCONV];
#pragma unroll
    for (int j = 0; j < KCONV; ++j) w[j] = __bfloat162float(a.conv_w[static_cast<int64_t>(c) * KCONV + j]);
    // win[j] = input at token t - (KCONV - 1) + j; inputs before token 0 come from the history.
    float win[KCONV];
#pragma unroll
    for (int j = 0; j < KCONV - 1; ++j) {
      const int t = t0 - (KCONV - 1) + j;
      win[j] = t >= 0 ? __bfloat162float(a.qkvz[static_cast<int64_t>(t) * a.ld_qkvz + c])
                      : __bfloat162float(a.conv_state[static_cast<int64_t>(c) * (KCONV - 1) + (t + KCONV - 1)]) * a.keep;
    }
    // The tile's inputs of this channel, all loads in flight at once.
    float xin[PREP_TOK];
#pragma unroll
    for (int tt = 0; tt < PREP_TOK; ++tt) {
      const int t = t0 + tt;
      xin[tt] = t < a.tokens ? __bfloat162float(a.qkvz[static_cast<int64_t>(t) * a.ld_qkvz + c]) : 0.f;
    }
#pragma unroll
    for (int tt = 0; tt < PREP_TOK; ++tt) {
      win[KCONV - 1] = xin[tt];
      // Python's sum over the taps: each addition rounds to bf16.
      float s = bf16r(__fmul_rn(win[0], w[0]));
#pragma unroll
      for (int j = 1; j < KCONV; ++j) s = bf16r(__fadd_rn(s, bf16r(__fmul_rn(win[j], w[j]))));
      xs[i * (PREP_TOK + 1) + tt] = t0 + tt < a.tokens ? bf16r(__fmul_rn(s, bf16r(sigmoidf_(s)))) : 0.f;
#pragma unroll
      for (int j = 0; j < KCONV - 1; ++j) win[j] = win[j + 1];
    }
  }
  __syncthreads();
  // L2 norms per (token, q|k), in place.
  const float inv_scale = static_cast<float>(sqrt(static_cast<double>(DK)));  // math.sqrt(k_head) as fp32
  for (int p = warp; p < 2 * PREP_TOK; p += blockDim.x / 32) {
    const int tt = p >> 1, which = p & 1;
    float* col = xs + (which * DK) * (PREP_TOK + 1) + tt;
    float ss = 0.f;
    for (int d = lane; d < DK; d += 32) ss = __fadd_rn(ss, __fmul_rn(col[d * (PREP_TOK + 1)], col[d * (PREP_TOK + 1)]));
    ss = warp_sum(ss);
    const float r = 1.0f / sqrtf(ss + 1e-6f);
    for (int d = lane; d < DK; d += 32) {
      const float v = __fmul_rn(col[d * (PREP_TOK + 1)], r);
      col[d * (PREP_TOK + 1)] = which == 0 ? __fdiv_rn(v, inv_scale) : v;
    }
  }
  __syncthreads();
  // q, k transposed: lane = token, so each row of 32 tokens is one 128-byte store.
  {
    const int t = t0 + lane;
    for (int d = warp; d < 2 * DK; d += blockDim.x / 32) {
      const int which = d >= DK, dd = d - which * DK;
      float* dst = (which ? a.kT : a.qT) + (static_cast<int64_t>(kh) * DK + dd) * a.tokens;
      if (t < a.tokens) dst[t] = xs[d * (PREP_TOK + 1) + lane];
    }
  }
  // v per value head, [head][token][dv].
  for (int idx = tid; idx < R * PREP_TOK * DV; idx += blockDim.x) {
    const int d = idx % DV, rest = idx / DV;
    const int tt = rest % PREP_TOK, j = rest / PREP_TOK;
    const int t = t0 + tt;
    if (t < a.tokens)
      a.v[(static_cast<int64_t>(h0 + j) * a.tokens + t) * DV + d] = xs[(2 * DK + j * DV + d) * (PREP_TOK + 1) + tt];
  }
  // Gates: beta = bf16(sigmoid(b)) * valid, g = -exp(A_log) * softplus(a + dt_bias) * valid.
  for (int idx = tid; idx < R * PREP_TOK; idx += blockDim.x) {
    const int j = idx / PREP_TOK, tt = idx % PREP_TOK;
    const int t = t0 + tt, h = h0 + j;
    if (t >= a.tokens) continue;
    const float valid = t < a.n_valid ? 1.0f : 0.0f;
    const float braw = __bfloat162float(a.ab[static_cast<int64_t>(t) * a.ld_ab + h]);
    const float araw = __bfloat162float(a.ab[static_cast<int64_t>(t) * a.ld_ab + a.num_v_heads + h]);
    a.beta[static_cast<int64_t>(h) * a.tokens + t] = __fmul_rn(bf16r(sigmoidf_(braw)), valid);
    a.g[static_cast<int64_t>(h) * a.tokens + t] =
        __fmul_rn(__fmul_rn(-expf(__bfloat162float(a.a_log[h])), softplusf_(__fadd_rn(araw, __bfloat162float(a.dt_bias[h])))),
                  valid);
  }
}

// ---------------------------------------------------------------------------------------------
// delta, phase A: everything of a sub-chunk that does not involve the state, for all (value head,
// sub-chunk) pairs at once. With gc the running sum of the sub-chunk's log decays:
//   Aqk[a][b] = (q_a . k_b) e^{gc_a - gc_b}            for a >= b, else 0
//   N[a][b]   = beta_a (k_a . k_b) e^{gc_a - gc_b}     for a > b
//   [u | w]   = (I + N)^-1 [beta v | beta e^{gc} k]    (the reference's u and w, model.py:110-116)
//   qg = q e^{gc},  kd = k e^{gc_last - gc},  el = e^{gc_last}
// go to the workspace, each matrix with padded rows so that phase B can bulk-copy it into shared
// memory as is. (I + N)^-1 is applied by blocked forward substitution: the four 16 x 16 diagonal
// blocks are inverted explicitly, one column of [u | w] per thread with the column in registers.
// ---------------------------------------------------------------------------------------------
template <int DK, int DV>
struct ChunkWs {
  static constexpr int RS = DK + 4;   // row stride of w, qg, kd (floats)
  static constexpr int AS = SUB + 4;  // row stride of Aqk
  static constexpr size_t AQK = 0;                               // [SUB][AS]
  static constexpr size_t U = AQK + SUB * AS;                    // [SUB][DV]
  static constexpr size_t W = U + SUB * DV;                      // [SUB][RS]
  static constexpr size_t QG = W + SUB * RS;                     // [SUB][RS]
  static constexpr size_t KD = QG + SUB * RS;                    // [SUB][RS]
  static constexpr size_t EL = KD + SUB * RS;                    // e^{gc_last} (4 floats)
  static constexpr size_t ITEM = EL + 4;                         // floats per (value head, sub-chunk)
  static_assert(AQK % 4 == 0 && U % 4 == 0 && W % 4 == 0 && QG % 4 == 0 && KD % 4 == 0 && EL % 4 == 0,
                "16-byte aligned pieces for the bulk copies");
};

template <int DK>
struct ChunkSmem {
  static constexpr size_t QT = 0;                                   // [DK][SUBP]
  static constexpr size_t KT = QT + sizeof(float) * DK * SUBP;      // [DK][SUBP]
  static constexpr size_t NT = KT + sizeof(float) * DK * SUBP;      // [SUB][SUBP] N^T
  static constexpr size_t INV = NT + sizeof(float) * SUB * SUBP;    // [4][16][16]
  static constexpr size_t VEC = INV + sizeof(float) * 4 * 16 * 16;  // gc, eg, beta, graw, wl [SUB] each
  static constexpr size_t TOTAL = VEC + sizeof(float) * 5 * SUB;
};

template <int DK, int DV>
__global__ void __launch_bounds__(256, 2) gdn_prefill_chunk_kernel(PrefillArgs a) {
  using S = ChunkSmem<DK>;
  using W = ChunkWs<DK, DV>;
  static_assert(DK + DV <= 256, "one [u | w] column per thread");
  extern __shared__ __align__(16) uint8_t smem[];
  float* qT = reinterpret_cast<float*>(smem + S::QT);
  float* kT = reinterpret_cast<float*>(smem + S::KT);
  float* nT = reinterpret_cast<float*>(smem + S::NT);
  float* inv = reinterpret_cast<float*>(smem + S::INV);
  float* gc = reinterpret_cast<float*>(smem + S::VEC);
  float* eg = gc + SUB;
  float* be = eg + SUB;
  float* graw = be + SUB;
  float* wl = graw + SUB;

  const int tid = threadIdx.x;
  const int h = blockIdx.x, c = blockIdx.y;
  const int R = a.num_v_heads / a.num_k_heads;
  const int kh = h / R;
  const int T = a.tokens;
  const int s0 = c * SUB, n = min(SUB, T - s0);
  float* item = a.chunks + (static_cast<size_t>(h) * gridDim.y + c) * W::ITEM;

  for (int i = tid; i < DK * SUB; i += 256) {
    const int d = i / SUB, t = i % SUB;
    const int64_t src = (static_cast<int64_t>(kh) * DK + d) * T + s0 + t;
    qT[d * SUBP + t] = t < n ? a.qT[src] : 0.f;
    kT[d * SUBP + t] = t < n ? a.kT[src] : 0.f;
  }
  if (tid < SUB) {
    be[tid] = tid < n ? a.beta[static_cast<int64_t>(h) * T + s0 + tid] : 0.f;
    graw[tid] = tid < n ? a.g[static_cast<int64_t>(h) * T + s0 + tid] : 0.f;
  }
  __syncthreads();
  if (tid == 0) {
    // Inclusive cumulative sum of the log decays (accumulated in double, rounded per element).
    double acc = 0.0;
    for (int t = 0; t < SUB; ++t) {
      acc += graw[t];
      gc[t] = static_cast<float>(acc);
    }
  }
  __syncthreads();
  if (tid < SUB) {
    eg[tid] = expf(gc[tid]);
    wl[tid] = expf(__fsub_rn(gc[SUB - 1], gc[tid]));
  }
  // Aqk (to the workspace) and N^T (to shared memory): the 64 x 64 products, 4 x 4 per thread.
  {
    const int ai = tid >> 4, bi = tid & 15;
    float accq[4][4], acck[4][4];
#pragma unroll
    for (int x = 0; x < 4; ++x)
#pragma unroll
      for (int y = 0; y < 4; ++y) accq[x][y] = acck[x][y] = 0.f;
#pragma unroll 4
    for (int d = 0; d < DK; ++d) {
      const float4 qa = *reinterpret_cast<const float4*>(qT + d * SUBP + 4 * ai);
      const float4 ka = *reinterpret_cast<const float4*>(kT + d * SUBP + 4 * ai);
      const float4 kb = *reinterpret_cast<const float4*>(kT + d * SUBP + 4 * bi);
      const float qv[4] = {qa.x, qa.y, qa.z, qa.w}, kv[4] = {ka.x, ka.y, ka.z, ka.w}, bv[4] = {kb.x, kb.y, kb.z, kb.w};
#pragma unroll
      for (int x = 0; x < 4; ++x)
#pragma unroll
        for (int y = 0; y < 4; ++y) {
          accq[x][y] = fmaf(qv[x], bv[y], accq[x][y]);
          acck[x][y] = fmaf(kv[x], bv[y], acck[x][y]);
        }
    }
    float aq[4][4];
#pragma unroll
    for (int y = 0; y < 4; ++y) {
      const int b = 4 * bi + y;
      float nn[4];
#pragma unroll
      for (int x = 0; x < 4; ++x) {
        const int a_ = 4 * ai + x;
        const float dec = a_ >= b ? expf(__fsub_rn(gc[a_], gc[b])) : 0.f;
        aq[x][y] = a_ >= b ? __fmul_rn(accq[x][y], dec) : 0.f;
        nn[x] = a_ > b ? __fmul_rn(__fmul_rn(be[a_], acck[x][y]), dec) : 0.f;
      }
      *reinterpret_cast<float4*>(nT + b * SUBP + 4 * ai) = make_float4(nn[0], nn[1], nn[2], nn[3]);
    }
#pragma unroll
    for (int x = 0; x < 4; ++x)
      *reinterpret_cast<float4*>(item + W::AQK + (4 * ai + x) * W::AS + 4 * bi) = make_float4(aq[x][0], aq[x][1], aq[x][2], aq[x][3]);
  }
  __syncthreads();  // N^T, eg and wl complete
  // Inverses of the four 16 x 16 unit lower diagonal blocks of I + N (a column per thread).
  if (tid < 64) {
    const int blk = tid >> 4, col_i = tid & 15, base = blk * 16;
    float col[16];
#pragma unroll
    for (int r = 0; r < 16; ++r) {
      float sacc = 0.f;
#pragma unroll
      for (int b = 0; b < r; ++b) sacc = fmaf(nT[(base + b) * SUBP + base + r], col[b], sacc);
      col[r] = r < col_i ? 0.f : (r == col_i ? 1.f : -sacc);
    }
#pragma unroll
    for (int r = 0; r < 16; ++r) inv[(blk * 16 + r) * 16 + col_i] = col[r];
  }
  // qg = q e^{gc}, kd = k e^{gc_last - gc}, token-major with padded rows. A warp covers 8 features x
  // 4 tokens: its shared-memory reads of the [d][t] tiles hit 32 distinct banks, its global writes are
  // four 32-byte runs.
  for (int i = tid; i < SUB * DK; i += 256) {
    const int l = i & 31, grp = i >> 5;
    const int d = (grp % (DK / 8)) * 8 + (l & 7), t = (grp / (DK / 8)) * 4 + (l >> 3);
    item[W::QG + t * W::RS + d] = __fmul_rn(qT[d * SUBP + t], eg[t]);
    item[W::KD + t * W::RS + d] = __fmul_rn(kT[d * SUBP + t], wl[t]);
  }
  if (tid == 0) item[W::EL] = eg[SUB - 1];
  __syncthreads();  // the inverses
  // [u | w] = (I + N)^-1 [beta v | beta e^{gc} k]: column j of the right-hand side in registers.
  if (tid < DV + DK) {
    const int j = tid;
    float x[SUB];
    if (j < DV) {
      const float* vsrc = a.v + (static_cast<int64_t>(h) * T + s0) * DV + j;
#pragma unroll
      for (int t = 0; t < SUB; ++t) x[t] = t < n ? __fmul_rn(be[t], vsrc[static_cast<int64_t>(t) * DV]) : 0.f;
    } else {
      const float* kcol = kT + (j - DV) * SUBP;  // 16-byte reads: a warp's 32 rows take the minimum 4 wavefronts
#pragma unroll
      for (int t = 0; t < SUB; t += 4) {
        const float4 k4 = *reinterpret_cast<const float4*>(kcol + t);
        const float kk[4] = {k4.x, k4.y, k4.z, k4.w};
#pragma unroll
        for (int e = 0; e < 4; ++e) x[t + e] = __fmul_rn(__fmul_rn(kk[e], be[t + e]), eg[t + e]);
      }
    }
#pragma unroll
    for (int blk = 0; blk < SUB / 16; ++blk) {
      float tv[16];
#pragma unroll
      for (int r = 0; r < 16; ++r) {
        const int row = blk * 16 + r;
        float sacc = x[row];
#pragma unroll
        for (int b = 0; b < blk * 16; ++b) sacc = fmaf(-nT[b * SUBP + row], x[b], sacc);
        tv[r] = sacc;
      }
#pragma unroll
      for (int r = 0; r < 16; ++r) {
        float v = 0.f;
#pragma unroll
        for (int cc = 0; cc <= r; ++cc) v = fmaf(inv[(blk * 16 + r) * 16 + cc], tv[cc], v);
        x[blk * 16 + r] = v;
      }
    }
    if (j < DV) {
#pragma unroll
      for (int t = 0; t < SUB; ++t) item[W::U + t * DV + j] = x[t];
    } else {
#pragma unroll
      for (int t = 0; t < SUB; ++t) item[W::W + t * W::RS + (j - DV)] = x[t];
    }
  }
}

// ---------------------------------------------------------------------------------------------
// delta, phase B: the state walk. One CTA per (value head, up to SDV state columns); the columns of S
// evolve independently given phase A's matrices, so the slices need no exchange. Three slices per
// head of 128 columns make 144 CTAs for 48 heads, one wave with one CTA per SM. The fp32 slice stays in
// shared memory across the chunk; per sub-chunk
//   v' = u - w S,   o = qg S + Aqk v' (bf16 out),   S = el S + kd^T v'
// with the inputs bulk-copied in while the previous step computes: qg and Aqk of the next sub-chunk
// during this one, kd (into w's buffer, once w is read) during o, and the next w during the next
// step's wait.
// ---------------------------------------------------------------------------------------------
template <int DK, int DV>
struct StateSmem {
  using W = ChunkWs<DK, DV>;
  static constexpr size_t ST = 0;                                         // [DK][SDV]
  static constexpr size_t WK = ST + sizeof(float) * DK * SDV;             // [SUB][RS] w, then kd
  static constexpr size_t QG = WK + sizeof(float) * SUB * W::RS;          // [SUB][RS] qg
  static constexpr size_t AQ = QG + sizeof(float) * SUB * W::RS;          // [SUB][AS] Aqk
  static constexpr size_t VP = AQ + sizeof(float) * SUB * W::AS;          // [SUB][SDV] v'
  static constexpr size_t BAR = VP + sizeof(float) * SUB * SDV;           // four mbarriers
  static constexpr size_t TOTAL = BAR + 32;
};

template <int DK, int DV>
__global__ void __launch_bounds__(STH, 1) gdn_prefill_state_kernel(PrefillArgs a) {
  using S = StateSmem<DK, DV>;
  using W = ChunkWs<DK, DV>;
  constexpr uint32_t RS_BYTES = sizeof(float) * SUB * W::RS;
  constexpr uint32_t AS_BYTES = sizeof(float) * SUB * W::AS;
  extern __shared__ __align__(16) uint8_t smem[];
  float* st = reinterpret_cast<float*>(smem + S::ST);
  float* wk = reinterpret_cast<float*>(smem + S::WK);
  float* qg = reinterpret_cast<float*>(smem + S::QG);
  float* aq = reinterpret_cast<float*>(smem + S::AQ);
  float* vp = reinterpret_cast<float*>(smem + S::VP);
  uint64_t* bar_w = reinterpret_cast<uint64_t*>(smem + S::BAR);
  uint64_t* bar_q = bar_w + 1;
  uint64_t* bar_k = bar_w + 2;
  uint64_t* bar_a = bar_w + 3;

  const int tid = threadIdx.x;
  const int h = blockIdx.x;
  const int c0 = blockIdx.y * SDV;  // first state column of this CTA
  const int ncols = min(SDV, DV - c0);  // a multiple of 4
  const int T = a.tokens;
  const int nsub = (T + SUB - 1) / SUB;
  const int64_t vd_all = static_cast<int64_t>(a.num_v_heads) * DV;
  const float* items = a.chunks + static_cast<size_t>(h) * nsub * W::ITEM;

  // The state slice, fp32, zero unless the row continues (start > 0).
  __nv_bfloat16* srow = a.state + static_cast<int64_t>(h) * DK * DV;
  for (int i = tid; i < DK * SDV; i += STH) {
    const int d = i / SDV, j = i % SDV;
    st[i] = j < ncols ? __fmul_rn(__bfloat162float(srow[d * DV + c0 + j]), a.keep) : 0.f;
  }
  if (tid == 0) {
    for (int i = 0; i < 4; ++i) mbar_init(bar_w + i, 1);
    fence_mbar_init();
  }
  __syncthreads();  // the barriers are initialised before anyone waits on them
  auto load = [&](uint64_t* bar, float* dst, int c, size_t off, uint32_t bytes) {
    mbar_arrive_expect_tx(bar, bytes);
    bulk_load(dst, items + static_cast<size_t>(c) * W::ITEM + off, bytes, bar);
  };
  if (tid == 0) {
    load(bar_w, wk, 0, W::W, RS_BYTES);
    load(bar_q, qg, 0, W::QG, RS_BYTES);
    load(bar_a, aq, 0, W::AQK, AS_BYTES);
  }

  // Thread tilings (STH threads): [SUB][SDV] outputs as RPT rows x 4 columns, [DK][SDV] as DPT x 4;
  // column groups past this slice's ncols compute zeros and store nothing.
  constexpr int CG = SDV / 4, RG = STH / CG, RPT = SUB / RG;
  constexpr int DG = STH / CG, DPT = DK / DG;
  static_assert(RPT >= 1 && DPT >= 1 && DK % DG == 0 && SUB % RG == 0 && RPT % 4 == 0, "tiling");
  const int ri = tid / CG, ci = tid % CG;
  const bool col_ok = 4 * ci < ncols;
  const int a0 = ri * RPT, d0 = ri * DPT;
  bool ok = true;

  for (int c = 0; c < nsub; ++c) {
    const float* it = items + static_cast<size_t>(c) * W::ITEM;
    const int s0 = c * SUB, n = min(SUB, T - s0);
    const uint32_t ph = c & 1;
    float4 u4[RPT];
#pragma unroll
    for (int x = 0; x < RPT; ++x)
      u4[x] = col_ok ? *reinterpret_cast<const float4*>(it + W::U + (a0 + x) * DV + c0 + 4 * ci) : make_float4(0.f, 0.f, 0.f, 0.f);
    const float el = it[W::EL];
    ok = ok && mbar_wait(bar_w, ph) && mbar_wait(bar_q, ph);
    // v' = u - w S and qg S, both against the state before this sub-chunk; four d per step.
    float accv[RPT][4], accq[RPT][4];
#pragma unroll
    for (int x = 0; x < RPT; ++x)
#pragma unroll
      for (int y = 0; y < 4; ++y) accv[x][y] = accq[x][y] = 0.f;
#pragma unroll 2
    for (int d = 0; d < DK; d += 4) {
      float s4[4][4];
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const float4 sv = *reinterpret_cast<const float4*>(st + (d + k) * SDV + 4 * ci);
        s4[k][0] = sv.x;
        s4[k][1] = sv.y;
        s4[k][2] = sv.z;
        s4[k][3] = sv.w;
      }
#pragma unroll
      for (int x = 0; x < RPT; ++x) {
        const float4 w4 = *reinterpret_cast<const float4*>(wk + (a0 + x) * W::RS + d);
        const float4 q4 = *reinterpret_cast<const float4*>(qg + (a0 + x) * W::RS + d);
        const float wx[4] = {w4.x, w4.y, w4.z, w4.w}, qx[4] = {q4.x, q4.y, q4.z, q4.w};
#pragma unroll
        for (int k = 0; k < 4; ++k)
#pragma unroll
          for (int y = 0; y < 4; ++y) {
            accv[x][y] = fmaf(wx[k], s4[k][y], accv[x][y]);
            accq[x][y] = fmaf(qx[k], s4[k][y], accq[x][y]);
          }
      }
    }
#pragma unroll
    for (int x = 0; x < RPT; ++x) {
      const float u[4] = {u4[x].x, u4[x].y, u4[x].z, u4[x].w};
      float v[4];
#pragma unroll
      for (int y = 0; y < 4; ++y) v[y] = __fsub_rn(u[y], accv[x][y]);
      *reinterpret_cast<float4*>(vp + (a0 + x) * SDV + 4 * ci) = make_float4(v[0], v[1], v[2], v[3]);
    }
    __syncthreads();  // v' complete; w and qg are read
    if (tid == 0 && ok) {
      load(bar_k, wk, c, W::KD, RS_BYTES);
      if (c + 1 < nsub) load(bar_q, qg, c + 1, W::QG, RS_BYTES);
    }
    ok = ok && mbar_wait(bar_a, ph);
    // o = qg S + Aqk v' (Aqk is zero above the diagonal), bf16 out; four b per step, the step past
    // a0 + RPT - 1 adding zeros.
    {
      float acc[RPT][4];
#pragma unroll
      for (int x = 0; x < RPT; ++x)
#pragma unroll
        for (int y = 0; y < 4; ++y) acc[x][y] = 0.f;
      for (int b = 0; b < a0 + RPT; b += 4) {
        float v4[4][4];
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          const float4 vv = *reinterpret_cast<const float4*>(vp + (b + k) * SDV + 4 * ci);
          v4[k][0] = vv.x;
          v4[k][1] = vv.y;
          v4[k][2] = vv.z;
          v4[k][3] = vv.w;
        }
#pragma unroll
        for (int x = 0; x < RPT; ++x) {
          const float4 m4 = *reinterpret_cast<const float4*>(aq + (a0 + x) * W::AS + b);
          const float m[4] = {m4.x, m4.y, m4.z, m4.w};
#pragma unroll
          for (int k = 0; k < 4; ++k)
#pragma unroll
            for (int y = 0; y < 4; ++y) acc[x][y] = fmaf(m[k], v4[k][y], acc[x][y]);
        }
      }
#pragma unroll
      for (int x = 0; x < RPT; ++x) {
        const int a_ = a0 + x;
        if (a_ < n && col_ok) {
          __nv_bfloat16* orow = a.o + static_cast<int64_t>(s0 + a_) * vd_all + static_cast<int64_t>(h) * DV + c0 + 4 * ci;
#pragma unroll
          for (int y = 0; y < 4; ++y) orow[y] = __float2bfloat16_rn(__fadd_rn(accq[x][y], acc[x][y]));
        }
      }
    }
    ok = ok && mbar_wait(bar_k, ph);
    // S = el S + kd^T v'.
    {
      float acc[DPT][4];
#pragma unroll
      for (int x = 0; x < DPT; ++x)
#pragma unroll
        for (int y = 0; y < 4; ++y) acc[x][y] = 0.f;
#pragma unroll 4
      for (int t = 0; t < SUB; ++t) {
        const float4 vv = *reinterpret_cast<const float4*>(vp + t * SDV + 4 * ci);
        const float v4[4] = {vv.x, vv.y, vv.z, vv.w};
        float kx[DPT];
        if constexpr (DPT % 4 == 0) {
#pragma unroll
          for (int x = 0; x < DPT; x += 4) {
            const float4 k4 = *reinterpret_cast<const float4*>(wk + t * W::RS + d0 + x);
            kx[x] = k4.x;
            kx[x + 1] = k4.y;
            kx[x + 2] = k4.z;
            kx[x + 3] = k4.w;
          }
        } else {
#pragma unroll
          for (int x = 0; x < DPT; ++x) kx[x] = wk[t * W::RS + d0 + x];
        }
#pragma unroll
        for (int x = 0; x < DPT; ++x)
#pragma unroll
          for (int y = 0; y < 4; ++y) acc[x][y] = fmaf(kx[x], v4[y], acc[x][y]);
      }
#pragma unroll
      for (int x = 0; x < DPT; ++x)
#pragma unroll
        for (int y = 0; y < 4; ++y) {
          float* p = st + (d0 + x) * SDV + 4 * ci + y;
          *p = __fadd_rn(__fmul_rn(*p, el), acc[x][y]);
        }
    }
    __syncthreads();  // S updated; kd, Aqk and v' are read
    if (tid == 0 && ok && c + 1 < nsub) {
      load(bar_w, wk, c + 1, W::W, RS_BYTES);
      load(bar_a, aq, c + 1, W::AQK, AS_BYTES);
    }
  }
  // A copy that timed out (recorded in the device error word) leaves the state untouched.
  if (__syncthreads_or(!ok)) return;
  for (int i = tid; i < DK * SDV; i += STH) {
    const int d = i / SDV, j = i % SDV;
    if (j < ncols) srow[d * DV + c0 + j] = __float2bfloat16_rn(st[i]);
  }
}

// ---------------------------------------------------------------------------------------------
// norm (+ conv carry)
// ---------------------------------------------------------------------------------------------
template <int DV>
__global__ void __launch_bounds__(256) gdn_prefill_norm_kernel(PrefillArgs a, int conv_dim) {
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int t = blockIdx.x;
  if (t == a.tokens) {
    // The conv state keeps window rows n_valid .. n_valid + KCONV - 2 of [history * keep, chunk].
    for (int c = tid; c < conv_dim; c += blockDim.x) {
      __nv_bfloat16* cs = a.conv_state + static_cast<int64_t>(c) * (KCONV - 1);
      __nv_bfloat16 val[KCONV - 1];
#pragma unroll
      for (int j = 0; j < KCONV - 1; ++j) {
        const int w = a.n_valid + j;
        val[j] = w < KCONV - 1 ? __float2bfloat16_rn(__bfloat162float(cs[w]) * a.keep)
                               : a.qkvz[static_cast<int64_t>(w - (KCONV - 1)) * a.ld_qkvz + c];
      }
#pragma unroll
      for (int j = 0; j < KCONV - 1; ++j) cs[j] = val[j];
    }
    return;
  }
  constexpr int CPL = DV / 32;
  const int64_t vd_all = static_cast<int64_t>(a.num_v_heads) * DV;
  const __nv_bfloat16* orow = a.o + static_cast<int64_t>(t) * vd_all;
  const __nv_bfloat16* zrow = a.qkvz + static_cast<int64_t>(t) * a.ld_qkvz + conv_dim;
  uint8_t* out = a.out + static_cast<int64_t>(t) * a.ld_out;
  for (int h = warp; h < a.num_v_heads; h += blockDim.x / 32) {
    float ob[CPL];
    float ss = 0.f;
#pragma unroll
    for (int i = 0; i < CPL; ++i) {
      ob[i] = __bfloat162float(orow[h * DV + lane * CPL + i]);
      ss = __fadd_rn(ss, __fmul_rn(ob[i], ob[i]));
    }
    ss = warp_sum(ss);
    const float r = 1.0f / sqrtf(__fadd_rn(__fdiv_rn(ss, static_cast<float>(DV)), a.eps));
#pragma unroll
    for (int i = 0; i < CPL; ++i) {
      const int c = lane * CPL + i;
      const float n1 = bf16r(__fmul_rn(ob[i], r));
      const float n2 = bf16r(__fmul_rn(__bfloat162float(a.norm_w[c]), n1));
      const float z = __bfloat162float(zrow[h * DV + c]);
      out[h * DV + c] = f32_to_e5m2(bf16r(__fmul_rn(n2, __fmul_rn(z, sigmoidf_(z)))));
    }
  }
}

size_t align256(size_t x) { return (x + 255) & ~size_t(255); }

struct WsLayout {
  size_t qT, kT, v, beta, g, o, chunks, total;
};

// Floats of phase A's output per (value head, sub-chunk): ChunkWs<dk, dv>::ITEM for the built shapes.
size_t chunk_item_floats(int dk, int dv) {
  return static_cast<size_t>(SUB) * (SUB + 4) + static_cast<size_t>(SUB) * dv + 3 * static_cast<size_t>(SUB) * (dk + 4) + 4;
}

WsLayout ws_layout(int64_t tokens, int hk, int hv, int dk, int dv) {
  WsLayout w{};
  size_t off = 0;
  w.qT = off;
  off = align256(off + sizeof(float) * hk * dk * tokens);
  w.kT = off;
  off = align256(off + sizeof(float) * hk * dk * tokens);
  w.v = off;
  off = align256(off + sizeof(float) * hv * tokens * dv);
  w.beta = off;
  off = align256(off + sizeof(float) * hv * tokens);
  w.g = off;
  off = align256(off + sizeof(float) * hv * tokens);
  w.o = off;
  off = align256(off + 2 * static_cast<size_t>(tokens) * hv * dv);
  w.chunks = off;
  off = align256(off + sizeof(float) * hv * static_cast<size_t>((tokens + SUB - 1) / SUB) * chunk_item_floats(dk, dv));
  w.total = off;
  return w;
}

template <int DK, int DV, int R>
int launch_prefill(PrefillArgs a, int conv_dim, cudaStream_t stream) {
  using CS = ChunkSmem<DK>;
  using SS = StateSmem<DK, DV>;
  static_assert(ChunkWs<DK, DV>::ITEM == (SUB * (SUB + 4) + SUB * DV + 3 * SUB * (DK + 4) + 4), "workspace size");
  static unsigned long long done_mask = 0;
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return q38host::cuda_status(e, "cudaGetDevice");
  const size_t prep_smem = sizeof(float) * (2 * DK + R * DV) * (PREP_TOK + 1);
  if (dev < 64 && !(done_mask & (1ull << dev))) {
    e = cudaFuncSetAttribute(gdn_prefill_prep_kernel<DK, DV, R>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             static_cast<int>(prep_smem));
    if (e == cudaSuccess)
      e = cudaFuncSetAttribute(gdn_prefill_chunk_kernel<DK, DV>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                               static_cast<int>(CS::TOTAL));
    if (e == cudaSuccess)
      e = cudaFuncSetAttribute(gdn_prefill_state_kernel<DK, DV>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                               static_cast<int>(SS::TOTAL));
    if (e != cudaSuccess) return q38host::cuda_status(e, "cudaFuncSetAttribute(gdn_prefill)");
    done_mask |= 1ull << dev;
  }
  dim3 gp((a.tokens + PREP_TOK - 1) / PREP_TOK, a.num_k_heads);
  static_assert(prep_threads<DK, DV, R>() <= PREP_MAX_THREADS, "prep CTA size");
  gdn_prefill_prep_kernel<DK, DV, R><<<gp, prep_threads<DK, DV, R>(), prep_smem, stream>>>(a);
  e = cudaGetLastError();
  if (e != cudaSuccess) return q38host::cuda_status(e, "gdn_prefill_prep launch");
  dim3 gc(a.num_v_heads, (a.tokens + SUB - 1) / SUB);
  gdn_prefill_chunk_kernel<DK, DV><<<gc, 256, CS::TOTAL, stream>>>(a);
  e = cudaGetLastError();
  if (e != cudaSuccess) return q38host::cuda_status(e, "gdn_prefill_chunk launch");
  dim3 gd(a.num_v_heads, (DV + SDV - 1) / SDV);
  gdn_prefill_state_kernel<DK, DV><<<gd, STH, SS::TOTAL, stream>>>(a);
  e = cudaGetLastError();
  if (e != cudaSuccess) return q38host::cuda_status(e, "gdn_prefill_state launch");
  gdn_prefill_norm_kernel<DV><<<a.tokens + 1, 256, 0, stream>>>(a, conv_dim);
  return q38host::cuda_status(cudaGetLastError(), "gdn_prefill_norm launch");
}

}  // namespace

extern "C" size_t q38_gdn_prefill_workspace_bytes(int64_t tokens, int num_k_heads, int num_v_heads, int head_k,
                                                  int head_v) {
  if (tokens <= 0 || num_k_heads <= 0 || num_v_heads <= 0 || head_k <= 0 || head_v <= 0) return 0;
  return ws_layout(tokens, num_k_heads, num_v_heads, head_k, head_v).total;
}

extern "C" int q38_gdn_prefill_chunk(const void* qkvz, int64_t ld_qkvz, const void* ab, int64_t ld_ab, void* conv_state,
                                     const void* conv_weight, const void* a_log, const void* dt_bias,
                                     const void* norm_weight, void* state, int64_t slot, int64_t state_rows,
                                     int64_t tokens, int64_t start, int64_t n_valid, void* out, int64_t ld_out,
                                     int num_k_heads, int num_v_heads, int head_k, int head_v, int conv_kernel,
                                     float eps, void* workspace, size_t workspace_bytes, q38_stream_t stream) {
  using namespace q38host;
  if (!qkvz || !ab || !conv_state || !conv_weight || !a_log || !dt_bias || !norm_weight || !state || !out || !workspace)
    return set_error("q38_gdn_prefill_chunk: null pointer"), Q38_ERR_ARG;
  if (tokens <= 0 || tokens > 65535 || n_valid < 0 || n_valid > tokens || start < 0)
    return set_error("q38_gdn_prefill_chunk: bad tokens %lld / n_valid %lld / start %lld", static_cast<long long>(tokens),
                     static_cast<long long>(n_valid), static_cast<long long>(start)),
           Q38_ERR_ARG;
  if (slot < 0 || slot >= state_rows) return set_error("q38_gdn_prefill_chunk: slot %lld out of range", static_cast<long long>(slot)), Q38_ERR_ARG;
  if (num_k_heads <= 0 || num_v_heads <= 0 || num_v_heads % num_k_heads)
    return set_error("q38_gdn_prefill_chunk: bad head counts"), Q38_ERR_ARG;
  if (conv_kernel != KCONV) return set_error("q38_gdn_prefill_chunk: conv kernel %d not built (4 is)", conv_kernel), Q38_ERR_ARG;
  const int64_t conv_dim = 2LL * num_k_heads * head_k + static_cast<int64_t>(num_v_heads) * head_v;
  if (ld_qkvz < conv_dim + static_cast<int64_t>(num_v_heads) * head_v || ld_ab < 2 * num_v_heads ||
      ld_out < static_cast<int64_t>(num_v_heads) * head_v)
    return set_error("q38_gdn_prefill_chunk: leading dimension too small"), Q38_ERR_ARG;
  const WsLayout w = ws_layout(tokens, num_k_heads, num_v_heads, head_k, head_v);
  if (workspace_bytes < w.total || (reinterpret_cast<uintptr_t>(workspace) & 255u) != 0)
    return set_error("q38_gdn_prefill_chunk: workspace needs %zu bytes, 256-byte aligned", w.total), Q38_ERR_ARG;
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  PrefillArgs a{};
  a.qkvz = static_cast<const __nv_bfloat16*>(qkvz);
  a.ld_qkvz = ld_qkvz;
  a.ab = static_cast<const __nv_bfloat16*>(ab);
  a.ld_ab = ld_ab;
  a.conv_state = static_cast<__nv_bfloat16*>(conv_state) + slot * conv_dim * (KCONV - 1);
  a.conv_w = static_cast<const __nv_bfloat16*>(conv_weight);
  a.a_log = static_cast<const __nv_bfloat16*>(a_log);
  a.dt_bias = static_cast<const __nv_bfloat16*>(dt_bias);
  a.norm_w = static_cast<const __nv_bfloat16*>(norm_weight);
  a.state = static_cast<__nv_bfloat16*>(state) + slot * static_cast<int64_t>(num_v_heads) * head_k * head_v;
  a.tokens = static_cast<int>(tokens);
  a.n_valid = static_cast<int>(n_valid);
  a.keep = start > 0 ? 1.0f : 0.0f;
  a.out = static_cast<uint8_t*>(out);
  a.ld_out = ld_out;
  a.num_k_heads = num_k_heads;
  a.num_v_heads = num_v_heads;
  a.eps = eps;
  a.qT = reinterpret_cast<float*>(ws + w.qT);
  a.kT = reinterpret_cast<float*>(ws + w.kT);
  a.v = reinterpret_cast<float*>(ws + w.v);
  a.beta = reinterpret_cast<float*>(ws + w.beta);
  a.g = reinterpret_cast<float*>(ws + w.g);
  a.o = reinterpret_cast<__nv_bfloat16*>(ws + w.o);
  a.chunks = reinterpret_cast<float*>(ws + w.chunks);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int rep = num_v_heads / num_k_heads;
  if (head_k == 128 && head_v == 128 && rep == 3) return launch_prefill<128, 128, 3>(a, static_cast<int>(conv_dim), s);
  if (head_k == 32 && head_v == 32 && rep == 3) return launch_prefill<32, 32, 3>(a, static_cast<int>(conv_dim), s);
  return set_error("q38_gdn_prefill_chunk: head dims %d/%d with %d value heads per key head not built", head_k, head_v, rep),
         Q38_ERR_UNSUPPORTED;
}

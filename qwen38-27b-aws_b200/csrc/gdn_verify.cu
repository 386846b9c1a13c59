// Gated delta rule, K verify tokens per row with commit-on-accept: GatedDeltaNetStep.verify
// (qwen38_inf2/model.py:376-454) and the CPU form of _commit_and_read (model.py:262-271).
//
// Two launches, the decode kernel's partition: one small CTA per (row, key head) convolves the K
// tokens' q and k channels (past the accepted tokens' inputs) and L2-normalises them into a workspace;
// then one CTA of 128 threads per (row, value head) owns that head's state tile, v channels and pending
// slices outright. Together:
//   1. commit: S' = bf16(S * e^{sum of the accepted tokens' log decays} * keep
//                         + sum_s (k_s e^{decays after s}) delta_s^T)   from the pending buffers the
//      last verify step kept (the closed form of applying those tokens one by one); the conv history
//      moves past the accepted tokens' inputs. A row with active 0 keeps both exactly.
//   2. the K new tokens: causal conv from that history, SiLU, L2 norms, gates; [k_t; q_t]^T S' for each
//      token, then the K x K chunk: delta_t = beta_t (v_t - e^{c_t} k_t^T S' - sum_{s<t} e^{c_t - c_s}
//      (k_t.k_s) delta_s), o_t = e^{c_t} q_t^T S' + sum_{s<=t} e^{c_t - c_s} (q_t.k_s) delta_s, with c
//      the running sum of log decays. S' itself is stored; the new tokens' k, delta, log decay and conv
//      inputs become the pending buffers for the next step to commit.
//   3. the gated RMS norm times SiLU(z), e5m2 for out_proj.
// Rounding follows the reference's CPU branch: the conv as decode (fp32 sum of bf16 products, one
// rounding), the committed state rounded to bf16 before it is read, fp32 elsewhere.
#include "gdn_common.cuh"

namespace {

using namespace q38;

constexpr int KCONV = 4;
constexpr int KMAX = 4;  // verify tokens per row built (the reference drafts K = 4)

struct VerifyArgs {
  const __nv_bfloat16* qkvz;  // [batch * K, ld_qkvz]: row b * K + t
  int64_t ld_qkvz;
  const __nv_bfloat16* ab;  // [batch * K, ld_ab]
  int64_t ld_ab;
  __nv_bfloat16* conv_state;  // [rows, conv_dim, KCONV - 1]
  const __nv_bfloat16* conv_w;
  const __nv_bfloat16* a_log;
  const __nv_bfloat16* dt_bias;
  const __nv_bfloat16* norm_w;
  __nv_bfloat16* state;  // [rows, num_v_heads, DK, DV]
  float* pending_key;    // [batch, K, num_v_heads, DK]
  float* pending_delta;  // [batch, K, num_v_heads, DV]
  float* pending_decay;  // [batch, K, num_v_heads]
  __nv_bfloat16* pending_input;  // [batch, K, conv_dim]
  const int32_t* position;
  const float* active;
  const int32_t* accepted;
  uint8_t* out;  // [batch * K, ld_out]
  int64_t ld_out;
  int num_k_heads, num_v_heads, head_v, K;
  float eps;
};

// One channel's conv for a verify step: the history is the KCONV - 1 inputs before the first uncommitted
// token (window [conv state, pending inputs] from `acc`, times keep; a row with active 0 keeps its conv
// state), then the K new inputs. Writes SiLU(conv) of each token to xs[t * stride], the new inputs to the
// pending buffer and, for an active row, the history to the conv state.
__device__ __forceinline__ void verify_conv_channel(const VerifyArgs& a, int b, int c, int conv_dim, int K, int acc,
                                                    bool on, float keep, float* xs, int stride) {
  constexpr int W = KCONV - 1 + KMAX;
  __nv_bfloat16* cs = a.conv_state + (static_cast<int64_t>(b) * conv_dim + c) * (KCONV - 1);
  float win[W];
#pragma unroll
  for (int j = 0; j < KCONV - 1; ++j) win[j] = __bfloat162float(cs[j]);
#pragma unroll
  for (int s = 0; s < KMAX; ++s)
    win[KCONV - 1 + s] = s < K ? __bfloat162float(a.pending_input[(static_cast<int64_t>(b) * K + s) * conv_dim + c]) : 0.f;
  float w2[W];
#pragma unroll
  for (int j = 0; j < KCONV - 1; ++j) {
    float h = win[j];
    if (on) {
      // win[acc + j] without a dynamic register index
#pragma unroll
      for (int s = 1; s <= KMAX; ++s)
        if (acc == s) h = win[s + j];
      h = __fmul_rn(h, keep);
    }
    w2[j] = h;
  }
  float cw[KCONV];
#pragma unroll
  for (int j = 0; j < KCONV; ++j) cw[j] = __bfloat162float(a.conv_w[static_cast<int64_t>(c) * KCONV + j]);
  // Every token's input is loaded before the pending buffer is overwritten (one round trip, not K).
  __nv_bfloat16 xin[KMAX];
#pragma unroll
  for (int t = 0; t < KMAX; ++t)
    if (t < K) xin[t] = a.qkvz[(static_cast<int64_t>(b) * K + t) * a.ld_qkvz + c];
#pragma unroll
  for (int t = 0; t < KMAX; ++t) {
    w2[KCONV - 1 + t] = 0.f;
    if (t < K) {
      w2[KCONV - 1 + t] = __bfloat162float(xin[t]);
      a.pending_input[(static_cast<int64_t>(b) * K + t) * conv_dim + c] = xin[t];
    }
  }
#pragma unroll
  for (int t = 0; t < KMAX; ++t) {
    if (t >= K) break;
    float sacc = 0.f;
#pragma unroll
    for (int j = 0; j < KCONV; ++j) sacc = __fadd_rn(sacc, bf16r(__fmul_rn(w2[t + j], cw[j])));
    const float conv = bf16r(sacc);
    xs[t * stride] = bf16r(__fmul_rn(conv, bf16r(sigmoidf_(conv))));
  }
  if (on) {
#pragma unroll
    for (int j = 0; j < KCONV - 1; ++j) cs[j] = __float2bfloat16_rn(w2[j]);
  }
}

// Kernel 1, one CTA of DK threads per (row, key head): the q and k channels' conv for the K tokens,
// their L2 norms (q / sqrt(dk)), into the workspace [row][key head][token][q | k][DK] (fp32).
template <int DK>
__global__ void __launch_bounds__(DK) gdn_verify_qk_kernel(VerifyArgs a, float* qk) {
  constexpr int NW = DK / 32;
  __shared__ float vals[2][KMAX][DK];
  __shared__ float part[2][KMAX][NW];
  const int kh = blockIdx.x, b = blockIdx.y, i = threadIdx.x, warp = i >> 5, lane = i & 31;
  const int K = a.K;
  const int pos = a.position[b];
  const bool on = a.active[b] > 0.5f;
  const float keep = (pos == 0 && on) ? 0.0f : 1.0f;
  int acc = a.accepted[b];
  acc = acc < 0 ? 0 : (acc > K ? K : acc);
  const int key_dim = a.num_k_heads * DK;
  const int conv_dim = 2 * key_dim + a.num_v_heads * a.head_v;
  verify_conv_channel(a, b, kh * DK + i, conv_dim, K, acc, on, keep, &vals[0][0][i], DK);
  verify_conv_channel(a, b, key_dim + kh * DK + i, conv_dim, K, acc, on, keep, &vals[1][0][i], DK);
  for (int t = 0; t < K; ++t) {
    const float sq = warp_sum(__fmul_rn(vals[0][t][i], vals[0][t][i]));
    const float sk = warp_sum(__fmul_rn(vals[1][t][i], vals[1][t][i]));
    if (lane == 0) {
      part[0][t][warp] = sq;
      part[1][t][warp] = sk;
    }
  }
  __syncthreads();
  const float inv_scale = static_cast<float>(sqrt(static_cast<double>(DK)));  // math.sqrt(k_head) as fp32
  float* dst = qk + (static_cast<int64_t>(b) * a.num_k_heads + kh) * K * 2 * DK;
  for (int t = 0; t < K; ++t) {
    float sq = 0.f, sk = 0.f;
#pragma unroll
    for (int w = 0; w < NW; ++w) {
      sq = __fadd_rn(sq, part[0][t][w]);
      sk = __fadd_rn(sk, part[1][t][w]);
    }
    dst[(t * 2 + 0) * DK + i] = __fdiv_rn(__fmul_rn(vals[0][t][i], 1.0f / sqrtf(sq + 1e-6f)), inv_scale);
    dst[(t * 2 + 1) * DK + i] = __fmul_rn(vals[1][t][i], 1.0f / sqrtf(sk + 1e-6f));
  }
}

template <int DK, int DV>
struct VerifySmem {
  static constexpr size_t TILE = static_cast<size_t>(DK) * DV * 2;
  static constexpr size_t FLOATS = static_cast<size_t>(KMAX) * DV        // xv: the K tokens' v (conv + SiLU)
                                   + 2 * KMAX * DK                       // qn, kn
                                   + KMAX * DK + KMAX * DV               // weighted pending keys, pending deltas
                                   + 4 * KMAX * DV                       // the 4 warps' k^T S' partials, then q^T S'
                                   + KMAX * DV                           // outputs before the norm
                                   + 2 * KMAX * KMAX + 2 * KMAX + KMAX + 4;  // dots, gates, commit weights, scale
  static constexpr size_t TOTAL = TILE + sizeof(float) * FLOATS + 16;
};

// Kernel 2, one CTA of 128 threads per (row, value head): the commit into its state tile, the head's v
// channels, the K x K chunk, the pending buffers and the gated norm.
template <int DK, int DV>
__global__ void __launch_bounds__(128) gdn_verify_kernel(VerifyArgs a, const float* qk) {
  using S = VerifySmem<DK, DV>;
  constexpr int ROWS_W = DK / 4;  // state rows per warp
  constexpr int CPL = DV / 32;    // state columns per lane
  constexpr uint32_t TILE_BYTES = DK * DV * 2;
  extern __shared__ __align__(128) uint8_t smem[];
  __nv_bfloat16* tile = reinterpret_cast<__nv_bfloat16*>(smem);
  float* xv = reinterpret_cast<float*>(smem + S::TILE);  // [KMAX][DV]
  float* qn = xv + KMAX * DV;                            // [KMAX][DK]
  float* kn = qn + KMAX * DK;                            // [KMAX][DK]
  float* wk = kn + KMAX * DK;                            // [KMAX][DK]
  float* dl = wk + KMAX * DK;                            // [KMAX][DV]
  float* red = dl + KMAX * DV;                           // [4][KMAX][DV], k^T S' partials, then q^T S'
  float* ob = red + 4 * KMAX * DV;                       // [KMAX][DV]
  float* dots = ob + KMAX * DV;                          // [2][KMAX][KMAX]
  float* gt = dots + 2 * KMAX * KMAX;                    // [KMAX][2] beta, log decay
  float* fw = gt + 2 * KMAX;                             // [KMAX] commit weights
  float* scl = fw + KMAX;                                // commit scale
  uint64_t* bar = reinterpret_cast<uint64_t*>((reinterpret_cast<uintptr_t>(scl + 4) + 7) & ~uintptr_t(7));

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int h = blockIdx.x, b = blockIdx.y;
  const int K = a.K;
  const int R = a.num_v_heads / a.num_k_heads;
  const int kh = h / R;
  const int pos = a.position[b];
  const bool on = a.active[b] > 0.5f;
  const float act = a.active[b];
  const float keep = (pos == 0 && on) ? 0.0f : 1.0f;
  int acc = a.accepted[b];
  acc = acc < 0 ? 0 : (acc > K ? K : acc);
  const int key_dim = a.num_k_heads * DK;
  const int conv_dim = 2 * key_dim + a.num_v_heads * DV;

  if (tid == 0) {
    mbar_init(bar, 1);
    fence_mbar_init();
    mbar_arrive_expect_tx(bar, TILE_BYTES);
    bulk_load(tile, a.state + (static_cast<int64_t>(b) * a.num_v_heads + h) * DK * DV, TILE_BYTES, bar);
    // Commit factors: the accepted tokens' log decays, summed in order, and what is left after each.
    float d[KMAX];
    float total = 0.f;
#pragma unroll
    for (int s = 0; s < KMAX; ++s) {
      d[s] = s < K ? __fmul_rn(a.pending_decay[(static_cast<int64_t>(b) * K + s) * a.num_v_heads + h], s < acc ? 1.f : 0.f)
                   : 0.f;
      if (s < K) total = __fadd_rn(total, d[s]);
    }
    scl[0] = on ? __fmul_rn(expf(total), keep) : 1.0f;
    float rem = total;
#pragma unroll
    for (int s = 0; s < KMAX; ++s) {
      if (s >= K) break;
      rem = __fsub_rn(rem, d[s]);
      fw[s] = __fmul_rn(__fmul_rn(__fmul_rn(expf(rem), s < acc ? 1.f : 0.f), keep), on ? 1.f : 0.f);
    }
  }
  // The head's v channels: history, the K tokens' conv and SiLU, conv state and pending inputs.
  for (int i = tid; i < DV; i += 128)
    verify_conv_channel(a, b, 2 * key_dim + h * DV + i, conv_dim, K, acc, on, keep, xv + i, DV);
  // This key head's normalised q and k of the K tokens, and this head's pending slices (read before
  // this step replaces them): 16-byte loads into registers first, stores after, one round trip.
  constexpr int QKV4 = (KMAX * 2 * DK / 4 + 127) / 128;       // float4 of q / k per thread
  constexpr int PV4 = (KMAX * (DK + DV) / 4 + 127) / 128;     // float4 of pending key / delta per thread
  const float4* src4 = reinterpret_cast<const float4*>(qk + (static_cast<int64_t>(b) * a.num_k_heads + kh) * K * 2 * DK);
  float4 rqk[QKV4], rpd[PV4];
#pragma unroll
  for (int j = 0; j < QKV4; ++j) {
    const int i4 = tid + 128 * j;
    if (i4 < K * 2 * DK / 4) rqk[j] = src4[i4];
  }
#pragma unroll
  for (int j = 0; j < PV4; ++j) {
    const int i4 = tid + 128 * j;
    if (i4 < K * (DK + DV) / 4) {
      const int s2 = i4 / ((DK + DV) / 4), e = (i4 % ((DK + DV) / 4)) * 4;
      const int64_t base = (static_cast<int64_t>(b) * K + s2) * a.num_v_heads + h;
      rpd[j] = e < DK ? *reinterpret_cast<const float4*>(a.pending_key + base * DK + e)
                      : *reinterpret_cast<const float4*>(a.pending_delta + base * DV + (e - DK));
    }
  }
#pragma unroll
  for (int j = 0; j < QKV4; ++j) {
    const int i4 = tid + 128 * j;
    if (i4 < K * 2 * DK / 4) {
      const int i = i4 * 4, t = i / (2 * DK), which = (i / DK) & 1, e = i % DK;
      *reinterpret_cast<float4*>((which ? kn : qn) + t * DK + e) = rqk[j];
    }
  }
  // Gates per token: beta = bf16(sigmoid(b)) * active, g = -exp(A_log) * softplus(a + dt_bias) * active.
  if (tid < K) {
    const int64_t r = static_cast<int64_t>(b) * K + tid;
    const float braw = __bfloat162float(a.ab[r * a.ld_ab + h]);
    const float araw = __bfloat162float(a.ab[r * a.ld_ab + a.num_v_heads + h]);
    gt[tid * 2 + 0] = __fmul_rn(bf16r(sigmoidf_(braw)), act);
    gt[tid * 2 + 1] = __fmul_rn(
        __fmul_rn(-expf(__bfloat162float(a.a_log[h])), softplusf_(__fadd_rn(araw, __bfloat162float(a.dt_bias[h])))), act);
  }
  __syncthreads();  // commit factors, v, q, k, gates
  // The pending slices, weighted for the commit.
#pragma unroll
  for (int j = 0; j < PV4; ++j) {
    const int i4 = tid + 128 * j;
    if (i4 < K * (DK + DV) / 4) {
      const int s2 = i4 / ((DK + DV) / 4), e = (i4 % ((DK + DV) / 4)) * 4;
      if (e < DK) {
        const float f = fw[s2];
        *reinterpret_cast<float4*>(wk + s2 * DK + e) =
            make_float4(__fmul_rn(rpd[j].x, f), __fmul_rn(rpd[j].y, f), __fmul_rn(rpd[j].z, f), __fmul_rn(rpd[j].w, f));
      } else {
        *reinterpret_cast<float4*>(dl + s2 * DV + (e - DK)) = rpd[j];
      }
    }
  }
  // k_t . k_s (s < t) and q_t . k_s (s <= t), one warp per dot.
  for (int p = warp; p < 2 * K * K; p += 4) {
    const int which = p / (K * K), t = (p / K) % K, s = p % K;
    const float* x = (which ? qn : kn) + t * DK;
    const float* y = kn + s * DK;
    float dsum = 0.f;
    for (int i = lane; i < DK; i += 32) dsum = fmaf(x[i], y[i], dsum);
    dsum = warp_sum(dsum);
    if (lane == 0) dots[(which * KMAX + t) * KMAX + s] = dsum;
  }
  const bool ok = mbar_wait(bar, 0);
  if (__syncthreads_or(!ok)) return;  // the copy timed out (recorded): nothing written

  // Commit S' = bf16(S * scale + sum_s w_s k_s delta_s^T) in place, and [k_t; q_t]^T S'.
  const int c0 = lane * CPL;
  const float scale = scl[0];
  float prod[2 * KMAX][CPL];
#pragma unroll
  for (int t = 0; t < 2 * KMAX; ++t)
#pragma unroll
    for (int e = 0; e < CPL; ++e) prod[t][e] = 0.f;
  // This thread's columns of the pending deltas are the same for every row: registers.
  float dlr[KMAX][CPL];
#pragma unroll
  for (int s = 0; s < KMAX; ++s)
#pragma unroll
    for (int e = 0; e < CPL; ++e) dlr[s][e] = s < K ? dl[s * DV + c0 + e] : 0.f;
#pragma unroll 4
  for (int r = 0; r < ROWS_W; ++r) {
    const int i = warp * ROWS_W + r;
    float sv[CPL];
    load_row<CPL>(tile + i * DV + c0, sv);
    float wki[KMAX];
#pragma unroll
    for (int s = 0; s < KMAX; ++s) wki[s] = s < K ? wk[s * DK + i] : 0.f;
#pragma unroll
    for (int e = 0; e < CPL; ++e) {
      float w = 0.f;
#pragma unroll
      for (int s = 0; s < KMAX; ++s)
        if (s < K) w = fmaf(wki[s], dlr[s][e], w);
      sv[e] = bf16r(__fadd_rn(__fmul_rn(sv[e], scale), w));
    }
    if (on) store_row<CPL>(tile + i * DV + c0, sv);
#pragma unroll
    for (int t = 0; t < KMAX; ++t) {
      if (t >= K) break;
      const float kt = kn[t * DK + i], qt = qn[t * DK + i];
#pragma unroll
      for (int e = 0; e < CPL; ++e) {
        prod[t][e] = fmaf(kt, sv[e], prod[t][e]);
        prod[KMAX + t][e] = fmaf(qt, sv[e], prod[KMAX + t][e]);
      }
    }
  }
  // The 4 warps' partials summed per column in warp order, k^T S' first, then q^T S' through the same
  // buffer (half the shared memory of both at once: 4 CTAs per SM instead of 3). One column per thread.
  static_assert(DV <= 128, "one state column per thread");
  const int c = tid;
  float ksum[KMAX], qsum[KMAX];
#pragma unroll
  for (int half = 0; half < 2; ++half) {
#pragma unroll
    for (int t = 0; t < KMAX; ++t) {
      if (t >= K) break;
#pragma unroll
      for (int e = 0; e < CPL; ++e) red[(warp * KMAX + t) * DV + c0 + e] = prod[half * KMAX + t][e];
    }
    if (half == 0) fence_proxy_async_shared();  // the committed tile is visible to the bulk copy engine
    __syncthreads();
    if (half == 0 && tid == 0 && on) {
      bulk_store(a.state + (static_cast<int64_t>(b) * a.num_v_heads + h) * DK * DV, tile, TILE_BYTES);
      bulk_commit();
    }
#pragma unroll
    for (int t = 0; t < KMAX; ++t) {
      float sum = 0.f;
      if (t < K && c < DV) {
#pragma unroll
        for (int w = 0; w < 4; ++w) sum = __fadd_rn(sum, red[(w * KMAX + t) * DV + c]);
      }
      (half == 0 ? ksum : qsum)[t] = sum;
    }
    __syncthreads();  // the partials are read before the buffer is reused
  }
  // The K x K chunk, one state column per thread.
  if (c < DV) {
    float cum[KMAX], dlt[KMAX];
#pragma unroll
    for (int t = 0; t < KMAX; ++t) {
      cum[t] = t == 0 ? gt[1] : __fadd_rn(cum[t - 1], gt[t * 2 + 1]);
      dlt[t] = 0.f;
    }
#pragma unroll
    for (int t = 0; t < KMAX; ++t) {
      if (t >= K) break;
      const float ks = ksum[t], qs = qsum[t];
      float dd = __fsub_rn(xv[t * DV + c], __fmul_rn(expf(cum[t]), ks));
#pragma unroll
      for (int s = 0; s < t; ++s)
        dd = __fsub_rn(dd, __fmul_rn(__fmul_rn(expf(__fsub_rn(cum[t], cum[s])), dots[(0 * KMAX + t) * KMAX + s]), dlt[s]));
      dlt[t] = __fmul_rn(dd, gt[t * 2 + 0]);
      float o = __fmul_rn(expf(cum[t]), qs);
#pragma unroll
      for (int s = 0; s <= t; ++s)
        o = __fadd_rn(o, __fmul_rn(__fmul_rn(expf(__fsub_rn(cum[t], cum[s])), dots[(1 * KMAX + t) * KMAX + s]), dlt[s]));
      ob[t * DV + c] = bf16r(o);
      a.pending_delta[((static_cast<int64_t>(b) * K + t) * a.num_v_heads + h) * DV + c] = dlt[t];
    }
  }
  for (int i = tid; i < K * DK; i += 128) {
    const int t = i / DK, e = i % DK;
    a.pending_key[((static_cast<int64_t>(b) * K + t) * a.num_v_heads + h) * DK + e] = kn[t * DK + e];
  }
  if (tid < K) a.pending_decay[(static_cast<int64_t>(b) * K + tid) * a.num_v_heads + h] = gt[tid * 2 + 1];
  __syncthreads();
  // Gated RMS norm of each token's output for this head, times SiLU(z); e5m2 out. Warp w: tokens w, w+4, ...
  for (int t = warp; t < K; t += 4) {
    float o[CPL];
    float ss = 0.f;
#pragma unroll
    for (int e = 0; e < CPL; ++e) {
      o[e] = ob[t * DV + c0 + e];
      ss = __fadd_rn(ss, __fmul_rn(o[e], o[e]));
    }
    ss = warp_sum(ss);
    const float r = 1.0f / sqrtf(__fadd_rn(__fdiv_rn(ss, static_cast<float>(DV)), a.eps));
    const int64_t row = static_cast<int64_t>(b) * K + t;
    const __nv_bfloat16* zrow = a.qkvz + row * a.ld_qkvz + conv_dim + h * DV;
    uint8_t* orow = a.out + row * a.ld_out + h * DV;
    float nwv[CPL], zv[CPL];  // loaded before any output store (one round trip)
#pragma unroll
    for (int e = 0; e < CPL; ++e) {
      nwv[e] = __bfloat162float(a.norm_w[c0 + e]);
      zv[e] = __bfloat162float(zrow[c0 + e]);
    }
#pragma unroll
    for (int e = 0; e < CPL; ++e) {
      const int c = c0 + e;
      const float n1 = bf16r(__fmul_rn(o[e], r));
      const float n2 = bf16r(__fmul_rn(nwv[e], n1));
      const float z = zv[e];
      orow[c] = f32_to_e5m2(bf16r(__fmul_rn(n2, __fmul_rn(z, sigmoidf_(z)))));
    }
  }
  if (tid == 0 && on) bulk_wait_read0();  // the tile must stay until the copy engine has read it
}

template <int DK, int DV>
int launch_verify(const VerifyArgs& a, int64_t batch, float* qk, cudaStream_t stream) {
  using S = VerifySmem<DK, DV>;
  static unsigned long long done_mask = 0;
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return q38host::cuda_status(e, "cudaGetDevice");
  if (dev < 64 && !(done_mask & (1ull << dev))) {
    e = cudaFuncSetAttribute(gdn_verify_kernel<DK, DV>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             static_cast<int>(S::TOTAL));
    if (e != cudaSuccess) return q38host::cuda_status(e, "cudaFuncSetAttribute(gdn_verify)");
    done_mask |= 1ull << dev;
  }
  gdn_verify_qk_kernel<DK><<<dim3(a.num_k_heads, static_cast<unsigned>(batch)), DK, 0, stream>>>(a, qk);
  e = cudaGetLastError();
  if (e != cudaSuccess) return q38host::cuda_status(e, "gdn_verify_qk launch");
  gdn_verify_kernel<DK, DV><<<dim3(a.num_v_heads, static_cast<unsigned>(batch)), 128, S::TOTAL, stream>>>(a, qk);
  return q38host::cuda_status(cudaGetLastError(), "gdn_verify launch");
}

}  // namespace

extern "C" size_t q38_gdn_verify_workspace_bytes(int64_t batch, int tokens, int num_k_heads, int head_k) {
  if (batch <= 0 || tokens <= 0 || num_k_heads <= 0 || head_k <= 0) return 0;
  return sizeof(float) * static_cast<size_t>(batch) * num_k_heads * tokens * 2 * head_k;
}

extern "C" int q38_gdn_verify_commit(const void* qkvz, int64_t ld_qkvz, const void* ab, int64_t ld_ab, void* conv_state,
                                     const void* conv_weight, const void* a_log, const void* dt_bias,
                                     const void* norm_weight, void* state, void* pending_key, void* pending_delta,
                                     void* pending_decay, void* pending_input, const int32_t* position,
                                     const float* active, const int32_t* accepted, void* out, int64_t ld_out,
                                     int64_t batch, int tokens, int num_k_heads, int num_v_heads, int head_k,
                                     int head_v, int conv_kernel, float eps, void* workspace, size_t workspace_bytes,
                                     q38_stream_t stream) {
  using namespace q38host;
  if (!qkvz || !ab || !conv_state || !conv_weight || !a_log || !dt_bias || !norm_weight || !state || !pending_key ||
      !pending_delta || !pending_decay || !pending_input || !position || !active || !accepted || !out || !workspace)
    return set_error("q38_gdn_verify_commit: null pointer"), Q38_ERR_ARG;
  if (batch <= 0 || batch > 65535 || tokens < 1 || tokens > KMAX)
    return set_error("q38_gdn_verify_commit: batch %lld / %d tokens per row (1..%d built)", static_cast<long long>(batch),
                     tokens, KMAX),
           Q38_ERR_ARG;
  if (num_k_heads <= 0 || num_v_heads <= 0 || num_v_heads % num_k_heads)
    return set_error("q38_gdn_verify_commit: bad head counts"), Q38_ERR_ARG;
  if (conv_kernel != KCONV) return set_error("q38_gdn_verify_commit: conv kernel %d not built (4 is)", conv_kernel), Q38_ERR_ARG;
  if ((reinterpret_cast<uintptr_t>(state) & 15u) != 0)
    return set_error("q38_gdn_verify_commit: state must be 16-byte aligned"), Q38_ERR_ARG;
  const int64_t conv_dim = 2LL * num_k_heads * head_k + static_cast<int64_t>(num_v_heads) * head_v;
  if (ld_qkvz < conv_dim + static_cast<int64_t>(num_v_heads) * head_v || ld_ab < 2 * num_v_heads ||
      ld_out < static_cast<int64_t>(num_v_heads) * head_v)
    return set_error("q38_gdn_verify_commit: leading dimension too small"), Q38_ERR_ARG;
  if (workspace_bytes < q38_gdn_verify_workspace_bytes(batch, tokens, num_k_heads, head_k) ||
      (reinterpret_cast<uintptr_t>(workspace) & 15u) != 0)
    return set_error("q38_gdn_verify_commit: workspace needs %zu bytes, 16-byte aligned",
                     q38_gdn_verify_workspace_bytes(batch, tokens, num_k_heads, head_k)),
           Q38_ERR_ARG;
  VerifyArgs a{};
  a.qkvz = static_cast<const __nv_bfloat16*>(qkvz);
  a.ld_qkvz = ld_qkvz;
  a.ab = static_cast<const __nv_bfloat16*>(ab);
  a.ld_ab = ld_ab;
  a.conv_state = static_cast<__nv_bfloat16*>(conv_state);
  a.conv_w = static_cast<const __nv_bfloat16*>(conv_weight);
  a.a_log = static_cast<const __nv_bfloat16*>(a_log);
  a.dt_bias = static_cast<const __nv_bfloat16*>(dt_bias);
  a.norm_w = static_cast<const __nv_bfloat16*>(norm_weight);
  a.state = static_cast<__nv_bfloat16*>(state);
  a.pending_key = static_cast<float*>(pending_key);
  a.pending_delta = static_cast<float*>(pending_delta);
  a.pending_decay = static_cast<float*>(pending_decay);
  a.pending_input = static_cast<__nv_bfloat16*>(pending_input);
  a.position = position;
  a.active = active;
  a.accepted = accepted;
  a.out = static_cast<uint8_t*>(out);
  a.ld_out = ld_out;
  a.num_k_heads = num_k_heads;
  a.num_v_heads = num_v_heads;
  a.head_v = head_v;
  a.K = tokens;
  a.eps = eps;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int rep = num_v_heads / num_k_heads;
  float* qk = static_cast<float*>(workspace);
  if (head_k == 128 && head_v == 128 && rep == 3) return launch_verify<128, 128>(a, batch, qk, s);
  if (head_k == 32 && head_v == 32 && rep == 3) return launch_verify<32, 32>(a, batch, qk, s);
  return set_error("q38_gdn_verify_commit: head dims %d/%d with %d value heads per key head not built", head_k, head_v,
                   rep),
         Q38_ERR_UNSUPPORTED;
}

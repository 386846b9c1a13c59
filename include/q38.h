/*
 * q38.h: C ABI of the B200 (sm_100a) kernels for the Qwen3.8 hybrid-decoder step.
 *
 * Every entry point takes raw device pointers, sizes and a CUDA stream (passed as an opaque
 * pointer, 0 for the legacy default stream), launches asynchronously on that stream, allocates
 * nothing, and returns an int status: Q38_OK (0) or a negative Q38_ERR_* code. q38_last_error()
 * gives the message of the last failure on the calling host thread.
 *
 * Numbers and layouts:
 *   bf16   : IEEE bfloat16, 2 bytes.
 *   e5m2   : FP8 E5M2 byte, the format the reference rounds every FP8 linear's input to
 *            (qwen38_inf2/model.py:85-87, :224).
 *   e4m3   : FP8 E4M3 (OCP e4m3fn) byte, the weight format.
 *   ue8m0  : one byte per 32 weights along K, value 2^(byte-127) (power-of-two group scale).
 *   Weights [out_features, in_features] are pre-tiled: 16 KB tiles of 128 rows x 128 bytes of K,
 *   ordered [row tile][K tile], each tile 128-byte swizzled (16-byte chunk c of tile row r stored at
 *   chunk c ^ (r % 8)), zero padded; q38_weight_tile_bytes gives the size. Their scales are pre-tiled
 *   into 512-byte blocks, one per (128 output rows, 128 K): byte (r % 32) * 16 + (r / 32) * 4 + (g % 4)
 *   holds row r's scale for K group g (q38_sf_tile_bytes).
 *
 * The reference's device path is NKI kernels called from PyTorch (qwen38_inf2/kernels.py); its
 * CPU branches (qwen38_inf2/model.py) define the arithmetic these kernels reproduce. Each function
 * below names the reference interface it replaces.
 */
#ifndef Q38_H
#define Q38_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define Q38_OK 0
#define Q38_ERR_ARG (-1)         /* bad pointer, size, alignment or unsupported shape */
#define Q38_ERR_CUDA (-2)        /* a CUDA runtime/driver call failed */
#define Q38_ERR_TIMEOUT (-3)     /* a bounded device wait gave up (set by kernels) */
#define Q38_ERR_UNSUPPORTED (-4) /* not built for this device */
#define Q38_ERR_DEVICE (-5)      /* a kernel recorded an error; see q38_device_status */

typedef void* q38_stream_t; /* a cudaStream_t */

/* Epilogues of q38_fp8_gemm. */
#define Q38_EPI_BF16 0     /* y = bf16(acc) */
#define Q38_EPI_RESIDUAL 1 /* y = bf16(residual + bf16(acc)); residual may alias y */

/* ABI version, bumped on any signature change. */
int q38_abi_version(void);

/*
 * Programmatic dependent launch for the decode path's kernels (GEMMs, lm_head, norms, gated delta and
 * attention decode): each may start while the previous kernel in its stream drains, running its
 * prologue and prefetching its weights, and waits on the device before touching activations. On by
 * default (the environment variable Q38_PDL=0 turns it off); applies to launches after the call.
 */
int q38_set_pdl(int enable);

/* Copies the last error message of this host thread into buf (NUL-terminated). Returns its length. */
int q38_last_error(char* buf, size_t n);

/* Reads (and with reset != 0 clears) the device error word that bounded waits set. Synchronises
 * the current device. Returns Q38_OK, a kernel's Q38_ERR_* code, or Q38_ERR_CUDA. */
int q38_device_status(int reset);

/*
 * y[t, f] = sum_k e5m2(x)[t, k] * e4m3(w)[f, k] * 2^(sf[f, k/32] - 127), fp32 accumulate, then the
 * epilogue. Replaces FP8Linear.forward (qwen38_inf2/model.py:211-229) and the NKI kernel
 * fp8_linear (qwen38_inf2/kernels.py:25-71, :175-196), whose CPU branch is
 * F.linear(fp8_round(x), fp8_to_float(W).T.to(bf16)). x is already e5m2 here: the producer of x
 * (norm, gated norm, attention, SiLU product) rounds it.
 *
 *   x        e5m2 [tokens, k]            (16-byte aligned, k % 16 == 0)
 *   w        e4m3 [features, k], pre-tiled (see above)
 *   w_sf     pre-tiled ue8m0 scales, ceil(features/128) * ceil(k/128) blocks of 512 bytes
 *   y        bf16 [tokens, ldy]
 *   residual bf16 [tokens, ldr] for Q38_EPI_RESIDUAL, else NULL
 *   splits   K splits (>= 1). With splits > 1 the partial sums go through `workspace`, of at least
 *            q38_fp8_gemm_workspace_bytes(tokens, features, splits) bytes, whose counter region
 *            must be zero before the first call (the kernel leaves it zero again).
 */
size_t q38_fp8_gemm_workspace_bytes(int64_t tokens, int64_t features, int splits);
int q38_fp8_gemm(const void* x, int64_t tokens, int64_t k, const void* w, const void* w_sf, int64_t features,
                 int epilogue, void* y, int64_t ldy, const void* residual, int64_t ldr, int splits, void* workspace,
                 size_t workspace_bytes, q38_stream_t stream);

/*
 * q38_fp8_gemm without a caller workspace, for callers that cannot allocate device memory: hosts whose
 * memory is owned by a framework pool, plugins that must not synchronise the device, and FFI bindings
 * that carry only input and output pointers. This entry point has no counterpart in the reference.
 * The split-K partial sums go to a fixed array inside the library, Q38_STATIC_SCRATCH_BYTES on every
 * GPU that loads it (kept until exit). Only calls that need the workspace epilogue use the array:
 * more than 8 K splits, or an output (or residual) that cannot be tensor-mapped (not 16-byte aligned,
 * or a row stride that is not a multiple of 8 elements); other calls run as q38_fp8_gemm does without
 * a workspace. Of the calls that use it, a shape whose q38_fp8_gemm_workspace_bytes exceeds the array
 * is refused with Q38_ERR_ARG. Every argument is checked on the host before the array is touched.
 * The first call on a device looks the array's address up once (cudaGetSymbolAddress), so make that
 * first call before any stream capture. All calls share the
 * one array: calls that overlap on the GPU (other streams, other host threads) race on it.
 * Arguments are those of q38_fp8_gemm without workspace and workspace_bytes.
 */
#define Q38_STATIC_SCRATCH_BYTES (16 * 1024 * 1024)
int q38_fp8_gemm_static_scratch(const void* x, int64_t tokens, int64_t k, const void* w, const void* w_sf,
                                int64_t features, int epilogue, void* y, int64_t ldy, const void* residual,
                                int64_t ldr, int splits, q38_stream_t stream);

/*
 * The same GEMM and epilogues (Q38_EPI_BF16, Q38_EPI_RESIDUAL) divided stream-K: one persistent CTA per
 * SM (2-SM pairs for 256-token tiles) and the K steps of all output tiles split evenly between them, so
 * every SM works for the whole launch whatever the tile count. A tile that one CTA computes whole takes
 * its epilogue from tensor memory; a tile split between CTAs leaves each part's fp32 partial in the
 * workspace and the last part to finish sums them in K order (deterministic) and applies the epilogue.
 * No CTA waits for another. Same FP8 formats as q38_fp8_gemm; the sum order over K differs from the
 * split-K form's (fp32 partial sums over other K ranges). The workspace (q38_fp8_gemm_streamk_workspace_bytes
 * for the shape on the current device, 0 on a bad shape or without a device) must be 16-byte aligned and
 * zero when first used; each call leaves its counters at zero again. Calls on one workspace must not
 * overlap. Replaces the row-parallel projections at TP = 1 (qwen38_inf2/model.py:259, :374, :639 with the
 * residual add of DecoderLayer.forward, model.py:918-930).
 */
size_t q38_fp8_gemm_streamk_workspace_bytes(int64_t tokens, int64_t features, int64_t k);
int q38_fp8_gemm_streamk(const void* x_q, int64_t tokens, int64_t k, const void* w, const void* w_sf,
                         int64_t features, int epilogue, void* y, int64_t ldy, const void* residual, int64_t ldr,
                         void* workspace, size_t workspace_bytes, q38_stream_t stream);

/* Bytes of the pre-tiled scale array of a [features, k] weight. */
size_t q38_sf_tile_bytes(int64_t features, int64_t k);

/* Bytes of a pre-tiled weight with `features` rows of `row_bytes` bytes (k for FP8, 2k for BF16). */
size_t q38_weight_tile_bytes(int64_t features, int64_t row_bytes);

/*
 * Decoder-layer input norms: h = bf16(rms_norm(x) * (1 + w)), written as bf16 (y_bf16, optional)
 * and as e5m2 (y_e5m2, optional). Replaces rms_norm (qwen38_inf2/model.py:54-57) as used by
 * DecoderLayer.forward (:918-930) and HeadStep.forward (:890-891), plus the e5m2 rounding of
 * fp8_round (:85-87) at the next linear.
 */
int q38_rmsnorm_quant(const void* x, int64_t ldx, const void* w, int64_t rows, int64_t n, float eps, void* y_bf16,
                      int64_t ldy, void* y_e5m2, int64_t ldq, q38_stream_t stream);

/*
 * y = bf16(bf16(rms_norm(x) * (1 + w)) / (1 + w_div)) for each of `rows` rows of n values (x, y bf16
 * with row strides ldx, ldy; w, w_div bf16 [n]): the MTP draft layer's output, its norm divided by the
 * model's final-norm weight (1 + w_div) so the head's final norm recovers it (MTPStep.forward,
 * qwen38_inf2/model.py:858-860).
 */
int q38_rmsnorm_divide(const void* x, int64_t ldx, const void* w, const void* w_div, int64_t rows, int64_t n, float eps,
                       void* y, int64_t ldy, q38_stream_t stream);

/*
 * MLP middle: h = e5m2(bf16(bf16(silu(g)) * u)) with g, u the bf16 gate and up projections
 * [rows, n] at gu and gu + n (row stride ld). Replaces silu(gate_proj(x)) * up_proj(x)
 * (qwen38_inf2/model.py:48-51, :259) and the NKI mlp_up epilogue (kernels.py:74-118).
 */
int q38_silu_mul_quant(const void* gu, int64_t ld, int64_t rows, int64_t n, void* y_e5m2, int64_t ldy,
                       q38_stream_t stream);

/*
 * y[r, o] = bf16(sum_k x[r, k] * w[o, k]) with BF16 x [rows, k] (contiguous) and a pre-tiled BF16
 * weight [n_out, k], fp32 accumulate on tcgen05 (kind::f16), split K as q38_fp8_gemm (same
 * workspace rules). Used for the gated delta rule's in_proj_b / in_proj_a, which stay BF16 and take
 * the unrounded normed input (qwen38_inf2/model.py:294-296, :333-337). With splits > 1 and a
 * workspace the split partials go through the workspace and the CTAs run in pairs on whichever SMs
 * are free (for a launch beside another kernel); without one, the splits of a tile form a thread-block
 * cluster. The result is the same bits either way.
 */
int q38_bf16_linear(const void* x, int64_t ldx, int64_t rows, int64_t k, const void* w, int64_t n_out, void* y,
                    int64_t ldy, int splits, void* workspace, size_t workspace_bytes, q38_stream_t stream);

/*
 * One decode token per row of the gated delta rule, everything between the input projections and
 * out_proj: causal conv window (kernel 4) + SiLU, q/k L2 norms (q / sqrt(dk)), key heads repeated to
 * value heads, beta = sigmoid(b), g = -exp(A_log) * softplus(a + dt_bias), the recurrent update
 * S = S*e^g*keep; delta = (v - S^T k) * beta; S += k delta^T; o = S^T q, and the gated RMS norm
 * times SiLU(z), rounded to e5m2 for out_proj. Replaces GatedDeltaNetStep.forward
 * (qwen38_inf2/model.py:347-374 with _split :322-331, _gates :333-337, _finish :339-345).
 *
 *   qkvz        bf16 [batch, ld_qkvz]: conv_dim qkv columns then value_dim z columns
 *   ab          bf16 [batch, ld_ab]: num_v_heads b columns then num_v_heads a columns
 *   conv_state  bf16 [batch, conv_dim, conv_kernel - 1], updated in place
 *   conv_weight bf16 [conv_dim, conv_kernel]
 *   a_log, dt_bias bf16 [num_v_heads]; norm_weight bf16 [head_v]
 *   state       bf16 [batch, num_v_heads, head_k, head_v], updated in place (rows with active 0
 *               keep theirs bit for bit)
 *   position    int32 [batch]; active float32 [batch]
 *   out         e5m2 [batch, ld_out], num_v_heads * head_v columns
 *   workspace   q38_gdn_decode_workspace_bytes(batch, num_k_heads, head_k) bytes, 16-byte aligned
 *               (the normalised q and k of each row's key heads between the two launches)
 */
size_t q38_gdn_decode_workspace_bytes(int64_t batch, int num_k_heads, int head_k);
int q38_gdn_decode(const void* qkvz, int64_t ld_qkvz, const void* ab, int64_t ld_ab, void* conv_state,
                   const void* conv_weight, const void* a_log, const void* dt_bias, const void* norm_weight,
                   void* state, const int32_t* position, const float* active, void* out, int64_t ld_out,
                   int64_t batch, int num_k_heads, int num_v_heads, int head_k, int head_v, int conv_kernel,
                   float eps, void* workspace, size_t workspace_bytes, q38_stream_t stream);

/*
 * A prefill chunk of one row (slot) through the gated delta rule: the causal conv over
 * [history * (start > 0), chunk] (bf16 products summed left to right in bf16), SiLU, L2 norms, the
 * gates masked to the first n_valid tokens, the chunked rule from the row's state * (start > 0), the
 * gated RMS norm times SiLU(z) rounded to e5m2 for out_proj; the row's state and conv state are
 * replaced by their values after the chunk (the conv state keeps inputs n_valid - 3 .. n_valid - 1 of
 * the window). Replaces GatedDeltaNetStep.prefill (qwen38_inf2/model.py:476-521, CPU branch; NKI
 * delta_prefill kernels.py:843-904) between its input and output projections.
 *
 *   qkvz, ab     as q38_gdn_decode, [tokens, ld] for the chunk's tokens
 *   conv_state   bf16 [state_rows, conv_dim, conv_kernel - 1]; state bf16 [state_rows, num_v_heads,
 *                head_k, head_v]: the slot's rows are read and replaced
 *   out          e5m2 [tokens, ld_out]
 *   workspace    q38_gdn_prefill_workspace_bytes(tokens, ...) bytes, 256-byte aligned
 */
size_t q38_gdn_prefill_workspace_bytes(int64_t tokens, int num_k_heads, int num_v_heads, int head_k, int head_v);
int q38_gdn_prefill_chunk(const void* qkvz, int64_t ld_qkvz, const void* ab, int64_t ld_ab, void* conv_state,
                          const void* conv_weight, const void* a_log, const void* dt_bias, const void* norm_weight,
                          void* state, int64_t slot, int64_t state_rows, int64_t tokens, int64_t start,
                          int64_t n_valid, void* out, int64_t ld_out, int num_k_heads, int num_v_heads, int head_k,
                          int head_v, int conv_kernel, float eps, void* workspace, size_t workspace_bytes,
                          q38_stream_t stream);

/*
 * Keys-first gated attention of a prefill chunk of one row: q/k RMS norms (1 + w), partial rotary,
 * queries scaled by head_dim^-0.5 in bf16; token t attends to cache positions < start and to chunk
 * tokens <= t; output times sigmoid(gate), e5m2 for o_proj. The chunk's keys and values are written to
 * the row's cache at start .. start + tokens - 1. Replaces FullAttentionStep.prefill
 * (qwen38_inf2/model.py:732-786 with blocked_attention :170-191; NKI prefill_attention
 * kernels.py:294-423) between its projections.
 *
 *   qkv      bf16 [tokens, ld_qkv], laid out as for q38_attn_decode
 *   cos, sin bf16 [tokens, rot_dim] for positions start .. start + tokens - 1
 *   k_cache, v_cache bf16 [cache_rows, num_kv_heads, max_seq, head_dim]
 *   out      e5m2 [tokens, ld_out]
 *   workspace q38_attn_prefill_workspace_bytes(tokens, num_q_heads, head_dim) bytes
 */
size_t q38_attn_prefill_workspace_bytes(int64_t tokens, int num_q_heads, int head_dim);
int q38_attn_prefill(const void* qkv, int64_t ld_qkv, const void* q_norm_weight, const void* k_norm_weight,
                     const void* cos, const void* sin, void* k_cache, void* v_cache, int64_t slot, int64_t cache_rows,
                     int64_t max_seq, int64_t tokens, int64_t start, void* out, int64_t ld_out, int num_q_heads,
                     int num_kv_heads, int head_dim, int rot_dim, float eps, void* workspace, size_t workspace_bytes,
                     q38_stream_t stream);

/*
 * q38_attn_prefill with the FP8 e4m3 cache (uint8 [cache_rows, num_kv_heads, max_seq, head_dim]): the
 * chunk's keys and values are written as e4m3 bytes of value / scale clamped to +-240, and every cached
 * key and value, the chunk's own included, is read back as bf16(e4m3 * scale) (FullAttentionStep.prefill
 * with kv_cache_format "fp8", qwen38_inf2/model.py:732-786 with _store / _load / _round_trip :579-593).
 */
int q38_attn_prefill_e4m3(const void* qkv, int64_t ld_qkv, const void* q_norm_weight, const void* k_norm_weight,
                          const void* cos, const void* sin, void* k_cache, void* v_cache, float k_scale, float v_scale,
                          int64_t slot, int64_t cache_rows, int64_t max_seq, int64_t tokens, int64_t start, void* out,
                          int64_t ld_out, int num_q_heads, int num_kv_heads, int head_dim, int rot_dim, float eps,
                          void* workspace, size_t workspace_bytes, q38_stream_t stream);

/*
 * K verify tokens per row through the gated delta rule with commit-on-accept: first the last verify
 * step's first accepted[b] tokens are committed to the row's state and conv state from the pending
 * buffers, then the K new tokens run from the committed state as one small chunk without changing it,
 * their updates (key, delta, log decay, conv input) replacing the pending buffers; out gets the gated
 * RMS norm times SiLU(z), e5m2, per token. Rows with active 0 keep their states exactly. Replaces
 * GatedDeltaNetStep.verify (qwen38_inf2/model.py:376-454) with _commit_and_read (:262-271; NKI
 * delta_verify_state kernels.py:936-968) between its projections.
 *
 *   qkvz, ab      as q38_gdn_decode with rows b * tokens + t
 *   pending_key   f32 [batch, tokens, num_v_heads, head_k]; pending_delta f32 [batch, tokens, num_v_heads,
 *                 head_v]; pending_decay f32 [batch, tokens, num_v_heads]; pending_input bf16 [batch, tokens,
 *                 conv_dim]: read (the commit), then replaced
 *   accepted      int32 [batch], 0 .. tokens; 0 after a decode or prefill step
 *   out           e5m2 [batch * tokens, ld_out]
 *   workspace     q38_gdn_verify_workspace_bytes(batch, tokens, num_k_heads, head_k) bytes, 16-byte aligned
 */
size_t q38_gdn_verify_workspace_bytes(int64_t batch, int tokens, int num_k_heads, int head_k);
int q38_gdn_verify_commit(const void* qkvz, int64_t ld_qkvz, const void* ab, int64_t ld_ab, void* conv_state,
                          const void* conv_weight, const void* a_log, const void* dt_bias, const void* norm_weight,
                          void* state, void* pending_key, void* pending_delta, void* pending_decay,
                          void* pending_input, const int32_t* position, const float* active, const int32_t* accepted,
                          void* out, int64_t ld_out, int64_t batch, int tokens, int num_k_heads, int num_v_heads,
                          int head_k, int head_v, int conv_kernel, float eps, void* workspace, size_t workspace_bytes,
                          q38_stream_t stream);

/*
 * K verify tokens per row of gated full attention with a BF16 KV cache: token t attends to cache
 * positions < position and to the step's own keys 0 .. t; the tokens' keys and values are written at
 * position .. position + tokens - 1 (rows with active 0 at the cache's last `tokens` positions).
 * Replaces FullAttentionStep.verify (qwen38_inf2/model.py:641-675; NKI verify_attention
 * kernels.py:468-488) between its projections.
 *
 *   qkv      bf16 [batch * tokens, ld_qkv], rows b * tokens + t, laid out as for q38_attn_decode
 *   cos, sin bf16 [batch * tokens, rot_dim]
 *   out      e5m2 [batch * tokens, ld_out]
 */
int q38_attn_verify(const void* qkv, int64_t ld_qkv, const void* q_norm_w, const void* k_norm_w, const void* cos,
                    const void* sin, void* k_cache, void* v_cache, int64_t max_seq, const int32_t* position,
                    const float* active, void* out, int64_t ld_out, int64_t batch, int tokens, int num_q_heads,
                    int num_kv_heads, int head_dim, int rot_dim, float eps, q38_stream_t stream);

/*
 * One decode token per row of gated full attention with a BF16 KV cache: q/k RMS norms (1 + w),
 * partial rotary on the first rot_dim dims, softmax attention over cache positions < position plus
 * the token's own key/value, times sigmoid(gate), rounded to e5m2 for o_proj; the token's key and
 * value are written at `position` (rows with active 0 write at max_seq - 1, as the reference does).
 * Replaces FullAttentionStep._project + forward (qwen38_inf2/model.py:565-577, :610-639) and the
 * NKI decode_attention (kernels.py:437-465, :491-644).
 *
 *   qkv      bf16 [batch, ld_qkv]: per q head [query head_dim | gate head_dim], then num_kv_heads
 *            keys, then num_kv_heads values
 *   cos, sin bf16 [batch, rot_dim]
 *   k_cache, v_cache bf16 [batch, num_kv_heads, max_seq, head_dim]
 *   out      e5m2 [batch, ld_out], num_q_heads * head_dim columns
 *   row_order int32 [batch], a permutation of the rows (q38_attn_row_order's), or NULL: the order in
 *            which the rows are scheduled. It changes no result, only how the grid's tail is filled.
 */
int q38_attn_decode(const void* qkv, int64_t ld_qkv, const void* q_norm_w, const void* k_norm_w, const void* cos,
                    const void* sin, void* k_cache, void* v_cache, int64_t max_seq, const int32_t* position,
                    const float* active, void* out, int64_t ld_out, int64_t batch, int num_q_heads,
                    int num_kv_heads, int head_dim, int rot_dim, float eps, const int32_t* row_order,
                    q38_stream_t stream);

/*
 * Gated full attention against a cache of any length, split along the cache: decode (tokens = 1) or
 * verify (tokens = K, each token attending to cache positions < position and to the step's own tokens
 * up to itself), with a BF16 cache or an FP8 e4m3 cache with static scales (kv_format Q38_KV_E4M3:
 * the cache holds e4m3 bytes of value / scale clamped to +-240 and reads back as bf16(e4m3 * scale),
 * the step's own keys and values taking the same round trip). The output and the cache writes are
 * those of q38_attn_decode / q38_attn_verify. Three launches: per (chunk of the cache, row, KV head) the
 * bf16 scores and their softmax statistics, then the bf16 weights times the values, then per (row, KV
 * head) the chunks' partials summed in chunk order, the own term and the gate. Replaces
 * FullAttentionStep.forward / verify (qwen38_inf2/model.py:610-675) with _store / _load / _round_trip
 * (:579-593) and the NKI decode / verify attention (kernels.py:437-488, :491-644) for long caches.
 *
 *   qkv, cos, sin, position, active, out   as q38_attn_verify (rows b * tokens + t)
 *   k_cache, v_cache   [batch, num_kv_heads, max_seq, head_dim], bf16 or e4m3 bytes
 *   k_scale, v_scale   the FP8 cache's scales (ignored for BF16)
 *   workspace          q38_attn_split_workspace_bytes(...) bytes, 16-byte aligned
 * groups x tokens <= 32, tokens <= 8.
 */
#define Q38_KV_BF16 0
#define Q38_KV_E4M3 1
size_t q38_attn_split_workspace_bytes(int64_t batch, int num_q_heads, int num_kv_heads, int tokens, int64_t max_seq,
                                      int head_dim);
int q38_attn_split(const void* qkv, int64_t ld_qkv, const void* q_norm_w, const void* k_norm_w, const void* cos,
                   const void* sin, void* k_cache, void* v_cache, int kv_format, float k_scale, float v_scale,
                   int64_t max_seq, const int32_t* position, const float* active, void* out, int64_t ld_out,
                   int64_t batch, int tokens, int num_q_heads, int num_kv_heads, int head_dim, int rot_dim, float eps,
                   void* workspace, size_t workspace_bytes, q38_stream_t stream);

/*
 * The longest-first schedule for q38_attn_decode: row_order int32 [batch] = the rows by decreasing
 * count of visible cache positions (min(position, max_seq) for active rows, none for inactive ones),
 * in tiles of 32, ties by row index. Positions and activity are the same for every attention layer
 * of a decode step, so one call per step serves all of them. batch <= 4096. No reference counterpart
 * (scheduling only).
 */
int q38_attn_row_order(const int32_t* position, const float* active, int64_t max_seq, int64_t batch,
                       int32_t* row_order, q38_stream_t stream);

/*
 * Tensor-parallel communicator for the fused GEMM + all-reduce. Each rank creates one exchange region
 * (cudaMalloc) holding the residual stream x bf16 [max_tokens, hidden], the receive slots and the
 * arrival flags; q38_comm_ipc_handle exports it, the host passes every rank's handle to every rank
 * (the handles of ranks 0 .. world - 1, back to back), and q38_comm_connect maps the peers' regions
 * over NVLink (CUDA IPC with peer access). No reference counterpart: it stands in for the NxD
 * collective plumbing behind the reference's all_reduce (qwen38_inf2/neuron.py:9, model.py:44-45).
 */
typedef void* q38_comm_t;
int q38_comm_init(int rank, int world, int64_t max_tokens, int64_t hidden, q38_comm_t* comm);
size_t q38_comm_ipc_handle_bytes(void);
int q38_comm_ipc_handle(q38_comm_t comm, void* handle, size_t handle_bytes);
int q38_comm_connect(q38_comm_t comm, const void* handles);
void* q38_comm_residual(q38_comm_t comm);  /* this rank's x, bf16 [max_tokens, hidden] */
int q38_comm_destroy(q38_comm_t comm);

/*
 * x += all_reduce(bf16(e5m2(x_q) @ W^T)) over the communicator's ranks, in one kernel per rank. Each
 * token row of the output has an owner rank that sums every rank's bf16 partial of it in rank order
 * (fp32, one bf16 rounding) and adds the residual (bf16). With 2 ranks both own every row: each pushes
 * its whole partial into the other's `part` slot over NVLink and both reduce (one crossing, no result
 * traffic). With more, row t is owned by rank t % world: the others push their partials of it to the
 * owner, which writes the new row into every rank's x directly. Data moves as plain 16-byte stores; a CTA
 * publishes each step with a system-scope release of the call's epoch into a per-CTA flag at the
 * receiver, which acquires it before reading. The epoch advances on the device (last CTA of the call)
 * and slots alternate by epoch parity, so calls replay inside CUDA graphs.
 * Every rank makes the same sequence of calls. x is the communicator's residual stream (rows 0 .. tokens - 1), so
 * features == hidden. Replaces the row-parallel projection plus all-reduce of o_proj / out_proj /
 * down_proj (qwen38_inf2/model.py:259, :374, :639 with the NxD reduce, neuron.py:9). Needs the whole
 * grid resident (returns Q38_ERR_UNSUPPORTED otherwise) and at most 8 K splits; a wait on a peer that
 * runs out (2 s) records Q38_ERR_TIMEOUT in the device error word.
 */
int q38_fp8_gemm_allreduce(const void* x_q, int64_t tokens, int64_t k, const void* w, const void* w_sf,
                           int64_t features, int splits, q38_comm_t comm, q38_stream_t stream);

/*
 * The MLP's gate and up projections with SiLU(gate) * up fused into the epilogue: x_q e5m2 [tokens, k]
 * times the FP8 weight whose 128-row tiles hold 64 gate rows then the 64 matching up rows
 * (FP8Weight.interleave_rows), y e5m2 [tokens, ldy] with features / 2 columns:
 * y = e5m2(bf16(bf16(g * bf16(sigmoid(g))) * u)), g and u the bf16 projections. Replaces
 * `silu(gate_proj(x)) * up_proj(x)` and down_proj's input rounding (qwen38_inf2/model.py:259, :85-87;
 * NKI mlp_up kernels.py:74-118).
 */
int q38_fp8_gemm_silu(const void* x_q, int64_t tokens, int64_t k, const void* w, const void* w_sf, int64_t features,
                      void* y, int64_t ldy, q38_stream_t stream);

/*
 * Save / restore of one slot's recurrent states for prefix reuse: row src_row of each of n_buffers
 * device buffers copied to row dst_row, in one launch (more than 96 buffers take more launches).
 * buffers[i] is a contiguous device array of rows[i] rows of row_bytes[i] bytes (a gated-delta layer's
 * recurrent state [rows, heads, dk, dv] or conv state [rows, conv_dim, kernel - 1]); the three arrays
 * are host memory. src_row == dst_row copies nothing. Replaces GatedDeltaNetStep.copy_states
 * (qwen38_inf2/model.py:456-464) over every layer (Qwen38Step.forward, model.py:987-990).
 */
int q38_copy_state_rows(void* const* buffers, const int64_t* row_bytes, const int64_t* rows, int n_buffers,
                        int64_t src_row, int64_t dst_row, q38_stream_t stream);

/*
 * lm_head candidates: maxima[r, j] = max over the `group` vocab rows v in group j of
 * sum_k x[r, k] * w[v, k], fp32 (x bf16 [rows, k], w bf16 [vocab, k] pre-tiled). Replaces HeadStep.forward's
 * logits and group maxima (qwen38_inf2/model.py:890-900) and the NKI lm_head_group_maxima
 * (kernels.py:126-172). group must be 32.
 */
int q38_lm_head_groupmax(const void* x, int64_t rows, int64_t k, const void* w, int64_t vocab, int group,
                         float* maxima, int64_t ld_max, q38_stream_t stream);

/*
 * The head's exact recheck on the device (ChipHead.next_tokens, qwen38_inf2/generate.py:186-208): for each
 * of `rows` rows, the `candidates` groups with the largest `maxima` (float [rows, ldm], `groups` groups of
 * 32 over the whole vocabulary; ties to the lower group), each of their 32 vocabulary rows scored in fp32
 * against rms_norm(hidden.float(), norm_w) (hidden bf16 [rows, ldh], norm_w bf16 [hidden_size]), and the
 * best token: the largest logit in a group (its first row on ties), groups taken in candidate order, a
 * strictly larger logit replacing the best. lm_head is this rank's vocabulary rows [vocab_first,
 * vocab_first + vocab_rows) in the tiled BF16 layout of q38_lm_head_groupmax; candidate groups outside
 * them score -inf with token -1. Outputs: tokens int32 [rows] (-1 where no logit is finite), and/or the
 * per-candidate slot_logits float / slot_tokens int32 [rows, candidates] for combining ranks (a max across
 * ranks, then q38_lm_head_pick). group must be 32, candidates 1..8.
 */
int q38_lm_head_recheck(const void* hidden, int64_t ldh, const void* norm_w, float eps, const float* maxima,
                        int64_t ldm, int64_t groups, const void* lm_head, int64_t vocab_first, int64_t vocab_rows,
                        int64_t hidden_size, int group, int candidates, int64_t rows, float* slot_logits,
                        int32_t* slot_tokens, int32_t* tokens, q38_stream_t stream);
/* out[i] = table[ids[i]]: bf16 rows of `hidden` values of the embedding table [vocab, hidden] for n int32
 * ids, into out [n, ldo] (ChipHead.embed_batch, qwen38_inf2/generate.py:183-184). An id outside the table
 * gives a zero row and records Q38_ERR_ARG in the device error word. */
int q38_embed_rows(const void* table, int64_t vocab, int64_t hidden, const int32_t* ids, int64_t n, void* out,
                   int64_t ldo, q38_stream_t stream);
/* tokens[r] from the per-candidate results of q38_lm_head_recheck (maximised across ranks): the candidate
 * slots in order, a strictly larger logit replacing the best so far; -1 where none is valid. */
int q38_lm_head_pick(const float* slot_logits, const int32_t* slot_tokens, int candidates, int64_t rows, int32_t* tokens,
                     q38_stream_t stream);

#ifdef __cplusplus
}
#endif

#endif /* Q38_H */

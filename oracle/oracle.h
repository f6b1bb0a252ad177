/* Test infrastructure — NOT part of the product.
 *
 * CPU restatement (IEEE double arithmetic, FP32 rounding at the reference's
 * stage boundaries) of welvet.metal's multi-head-attention forward path and of
 * the weight codecs it uses. Only tests/, __graft_entry__.smoke() and bench.py's
 * CPU-baseline / reference legs load this library, and only as the checker.
 *
 * Stage boundaries follow src/layers/mha/mha.cpp:138-205: q/k/v are rounded to
 * FP32 by the Dense projections, attention runs at (emulated) f64 and rounds
 * its output to FP32, and the output projection rounds to FP32 again.
 */
#ifndef WELVET_ORACLE_H
#define WELVET_ORACLE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Mirrors welvet::mha::Config (include/welvet/mha.hpp:39-64) plus the sequence
 * mode. per_sequence = 0 reproduces the reference's stream semantics
 * (shaders/ops_mha.metal:58-80: positions continue across the batch and keys
 * come from a ring of max_seq_len slots); per_sequence = 1 treats each batch
 * row as an independent sequence starting at position 0. */
typedef struct oracle_mha_cfg {
  int32_t d_model, num_heads, num_kv_heads, head_dim, max_seq_len;
  int32_t mask, pos, softmax, window, prefix_len, window_causal;
  double rope_theta, scale_override;
  int32_t per_sequence;
} oracle_mha_cfg;

/* Defaults and checks of validate() (src/layers/mha/mha.cpp:63-94).
 * Returns the reference status code (0 ok, 1 invalid). */
int32_t oracle_mha_validate(oracle_mha_cfg* cfg, char* msg, int32_t msg_len);

/* y[m,n] = fl32( sum_k double(W[n,k]) * double(x[m,k]) ), k ascending
 * (shaders/welvet_dense.metal:54-85, Linear activation, no bias). */
void oracle_dense(const float* x, const float* W, float* y, int64_t M, int64_t K, int64_t N,
                  int32_t threads);

/* Attention forward (shaders/ops_mha.metal:31-127). q [B*T, qd], k/v [B*T, kd],
 * out [B*T, qd], all FP32; RoPE is applied inside, as in the reference. */
int32_t oracle_attention(const oracle_mha_cfg* cfg, int32_t batch, int32_t seq, const float* q,
                         const float* k, const float* v, float* out, int32_t threads);

/* Full MHA forward (src/layers/mha/mha.cpp:138-205) on already-decoded FP32 weights
 * Wq [qd,d], Wk/Wv [kd,d], Wo [d,qd]; x [B*T,d]; pre [B*T,qd]; post [B*T,d].
 * q_out/k_out/v_out (optional, may be NULL) receive the FP32 projections. */
int32_t oracle_mha_forward(const oracle_mha_cfg* cfg, int32_t batch, int32_t seq, const float* Wq,
                           const float* Wk, const float* Wv, const float* Wo, const float* x,
                           float* pre, float* post, float* q_out, float* k_out, float* v_out,
                           int32_t threads);

/* Decode (extension; the reference has no KV cache): one new token per sequence b
 * at position ctx_len[b]. k_cache/v_cache hold, per sequence, cache_stride rows of
 * kd values, already position-encoded (keys after RoPE), rows 0..ctx_len[b]-1 valid.
 * The new token's q/k get RoPE at position ctx_len[b]; it attends to the cached rows
 * and to itself (causal, per-sequence). x_new [B,d]; pre [B,qd]; post [B,d];
 * k_new/v_new (optional) receive the new token's key (after RoPE) and value. */
int32_t oracle_mha_decode(const oracle_mha_cfg* cfg, int32_t batch, const int32_t* ctx_len,
                          int64_t cache_stride, const float* k_cache, const float* v_cache,
                          const float* Wq, const float* Wk, const float* Wv, const float* Wo,
                          const float* x_new, float* pre, float* post, float* k_new,
                          float* v_new, int32_t threads);

/* ---- codecs (src/core/float_codecs.cpp, src/weights/native_codec.cpp) ---- */
uint16_t oracle_bf16_encode(float f);  /* truncating, float_codecs.cpp:53 */
float oracle_bf16_decode(uint16_t h);  /* float_codecs.cpp:55 */
uint16_t oracle_f16_encode(float f);   /* float_codecs.cpp:23-35 */
float oracle_f16_decode(uint16_t h);   /* float_codecs.cpp:37-51 */
uint8_t oracle_e4m3_encode(float f);   /* float_codecs.cpp:57-97 */
float oracle_e4m3_decode(uint8_t b);   /* float_codecs.cpp:99-117 */
uint8_t oracle_e5m2_encode(float f);   /* float_codecs.cpp:119-158 */
float oracle_e5m2_decode(uint8_t b);   /* float_codecs.cpp:160-181 */
float oracle_nf4_level(int32_t code);  /* kNf4, native_codec.cpp:93-110 */

/* FormatNone encode of one weight matrix (native_codec.cpp:189-560 for the dtypes
 * below). Returns bytes written to `out` (caller sizes it as 8*n), or -2 for a dtype
 * this restatement does not cover. scale as WeightStore::scale. */
int64_t oracle_encode(int32_t dtype, const float* w, int64_t n, uint8_t* out, float* scale);
/* weight_at() decode of every element (native_codec.cpp:562-813). */
int32_t oracle_decode(int32_t dtype, const uint8_t* raw, int64_t n, float scale, float* out);
// decode(encode(w)) for every FormatNone dtype 0-33 (0 ok, -2 unsupported).
int32_t oracle_roundtrip(int32_t dtype, const float* w, int64_t n, float* out);

/* Extension formats (no reference counterpart; element codes use the reference
 * converters above):
 * FP8-E4M3 with one FP32 scale per output row: scale[r] = absmax(row)/448 (1 if 0),
 * code = e4m3_encode(w / scale[r]); decode = e4m3_decode(code) * scale[r].
 * NF4 with one FP32 absmax per 64 consecutive elements (1 if 0), code = nearest kNf4
 * level of w/absmax (first minimum), two codes per byte, low nibble = even element;
 * decode = kNf4[code] * absmax. */
void oracle_fp8_rowscale_encode(const float* w, int64_t rows, int64_t cols, uint8_t* codes,
                                float* scales);
void oracle_fp8_rowscale_decode(const uint8_t* codes, const float* scales, int64_t rows,
                                int64_t cols, float* out);
void oracle_nf4_block_encode(const float* w, int64_t n, int32_t block, uint8_t* packed,
                             float* absmax);
void oracle_nf4_block_decode(const uint8_t* packed, const float* absmax, int64_t n, int32_t block,
                             float* out);

/* welvet_mha_normalbp_f32 (src/interop/c_abi.cpp:249-325) on decoded FP32 weights,
 * the reference's stream semantics: forward, MSE loss/gradient against
 * grad_or_target (use_target) or grad_or_target as dL/dpost, mha::backward_f32
 * (dense gradients, op_attention backward), SGD with rate lr for Float32 storage
 * (sgd_f32 = 1; otherwise the step is not restated and 2 is returned when lr != 0),
 * weight export. dW / W_after = concat(Q, K, V, O). */
int32_t oracle_mha_normalbp(const oracle_mha_cfg* cfg, int32_t batch, int32_t seq, const float* Wq,
                            const float* Wk, const float* Wv, const float* Wo, const float* x,
                            const float* grad_or_target, int32_t use_target, double lr, int32_t sgd_f32,
                            float* pre, float* post, float* dX, float* dW, float* W_after, double* loss,
                            int32_t threads);

/* Transformer-block forwards (block_oracle.cpp), on decoded FP32 weights. */
/* act_value of shaders/ops_common.metal:83-105 (Activation ids: -1 Linear, 0 ReLU,
 * 1 Silu, 2 GELU, 3 Tanh, 4 Sigmoid, 5 LeakyReLU, 6 ReLU2). */
float oracle_act_value(float v, int32_t act);
/* RMSNorm (layernorm = 0) / LayerNorm (1) over rows of dim: pre = x-hat, post =
 * x-hat * gamma (+ beta) (shaders/ops_norm.metal:2-26); eps <= 0 -> the validate()
 * default (1e-6 / 1e-5). */
int32_t oracle_norm_forward(int32_t layernorm, int64_t rows, int32_t dim, double eps,
                            const float* gamma, const float* beta, const float* x, float* pre,
                            float* post);
/* SwiGLU (swiglu.cpp:93-143): pre = h = silu(x Gate^T) * (x Up^T), post = h Down^T. */
int32_t oracle_swiglu_forward(int64_t tokens, int32_t in, int32_t inter, const float* Gate,
                              const float* Up, const float* Down, const float* x, float* pre,
                              float* post, int32_t threads);
/* Embedding (ops_embedding.metal:1-8): row abs(int(x[t*in_last])) % vocab of W, act applied. */
int32_t oracle_embedding_forward(int64_t tokens, int32_t vocab, int32_t emb, int32_t in_last,
                                 int32_t act, const float* W, const float* x, float* pre,
                                 float* post);

#ifdef __cplusplus
}
#endif
#endif

#pragma once

/* welvet B200 extension ABI (libwelvet_b200.so). Not part of the reference's
 * include/welvet_c.h; every entry point states the reference interface it
 * generalises, or that it has none.
 *
 * Conventions: plain pointers and sizes only. `on_device` = 1 means the buffer
 * arguments are CUDA device pointers and the call is asynchronous on `stream`
 * (a cudaStream_t, NULL = legacy default stream); 0 means host pointers, copied
 * in and out inside the call, which returns after the results are on the host.
 * Activations are FP32 when the layer's precision is 0 and BF16 (uint16 bit
 * patterns) when it is 1. Statuses follow welvet_c.h (code 4 = CUDA/NCCL error,
 * including a device-side timeout reported by a kernel's error word). */

#include "welvet_c.h"

#ifdef __cplusplus
extern "C" {
#endif

/* welvet::mha::Config (reference include/welvet/mha.hpp:39-64) plus the B200
 * execution choices. seq_mode 0 keeps the reference's stream semantics
 * (shaders/ops_mha.metal:58-80); 1 treats each batch row as an independent
 * sequence starting at position 0 (the usual LLM batch). */
typedef struct welvet_b200_mha_config {
  int32_t d_model, num_heads, num_kv_heads, head_dim, max_seq_len;
  int32_t mask, pos, softmax, window, prefix_len, window_causal;
  double rope_theta, scale_override;
  int32_t seq_mode;      /* 0 stream (reference), 1 per sequence */
  int32_t precision;     /* 0 FP32 activations (3xTF32 tensor cores), 1 BF16 */
  int32_t weight_format; /* precision 1 only: 0 BF16 (from the decoded dtype), 1 FP8-E4M3 with
                            one FP32 scale per output channel, 2 NF4 with one FP32 absmax per
                            64 weights, 3 the reference's FormatNone codes of the mount's dtype
                            kept resident (Int8 9, Int4 14 or FP4 16; per-tensor scale) and
                            dequantised inside the GEMM mainloop */
  int32_t head_begin, head_count; /* this rank's query heads; head_count 0 = all heads */
  int32_t device;                 /* CUDA ordinal; -1 = current device */
} welvet_b200_mha_config;

typedef struct welvet_b200_mha welvet_b200_mha;
typedef struct welvet_b200_kv welvet_b200_kv;

/* Fills `cfg` with the defaults of reference mha::decoder_causal
 * (src/layers/mha/mha.cpp:96-106): causal mask, RoPE, theta 10000. */
WELVET_API void welvet_b200_mha_config_default(welvet_b200_mha_config* cfg, int32_t d_model,
                                               int32_t num_heads, int32_t num_kv_heads);

/* Resident layer (generalises reference mha::new_configured,
 * src/layers/mha/mha.cpp:108-136, plus the Dense resident mount of
 * src/layers/dense/dense.cpp:50-97): weights are encoded once to `dtype`
 * (FormatNone ids of reference include/welvet/dtype.hpp), decoded on the GPU and
 * kept in HBM in the layer's compute format. Q/K/V/O are the full FP32 matrices
 * (host or device per weights_on_device); a head shard keeps only its slices. */
WELVET_API welvet_status welvet_b200_mha_mount(const welvet_b200_mha_config* cfg, int32_t dtype,
                                               const float* Q, const float* K, const float* V,
                                               const float* O, int32_t weights_on_device,
                                               welvet_b200_mha** out);
WELVET_API void welvet_b200_mha_release(welvet_b200_mha* layer);

/* Forward of reference mha::forward (src/layers/mha/mha.cpp:138-205) on a resident
 * layer: x [batch*seq, d_model] -> pre [batch*seq, q_dim_local], post
 * [batch*seq, d_model]. pre may be NULL. With a communicator attached, post is the
 * sum over ranks (all-reduce after the row-sharded output projection). */
WELVET_API welvet_status welvet_b200_mha_forward(welvet_b200_mha* layer, int32_t batch,
                                                 int32_t seq, const void* x, void* pre, void* post,
                                                 int32_t on_device, void* stream);

/* Forward with row-sharded host buffers (no reference counterpart: the reference
 * is single-device). For a head-sharded layer with a communicator of N ranks in
 * per-sequence mode: every rank passes its own batch_local sequences (rank r holds
 * sequences [r * batch_local, (r + 1) * batch_local) of the whole batch of
 * N * batch_local), x [batch_local*seq, d_model] in and post [batch_local*seq,
 * d_model] out, host memory (pinned for full speed), synchronous. post receives the
 * sum over ranks of those rows, as welvet_b200_mha_forward would give for them. The
 * layer all-gathers the input rows and reduce-scatters the output rows over NVLink,
 * so each GPU moves 1/N of x and post over PCIe. Without a communicator (or with
 * one rank) it is the host-buffer forward of batch_local sequences. */
WELVET_API welvet_status welvet_b200_mha_forward_rows(welvet_b200_mha* layer, int32_t batch_local,
                                                      int32_t seq, const void* x, void* post);

/* Output collective of welvet_b200_mha_forward with device buffers and a
 * communicator of N ranks (no reference counterpart: the reference is
 * single-device). mode 0 (default): all-reduce, every rank's post holds every
 * summed row. mode 1: reduce-scatter, half the NVLink bytes: the forward runs the
 * batch in chunks of whole sequences (4 chunks of ceil(batch/4) sequences when
 * batch > 1 in per-sequence mode, else one chunk of all rows), each chunk's rows
 * must divide by N, and rank r's post holds the summed rows [c0 + r*n/N,
 * c0 + (r+1)*n/N) of each chunk (c0 its first row, n its rows); the other rows hold
 * this rank's partial sums (a sequence-sharded output, as a sequence-parallel
 * next layer consumes it). mode 2: the same sequence-sharded output through an
 * exchange of the attention output instead of the partial sums: each chunk's
 * attention rows [c0 + r*n/N, c0 + (r+1)*n/N) of every rank's heads go to rank r
 * (copy engines over NVLink peer memory, q_dim/d_model of mode 1's bytes), which
 * runs the output projection over every head for its own rows only, so its rows
 * equal the single-GPU layer's bit for bit; the other rows of post are not
 * written. Needs BF16 activations, BF16 (weight format 0) weights, equal head
 * shards and no `pre`; otherwise the call runs as mode 1. The first mode-2 forward
 * gathers every rank's Wo columns (d_model x q_dim BF16 per rank) and sets up the
 * receive areas: collective, like every forward with a communicator.
 * Host-buffer forwards and decode always all-reduce. Code 1 for another mode. */
WELVET_API welvet_status welvet_b200_mha_set_output_mode(welvet_b200_mha* layer, int32_t mode);

/* Reads and clears the device error word of the layer's device after a
 * synchronisation; code 4 with the kernel's reason when a device-side bounded wait
 * expired or a bound check failed. No reference counterpart. */
WELVET_API welvet_status welvet_b200_mha_check(welvet_b200_mha* layer);

/* ---- KV cache (no reference counterpart: the reference has no KV cache) ----
 * Paged: pages of 16 tokens, pools laid out [page][kv_head][16][head_dim] in the
 * layer's precision; each of max_batch sequences owns ceil(max_ctx/16) pages. */
WELVET_API welvet_status welvet_b200_kv_create(welvet_b200_mha* layer, int32_t max_batch,
                                               int32_t max_ctx, welvet_b200_kv** out);
WELVET_API void welvet_b200_kv_release(welvet_b200_kv* kv);
/* Sets the cached length of `batch` sequences to ctx_len and writes their rows
 * [0, ctx_len) from k, v [batch, ctx_len, kv_dim_local] (keys as cached, i.e. after
 * position encoding). k/v NULL only sets the lengths. */
WELVET_API welvet_status welvet_b200_kv_fill(welvet_b200_kv* kv, int32_t batch, int32_t ctx_len,
                                             const void* k, const void* v, int32_t on_device,
                                             void* stream);
/* Per-sequence prefill: forward of `seq` tokens per sequence (positions 0..seq-1)
 * that also writes their keys/values into the cache (cached length := seq). */
WELVET_API welvet_status welvet_b200_mha_prefill(welvet_b200_mha* layer, welvet_b200_kv* kv,
                                                 int32_t batch, int32_t seq, const void* x,
                                                 void* pre, void* post, int32_t on_device,
                                                 void* stream);
/* One decode step: x_new [batch, d_model], one token per sequence at position
 * ctx_len[b]; appends its key/value, attends over the cache (split-KV), then the
 * output projection. pre [batch, q_dim_local] may be NULL. */
WELVET_API welvet_status welvet_b200_mha_decode(welvet_b200_mha* layer, welvet_b200_kv* kv,
                                                int32_t batch, const void* x_new, void* pre,
                                                void* post, int32_t on_device, void* stream);

/* ---- multi-GPU (no reference counterpart: the reference is single-device) ----
 * One process per GPU. Rank 0 creates the id, the caller distributes it; every
 * rank attaches an NCCL communicator to its head-sharded layer. */
WELVET_API welvet_status welvet_b200_comm_unique_id(uint8_t id[128]);
WELVET_API welvet_status welvet_b200_comm_attach(welvet_b200_mha* layer, const uint8_t id[128],
                                                 int32_t nranks, int32_t rank);

/* ---- kernel-level entry points (device pointers, asynchronous on `stream`) ----
 * Used by the parity tests and the benchmark to exercise one kernel at a time.
 * No reference counterparts except where cited. Each returns code 4 on a launch
 * failure; device-side faults show up in welvet_b200_device_check. */

/* C[M,N] = A[M,K] B[N,K]^T (reference Dense MatVec, shaders/welvet_dense.metal:54-85).
 * kind 0: A,B bf16 -> out bf16 (out_bf16=1) or fp32; kind 1: 3xTF32 with A=(a,a_lo),
 * B=(b,b_lo) fp32 TF32 splits -> out fp32; kind 2: A bf16, B FP8-E4M3 codes with
 * per-row scale b_scale [N], decoded by the hardware E4M3 conversion: equal to the
 * reference decoder except that subnormal codes give their IEEE value (the reference
 * gives +-0; below 2^-6/448 of the row's absmax) and 0x7f/0xff are not accepted
 * (neither encoder emits them); a mounted layer normalises its codes so that its
 * dequantised weights equal the reference decoder's exactly; kind 3: A bf16, B NF4
 * packed [N, K/2] with b_scale [N, K/64]; kinds 4 / 5 / 6: A bf16, B the
 * reference's FormatNone Int8 codes [N, K] / Int4 codes [N, K/2] / FP4 (E2M1) codes
 * [N, K/2] (src/weights/native_codec.cpp pack_native, two per byte low nibble first)
 * dequantised in shared memory inside the mainloop, b_scale [N] the per-row scale
 * applied in the epilogue (may be NULL for FP4). */
WELVET_API welvet_status welvet_b200_gemm(int32_t kind, int32_t M, int32_t N, int32_t K,
                                          const void* a, const void* a_lo, const void* b,
                                          const void* b_lo, const float* b_scale, void* out,
                                          int32_t out_bf16, void* stream);
/* FP32 -> (hi, lo) TF32 split, hi + lo == x exactly. */
WELVET_API welvet_status welvet_b200_split_tf32(const float* x, float* hi, float* lo, int64_t n,
                                                void* stream);
/* Attention forward over token-major q [*, q_dim], k/v [*, kv_dim] (RoPE already
 * applied) -> out [*, q_dim] (reference op_attention forward,
 * shaders/ops_mha.metal:31-127). impl 0 = best available, 1 = CUDA-core kernel,
 * 2 = tensor-core kernel (fails when unsupported; the persistent form, one CTA per
 * SM looping over query tiles), 3 = tensor-core kernel on CTA pairs (head_dim 128,
 * seq a multiple of 256), 4 = tensor-core kernel with one CTA per query tile. The
 * persistent form counts its tiles in one per-device word: calls of impl 0/2 on
 * one device must not overlap in time (one stream, or ordered streams). */
WELVET_API welvet_status welvet_b200_attention(const welvet_b200_mha_config* cfg, int32_t batch,
                                               int32_t seq, const void* q, const void* k,
                                               const void* v, void* out, int32_t impl,
                                               void* stream);
/* The same forward for an FP32 configuration on the tensor cores (3xTF32, head_dim
 * 64): q/k/v given as their TF32 split (hi, lo from welvet_b200_split_tf32, same
 * layouts as above); out FP32, and its TF32 split into out_hi / out_lo when both
 * are given. Code 2 when the configuration is outside the kernel (head_dim,
 * stream ring wrap, alignment). Reference: shaders/ops_mha.metal:31-127. */
WELVET_API welvet_status welvet_b200_attention_tf32(const welvet_b200_mha_config* cfg, int32_t batch,
                                                    int32_t seq, const float* q_hi, const float* q_lo,
                                                    const float* k_hi, const float* k_lo,
                                                    const float* v_hi, const float* v_lo, float* out,
                                                    float* out_hi, float* out_lo, void* stream);
/* Codec kernels, bit-exact to the reference converters
 * (src/core/float_codecs.cpp, src/weights/native_codec.cpp:189-813):
 * roundtrip: out = decode(encode(w)) for any FormatNone dtype 0-33 (per-tensor
 * absmax / min / max computed on the device; out may equal w); encode/decode: the
 * stored bytes of dtypes 0-5 and 26 (nf4 scale = absmax); encode also dtypes 9, 14
 * and 16 (Int8 / Int4 / FP4 bytes, the per-tensor scale to scale_out[0]). */
WELVET_API welvet_status welvet_b200_codec_roundtrip(int32_t dtype, const float* w, float* out,
                                                     int64_t n, void* stream);
WELVET_API welvet_status welvet_b200_codec_encode(int32_t dtype, const float* w, void* codes,
                                                  float* scale_out, int64_t n, void* stream);
WELVET_API welvet_status welvet_b200_codec_decode(int32_t dtype, const void* codes,
                                                  const float* scale, float* out, int64_t n,
                                                  void* stream);
/* Extension weight formats (encode on the GPU; out_bf16 selects the decode type). */
WELVET_API welvet_status welvet_b200_fp8_rowscale_encode(const float* w, int32_t rows,
                                                         int32_t cols, uint8_t* codes,
                                                         float* scales, void* stream);
WELVET_API welvet_status welvet_b200_fp8_rowscale_decode(const uint8_t* codes,
                                                         const float* scales, int32_t rows,
                                                         int32_t cols, void* out,
                                                         int32_t out_bf16, void* stream);
WELVET_API welvet_status welvet_b200_nf4_block_encode(const float* w, int64_t n, uint8_t* packed,
                                                      float* absmax, void* stream);
WELVET_API welvet_status welvet_b200_nf4_block_decode(const uint8_t* packed, const float* absmax,
                                                      int64_t n, void* out, int32_t out_bf16,
                                                      void* stream);
/* Deterministic synthetic data on the device: element i of counter stream `seed`
 * (SplitMix64), kind 0 uniform(-a, a), kind 1 normal(0, a). */
WELVET_API welvet_status welvet_b200_fill_synthetic(void* dst, int32_t is_bf16, int64_t n,
                                                    uint64_t seed, uint64_t offset, int32_t kind,
                                                    double a, void* stream);
/* Reads and clears the current device's error word (synchronises the device). */
WELVET_API welvet_status welvet_b200_device_check(void);
/* Bounded-wait probe (no reference counterpart; the reference reports failures as
 * status codes, include/welvet/status.hpp:8-30, and this checks the device side of
 * that contract): launches one kernel whose thread waits on an mbarrier that
 * nothing arrives at, through the bounded wait every pipeline kernel here uses,
 * with limit_ns (1 ns .. 10 s) instead of the library's 4 s. The wait runs out,
 * the kernel records "device wait timeout" in the current device's error word and
 * returns without trapping; welvet_b200_device_check then returns code 4 and the
 * device stays usable. Code 1 for a limit out of range. */
WELVET_API welvet_status welvet_b200_wait_probe(uint64_t limit_ns, void* stream);
/* Number of kernel launches this library issued since the last reset
 * (benchmark accounting). No reference counterpart. */
WELVET_API int64_t welvet_b200_launch_count(int32_t reset);
/* Live per-kernel timing (no reference counterpart; the reference times whole calls
 * with steady_clock, tools/dense_fwd/main.cpp:198-216). When enabled, each hot kernel
 * of forward / decode is bracketed by CUDA events on its launch stream.
 * welvet_b200_profile_read synchronises and returns, per kernel id, the summed
 * milliseconds and launch counts (14 slots: 0 QKV GEMM, 1 prefill attention, 2 O GEMM,
 * 3 decode attention, 4 decode QKV GEMM, 5 decode O GEMM, 6 all-reduce, 7 other,
 * 8 SwiGLU Gate|Up GEMM, 9 SwiGLU Down GEMM, 10 RMSNorm/LayerNorm, 11 embedding,
 * 12 NormalBP attention backward, 13 NormalBP gradient GEMMs). */
WELVET_API void welvet_b200_profile_enable(int32_t on);
WELVET_API void welvet_b200_profile_read(double ms[14], int64_t counts[14], int32_t reset);

/* ---- decode attention without allocation (no counterpart in the reference) ----
 * Split-KV decode attention of one new query per sequence over a paged KV cache,
 * the same kernels as the decode step of welvet_b200_mha_decode, with the split
 * partials in a fixed per-device array of WELVET_B200_DECODE_STATIC_FLOATS floats
 * (4 MiB) instead of allocated memory: for callers that may not let a library
 * allocate device memory while decoding (HBM reserved up front by their own pool;
 * a framework whose caching allocator accounts for all device memory).
 * All buffers are device memory; asynchronous on `stream`.
 *   cfg         heads, KV heads, head_dim, scale, ALiBi / sigmoid, precision
 *               (1: BF16 buffers, 0: FP32), head shard; causal mask only.
 *   q           [batch, ldq], RoPE applied, the shard's heads from column 0.
 *   k_pool/v_pool [page][kv_heads][16][head_dim]; block_table [batch, max_pages]
 *               int32 page ids; ctx_len [batch] int32 keys per sequence
 *               (including the new one), each in [1, max_ctx].
 *   out         [batch, ldo].
 * Needs batch*heads*(head_dim+2) <= WELVET_B200_DECODE_STATIC_FLOATS (else code 1,
 * nothing launched); fewer KV splits are used when the default count does not fit.
 * The array need not start at zero. Calls on one device share it: calls that
 * overlap in time race, so issue them on one stream. The first call on a device
 * does the set-up (symbol lookup, module loading): make it before stream capture. */
#define WELVET_B200_DECODE_STATIC_FLOATS (1 << 20)
WELVET_API welvet_status welvet_b200_decode_attention_static(const welvet_b200_mha_config* cfg, int32_t batch,
                                                             int32_t max_ctx, const void* q, int32_t ldq,
                                                             const void* k_pool, const void* v_pool,
                                                             const int32_t* block_table, int32_t max_pages,
                                                             const int32_t* ctx_len, void* out, int32_t ldo,
                                                             void* stream);

/* ---- transformer-block forwards around the MHA (extension; the reference's
 * one-shot entries are in welvet_c.h) ----
 * Resident SwiGLU feed-forward (src/layers/swiglu/swiglu.cpp:93-143): Gate/Up
 * [intermediate_dim, input_dim] and Down [input_dim, intermediate_dim] FP32 inits
 * decoded as FormatNone `dtype` (0-33) once, then packed for the tensor cores;
 * precision 0 = FP32 (3xTF32 GEMMs), 1 = BF16 operands. forward: x [tokens,
 * input_dim], pre = h = SiLU(x Gate^T) * (x Up^T) [tokens, intermediate_dim] (may
 * be NULL), post = h Down^T [tokens, input_dim], device buffers of the layer's
 * precision, asynchronous on `stream`; forward_host: FP32 host buffers,
 * synchronous (FP32 layers). */
typedef struct welvet_b200_swiglu welvet_b200_swiglu;
WELVET_API welvet_status welvet_b200_swiglu_mount(int32_t input_dim, int32_t intermediate_dim,
                                                  int32_t precision, int32_t device, int32_t dtype,
                                                  const float* Gate, const float* Up,
                                                  const float* Down, int32_t weights_on_device,
                                                  welvet_b200_swiglu** out);
WELVET_API welvet_status welvet_b200_swiglu_forward(welvet_b200_swiglu* layer, int64_t tokens,
                                                    const void* x, void* pre, void* post,
                                                    void* stream);
WELVET_API welvet_status welvet_b200_swiglu_forward_host(welvet_b200_swiglu* layer, int64_t tokens,
                                                         const float* x, float* pre, float* post);
WELVET_API void welvet_b200_swiglu_release(welvet_b200_swiglu* layer);
/* RMSNorm (layernorm = 0) / LayerNorm (1) forward over `rows` rows of `dim`
 * (shaders/ops_norm.metal:2-26): pre = x-hat (may be NULL), post = x-hat * gamma
 * (+ beta); gamma/beta are decoded FP32 weights in device memory
 * (welvet_b200_codec_roundtrip); x/pre/post FP32, or BF16 when io_bf16; eps <= 0
 * selects the reference default (1e-6 / 1e-5). Statistics in FP64. */
WELVET_API welvet_status welvet_b200_norm_forward(int32_t layernorm, int64_t rows, int32_t dim,
                                                  double eps, const float* gamma,
                                                  const float* beta, const void* x, void* pre,
                                                  void* post, int32_t io_bf16, void* stream);
/* Embedding gather (shaders/ops_embedding.metal:1-8): out[t] = act(W[abs(int(x[t *
 * in_last])) % vocab]) over decoded FP32 weights W [vocab, emb] (device); x holds the
 * ids as floats; act is the reference's Activation id (-1 Linear, 0 ReLU, 1 SiLU,
 * 2 GELU, 3 Tanh, 4 Sigmoid, 5 LeakyReLU, 6 ReLU2). */
WELVET_API welvet_status welvet_b200_embedding_forward(int64_t tokens, int32_t vocab, int32_t emb,
                                                       int32_t in_last, int32_t act, const float* W,
                                                       const float* x, void* out, int32_t out_bf16,
                                                       void* stream);

#ifdef __cplusplus
}
#endif

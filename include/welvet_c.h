#pragma once

/* welvet C ABI — the multi-head-attention forward subset, served by the B200
 * (sm_100a) CUDA backend in libwelvet_b200.so.
 *
 * Every declaration below has the same name, signature, argument meaning and
 * status semantics as the reference header include/welvet_c.h of
 * openfluke/welvet.metal; the line of the reference each one replaces is cited.
 * Besides the MHA forward it serves the MHA NormalBP leaf and the forward entries
 * of the transformer block around it (SwiGLU, RMSNorm, LayerNorm, Embedding). The
 * reference's other entry points (Dense/CNN/recurrent families, the other NormalBP
 * leaves) are not part of this library. Model sessions (WMN1) are served for models
 * whose layers are MHA cells; their training entry points answer code 2. */

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define WELVET_API __attribute__((visibility("default")))

/* Reference include/welvet_c.h:22-25. code: 0 ok, 1 invalid argument,
 * 2 unsupported, 3 gap, 4 internal (CUDA/NCCL failures map here). */
typedef struct welvet_status {
  int32_t code;
  char message[256];
} welvet_status;

/* Reference include/welvet_c.h:28 (impl src/interop/c_abi.cpp:79-82). */
WELVET_API const char* welvet_version(void);
/* Reference include/welvet_c.h:29. Returns "cuda:<device name>:sm_<cc>:welvet-b200"
 * (the reference returns "metal:..."). */
WELVET_API const char* welvet_runtime_identity(void);
/* Reference include/welvet_c.h:31 (impl c_abi.cpp:90-94): selects/initialises
 * the compute device; the name is kept for ABI compatibility. */
WELVET_API welvet_status welvet_metal_init(void);
/* Reference include/welvet_c.h:32: 1 when a usable sm_100 device is present. */
WELVET_API int32_t welvet_metal_available(void);

/* Reference include/welvet_c.h:87-92 (impl src/interop/c_abi.cpp:209-247).
 * MHA ModeSelf forward. Q [q_dim, d_model], K/V [kv_dim, d_model], O [d_model, q_dim]
 * are FP32 initial weights, encoded to `dtype` (FormatNone) and decoded exactly as the
 * reference does; x [batch*seq*d_model]; outputs pre [batch*seq*q_dim] (attention
 * output) and post [batch*seq*d_model]. num_kv_heads/head_dim/max_seq_len <= 0 select
 * the defaults; mask 0/1 causal, 2 bidirectional, 3 sliding window (window =
 * max_seq_len), 4 prefix-LM (prefix 0), 5 custom (causal); pos 0 RoPE, 1 none,
 * 2 ALiBi, 3 RoPE+ALiBi; backend is ignored. Batches form one stream of positions
 * with a max_seq_len ring of keys, exactly as the reference attention kernel.
 * All pointers are host memory owned by the caller; nothing is retained. */
WELVET_API welvet_status welvet_mha_forward_f32(
    int32_t batch, int32_t seq, int32_t d_model, int32_t num_heads, int32_t num_kv_heads,
    int32_t head_dim, int32_t max_seq_len, int32_t mask, int32_t pos, int32_t dtype, int32_t backend,
    const float* Q, const float* K, const float* V, const float* O, const float* x, float* pre,
    float* post);

/* Reference include/welvet_c.h:94-103 (impl src/interop/c_abi.cpp:249-325). MHA NormalBP
 * leaf: forward, then dL/dpost = MSE gradient against grad_or_target (use_target = 1,
 * *loss = the MSE) or grad_or_target itself (use_target = 0, *loss = 0), the backward
 * with the reference's stream semantics, SGD with rate lr (Float32 storage; other
 * dtypes need lr = 0 here, status 2 otherwise), the weight export. Outputs pre
 * [batch*seq*q_dim], post and dX [batch*seq*d_model], dW and W_after = concat(Q, K,
 * V, O). Host memory, synchronous, nothing retained. */
WELVET_API welvet_status welvet_mha_normalbp_f32(
    int32_t batch, int32_t seq, int32_t d_model, int32_t num_heads, int32_t num_kv_heads,
    int32_t head_dim, int32_t max_seq_len, int32_t mask, int32_t pos, int32_t dtype, int32_t backend,
    const float* Q, const float* K, const float* V, const float* O, const float* x,
    const float* grad_or_target, int32_t use_target, double lr, float* pre, float* post, float* dX,
    float* dW, float* W_after, double* loss);

/* Reference include/welvet_c.h:105-109 (impl src/interop/c_abi.cpp:326-361).
 * SwiGLU forward: Gate/Up [intermediate_dim, input_dim], Down [input_dim,
 * intermediate_dim] FP32 inits encoded to `dtype`; x [batch*seq*input_dim];
 * pre = h = SiLU(x Gate^T) * (x Up^T) [batch*seq*intermediate_dim], post = h Down^T
 * [batch*seq*input_dim]. Host memory, synchronous, nothing retained. */
WELVET_API welvet_status welvet_swiglu_forward_f32(
    int32_t batch, int32_t seq, int32_t input_dim, int32_t intermediate_dim, int32_t dtype,
    int32_t backend, const float* Gate, const float* Up, const float* Down, const float* x,
    float* pre, float* post);

/* Reference include/welvet_c.h:121-124 (impl c_abi.cpp:437-469). RMSNorm forward:
 * gamma [dim] encoded to `dtype`; pre = x / rms(x), post = pre * gamma, each
 * [batch*seq*dim]; eps <= 0 selects 1e-6. */
WELVET_API welvet_status welvet_rmsnorm_forward_f32(int32_t batch, int32_t seq, int32_t dim,
                                                    double eps, int32_t dtype, int32_t backend,
                                                    const float* gamma, const float* x,
                                                    float* pre, float* post);

/* Reference include/welvet_c.h:135-138 (impl c_abi.cpp:543-577). LayerNorm forward:
 * pre = (x - mean) / sqrt(var + eps), post = pre * gamma + beta; eps <= 0 selects 1e-5. */
WELVET_API welvet_status welvet_layernorm_forward_f32(int32_t batch, int32_t seq, int32_t dim,
                                                      double eps, int32_t dtype, int32_t backend,
                                                      const float* gamma, const float* beta,
                                                      const float* x, float* pre, float* post);

/* Reference include/welvet_c.h:168-172 (impl c_abi.cpp:792-832). Embedding gather:
 * W [vocab, emb] encoded to `dtype`; token t's id is abs(int(x[t*in_last])) % vocab
 * (in_rank 1: seq_len tokens; 2: batch*seq_len; 3: batch*seq_len with in_last 1 or
 * emb); pre = post = act(W[id]) [tokens*emb]. */
WELVET_API welvet_status welvet_embedding_forward_f32(
    int32_t batch, int32_t vocab, int32_t emb, int32_t seq_len, int32_t in_rank, int32_t in_last,
    int32_t act, int32_t dtype, int32_t backend, const float* W, const float* x, float* pre,
    float* post);

/* Versioned model sessions (reference include/welvet_c.h:36-56, impl
 * src/interop/model_session.cpp:319-576). welvet_model_mount reads a WMN1
 * descriptor (root Stack = 0 or Grid = 2, MHA and nested-Stack children,
 * Cameral controls, native Store snapshots, grid cell metadata; the byte layout of
 * the reference's model_wire.hpp / child_wire.hpp) and mounts every MHA child as a
 * resident B200 layer whose weights are the snapshots' stores (Q, K, V, O). Inputs
 * and outputs are the reference's tensor wires (rank, dims, FP32 values; outputs
 * add the element count). Buffers are copied during calls; one call at a time per
 * session (a per-session lock). Root Parallel, other layer kinds, and the training
 * / proxy / sync entry points answer code 2. */
typedef struct welvet_model_session welvet_model_session;
typedef struct welvet_metal_blob { uint8_t* data; size_t size; } welvet_metal_blob;
WELVET_API int32_t welvet_model_abi_version(void);
WELVET_API welvet_status welvet_model_mount(const uint8_t*, size_t, welvet_model_session**);
WELVET_API welvet_status welvet_model_forward(welvet_model_session*, const uint8_t*, size_t, welvet_metal_blob*);
WELVET_API welvet_status welvet_model_train_credit(welvet_model_session*, int32_t, double, const uint8_t*, size_t);
WELVET_API welvet_status welvet_model_dense_proxy(welvet_model_session*, int32_t, const uint8_t*, size_t, welvet_metal_blob*);
WELVET_API welvet_status welvet_model_forward_pair(welvet_model_session*, const uint8_t*, size_t, welvet_metal_blob*);
WELVET_API welvet_status welvet_model_backward(welvet_model_session*, const uint8_t*, size_t, welvet_metal_blob*);
WELVET_API welvet_status welvet_model_apply_sgd(welvet_model_session*, double, const uint8_t*, size_t);
WELVET_API welvet_status welvet_model_train_mse(welvet_model_session*, int32_t mode, double lr, int32_t ticks, const uint8_t*, size_t, double* loss);
WELVET_API welvet_status welvet_model_export_weights(welvet_model_session*, welvet_metal_blob*);
WELVET_API welvet_status welvet_model_sync(welvet_model_session*, int32_t event);
WELVET_API void welvet_model_release(welvet_model_session*);
WELVET_API void welvet_metal_blob_free(welvet_metal_blob*);

#ifdef __cplusplus
}
#endif

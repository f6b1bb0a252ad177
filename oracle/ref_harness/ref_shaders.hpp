// Test infrastructure (builds oracle/_ref only): host entry points for the
// reference shader kernels compiled as C++ (see ref_shaders.cpp).
#pragma once
#include <cstdint>

namespace refshader {
// welvet_dense_matvec_softdouble_batch (shaders/welvet_dense.metal:54-85), one gid.
void dense_matvec(const float* W_xy, const float* x, float* y, uint32_t in_dim, uint32_t out_dim,
                  uint32_t batch, uint32_t gid);
// welvet_dense_bias_act (shaders/welvet_dense.metal:87-105), one gid.
void dense_bias_act(float* pre, float* post, const float* bias_xy, uint32_t out_dim,
                    uint32_t batch, int32_t act, uint32_t bias_len, uint32_t gid);
// op_attention (shaders/ops_mha.metal:31-176), one thread id; OP_ARGS buffers a..j.
void op_attention_kernel(float* const bufs[8], const int32_t* c, const float* r, uint32_t tid);
// One thread id of the OP_ARGS kernel `name` (op_attention, op_swiglu,
// op_norm_forward, op_embedding_forward); false for any other name.
bool op_kernel(const char* name, float* const bufs[8], const int32_t* c, const float* r, uint32_t tid);
} // namespace refshader

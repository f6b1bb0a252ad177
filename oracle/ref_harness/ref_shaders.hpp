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
// Backward / training kernels of welvet_dense.metal, one gid each.
void dense_act_deriv(const float* gy, const float* pre, float* d_pre, uint32_t out_dim, uint32_t batch,
                     int32_t act, uint32_t gid);
void dense_matvect(const float* W_xy, const float* gy, float* gx, uint32_t in_dim, uint32_t out_dim,
                   uint32_t batch, uint32_t gid);
void dense_outer(const float* gy, const float* x, float* dW, uint32_t in_dim, uint32_t out_dim, uint32_t batch,
                 uint32_t gid);
void mse_loss(const float* pred, const float* target, float* loss2, uint32_t n);
void mse_grad(const float* pred, const float* target, float* grad, uint32_t n, uint32_t gid);
void sgd_f32_f64_grad(float* weights, const float* grad_xy, const float* lr_xy, uint32_t n, uint32_t gid);
// One thread id of the OP_ARGS kernel `name` (op_attention, op_swiglu,
// op_norm_forward, op_embedding_forward, op_add3); false for any other name.
bool op_kernel(const char* name, float* const bufs[8], const int32_t* c, const float* r, uint32_t tid);
} // namespace refshader

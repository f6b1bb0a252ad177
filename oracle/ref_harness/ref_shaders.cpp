// Test infrastructure (builds oracle/_ref only). Compiles the reference's own
// soft-double shader sources — welvet_dense.metal, then ops_common.metal,
// ops_embedding.metal, ops_mha.metal and ops_norm.metal in the sorted order of the
// reference's ops_*.metal glob (CMakeLists.txt:118-129) — as host C++ through the
// MSL shim in oracle/msl_shim, and exposes the kernels that the MHA, SwiGLU,
// RMSNorm/LayerNorm and Embedding forwards dispatch as plain functions. The
// shader files are read where they lie; nothing is copied.
#include <metal_stdlib>

#include <cstring>

#include "welvet_dense.metal"
#include "ops_common.metal"
#include "ops_embedding.metal"
#include "ops_mha.metal"
#include "ops_norm.metal"

// Declared (not defined) by welvet_dense.metal and used by the MSE-loss kernel to
// hand the soft-double loss to the host as an IEEE double (ops_storage.metal
// defines it; here the pair is summed in double, exact to the last bit or one).
namespace native_gpu {
inline ulong pack_sd(float2 value) {
  const double d = (double)value.x + (double)value.y;
  ulong u = 0;
  std::memcpy(&u, &d, sizeof(d));
  return u;
}
} // namespace native_gpu

#undef kernel
#undef device
#undef thread
#undef constant

#include "ref_shaders.hpp"

namespace refshader {

void dense_matvec(const float* W_xy, const float* x, float* y, uint32_t in_dim, uint32_t out_dim,
                  uint32_t batch, uint32_t gid) {
  welvet_dense_matvec_softdouble_batch(reinterpret_cast<const float2*>(W_xy), x, y, in_dim,
                                       out_dim, batch, gid);
}

void dense_bias_act(float* pre, float* post, const float* bias_xy, uint32_t out_dim,
                    uint32_t batch, int32_t act, uint32_t bias_len, uint32_t gid) {
  welvet_dense_bias_act(pre, post, reinterpret_cast<const float2*>(bias_xy), out_dim, batch, act,
                        bias_len, gid);
}

void op_attention_kernel(float* const bufs[8], const int32_t* c, const float* r, uint32_t tid) {
  op_attention(bufs[0], bufs[1], bufs[2], bufs[3], bufs[4], bufs[5], bufs[6], bufs[7], c, r, tid);
}

void dense_act_deriv(const float* gy, const float* pre, float* d_pre, uint32_t out_dim, uint32_t batch,
                     int32_t act, uint32_t gid) {
  welvet_dense_act_deriv(gy, pre, d_pre, out_dim, batch, act, gid);
}
void dense_matvect(const float* W_xy, const float* gy, float* gx, uint32_t in_dim, uint32_t out_dim,
                   uint32_t batch, uint32_t gid) {
  welvet_dense_matvect_softdouble_batch(reinterpret_cast<const float2*>(W_xy), gy, gx, in_dim, out_dim, batch,
                                        gid);
}
void dense_outer(const float* gy, const float* x, float* dW, uint32_t in_dim, uint32_t out_dim, uint32_t batch,
                 uint32_t gid) {
  welvet_dense_outer_batch(gy, x, dW, in_dim, out_dim, batch, gid);
}
void mse_loss(const float* pred, const float* target, float* loss2, uint32_t n) {
  welvet_mse_loss(pred, target, reinterpret_cast<float2*>(loss2), n, 0);
}
void mse_grad(const float* pred, const float* target, float* grad, uint32_t n, uint32_t gid) {
  welvet_mse_grad(pred, target, grad, n, gid);
}
void sgd_f32_f64_grad(float* weights, const float* grad_xy, const float* lr_xy, uint32_t n, uint32_t gid) {
  const float2 lr(lr_xy[0], lr_xy[1]);
  welvet_sgd_f32_f64_grad(weights, reinterpret_cast<const float2*>(grad_xy), lr, n, gid);
}

bool op_kernel(const char* name, float* const bufs[8], const int32_t* c, const float* r, uint32_t tid) {
#define WV_OP(k)                                                                                   \
  if (std::strcmp(name, #k) == 0) {                                                                \
    k(bufs[0], bufs[1], bufs[2], bufs[3], bufs[4], bufs[5], bufs[6], bufs[7], c, r, tid);          \
    return true;                                                                                   \
  }
  WV_OP(op_attention)
  WV_OP(op_swiglu)
  WV_OP(op_norm_forward)
  WV_OP(op_embedding_forward)
  WV_OP(op_add3)
#undef WV_OP
  return false;
}

} // namespace refshader

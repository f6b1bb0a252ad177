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

// Declared (not defined) by welvet_dense.metal; only the MSE-loss kernel uses it.
namespace native_gpu {
inline ulong pack_sd(float2 value) {
  ulong u = 0;
  std::memcpy(&u, &value, sizeof(value));
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
#undef WV_OP
  return false;
}

} // namespace refshader

// Test infrastructure — NOT part of the product. FP64 restatement of the
// reference's transformer-block forwards around the MHA: RMSNorm / LayerNorm
// (src/layers/rmsnorm/rmsnorm.cpp, src/layers/layernorm/layernorm.cpp,
// shaders/ops_norm.metal:2-26), SwiGLU (src/layers/swiglu/swiglu.cpp:93-143,
// shaders/ops_common.metal:27-38) and Embedding (src/layers/embedding/embedding.cpp,
// shaders/ops_embedding.metal:1-8), with the activations of
// shaders/ops_common.metal:83-105. The shaders' float2 soft-double arithmetic is
// restated in IEEE double; values are rounded to FP32 where the shaders call
// sd_to_float or do float arithmetic. Weights arrive already decoded
// (oracle_roundtrip of the FP32 inits).
#include "oracle.h"

#include <cmath>
#include <cstdlib>
#include <vector>

namespace {

// act_value (ops_common.metal:83-105): soft-double for Silu, GELU (tanh form),
// Tanh, Sigmoid, LeakyReLU; float for ReLU and ReLU2; identity otherwise (Linear).
float act_value(float v, int act) {
  const double x = v;
  auto sigmoid = [](double t) { return 1.0 / (1.0 + std::exp(-t)); };
  auto tanh_c = [](double t) { return t > 18 ? 1.0 : (t < -18 ? -1.0 : std::tanh(t)); };
  switch (act) {
  case 1: return (float)(x * sigmoid(x));
  case 3: return (float)tanh_c(x);
  case 4: return (float)sigmoid(x);
  case 2: {
    // float2 constants (hi + lo) of the shader
    const double c3 = 0.044714998453855515 + 1.5461444832776117e-09;
    const double c = 0.7978845834732056 + -2.2670340160679814e-08;
    const double u = (x + x * x * x * c3) * c;
    return (float)(x * 0.5 * (1.0 + tanh_c(u)));
  }
  case 0: return v > 0.0f ? v : 0.0f;
  case 6: return v < 0 ? 0.0f : v * v;
  case 5: return v < 0 ? (float)(x * (0.009999999776482582 + 2.2351741811588166e-10)) : v;
  default: return v;
  }
}

}  // namespace

float oracle_act_value(float v, int32_t act) { return act_value(v, act); }

int32_t oracle_norm_forward(int32_t layernorm, int64_t rows, int32_t dim, double eps,
                            const float* gamma, const float* beta, const float* x, float* pre,
                            float* post) {
  if (rows <= 0 || dim <= 0) return 1;
  // validate(): eps <= 0 -> 1e-6 (RMSNorm, rmsnorm.cpp) / 1e-5 (LayerNorm, layernorm.cpp:56-57)
  if (eps <= 0) eps = layernorm ? 1e-5 : 1e-6;
  for (int64_t r = 0; r < rows; ++r) {
    const float* xr = x + r * dim;
    double sum = 0, sq = 0;
    for (int i = 0; i < dim; ++i) {
      sum += xr[i];
      sq += (double)xr[i] * (double)xr[i];
    }
    const double mean = layernorm ? sum / dim : 0.0;
    const double var = sq / dim - mean * mean;
    const double inv = 1.0 / std::sqrt(var + eps);
    for (int i = 0; i < dim; ++i) {
      const double xh = ((double)xr[i] - mean) * inv;
      pre[r * dim + i] = (float)xh;
      double y = xh * (double)gamma[i];
      if (layernorm) y += (double)beta[i];
      post[r * dim + i] = (float)y;
    }
  }
  return 0;
}

int32_t oracle_swiglu_forward(int64_t tokens, int32_t in, int32_t inter, const float* Gate,
                              const float* Up, const float* Down, const float* x, float* pre,
                              float* post, int32_t threads) {
  if (tokens <= 0 || in <= 0 || inter <= 0) return 1;
  std::vector<float> g((size_t)tokens * inter), u((size_t)tokens * inter);
  oracle_dense(x, Gate, g.data(), tokens, in, inter, threads);
  oracle_dense(x, Up, u.data(), tokens, in, inter, threads);
  // op_swiglu: float s = act_value(gate_pre, Silu); h = s * up_post in float
  for (int64_t i = 0; i < tokens * inter; ++i) pre[i] = act_value(g[i], 1) * u[i];
  oracle_dense(pre, Down, post, tokens, inter, in, threads);
  return 0;
}

int32_t oracle_embedding_forward(int64_t tokens, int32_t vocab, int32_t emb, int32_t in_last,
                                 int32_t act, const float* W, const float* x, float* pre,
                                 float* post) {
  if (tokens <= 0 || vocab <= 0 || emb <= 0 || in_last <= 0) return 1;
  for (int64_t t = 0; t < tokens; ++t) {
    // id = abs(int(x[tok * in_last])) % vocab (ops_embedding.metal:4)
    const int id = std::abs((int)x[t * in_last]) % vocab;
    for (int c = 0; c < emb; ++c) {
      const float v = act_value(W[(int64_t)id * emb + c], act);
      pre[t * emb + c] = v;
      post[t * emb + c] = v;
    }
  }
  return 0;
}

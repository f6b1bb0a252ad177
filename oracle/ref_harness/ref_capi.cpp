// Test infrastructure (builds oracle/_ref only). C entry points over the
// reference's own host code, compiled from its sources, so Python tests can
// call it through ctypes:
//  - ref_mha_forward_f32: the body of welvet_mha_forward_f32
//    (src/interop/c_abi.cpp:209-247) — config fill, mha::new_configured,
//    mha::forward — running the reference shaders on the CPU executor.
//  - ref_mha_forward_cfg: the same with every mha::Config field settable.
//  - ref_weight_roundtrip: WeightStore::make + native bytes + export_f32.
//  - ref_mha_normalbp_f32: the body of welvet_mha_normalbp_f32
//    (src/interop/c_abi.cpp:249-325) — forward, MSE or the given gradient,
//    mha::backward_f32, SGD, weight export (MSE through metal::mse_f32 as
//    src/runtime/training.cpp:43-57 does).
//  - ref_swiglu_forward_f32, ref_rmsnorm_forward_f32, ref_layernorm_forward_f32,
//    ref_embedding_forward_f32: the bodies of the reference's block forward entries
//    (src/interop/c_abi.cpp:326-361, 437-469, 543-577, 792-832).
//  - the scalar converters of include/welvet/float_codecs.hpp.
#include "welvet/embedding.hpp"
#include "welvet/float_codecs.hpp"
#include "welvet/layernorm.hpp"
#include "welvet/metal/training.hpp"
#include "welvet/mha.hpp"
#include "welvet/rmsnorm.hpp"
#include "welvet/swiglu.hpp"
#include "welvet/weights.hpp"

#include <cstdio>
#include <cstring>

extern "C" {

struct ref_status {
  int32_t code;
  char message[256];
};

static ref_status to_status(const welvet::Status& st) {
  ref_status out{};
  out.code = static_cast<int32_t>(st.code);
  std::snprintf(out.message, sizeof(out.message), "%s", st.message.c_str());
  return out;
}

ref_status ref_mha_forward_cfg(int32_t batch, int32_t seq, int32_t d_model, int32_t num_heads,
                               int32_t num_kv_heads, int32_t head_dim, int32_t max_seq_len,
                               int32_t mask, int32_t pos, int32_t softmax, int32_t window,
                               int32_t prefix_len, int32_t window_causal, double rope_theta,
                               double scale_override, int32_t dtype, const float* Q,
                               const float* K, const float* V, const float* O, const float* x,
                               float* pre, float* post) {
  welvet::mha::Config cfg;
  cfg.d_model = d_model;
  cfg.num_heads = num_heads;
  cfg.num_kv_heads = num_kv_heads;
  cfg.head_dim = head_dim;
  cfg.max_seq_len = max_seq_len;
  cfg.mask = static_cast<welvet::mha::MaskKind>(mask);
  cfg.pos = static_cast<welvet::mha::PosKind>(pos);
  cfg.softmax = static_cast<welvet::mha::SoftmaxKind>(softmax);
  cfg.mode = welvet::mha::AttnMode::Self;
  cfg.causal = (cfg.mask == welvet::mha::MaskKind::Causal);
  cfg.window = window;
  cfg.prefix_len = prefix_len;
  cfg.window_causal = window_causal != 0;
  cfg.rope_theta = rope_theta;
  cfg.scale_override = scale_override;
  welvet::mha::Layer layer;
  auto st = welvet::mha::new_configured(cfg, static_cast<welvet::DType>(dtype), Q, K, V, O, &layer);
  if (!st) return to_status(st);
  welvet::TensorF32 input;
  input.shape = {batch, seq, d_model};
  input.data.assign(x, x + static_cast<std::size_t>(batch) * seq * d_model);
  welvet::TensorF32 pre_t, post_t;
  st = welvet::mha::forward(layer, input, &pre_t, &post_t);
  if (!st) return to_status(st);
  std::memcpy(pre, pre_t.data.data(), pre_t.data.size() * sizeof(float));
  std::memcpy(post, post_t.data.data(), post_t.data.size() * sizeof(float));
  return to_status(welvet::Status::Ok());
}

// Argument checks and Config fill of c_abi.cpp:213-231; window/prefix are not
// settable through this entry, and window_causal keeps its default (true).
ref_status ref_mha_forward_f32(int32_t batch, int32_t seq, int32_t d_model, int32_t num_heads,
                               int32_t num_kv_heads, int32_t head_dim, int32_t max_seq_len,
                               int32_t mask, int32_t pos, int32_t dtype, int32_t /*backend*/,
                               const float* Q, const float* K, const float* V, const float* O,
                               const float* x, float* pre, float* post) {
  if (batch <= 0 || seq <= 0 || d_model <= 0 || num_heads <= 0 || !Q || !K || !V || !O || !x ||
      !pre || !post) {
    ref_status st{};
    st.code = 1;
    std::snprintf(st.message, sizeof(st.message), "mha: invalid argument");
    return st;
  }
  return ref_mha_forward_cfg(batch, seq, d_model, num_heads, num_kv_heads, head_dim, max_seq_len,
                             mask, pos, 0, 0, 0, 1, 10000.0, 0.0, dtype, Q, K, V, O, x, pre,
                             post);
}

// Encodes rows*cols FP32 weights as `dtype` with the reference WeightStore and
// returns its native bytes (native_len in/out: capacity, then size), scale and
// the decoded FP32 matrix (export_f32).
ref_status ref_weight_roundtrip(int32_t dtype, int32_t rows, int32_t cols, const float* w,
                                uint8_t* native, int64_t* native_len, float* scale,
                                float* decoded) {
  welvet::WeightStore s;
  auto st = welvet::WeightStore::make(rows, cols, static_cast<welvet::DType>(dtype), w, &s);
  if (!st) return to_status(st);
  const auto& bytes = s.native;
  if (dtype == static_cast<int32_t>(welvet::DType::Float32)) {
    *native_len = 0;
  } else {
    if ((int64_t)bytes.size() > *native_len) {
      ref_status e{};
      e.code = 1;
      std::snprintf(e.message, sizeof(e.message), "native buffer too small");
      return e;
    }
    std::memcpy(native, bytes.data(), bytes.size());
    *native_len = (int64_t)bytes.size();
  }
  *scale = s.scale;
  return to_status(s.export_f32(decoded));
}


static ref_status invalid(const char* msg) {
  ref_status st{};
  st.code = 1;
  std::snprintf(st.message, sizeof(st.message), "%s", msg);
  return st;
}

// [batch, dim] when seq == 1, else [batch, seq, dim], as the reference entries shape x.
static welvet::TensorF32 block_input(int32_t batch, int32_t seq, int32_t dim, const float* x) {
  welvet::TensorF32 input;
  if (seq == 1)
    input.shape = {batch, dim};
  else
    input.shape = {batch, seq, dim};
  input.data.assign(x, x + static_cast<std::size_t>(batch) * seq * dim);
  return input;
}

static ref_status copy_out(const welvet::TensorF32& pre_t, const welvet::TensorF32& post_t, float* pre,
                           float* post) {
  std::memcpy(pre, pre_t.data.data(), pre_t.data.size() * sizeof(float));
  std::memcpy(post, post_t.data.data(), post_t.data.size() * sizeof(float));
  return to_status(welvet::Status::Ok());
}

ref_status ref_swiglu_forward_f32(int32_t batch, int32_t seq, int32_t input_dim, int32_t intermediate_dim,
                                  int32_t dtype, const float* Gate, const float* Up, const float* Down,
                                  const float* x, float* pre, float* post) {
  if (batch <= 0 || seq <= 0 || input_dim <= 0 || intermediate_dim <= 0 || !Gate || !Up || !Down || !x ||
      !pre || !post)
    return invalid("swiglu: invalid argument");
  welvet::swiglu::Config cfg;
  cfg.input_dim = input_dim;
  cfg.intermediate_dim = intermediate_dim;
  welvet::swiglu::Layer layer;
  auto st = welvet::swiglu::new_configured(cfg, static_cast<welvet::DType>(dtype), Gate, Up, Down, &layer);
  if (!st) return to_status(st);
  welvet::TensorF32 pre_t, post_t;
  st = welvet::swiglu::forward(layer, block_input(batch, seq, input_dim, x), &pre_t, &post_t);
  if (!st) return to_status(st);
  return copy_out(pre_t, post_t, pre, post);
}

ref_status ref_rmsnorm_forward_f32(int32_t batch, int32_t seq, int32_t dim, double eps, int32_t dtype,
                                   const float* gamma, const float* x, float* pre, float* post) {
  if (batch <= 0 || seq <= 0 || dim <= 0 || !gamma || !x || !pre || !post)
    return invalid("rmsnorm: invalid argument");
  welvet::rmsnorm::Config cfg;
  cfg.dim = dim;
  cfg.eps = eps;
  welvet::rmsnorm::Layer layer;
  auto st = welvet::rmsnorm::new_configured(cfg, static_cast<welvet::DType>(dtype), gamma, &layer);
  if (!st) return to_status(st);
  welvet::TensorF32 pre_t, post_t;
  st = welvet::rmsnorm::forward(layer, block_input(batch, seq, dim, x), &pre_t, &post_t);
  if (!st) return to_status(st);
  return copy_out(pre_t, post_t, pre, post);
}

ref_status ref_layernorm_forward_f32(int32_t batch, int32_t seq, int32_t dim, double eps, int32_t dtype,
                                     const float* gamma, const float* beta, const float* x, float* pre,
                                     float* post) {
  if (batch <= 0 || seq <= 0 || dim <= 0 || !gamma || !beta || !x || !pre || !post)
    return invalid("layernorm: invalid argument");
  welvet::layernorm::Config cfg;
  cfg.dim = dim;
  cfg.eps = eps;
  welvet::layernorm::Layer layer;
  auto st =
      welvet::layernorm::new_configured(cfg, static_cast<welvet::DType>(dtype), gamma, beta, &layer);
  if (!st) return to_status(st);
  welvet::TensorF32 pre_t, post_t;
  st = welvet::layernorm::forward(layer, block_input(batch, seq, dim, x), &pre_t, &post_t);
  if (!st) return to_status(st);
  return copy_out(pre_t, post_t, pre, post);
}

ref_status ref_embedding_forward_f32(int32_t batch, int32_t vocab, int32_t emb, int32_t seq_len,
                                     int32_t in_rank, int32_t in_last, int32_t act, int32_t dtype,
                                     const float* W, const float* x, float* pre, float* post) {
  if (batch <= 0 || vocab <= 0 || emb <= 0 || seq_len <= 0 || in_last <= 0 || !W || !x || !pre || !post)
    return invalid("embedding: invalid argument");
  if (in_rank < 1 || in_rank > 3) return invalid("embedding: bad in_rank");
  welvet::embedding::Config cfg;
  cfg.vocab_size = vocab;
  cfg.embedding_dim = emb;
  cfg.seq_len = seq_len;
  welvet::embedding::Layer layer;
  auto st = welvet::embedding::new_configured(cfg, static_cast<welvet::DType>(dtype),
                                              static_cast<welvet::Activation>(act), W, &layer);
  if (!st) return to_status(st);
  welvet::TensorF32 input;
  if (in_rank == 1)
    input.shape = {seq_len};
  else if (in_rank == 2)
    input.shape = {batch, seq_len};
  else
    input.shape = {batch, seq_len, in_last};
  input.data.assign(x, x + static_cast<std::size_t>(batch) * seq_len * in_last);
  welvet::TensorF32 pre_t, post_t;
  st = welvet::embedding::forward(layer, input, &pre_t, &post_t);
  if (!st) return to_status(st);
  return copy_out(pre_t, post_t, pre, post);
}

ref_status ref_mha_normalbp_f32(int32_t batch, int32_t seq, int32_t d_model, int32_t num_heads,
                                int32_t num_kv_heads, int32_t head_dim, int32_t max_seq_len, int32_t mask,
                                int32_t pos, int32_t dtype, const float* Q, const float* K, const float* V,
                                const float* O, const float* x, const float* grad_or_target, int32_t use_target,
                                double lr, float* pre, float* post, float* dX, float* dW, float* W_after,
                                double* loss) {
  if (batch <= 0 || seq <= 0 || d_model <= 0 || num_heads <= 0 || !Q || !K || !V || !O || !x ||
      !grad_or_target || !pre || !post || !dX || !dW || !W_after || !loss)
    return invalid("mha nbp: invalid argument");
  welvet::mha::Config cfg;
  cfg.d_model = d_model;
  cfg.num_heads = num_heads;
  cfg.num_kv_heads = num_kv_heads;
  cfg.head_dim = head_dim;
  cfg.max_seq_len = max_seq_len;
  cfg.mask = static_cast<welvet::mha::MaskKind>(mask);
  cfg.pos = static_cast<welvet::mha::PosKind>(pos);
  cfg.mode = welvet::mha::AttnMode::Self;
  cfg.causal = (cfg.mask == welvet::mha::MaskKind::Causal);
  welvet::mha::Layer layer;
  auto st = welvet::mha::new_configured(cfg, static_cast<welvet::DType>(dtype), Q, K, V, O, &layer);
  if (!st) return to_status(st);
  welvet::TensorF32 input;
  input.shape = {batch, seq, d_model};
  const std::size_t n = static_cast<std::size_t>(batch) * seq * d_model;
  input.data.assign(x, x + n);
  welvet::TensorF32 pre_t, post_t;
  st = welvet::mha::forward(layer, input, &pre_t, &post_t);
  if (!st) return to_status(st);
  welvet::TensorF32 gy;
  gy.shape = post_t.shape;
  gy.data.assign(grad_or_target, grad_or_target + n);
  *loss = 0.0;
  if (use_target) {
    st = welvet::metal::mse_f32(post_t.data.data(), gy.data.data(), n, loss, nullptr);
    if (!st) return to_status(st);
    welvet::TensorF32 g = post_t;
    st = welvet::metal::mse_f32(post_t.data.data(), gy.data.data(), n, nullptr, g.data.data());
    if (!st) return to_status(st);
    gy = std::move(g);
  }
  welvet::TensorF32 dx_t, dw_t;
  st = welvet::mha::backward_f32(layer, gy, input, pre_t, &dx_t, &dw_t);
  if (!st) return to_status(st);
  if (lr != 0.0) {
    st = welvet::mha::apply_grad_sgd(&layer, dw_t, lr);
    if (!st) return to_status(st);
  }
  st = welvet::mha::export_weights_f32(layer, W_after);
  if (!st) return to_status(st);
  std::memcpy(pre, pre_t.data.data(), pre_t.data.size() * sizeof(float));
  std::memcpy(post, post_t.data.data(), post_t.data.size() * sizeof(float));
  std::memcpy(dX, dx_t.data.data(), dx_t.data.size() * sizeof(float));
  std::memcpy(dW, dw_t.data.data(), dw_t.data.size() * sizeof(float));
  return to_status(welvet::Status::Ok());
}

uint8_t ref_fp8e4m3_encode(float f) { return welvet::float32_to_fp8e4m3(f); }
float ref_fp8e4m3_decode(uint8_t b) { return welvet::fp8e4m3_to_float32(b); }
uint8_t ref_fp8e5m2_encode(float f) { return welvet::float32_to_fp8e5m2(f); }
float ref_fp8e5m2_decode(uint8_t b) { return welvet::fp8e5m2_to_float32(b); }
uint16_t ref_bf16_encode(float f) { return welvet::float32_to_bfloat16(f); }
float ref_bf16_decode(uint16_t h) { return welvet::bfloat16_to_float32(h); }
uint16_t ref_f16_encode(float f) { return welvet::float32_to_float16(f); }
float ref_f16_decode(uint16_t h) { return welvet::float16_to_float32(h); }

} // extern "C"

#pragma once
// C++ layer API of the MHA forward (reference include/welvet/mha.hpp:10-98, same
// names, signatures, enum values and defaults), running on the B200 engine of
// libwelvet_b200.so.
//
// new_configured encodes the FP32 inits to `dt` (FormatNone), decodes them on the
// GPU and keeps the layer's weights resident in HBM (the reference builds four
// Dense layers that mount on their first forward, src/layers/dense/dense.cpp:50-97).
// forward runs the reference's stream semantics (positions b*T + t, keys from a
// max_seq_len ring) in FP32 (3xTF32 projections), host tensors in and out, like
// reference mha::forward (src/layers/mha/mha.cpp:138-205).
//
// Differences a caller can see: Layer holds the resident session instead of four
// dense::Layer members; the attention settings (mask, pos, softmax, window,
// prefix, theta, scale, max_seq_len) are fixed when the layer is mounted, so a
// forward after they were edited in layer.cfg returns code 2 (call new_configured
// again); the backward / SGD / export members of the reference header are not
// part of this API (the MHA NormalBP leaf is welvet_mha_normalbp_f32 in welvet_c.h).
#include <cstdint>
#include <memory>

#include "welvet/dtype.hpp"
#include "welvet/export.hpp"
#include "welvet/status.hpp"
#include "welvet/tensor.hpp"

struct welvet_b200_mha;

namespace welvet::mha {

enum class MaskKind : int32_t { Unspecified = 0, Causal = 1, Bidirectional = 2, SlidingWindow = 3, PrefixLM = 4, Custom = 5 };
enum class PosKind : int32_t { RoPE = 0, None = 1, ALiBi = 2, RoPEALiBi = 3 };
enum class AttnMode : int32_t { Self = 0, Cross = 1 };
enum class SoftmaxKind : int32_t { Standard = 0, Sigmoid = 1 };

struct Config {
  int d_model = 0;
  int num_heads = 0;
  int num_kv_heads = 0;  // 0 -> num_heads
  int head_dim = 0;      // 0 -> d_model / num_heads
  int max_seq_len = 0;   // 0 -> 512

  MaskKind mask = MaskKind::Causal;
  PosKind pos = PosKind::RoPE;
  AttnMode mode = AttnMode::Self;
  SoftmaxKind softmax = SoftmaxKind::Standard;

  bool causal = true;
  int window = 0;
  bool window_causal = true;
  int prefix_len = 0;
  double rope_theta = 10000.0;
  double scale_override = 0.0;

  int q_dim() const { return num_heads * head_dim; }
  int kv_dim() const { return num_kv_heads * head_dim; }
  int heads_per_kv() const { return num_heads / num_kv_heads; }
  WELVET_CXX_API double scale() const;
  bool uses_rope() const { return pos == PosKind::RoPE || pos == PosKind::RoPEALiBi; }
  bool uses_alibi() const { return pos == PosKind::ALiBi || pos == PosKind::RoPEALiBi; }
};

// Defaults and checks of reference validate (src/layers/mha/mha.cpp:63-94).
WELVET_CXX_API Status validate(Config* cfg);
// Causal mask, RoPE, self attention (src/layers/mha/mha.cpp:96-106).
WELVET_CXX_API Config decoder_causal(int d_model, int num_heads, int num_kv_heads);

struct Layer {
  Config cfg{};
  DType dtype = DType::Float32;
  std::shared_ptr<welvet_b200_mha> session;  // resident weights on the GPU; shared by copies
  Config mounted{};                           // cfg as it was when the weights were mounted
};

// Q [q_dim, d], K/V [kv_dim, d], O [d, q_dim] row-major FP32 inits (W[out, in]).
WELVET_CXX_API Status new_configured(const Config& cfg, DType dt, const float* q_init, const float* k_init,
                                     const float* v_init, const float* o_init, Layer* out);

// input [batch, seq, d] or [seq, d]; pre = attention output [batch, seq, q_dim],
// post = O(attention) [batch, seq, d_model].
WELVET_CXX_API Status forward(Layer& layer, const TensorF32& input, TensorF32* pre, TensorF32* post);

}  // namespace welvet::mha

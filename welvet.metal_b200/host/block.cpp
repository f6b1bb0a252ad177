// Host side of the transformer-block forwards around the MHA: the reference's
// SwiGLU, RMSNorm, LayerNorm and Embedding C entries (src/interop/c_abi.cpp:326-361,
// 437-469, 543-577, 792-832) with their argument checks and status codes, a
// resident SwiGLU layer (weights decoded, packed and uploaded once, forward many),
// and device-pointer entries for pipelines that keep activations in HBM.
#include <cuda_runtime.h>

#include <cstdio>
#include <cstring>

#include "../../include/welvet_b200.h"
#include "../../include/welvet_c.h"
#include "engine.hpp"

namespace wv {
namespace {

inline int round_up(int v, int m) { return (v + m - 1) / m * m; }

welvet_status status_c(int code, const char* msg) {
  welvet_status st{};
  st.code = code;
  std::snprintf(st.message, sizeof(st.message), "%s", msg);
  return st;
}

// Decodes n FP32 weights (host or device) as FormatNone `dtype` into dst (device).
Status decode_weights(DeviceCtx* d, int dtype, const float* src, bool on_device, float* dst, int64_t n,
                      cudaStream_t s) {
  WV_CUDA(cudaMemcpyAsync(dst, src, (size_t)n * 4, on_device ? cudaMemcpyDeviceToDevice : cudaMemcpyHostToDevice,
                          s),
          "weights upload");
  const float* stats = nullptr;
  if (codec_needs_stats(dtype)) {
    WV_CUDA(stats_f32(dst, n, d->scalars, d->scratch, s), "tensor stats");
    count_launch(2);
    stats = d->scalars;
  }
  if (dtype != 1) {
    WV_CUDA(codec_roundtrip_f32(dtype, dst, dst, n, stats, s), "codec roundtrip");
    count_launch();
  }
  return Status::ok();
}

}  // namespace

// Resident SwiGLU feed-forward (swiglu.cpp:93-143): h = SiLU(x Gate^T) * (x Up^T),
// post = h Down^T. FP32 (3xTF32 tensor-core GEMMs) or BF16 operands. The Gate|Up
// GEMM writes h directly through its SwiGLU epilogue; `in` is padded to a multiple
// of 4 and `inter` to a multiple of 32 with zero weights (exact).
struct Swiglu {
  DeviceCtx* d = nullptr;
  int in = 0, inter = 0, in_p = 0, inter_p = 0, precision = 0;
  DevBuf gu, gu_lo, dn, dn_lo;            // packed weights (TF32 hi/lo, or bf16 in gu/dn)
  DevBuf xa, xa_lo, h, h_hi, h_lo, post;  // per-call operands (grown on demand)
  DevBuf stage_x, stage_pre;              // host I/O staging
};

Status swiglu_mount(int in, int inter, int precision, int device, int dtype, const float* Gate, const float* Up,
                    const float* Down, bool on_device, Swiglu** out) {
  if (in <= 0 || inter <= 0 || !Gate || !Up || !Down || !out) return Status::err(1, "swiglu: invalid argument");
  if (!codec_dtype_supported(dtype))
    return Status::err(2, "swiglu Gate: dense FormatNone forward unsupported for dtype " + std::to_string(dtype));
  if (precision != 0 && precision != 1) return Status::err(1, "swiglu: precision must be 0 (FP32) or 1 (BF16)");
  DeviceCtx* d = nullptr;
  WV_TRY(device_ctx(device, &d));
  auto* L = new Swiglu();
  std::unique_ptr<Swiglu> guard(L);
  L->d = d;
  L->in = in;
  L->inter = inter;
  L->in_p = round_up(in, precision ? 8 : 4);
  L->inter_p = round_up(inter, 32);
  L->precision = precision;
  cudaStream_t s = 0;
  const int64_t ng = (int64_t)inter * in, nd = (int64_t)in * inter;
  DevBuf g, u, dn_raw, tmp;
  WV_TRY(g.ensure(ng * 4));
  WV_TRY(u.ensure(ng * 4));
  WV_TRY(dn_raw.ensure(nd * 4));
  WV_TRY(decode_weights(d, dtype, Gate, on_device, g.as<float>(), ng, s));
  WV_TRY(decode_weights(d, dtype, Up, on_device, u.as<float>(), ng, s));
  WV_TRY(decode_weights(d, dtype, Down, on_device, dn_raw.as<float>(), nd, s));
  const int64_t n_gu = (int64_t)2 * L->inter_p * L->in_p, n_dn = (int64_t)in * L->inter_p;
  WV_TRY(tmp.ensure(std::max(n_gu, n_dn) * 4));
  WV_CUDA(swiglu_pack_gate_up(g.as<float>(), u.as<float>(), tmp.as<float>(), inter, in, L->inter_p, L->in_p, s),
          "pack gate/up");
  count_launch();
  if (precision == 0) {
    WV_TRY(L->gu.ensure(n_gu * 4));
    WV_TRY(L->gu_lo.ensure(n_gu * 4));
    WV_CUDA(split_tf32(tmp.as<float>(), L->gu.as<float>(), L->gu_lo.as<float>(), n_gu, s), "split gate/up");
  } else {
    WV_TRY(L->gu.ensure(n_gu * 2));
    WV_CUDA(cast_f32_bf16(tmp.as<float>(), L->gu.p, n_gu, s), "cast gate/up");
  }
  count_launch();
  WV_CUDA(pad_cols(dn_raw.as<float>(), tmp.as<float>(), in, inter, L->inter_p, s), "pad down");
  count_launch();
  if (precision == 0) {
    WV_TRY(L->dn.ensure(n_dn * 4));
    WV_TRY(L->dn_lo.ensure(n_dn * 4));
    WV_CUDA(split_tf32(tmp.as<float>(), L->dn.as<float>(), L->dn_lo.as<float>(), n_dn, s), "split down");
  } else {
    WV_TRY(L->dn.ensure(n_dn * 2));
    WV_CUDA(cast_f32_bf16(tmp.as<float>(), L->dn.p, n_dn, s), "cast down");
  }
  count_launch();
  WV_CUDA(cudaStreamSynchronize(s), "swiglu mount");
  *out = guard.release();
  return Status::ok();
}

// x [tokens, in], pre = h [tokens, inter] (may be null), post [tokens, in]: FP32
// arrays for precision 0, BF16 for precision 1; device memory unless `host`
// (then FP32 host memory, copied in and out on `s`, which is synchronised).
Status swiglu_forward(Swiglu* L, int64_t tokens, const void* x, void* pre, void* post, bool host, cudaStream_t s) {
  if (!L || tokens <= 0 || !x || !post) return Status::err(1, "swiglu: invalid argument");
  if (tokens > (1ll << 31) - 1) return Status::err(1, "swiglu: too many tokens");
  const int M = (int)tokens;
  const bool f32 = L->precision == 0;
  const size_t es = f32 ? 4 : 2;
  const void* xd = x;
  if (host) {
    WV_TRY(L->stage_x.ensure((size_t)M * L->in * 4));
    WV_CUDA(cudaMemcpyAsync(L->stage_x.p, x, (size_t)M * L->in * 4, cudaMemcpyHostToDevice, s), "x upload");
    xd = L->stage_x.p;
  }
  // A operand of the Gate|Up GEMM: BF16 x is used in place when its rows are
  // 16-byte aligned; otherwise a zero-padded copy (TF32 pairs or BF16)
  const void* xa = xd;
  const bool x_direct = !f32 && !host && L->in_p == L->in && (reinterpret_cast<uintptr_t>(xd) & 15) == 0;
  if (!x_direct) {
    WV_TRY(L->xa.ensure((size_t)M * L->in_p * es));
    if (f32) WV_TRY(L->xa_lo.ensure((size_t)M * L->in_p * 4));
    WV_CUDA(pad_operand(xd, (host || f32) ? 0 : 1, M, L->in, L->in_p, f32 ? L->xa.as<float>() : nullptr,
                        f32 ? L->xa_lo.as<float>() : nullptr, f32 ? nullptr : L->xa.p, s),
            "pad x");
    count_launch();
    xa = L->xa.p;
  }
  // h: written by the Gate|Up epilogue straight into the caller's pre (device) when
  // its rows can be the Down GEMM's A operand (16-byte aligned), else into [M, inter_p]
  // and copied out; the FP32 layer also keeps h's TF32 split at the same stride
  const int align = f32 ? 4 : 8;
  const bool h_direct = pre && !host && L->inter % align == 0 && (reinterpret_cast<uintptr_t>(pre) & 15) == 0;
  const int ld_h = h_direct ? L->inter : L->inter_p;
  void* h = h_direct ? pre : nullptr;
  if (!h_direct) {
    WV_TRY(L->h.ensure((size_t)M * ld_h * es));
    h = L->h.p;
  }
  if (f32) {
    WV_TRY(L->h_hi.ensure((size_t)M * ld_h * 4));
    WV_TRY(L->h_lo.ensure((size_t)M * ld_h * 4));
  }
  GemmArgs g1;
  g1.kind = f32 ? kGemmTF32x3 : kGemmBF16;
  g1.M = M;
  g1.N = 2 * L->inter_p;
  g1.K = L->in_p;
  g1.a = xa;
  g1.a_lo = f32 ? L->xa_lo.p : nullptr;
  g1.lda = x_direct ? L->in : L->in_p;
  g1.b = L->gu.p;
  g1.b_lo = f32 ? L->gu_lo.p : nullptr;
  g1.ldb = L->in_p;
  g1.out = h;
  g1.ldo = ld_h;
  g1.swiglu_cols = h_direct ? L->inter : L->inter_p;
  g1.out_bf16 = f32 ? 0 : 1;
  g1.out_hi = f32 ? L->h_hi.as<float>() : nullptr;
  g1.out_lo = f32 ? L->h_lo.as<float>() : nullptr;
  g1.swiglu = 1;
  g1.err = L->d->err;
  g1.sm_count = L->d->sm_count;
  if (!gemm_tc_supported(g1)) return Status::err(4, "swiglu: Gate|Up GEMM operands not TMA-aligned");
  prof_begin(kProfGemmGateUp, s);
  WV_CUDA(gemm_tc(g1, s), "swiglu gate|up gemm");
  prof_end(kProfGemmGateUp, s);
  count_launch();
  void* post_d = post;
  if (host) {
    WV_TRY(L->post.ensure((size_t)M * L->in * 4));
    post_d = L->post.p;
  }
  GemmArgs g2;
  g2.kind = g1.kind;
  g2.M = M;
  g2.N = L->in;
  g2.K = ld_h;
  g2.a = f32 ? L->h_hi.p : h;
  g2.a_lo = f32 ? L->h_lo.p : nullptr;
  g2.lda = ld_h;
  g2.b = L->dn.p;
  g2.b_lo = f32 ? L->dn_lo.p : nullptr;
  g2.ldb = L->inter_p;
  g2.out = post_d;
  g2.ldo = L->in;
  g2.out_bf16 = f32 ? 0 : 1;
  g2.err = L->d->err;
  g2.sm_count = L->d->sm_count;
  if (!gemm_tc_supported(g2)) return Status::err(4, "swiglu: Down GEMM operands not TMA-aligned");
  prof_begin(kProfGemmDown, s);
  WV_CUDA(gemm_tc(g2, s), "swiglu down gemm");
  prof_end(kProfGemmDown, s);
  count_launch();
  if (pre && !h_direct) {
    WV_CUDA(cudaMemcpy2DAsync(pre, (size_t)L->inter * es, h, (size_t)ld_h * es, (size_t)L->inter * es, M,
                              host ? cudaMemcpyDeviceToHost : cudaMemcpyDeviceToDevice, s),
            "pre copy");
  }
  if (host) {
    WV_CUDA(cudaMemcpyAsync(post, post_d, (size_t)M * L->in * 4, cudaMemcpyDeviceToHost, s), "post download");
    WV_CUDA(cudaStreamSynchronize(s), "swiglu forward");
    WV_TRY(check_device_error(L->d));
  }
  return Status::ok();
}

void swiglu_release(Swiglu* L) { delete L; }

// One-shot norm over host buffers: upload, decode gamma/beta, kernel, download.
Status norm_forward_host(int layernorm, int batch, int seq, int dim, double eps, int dtype, const float* gamma,
                         const float* beta, const float* x, float* pre, float* post) {
  const char* name = layernorm ? "layernorm" : "rmsnorm";
  if (!codec_dtype_supported(dtype))
    return Status::err(3, std::string(name) + " gamma: gap? pack_native unknown");
  if (eps <= 0) eps = layernorm ? 1e-5 : 1e-6;  // validate() defaults
  DeviceCtx* d = nullptr;
  WV_TRY(device_ctx(-1, &d));
  cudaStream_t s = 0;
  const int64_t n = (int64_t)batch * seq * dim;
  DevBuf w, xb, pb, qb;
  WV_TRY(w.ensure((size_t)2 * dim * 4));
  WV_TRY(xb.ensure((size_t)n * 4));
  WV_TRY(pb.ensure((size_t)n * 4));
  WV_TRY(qb.ensure((size_t)n * 4));
  WV_TRY(decode_weights(d, dtype, gamma, false, w.as<float>(), dim, s));
  if (layernorm) WV_TRY(decode_weights(d, dtype, beta, false, w.as<float>() + dim, dim, s));
  WV_CUDA(cudaMemcpyAsync(xb.p, x, (size_t)n * 4, cudaMemcpyHostToDevice, s), "x upload");
  NormArgs a;
  a.rows = (int64_t)batch * seq;
  a.dim = dim;
  a.eps = eps;
  a.x = xb.p;
  a.gamma = w.as<float>();
  a.beta = layernorm ? w.as<float>() + dim : nullptr;
  a.pre = pb.p;
  a.post = qb.p;
  prof_begin(kProfNorm, s);
  WV_CUDA(norm_forward(a, layernorm, s), "norm forward");
  prof_end(kProfNorm, s);
  count_launch();
  WV_CUDA(cudaMemcpyAsync(pre, pb.p, (size_t)n * 4, cudaMemcpyDeviceToHost, s), "pre download");
  WV_CUDA(cudaMemcpyAsync(post, qb.p, (size_t)n * 4, cudaMemcpyDeviceToHost, s), "post download");
  WV_CUDA(cudaStreamSynchronize(s), "norm forward");
  return check_device_error(d);
}

Status embedding_forward_host(int batch, int vocab, int emb, int seq_len, int in_rank, int in_last, int act,
                              int dtype, const float* W, const float* x, float* pre, float* post) {
  if (!codec_dtype_supported(dtype)) return Status::err(3, "embedding weights: gap? pack_native unknown");
  // parse_layout (embedding.cpp): rank 3 needs in_last 1 or emb
  if (in_rank == 3 && in_last != 1 && in_last != emb)
    return Status::err(1, "embedding: input last dim want 1 or emb");
  if (in_rank < 3) in_last = 1;
  const int64_t tokens = in_rank == 1 ? seq_len : (int64_t)batch * seq_len;
  DeviceCtx* d = nullptr;
  WV_TRY(device_ctx(-1, &d));
  cudaStream_t s = 0;
  const int64_t nw = (int64_t)vocab * emb, nx = tokens * in_last, no = tokens * emb;
  DevBuf wb, xb, ob;
  WV_TRY(wb.ensure((size_t)nw * 4));
  WV_TRY(xb.ensure((size_t)nx * 4));
  WV_TRY(ob.ensure((size_t)no * 4));
  WV_TRY(decode_weights(d, dtype, W, false, wb.as<float>(), nw, s));
  WV_CUDA(cudaMemcpyAsync(xb.p, x, (size_t)nx * 4, cudaMemcpyHostToDevice, s), "ids upload");
  EmbedArgs a;
  a.tokens = tokens;
  a.vocab = vocab;
  a.emb = emb;
  a.in_last = in_last;
  a.act = act;
  a.W = wb.as<float>();
  a.x = xb.as<float>();
  a.out = ob.p;
  prof_begin(kProfEmbedding, s);
  WV_CUDA(embedding_forward(a, s), "embedding forward");
  prof_end(kProfEmbedding, s);
  count_launch();
  WV_CUDA(cudaMemcpyAsync(pre, ob.p, (size_t)no * 4, cudaMemcpyDeviceToHost, s), "pre download");
  WV_CUDA(cudaMemcpyAsync(post, ob.p, (size_t)no * 4, cudaMemcpyDeviceToHost, s), "post download");
  WV_CUDA(cudaStreamSynchronize(s), "embedding forward");
  return check_device_error(d);
}

}  // namespace wv

using wv::Status;

extern "C" {

struct welvet_b200_swiglu {
  wv::Swiglu* impl;
};

// Reference src/interop/c_abi.cpp:326-361.
welvet_status welvet_swiglu_forward_f32(int32_t batch, int32_t seq, int32_t input_dim, int32_t intermediate_dim,
                                        int32_t dtype, int32_t /*backend*/, const float* Gate, const float* Up,
                                        const float* Down, const float* x, float* pre, float* post) {
  wv::DeviceRestore restore_device;
  if (batch <= 0 || seq <= 0 || input_dim <= 0 || intermediate_dim <= 0 || !Gate || !Up || !Down || !x || !pre ||
      !post)
    return wv::status_c(1, "swiglu: invalid argument");
  wv::Swiglu* L = nullptr;
  Status st = wv::swiglu_mount(input_dim, intermediate_dim, 0, -1, dtype, Gate, Up, Down, false, &L);
  if (!st) return wv::to_c(st);
  st = wv::swiglu_forward(L, (int64_t)batch * seq, x, pre, post, true, 0);
  wv::swiglu_release(L);
  return wv::to_c(st);
}

// Reference src/interop/c_abi.cpp:437-469.
welvet_status welvet_rmsnorm_forward_f32(int32_t batch, int32_t seq, int32_t dim, double eps, int32_t dtype,
                                         int32_t /*backend*/, const float* gamma, const float* x, float* pre,
                                         float* post) {
  if (batch <= 0 || seq <= 0 || dim <= 0 || !gamma || !x || !pre || !post)
    return wv::status_c(1, "rmsnorm: invalid argument");
  return wv::to_c(wv::norm_forward_host(0, batch, seq, dim, eps, dtype, gamma, nullptr, x, pre, post));
}

// Reference src/interop/c_abi.cpp:543-577.
welvet_status welvet_layernorm_forward_f32(int32_t batch, int32_t seq, int32_t dim, double eps, int32_t dtype,
                                           int32_t /*backend*/, const float* gamma, const float* beta,
                                           const float* x, float* pre, float* post) {
  if (batch <= 0 || seq <= 0 || dim <= 0 || !gamma || !beta || !x || !pre || !post)
    return wv::status_c(1, "layernorm: invalid argument");
  return wv::to_c(wv::norm_forward_host(1, batch, seq, dim, eps, dtype, gamma, beta, x, pre, post));
}

// Reference src/interop/c_abi.cpp:792-832.
welvet_status welvet_embedding_forward_f32(int32_t batch, int32_t vocab, int32_t emb, int32_t seq_len,
                                           int32_t in_rank, int32_t in_last, int32_t act, int32_t dtype,
                                           int32_t /*backend*/, const float* W, const float* x, float* pre,
                                           float* post) {
  if (batch <= 0 || vocab <= 0 || emb <= 0 || seq_len <= 0 || in_last <= 0 || !W || !x || !pre || !post)
    return wv::status_c(1, "embedding: invalid argument");
  if (in_rank < 1 || in_rank > 3) return wv::status_c(1, "embedding: bad in_rank");
  return wv::to_c(
      wv::embedding_forward_host(batch, vocab, emb, seq_len, in_rank, in_last, act, dtype, W, x, pre, post));
}

welvet_status welvet_b200_swiglu_mount(int32_t input_dim, int32_t intermediate_dim, int32_t precision,
                                       int32_t device, int32_t dtype, const float* Gate, const float* Up,
                                       const float* Down, int32_t weights_on_device, welvet_b200_swiglu** out) {
  wv::DeviceRestore restore_device;
  if (!out) return wv::status_c(1, "swiglu: invalid argument");
  wv::Swiglu* L = nullptr;
  Status st = wv::swiglu_mount(input_dim, intermediate_dim, precision, device, dtype, Gate, Up, Down,
                               weights_on_device != 0, &L);
  if (!st) return wv::to_c(st);
  *out = new welvet_b200_swiglu{L};
  return wv::to_c(st);
}

welvet_status welvet_b200_swiglu_forward(welvet_b200_swiglu* layer, int64_t tokens, const void* x, void* pre,
                                         void* post, void* stream) {
  wv::DeviceRestore restore_device;
  if (!layer) return wv::status_c(1, "swiglu: invalid argument");
  return wv::to_c(wv::swiglu_forward(layer->impl, tokens, x, pre, post, false, static_cast<cudaStream_t>(stream)));
}

welvet_status welvet_b200_swiglu_forward_host(welvet_b200_swiglu* layer, int64_t tokens, const float* x,
                                              float* pre, float* post) {
  wv::DeviceRestore restore_device;
  if (!layer) return wv::status_c(1, "swiglu: invalid argument");
  if (layer->impl->precision != 0) return wv::status_c(2, "swiglu: host buffers need the FP32 layer");
  return wv::to_c(wv::swiglu_forward(layer->impl, tokens, x, pre, post, true, 0));
}

void welvet_b200_swiglu_release(welvet_b200_swiglu* layer) {
  wv::DeviceRestore restore_device;
  if (!layer) return;
  cudaDeviceSynchronize();
  wv::swiglu_release(layer->impl);
  delete layer;
}

welvet_status welvet_b200_norm_forward(int32_t layernorm, int64_t rows, int32_t dim, double eps, const float* gamma,
                                       const float* beta, const void* x, void* pre, void* post, int32_t io_bf16,
                                       void* stream) {
  if (rows <= 0 || dim <= 0 || !gamma || (layernorm && !beta) || !x || !post)
    return wv::status_c(1, layernorm ? "layernorm: invalid argument" : "rmsnorm: invalid argument");
  if (eps <= 0) eps = layernorm ? 1e-5 : 1e-6;
  wv::NormArgs a;
  a.rows = rows;
  a.dim = dim;
  a.eps = eps;
  a.x = x;
  a.x_bf16 = io_bf16 != 0;
  a.gamma = gamma;
  a.beta = layernorm ? beta : nullptr;
  a.pre = pre;
  a.post = post;
  a.out_bf16 = io_bf16 != 0;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  wv::prof_begin(wv::kProfNorm, s);
  cudaError_t e = wv::norm_forward(a, layernorm != 0, s);
  wv::prof_end(wv::kProfNorm, s);
  wv::count_launch();
  return wv::to_c(e == cudaSuccess ? Status::ok() : wv::cuda_status(e, "norm forward"));
}

welvet_status welvet_b200_embedding_forward(int64_t tokens, int32_t vocab, int32_t emb, int32_t in_last,
                                            int32_t act, const float* W, const float* x, void* out,
                                            int32_t out_bf16, void* stream) {
  if (tokens <= 0 || vocab <= 0 || emb <= 0 || in_last <= 0 || !W || !x || !out)
    return wv::status_c(1, "embedding: invalid argument");
  wv::EmbedArgs a;
  a.tokens = tokens;
  a.vocab = vocab;
  a.emb = emb;
  a.in_last = in_last;
  a.act = act;
  a.W = W;
  a.x = x;
  a.out = out;
  a.out_bf16 = out_bf16 != 0;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  wv::prof_begin(wv::kProfEmbedding, s);
  cudaError_t e = wv::embedding_forward(a, s);
  wv::prof_end(wv::kProfEmbedding, s);
  wv::count_launch();
  return wv::to_c(e == cudaSuccess ? Status::ok() : wv::cuda_status(e, "embedding forward"));
}

}  // extern "C"

// extern "C" entry points: the welvet_c.h MHA subset (drop-in for the
// reference's src/interop/c_abi.cpp MHA entries) and the welvet_b200.h extension.
#include <climits>
#include <cstdio>
#include <cstring>
#include <memory>
#include <mutex>
#include <string>

#include "engine.hpp"

using wv::Status;

namespace {

const char* kVersion = "0.71";

welvet_status ok_status() { return wv::to_c(Status::ok()); }

cudaStream_t as_stream(void* s) { return static_cast<cudaStream_t>(s); }

welvet_status launch_status(cudaError_t e, const char* what) {
  if (e == cudaSuccess) return ok_status();
  return wv::to_c(wv::cuda_status(e, what));
}

} // namespace

struct welvet_b200_mha {
  wv::Mha* m = nullptr;
};
struct welvet_b200_kv {
  wv::Kv* kv = nullptr;
};

extern "C" {

// ------------------------------------------------------------- welvet_c.h
const char* welvet_version(void) { return kVersion; }

const char* welvet_runtime_identity(void) {
  static thread_local std::string id;
  int dev = 0;
  cudaDeviceProp prop{};
  if (cudaGetDevice(&dev) != cudaSuccess || cudaGetDeviceProperties(&prop, dev) != cudaSuccess) {
    id = "cuda:unavailable:welvet-b200";
    cudaGetLastError();
  } else {
    char buf[160];
    std::snprintf(buf, sizeof(buf), "cuda:%s:sm_%d%d:welvet-b200", prop.name, prop.major, prop.minor);
    id = buf;
  }
  return id.c_str();
}

welvet_status welvet_metal_init(void) {
  wv::DeviceCtx* d = nullptr;
  return wv::to_c(wv::device_ctx(-1, &d));
}

int32_t welvet_metal_available(void) {
  int n = 0;
  if (cudaGetDeviceCount(&n) != cudaSuccess) {
    cudaGetLastError();
    return 0;
  }
  for (int i = 0; i < n; ++i) {
    cudaDeviceProp prop{};
    if (cudaGetDeviceProperties(&prop, i) == cudaSuccess && prop.major == 10) return 1;
  }
  return 0;
}

// Reference src/interop/c_abi.cpp:209-247: argument checks, Config fill, layer
// construction (encode every weight to `dtype`), forward, copy-out. Nothing retained.
welvet_status welvet_mha_forward_f32(int32_t batch, int32_t seq, int32_t d_model, int32_t num_heads,
                                     int32_t num_kv_heads, int32_t head_dim, int32_t max_seq_len,
                                     int32_t mask, int32_t pos, int32_t dtype, int32_t /*backend*/,
                                     const float* Q, const float* K, const float* V, const float* O,
                                     const float* x, float* pre, float* post) {
  wv::DeviceRestore restore_device;
  if (batch <= 0 || seq <= 0 || d_model <= 0 || num_heads <= 0 || !Q || !K || !V || !O || !x || !pre ||
      !post) {
    welvet_status st{};
    st.code = 1;
    std::snprintf(st.message, sizeof(st.message), "mha: invalid argument");
    return st;
  }
  if (dtype < 0 || dtype >= 34) {
    welvet_status st{};
    st.code = 2;
    std::snprintf(st.message, sizeof(st.message),
                  "mha Q: dense FormatNone forward unsupported for dtype %d", dtype);
    return st;
  }
  welvet_b200_mha_config cfg{};
  cfg.d_model = d_model;
  cfg.num_heads = num_heads;
  cfg.num_kv_heads = num_kv_heads;
  cfg.head_dim = head_dim;
  cfg.max_seq_len = max_seq_len;
  cfg.mask = mask;
  cfg.pos = pos;
  cfg.softmax = 0;
  cfg.window = 0;
  cfg.prefix_len = 0;
  cfg.window_causal = 1;  // Config default (mha.hpp:53), passed as c[11] = window_causal || causal
  cfg.rope_theta = 10000.0;
  cfg.scale_override = 0.0;
  cfg.seq_mode = 0;
  cfg.precision = 0;
  cfg.weight_format = 0;
  cfg.device = -1;
  wv::Mha* m = nullptr;
  Status st = wv::mha_mount(cfg, dtype, Q, K, V, O, false, &m);
  if (!st) return wv::to_c(st);
  std::unique_ptr<wv::Mha> hold(m);
  st = wv::mha_forward(m, batch, seq, x, pre, post, false, 0);
  return wv::to_c(st);
}

// -------------------------------------------------------------- extension
void welvet_b200_mha_config_default(welvet_b200_mha_config* cfg, int32_t d_model, int32_t num_heads,
                                    int32_t num_kv_heads) {
  if (!cfg) return;
  std::memset(cfg, 0, sizeof(*cfg));
  cfg->d_model = d_model;
  cfg->num_heads = num_heads;
  cfg->num_kv_heads = num_kv_heads;
  cfg->mask = 1;
  cfg->pos = 0;
  cfg->window_causal = 1;
  cfg->rope_theta = 10000.0;
  cfg->seq_mode = 1;
  cfg->device = -1;
}

welvet_status welvet_b200_mha_mount(const welvet_b200_mha_config* cfg, int32_t dtype, const float* Q,
                                    const float* K, const float* V, const float* O, int32_t weights_on_device,
                                    welvet_b200_mha** out) {
  wv::DeviceRestore restore_device;
  if (!cfg || !out) return wv::to_c(Status::err(1, "mha: invalid argument"));
  wv::Mha* m = nullptr;
  Status st = wv::mha_mount(*cfg, dtype, Q, K, V, O, weights_on_device != 0, &m);
  if (!st) return wv::to_c(st);
  *out = new welvet_b200_mha{m};
  return ok_status();
}

void welvet_b200_mha_release(welvet_b200_mha* layer) {
  wv::DeviceRestore restore_device;
  if (!layer) return;
  delete layer->m;
  delete layer;
}

welvet_status welvet_b200_mha_forward(welvet_b200_mha* layer, int32_t batch, int32_t seq, const void* x,
                                      void* pre, void* post, int32_t on_device, void* stream) {
  wv::DeviceRestore restore_device;
  if (!layer) return wv::to_c(Status::err(1, "mha: nil layer"));
  return wv::to_c(wv::mha_forward(layer->m, batch, seq, x, pre, post, on_device != 0, as_stream(stream)));
}

welvet_status welvet_b200_mha_forward_rows(welvet_b200_mha* layer, int32_t batch_local, int32_t seq, const void* x,
                                           void* post) {
  wv::DeviceRestore restore_device;
  if (!layer) return wv::to_c(Status::err(1, "mha: nil layer"));
  wv::Mha* m = layer->m;
  const bool sharded = m->comm && m->nranks > 1;
  if (batch_local <= 0 || (sharded && (int64_t)batch_local * m->nranks > INT32_MAX))
    return wv::to_c(Status::err(1, "mha: invalid argument"));
  const int batch = sharded ? batch_local * m->nranks : batch_local;
  return wv::to_c(wv::mha_forward(m, batch, seq, x, nullptr, post, false, nullptr, nullptr, sharded));
}

welvet_status welvet_b200_mha_set_output_mode(welvet_b200_mha* layer, int32_t mode) {
  if (!layer || mode < 0 || mode > 2) return wv::to_c(Status::err(1, "mha: invalid output mode"));
  std::lock_guard<std::mutex> lock(layer->m->mu);
  layer->m->out_mode = mode;
  return ok_status();
}

welvet_status welvet_b200_mha_check(welvet_b200_mha* layer) {
  wv::DeviceRestore restore_device;
  if (!layer) return wv::to_c(Status::err(1, "mha: nil layer"));
  Status st = wv::check_device_error(layer->m->dev);
  if (!st) return wv::to_c(st);
  return wv::to_c(wv::comm_poll(layer->m));
}

welvet_status welvet_b200_kv_create(welvet_b200_mha* layer, int32_t max_batch, int32_t max_ctx,
                                    welvet_b200_kv** out) {
  wv::DeviceRestore restore_device;
  if (!layer || !out) return wv::to_c(Status::err(1, "kv: invalid argument"));
  wv::Kv* kv = nullptr;
  Status st = wv::kv_create(layer->m, max_batch, max_ctx, &kv);
  if (!st) return wv::to_c(st);
  *out = new welvet_b200_kv{kv};
  return ok_status();
}

void welvet_b200_kv_release(welvet_b200_kv* kv) {
  wv::DeviceRestore restore_device;
  if (!kv) return;
  delete kv->kv;
  delete kv;
}

welvet_status welvet_b200_kv_fill(welvet_b200_kv* kv, int32_t batch, int32_t ctx_len, const void* k,
                                  const void* v, int32_t on_device, void* stream) {
  wv::DeviceRestore restore_device;
  if (!kv) return wv::to_c(Status::err(1, "kv: nil cache"));
  return wv::to_c(wv::kv_fill(kv->kv, batch, ctx_len, k, v, on_device != 0, as_stream(stream)));
}

welvet_status welvet_b200_mha_prefill(welvet_b200_mha* layer, welvet_b200_kv* kv, int32_t batch, int32_t seq,
                                      const void* x, void* pre, void* post, int32_t on_device, void* stream) {
  wv::DeviceRestore restore_device;
  if (!layer || !kv) return wv::to_c(Status::err(1, "mha prefill: invalid argument"));
  if (layer->m->cfg.c.seq_mode != 1)
    return wv::to_c(Status::err(1, "mha prefill: needs seq_mode 1 (per-sequence positions)"));
  if (batch > kv->kv->max_batch || seq > kv->kv->max_ctx)
    return wv::to_c(Status::err(1, "mha prefill: exceeds the KV cache"));
  return wv::to_c(wv::mha_forward(layer->m, batch, seq, x, pre, post, on_device != 0, as_stream(stream), kv->kv));
}

welvet_status welvet_b200_mha_decode(welvet_b200_mha* layer, welvet_b200_kv* kv, int32_t batch, const void* x_new,
                                     void* pre, void* post, int32_t on_device, void* stream) {
  wv::DeviceRestore restore_device;
  if (!layer || !kv) return wv::to_c(Status::err(1, "mha decode: invalid argument"));
  return wv::to_c(wv::mha_decode(layer->m, kv->kv, batch, x_new, pre, post, on_device != 0, as_stream(stream)));
}

welvet_status welvet_b200_comm_unique_id(uint8_t id[128]) { return wv::to_c(wv::comm_unique_id(id)); }

welvet_status welvet_b200_comm_attach(welvet_b200_mha* layer, const uint8_t id[128], int32_t nranks,
                                      int32_t rank) {
  wv::DeviceRestore restore_device;
  if (!layer) return wv::to_c(Status::err(1, "comm: nil layer"));
  return wv::to_c(wv::comm_attach(layer->m, id, nranks, rank));
}

// ------------------------------------------------------- kernel-level entries
welvet_status welvet_b200_gemm(int32_t kind, int32_t M, int32_t N, int32_t K, const void* a, const void* a_lo,
                               const void* b, const void* b_lo, const float* b_scale, void* out, int32_t out_bf16,
                               void* stream) {
  wv::DeviceCtx* d = nullptr;
  Status st = wv::device_ctx(-1, &d);
  if (!st) return wv::to_c(st);
  wv::GemmArgs g;
  g.kind = kind;
  g.M = M;
  g.N = N;
  g.K = K;
  g.a = a;
  g.a_lo = a_lo;
  g.lda = K;
  g.b = b;
  g.b_lo = b_lo;
  g.ldb = K;
  g.b_scale = b_scale;
  g.out = out;
  g.ldo = N;
  g.out_bf16 = out_bf16;
  g.err = d->err;
  g.sm_count = d->sm_count;
  if (!wv::gemm_tc_supported(g)) return wv::to_c(Status::err(2, "gemm: shape/alignment not supported by TMA"));
  wv::count_launch();
  return launch_status(wv::gemm_tc(g, as_stream(stream)), "gemm_tc");
}

welvet_status welvet_b200_split_tf32(const float* x, float* hi, float* lo, int64_t n, void* stream) {
  wv::count_launch();
  return launch_status(wv::split_tf32(x, hi, lo, n, as_stream(stream)), "split_tf32");
}

namespace {
// Attention arguments of a kernel-level call: q/k/v/out token-major with the
// configuration's natural row strides.
Status attention_args(const welvet_b200_mha_config* cfgp, int32_t batch, int32_t seq, const void* q, const void* k,
                      const void* v, void* out, wv::AttnArgs* out_args) {
  if (!cfgp || !q || !k || !v || !out || batch <= 0 || seq <= 0) return Status::err(1, "attention: invalid argument");
  wv::Cfg c;
  Status st = wv::resolve_config(*cfgp, &c);
  if (!st) return st;
  wv::DeviceCtx* d = nullptr;
  st = wv::device_ctx(c.c.device, &d);
  if (!st) return st;
  wv::AttnArgs& a = *out_args;
  a.q = q;
  a.k = k;
  a.v = v;
  a.ldq = c.qd;
  a.ldk = c.kd;
  a.out = out;
  a.ldo = c.qd;
  a.is_bf16 = c.c.precision == 1;
  a.batch = batch;
  a.seq = seq;
  a.num_heads = c.c.num_heads;
  a.num_kv_heads = c.nk;
  a.head_dim = c.hd;
  a.stream_mode = c.c.seq_mode == 0;
  a.mask = c.c.mask;
  a.window = c.c.window;
  a.max_seq_len = c.msl;
  a.prefix_len = c.c.prefix_len;
  a.window_causal = c.c.window_causal;
  a.alibi = c.alibi;
  a.sigmoid = c.c.softmax == 1;
  a.head_base = 0;
  a.total_heads = c.c.num_heads;
  a.scale = c.scale;
  a.err = d->err;
  a.sm_count = d->sm_count;
  a.tile_ctr = d->tile_ctr;
  return Status::ok();
}
}  // namespace

welvet_status welvet_b200_attention(const welvet_b200_mha_config* cfgp, int32_t batch, int32_t seq, const void* q,
                                    const void* k, const void* v, void* out, int32_t impl, void* stream) {
  wv::DeviceRestore restore_device;
  wv::AttnArgs a;
  Status st = attention_args(cfgp, batch, seq, q, k, v, out, &a);
  if (!st) return wv::to_c(st);
  wv::count_launch();
  if (impl == 3) {  // tensor-core kernel on CTA pairs (M = 256 UMMAs)
    if (!wv::attn_tc_pair_supported(a))
      return wv::to_c(Status::err(2, "attention: CTA-pair tensor-core kernel unsupported here"));
    a.pair = 1;
    return launch_status(wv::attn_prefill_tc(a, as_stream(stream)), "attn_prefill_tc (pairs)");
  }
  if (impl == 2 || impl == 4 || (impl == 0 && wv::attn_tc_supported(a))) {
    if (!wv::attn_tc_supported(a)) return wv::to_c(Status::err(2, "attention: tensor-core kernel unsupported here"));
    if (impl == 2 || impl == 4) a.pair = 0;
    if (impl == 4) a.tile_ctr = nullptr;  // one CTA per query tile
    return launch_status(wv::attn_prefill_tc(a, as_stream(stream)), "attn_prefill_tc");
  }
  return launch_status(wv::attn_prefill_simt(a, as_stream(stream)), "attn_prefill_simt");
}

welvet_status welvet_b200_attention_tf32(const welvet_b200_mha_config* cfgp, int32_t batch, int32_t seq,
                                         const float* q_hi, const float* q_lo, const float* k_hi, const float* k_lo,
                                         const float* v_hi, const float* v_lo, float* out, float* out_hi,
                                         float* out_lo, void* stream) {
  wv::DeviceRestore restore_device;
  wv::AttnArgs a;
  Status st = attention_args(cfgp, batch, seq, q_hi, k_hi, v_hi, out, &a);
  if (!st) return wv::to_c(st);
  if (!q_lo || !k_lo || !v_lo || (out_hi == nullptr) != (out_lo == nullptr))
    return wv::to_c(Status::err(1, "attention: invalid argument"));
  a.q_lo = q_lo;
  a.k_lo = k_lo;
  a.v_lo = v_lo;
  a.out_hi = out_hi;
  a.out_lo = out_lo;
  if (!wv::attn_tf32_supported(a)) return wv::to_c(Status::err(2, "attention: 3xTF32 kernel unsupported here"));
  wv::count_launch();
  return launch_status(wv::attn_prefill_tf32(a, as_stream(stream)), "attn_prefill_tf32");
}

welvet_status welvet_b200_codec_roundtrip(int32_t dtype, const float* w, float* out, int64_t n, void* stream) {
  wv::DeviceCtx* d = nullptr;
  Status st = wv::device_ctx(-1, &d);
  if (!st) return wv::to_c(st);
  if (!wv::codec_dtype_supported(dtype) || n < 0 || (n > 0 && (!w || !out)))
    return wv::to_c(Status::err(1, "codec_roundtrip: invalid argument"));
  cudaStream_t s = as_stream(stream);
  const float* stats = nullptr;
  if (wv::codec_needs_stats(dtype) && n > 0) {
    cudaError_t e = wv::stats_f32(w, n, d->scalars, d->scratch, s);
    if (e != cudaSuccess) return launch_status(e, "tensor stats");
    stats = d->scalars;
    wv::count_launch(2);
  }
  wv::count_launch();
  return launch_status(wv::codec_roundtrip_f32(dtype, w, out, n, stats, s), "codec_roundtrip");
}

welvet_status welvet_b200_codec_encode(int32_t dtype, const float* w, void* codes, float* scale_out, int64_t n,
                                       void* stream) {
  wv::DeviceCtx* d = nullptr;
  Status st = wv::device_ctx(-1, &d);
  if (!st) return wv::to_c(st);
  cudaStream_t s = as_stream(stream);
  if (dtype == 9 || dtype == 14 || dtype == 16) {
    // Int8 / Int4 / FP4 bytes of pack_native with the per-tensor scale (the codes the
    // dequantising GEMM keeps resident); scale_out receives the scale (n / 1 row)
    if (!scale_out || n <= 0 || n > INT32_MAX) return wv::to_c(Status::err(1, "codec: invalid argument"));
    cudaError_t e = wv::stats_f32(w, n, d->scalars, d->scratch, s);
    if (e != cudaSuccess) return launch_status(e, "stats");
    wv::count_launch(3);
    return launch_status(wv::formatnone_codes_encode(dtype, w, n, (int)n, d->scalars,
                                                     static_cast<uint8_t*>(codes), scale_out, s),
                         "formatnone codes");
  }
  if (dtype == 26) {
    if (!scale_out) return wv::to_c(Status::err(1, "codec: nf4 needs scale_out"));
    cudaError_t e = wv::absmax_f32(w, n, scale_out, d->scratch, s);
    if (e != cudaSuccess) return launch_status(e, "absmax");
    wv::count_launch(2);
  }
  wv::count_launch();
  return launch_status(wv::codec_encode(dtype, w, codes, n, scale_out, s), "codec_encode");
}

welvet_status welvet_b200_codec_decode(int32_t dtype, const void* codes, const float* scale, float* out, int64_t n,
                                       void* stream) {
  wv::count_launch();
  return launch_status(wv::codec_decode(dtype, codes, out, n, scale, as_stream(stream)), "codec_decode");
}

welvet_status welvet_b200_fp8_rowscale_encode(const float* w, int32_t rows, int32_t cols, uint8_t* codes,
                                              float* scales, void* stream) {
  wv::count_launch();
  return launch_status(wv::fp8_rowscale_encode(w, rows, cols, codes, scales, as_stream(stream)), "fp8 encode");
}
welvet_status welvet_b200_fp8_rowscale_decode(const uint8_t* codes, const float* scales, int32_t rows, int32_t cols,
                                              void* out, int32_t out_bf16, void* stream) {
  wv::count_launch();
  return launch_status(wv::fp8_rowscale_decode(codes, scales, rows, cols, out, out_bf16, as_stream(stream)),
                       "fp8 decode");
}
welvet_status welvet_b200_nf4_block_encode(const float* w, int64_t n, uint8_t* packed, float* absmax, void* stream) {
  wv::count_launch();
  return launch_status(wv::nf4_block_encode(w, n, packed, absmax, as_stream(stream)), "nf4 encode");
}
welvet_status welvet_b200_nf4_block_decode(const uint8_t* packed, const float* absmax, int64_t n, void* out,
                                           int32_t out_bf16, void* stream) {
  wv::count_launch();
  return launch_status(wv::nf4_block_decode(packed, absmax, n, out, out_bf16, as_stream(stream)), "nf4 decode");
}

welvet_status welvet_b200_fill_synthetic(void* dst, int32_t is_bf16, int64_t n, uint64_t seed, uint64_t offset,
                                         int32_t kind, double a, void* stream) {
  wv::count_launch();
  return launch_status(wv::fill_synthetic(dst, is_bf16, n, seed, offset, kind, a, as_stream(stream)), "fill");
}

welvet_status welvet_b200_device_check(void) {
  wv::DeviceCtx* d = nullptr;
  Status st = wv::device_ctx(-1, &d);
  if (!st) return wv::to_c(st);
  return wv::to_c(wv::check_device_error(d));
}

welvet_status welvet_b200_wait_probe(uint64_t limit_ns, void* stream) {
  if (limit_ns == 0 || limit_ns > 10000000000ull) return wv::to_c(Status::err(1, "wait probe: limit out of range"));
  wv::DeviceCtx* d = nullptr;
  Status st = wv::device_ctx(-1, &d);
  if (!st) return wv::to_c(st);
  wv::count_launch();
  return launch_status(wv::wait_probe(d->err, limit_ns, as_stream(stream)), "wait_probe");
}

int64_t welvet_b200_launch_count(int32_t reset) {
  if (reset) return wv::g_launches.exchange(0);
  return wv::g_launches.load();
}

void welvet_b200_profile_enable(int32_t on) { wv::prof_enable(on != 0); }

void welvet_b200_profile_read(double ms[14], int64_t counts[14], int32_t reset) {
  wv::prof_read(ms, counts, reset != 0);
}

} // extern "C"

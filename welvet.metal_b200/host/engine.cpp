// Host orchestration of the MHA forward on B200. See engine.hpp.
//
// Weight layouts in HBM (per layer, for this rank's head shard):
//   wqkv  [nqkv, d]   rows = Wq[heads h0..h0+hc) | Wk[kv heads] | Wv[kv heads]
//                     precision 0: TF32 hi part (fp32), wqkv_lo the lo part
//                     precision 1: bf16, or FP8 codes (+ wqkv_scale [nqkv]) or
//                     NF4 packed [nqkv, d/2] (+ wqkv_scale [nqkv, d/64])
//   wo    [d, qd_l]   the Wo columns of this shard (row-sharded output projection)
// Activations are token-major: x [M, d], qkv [M, nqkv], attn [M, qd_l], post [M, d].
#include "engine.hpp"

#include <algorithm>
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <map>

namespace wv {

std::atomic<int64_t> g_launches{0};

// ---------------------------------------------------------------- profiler
namespace {
struct ProfState {
  std::mutex mu;
  bool on = false;
  struct Rec {
    int id;
    cudaEvent_t a, b;
    bool closed;
  };
  std::vector<Rec> pending;
  std::vector<cudaEvent_t> pool;
  double ms[kProfCount] = {};
  int64_t counts[kProfCount] = {};
  cudaEvent_t get() {
    if (!pool.empty()) {
      cudaEvent_t e = pool.back();
      pool.pop_back();
      return e;
    }
    cudaEvent_t e = nullptr;
    cudaEventCreate(&e);
    return e;
  }
};
ProfState g_prof;
} // namespace

void prof_enable(bool on) {
  std::lock_guard<std::mutex> lock(g_prof.mu);
  g_prof.on = on;
}
bool prof_on() { return g_prof.on; }
void prof_begin(int id, cudaStream_t s) {
  if (!g_prof.on) return;
  std::lock_guard<std::mutex> lock(g_prof.mu);
  ProfState::Rec r{id, g_prof.get(), g_prof.get(), false};
  cudaEventRecord(r.a, s);
  g_prof.pending.push_back(r);
}
void prof_end(int id, cudaStream_t s) {
  if (!g_prof.on) return;
  std::lock_guard<std::mutex> lock(g_prof.mu);
  for (auto it = g_prof.pending.rbegin(); it != g_prof.pending.rend(); ++it)
    if (it->id == id && !it->closed) {
      cudaEventRecord(it->b, s);
      it->closed = true;
      return;
    }
}
void prof_read(double* ms, int64_t* counts, bool reset) {
  std::lock_guard<std::mutex> lock(g_prof.mu);
  for (auto& r : g_prof.pending) {
    if (r.closed) {
      cudaEventSynchronize(r.b);
      float t = 0.f;
      if (cudaEventElapsedTime(&t, r.a, r.b) == cudaSuccess) {
        g_prof.ms[r.id] += t;
        g_prof.counts[r.id] += 1;
      }
    }
    g_prof.pool.push_back(r.a);
    g_prof.pool.push_back(r.b);
  }
  g_prof.pending.clear();
  for (int i = 0; i < kProfCount; ++i) {
    if (ms) ms[i] = g_prof.ms[i];
    if (counts) counts[i] = g_prof.counts[i];
    if (reset) {
      g_prof.ms[i] = 0;
      g_prof.counts[i] = 0;
    }
  }
}

welvet_status to_c(const Status& s) {
  welvet_status out{};
  out.code = s.code;
  std::snprintf(out.message, sizeof(out.message), "%s", s.msg.c_str());
  return out;
}

Status cuda_status(cudaError_t e, const char* what) {
  return Status::err(4, std::string("cuda: ") + what + ": " + cudaGetErrorString(e));
}

namespace {
using PrimaryCtxStateFn = int (*)(int dev, unsigned int* flags, int* active);
PrimaryCtxStateFn primary_ctx_state_fn() {
  static PrimaryCtxStateFn fn = [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q{};
    if (cudaGetDriverEntryPoint("cuDevicePrimaryCtxGetState", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      return reinterpret_cast<PrimaryCtxStateFn>(p);
    return static_cast<PrimaryCtxStateFn>(nullptr);
  }();
  return fn;
}
}  // namespace

DeviceRestore::DeviceRestore() {
  if (cudaGetDevice(&dev_) != cudaSuccess) dev_ = -1;
}

DeviceRestore::~DeviceRestore() {
  if (dev_ < 0) return;
  int now = -1;
  if (cudaGetDevice(&now) != cudaSuccess || now == dev_) return;
  unsigned int flags = 0;
  int active = 0;
  PrimaryCtxStateFn fn = primary_ctx_state_fn();
  if (!fn || fn(dev_, &flags, &active) != 0 || !active) return;
  cudaSetDevice(dev_);
}

// True for host memory the device copies from or to asynchronously (page-locked);
// false for pageable memory, whose device-to-host copies hold the calling thread
// until the copy has run.
bool host_pinned(const void* p) {
  if (!p) return true;
  cudaPointerAttributes a{};
  if (cudaPointerGetAttributes(&a, p) != cudaSuccess) {
    cudaGetLastError();
    return false;
  }
  return a.type == cudaMemoryTypeHost;
}

// ------------------------------------------------------------------ devices
namespace {
std::mutex g_dev_mu;
std::map<int, DeviceCtx*> g_devs;

const char* err_reason(uint32_t code) {
  switch (code) {
  case kErrWaitFull: return "device wait timeout (TMA stage)";
  case kErrWaitEmpty: return "device wait timeout (free stage)";
  case kErrWaitAccFull: return "device wait timeout (accumulator full)";
  case kErrWaitAccEmpty: return "device wait timeout (accumulator empty)";
  case kErrWaitOther: return "device wait timeout";
  case kErrPeerWait: return "peer rank's data did not arrive (peer-memory all-reduce)";
  case 0x100: return "RoPE position outside the table";
  default: return "device error";
  }
}
} // namespace

Status device_ctx(int device, DeviceCtx** out) {
  if (device < 0) WV_CUDA(cudaGetDevice(&device), "cudaGetDevice");
  std::lock_guard<std::mutex> lock(g_dev_mu);
  auto it = g_devs.find(device);
  if (it != g_devs.end()) {
    *out = it->second;
    return cudaSetDevice(device) == cudaSuccess ? Status::ok() : Status::err(4, "cudaSetDevice");
  }
  WV_CUDA(cudaSetDevice(device), "cudaSetDevice");
  cudaDeviceProp prop{};
  WV_CUDA(cudaGetDeviceProperties(&prop, device), "cudaGetDeviceProperties");
  if (prop.major < 10)
    return Status::err(2, std::string("device ") + prop.name + " is not sm_100 (Blackwell)");
  auto* d = new DeviceCtx();
  d->device = device;
  d->sm_count = prop.multiProcessorCount;
  d->cc_major = prop.major;
  d->cc_minor = prop.minor;
  d->name = prop.name;
  WV_CUDA(cudaMalloc(&d->err, 256), "cudaMalloc err");
  WV_CUDA(cudaMemset(d->err, 0, 256), "cudaMemset err");
  WV_CUDA(cudaMalloc(&d->scratch, 4096 * sizeof(float)), "cudaMalloc scratch");
  WV_CUDA(cudaMalloc(&d->scalars, 64 * sizeof(float)), "cudaMalloc scalars");
  WV_CUDA(cudaMalloc(&d->tile_ctr, 256), "cudaMalloc tile counter");
  WV_CUDA(cudaDeviceSynchronize(), "init");
  g_devs[device] = d;
  *out = d;
  return Status::ok();
}

Status check_device_error(DeviceCtx* d) {
  WV_CUDA(cudaSetDevice(d->device), "cudaSetDevice");
  WV_CUDA(cudaDeviceSynchronize(), "synchronize");
  uint32_t code = 0;
  WV_CUDA(cudaMemcpy(&code, d->err, 4, cudaMemcpyDeviceToHost), "read error word");
  uint32_t static_code = 0;
  WV_TRY(take_static_decode_error(&static_code));
  if (!code) code = static_code;
  if (code) {
    cudaMemset(d->err, 0, 4);
    char buf[96];
    std::snprintf(buf, sizeof(buf), "kernel error 0x%x: %s", code, err_reason(code));
    return Status::err(4, buf);
  }
  return Status::ok();
}

// ------------------------------------------------------------------- config
Status resolve_config(const welvet_b200_mha_config& in, Cfg* out) {
  Cfg r;
  r.c = in;
  auto& c = r.c;
  if (c.d_model <= 0 || c.num_heads <= 0)
    return Status::err(1, "mha: need DModel>0 and NumHeads>0");
  if (c.head_dim <= 0) {
    if (c.d_model % c.num_heads != 0)
      return Status::err(1, "mha: HeadDim unset and DModel%NumHeads!=0");
    c.head_dim = c.d_model / c.num_heads;
  }
  if (c.num_kv_heads <= 0) c.num_kv_heads = c.num_heads;
  if (c.num_heads % c.num_kv_heads != 0)
    return Status::err(1, "mha: NumHeads not divisible by NumKVHeads");
  if (c.max_seq_len <= 0) c.max_seq_len = 512;
  if (c.mask == 0) c.mask = 1;
  if (c.rope_theta <= 0) c.rope_theta = 10000;
  if (c.softmax != 0 && c.softmax != 1) return Status::err(1, "mha: unknown Softmax");
  if (c.precision != 0 && c.precision != 1) return Status::err(1, "mha: precision must be 0 or 1");
  if (c.weight_format < 0 || c.weight_format > 3 || (c.precision == 0 && c.weight_format != 0))
    return Status::err(1, "mha: weight_format 1/2/3 need precision 1 (BF16)");
  r.hd = c.head_dim;
  r.nk = c.num_kv_heads;
  r.msl = c.max_seq_len;
  r.group = c.num_heads / c.num_kv_heads;
  r.qd = c.num_heads * r.hd;
  r.kd = r.nk * r.hd;
  // ops_mha.metal:46-48: the override is used unless its float high part is 0.
  r.scale = ((float)c.scale_override != 0.f) ? (float)c.scale_override
                                               : (float)(1.0 / std::sqrt((double)r.hd));
  r.rope = c.pos == 0 || c.pos == 3;
  r.alibi = c.pos == 2 || c.pos == 3;
  if (c.head_count == 0) {
    c.head_begin = 0;
    c.head_count = c.num_heads;
  }
  if (c.head_begin < 0 || c.head_count < 0 || c.head_begin + c.head_count > c.num_heads)
    return Status::err(1, "mha: head shard outside [0, num_heads)");
  if (c.head_count != c.num_heads &&
      (c.head_begin % r.group != 0 || c.head_count % r.group != 0))
    return Status::err(1, "mha: head shard must cover whole KV groups");
  *out = r;
  return Status::ok();
}

// -------------------------------------------------------------------- mount
Mha::~Mha() {
  comm_release(this);
  for (auto& e : io_ev)
    if (e) cudaEventDestroy(e);
  for (auto& e : gather_ev)
    if (e) cudaEventDestroy(e);
  if (io_in) cudaStreamDestroy(io_in);
  if (io_out) cudaStreamDestroy(io_out);
}

namespace {

// Encode -> decode of one full FP32 matrix on the device (FormatNone dtype), in place.
Status roundtrip_inplace(DeviceCtx* d, int dtype, float* w, int64_t n, cudaStream_t s) {
  if (!codec_dtype_supported(dtype)) {
    char buf[128];
    std::snprintf(buf, sizeof(buf), "mha: weight dtype %d is not a FormatNone dtype (0-33)", dtype);
    return Status::err(2, buf);
  }
  if (dtype == 1) return Status::ok();
  const float* stats = nullptr;
  if (codec_needs_stats(dtype)) {
    WV_CUDA(stats_f32(w, n, d->scalars, d->scratch, s), "tensor stats");
    count_launch(2);
    stats = d->scalars;
  }
  WV_CUDA(codec_roundtrip_f32(dtype, w, w, n, stats, s), "codec roundtrip");
  count_launch();
  return Status::ok();
}

} // namespace

Status mha_mount(const welvet_b200_mha_config& cin, int dtype, const float* Q, const float* K,
                 const float* V, const float* O, bool on_device, Mha** out) {
  if (!Q || !K || !V || !O || !out) return Status::err(1, "mha: invalid argument");
  Cfg cfg;
  WV_TRY(resolve_config(cin, &cfg));
  DeviceCtx* d = nullptr;
  WV_TRY(device_ctx(cfg.c.device, &d));
  auto m = std::make_unique<Mha>();
  m->cfg = cfg;
  m->dev = d;
  m->precision = cfg.c.precision;
  m->wfmt = cfg.c.weight_format;
  m->h0 = cfg.c.head_begin;
  m->hc = cfg.c.head_count;
  m->kh0 = m->h0 / cfg.group;
  m->khc = std::max(1, m->hc / cfg.group);
  m->qd_l = m->hc * cfg.hd;
  m->kd_l = m->khc * cfg.hd;
  m->nqkv = m->qd_l + 2 * m->kd_l;
  const int dm = cfg.c.d_model, hd = cfg.hd;
  const int64_t nq = (int64_t)cfg.qd * dm, nkv = (int64_t)cfg.kd * dm, no = (int64_t)dm * cfg.qd;
  cudaStream_t s = 0;

  // Full FP32 matrices on the device.
  DevBuf fq, fk, fv, fo;
  WV_TRY(fq.ensure(nq * 4));
  WV_TRY(fk.ensure(nkv * 4));
  WV_TRY(fv.ensure(nkv * 4));
  WV_TRY(fo.ensure(no * 4));
  const cudaMemcpyKind kind = on_device ? cudaMemcpyDeviceToDevice : cudaMemcpyHostToDevice;
  WV_CUDA(cudaMemcpyAsync(fq.p, Q, nq * 4, kind, s), "upload Q");
  WV_CUDA(cudaMemcpyAsync(fk.p, K, nkv * 4, kind, s), "upload K");
  WV_CUDA(cudaMemcpyAsync(fv.p, V, nkv * 4, kind, s), "upload V");
  WV_CUDA(cudaMemcpyAsync(fo.p, O, no * 4, kind, s), "upload O");

  const size_t qrow0 = (size_t)m->h0 * hd, krow0 = (size_t)m->kh0 * hd;
  if (m->wfmt == 0) {
    // FormatNone dtype round trip of each full matrix (reference WeightStore::make
    // + decode_row_f64, src/weights/store.cpp:7-22, native_codec.cpp:835-870).
    WV_TRY(roundtrip_inplace(d, dtype, fq.as<float>(), nq, s));
    WV_TRY(roundtrip_inplace(d, dtype, fk.as<float>(), nkv, s));
    WV_TRY(roundtrip_inplace(d, dtype, fv.as<float>(), nkv, s));
    WV_TRY(roundtrip_inplace(d, dtype, fo.as<float>(), no, s));
    // Shard slices: W_qkv [nqkv, d] and Wo [d, qd_l].
    DevBuf wqkv32, wo32;
    WV_TRY(wqkv32.ensure((size_t)m->nqkv * dm * 4));
    WV_TRY(wo32.ensure((size_t)dm * m->qd_l * 4));
    float* dst = wqkv32.as<float>();
    WV_CUDA(cudaMemcpyAsync(dst, fq.as<float>() + qrow0 * dm, (size_t)m->qd_l * dm * 4,
                            cudaMemcpyDeviceToDevice, s), "slice Wq");
    WV_CUDA(cudaMemcpyAsync(dst + (size_t)m->qd_l * dm, fk.as<float>() + krow0 * dm,
                            (size_t)m->kd_l * dm * 4, cudaMemcpyDeviceToDevice, s), "slice Wk");
    WV_CUDA(cudaMemcpyAsync(dst + (size_t)(m->qd_l + m->kd_l) * dm, fv.as<float>() + krow0 * dm,
                            (size_t)m->kd_l * dm * 4, cudaMemcpyDeviceToDevice, s), "slice Wv");
    WV_CUDA(cudaMemcpy2DAsync(wo32.p, (size_t)m->qd_l * 4, fo.as<float>() + qrow0,
                              (size_t)cfg.qd * 4, (size_t)m->qd_l * 4, dm,
                              cudaMemcpyDeviceToDevice, s), "slice Wo");
    const int64_t n1 = (int64_t)m->nqkv * dm, n2 = (int64_t)dm * m->qd_l;
    if (m->precision == 0) {
      WV_TRY(m->wqkv.ensure(n1 * 4));
      WV_TRY(m->wqkv_lo.ensure(n1 * 4));
      WV_TRY(m->wo.ensure(n2 * 4));
      WV_TRY(m->wo_lo.ensure(n2 * 4));
      WV_CUDA(split_tf32(wqkv32.as<float>(), m->wqkv.as<float>(), m->wqkv_lo.as<float>(), n1, s), "split");
      WV_CUDA(split_tf32(wo32.as<float>(), m->wo.as<float>(), m->wo_lo.as<float>(), n2, s), "split");
      count_launch(2);
    } else {
      WV_TRY(m->wqkv.ensure(n1 * 2));
      WV_TRY(m->wo.ensure(n2 * 2));
      WV_CUDA(cast_f32_bf16(wqkv32.as<float>(), m->wqkv.p, n1, s), "cast");
      WV_CUDA(cast_f32_bf16(wo32.as<float>(), m->wo.p, n2, s), "cast");
      count_launch(2);
    }
    WV_CUDA(cudaStreamSynchronize(s), "mount");
  } else {
    // Extension formats encode the FP32 inits directly. Scales are computed on the
    // full matrices, then the shard's slice of codes and scales is kept.
    // weight_format 3 keeps the reference's own FormatNone codes of `dtype` (Int8,
    // Int4 or FP4) with the per-tensor scale of each matrix as a per-row scale.
    if (m->wfmt == 3 && dtype != 9 && dtype != 14 && dtype != 16)
      return Status::err(2, "mha: weight_format 3 keeps Int8 (9), Int4 (14) or FP4 (16) codes");
    m->wdtype = dtype;
    const bool fp8 = m->wfmt == 1 || (m->wfmt == 3 && dtype == 9);  // one byte per code
    const bool rowscale = m->wfmt != 2;                               // one scale per row
    if (dm % 64 || cfg.qd % 64 || (m->qd_l % 64))
      return Status::err(2, "mha: FP8/NF4/FormatNone-code weight formats need d_model and head slices % 64 == 0");
    DevBuf cq, ck, cv, co, sq, sk, sv, so;
    auto enc = [&](const DevBuf& w, int rows, int cols, DevBuf& codes, DevBuf& sc) -> Status {
      const int64_t n = (int64_t)rows * cols;
      WV_TRY(codes.ensure(fp8 ? n : n / 2));
      WV_TRY(sc.ensure(rowscale ? (size_t)rows * 4 : (size_t)(n / 64) * 4));
      if (m->wfmt == 3) {
        WV_CUDA(stats_f32(w.as<float>(), n, d->scalars, d->scratch, s), "stats");
        WV_CUDA(formatnone_codes_encode(dtype, w.as<float>(), n, cols, d->scalars, codes.as<uint8_t>(),
                                        sc.as<float>(), s), "formatnone codes");
        count_launch(2);
      } else if (fp8) {
        WV_CUDA(fp8_rowscale_encode(w.as<float>(), rows, cols, codes.as<uint8_t>(), sc.as<float>(), s), "fp8 enc");
        // the dequantising GEMM decodes with the hardware E4M3 conversion
        WV_CUDA(fp8_normalize(codes.as<uint8_t>(), n, s), "fp8 normalize");
        count_launch();
      } else
        WV_CUDA(nf4_block_encode(w.as<float>(), n, codes.as<uint8_t>(), sc.as<float>(), s), "nf4 enc");
      count_launch();
      return Status::ok();
    };
    WV_TRY(enc(fq, cfg.qd, dm, cq, sq));
    WV_TRY(enc(fk, cfg.kd, dm, ck, sk));
    WV_TRY(enc(fv, cfg.kd, dm, cv, sv));
    WV_TRY(enc(fo, dm, cfg.qd, co, so));
    const size_t rb = fp8 ? (size_t)dm : (size_t)dm / 2;   // code bytes per W_qkv row
    const size_t srow = rowscale ? 1 : (size_t)dm / 64;    // scales per W_qkv row
    WV_TRY(m->wqkv.ensure((size_t)m->nqkv * rb));
    WV_TRY(m->wqkv_scale.ensure((size_t)m->nqkv * srow * 4));
    auto cp = [&](void* dstp, const void* srcp, size_t bytes) -> Status {
      WV_CUDA(cudaMemcpyAsync(dstp, srcp, bytes, cudaMemcpyDeviceToDevice, s), "slice codes");
      return Status::ok();
    };
    uint8_t* wc = m->wqkv.as<uint8_t>();
    float* wsc = m->wqkv_scale.as<float>();
    WV_TRY(cp(wc, cq.as<uint8_t>() + qrow0 * rb, (size_t)m->qd_l * rb));
    WV_TRY(cp(wc + (size_t)m->qd_l * rb, ck.as<uint8_t>() + krow0 * rb, (size_t)m->kd_l * rb));
    WV_TRY(cp(wc + (size_t)(m->qd_l + m->kd_l) * rb, cv.as<uint8_t>() + krow0 * rb, (size_t)m->kd_l * rb));
    WV_TRY(cp(wsc, sq.as<float>() + qrow0 * srow, (size_t)m->qd_l * srow * 4));
    WV_TRY(cp(wsc + (size_t)m->qd_l * srow, sk.as<float>() + krow0 * srow, (size_t)m->kd_l * srow * 4));
    WV_TRY(cp(wsc + (size_t)(m->qd_l + m->kd_l) * srow, sv.as<float>() + krow0 * srow,
              (size_t)m->kd_l * srow * 4));
    // Wo [d, qd]: keep columns [qrow0, qrow0 + qd_l) of every row.
    const size_t ob = fp8 ? (size_t)cfg.qd : (size_t)cfg.qd / 2, ob_l = fp8 ? (size_t)m->qd_l : (size_t)m->qd_l / 2;
    const size_t oc0 = fp8 ? qrow0 : qrow0 / 2;
    WV_TRY(m->wo.ensure((size_t)dm * ob_l));
    WV_CUDA(cudaMemcpy2DAsync(m->wo.p, ob_l, co.as<uint8_t>() + oc0, ob, ob_l, dm,
                              cudaMemcpyDeviceToDevice, s), "slice Wo codes");
    if (rowscale) {
      WV_TRY(m->wo_scale.ensure((size_t)dm * 4));
      WV_TRY(cp(m->wo_scale.p, so.p, (size_t)dm * 4));
    } else {
      const size_t sb = (size_t)cfg.qd / 64, sb_l = (size_t)m->qd_l / 64;
      WV_TRY(m->wo_scale.ensure((size_t)dm * sb_l * 4));
      WV_CUDA(cudaMemcpy2DAsync(m->wo_scale.p, sb_l * 4, so.as<float>() + qrow0 / 64, sb * 4, sb_l * 4, dm,
                                cudaMemcpyDeviceToDevice, s), "slice Wo absmax");
    }
    WV_CUDA(cudaStreamSynchronize(s), "mount");
  }
  WV_TRY(check_device_error(d));
  *out = m.release();
  return Status::ok();
}

// ------------------------------------------------------------------ forward
namespace {

// Copy streams and events of the chunked host-buffer forward (created on first use).
Status ensure_io_streams(Mha* m) {
  if (m->io_in) return Status::ok();
  WV_CUDA(cudaStreamCreateWithFlags(&m->io_in, cudaStreamNonBlocking), "io stream");
  WV_CUDA(cudaStreamCreateWithFlags(&m->io_out, cudaStreamNonBlocking), "io stream");
  for (auto& e : m->io_ev) WV_CUDA(cudaEventCreateWithFlags(&e, cudaEventDisableTiming), "io event");
  for (auto& e : m->gather_ev) WV_CUDA(cudaEventCreateWithFlags(&e, cudaEventDisableTiming), "io event");
  for (auto& e : m->chunk_done)  // shared with the communicator path
    if (!e) WV_CUDA(cudaEventCreateWithFlags(&e, cudaEventDisableTiming), "chunk event");
  return Status::ok();
}

Status ensure_rope(Mha* m, int max_pos, cudaStream_t s) {
  if (!m->cfg.rope || m->cfg.hd < 2) return Status::ok();
  if (max_pos <= m->rope_max_pos) return Status::ok();
  const int want = std::max(max_pos, std::max(m->rope_max_pos * 2, 1024));
  // The table may be in use by work queued on another stream of this layer.
  WV_CUDA(cudaDeviceSynchronize(), "rope table sync");
  WV_TRY(m->rope_tab.ensure((size_t)want * (m->cfg.hd / 2) * sizeof(float2)));
  WV_CUDA(rope_table(m->rope_tab.as<float2>(), want, m->cfg.hd, m->cfg.c.rope_theta, s), "rope table");
  count_launch();
  m->rope_max_pos = want;
  return Status::ok();
}

// One projection: out[M, N] = A[M, K] * W[N, K]^T with the layer's format.
// RoPE (rope_cols > 0) and the KV scatter (kv) are fused where the tensor-core
// path allows, applied by separate kernels otherwise.
struct Proj {
  const void* a = nullptr;
  const void* a_lo = nullptr;
  int M = 0, K = 0, lda = 0;
  const void* w = nullptr;
  const void* w_lo = nullptr;
  const float* w_scale = nullptr;
  int N = 0;
  void* out = nullptr;
  int ldo = 0;
  float* out_hi = nullptr;
  float* out_lo = nullptr;
  int rope_cols = 0;
  const int* positions = nullptr;
  int pos_mod = 0;
  bool splitk = false;  // few rows (decode): split K over the SMs through m->splitk_ws
  bool split_only = false;  // with out_hi: out is not needed (written only if RoPE is unfused)
  // Decode: the K and V column ranges [kv_col0, kv_col0 + 2 kv_dim) may go straight
  // to the KV page pools (row b to slot kv_slot[b]) when the kernel can scatter them.
  void* kv_k = nullptr;
  void* kv_v = nullptr;
  const int* kv_slot = nullptr;
  int kv_col0 = 0, kv_dim = 0;
};

// Chunks of a device-buffer forward with a communicator: 4, or WELVET_B200_FORWARD_CHUNKS
// (1-16): more chunks leave less of the last chunk's collective exposed at the end,
// at a few launches per chunk.
int device_chunks() {
  static const int n = [] {
    const char* v = std::getenv("WELVET_B200_FORWARD_CHUNKS");
    const int c = v ? std::atoi(v) : 0;
    return c >= 1 && c <= Mha::kMaxChunks ? c : 4;
  }();
  return n;
}

// Few-row BF16 projections (decode) run as a GEMV streaming the weights at HBM rate
// unless WELVET_B200_DECODE_GEMV=0 selects the split-K tensor-core GEMM.
bool decode_gemv_enabled() {
  static const bool on = [] {
    const char* v = std::getenv("WELVET_B200_DECODE_GEMV");
    return !(v && v[0] == '0');
  }();
  return on;
}

// *kv_done (optional) tells whether the K/V columns went to the page pools.
Status run_proj(Mha* m, const Proj& pj, cudaStream_t s, bool* kv_done = nullptr) {
  if (kv_done) *kv_done = false;
  const bool f32 = m->precision == 0;
  GemmArgs g;
  g.kind = f32 ? kGemmTF32x3
              : m->wfmt == 1 ? kGemmFP8
              : m->wfmt == 2 ? kGemmNF4
              : m->wfmt == 3 ? (m->wdtype == 9 ? kGemmI8 : m->wdtype == 14 ? kGemmI4 : kGemmFP4)
                             : kGemmBF16;
  g.M = pj.M;
  g.N = pj.N;
  g.K = pj.K;
  g.a = pj.a;
  g.a_lo = pj.a_lo;
  g.lda = pj.lda;
  g.b = pj.w;
  g.b_lo = pj.w_lo;
  g.ldb = pj.K;
  g.b_scale = pj.w_scale;
  g.out = pj.out;
  g.ldo = pj.ldo;
  g.out_bf16 = f32 ? 0 : 1;
  g.out_hi = pj.out_hi;
  g.out_lo = pj.out_lo;
  g.err = m->dev->err;
  g.split_only = pj.split_only ? 1 : 0;
  g.sm_count = m->dev->sm_count;
  const bool rope = pj.rope_cols > 0 && m->cfg.rope;
  if (rope) {
    g.rope_tab = m->rope_tab.as<float2>();
    g.rope_cols = pj.rope_cols;
    g.head_dim = m->cfg.hd;
    g.rope_max_pos = m->rope_max_pos;
    g.positions = pj.positions;
    g.pos_mod = pj.pos_mod;
  }
  const int hd = m->cfg.hd;
  if (pj.splitk && !f32 && decode_gemv_enabled()) {
    GemmArgs v = g;
    v.head_dim = hd;
    v.kv_k = pj.kv_k;
    v.kv_v = pj.kv_v;
    v.kv_slot = pj.kv_slot;
    v.kv_col0 = pj.kv_col0;
    v.kv_dim = pj.kv_dim;
    if (gemv_decode_supported(v)) {
      WV_CUDA(gemv_decode(v, s), "gemv_decode");
      count_launch();
      if (kv_done) *kv_done = pj.kv_k != nullptr;
      return Status::ok();
    }
  }
  const int bn = f32 ? 128 : 256;
  const bool fused_rope = rope && (hd == 64 || hd == 128 || hd == 256) && bn % hd == 0;
  if (rope && !fused_rope) g.split_only = 0;  // rope_apply rotates out, then re-splits it
  if (gemm_tc_supported(g)) {
    if (pj.splitk) {
      const size_t floats = gemm_tc_splitk_floats(g);
      if (floats) {
        WV_TRY(m->splitk_ws.ensure(floats * sizeof(float)));
        g.splitk_ws = m->splitk_ws.as<float>();
        g.splitk_ws_floats = floats;
      }
    }
    WV_CUDA(gemm_tc(g, s), "gemm_tc");
    count_launch(gemm_tc_launches(g));
  } else {
    if (g.kind == kGemmFP8 || g.kind == kGemmNF4)
      return Status::err(2, "mha: quantised weight GEMM needs TMA-aligned shapes");
    WV_CUDA(gemm_simt(g, s), "gemm_simt");
    count_launch();
  }
  if (rope && !(fused_rope && gemm_tc_supported(g))) {
    WV_CUDA(rope_apply(pj.out, f32 ? 0 : 1, pj.M, pj.ldo, pj.rope_cols, hd, m->rope_tab.as<float2>(),
                       m->rope_max_pos, pj.positions, pj.pos_mod, s), "rope");
    count_launch();
    if (pj.out_hi) {  // keep the TF32 split in step with the rotated values
      WV_CUDA(split_tf32(static_cast<const float*>(pj.out), pj.out_hi, pj.out_lo, (int64_t)pj.M * pj.ldo, s),
              "split");
      count_launch();
    }
  }
  return Status::ok();
}

AttnArgs attn_args(Mha* m, int batch, int seq, bool stream_mode) {
  AttnArgs a;
  const auto& c = m->cfg;
  a.batch = batch;
  a.seq = seq;
  a.num_heads = m->hc;
  a.num_kv_heads = m->khc;
  a.head_dim = c.hd;
  a.stream_mode = stream_mode ? 1 : 0;
  a.mask = c.c.mask;
  a.window = c.c.window;
  a.max_seq_len = c.msl;
  a.prefix_len = c.c.prefix_len;
  a.window_causal = c.c.window_causal;
  a.alibi = c.alibi;
  a.sigmoid = c.c.softmax == 1;
  a.head_base = m->h0;
  a.total_heads = c.c.num_heads;
  a.scale = c.scale;
  a.is_bf16 = m->precision == 1;
  a.err = m->dev->err;
  a.sm_count = m->dev->sm_count;
  a.tile_ctr = m->attn_ctr.as<int>();  // null until mha_forward sized it
  return a;
}

Status run_attention(Mha* m, AttnArgs a, cudaStream_t s) {
  (void)m;
  cudaError_t e = cudaErrorNotSupported;
  if (attn_tf32_supported(a)) e = attn_prefill_tf32(a, s);
  else if (attn_tc_supported(a)) e = attn_prefill_tc(a, s);
  if (e == cudaErrorNotSupported) {  // shape/mode outside the tensor-core kernel, or its
    cudaGetLastError();               // register split does not fit this build
    e = attn_prefill_simt(a, s);
  }
  WV_CUDA(e, "attention prefill");
  count_launch();
  return Status::ok();
}

} // namespace

// New weights for a mounted FP32 layer that holds every head in the FormatNone
// layout (precision 0, weight format 0): already decoded device matrices W_qkv
// [q_dim + 2 kv_dim, d_model] (rows Q | K | V) and Wo [d_model, q_dim] are split
// into the layer's TF32 pairs in place; nothing is allocated.
Status mha_reload_fp32(Mha* m, const float* wqkv, const float* wo, cudaStream_t s) {
  if (!m || !wqkv || !wo) return Status::err(1, "mha: invalid argument");
  if (m->precision != 0 || m->wfmt != 0 || m->qd_l != m->cfg.qd || m->kd_l != m->cfg.kd)
    return Status::err(2, "mha: weight reload needs an FP32 layer holding every head");
  std::lock_guard<std::mutex> lock(m->mu);
  const int64_t dm = m->cfg.c.d_model;
  WV_CUDA(split_tf32(wqkv, m->wqkv.as<float>(), m->wqkv_lo.as<float>(), (int64_t)m->nqkv * dm, s), "split");
  WV_CUDA(split_tf32(wo, m->wo.as<float>(), m->wo_lo.as<float>(), dm * m->qd_l, s), "split");
  count_launch(2);
  return Status::ok();
}

Status mha_forward(Mha* m, int batch, int seq, const void* x, void* pre, void* post, bool on_device,
                   cudaStream_t s, Kv* kv, bool rows) {
  if (!m || !x || !post || batch <= 0 || seq <= 0) return Status::err(1, "mha: invalid argument");
  std::lock_guard<std::mutex> lock(m->mu);
  const auto& c = m->cfg;
  const bool stream_mode = c.c.seq_mode == 0;
  // Row-sharded host I/O: rank r's sequences are [r * batch / N, (r + 1) * batch / N).
  const bool rows_io = rows && m->comm && m->nranks > 1;
  if (rows_io) {
    if (on_device || stream_mode || kv || pre)
      return Status::err(2, "mha: row-sharded I/O needs host buffers, per-sequence mode and no pre");
    if (batch % m->nranks) return Status::err(1, "mha: batch not divisible by the ranks");
  }
  if (stream_mode && seq > c.msl) return Status::err(1, "mha: seq > MaxSeqLen");  // mha.cpp:159-161
  WV_CUDA(cudaSetDevice(m->dev->device), "cudaSetDevice");
  const int64_t M = (int64_t)batch * seq;
  // Rows are 32-bit TMA coordinates; element offsets are 64-bit everywhere.
  if (M >= (int64_t{1} << 30)) return Status::err(1, "mha: batch*seq too large");
  const int dm = c.c.d_model;
  const bool f32 = m->precision == 0;
  const size_t es = f32 ? 4 : 2;

  // Host buffers: stage through device copies inside the call.
  const void* xd = x;
  void* pred = pre;
  void* postd = post;
  // With a communicator attached, or with host buffers, and independent sequences
  // (per-sequence mode, no KV prefill) the batch runs in chunks: the all-reduce of
  // chunk i (comm_stream) and its device->host copy (io_out) overlap the next
  // chunk's projections and attention (stream s), whose input copy (io_in) ran
  // during the previous chunk.
  const bool chunked = (m->comm || !on_device) && !stream_mode && !kv && batch > 1;
  // Pageable host outputs with a communicator: a device-to-host copy queued behind a
  // collective would hold this thread until the collective ends, i.e. forever if a
  // peer rank stopped. Their copies wait until the bounded wait (comm_wait) has seen
  // the collectives finish.
  const bool defer_d2h = !on_device && m->comm && m->nranks > 1 && (!host_pinned(post) || !host_pinned(pre));
  // Host copies (about 40 ms per 2 GB each way on PCIe) want more, smaller chunks
  // than the all-reduce does.
  int chunks = chunked ? std::min(batch, on_device ? device_chunks() : Mha::kMaxChunks) : 1;
  // rows_io: chunk i takes bcl sequences of every rank (rank-major), bcl of this rank
  const int nr = rows_io ? m->nranks : 1, b_local = batch / nr;
  const int bcl = rows_io ? (b_local + std::min(b_local, Mha::kMaxChunks) - 1) / std::min(b_local, Mha::kMaxChunks)
                          : 0;
  if (rows_io) chunks = (b_local + bcl - 1) / bcl;
  if (!on_device) {
    WV_TRY(m->x_io.ensure(M * dm * es));
    WV_TRY(m->post_io.ensure(M * dm * es));
    if (!chunked) WV_CUDA(cudaMemcpyAsync(m->x_io.p, x, M * dm * es, cudaMemcpyHostToDevice, s), "H2D x");
    else WV_TRY(ensure_io_streams(m));
    xd = m->x_io.p;
    postd = m->post_io.p;
    pred = nullptr;
    if (pre) {  // attention output of every chunk lands here, copied back below
      WV_TRY(m->pre_io.ensure(M * m->qd_l * es));
      pred = m->pre_io.p;
    }
  }
  const int bc_max = rows_io ? bcl * nr : (batch + chunks - 1) / chunks;
  const int64_t Mc_max = (int64_t)bc_max * seq;
  WV_TRY(m->qkv.ensure(Mc_max * m->nqkv * es));
  if (!pred) WV_TRY(m->attn.ensure(Mc_max * m->qd_l * es));
  if (f32) {
    WV_TRY(m->x_hi.ensure(Mc_max * dm * 4));
    WV_TRY(m->x_lo.ensure(Mc_max * dm * 4));
    WV_TRY(m->attn_hi.ensure(Mc_max * m->qd_l * 4));
    WV_TRY(m->attn_lo.ensure(Mc_max * m->qd_l * 4));
  }
  // FP32 attention on the tensor cores (3xTF32) reads the TF32 split of Q, K and
  // V, written by the QKV projection's epilogue.
  bool tf32_attn = false;
  if (f32) {
    AttnArgs t = attn_args(m, bc_max, seq, stream_mode);
    t.q = t.k = t.v = t.q_lo = t.k_lo = t.v_lo = m->qkv.p;  // alignment stand-ins
    t.ldq = t.ldk = m->nqkv;
    t.out = pred ? pred : m->attn.p;
    t.ldo = m->qd_l;
    t.out_hi = m->attn_hi.as<float>();
    t.out_lo = m->attn_lo.as<float>();
    tf32_attn = attn_tf32_supported(t);
    if (tf32_attn) {
      WV_TRY(m->qkv_hi.ensure(Mc_max * m->nqkv * 4));
      WV_TRY(m->qkv_lo.ensure(Mc_max * m->nqkv * 4));
    }
  }
  if (!f32) WV_TRY(m->attn_ctr.ensure(256));  // the persistent attention's tile counter
  // RoPE positions: stream mode -> row index (global position), else row % seq.
  const int max_pos = stream_mode ? (int)M : seq;
  WV_TRY(ensure_rope(m, max_pos, s));

  // QKV projection, attention and O projection of sequences [b0, b0 + bc); with
  // with_o false the attention output goes to attn_at and the O projection is left
  // to the caller (the attention-output exchange).
  auto run_rows = [&](int b0, int bc, void* attn_at = nullptr, bool with_o = true) -> Status {
    const int64_t r0 = (int64_t)b0 * seq, Mc = (int64_t)bc * seq;
    const void* xc = static_cast<const char*>(xd) + r0 * dm * es;
    void* attn = attn_at ? attn_at
                 : pred  ? static_cast<void*>(static_cast<char*>(pred) + r0 * m->qd_l * es)
                         : m->attn.p;
    Proj q;
    q.M = (int)Mc;
    q.K = dm;
    q.lda = dm;
    q.N = m->nqkv;
    q.out = m->qkv.p;
    q.ldo = m->nqkv;
    q.rope_cols = m->qd_l + m->kd_l;
    q.pos_mod = stream_mode ? 0 : seq;
    q.w = m->wqkv.p;
    q.w_lo = m->wqkv_lo.p;
    q.w_scale = m->wqkv_scale.as<float>();
    if (tf32_attn) {
      q.out_hi = m->qkv_hi.as<float>();
      q.out_lo = m->qkv_lo.as<float>();
      q.split_only = kv == nullptr;  // the KV cache takes the FP32 rows
    }
    if (f32) {
      WV_CUDA(split_tf32(static_cast<const float*>(xc), m->x_hi.as<float>(), m->x_lo.as<float>(), Mc * dm, s),
              "split x");
      count_launch();
      q.a = m->x_hi.p;
      q.a_lo = m->x_lo.p;
    } else {
      q.a = xc;
    }
    prof_begin(kProfGemmQkv, s);
    WV_TRY(run_proj(m, q, s));
    prof_end(kProfGemmQkv, s);

    if (kv) {  // prefill: K/V rows into the cache pages of each sequence (single chunk)
      WV_TRY(m->slots.ensure(M * 4));
      WV_CUDA(make_prefill_slots(m->slots.as<int>(), batch, seq, kv->pages_per_seq, s), "slots");
      const char* base = static_cast<const char*>(m->qkv.p);
      WV_CUDA(kv_append(base + (size_t)m->qd_l * es, base + (size_t)(m->qd_l + m->kd_l) * es, m->nqkv, (int)M,
                        m->kd_l, c.hd, f32 ? 0 : 1, m->slots.as<int>(), kv->k_pool.p, kv->v_pool.p, s),
              "kv append");
      WV_CUDA(set_ctx(kv->ctx_len.as<int>(), batch, seq, s), "ctx");
      count_launch(3);
      for (int b = 0; b < batch; ++b) kv->ctx_host[b] = seq;
    }

    AttnArgs a = attn_args(m, bc, seq, stream_mode);
    const char* base = static_cast<const char*>(m->qkv.p);
    a.q = base;
    a.k = base + (size_t)m->qd_l * es;
    a.v = base + (size_t)(m->qd_l + m->kd_l) * es;
    a.ldq = a.ldk = m->nqkv;
    a.out = attn;
    a.ldo = m->qd_l;
    if (f32) {
      a.out_hi = m->attn_hi.as<float>();
      a.out_lo = m->attn_lo.as<float>();
    }
    if (tf32_attn) {  // (every chunk qualifies when the largest one does)
      const char* hb = static_cast<const char*>(m->qkv_hi.p);
      const char* lb = static_cast<const char*>(m->qkv_lo.p);
      a.q = hb;
      a.k = hb + (size_t)m->qd_l * es;
      a.v = hb + (size_t)(m->qd_l + m->kd_l) * es;
      a.q_lo = lb;
      a.k_lo = lb + (size_t)m->qd_l * es;
      a.v_lo = lb + (size_t)(m->qd_l + m->kd_l) * es;
      if (!attn_tf32_supported(a)) return Status::err(4, "mha: 3xTF32 attention refused a chunk");
    }
    prof_begin(kProfAttnPrefill, s);
    WV_TRY(run_attention(m, a, s));
    prof_end(kProfAttnPrefill, s);
    if (!with_o) return Status::ok();

    Proj o;
    o.M = (int)Mc;
    o.K = m->qd_l;
    o.lda = m->qd_l;
    o.N = dm;
    o.out = static_cast<char*>(postd) + r0 * dm * es;
    o.ldo = dm;
    o.w = m->wo.p;
    o.w_lo = m->wo_lo.p;
    o.w_scale = m->wo_scale.as<float>();
    if (f32) {
      o.a = m->attn_hi.p;
      o.a_lo = m->attn_lo.p;
    } else {
      o.a = attn;
    }
    prof_begin(kProfGemmO, s);
    WV_TRY(run_proj(m, o, s));
    prof_end(kProfGemmO, s);
    return Status::ok();
  };

  // Reduce-scatter output (device buffers): chunk rows split evenly over the ranks,
  // rank r keeps the r-th slice of each chunk summed; other rows hold its partial
  // (mode 1), or are not written (mode 2, the attention-output exchange).
  const bool rs_out = m->comm && m->nranks > 1 && m->out_mode >= 1 && on_device && !rows_io;
  if (rs_out && ((int64_t)bc_max * seq % m->nranks || M % m->nranks ||
                 (int64_t)(batch - (int64_t)(chunks - 1) * bc_max) * seq % m->nranks))
    return Status::err(1, "mha: reduce-scatter output needs every chunk's rows divisible by the ranks");
  // Reduce-scatter through copy engines and peer memory when the layer can take it
  // (chunked calls), else NCCL's.
  const bool peer_rs = rs_out && chunks > 1 && comm_peer_rs_ok(m) &&
                       ((int64_t)bc_max * seq / m->nranks) * dm * (int64_t)es % 16 == 0;
  // Attention-output exchange (mode 2): the chunk's attention rows go to their
  // owners, which run the output projection over every head (K = q_dim) for their
  // own rows only; without it the layer takes mode 1.
  const bool xa = rs_out && m->out_mode == 2 && chunks > 1 && comm_xa_ok(m) && !pre;
  auto reduce_out = [&](char* base, int64_t rows, cudaStream_t st) -> Status {
    if (rs_out) return comm_reducescatter(m, base, (size_t)(rows / m->nranks) * dm, !f32, st);
    return comm_allreduce(m, base, (size_t)rows * dm, !f32, st);
  };
  // Row-sharded host I/O takes the exchange too: chunk i's row slice p is rank p's
  // own sequences, so each rank projects and copies down exactly its rows.
  const bool xa_rows = rows_io && comm_xa_ok(m);
  // Exchange state: chunk i's receive slot (A operand of its output projection) and
  // the rows of post that projection writes.
  const void* a_slot[Mha::kMaxChunks] = {};
  int64_t o_row0[Mha::kMaxChunks] = {}, o_rows[Mha::kMaxChunks] = {};
  auto o_proj = [&](int i) -> Status {
    WV_TRY(comm_xa_wait(m, i, s));
    Proj o;
    o.M = (int)o_rows[i];
    o.K = m->cfg.qd;
    o.lda = m->cfg.qd;
    o.N = dm;
    o.out = static_cast<char*>(postd) + o_row0[i] * dm * es;
    o.ldo = dm;
    o.w = m->wo_full.p;
    o.a = a_slot[i];
    prof_begin(kProfGemmO, s);
    WV_TRY(run_proj(m, o, s));
    prof_end(kProfGemmO, s);
    return Status::ok();
  };
  if (xa || xa_rows) WV_TRY(m->attn.ensure((size_t)M * m->qd_l * es));
  if (xa) {
    // Per chunk: QKV projection and attention into attn (every chunk's rows kept
    // until its copies have read them), the exchange's copies, then the previous
    // chunk's output projection once its blocks have landed; so chunk i's transfers
    // overlap chunk i + 1's projections and attention.
    int n_done = 0;
    for (int i = 0, b0 = 0; i < chunks && b0 < batch; ++i, b0 += bc_max, ++n_done) {
      const int bc = std::min(bc_max, batch - b0);
      const int64_t r0 = (int64_t)b0 * seq, rows = (int64_t)bc * seq;
      char* attn_i = m->attn.as<char>() + r0 * m->qd_l * es;
      WV_TRY(run_rows(b0, bc, attn_i, false));
      WV_CUDA(cudaEventRecord(m->chunk_done[i], s), "event");
      prof_begin(kProfAllReduce, s);
      WV_TRY(comm_xa_chunk(m, attn_i, rows, Mc_max, i, chunks, m->chunk_done[i], s, &a_slot[i]));
      prof_end(kProfAllReduce, s);
      o_rows[i] = rows / m->nranks;
      o_row0[i] = r0 + m->rank * o_rows[i];
      if (i > 0) WV_TRY(o_proj(i - 1));
    }
    WV_TRY(o_proj(n_done - 1));
    WV_TRY(comm_xa_finish(m, s));  // the copies have read every chunk's rows
  } else if (chunks == 1 && !rows_io) {
    WV_TRY(run_rows(0, batch));
    if (m->comm) {
      prof_begin(kProfAllReduce, s);
      WV_TRY(reduce_out(static_cast<char*>(postd), M, s));
      prof_end(kProfAllReduce, s);
    }
  } else {
    // The helper streams first wait for what s did before this call (the previous
    // forward's readers of the staging buffers and of post).
    const bool host = !on_device;
    WV_CUDA(cudaEventRecord(m->chunk_done[0], s), "event");
    if (m->comm) WV_CUDA(cudaStreamWaitEvent(m->comm_stream, m->chunk_done[0], 0), "wait");
    if (host) {
      WV_CUDA(cudaStreamWaitEvent(m->io_in, m->chunk_done[0], 0), "wait");
      WV_CUDA(cudaStreamWaitEvent(m->io_out, m->chunk_done[0], 0), "wait");
    }
    // rows_io: this rank's rows of chunk i go up and are all-gathered (comm_stream)
    // one chunk ahead of the compute, so that the gather of chunk i + 1 runs
    // during chunk i and precedes chunk i's reduce-scatter on comm_stream.
    auto gather_chunk = [&](int i) -> Status {
      const int b0 = i * bc_max, bc = std::min(bc_max, batch - b0);
      const int64_t r0 = (int64_t)b0 * seq, own = (int64_t)(bc / nr) * seq;
      WV_CUDA(cudaMemcpyAsync(static_cast<char*>(m->x_io.p) + (r0 + m->rank * own) * dm * es,
                              static_cast<const char*>(x) + (int64_t)i * bcl * seq * dm * es, own * dm * es,
                              cudaMemcpyHostToDevice, m->io_in), "H2D x rows");
      WV_CUDA(cudaEventRecord(m->io_ev[i], m->io_in), "event");
      WV_CUDA(cudaStreamWaitEvent(m->comm_stream, m->io_ev[i], 0), "wait");
      WV_TRY(comm_allgather(m, static_cast<char*>(m->x_io.p) + r0 * dm * es, (size_t)own * dm, !f32,
                            m->comm_stream));
      WV_CUDA(cudaEventRecord(m->gather_ev[i], m->comm_stream), "event");
      return Status::ok();
    };
    // xa_rows: this rank's rows of chunk i (projected on s) go down on io_out
    auto rows_down = [&](int i) -> Status {
      if (defer_d2h) return Status::ok();
      WV_CUDA(cudaEventRecord(m->io_ev[Mha::kMaxChunks + i], s), "event");
      WV_CUDA(cudaStreamWaitEvent(m->io_out, m->io_ev[Mha::kMaxChunks + i], 0), "wait");
      WV_CUDA(cudaMemcpyAsync(static_cast<char*>(post) + (int64_t)i * bcl * seq * dm * es,
                              static_cast<char*>(postd) + o_row0[i] * dm * es, o_rows[i] * dm * es,
                              cudaMemcpyDeviceToHost, m->io_out), "D2H post rows");
      return Status::ok();
    };
    int xa_done = 0;
    if (rows_io) WV_TRY(gather_chunk(0));
    for (int i = 0, b0 = 0; i < chunks && b0 < batch; ++i, b0 += bc_max) {
      const int bc = std::min(bc_max, batch - b0);
      const int64_t r0 = (int64_t)b0 * seq, rows = (int64_t)bc * seq;
      if (rows_io && xa_rows) {
        // attention rows out to their owners, then the previous chunk's output
        // projection over every head and its rows down to the host
        const int64_t own = rows / nr;
        WV_CUDA(cudaStreamWaitEvent(s, m->gather_ev[i], 0), "wait");
        char* attn_i = m->attn.as<char>() + r0 * m->qd_l * es;
        WV_TRY(run_rows(b0, bc, attn_i, false));
        WV_CUDA(cudaEventRecord(m->chunk_done[i], s), "event");
        if (i + 1 < chunks) WV_TRY(gather_chunk(i + 1));
        prof_begin(kProfAllReduce, s);
        WV_TRY(comm_xa_chunk(m, attn_i, rows, Mc_max, i, chunks, m->chunk_done[i], s, &a_slot[i]));
        prof_end(kProfAllReduce, s);
        o_rows[i] = own;
        o_row0[i] = r0 + m->rank * own;
        if (i > 0) {
          WV_TRY(o_proj(i - 1));
          WV_TRY(rows_down(i - 1));
        }
        ++xa_done;
        continue;
      }
      if (rows_io) {
        const int64_t own = rows / nr;
        WV_CUDA(cudaStreamWaitEvent(s, m->gather_ev[i], 0), "wait");
        WV_TRY(run_rows(b0, bc));
        WV_CUDA(cudaEventRecord(m->chunk_done[i], s), "event");
        if (i + 1 < chunks) WV_TRY(gather_chunk(i + 1));
        WV_CUDA(cudaStreamWaitEvent(m->comm_stream, m->chunk_done[i], 0), "wait");
        prof_begin(kProfAllReduce, m->comm_stream);
        WV_TRY(comm_reducescatter(m, static_cast<char*>(postd) + r0 * dm * es, (size_t)own * dm, !f32,
                                  m->comm_stream));
        prof_end(kProfAllReduce, m->comm_stream);
        if (!defer_d2h) {
          WV_CUDA(cudaEventRecord(m->io_ev[Mha::kMaxChunks + i], m->comm_stream), "event");
          WV_CUDA(cudaStreamWaitEvent(m->io_out, m->io_ev[Mha::kMaxChunks + i], 0), "wait");
          WV_CUDA(cudaMemcpyAsync(static_cast<char*>(post) + (int64_t)i * bcl * seq * dm * es,
                                  static_cast<char*>(postd) + (r0 + m->rank * own) * dm * es, own * dm * es,
                                  cudaMemcpyDeviceToHost, m->io_out), "D2H post rows");
        }
        continue;
      }
      if (host) {
        WV_CUDA(cudaMemcpyAsync(static_cast<char*>(m->x_io.p) + r0 * dm * es, static_cast<const char*>(x) + r0 * dm * es,
                                rows * dm * es, cudaMemcpyHostToDevice, m->io_in), "H2D x");
        WV_CUDA(cudaEventRecord(m->io_ev[i], m->io_in), "event");
        WV_CUDA(cudaStreamWaitEvent(s, m->io_ev[i], 0), "wait");
      }
      WV_TRY(run_rows(b0, bc));
      WV_CUDA(cudaEventRecord(m->chunk_done[i], s), "event");
      cudaEvent_t out_ready = m->chunk_done[i];
      if (m->comm) {
        WV_CUDA(cudaStreamWaitEvent(m->comm_stream, m->chunk_done[i], 0), "wait");
        prof_begin(kProfAllReduce, m->comm_stream);
        if (peer_rs) {
          WV_TRY(comm_peer_rs_chunk(m, static_cast<char*>(postd) + r0 * dm * es, rows, (int64_t)bc_max * seq, dm,
                                    !f32, i, chunks, m->chunk_done[i], m->comm_stream));
        } else {
          WV_TRY(reduce_out(static_cast<char*>(postd) + r0 * dm * es, rows, m->comm_stream));
        }
        prof_end(kProfAllReduce, m->comm_stream);
        if (host) {
          WV_CUDA(cudaEventRecord(m->io_ev[Mha::kMaxChunks + i], m->comm_stream), "event");
          out_ready = m->io_ev[Mha::kMaxChunks + i];
        }
      }
      if (host && !defer_d2h) {
        WV_CUDA(cudaStreamWaitEvent(m->io_out, out_ready, 0), "wait");
        WV_CUDA(cudaMemcpyAsync(static_cast<char*>(post) + r0 * dm * es, static_cast<char*>(postd) + r0 * dm * es,
                                rows * dm * es, cudaMemcpyDeviceToHost, m->io_out), "D2H post");
        if (pre)
          WV_CUDA(cudaMemcpyAsync(static_cast<char*>(pre) + r0 * m->qd_l * es,
                                  static_cast<char*>(pred) + r0 * m->qd_l * es, rows * m->qd_l * es,
                                  cudaMemcpyDeviceToHost, m->io_out), "D2H pre");
      }
    }
    if (xa_done > 0) {
      WV_TRY(o_proj(xa_done - 1));
      WV_TRY(rows_down(xa_done - 1));
      WV_TRY(comm_xa_finish(m, s));  // the copies have read every chunk's rows
    }
    if (m->comm) {
      WV_CUDA(cudaEventRecord(m->comm_done, m->comm_stream), "event");
      WV_CUDA(cudaStreamWaitEvent(s, m->comm_done, 0), "wait");
    }
    if (peer_rs) WV_TRY(comm_peer_rs_finish(m, s));  // the copies have read every chunk's rows
    if (host) {
      WV_CUDA(cudaEventRecord(m->io_ev[2 * Mha::kMaxChunks], m->io_out), "event");
      WV_CUDA(cudaStreamWaitEvent(s, m->io_ev[2 * Mha::kMaxChunks], 0), "wait");
    }
  }

  if (!on_device) {
    if (defer_d2h) {
      WV_TRY(comm_wait(m, s, "forward"));  // every collective finished (or code 4)
      if (rows_io) {
        for (int i = 0, b0 = 0; i < chunks && b0 < batch; ++i, b0 += bc_max) {
          const int64_t r0 = (int64_t)b0 * seq, own = (int64_t)(std::min(bc_max, batch - b0) / nr) * seq;
          WV_CUDA(cudaMemcpy(static_cast<char*>(post) + (int64_t)i * bcl * seq * dm * es,
                             static_cast<char*>(postd) + (r0 + m->rank * own) * dm * es, own * dm * es,
                             cudaMemcpyDeviceToHost), "D2H post rows");
        }
      } else {
        WV_CUDA(cudaMemcpy(post, postd, M * dm * es, cudaMemcpyDeviceToHost), "D2H post");
        if (pre) WV_CUDA(cudaMemcpy(pre, pred, M * m->qd_l * es, cudaMemcpyDeviceToHost), "D2H pre");
      }
    } else {
      if (!chunked) {
        WV_CUDA(cudaMemcpyAsync(post, postd, M * dm * es, cudaMemcpyDeviceToHost, s), "D2H post");
        if (pre) WV_CUDA(cudaMemcpyAsync(pre, pred, M * m->qd_l * es, cudaMemcpyDeviceToHost, s), "D2H pre");
      }
      WV_TRY(comm_wait(m, s, "forward"));
    }
    WV_TRY(check_device_error(m->dev));
  }
  return Status::ok();
}

// ------------------------------------------------------------------ KV cache
Status kv_create(Mha* m, int max_batch, int max_ctx, Kv** out) {
  if (!m || max_batch <= 0 || max_ctx <= 0 || !out) return Status::err(1, "kv: invalid argument");
  WV_CUDA(cudaSetDevice(m->dev->device), "cudaSetDevice");
  auto kv = std::make_unique<Kv>();
  kv->layer = m;
  kv->max_batch = max_batch;
  kv->max_ctx = max_ctx;
  kv->pages_per_seq = (max_ctx + kPageTokens - 1) / kPageTokens;
  const size_t es = m->precision == 0 ? 4 : 2;
  const size_t pool = (size_t)max_batch * kv->pages_per_seq * kPageTokens * m->kd_l * es;
  WV_TRY(kv->k_pool.ensure(pool));
  WV_TRY(kv->v_pool.ensure(pool));
  WV_TRY(kv->block_table.ensure((size_t)max_batch * kv->pages_per_seq * 4));
  WV_TRY(kv->ctx_len.ensure((size_t)max_batch * 4));
  WV_CUDA(make_block_table(kv->block_table.as<int>(), max_batch, kv->pages_per_seq, 0), "block table");
  WV_CUDA(set_ctx(kv->ctx_len.as<int>(), max_batch, 0, 0), "ctx");
  count_launch(2);
  WV_CUDA(cudaDeviceSynchronize(), "kv create");
  kv->ctx_host.assign(max_batch, 0);
  *out = kv.release();
  return Status::ok();
}

Status kv_fill(Kv* kv, int batch, int ctx, const void* k, const void* v, bool on_device, cudaStream_t s) {
  if (!kv || batch <= 0 || batch > kv->max_batch || ctx < 0 || ctx > kv->max_ctx)
    return Status::err(1, "kv: invalid fill");
  Mha* m = kv->layer;
  std::lock_guard<std::mutex> lock(m->mu);
  WV_CUDA(cudaSetDevice(m->dev->device), "cudaSetDevice");
  const size_t es = m->precision == 0 ? 4 : 2;
  const int64_t rows = (int64_t)batch * ctx;
  if (k && v && rows > 0) {
    const void* kd = k;
    const void* vd = v;
    DevBuf tk, tv;
    if (!on_device) {
      WV_TRY(tk.ensure(rows * m->kd_l * es));
      WV_TRY(tv.ensure(rows * m->kd_l * es));
      WV_CUDA(cudaMemcpyAsync(tk.p, k, rows * m->kd_l * es, cudaMemcpyHostToDevice, s), "H2D k");
      WV_CUDA(cudaMemcpyAsync(tv.p, v, rows * m->kd_l * es, cudaMemcpyHostToDevice, s), "H2D v");
      kd = tk.p;
      vd = tv.p;
    }
    WV_TRY(m->slots.ensure(rows * 4));
    WV_CUDA(make_prefill_slots(m->slots.as<int>(), batch, ctx, kv->pages_per_seq, s), "slots");
    WV_CUDA(kv_append(kd, vd, m->kd_l, (int)rows, m->kd_l, m->cfg.hd, m->precision == 1, m->slots.as<int>(),
                      kv->k_pool.p, kv->v_pool.p, s), "kv append");
    count_launch(2);
    if (!on_device) WV_CUDA(cudaStreamSynchronize(s), "kv fill");
  }
  WV_CUDA(set_ctx(kv->ctx_len.as<int>(), batch, ctx, s), "ctx");
  count_launch();
  for (int b = 0; b < batch; ++b) kv->ctx_host[b] = ctx;
  if (!on_device) WV_CUDA(cudaStreamSynchronize(s), "kv fill");
  return Status::ok();
}

Status mha_decode(Mha* m, Kv* kv, int batch, const void* x, void* pre, void* post, bool on_device,
                  cudaStream_t s) {
  if (!m || !kv || kv->layer != m || !x || !post || batch <= 0 || batch > kv->max_batch)
    return Status::err(1, "mha decode: invalid argument");
  std::lock_guard<std::mutex> lock(m->mu);
  WV_CUDA(cudaSetDevice(m->dev->device), "cudaSetDevice");
  const auto& c = m->cfg;
  const int dm = c.c.d_model;
  const bool f32 = m->precision == 0;
  const size_t es = f32 ? 4 : 2;
  int max_ctx = 0;
  for (int b = 0; b < batch; ++b) max_ctx = std::max(max_ctx, kv->ctx_host[b]);
  if (max_ctx + 1 > kv->max_ctx) return Status::err(1, "mha decode: KV cache full");
  WV_TRY(ensure_rope(m, max_ctx + 1, s));

  const void* xd = x;
  void* postd = post;
  if (!on_device) {
    WV_TRY(m->x_io.ensure((size_t)batch * dm * es));
    WV_TRY(m->post_io.ensure((size_t)batch * dm * es));
    WV_CUDA(cudaMemcpyAsync(m->x_io.p, x, (size_t)batch * dm * es, cudaMemcpyHostToDevice, s), "H2D x");
    xd = m->x_io.p;
    postd = m->post_io.p;
  }
  WV_TRY(m->positions.ensure((size_t)batch * 4));
  WV_TRY(m->slots.ensure((size_t)batch * 4));
  // positions[b] = ctx[b]; slots[b] = page slot of that position; ctx[b] += 1
  WV_CUDA(make_decode_rows(kv->ctx_len.as<int>(), m->positions.as<int>(), m->slots.as<int>(), batch,
                           kv->pages_per_seq, s), "decode rows");
  count_launch();
  WV_TRY(m->qkv.ensure((size_t)batch * m->nqkv * es));

  Proj q;
  q.M = batch;
  q.K = dm;
  q.lda = dm;
  q.N = m->nqkv;
  q.out = m->qkv.p;
  q.ldo = m->nqkv;
  q.rope_cols = m->qd_l + m->kd_l;
  q.positions = m->positions.as<int>();
  q.splitk = true;
  q.w = m->wqkv.p;
  q.w_lo = m->wqkv_lo.p;
  q.w_scale = m->wqkv_scale.as<float>();
  if (f32) {
    WV_TRY(m->x_hi.ensure((size_t)batch * dm * 4));
    WV_TRY(m->x_lo.ensure((size_t)batch * dm * 4));
    WV_CUDA(split_tf32(static_cast<const float*>(xd), m->x_hi.as<float>(), m->x_lo.as<float>(),
                       (int64_t)batch * dm, s), "split x");
    count_launch();
    q.a = m->x_hi.p;
    q.a_lo = m->x_lo.p;
  } else {
    q.a = xd;
  }
  q.kv_k = kv->k_pool.p;
  q.kv_v = kv->v_pool.p;
  q.kv_slot = m->slots.as<int>();
  q.kv_col0 = m->qd_l;
  q.kv_dim = m->kd_l;
  bool kv_done = false;
  prof_begin(kProfGemmQkvDecode, s);
  WV_TRY(run_proj(m, q, s, &kv_done));
  prof_end(kProfGemmQkvDecode, s);
  if (!kv_done) {
    const char* base = static_cast<const char*>(m->qkv.p);
    WV_CUDA(kv_append(base + (size_t)m->qd_l * es, base + (size_t)(m->qd_l + m->kd_l) * es, m->nqkv, batch,
                      m->kd_l, c.hd, f32 ? 0 : 1, m->slots.as<int>(), kv->k_pool.p, kv->v_pool.p, s),
            "kv append");
    count_launch();
  }

  void* attn = pre;
  if (!attn || !on_device) {
    WV_TRY(m->attn.ensure((size_t)batch * m->qd_l * es));
    attn = m->attn.p;
  }
  DecodeArgs d;
  d.q = m->qkv.p;
  d.ldq = m->nqkv;
  d.k_pool = kv->k_pool.p;
  d.v_pool = kv->v_pool.p;
  d.block_table = kv->block_table.as<int>();
  d.max_pages = kv->pages_per_seq;
  d.ctx_len = kv->ctx_len.as<int>();
  d.out = attn;
  d.ldo = m->qd_l;
  d.is_bf16 = f32 ? 0 : 1;
  d.batch = batch;
  d.num_heads = m->hc;
  d.num_kv_heads = m->khc;
  d.head_dim = c.hd;
  d.alibi = c.alibi;
  d.sigmoid = c.c.softmax == 1;
  d.head_base = m->h0;
  d.total_heads = c.c.num_heads;
  d.scale = c.scale;
  d.max_ctx = max_ctx + 1;
  d.pool_rows = (int64_t)kv->max_batch * kv->pages_per_seq * m->khc * kPageTokens;
  d.err = m->dev->err;
  d.sm_count = m->dev->sm_count;
  WV_TRY(kv->scratch.ensure(decode_scratch_floats(d) * 4));
  d.partial = kv->scratch.as<float>();
  prof_begin(kProfAttnDecode, s);
  WV_CUDA(attn_decode(d, s), "attn_decode");
  prof_end(kProfAttnDecode, s);
  count_launch(2);

  Proj o;
  o.M = batch;
  o.K = m->qd_l;
  o.lda = m->qd_l;
  o.N = dm;
  o.out = postd;
  o.ldo = dm;
  o.w = m->wo.p;
  o.w_lo = m->wo_lo.p;
  o.w_scale = m->wo_scale.as<float>();
  o.splitk = true;
  if (f32) {
    WV_TRY(m->attn_hi.ensure((size_t)batch * m->qd_l * 4));
    WV_TRY(m->attn_lo.ensure((size_t)batch * m->qd_l * 4));
    WV_CUDA(split_tf32(static_cast<const float*>(attn), m->attn_hi.as<float>(), m->attn_lo.as<float>(),
                       (int64_t)batch * m->qd_l, s), "split attn");
    count_launch();
    o.a = m->attn_hi.p;
    o.a_lo = m->attn_lo.p;
  } else {
    o.a = attn;
  }
  prof_begin(kProfGemmODecode, s);
  WV_TRY(run_proj(m, o, s));
  prof_end(kProfGemmODecode, s);
  if (m->comm) {
    // The decode output (batch x d_model) is small: one peer-memory kernel over
    // NVLink instead of NCCL when the layer can take it.
    const size_t count = (size_t)batch * dm;
    prof_begin(kProfAllReduce, s);
    if (comm_peer_ok(m, count * es)) WV_TRY(comm_peer_allreduce(m, postd, count, !f32, s));
    else WV_TRY(comm_allreduce(m, postd, count, !f32, s));
    prof_end(kProfAllReduce, s);
  }
  for (int b = 0; b < batch; ++b) kv->ctx_host[b] += 1;
  if (!on_device) {
    // pageable outputs with a communicator: copy only after the bounded wait (see
    // mha_forward)
    const bool defer_d2h = m->comm && m->nranks > 1 && (!host_pinned(post) || !host_pinned(pre));
    if (defer_d2h) WV_TRY(comm_wait(m, s, "decode"));
    WV_CUDA(cudaMemcpyAsync(post, postd, (size_t)batch * dm * es, cudaMemcpyDeviceToHost, s), "D2H post");
    if (pre) WV_CUDA(cudaMemcpyAsync(pre, attn, (size_t)batch * m->qd_l * es, cudaMemcpyDeviceToHost, s), "D2H pre");
    WV_TRY(comm_wait(m, s, "decode"));
    WV_TRY(check_device_error(m->dev));
  }
  return Status::ok();
}

} // namespace wv

// welvet_mha_normalbp_f32 on the B200 (reference src/interop/c_abi.cpp:249-325,
// src/layers/mha/mha.cpp:212-369): forward through the resident FP32 layer,
// MSE loss and gradient (or the caller's dL/dpost), the backward — dense
// gradients as 3xTF32 tensor-core GEMMs over transposed operands, the attention
// backward with the reference's stream semantics (csrc/mha_bwd.cu) — SGD of FP32
// storage and the weight export. One call, synchronous, host buffers.
#include <cuda_runtime.h>

#include <cmath>
#include <cstdio>
#include <cstring>
#include <map>
#include <memory>
#include <mutex>
#include <vector>

#include "../../include/welvet_c.h"
#include "engine.hpp"

namespace wv {
namespace {

inline int64_t round4(int64_t v) { return (v + 3) / 4 * 4; }

// A TF32 hi/lo operand [rows, k_p] (contiguous, zero padded).
struct Operand {
  DevBuf hi, lo;
  Status make(size_t elems) {
    WV_TRY(hi.ensure(elems * 4));
    return lo.ensure(elems * 4);
  }
};

// src [rows, cols] -> operand [rows, round4(cols)]
Status op_rows(Operand& o, const float* src, int64_t rows, int cols, cudaStream_t s) {
  const int cp = (int)round4(cols);
  WV_TRY(o.make((size_t)rows * cp));
  WV_CUDA(pad_operand(src, 0, rows, cols, cp, o.hi.as<float>(), o.lo.as<float>(), nullptr, s), "pad operand");
  count_launch();
  return Status::ok();
}
// src [rows, cols] -> operand [cols, round4(rows)] (transposed)
Status op_cols(Operand& o, const float* src, int64_t rows, int cols, cudaStream_t s) {
  const int64_t rp = round4(rows);
  WV_TRY(o.make((size_t)cols * rp));
  WV_CUDA(transpose_split(src, rows, cols, rp, o.hi.as<float>(), o.lo.as<float>(), s), "transpose operand");
  count_launch();
  return Status::ok();
}

// C[M, N] (row stride ldc) = A[M, K] B[N, K]^T in FP32 (3xTF32 UMMA), operands
// prepared by op_rows / op_cols with K padded to kp.
Status gemm_f32(DeviceCtx* d, int M, int N, int kp, const Operand& A, const Operand& B, float* C, int ldc,
                cudaStream_t s) {
  GemmArgs g;
  g.kind = kGemmTF32x3;
  g.M = M;
  g.N = N;
  g.K = kp;
  g.a = A.hi.p;
  g.a_lo = A.lo.p;
  g.lda = kp;
  g.b = B.hi.p;
  g.b_lo = B.lo.p;
  g.ldb = kp;
  g.out = C;
  g.ldo = ldc;
  g.err = d->err;
  g.sm_count = d->sm_count;
  if (!gemm_tc_supported(g)) return Status::err(4, "mha nbp: gradient GEMM operands not TMA-aligned");
  prof_begin(kProfGemmGrad, s);
  WV_CUDA(gemm_tc(g, s), "gradient gemm");
  prof_end(kProfGemmGrad, s);
  count_launch();
  return Status::ok();
}

Status decode_to(DeviceCtx* d, int dtype, const float* src, float* dst, int64_t n, cudaStream_t s) {
  WV_CUDA(cudaMemcpyAsync(dst, src, (size_t)n * 4, cudaMemcpyHostToDevice, s), "weights upload");
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

// The device buffers of a call and the forward layer of its configuration, kept
// per device and reused by later calls: buffers grow on demand and are never freed
// (they live until the process exits); a later call of the same configuration
// only loads its weights into the layer, so a repeated call of one shape allocates
// nothing. The mutex serialises calls on one device.
struct Workspace {
  std::mutex mu;
  std::unique_ptr<Mha> layer;  // the FP32 forward layer of the last call's configuration
  welvet_b200_mha_config layer_cfg{};
  DevBuf wqkv, wo, xb, preb, postb, gy, tgt, qkv, gattn, G, dxb, dwb, wab, part;
  DevBuf ck, cv, qb, gyb, gq, gk, gv, scr, pq, pkv;
  Operand a1, b1, a2, b2;
};

bool same_config(const welvet_b200_mha_config& a, const welvet_b200_mha_config& b) {
  return a.d_model == b.d_model && a.num_heads == b.num_heads && a.num_kv_heads == b.num_kv_heads &&
         a.head_dim == b.head_dim && a.max_seq_len == b.max_seq_len && a.mask == b.mask && a.pos == b.pos &&
         a.softmax == b.softmax && a.window == b.window && a.prefix_len == b.prefix_len &&
         a.window_causal == b.window_causal && a.rope_theta == b.rope_theta &&
         a.scale_override == b.scale_override && a.seq_mode == b.seq_mode && a.precision == b.precision &&
         a.weight_format == b.weight_format && a.head_begin == b.head_begin && a.head_count == b.head_count &&
         a.device == b.device;
}

Workspace* workspace(int device) {
  static std::mutex mu;
  static std::map<int, Workspace*> by_device;
  std::lock_guard<std::mutex> lock(mu);
  Workspace*& w = by_device[device];
  if (!w) w = new Workspace();
  return w;
}

}  // namespace

Status mha_normalbp(const welvet_b200_mha_config& cin, int dtype, int B, int T, const float* Q, const float* K,
                    const float* V, const float* O, const float* x, const float* grad_or_target, bool use_target,
                    double lr, float* pre, float* post, float* dX, float* dW, float* W_after, double* loss) {
  if (!codec_dtype_supported(dtype)) {
    char buf[96];
    std::snprintf(buf, sizeof(buf), "mha nbp: bad dtype %d", dtype);
    return Status::err(1, buf);
  }
  if (lr != 0.0 && dtype != 1) {
    char buf[160];
    std::snprintf(buf, sizeof(buf),
                  "mha nbp: SGD of FormatNone dtype %d storage is not implemented on the B200 path (Float32 only)",
                  dtype);
    return Status::err(2, buf);
  }
  if (!std::isfinite(lr)) return Status::err(1, "weights: bad SGD arguments");
  Cfg cfg;
  WV_TRY(resolve_config(cin, &cfg));
  if (T > cfg.msl) return Status::err(1, "mha: seq > MaxSeqLen");
  DeviceCtx* d = nullptr;
  WV_TRY(device_ctx(cin.device, &d));
  Workspace* ws = workspace(d->device);
  std::lock_guard<std::mutex> lock(ws->mu);
  cudaStream_t s = 0;
  const int dm = cin.d_model, qd = cfg.qd, kd = cfg.kd, nqkv = qd + 2 * kd;
  const int64_t M = (int64_t)B * T, n = M * dm;
  const int64_t nq = (int64_t)qd * dm, nk = (int64_t)kd * dm;
  // decoded weights: Wqkv [nqkv, d] (Q, K, V rows) and Wo [d, qd]
  DevBuf &wqkv = ws->wqkv, &wo = ws->wo, &xb = ws->xb, &preb = ws->preb, &postb = ws->postb, &gy = ws->gy,
         &tgt = ws->tgt, &qkv = ws->qkv, &gattn = ws->gattn, &G = ws->G, &dxb = ws->dxb, &dwb = ws->dwb,
         &wab = ws->wab, &part = ws->part;
  WV_TRY(wqkv.ensure((size_t)nqkv * dm * 4));
  WV_TRY(wo.ensure((size_t)nq * 4));
  float* Wq = wqkv.as<float>();
  float* Wk = Wq + nq;
  float* Wv = Wk + nk;
  WV_TRY(decode_to(d, dtype, Q, Wq, nq, s));
  WV_TRY(decode_to(d, dtype, K, Wk, nk, s));
  WV_TRY(decode_to(d, dtype, V, Wv, nk, s));
  WV_TRY(decode_to(d, dtype, O, wo.as<float>(), nq, s));
  // forward (the resident layer on the decoded weights, stream semantics)
  WV_TRY(xb.ensure((size_t)n * 4));
  WV_TRY(preb.ensure((size_t)M * qd * 4));
  WV_TRY(postb.ensure((size_t)n * 4));
  WV_CUDA(cudaMemcpyAsync(xb.p, x, (size_t)n * 4, cudaMemcpyHostToDevice, s), "x upload");
  if (ws->layer && same_config(ws->layer_cfg, cin)) {
    WV_TRY(mha_reload_fp32(ws->layer.get(), Wq, wo.as<float>(), s));
  } else {
    ws->layer.reset();
    Mha* m = nullptr;
    WV_TRY(mha_mount(cin, 1, Wq, Wk, Wv, wo.as<float>(), true, &m));
    ws->layer.reset(m);
    ws->layer_cfg = cin;
  }
  WV_TRY(mha_forward(ws->layer.get(), B, T, xb.p, preb.p, postb.p, true, s));
  // dL/dpost
  WV_TRY(gy.ensure((size_t)n * 4));
  *loss = 0.0;
  if (use_target) {
    WV_TRY(tgt.ensure((size_t)n * 4));
    const int pg = mse_grid(n);
    WV_TRY(part.ensure((size_t)pg * 8));
    WV_CUDA(cudaMemcpyAsync(tgt.p, grad_or_target, (size_t)n * 4, cudaMemcpyHostToDevice, s), "target upload");
    WV_CUDA(mse_grad(postb.as<float>(), tgt.as<float>(), gy.as<float>(), part.as<double>(), n, s), "mse");
    count_launch();
    std::vector<double> ph((size_t)pg);
    WV_CUDA(cudaMemcpyAsync(ph.data(), part.p, (size_t)pg * 8, cudaMemcpyDeviceToHost, s), "mse download");
    WV_CUDA(cudaStreamSynchronize(s), "mse");
    double s2 = 0;
    for (double v : ph) s2 += v;
    *loss = s2 / (double)n;
  } else {
    WV_CUDA(cudaMemcpyAsync(gy.p, grad_or_target, (size_t)n * 4, cudaMemcpyHostToDevice, s), "grad upload");
  }
  const int64_t Mp = round4(M);
  const int dp = (int)round4(dm), qdp = (int)round4(qd), nqkvp = (int)round4(nqkv);
  Operand &a1 = ws->a1, &b1 = ws->b1, &a2 = ws->a2, &b2 = ws->b2;
  // grad_attn [M, qd] = gy [M, d] . Wo [d, qd]
  WV_TRY(gattn.ensure((size_t)M * qd * 4));
  WV_TRY(op_rows(a1, gy.as<float>(), M, dm, s));
  WV_TRY(op_cols(b1, wo.as<float>(), dm, qd, s));
  WV_TRY(gemm_f32(d, (int)M, qd, dp, a1, b1, gattn.as<float>(), qd, s));
  // dWo [d, qd] = gy^T [d, M] . pre [M, qd]
  WV_TRY(dwb.ensure((size_t)(2 * nq + 2 * nk) * 4));
  float* dWo = dwb.as<float>() + nq + 2 * nk;
  WV_TRY(op_cols(a2, gy.as<float>(), M, dm, s));
  WV_TRY(op_cols(b2, preb.as<float>(), M, qd, s));
  WV_TRY(gemm_f32(d, dm, qd, (int)Mp, a2, b2, dWo, qd, s));
  // q | k | v projections without RoPE (the backward recomputes them, mha.cpp:266-275)
  WV_TRY(qkv.ensure((size_t)M * nqkv * 4));
  WV_TRY(op_rows(a1, xb.as<float>(), M, dm, s));
  WV_TRY(op_rows(b1, wqkv.as<float>(), nqkv, dm, s));
  WV_TRY(gemm_f32(d, (int)M, nqkv, dp, a1, b1, qkv.as<float>(), nqkv, s));
  // attention backward -> G = [gq | gk | gv] [M, nqkv]
  WV_TRY(G.ensure((size_t)M * nqkv * 4));
  {
    float amax = 0.f;
    WV_CUDA(absmax_f32(gattn.as<float>(), M * qd, d->scalars, d->scratch, s), "absmax");
    count_launch(2);
    WV_CUDA(cudaMemcpyAsync(&amax, d->scalars, 4, cudaMemcpyDeviceToHost, s), "absmax download");
    WV_CUDA(cudaStreamSynchronize(s), "absmax");
    BwdArgs a;
    a.B = B;
    a.T = T;
    a.M = M;
    a.nh = cin.num_heads;
    a.nk = cfg.nk;
    a.hd = cfg.hd;
    a.qd = qd;
    a.kd = kd;
    a.msl = cfg.msl;
    a.mask = cfg.c.mask;
    a.window = cfg.c.window;
    a.window_causal = cfg.c.window_causal;
    a.prefix = cfg.c.prefix_len;
    a.rope = cfg.rope;
    a.alibi = cfg.alibi;
    a.sigmoid = cfg.c.softmax == 1;
    a.theta = cfg.c.rope_theta;
    const float sh = (float)cfg.c.scale_override;
    a.scale = sh == 0.0f ? 1.0 / std::sqrt((double)cfg.hd) : cfg.c.scale_override;
    a.shift = amax < 1e-20f ? 64 : 0;
    a.qkv = qkv.as<float>();
    a.ld_qkv = nqkv;
    a.grad_attn = gattn.as<float>();
    a.kvmax = (int)M;
    DevBuf &ck = ws->ck, &cv = ws->cv, &qb = ws->qb, &gyb = ws->gyb, &gq = ws->gq, &gk = ws->gk, &gv = ws->gv,
           &scr = ws->scr, &pq = ws->pq, &pkv = ws->pkv;
    WV_TRY(ck.ensure((size_t)a.msl * kd * 8));
    WV_TRY(cv.ensure((size_t)a.msl * kd * 8));
    WV_TRY(qb.ensure((size_t)T * qd * 8));
    WV_TRY(gyb.ensure((size_t)T * qd * 8));
    WV_TRY(pq.ensure((size_t)kMaxSplit * T * qd * 8));
    WV_TRY(pkv.ensure((size_t)2 * kMaxSplit * a.msl * kd * 8));
    WV_TRY(gq.ensure((size_t)T * qd * 8));
    WV_TRY(gk.ensure((size_t)a.msl * kd * 8));
    WV_TRY(gv.ensure((size_t)a.msl * kd * 8));
    WV_TRY(scr.ensure((size_t)T * a.nh * 2 * a.kvmax * 8));
    a.ck = ck.as<double>();
    a.cv = cv.as<double>();
    a.qb = qb.as<double>();
    a.gyb = gyb.as<double>();
    a.part_q = pq.as<double>();
    a.part_kv = pkv.as<double>();
    a.gq = gq.as<double>();
    a.gk = gk.as<double>();
    a.gv = gv.as<double>();
    a.scratch = scr.as<double>();
    a.g_q = G.as<float>();
    a.g_k = G.as<float>() + qd;
    a.g_v = G.as<float>() + qd + kd;
    a.ld_g = nqkv;
    prof_begin(kProfAttnBwd, s);
    WV_CUDA(attn_backward(a, s), "attention backward");
    prof_end(kProfAttnBwd, s);
    count_launch(attn_backward_launches(a));
  }
  // dX [M, d] = G [M, nqkv] . Wqkv [nqkv, d]   (the three input gradients summed)
  WV_TRY(dxb.ensure((size_t)n * 4));
  WV_TRY(op_rows(a1, G.as<float>(), M, nqkv, s));
  WV_TRY(op_cols(b1, wqkv.as<float>(), nqkv, dm, s));
  WV_TRY(gemm_f32(d, (int)M, dm, nqkvp, a1, b1, dxb.as<float>(), dm, s));
  // dWqkv [nqkv, d] = G^T [nqkv, M] . x [M, d]  -> dW = concat(Q, K, V, O)
  WV_TRY(op_cols(a2, G.as<float>(), M, nqkv, s));
  WV_TRY(op_cols(b2, xb.as<float>(), M, dm, s));
  WV_TRY(gemm_f32(d, nqkv, dm, (int)Mp, a2, b2, dwb.as<float>(), dm, s));
  // SGD and export
  const int64_t nw = 2 * nq + 2 * nk;
  WV_TRY(wab.ensure((size_t)nw * 4));
  WV_CUDA(cudaMemcpyAsync(wab.p, wqkv.p, (size_t)(nq + 2 * nk) * 4, cudaMemcpyDeviceToDevice, s), "export qkv");
  WV_CUDA(cudaMemcpyAsync(wab.as<float>() + nq + 2 * nk, wo.p, (size_t)nq * 4, cudaMemcpyDeviceToDevice, s),
          "export o");
  if (lr != 0.0) {
    WV_CUDA(sgd_f32(wab.as<float>(), dwb.as<float>(), wab.as<float>(), nw, lr, s), "sgd");
    count_launch();
  }
  WV_CUDA(cudaMemcpyAsync(pre, preb.p, (size_t)M * qd * 4, cudaMemcpyDeviceToHost, s), "pre download");
  WV_CUDA(cudaMemcpyAsync(post, postb.p, (size_t)n * 4, cudaMemcpyDeviceToHost, s), "post download");
  WV_CUDA(cudaMemcpyAsync(dX, dxb.p, (size_t)n * 4, cudaMemcpyDeviceToHost, s), "dX download");
  WV_CUDA(cudaMemcpyAsync(dW, dwb.p, (size_t)nw * 4, cudaMemcpyDeviceToHost, s), "dW download");
  WV_CUDA(cudaMemcpyAsync(W_after, wab.p, (size_t)nw * 4, cudaMemcpyDeviceToHost, s), "W download");
  WV_CUDA(cudaStreamSynchronize(s), "mha nbp");
  return check_device_error(d);
}

}  // namespace wv

extern "C" {

// Reference include/welvet_c.h:94-103, src/interop/c_abi.cpp:249-325.
welvet_status welvet_mha_normalbp_f32(int32_t batch, int32_t seq, int32_t d_model, int32_t num_heads,
                                      int32_t num_kv_heads, int32_t head_dim, int32_t max_seq_len, int32_t mask,
                                      int32_t pos, int32_t dtype, int32_t /*backend*/, const float* Q,
                                      const float* K, const float* V, const float* O, const float* x,
                                      const float* grad_or_target, int32_t use_target, double lr, float* pre,
                                      float* post, float* dX, float* dW, float* W_after, double* loss) {
  wv::DeviceRestore restore_device;
  if (batch <= 0 || seq <= 0 || d_model <= 0 || num_heads <= 0 || !Q || !K || !V || !O || !x ||
      !grad_or_target || !pre || !post || !dX || !dW || !W_after || !loss) {
    welvet_status st{};
    st.code = 1;
    std::snprintf(st.message, sizeof(st.message), "mha nbp: invalid argument");
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
  cfg.window_causal = 1;
  cfg.rope_theta = 10000.0;
  cfg.device = -1;
  return wv::to_c(wv::mha_normalbp(cfg, dtype, batch, seq, Q, K, V, O, x, grad_or_target, use_target != 0, lr,
                                   pre, post, dX, dW, W_after, loss));
}

}  // extern "C"

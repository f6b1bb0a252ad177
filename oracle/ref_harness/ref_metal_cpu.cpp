// Test infrastructure (builds oracle/_ref only). A CPU executor that stands in
// for the reference's Metal device layer (src/metal/ops.mm, src/metal/matvec.mm)
// so that the reference's unmodified host code (src/layers/mha/mha.cpp,
// src/layers/dense/dense.cpp, src/layers/{swiglu,rmsnorm,layernorm,embedding}/*.cpp,
// src/weights/*.cpp) runs its own shader kernels on the CPU. Dispatch follows the reference: `run` copies every argument into a
// fresh buffer, runs `threads` invocations and copies writable buffers back
// (ops.mm:13-88); the resident Dense path runs matvec then bias_act over
// batch*rows invocations (matvec.mm:332-400). Invocations of one dispatch are
// independent, so they are spread over host threads.
#include "welvet/metal/matvec.hpp"
#include "welvet/metal/ops.hpp"
#include "welvet/metal/training.hpp"

#include "ref_shaders.hpp"

#include <algorithm>
#include <cmath>
#include <atomic>
#include <cstring>
#include <string>
#include <thread>
#include <vector>

namespace {

struct HostResident {
  std::vector<float> w_xy, bias_xy, x, pre, post;
};

template <class F> void dispatch(std::size_t n, F&& fn) {
  const unsigned hw = std::max(1u, std::thread::hardware_concurrency());
  if (n < 64 || hw == 1) {
    for (std::size_t i = 0; i < n; ++i) fn((uint32_t)i);
    return;
  }
  std::atomic<std::size_t> next{0};
  std::vector<std::thread> pool;
  for (unsigned t = 0; t < hw; ++t)
    pool.emplace_back([&]() {
      for (std::size_t i = next.fetch_add(1); i < n; i = next.fetch_add(1)) fn((uint32_t)i);
    });
  for (auto& th : pool) th.join();
}

} // namespace

namespace welvet::metal {

Status require_dense_compute() { return Status::Ok(); }

Status run(const char* kernel, std::initializer_list<Arg> args, std::initializer_list<int32_t> ints,
           std::initializer_list<float> reals, std::size_t threads) {
  if (args.size() > 8 || ints.size() > 64 || reals.size() > 64 || !threads)
    return Status::Err(StatusCode::InvalidArgument, "Metal op: invalid argument count");
  std::vector<std::vector<float>> storage;
  storage.reserve(8);
  float* bufs[8] = {};
  unsigned idx = 0;
  for (const auto& a : args) {
    std::vector<float> b(std::max<std::size_t>(1, (a.bytes + 3) / 4), 0.0f);
    if (a.bytes) std::memcpy(b.data(), a.input, a.bytes);
    storage.push_back(std::move(b));
    bufs[idx++] = storage.back().data();
  }
  static float dummy[1] = {0};
  for (; idx < 8; ++idx) bufs[idx] = dummy;
  int32_t ci[64] = {};
  float cr[64] = {};
  std::copy(ints.begin(), ints.end(), ci);
  std::copy(reals.begin(), reals.end(), cr);
  if (std::string(kernel) == "op_attention") {
    // one invocation does all the work (tid 0); the others return at once
    for (std::size_t t = 0; t < threads; ++t)
      refshader::op_attention_kernel(bufs, ci, cr, (uint32_t)t);
  } else if (std::string(kernel) == "op_swiglu" || std::string(kernel) == "op_norm_forward" ||
             std::string(kernel) == "op_embedding_forward" || std::string(kernel) == "op_add3") {
    dispatch(threads, [&](uint32_t t) { refshader::op_kernel(kernel, bufs, ci, cr, t); });
  } else {
    return Status::Err(StatusCode::Unsupported,
                       std::string("cpu executor: kernel not on the block forward paths: ") + kernel);
  }
  idx = 0;
  for (const auto& a : args) {
    if (a.output && a.bytes) std::memcpy(a.output, bufs[idx], a.bytes);
    ++idx;
  }
  return Status::Ok();
}

Status resident_mount(ResidentDense* r, const float* W_xy, const float* bias_xy, int32_t bias_len,
                      int32_t batch, int32_t rows, int32_t cols, Activation act) {
  if (!r || !W_xy) return Status::Err(StatusCode::InvalidArgument, "null resident mount");
  if (batch <= 0 || rows <= 0 || cols <= 0)
    return Status::Err(StatusCode::InvalidArgument, "bad resident dims");
  resident_release(r);
  auto* h = new HostResident();
  h->w_xy.assign(W_xy, W_xy + (std::size_t)rows * cols * 2);
  if (bias_len > 0)
    h->bias_xy.assign(bias_xy, bias_xy + (std::size_t)bias_len * 2);
  else
    h->bias_xy.assign(2, 0.0f);
  h->x.resize((std::size_t)batch * cols);
  h->pre.resize((std::size_t)batch * rows);
  h->post.resize((std::size_t)batch * rows);
  r->buf_w = h;
  r->batch = batch;
  r->rows = rows;
  r->cols = cols;
  r->bias_len = bias_len;
  r->act = act;
  return Status::Ok();
}

Status resident_reload_w(ResidentDense* r, const float* W_xy, const float* bias_xy,
                         int32_t bias_len) {
  if (!r || !r->buf_w || !W_xy) return Status::Err(StatusCode::InvalidArgument, "null reload");
  auto* h = static_cast<HostResident*>(r->buf_w);
  std::memcpy(h->w_xy.data(), W_xy, h->w_xy.size() * 4);
  if (bias_len > 0 && bias_xy) std::memcpy(h->bias_xy.data(), bias_xy, (std::size_t)bias_len * 8);
  return Status::Ok();
}

Status resident_execute(ResidentDense* r, const float* x, float* pre, float* post) {
  if (!r || !r->buf_w || !x || !pre || !post)
    return Status::Err(StatusCode::InvalidArgument, "null resident execute");
  auto* h = static_cast<HostResident*>(r->buf_w);
  std::memcpy(h->x.data(), x, h->x.size() * 4);
  const std::size_t total = (std::size_t)r->batch * r->rows;
  const uint32_t in = (uint32_t)r->cols, out = (uint32_t)r->rows, batch = (uint32_t)r->batch;
  dispatch(total, [&](uint32_t gid) {
    refshader::dense_matvec(h->w_xy.data(), h->x.data(), h->pre.data(), in, out, batch, gid);
  });
  dispatch(total, [&](uint32_t gid) {
    refshader::dense_bias_act(h->pre.data(), h->post.data(), h->bias_xy.data(), out, batch,
                              (int32_t)r->act, (uint32_t)r->bias_len, gid);
  });
  std::memcpy(pre, h->pre.data(), total * 4);
  std::memcpy(post, h->post.data(), total * 4);
  return Status::Ok();
}

// matvec.mm:402-490: act' (Linear when `linear`), then gx = W^T d_pre and
// dW = d_pre^T x, each kernel over its own grid.
Status resident_backward(ResidentDense* r, const float* grad_out, const float* input, const float* pre,
                         float* grad_in, float* grad_w, bool linear) {
  if (!r || !r->buf_w || !grad_out || !input || !pre || !grad_in || !grad_w)
    return Status::Err(StatusCode::InvalidArgument, "null resident backward");
  auto* h = static_cast<HostResident*>(r->buf_w);
  const uint32_t in = (uint32_t)r->cols, out = (uint32_t)r->rows, batch = (uint32_t)r->batch;
  const int32_t act = linear ? (int32_t)Activation::Linear : (int32_t)r->act;
  std::vector<float> d_pre((std::size_t)batch * out);
  dispatch((std::size_t)batch * out,
           [&](uint32_t gid) { refshader::dense_act_deriv(grad_out, pre, d_pre.data(), out, batch, act, gid); });
  dispatch((std::size_t)batch * in,
           [&](uint32_t gid) { refshader::dense_matvect(h->w_xy.data(), d_pre.data(), grad_in, in, out, batch, gid); });
  dispatch((std::size_t)out * in,
           [&](uint32_t gid) { refshader::dense_outer(d_pre.data(), input, grad_w, in, out, batch, gid); });
  return Status::Ok();
}

void resident_release(ResidentDense* r) {
  if (r && r->buf_w) {
    delete static_cast<HostResident*>(r->buf_w);
    r->buf_w = nullptr;
  }
}

// training.mm:75-128: gradients split to float2 pairs on the host, the update runs
// in welvet_sgd_f32_f64_grad.
Status sgd_f32_f64_grad(float* weights, const double* grad, std::size_t n, double lr) {
  if (!weights || !grad || !n) return Status::Err(StatusCode::InvalidArgument, "Metal SGD: gradient size");
  std::vector<float> xy(n * 2);
  for (std::size_t i = 0; i < n; ++i) {
    if (!std::isfinite(grad[i]) || std::abs(grad[i]) > 3.4028234663852886e38)
      return Status::Err(StatusCode::Unsupported, "Metal SGD: gradient exceeds soft-double range");
    split_double(grad[i], &xy[2 * i], &xy[2 * i + 1]);
  }
  float rate[2];
  split_double(lr, &rate[0], &rate[1]);
  dispatch(n, [&](uint32_t gid) { refshader::sgd_f32_f64_grad(weights, xy.data(), rate, (uint32_t)n, gid); });
  return Status::Ok();
}

// training.mm:130-180: the loss kernel (one thread, serial order) and the gradient.
Status mse_f32(const float* pred, const float* target, std::size_t n, double* loss, float* grad) {
  if (!pred || !target || (!loss && !grad) || !n)
    return Status::Err(StatusCode::InvalidArgument, "Metal MSE: invalid arguments");
  if (loss) {
    float l2[2] = {0.f, 0.f};
    refshader::mse_loss(pred, target, l2, (uint32_t)n);
    std::memcpy(loss, l2, sizeof(double));
  }
  if (grad) dispatch(n, [&](uint32_t gid) { refshader::mse_grad(pred, target, grad, (uint32_t)n, gid); });
  return Status::Ok();
}

} // namespace welvet::metal

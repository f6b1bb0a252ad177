// Test infrastructure — NOT part of the product. FP64 restatement of the
// welvet.metal MHA forward (see oracle.h). Every function cites the reference
// lines it restates. The reference emulates f64 with float2 "soft-double"
// arithmetic (shaders/welvet_dense.metal:1-3); this file uses IEEE double,
// which is the Go float64 contract those shaders emulate.
#include "oracle.h"

#include <algorithm>
#include <atomic>
#include <cmath>
#include <cstdio>
#include <cstring>
#include <thread>
#include <vector>

namespace {

template <class F> void parallel_for(int64_t n, int threads, F&& fn) {
  if (threads <= 0) threads = (int)std::max(1u, std::thread::hardware_concurrency());
  if (threads == 1 || n <= 1) {
    for (int64_t i = 0; i < n; ++i) fn(i);
    return;
  }
  std::atomic<int64_t> next{0};
  std::vector<std::thread> pool;
  const int nt = (int)std::min<int64_t>(threads, n);
  for (int t = 0; t < nt; ++t)
    pool.emplace_back([&]() {
      for (int64_t i = next.fetch_add(1); i < n; i = next.fetch_add(1)) fn(i);
    });
  for (auto& th : pool) th.join();
}

void set_msg(char* msg, int32_t len, const char* s) {
  if (msg && len > 0) std::snprintf(msg, (size_t)len, "%s", s);
}

// attn_allow (shaders/ops_mha.metal:1-12). c[6] mask, c[9] window, c[5] MSL,
// c[11] window_causal, c[10] prefix length.
inline bool allow(const oracle_mha_cfg& c, int q, int k) {
  const int mask = c.mask;
  if (mask == 2) return true;
  if (mask == 3) {
    const int w = c.window > 0 ? c.window : c.max_seq_len;
    return c.window_causal ? (k <= q && k >= q - w + 1) : (std::abs(q - k) < w);
  }
  if (mask == 4 && q < c.prefix_len && k < c.prefix_len) return true;
  return k <= q;
}

// The reference carries scale as float2 split of scale_override and falls back
// to 1/sqrt(HD) only when its high part is 0 (ops_mha.metal:46-48).
inline double attn_scale(const oracle_mha_cfg& c) {
  const float hi = (float)c.scale_override;
  if (hi == 0.0f) return 1.0 / std::sqrt((double)c.head_dim);
  return c.scale_override;
}

// rope_gpu (ops_mha.metal:13-30), forward direction, in double. The exponent
// 2i/hd is a float32 division in the reference and is kept so.
void rope_inplace(double* v, int pos, int nh, int hd, double theta) {
  const int half = hd / 2;
  if (half < 1 || (float)theta <= 0.0f) return;
  const double ltheta = std::log(theta);
  for (int head = 0; head < nh; ++head)
    for (int i = 0; i < half; ++i) {
      const float e = (float)(2 * i) / (float)hd;
      const double power = std::exp(ltheta * (double)e);
      const double angle = (double)pos / power;
      const double cs = std::cos(angle), sn = std::sin(angle);
      double* a = v + (size_t)head * hd + i;
      double* b = a + half;
      const double x = *a, y = *b;
      *a = x * cs - y * sn;
      *b = x * sn + y * cs;
    }
}

// rope_gpu with reverse = true (ops_mha.metal:21-23): the transposed rotation,
// applied to gradients.
void rope_reverse_inplace(double* v, int pos, int nh, int hd, double theta) {
  const int half = hd / 2;
  if (half < 1 || (float)theta <= 0.0f) return;
  const double ltheta = std::log(theta);
  for (int head = 0; head < nh; ++head)
    for (int i = 0; i < half; ++i) {
      const float e = (float)(2 * i) / (float)hd;
      const double power = std::exp(ltheta * (double)e);
      const double angle = (double)pos / power;
      const double cs = std::cos(angle), sn = std::sin(angle);
      double* a = v + (size_t)head * hd + i;
      double* b = a + half;
      const double x = *a, y = *b;
      *a = x * cs + y * sn;
      *b = -x * sn + y * cs;
    }
}

// ALiBi slope 2^(-8(h+1)/NH) with the exponent rounded to float32 as in
// ops_mha.metal:96-97.
inline double alibi_slope(int head, int nh) {
  const float e = -(float)(head + 1) * 8.0f / (float)nh;
  return std::exp2((double)e);
}

// One query row: scores over allowed keys, softmax (or sigmoid), P·V, rounded
// to float (ops_mha.metal:81-127). key(kidx) returns the rotated key of key
// index kidx; val(kidx) the value row; both already offset to the kv head.
template <class KeyFn, class ValFn>
void attend_row(const oracle_mha_cfg& c, int head, int pos, int kvlen, const double* q,
                KeyFn key, ValFn val, double scale, float* out, std::vector<double>& score,
                std::vector<char>& ok) {
  const int hd = c.head_dim;
  const bool alibi = c.pos == 2 || c.pos == 3;
  score.assign((size_t)kvlen, 0.0);
  ok.assign((size_t)kvlen, 0);
  int count = 0;
  double mx = -1e300;
  for (int k = 0; k < kvlen; ++k) {
    if (!allow(c, pos, k)) continue;
    const double* kr = key(k);
    double dot = 0;
    for (int z = 0; z < hd; ++z) dot += q[z] * kr[z];
    double sc = dot * scale;
    if (alibi) sc += -alibi_slope(head, c.num_heads) * (double)(float)std::abs(pos - k);
    score[(size_t)k] = sc;
    ok[(size_t)k] = 1;
    mx = std::max(mx, sc);
    ++count;
  }
  if (!count) {
    for (int z = 0; z < hd; ++z) out[z] = 0.0f;
    return;
  }
  const bool sigmoid = c.softmax == 1;
  double sum = 0;
  for (int k = 0; k < kvlen; ++k)
    if (ok[(size_t)k]) {
      const double s = score[(size_t)k];
      score[(size_t)k] = sigmoid ? 1.0 / (1.0 + std::exp(-s)) : std::exp(s - mx);
      sum += score[(size_t)k];
    }
  if (!sigmoid)
    for (int k = 0; k < kvlen; ++k)
      if (ok[(size_t)k]) score[(size_t)k] /= sum;
  for (int z = 0; z < hd; ++z) {
    double o = 0;
    for (int k = 0; k < kvlen; ++k)
      if (ok[(size_t)k]) o += score[(size_t)k] * val(k)[z];
    out[z] = (float)o;
  }
}

} // namespace

extern "C" {

int32_t oracle_mha_validate(oracle_mha_cfg* c, char* msg, int32_t msg_len) {
  if (!c) {
    set_msg(msg, msg_len, "mha: nil config");
    return 1;
  }
  if (c->d_model <= 0 || c->num_heads <= 0) {
    set_msg(msg, msg_len, "mha: need DModel>0 and NumHeads>0");
    return 1;
  }
  if (c->head_dim <= 0) {
    if (c->d_model % c->num_heads != 0) {
      set_msg(msg, msg_len, "mha: HeadDim unset and DModel%NumHeads!=0");
      return 1;
    }
    c->head_dim = c->d_model / c->num_heads;
  }
  if (c->num_kv_heads <= 0) c->num_kv_heads = c->num_heads;
  if (c->num_heads % c->num_kv_heads != 0) {
    set_msg(msg, msg_len, "mha: NumHeads not divisible by NumKVHeads");
    return 1;
  }
  if (c->max_seq_len <= 0) c->max_seq_len = 512;
  if (c->mask == 0) c->mask = 1;
  if (c->rope_theta <= 0) c->rope_theta = 10000;
  if (c->softmax != 0 && c->softmax != 1) {
    set_msg(msg, msg_len, "mha: unknown Softmax");
    return 1;
  }
  return 0;
}

void oracle_dense(const float* x, const float* W, float* y, int64_t M, int64_t K, int64_t N,
                  int32_t threads) {
  // One work item per 8 output rows keeps x rows hot in cache.
  const int64_t rows_per = 8;
  parallel_for((M + rows_per - 1) / rows_per, threads, [&](int64_t blk) {
    const int64_t m0 = blk * rows_per, m1 = std::min(M, m0 + rows_per);
    for (int64_t m = m0; m < m1; ++m) {
      const float* xr = x + m * K;
      for (int64_t n = 0; n < N; ++n) {
        const float* wr = W + n * K;
        double acc = 0;
        for (int64_t k = 0; k < K; ++k) acc += (double)wr[k] * (double)xr[k];
        y[m * N + n] = (float)acc;
      }
    }
  });
}

int32_t oracle_attention(const oracle_mha_cfg* cfg, int32_t B, int32_t T, const float* q,
                         const float* k, const float* v, float* out, int32_t threads) {
  oracle_mha_cfg c = *cfg;
  if (oracle_mha_validate(&c, nullptr, 0)) return 1;
  const int NH = c.num_heads, NK = c.num_kv_heads, HD = c.head_dim, MSL = c.max_seq_len;
  const int QD = NH * HD, KD = NK * HD, group = NH / NK;
  const bool rope = c.pos == 0 || c.pos == 3;
  const double scale = attn_scale(c);
  const int64_t M = (int64_t)B * T;

  // Rotate every q row and every key row once, at the position the reference
  // rotates it with (its own position: ops_mha.metal:68-80).
  std::vector<double> qr((size_t)M * QD), kr((size_t)M * KD), vr((size_t)M * KD);
  parallel_for(M, threads, [&](int64_t tok) {
    const int pos = c.per_sequence ? (int)(tok % T) : (int)tok;
    double* qd = &qr[(size_t)tok * QD];
    double* kd = &kr[(size_t)tok * KD];
    for (int i = 0; i < QD; ++i) qd[i] = q[tok * QD + i];
    for (int i = 0; i < KD; ++i) {
      kd[i] = k[tok * KD + i];
      vr[(size_t)tok * KD + i] = v[tok * KD + i];
    }
    if (rope) {
      rope_inplace(qd, pos, NH, HD, c.rope_theta);
      rope_inplace(kd, pos, NK, HD, c.rope_theta);
    }
  });

  parallel_for((int64_t)B * NH, threads, [&](int64_t item) {
    const int b = (int)(item / NH), head = (int)(item % NH), kh = head / group;
    std::vector<double> score;
    std::vector<char> ok;
    for (int t = 0; t < T; ++t) {
      const int64_t tok = (int64_t)b * T + t;
      const double* qrow = &qr[(size_t)tok * QD + (size_t)head * HD];
      float* orow = out + tok * QD + (int64_t)head * HD;
      if (c.per_sequence) {
        const int64_t base = (int64_t)b * T;
        attend_row(
            c, head, t, T, qrow,
            [&](int kk) { return &kr[(size_t)(base + kk) * KD + (size_t)kh * HD]; },
            [&](int kk) { return &vr[(size_t)(base + kk) * KD + (size_t)kh * HD]; }, scale, orow,
            score, ok);
      } else {
        // Stream mode: key index kk reads ring slot kk % MSL, which after batch b's
        // writes holds the latest position p <= (b+1)T-1 with p == kk (mod MSL).
        const int last = (b + 1) * T - 1;
        auto src = [&](int kk) {
          const int s = kk % MSL;
          return (int64_t)s + (int64_t)MSL * ((last - s) / MSL);
        };
        attend_row(
            c, head, (int)tok, (b + 1) * T, qrow,
            [&](int kk) { return &kr[(size_t)src(kk) * KD + (size_t)kh * HD]; },
            [&](int kk) { return &vr[(size_t)src(kk) * KD + (size_t)kh * HD]; }, scale, orow,
            score, ok);
      }
    }
  });
  return 0;
}

int32_t oracle_mha_forward(const oracle_mha_cfg* cfg, int32_t B, int32_t T, const float* Wq,
                           const float* Wk, const float* Wv, const float* Wo, const float* x,
                           float* pre, float* post, float* q_out, float* k_out, float* v_out,
                           int32_t threads) {
  oracle_mha_cfg c = *cfg;
  if (oracle_mha_validate(&c, nullptr, 0)) return 1;
  if (B <= 0 || T <= 0) return 1;
  if (T > c.max_seq_len) return 1; // mha.cpp:159-161
  const int64_t M = (int64_t)B * T;
  const int d = c.d_model, QD = c.num_heads * c.head_dim, KD = c.num_kv_heads * c.head_dim;
  std::vector<float> q((size_t)M * QD), k((size_t)M * KD), v((size_t)M * KD);
  oracle_dense(x, Wq, q.data(), M, d, QD, threads);
  oracle_dense(x, Wk, k.data(), M, d, KD, threads);
  oracle_dense(x, Wv, v.data(), M, d, KD, threads);
  if (q_out) std::memcpy(q_out, q.data(), q.size() * 4);
  if (k_out) std::memcpy(k_out, k.data(), k.size() * 4);
  if (v_out) std::memcpy(v_out, v.data(), v.size() * 4);
  if (int32_t st = oracle_attention(&c, B, T, q.data(), k.data(), v.data(), pre, threads)) return st;
  oracle_dense(pre, Wo, post, M, QD, d, threads);
  return 0;
}

int32_t oracle_mha_decode(const oracle_mha_cfg* cfg, int32_t B, const int32_t* ctx_len,
                          int64_t cache_stride, const float* k_cache, const float* v_cache,
                          const float* Wq, const float* Wk, const float* Wv, const float* Wo,
                          const float* x_new, float* pre, float* post, float* k_new_out,
                          float* v_new_out, int32_t threads) {
  oracle_mha_cfg c = *cfg;
  if (oracle_mha_validate(&c, nullptr, 0)) return 1;
  const int d = c.d_model, NH = c.num_heads, HD = c.head_dim, QD = NH * HD;
  const int NK = c.num_kv_heads, KD = NK * HD, group = NH / NK;
  const bool rope = c.pos == 0 || c.pos == 3;
  const double scale = attn_scale(c);
  std::vector<float> q((size_t)B * QD), k((size_t)B * KD), v((size_t)B * KD);
  oracle_dense(x_new, Wq, q.data(), B, d, QD, threads);
  oracle_dense(x_new, Wk, k.data(), B, d, KD, threads);
  oracle_dense(x_new, Wv, v.data(), B, d, KD, threads);
  std::vector<double> qr((size_t)B * QD), kr((size_t)B * KD), vr((size_t)B * KD);
  for (int b = 0; b < B; ++b) {
    for (int i = 0; i < QD; ++i) qr[(size_t)b * QD + i] = q[(size_t)b * QD + i];
    for (int i = 0; i < KD; ++i) {
      kr[(size_t)b * KD + i] = k[(size_t)b * KD + i];
      vr[(size_t)b * KD + i] = v[(size_t)b * KD + i];
    }
    if (rope) {
      rope_inplace(&qr[(size_t)b * QD], ctx_len[b], NH, HD, c.rope_theta);
      rope_inplace(&kr[(size_t)b * KD], ctx_len[b], NK, HD, c.rope_theta);
    }
    if (k_new_out)
      for (int i = 0; i < KD; ++i) k_new_out[(size_t)b * KD + i] = (float)kr[(size_t)b * KD + i];
    if (v_new_out)
      for (int i = 0; i < KD; ++i) v_new_out[(size_t)b * KD + i] = v[(size_t)b * KD + i];
  }
  parallel_for((int64_t)B * NH, threads, [&](int64_t item) {
    const int b = (int)(item / NH), head = (int)(item % NH), kh = head / group;
    const int L = ctx_len[b];
    std::vector<double> kc((size_t)(L + 1) * HD), vc((size_t)(L + 1) * HD);
    for (int p = 0; p < L; ++p)
      for (int z = 0; z < HD; ++z) {
        const int64_t off = ((int64_t)b * cache_stride + p) * KD + (int64_t)kh * HD + z;
        kc[(size_t)p * HD + z] = k_cache[off];
        vc[(size_t)p * HD + z] = v_cache[off];
      }
    for (int z = 0; z < HD; ++z) {
      kc[(size_t)L * HD + z] = kr[(size_t)b * KD + (size_t)kh * HD + z];
      vc[(size_t)L * HD + z] = vr[(size_t)b * KD + (size_t)kh * HD + z];
    }
    std::vector<double> score;
    std::vector<char> ok;
    oracle_mha_cfg cc = c;
    cc.per_sequence = 1;
    attend_row(
        cc, head, L, L + 1, &qr[(size_t)b * QD + (size_t)head * HD],
        [&](int kk) { return &kc[(size_t)kk * HD]; }, [&](int kk) { return &vc[(size_t)kk * HD]; },
        scale, pre + (int64_t)b * QD + (int64_t)head * HD, score, ok);
  });
  oracle_dense(pre, Wo, post, B, QD, d, threads);
  return 0;
}

} // extern "C"

// ------------------------------------------------------------------ backward
namespace {

// welvet_dense_matvect_softdouble_batch (welvet_dense.metal:122-154): gx[m,i] =
// fl32(sum_o W[o,i] * gy[m,o]), o ascending (the power-of-two pre-scaling of tiny
// operands is exact and has no effect in double).
void dense_grad_in(const float* gy, const float* W, float* gx, int64_t M, int64_t out, int64_t in,
                   int threads) {
  parallel_for(M, threads, [&](int64_t m) {
    for (int64_t i = 0; i < in; ++i) {
      double acc = 0;
      for (int64_t o = 0; o < out; ++o) acc += (double)W[o * in + i] * (double)gy[m * out + o];
      gx[m * in + i] = (float)acc;
    }
  });
}

// welvet_dense_outer_batch (welvet_dense.metal:156-184): dW[o,i] accumulated over
// the batch in FP32, each exact product added with one rounding, batch ascending.
void dense_grad_w(const float* gy, const float* x, float* dW, int64_t M, int64_t out, int64_t in,
                  int threads) {
  parallel_for(out, threads, [&](int64_t o) {
    for (int64_t i = 0; i < in; ++i) {
      float acc = 0.0f;
      for (int64_t m = 0; m < M; ++m)
        acc = (float)((double)acc + (double)gy[m * out + o] * (double)x[m * in + i]);
      dW[o * in + i] = acc;
    }
  });
}

// op_attention with back = 1 (ops_mha.metal:31-175), the reference's stream
// semantics: per batch the key/value ring is cleared and refilled with that
// batch's rotated keys only (keys of earlier positions read as zero vectors but
// still take part in the softmax), q gradients are rotated back per batch, key
// gradients accumulate in the ring across batches (each batch rotates back the
// slots of its own positions when it ends), and the token gradients are read
// from the ring slots at the end. Gradients are scaled by 2^64 when every
// attention gradient is below 1e-20.
void attention_backward(const oracle_mha_cfg& c, int B, int T, const float* q, const float* k, const float* v,
                        const float* e, float* gq_out, float* gk_out, float* gv_out) {
  const int NH = c.num_heads, NK = c.num_kv_heads, HD = c.head_dim, MSL = c.max_seq_len;
  const int QD = NH * HD, KD = NK * HD, group = NH / NK;
  const bool rope = c.pos == 0 || c.pos == 3, alibi = c.pos == 2 || c.pos == 3;
  const bool sigmoid = c.softmax == 1;
  const double scale = attn_scale(c);
  const int64_t M = (int64_t)B * T;
  float maxgrad = 0;
  for (int64_t i = 0; i < M * QD; ++i) maxgrad = std::max(maxgrad, std::fabs(e[i]));
  const int shift = maxgrad < 1e-20f ? 64 : 0;
  std::vector<double> ck((size_t)MSL * KD), cv((size_t)MSL * KD), qb((size_t)T * QD), gq((size_t)T * QD);
  std::vector<double> gk((size_t)MSL * KD, 0.0), gv((size_t)MSL * KD, 0.0);
  std::vector<double> score((size_t)M), dw((size_t)M);
  std::vector<char> ok((size_t)M);
  for (int b = 0; b < B; ++b) {
    const int base = b * T, kvlen = base + T;
    std::fill(ck.begin(), ck.end(), 0.0);
    std::fill(cv.begin(), cv.end(), 0.0);
    std::fill(gq.begin(), gq.end(), 0.0);
    for (int t = 0; t < T; ++t) {
      const int pos = base + t;
      const int64_t tok = base + t;
      const size_t slot = (size_t)(pos % MSL) * KD;
      for (int i = 0; i < QD; ++i) qb[(size_t)t * QD + i] = q[tok * QD + i];
      for (int i = 0; i < KD; ++i) {
        ck[slot + i] = k[tok * KD + i];
        cv[slot + i] = v[tok * KD + i];
      }
      if (rope) {
        rope_inplace(&qb[(size_t)t * QD], pos, NH, HD, c.rope_theta);
        rope_inplace(&ck[slot], pos, NK, HD, c.rope_theta);
      }
    }
    for (int head = 0; head < NH; ++head)
      for (int t = 0; t < T; ++t) {
        const int pos = base + t, kh = head / group;
        const size_t qo = (size_t)t * QD + (size_t)head * HD;
        int count = 0;
        double mx = -1e300;
        for (int kk = 0; kk < kvlen; ++kk) {
          ok[(size_t)kk] = allow(c, pos, kk);
          if (!ok[(size_t)kk]) continue;
          const double* kr = &ck[(size_t)(kk % MSL) * KD + (size_t)kh * HD];
          double dot = 0;
          for (int z = 0; z < HD; ++z) dot += qb[qo + z] * kr[z];
          double sc = dot * scale;
          if (alibi) sc += -alibi_slope(head, NH) * (double)(float)std::abs(pos - kk);
          score[(size_t)kk] = sc;
          mx = std::max(mx, sc);
          ++count;
        }
        if (!count) continue;
        double sum = 0;
        for (int kk = 0; kk < kvlen; ++kk)
          if (ok[(size_t)kk]) {
            const double s0 = score[(size_t)kk];
            score[(size_t)kk] = sigmoid ? 1.0 / (1.0 + std::exp(-s0)) : std::exp(s0 - mx);
            sum += score[(size_t)kk];
          }
        if (!sigmoid)
          for (int kk = 0; kk < kvlen; ++kk)
            if (ok[(size_t)kk]) score[(size_t)kk] /= sum;
        const float* grow = e + (int64_t)pos * QD + (int64_t)head * HD;
        double sumdw = 0;
        for (int kk = 0; kk < kvlen; ++kk) {
          dw[(size_t)kk] = 0;
          if (!ok[(size_t)kk]) continue;
          const size_t vi0 = (size_t)(kk % MSL) * KD + (size_t)kh * HD;
          for (int z = 0; z < HD; ++z) {
            const double gyz = std::ldexp((double)grow[z], shift);
            gv[vi0 + z] += score[(size_t)kk] * gyz;
            dw[(size_t)kk] += cv[vi0 + z] * gyz;
          }
          sumdw += dw[(size_t)kk] * score[(size_t)kk];
        }
        for (int kk = 0; kk < kvlen; ++kk)
          if (ok[(size_t)kk]) {
            const double sc = score[(size_t)kk];
            double delta = sigmoid ? dw[(size_t)kk] * sc * (1.0 - sc) : sc * (dw[(size_t)kk] - sumdw);
            delta *= scale;
            const size_t ki0 = (size_t)(kk % MSL) * KD + (size_t)kh * HD;
            for (int z = 0; z < HD; ++z) {
              gq[qo + z] += delta * ck[ki0 + z];
              gk[ki0 + z] += delta * qb[qo + z];
            }
          }
      }
    for (int t = 0; t < T; ++t) {
      const int pos = base + t;
      if (rope) rope_reverse_inplace(&gq[(size_t)t * QD], pos, NH, HD, c.rope_theta);
      for (int i = 0; i < QD; ++i)
        gq_out[(int64_t)(base + t) * QD + i] = std::ldexp((float)gq[(size_t)t * QD + i], -shift);
    }
    if (rope)
      for (int t = 0; t < T; ++t)
        rope_reverse_inplace(&gk[(size_t)((base + t) % MSL) * KD], base + t, NK, HD, c.rope_theta);
  }
  for (int64_t tok = 0; tok < M; ++tok)
    for (int i = 0; i < KD; ++i) {
      gk_out[tok * KD + i] = std::ldexp((float)gk[(size_t)(tok % MSL) * KD + i], -shift);
      gv_out[tok * KD + i] = std::ldexp((float)gv[(size_t)(tok % MSL) * KD + i], -shift);
    }
}

}  // namespace

extern "C" int32_t oracle_mha_normalbp(const oracle_mha_cfg* cfg, int32_t B, int32_t T, const float* Wq,
                                       const float* Wk, const float* Wv, const float* Wo, const float* x,
                                       const float* grad_or_target, int32_t use_target, double lr,
                                       int32_t sgd_f32, float* pre, float* post, float* dX, float* dW,
                                       float* W_after, double* loss, int32_t threads) {
  oracle_mha_cfg c = *cfg;
  c.per_sequence = 0;  // the reference's stream semantics throughout
  if (oracle_mha_validate(&c, nullptr, 0)) return 1;
  if (B <= 0 || T <= 0 || T > c.max_seq_len) return 1;
  const int64_t M = (int64_t)B * T;
  const int d = c.d_model, QD = c.num_heads * c.head_dim, KD = c.num_kv_heads * c.head_dim;
  const int64_t n = M * d;
  std::vector<float> q((size_t)M * QD), k((size_t)M * KD), v((size_t)M * KD);
  if (int32_t st = oracle_mha_forward(&c, B, T, Wq, Wk, Wv, Wo, x, pre, post, q.data(), k.data(), v.data(),
                                      threads))
    return st;
  // MSE (welvet_mse_loss / welvet_mse_grad, welvet_dense.metal:193-215): exact
  // differences, the loss in double, gradient 2 d / n rounded once.
  std::vector<float> gy((size_t)n);
  *loss = 0.0;
  if (use_target) {
    double s2 = 0;
    for (int64_t i = 0; i < n; ++i) {
      const double dd = (double)post[i] - (double)grad_or_target[i];
      s2 += dd * dd;
      gy[(size_t)i] = (float)(2.0 * dd / (double)n);
    }
    *loss = s2 / (double)n;
  } else {
    std::memcpy(gy.data(), grad_or_target, (size_t)n * 4);
  }
  // mha::backward_f32 (src/layers/mha/mha.cpp:212-333)
  std::vector<float> gattn((size_t)M * QD);
  dense_grad_in(gy.data(), Wo, gattn.data(), M, d, QD, threads);
  const int64_t nq = (int64_t)QD * d, nk = (int64_t)KD * d;
  float* dWq = dW;
  float* dWk = dW + nq;
  float* dWv = dWk + nk;
  float* dWo = dWv + nk;
  dense_grad_w(gy.data(), pre, dWo, M, d, QD, threads);
  std::vector<float> gq((size_t)M * QD), gk((size_t)M * KD), gv((size_t)M * KD);
  attention_backward(c, B, T, q.data(), k.data(), v.data(), gattn.data(), gq.data(), gk.data(), gv.data());
  std::vector<float> gxq((size_t)n), gxk((size_t)n), gxv((size_t)n);
  dense_grad_in(gq.data(), Wq, gxq.data(), M, QD, d, threads);
  dense_grad_in(gk.data(), Wk, gxk.data(), M, KD, d, threads);
  dense_grad_in(gv.data(), Wv, gxv.data(), M, KD, d, threads);
  for (int64_t i = 0; i < n; ++i)  // op_add3: one rounding of the three-way sum
    dX[i] = (float)((double)gxq[(size_t)i] + (double)gxk[(size_t)i] + (double)gxv[(size_t)i]);
  dense_grad_w(gq.data(), x, dWq, M, QD, d, threads);
  dense_grad_w(gk.data(), x, dWk, M, KD, d, threads);
  dense_grad_w(gv.data(), x, dWv, M, KD, d, threads);
  // SGD (welvet_sgd_f32_f64_grad, welvet_dense.metal:263-281) then export: the step
  // lr * g rounded to FP32 once, subtracted in FP32. Other stored dtypes update their
  // native bytes (op_native_sgd), not restated here.
  const float* Ws[4] = {Wq, Wk, Wv, Wo};
  const int64_t ns[4] = {nq, nk, nk, nq};
  int64_t off = 0;
  for (int w = 0; w < 4; ++w) {
    for (int64_t i = 0; i < ns[w]; ++i) {
      float val = Ws[w][i];
      if (lr != 0.0) {
        const float g = dW[off + i];
        const float step = std::fabs(g) < 1e-20f ? std::ldexp((float)(lr * std::ldexp((double)g, 64)), -64)
                                                 : (float)(lr * (double)g);
        val = val - step;
      }
      W_after[off + i] = val;
    }
    off += ns[w];
  }
  if (lr != 0.0 && !sgd_f32) return 2;
  return 0;
}

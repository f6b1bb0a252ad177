// CPU check of the FormatNone round trips that the device kernels run
// (welvet.metal_b200/csrc/formatnone.cuh, compiled here for the host without
// contraction) against the C restatement of the reference's WeightStore round
// trip (oracle/liboracle.so: oracle_roundtrip). Test infrastructure, built and
// run by tests/test_formatnone_formulas.py.
//
//   formatnone_check [stride]
//
// Dtypes without per-tensor statistics are checked on every stride-th FP32 bit
// pattern; the others on every stride-th float of five ranges [min, max], each
// chunk carrying its range's endpoints so that the oracle's statistics are the
// range's. stride 1 enumerates every input. Both also take every pattern whose
// low 12 bits are 0x000, 0x001, 0x7ff, 0x800, 0x801 or 0xfff (all 2^20 high
// parts): the exact halves of every mantissa truncation point from bit 12 up,
// and their neighbours, where rounding ties are decided.
#include <cstdio>
#include <cstdlib>
#include <utility>
#include <vector>

#include "formatnone.cuh"

extern "C" int32_t oracle_roundtrip(int32_t dtype, const float* w, int64_t n, float* out);

namespace {

using Fn = float (*)(float, const wv::RtStats&, const float*);
template <int... D>
std::vector<Fn> table(std::integer_sequence<int, D...>) {
  return {&wv::rt_elem<D>...};
}

struct Checker {
  int dtype;
  Fn fn;
  wv::RtStats st;
  const float* nf4;
  float lo, hi;  // appended to every chunk when the dtype reads statistics
  bool stats;
  std::vector<float> w, out;
  uint64_t checked = 0, bad = 0;

  void flush() {
    if (w.empty()) return;
    const size_t n = w.size();
    if (stats) {
      w.push_back(lo);
      w.push_back(hi);
    }
    out.resize(w.size());
    if (oracle_roundtrip(dtype, w.data(), (int64_t)w.size(), out.data()) != 0) {
      std::printf("dtype %d: oracle refused\n", dtype);
      std::exit(2);
    }
    for (size_t i = 0; i < n; ++i) {
      const float g = fn(w[i], st, nf4);
      if (wv::f2u(g) != wv::f2u(out[i])) {
        if (bad < 5)
          std::printf("dtype %d: w=%a (0x%08x) device formula %a, oracle %a\n", dtype, w[i], wv::f2u(w[i]), g,
                      out[i]);
        ++bad;
      }
    }
    checked += n;
    w.clear();
  }
  void add(float v) {
    w.push_back(v);
    if (w.size() == (1u << 20)) flush();
  }
  // every stride-th float of [m0, m1] (0 <= m0 <= m1), with the given sign
  void magnitudes(float m0, float m1, bool negative, uint64_t stride) {
    for (uint64_t u = wv::f2u(m0); u <= wv::f2u(m1); u += stride) add(negative ? -wv::u2f((uint32_t)u) : wv::u2f((uint32_t)u));
  }
  // the rounding-boundary patterns, those inside [lo, hi] when statistics apply
  void boundaries() {
    const uint32_t low[6] = {0x000u, 0x001u, 0x7ffu, 0x800u, 0x801u, 0xfffu};
    for (uint32_t h = 0; h < (1u << 20); ++h)
      for (uint32_t l : low) {
        const float v = wv::u2f((h << 12) | l);
        if (!stats || (v >= lo && v <= hi)) add(v);
      }
  }
};

}  // namespace

int main(int argc, char** argv) {
  const uint64_t stride = argc > 1 ? std::strtoull(argv[1], nullptr, 10) : 1021;
  const auto fns = table(std::make_integer_sequence<int, 34>{});
  float nf4[17];
  wv::nf4_table(nf4);
  const float ranges[5][2] = {{-1.f, 1.f}, {0.25f, 3.f}, {-7.5f, -0.001f}, {0.f, 1.f}, {-0.1f, 3.5f}};
  uint64_t total_bad = 0;
  for (int dt = 0; dt < 34; ++dt) {
    uint64_t checked = 0, bad = 0;
    if (!wv::formatnone_needs_stats(dt)) {
      Checker c{dt, fns[dt], {1.f, 0.f, 1.f}, nf4, 0.f, 0.f, false};
      for (uint64_t b = 0; b <= 0xffffffffull; b += stride) c.add(wv::u2f((uint32_t)b));
      c.boundaries();
      c.flush();
      checked = c.checked;
      bad = c.bad;
    } else {
      for (const auto& r : ranges) {
        const float mn = r[0], mx = r[1];
        const float span = (mx - mn) == 0.f ? 1.f : (mx - mn);
        const float amax = std::fmax(std::fabs(mn), std::fabs(mx));
        Checker c{dt, fns[dt], {amax, mn, span}, nf4, mn, mx, true};
        if (mn < 0.f) c.magnitudes(mx < 0.f ? -mx : 0.f, -mn, true, stride);
        if (mx >= 0.f) c.magnitudes(mn > 0.f ? mn : 0.f, mx, false, stride);
        c.boundaries();
        c.flush();
        checked += c.checked;
        bad += c.bad;
      }
    }
    std::printf("dtype %2d: %llu inputs, %llu mismatches\n", dt, (unsigned long long)checked,
                (unsigned long long)bad);
    total_bad += bad;
  }
  return total_bad ? 1 : 0;
}

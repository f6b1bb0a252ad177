// welvet_dense_fwd for the B200 MHA path: the stdin -> stdout binary wires the
// w2a harness drives (reference tools/dense_fwd/main.cpp, volume_fwd.cpp), for the
// two MHA forward wires:
//
//   WVM1 -> WVMO  one-shot MHA forward through welvet_mha_forward_f32
//                 (main.cpp:153-233): 11 int32 (batch, seq, d_model, num_heads,
//                 num_kv, head_dim, msl, mask, pos, dtype, backend), then Q, K, V, O
//                 and x as FP32; out "WVMO", int32 pre_n, pre, int32 post_n, post.
//                 --bench=N: 3 warm-up calls, N timed calls, "WVB1" int64 ns int32 N
//                 before the output.
//   WMV1 -> WVFO  a volume of MHA cells (volume_fwd.cpp:209-300): 7 int32 (depth,
//                 rows, cols, layers_per_cell, batch, backend, n_links), n_links x 8
//                 int32 remote links, per cell in hop order an int32 enabled flag and
//                 for enabled cells 9 int32 (seq, d_model, num_heads, num_kv,
//                 head_dim, msl, mask, pos, dtype) and Q, K, V, O; then x [batch,
//                 seq, d] of the first enabled cell. Mounted once (mha::new_configured
//                 + architecture::bind_mha), run by runtime::forward::volume_dense;
//                 out "WVFO", int32 n, output. --bench=N: "WVB2" int64 mount_ns int64
//                 exec_ns int32 N first.
//
// Exit codes as the reference's tool: 0 ok, 1 the library returned an error (its
// message on stderr), 2 malformed wire or usage. Other wires of the reference's
// tool (Dense, norms, training, ...) are not part of this path: "unsupported wire".
#include <chrono>
#include <cstdint>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <functional>
#include <string>
#include <vector>

#include "welvet/architecture.hpp"
#include "welvet/mha.hpp"
#include "welvet/runtime/forward.hpp"
#include "welvet_c.h"

namespace {

bool read_exact(void* p, size_t n) { return std::fread(p, 1, n, stdin) == n; }
template <typename T>
bool read_n(T* p, size_t n) {
  return read_exact(static_cast<void*>(p), n * sizeof(T));
}
bool write_exact(const void* p, size_t n) { return std::fwrite(p, 1, n, stdout) == n; }
template <typename T>
bool write_n(const T* p, size_t n) {
  return write_exact(static_cast<const void*>(p), n * sizeof(T));
}

int64_t now_ns() {
  return std::chrono::duration_cast<std::chrono::nanoseconds>(
             std::chrono::steady_clock::now().time_since_epoch())
      .count();
}

void usage() {
  std::fprintf(stderr,
               "welvet_dense_fwd (welvet B200 MHA path)\n"
               "  --version | --identity | --help\n"
               "  --bench=N -> WVB1 (WVM1) / WVB2 mount_ns+exec_ns (WMV1)\n"
               "  stdin WVM1 -> WVMO | WMV1 -> WVFO\n");
}

// Sizes of an MHA cell's weights (defaults of the reference tool: head_dim 0 ->
// d/heads, num_kv 0 -> heads).
struct Dims {
  int hd = 0, q_dim = 0, kv_dim = 0;
};
bool dims(int d_model, int num_heads, int num_kv, int head_dim, Dims* out) {
  if (num_heads <= 0 || d_model <= 0) return false;
  if (head_dim <= 0 && d_model % num_heads != 0) return false;
  out->hd = head_dim > 0 ? head_dim : d_model / num_heads;
  const int kv = num_kv > 0 ? num_kv : num_heads;
  out->q_dim = num_heads * out->hd;
  out->kv_dim = kv * out->hd;
  return true;
}

int run_mha(int bench_iters) {
  int32_t h[11];
  if (!read_n(h, 11)) {
    std::fprintf(stderr, "welvet_dense_fwd: short WVM1 header\n");
    return 2;
  }
  const int32_t batch = h[0], seq = h[1], d_model = h[2], num_heads = h[3], num_kv = h[4], head_dim = h[5],
                msl = h[6], mask = h[7], pos = h[8], dtype = h[9], backend = h[10];
  Dims dm;
  if (num_heads <= 0 || d_model <= 0 || d_model % num_heads != 0 || !dims(d_model, num_heads, num_kv, head_dim, &dm) ||
      batch <= 0 || seq <= 0) {
    std::fprintf(stderr, "welvet_dense_fwd: bad mha dims\n");
    return 2;
  }
  std::vector<float> Q((size_t)dm.q_dim * d_model), K((size_t)dm.kv_dim * d_model), V((size_t)dm.kv_dim * d_model),
      O((size_t)d_model * dm.q_dim);
  if (!read_n(Q.data(), Q.size()) || !read_n(K.data(), K.size()) || !read_n(V.data(), V.size()) ||
      !read_n(O.data(), O.size())) {
    std::fprintf(stderr, "welvet_dense_fwd: short WVM1 weights\n");
    return 2;
  }
  std::vector<float> x((size_t)batch * seq * d_model);
  if (!read_n(x.data(), x.size())) {
    std::fprintf(stderr, "welvet_dense_fwd: short WVM1 input\n");
    return 2;
  }
  std::vector<float> pre((size_t)batch * seq * dm.q_dim), post((size_t)batch * seq * d_model);
  auto once = [&]() {
    return welvet_mha_forward_f32(batch, seq, d_model, num_heads, num_kv, head_dim, msl, mask, pos, dtype, backend,
                                  Q.data(), K.data(), V.data(), O.data(), x.data(), pre.data(), post.data());
  };
  if (bench_iters > 0) {
    for (int i = 0; i < 3; ++i) {
      const welvet_status st = once();
      if (st.code != 0) {
        std::fprintf(stderr, "welvet_dense_fwd: %s\n", st.message);
        return 1;
      }
    }
    const int64_t t0 = now_ns();
    for (int i = 0; i < bench_iters; ++i) {
      const welvet_status st = once();
      if (st.code != 0) {
        std::fprintf(stderr, "welvet_dense_fwd: %s\n", st.message);
        return 1;
      }
    }
    const int64_t ns = now_ns() - t0;
    const int32_t iters = bench_iters;
    if (!write_exact("WVB1", 4) || !write_n(&ns, 1) || !write_n(&iters, 1)) return 2;
  } else {
    const welvet_status st = once();
    if (st.code != 0) {
      std::fprintf(stderr, "welvet_dense_fwd: %s\n", st.message);
      return 1;
    }
  }
  const int32_t pre_n = (int32_t)pre.size(), post_n = (int32_t)post.size();
  if (!write_exact("WVMO", 4) || !write_n(&pre_n, 1) || !write_n(pre.data(), pre.size()) || !write_n(&post_n, 1) ||
      !write_n(post.data(), post.size()))
    return 2;
  return 0;
}

int run_volume_mha(int bench_iters) {
  namespace arch = welvet::architecture;
  int32_t g[7];
  if (!read_n(g, 7)) {
    std::fprintf(stderr, "welvet_dense_fwd: short WMV1 header\n");
    return 2;
  }
  const int32_t depth = g[0], rows = g[1], cols = g[2], lpc = g[3], batch = g[4], n_links = g[6];
  if (batch <= 0) {
    std::fprintf(stderr, "welvet_dense_fwd: bad batch\n");
    return 2;
  }
  if (n_links < 0 || n_links > (1 << 20)) {
    std::fprintf(stderr, "welvet_dense_fwd: bad link count\n");
    return 2;
  }
  std::vector<int32_t> links((size_t)n_links * 8);
  if (n_links > 0 && !read_n(links.data(), links.size())) return 2;

  struct CellWire {
    bool enabled = false;
    int32_t seq = 0, d_model = 0, num_heads = 0, num_kv = 0, head_dim = 0, msl = 0, mask = 0, pos = 0, dtype = 1;
    arch::Coord coord{};
    std::vector<float> Q, K, V, O;
  };
  const auto hops = arch::hop_order(arch::new_grid(depth, rows, cols, lpc));
  std::vector<CellWire> cells;
  cells.reserve(hops.size());
  int first_seq = -1, first_d = -1;
  for (const auto& coord : hops) {
    CellWire c;
    c.coord = coord;
    int32_t en = 0;
    if (!read_n(&en, 1)) return 2;
    c.enabled = en != 0;
    if (!c.enabled) {
      cells.push_back(std::move(c));
      continue;
    }
    int32_t f[9];
    if (!read_n(f, 9)) return 2;
    c.seq = f[0];
    c.d_model = f[1];
    c.num_heads = f[2];
    c.num_kv = f[3];
    c.head_dim = f[4];
    c.msl = f[5];
    c.mask = f[6];
    c.pos = f[7];
    c.dtype = f[8];
    Dims dm;
    if (!dims(c.d_model, c.num_heads, c.num_kv, c.head_dim, &dm)) {
      std::fprintf(stderr, "welvet_dense_fwd: bad mha dims\n");
      return 2;
    }
    c.Q.resize((size_t)dm.q_dim * c.d_model);
    c.K.resize((size_t)dm.kv_dim * c.d_model);
    c.V.resize((size_t)dm.kv_dim * c.d_model);
    c.O.resize((size_t)c.d_model * dm.q_dim);
    if (!read_n(c.Q.data(), c.Q.size()) || !read_n(c.K.data(), c.K.size()) || !read_n(c.V.data(), c.V.size()) ||
        !read_n(c.O.data(), c.O.size()))
      return 2;
    if (first_seq < 0) {
      first_seq = c.seq;
      first_d = c.d_model;
    }
    cells.push_back(std::move(c));
  }
  if (first_seq < 0) return 1;
  if (first_seq <= 0) {
    std::fprintf(stderr, "welvet_dense_fwd: bad seq\n");
    return 2;
  }
  welvet::TensorF32 input;
  input.shape = {batch, first_seq, first_d};
  input.data.resize((size_t)batch * first_seq * first_d);
  if (!read_n(input.data.data(), input.data.size())) return 2;

  const int64_t tm0 = now_ns();
  arch::Grid grid = arch::new_grid(depth, rows, cols, lpc);
  for (int32_t i = 0; i < n_links; ++i) {
    const int32_t* L = links.data() + (size_t)i * 8;
    const welvet::Status st = arch::set_remote_link(grid, L[0], L[1], L[2], L[3], L[4], L[5], L[6], L[7]);
    if (!st) {
      std::fprintf(stderr, "welvet_dense_fwd: %s\n", st.message.c_str());
      return 1;
    }
  }
  for (const auto& c : cells) {
    if (!c.enabled) continue;
    welvet::mha::Config cfg;
    cfg.d_model = c.d_model;
    cfg.num_heads = c.num_heads;
    cfg.num_kv_heads = c.num_kv;
    cfg.head_dim = c.head_dim;
    cfg.max_seq_len = c.msl;
    cfg.mask = static_cast<welvet::mha::MaskKind>(c.mask);
    cfg.pos = static_cast<welvet::mha::PosKind>(c.pos);
    cfg.mode = welvet::mha::AttnMode::Self;
    cfg.causal = cfg.mask == welvet::mha::MaskKind::Causal;
    welvet::mha::Layer layer;
    welvet::Status st = welvet::mha::new_configured(cfg, static_cast<welvet::DType>(c.dtype), c.Q.data(),
                                                    c.K.data(), c.V.data(), c.O.data(), &layer);
    if (!st) {
      std::fprintf(stderr, "welvet_dense_fwd: %s\n", st.message.c_str());
      return 1;
    }
    st = arch::bind_mha(grid, c.coord.z, c.coord.y, c.coord.x, c.coord.l, std::move(layer));
    if (!st) {
      std::fprintf(stderr, "welvet_dense_fwd: %s\n", st.message.c_str());
      return 1;
    }
  }
  const int64_t mount_ns = now_ns() - tm0;

  welvet::runtime::forward::Result result;
  auto once = [&]() { return welvet::runtime::forward::volume_dense(grid, input, &result); };
  if (bench_iters > 0) {
    for (int i = 0; i < 3; ++i) {
      const welvet::Status st = once();
      if (!st) {
        std::fprintf(stderr, "welvet_dense_fwd: %s\n", st.message.c_str());
        return 1;
      }
    }
    const int64_t te0 = now_ns();
    for (int i = 0; i < bench_iters; ++i) {
      const welvet::Status st = once();
      if (!st) {
        std::fprintf(stderr, "welvet_dense_fwd: %s\n", st.message.c_str());
        return 1;
      }
    }
    const int64_t exec_ns = now_ns() - te0;
    const int32_t iters = bench_iters;
    if (!write_exact("WVB2", 4) || !write_n(&mount_ns, 1) || !write_n(&exec_ns, 1) || !write_n(&iters, 1))
      return 2;
  } else {
    const welvet::Status st = once();
    if (!st) {
      std::fprintf(stderr, "welvet_dense_fwd: %s\n", st.message.c_str());
      return 1;
    }
  }
  const int32_t n = (int32_t)result.output.data.size();
  if (!write_exact("WVFO", 4) || !write_n(&n, 1) || !write_n(result.output.data.data(), result.output.data.size()))
    return 2;
  return 0;
}

}  // namespace

int main(int argc, char** argv) {
  int bench_iters = 0;
  for (int i = 1; i < argc; ++i) {
    const std::string a = argv[i];
    if (a == "--version" || a == "-v") {
      std::printf("%s\n", welvet_version());
      return 0;
    }
    if (a == "--identity") {
      const welvet_status st = welvet_metal_init();
      if (st.code != 0) {
        std::fprintf(stderr, "%s\n", st.message);
        return 1;
      }
      std::printf("%s\n", welvet_runtime_identity());
      return 0;
    }
    if (a == "--help" || a == "-h") {
      usage();
      return 0;
    }
    if (a.rfind("--bench=", 0) == 0) {
      bench_iters = std::atoi(a.c_str() + 8);
      continue;
    }
    std::fprintf(stderr, "unknown arg %s\n", a.c_str());
    usage();
    return 2;
  }
  char magic[4];
  if (!read_exact(magic, 4)) {
    usage();
    return 2;
  }
  if (std::memcmp(magic, "WVM1", 4) == 0) return run_mha(bench_iters);
  if (std::memcmp(magic, "WMV1", 4) == 0) return run_volume_mha(bench_iters);
  std::fprintf(stderr, "welvet_dense_fwd: unsupported wire %.4s (this tool carries the MHA forward wires "
                       "WVM1 and WMV1)\n", magic);
  return 2;
}

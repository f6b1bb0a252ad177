// The C++ layer / volume API of the MHA path (include/welvet/mha.hpp,
// include/welvet/architecture.hpp, include/welvet/runtime/forward.hpp) on top of
// this library's resident-layer C ABI (include/welvet_b200.h). Names, signatures,
// defaults, status codes and messages follow the reference's
// src/layers/mha/mha.cpp, src/architecture/grid.cpp and src/runtime/forward.cpp
// so that a C++ caller of the reference (and the w2a wire tool) can switch; the
// work runs on the B200 kernels through welvet_b200_mha_mount / _forward.
#include <cmath>
#include <map>
#include <sstream>
#include <string>
#include <utility>

#include "welvet/architecture.hpp"
#include "welvet/mha.hpp"
#include "welvet/runtime/forward.hpp"
#include "welvet_b200.h"

namespace welvet {

TensorF32 TensorF32::zeros(int64_t a, int64_t b) {
  TensorF32 t;
  t.shape = {a, b};
  t.data.assign(static_cast<std::size_t>(a * b), 0.0f);
  return t;
}

namespace {
Status from_c(const welvet_status& s) {
  return Status{static_cast<StatusCode>(s.code), std::string(s.message)};
}
}  // namespace

// ------------------------------------------------------------------ mha layer
namespace mha {

double Config::scale() const {
  if (scale_override > 0) return scale_override;
  return 1.0 / std::sqrt(static_cast<double>(head_dim));
}

// Defaults and checks in the reference's order (src/layers/mha/mha.cpp:63-94).
Status validate(Config* cfg) {
  if (!cfg) return Status::Err(StatusCode::InvalidArgument, "mha: nil config");
  if (cfg->d_model <= 0 || cfg->num_heads <= 0)
    return Status::Err(StatusCode::InvalidArgument, "mha: need DModel>0 and NumHeads>0");
  if (cfg->head_dim <= 0) {
    if (cfg->d_model % cfg->num_heads != 0)
      return Status::Err(StatusCode::InvalidArgument, "mha: HeadDim unset and DModel%NumHeads!=0");
    cfg->head_dim = cfg->d_model / cfg->num_heads;
  }
  if (cfg->num_kv_heads <= 0) cfg->num_kv_heads = cfg->num_heads;
  if (cfg->num_heads % cfg->num_kv_heads != 0)
    return Status::Err(StatusCode::InvalidArgument, "mha: NumHeads not divisible by NumKVHeads");
  if (cfg->max_seq_len <= 0) cfg->max_seq_len = 512;
  if (cfg->mask == MaskKind::Unspecified) cfg->mask = MaskKind::Causal;
  if (cfg->mask == MaskKind::Causal) cfg->causal = true;
  if (cfg->rope_theta <= 0) cfg->rope_theta = 10000;
  if (cfg->softmax != SoftmaxKind::Standard && cfg->softmax != SoftmaxKind::Sigmoid)
    return Status::Err(StatusCode::InvalidArgument, "mha: unknown Softmax");
  return Status::Ok();
}

Config decoder_causal(int d_model, int num_heads, int num_kv_heads) {
  Config c;
  c.d_model = d_model;
  c.num_heads = num_heads;
  c.num_kv_heads = num_kv_heads;
  c.mask = MaskKind::Causal;
  c.pos = PosKind::RoPE;
  c.mode = AttnMode::Self;
  c.causal = true;
  return c;
}

namespace {

// The engine's configuration of a validated Config: the reference's stream
// semantics in FP32 on the current device; the window's causal flag is the
// reference's `window_causal || causal` (mha.cpp:183-191, c[11]).
welvet_b200_mha_config engine_config(const Config& c) {
  welvet_b200_mha_config e{};
  welvet_b200_mha_config_default(&e, c.d_model, c.num_heads, c.num_kv_heads);
  e.head_dim = c.head_dim;
  e.max_seq_len = c.max_seq_len;
  e.mask = static_cast<int32_t>(c.mask);
  e.pos = static_cast<int32_t>(c.pos);
  e.softmax = static_cast<int32_t>(c.softmax);
  e.window = c.window;
  e.prefix_len = c.prefix_len;
  e.window_causal = (c.window_causal || c.causal) ? 1 : 0;
  e.rope_theta = c.rope_theta;
  e.scale_override = c.scale_override;
  e.seq_mode = 0;
  e.precision = 0;
  e.weight_format = 0;
  e.head_begin = 0;
  e.head_count = 0;
  e.device = -1;
  return e;
}

bool same_mount(const Config& a, const Config& b) {
  return a.d_model == b.d_model && a.num_heads == b.num_heads && a.num_kv_heads == b.num_kv_heads &&
         a.head_dim == b.head_dim && a.max_seq_len == b.max_seq_len && a.mask == b.mask && a.pos == b.pos &&
         a.softmax == b.softmax && a.window == b.window && a.prefix_len == b.prefix_len &&
         (a.window_causal || a.causal) == (b.window_causal || b.causal) && a.rope_theta == b.rope_theta &&
         a.scale_override == b.scale_override;
}

}  // namespace

Status new_configured(const Config& cfg_in, DType dt, const float* q_init, const float* k_init,
                      const float* v_init, const float* o_init, Layer* out) {
  if (!out) return Status::Err(StatusCode::InvalidArgument, "mha: nil out");
  Config cfg = cfg_in;
  if (auto st = validate(&cfg); !st) return st;
  if (!q_init || !k_init || !v_init || !o_init)
    return Status::Err(StatusCode::InvalidArgument, "mha: nil weight init");
  const welvet_b200_mha_config ec = engine_config(cfg);
  welvet_b200_mha* h = nullptr;
  const welvet_status st =
      welvet_b200_mha_mount(&ec, static_cast<int32_t>(dt), q_init, k_init, v_init, o_init, 0, &h);
  if (st.code != 0) return from_c(st);
  Layer layer;
  layer.cfg = cfg;
  layer.dtype = dt;
  layer.session = std::shared_ptr<welvet_b200_mha>(h, welvet_b200_mha_release);
  layer.mounted = cfg;
  *out = std::move(layer);
  return Status::Ok();
}

Status forward(Layer& layer, const TensorF32& input, TensorF32* pre, TensorF32* post) {
  if (!pre || !post) return Status::Err(StatusCode::InvalidArgument, "mha: nil pre/post");
  Config cfg = layer.cfg;
  if (auto st = validate(&cfg); !st) return st;
  if (cfg.mode != AttnMode::Self) return Status::Gap("mha forward: ModeCross not in baseline");
  if (!layer.session)
    return Status::Err(StatusCode::InvalidArgument, "mha: layer has no mounted weights (new_configured)");
  if (!same_mount(cfg, layer.mounted))
    return Status::Err(StatusCode::Unsupported,
                       "mha: config changed after new_configured; mount the layer again");
  // layout of reference parse_layout (mha.cpp:18-47)
  if (input.data.empty()) return Status::Err(StatusCode::InvalidArgument, "mha: empty input");
  int batch = 0, seq = 0;
  if (input.shape.size() == 3) {
    batch = static_cast<int>(input.shape[0]);
    seq = static_cast<int>(input.shape[1]);
    if (static_cast<int>(input.shape[2]) != cfg.d_model)
      return Status::Err(StatusCode::InvalidArgument, "mha: last dim != d_model");
  } else if (input.shape.size() == 2) {
    batch = 1;
    if (static_cast<int>(input.shape[1]) != cfg.d_model)
      return Status::Err(StatusCode::InvalidArgument, "mha: width != d_model");
    seq = static_cast<int>(input.shape[0]);
  } else {
    return Status::Err(StatusCode::InvalidArgument, "mha: need [batch,seq,d] or [seq,d]");
  }
  if (batch <= 0 || seq <= 0) return Status::Err(StatusCode::InvalidArgument, "mha: bad batch/seq");
  const int64_t rows = static_cast<int64_t>(batch) * seq;
  if (static_cast<int64_t>(input.data.size()) < rows * cfg.d_model)
    return Status::Err(StatusCode::InvalidArgument, "mha: short data");
  if (seq > cfg.max_seq_len) return Status::Err(StatusCode::InvalidArgument, "mha: seq > MaxSeqLen");

  TensorF32 p, q;
  p.shape = {batch, seq, cfg.q_dim()};
  p.data.assign(static_cast<std::size_t>(rows * cfg.q_dim()), 0.0f);
  q.shape = {batch, seq, cfg.d_model};
  q.data.assign(static_cast<std::size_t>(rows * cfg.d_model), 0.0f);
  const welvet_status st = welvet_b200_mha_forward(layer.session.get(), batch, seq, input.data.data(),
                                                   p.data.data(), q.data.data(), 0, nullptr);
  if (st.code != 0) return from_c(st);
  *pre = std::move(p);
  *post = std::move(q);
  return Status::Ok();
}

}  // namespace mha

// --------------------------------------------------------------- architecture
namespace architecture {
namespace {

Status bad_coord(const char* which, int z, int y, int x, int l) {
  std::ostringstream oss;
  oss << "architecture: bad " << which << " coord z=" << z << " y=" << y << " x=" << x << " l=" << l;
  return Status::Err(StatusCode::InvalidArgument, oss.str());
}

}  // namespace

Grid new_grid(int depth, int rows, int cols, int layers_per_cell) {
  Grid g;
  g.depth = depth < 1 ? 1 : depth;
  g.rows = rows < 1 ? 1 : rows;
  g.cols = cols < 1 ? 1 : cols;
  g.layers_per_cell = layers_per_cell < 1 ? 1 : layers_per_cell;
  g.cells.resize(static_cast<std::size_t>(stack_layer_count(g)));
  for (const Coord& c : hop_order(g)) {
    Cell& cell = g.cells[static_cast<std::size_t>(index(g, c.z, c.y, c.x, c.l))];
    cell.meta.z = c.z;
    cell.meta.y = c.y;
    cell.meta.x = c.x;
    cell.meta.l = c.l;
  }
  return g;
}

int index(const Grid& g, int z, int y, int x, int l) {
  return ((z * g.rows + y) * g.cols + x) * g.layers_per_cell + l;
}

Cell* at(Grid& g, int z, int y, int x, int l) {
  if (z < 0 || z >= g.depth || y < 0 || y >= g.rows || x < 0 || x >= g.cols || l < 0 || l >= g.layers_per_cell)
    return nullptr;
  const int i = index(g, z, y, x, l);
  if (i < 0 || i >= static_cast<int>(g.cells.size())) return nullptr;
  return &g.cells[static_cast<std::size_t>(i)];
}

const Cell* at(const Grid& g, int z, int y, int x, int l) { return at(const_cast<Grid&>(g), z, y, x, l); }

std::vector<Coord> hop_order(const Grid& g) {
  std::vector<Coord> out;
  out.reserve(static_cast<std::size_t>(stack_layer_count(g)));
  for (int z = 0; z < g.depth; ++z)
    for (int y = 0; y < g.rows; ++y)
      for (int x = 0; x < g.cols; ++x)
        for (int l = 0; l < g.layers_per_cell; ++l) out.push_back(Coord{z, y, x, l});
  return out;
}

Status set_remote_link(Grid& g, int z, int y, int x, int l, int tz, int ty, int tx, int tl) {
  Cell* c = at(g, z, y, x, l);
  if (!c) return bad_coord("source", z, y, x, l);
  if (!at(g, tz, ty, tx, tl)) return bad_coord("target", tz, ty, tx, tl);
  c->is_remote_link = true;
  c->target_z = tz;
  c->target_y = ty;
  c->target_x = tx;
  c->target_l = tl;
  return Status::Ok();
}

Status bind_mha(Grid& g, int z, int y, int x, int l, mha::Layer op) {
  Cell* c = at(g, z, y, x, l);
  if (!c) return bad_coord("bind", z, y, x, l);
  c->meta.type = LayerType::MultiHeadAttention;
  c->meta.dtype = op.dtype;
  c->meta.z = z;
  c->meta.y = y;
  c->meta.x = x;
  c->meta.l = l;
  c->op_kind = OpKind::MHA;
  c->mha_op = std::move(op);
  return Status::Ok();
}

}  // namespace architecture

// -------------------------------------------------------------- volume forward
namespace runtime::forward {
namespace {
struct CoordLess {
  bool operator()(const architecture::Coord& a, const architecture::Coord& b) const {
    if (a.z != b.z) return a.z < b.z;
    if (a.y != b.y) return a.y < b.y;
    if (a.x != b.x) return a.x < b.x;
    return a.l < b.l;
  }
};
}  // namespace

Status cell(architecture::Cell& c, const TensorF32& in, TensorF32* pre, TensorF32* post) {
  if (c.op_kind == architecture::OpKind::MHA) return mha::forward(c.mha_op, in, pre, post);
  return Status::Gap("runtime.forward: unsupported cell Op");
}

// Reference src/runtime/forward.cpp:74-132.
Status volume_dense(architecture::Grid& g, const TensorF32& input, Result* out) {
  if (!out) return Status::Err(StatusCode::InvalidArgument, "runtime.forward: nil result");
  if (input.data.empty()) return Status::Err(StatusCode::InvalidArgument, "runtime.forward: empty input");
  TensorF32 current = input;
  std::map<architecture::Coord, TensorF32, CoordLess> posts;
  Result result;
  for (const auto& coord : architecture::hop_order(g)) {
    architecture::Cell* c = architecture::at(g, coord.z, coord.y, coord.x, coord.l);
    if (!c || c->meta.is_disabled) continue;
    if (c->op_kind == architecture::OpKind::None) {
      std::ostringstream oss;
      oss << "runtime.forward: no op at z=" << coord.z << " y=" << coord.y << " x=" << coord.x
          << " l=" << coord.l;
      return Status::Err(StatusCode::InvalidArgument, oss.str());
    }
    const TensorF32* in = &current;
    TensorF32 remote;
    if (c->is_remote_link) {
      const architecture::Coord tc{c->target_z, c->target_y, c->target_x, c->target_l};
      auto it = posts.find(tc);
      if (it == posts.end()) {
        std::ostringstream oss;
        oss << "runtime.forward: remote hop has no recorded activation → z=" << tc.z << " y=" << tc.y
            << " x=" << tc.x << " l=" << tc.l;
        return Status::Err(StatusCode::InvalidArgument, oss.str());
      }
      remote = it->second;
      in = &remote;
    }
    TensorF32 pre, post;
    if (Status st = cell(*c, *in, &pre, &post); !st) return st;
    Step step;
    step.coord = coord;
    step.input = *in;
    step.pre = std::move(pre);
    step.post = post;
    posts[coord] = post;
    current = std::move(post);
    result.steps.push_back(std::move(step));
  }
  if (result.steps.empty())
    return Status::Err(StatusCode::InvalidArgument, "runtime.forward: grid has no enabled cells with ops");
  result.output = std::move(current);
  *out = std::move(result);
  return Status::Ok();
}

}  // namespace runtime::forward
}  // namespace welvet

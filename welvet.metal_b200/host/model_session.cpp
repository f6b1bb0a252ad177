// WMN1 model sessions for models built of MHA cells (the reference's
// src/interop/model_session.cpp:319-576 with the descriptor grammar of
// include/welvet/interop/model_wire.hpp and child_wire.hpp): welvet_model_mount
// reads the descriptor — root kind, child count, four grid dimensions, the
// recursive children, the Cameral controls of the root and of every child, the
// native Store snapshots and, for a Grid root, six integers of metadata per cell —
// and mounts each MHA child as a resident B200 layer through the C++ layer API
// (welvet::mha::new_configured) with the weights of its four stores (Q, K, V, O,
// the order of the reference's store collection). welvet_model_forward runs a
// Stack root child by child and a Grid root through runtime::forward::volume_dense.
//
// The stores' FP32 payloads are encoded to the store dtype and decoded on the GPU
// (bit-exact FormatNone round trip), which equals the reference's decode of the
// snapshot's native bytes whenever those bytes are the encoding of the payload (a
// model exported at mount, as the Go side writes it). The snapshots are kept as
// read, so welvet_model_export_weights returns them unchanged (NWS1): the forward
// path does not train. The Cameral controls steer training only; they are parsed
// and not used. A Parallel root, layer kinds other than MHA and nested Stacks, and
// the training, proxy and sync entry points answer code 2.
#include <cmath>
#include <cstdlib>
#include <cstdio>
#include <cstring>
#include <functional>
#include <memory>
#include <mutex>
#include <stdexcept>
#include <string>
#include <vector>

#include "welvet/architecture.hpp"
#include "welvet/mha.hpp"
#include "welvet/runtime/forward.hpp"
#include "welvet_c.h"

using welvet::Status;
using welvet::StatusCode;
using welvet::TensorF32;

namespace {

constexpr uint32_t kWmn1 = 0x314e4d57;  // "WMN1"
constexpr uint32_t kNws1 = 0x3153574e;  // "NWS1"
constexpr int32_t kKindNone = 0, kKindMha = 7, kKindNestedStack = 19;

// An error that carries a reference status code (unsupported model parts: 2).
struct CodedError : std::runtime_error {
  int code;
  CodedError(int c, const std::string& m) : std::runtime_error(m), code(c) {}
};
void require(bool ok, const char* why) {
  if (!ok) throw std::invalid_argument(why);
}
void good(const Status& s) {
  if (!s) throw CodedError(static_cast<int>(s.code), s.message);
}

struct Reader {
  const uint8_t* p;
  size_t left;
  int depth = 0;
  template <class T> void read(T* out, size_t n) {
    require(n <= left / sizeof(T), "truncated descriptor");
    if (n) std::memcpy(out, p, n * sizeof(T));
    p += n * sizeof(T);
    left -= n * sizeof(T);
  }
  template <class T> T one() {
    T v{};
    read(&v, 1);
    return v;
  }
  template <class T> std::vector<T> vec() {
    const int32_t n = one<int32_t>();
    require(n >= 0 && size_t(n) <= left / sizeof(T), "invalid vector length");
    std::vector<T> v(n);
    read(v.data(), v.size());
    return v;
  }
  void skip_floats(int64_t n) {
    require(n >= 0 && n <= (int64_t(1) << 26) && size_t(n) <= left / 4, "invalid model payload size");
    p += n * 4;
    left -= n * 4;
  }
};

struct Writer {
  std::vector<uint8_t> data;
  template <class T> void one(T v) {
    const auto* b = reinterpret_cast<const uint8_t*>(&v);
    data.insert(data.end(), b, b + sizeof(T));
  }
  template <class T> void vec(const std::vector<T>& v) {
    one(int32_t(v.size()));
    const auto* b = reinterpret_cast<const uint8_t*>(v.data());
    if (!v.empty()) data.insert(data.end(), b, b + v.size() * sizeof(T));
  }
};

// A native WeightStore snapshot (model_session.cpp read_store / write_store).
struct Store {
  int32_t dt = 1, rows = 0, cols = 0;
  float scale = 0.f;
  std::vector<float> f32;
  std::vector<uint8_t> native;
  std::vector<double> bias;
};

struct Child {
  int32_t kind = kKindNone;
  welvet::mha::Config cfg{};
  int32_t dtype = 1;
  std::vector<Child> nested;
  Store store[4];  // MHA: Q, K, V, O
  welvet::mha::Layer layer;
};

// child_wire.hpp read_child for the kinds this library serves.
void read_child(Reader& r, Child* c) {
  require(++r.depth <= 64, "model nesting exceeds 64");
  c->kind = r.one<int32_t>();
  if (c->kind == kKindMha) {
    int32_t v[9];
    r.read(v, 9);  // seq, d_model, heads, kv heads, head_dim, msl, mask, pos, dtype
    const int32_t seq = v[0], d = v[1], heads = v[2], kv = v[3], hd_in = v[4], msl = v[5];
    require(heads > 0 && d > 0 && kv >= 0 && hd_in >= 0, "invalid model child");
    const int hd = hd_in > 0 ? hd_in : d / heads;
    const int kvh = kv > 0 ? kv : heads;
    welvet::mha::Config cfg = welvet::mha::decoder_causal(d, heads, kvh);
    cfg.max_seq_len = msl > 0 ? msl : seq;
    cfg.mask = static_cast<welvet::mha::MaskKind>(v[6]);
    cfg.pos = static_cast<welvet::mha::PosKind>(v[7]);
    if (hd_in > 0) cfg.head_dim = hd_in;
    c->cfg = cfg;
    c->dtype = v[8];
    // the child's FP32 inits (the stores that follow define the weights)
    const int64_t qd = int64_t(heads) * hd, kd = int64_t(kvh) * hd;
    r.skip_floats(qd * d);
    r.skip_floats(kd * d);
    r.skip_floats(kd * d);
    r.skip_floats(int64_t(d) * qd);
  } else if (c->kind == kKindNestedStack) {
    const int32_t n = r.one<int32_t>();
    require(n > 0 && n <= 4096, "invalid model child");
    c->nested.resize(n);
    for (auto& ch : c->nested) read_child(r, &ch);
  } else if (c->kind != kKindNone) {
    throw CodedError(2, "model child kind " + std::to_string(c->kind) +
                            " is not served by this library (MHA and nested Stack children only)");
  }
  --r.depth;
}

// model_wire.hpp read_cam_controls: training controls, consumed and not used here.
void read_controls(Reader& r) {
  int32_t n = r.one<int32_t>();
  require(n >= 0 && n <= 4096, "invalid controls");
  for (int i = 0; i < n; ++i) {
    const int32_t m = r.one<int32_t>();
    require(m >= 0 && m <= 33, "invalid controls");
  }
  n = r.one<int32_t>();
  require(n >= 0 && n <= 4096, "invalid controls");
  std::vector<double> lrs(n);
  r.read(lrs.data(), lrs.size());
  double tail[3];
  r.read(tail, 3);  // shadow_coef, surprise_thresh, last_loss
  if (!r.one<int32_t>()) return;  // no CamSync configuration
  r.one<int32_t>();               // enabled
  r.one<double>();                // alpha
  const int32_t when = r.one<int32_t>();
  require(when >= 0 && when <= 3, "invalid controls");
  n = r.one<int32_t>();
  require(n >= 0 && n <= 4096, "invalid controls");
  std::vector<double> alpha(n);
  r.read(alpha.data(), alpha.size());
  n = r.one<int32_t>();
  require(n >= 0 && n <= 4096, "invalid controls");
  for (int g = 0; g < n; ++g) {
    const int32_t cnt = r.one<int32_t>();
    require(cnt >= 0 && cnt <= 4096, "invalid controls");
    std::vector<int32_t> grp(cnt);
    r.read(grp.data(), grp.size());
  }
  n = r.one<int32_t>();
  require(n >= 0 && n <= 4096, "invalid controls");
  std::vector<int32_t> cross(6 * size_t(n));
  r.read(cross.data(), cross.size());
}
void read_cam_tree(Reader& r, Child& c) {
  read_controls(r);
  for (auto& ch : c.nested) read_cam_tree(r, ch);
}

void collect_stores(Child& c, std::vector<Store*>* out) {
  if (c.kind == kKindMha)
    for (auto& s : c.store) out->push_back(&s);
  for (auto& ch : c.nested) collect_stores(ch, out);
}

void read_store(Reader& r, Store& s, int32_t rows, int32_t cols) {
  s.dt = r.one<int32_t>();
  s.rows = r.one<int32_t>();
  s.cols = r.one<int32_t>();
  s.scale = r.one<float>();
  require(s.dt >= 0 && s.dt <= 33 && s.rows == rows && s.cols == cols && std::isfinite(s.scale),
          "native store metadata mismatch");
  s.f32 = r.vec<float>();
  s.native = r.vec<uint8_t>();
  s.bias = r.vec<double>();
  require(s.f32.size() == size_t(rows) * size_t(cols), "native store payload length mismatch");
}
void write_store(Writer& w, const Store& s) {
  w.one(s.dt);
  w.one(s.rows);
  w.one(s.cols);
  w.one(s.scale);
  w.vec(s.f32);
  w.vec(s.native);
  w.vec(s.bias);
}

// Shapes of the four dense stores of an MHA child ([out, in] as dense::new_layer).
void mha_store_shapes(const Child& c, int32_t rows[4], int32_t cols[4]) {
  welvet::mha::Config cfg = c.cfg;
  good(welvet::mha::validate(&cfg));
  const int d = cfg.d_model, qd = cfg.q_dim(), kd = cfg.kv_dim();
  const int32_t r_[4] = {qd, kd, kd, d}, c_[4] = {d, d, d, qd};
  for (int i = 0; i < 4; ++i) {
    rows[i] = r_[i];
    cols[i] = c_[i];
  }
}

void mount_children(Child& c) {
  if (c.kind == kKindMha) {
    const int32_t dt = c.store[0].dt;
    for (const auto& s : c.store)
      if (s.dt != dt)
        throw CodedError(2, "mha child with different store dtypes per projection is not served");
    good(welvet::mha::new_configured(c.cfg, static_cast<welvet::DType>(dt), c.store[0].f32.data(),
                                     c.store[1].f32.data(), c.store[2].f32.data(), c.store[3].f32.data(),
                                     &c.layer));
  }
  for (auto& ch : c.nested) mount_children(ch);
}

void flatten(Child& c, std::vector<Child*>* ops) {
  if (c.kind == kKindNestedStack) {
    for (auto& ch : c.nested) flatten(ch, ops);
  } else if (c.kind != kKindNone) {
    ops->push_back(&c);
  }
}

TensorF32 read_tensor(Reader& r) {
  TensorF32 t;
  const int32_t rank = r.one<int32_t>();
  require(rank > 0 && rank <= 5, "tensor rank must be 1..5");
  size_t n = 1;
  for (int i = 0; i < rank; ++i) {
    const int32_t d = r.one<int32_t>();
    require(d > 0 && n <= size_t(1 << 26) / size_t(d), "invalid tensor shape");
    n *= size_t(d);
    t.shape.push_back(d);
  }
  require(n <= r.left / 4, "short tensor data");
  t.data.resize(n);
  r.read(t.data.data(), n);
  return t;
}
void write_tensor(Writer& w, const TensorF32& t) {
  w.one(int32_t(t.shape.size()));
  for (auto d : t.shape) w.one(int32_t(d));
  w.vec(t.data);
}

void to_blob(Writer& w, welvet_metal_blob* out) {
  require(out != nullptr, "null output");
  out->data = nullptr;
  out->size = 0;
  void* p = std::malloc(w.data.size() ? w.data.size() : 1);
  if (!p) throw std::bad_alloc();
  if (!w.data.empty()) std::memcpy(p, w.data.data(), w.data.size());
  out->data = static_cast<uint8_t*>(p);
  out->size = w.data.size();
}

welvet_status make_status(int code, const char* msg) {
  welvet_status st{};
  st.code = code;
  if (msg) std::snprintf(st.message, sizeof(st.message), "%s", msg);
  return st;
}

template <class F> welvet_status guarded(F fn) {
  try {
    fn();
    return make_status(0, nullptr);
  } catch (const CodedError& e) {
    return make_status(e.code, e.what());
  } catch (const std::invalid_argument& e) {
    return make_status(1, e.what());
  } catch (const std::exception& e) {
    return make_status(4, e.what());
  } catch (...) {
    return make_status(4, "unknown native session failure");
  }
}

Status stack_forward(std::vector<Child>& children, const TensorF32& x, TensorF32* pre, TensorF32* post) {
  std::vector<Child*> ops;
  for (auto& c : children) flatten(c, &ops);
  if (ops.empty()) {
    *pre = x;
    *post = x;
    return Status::Ok();
  }
  TensorF32 current = x, last_pre;
  for (Child* c : ops) {
    TensorF32 p, o;
    Status st = welvet::mha::forward(c->layer, current, &p, &o);
    if (!st) return Status::Err(st.code, std::string("stack fwd: ") + st.message);
    last_pre = std::move(p);
    current = std::move(o);
  }
  *pre = std::move(last_pre);
  *post = std::move(current);
  return Status::Ok();
}

}  // namespace

struct welvet_model_session {
  int root = 0;
  std::vector<Child> children;  // Stack root
  welvet::architecture::Grid grid;  // Grid root (cells hold the mounted layers)
  std::vector<Store> grid_stores;   // Grid root: snapshots in descriptor order, for export
  std::mutex mu;
};

extern "C" {

int32_t welvet_model_abi_version(void) { return 1; }

welvet_status welvet_model_mount(const uint8_t* descriptor, size_t size, welvet_model_session** out) {
  if (out) *out = nullptr;
  return guarded([&] {
    require(out && descriptor && size >= 28 && size <= (1u << 28), "invalid mount arguments");
    Reader r{descriptor, size};
    require(r.one<uint32_t>() == kWmn1, "unsupported model descriptor version");
    auto s = std::make_unique<welvet_model_session>();
    s->root = r.one<int32_t>();
    const int32_t count = r.one<int32_t>();
    require(s->root >= 0 && s->root <= 2 && count > 0 && count <= 4096, "invalid model root/count");
    if (s->root == 1) throw CodedError(2, "Parallel model roots are not served by this library");
    int32_t dims[4];
    r.read(dims, 4);
    s->children.resize(count);
    for (auto& c : s->children) read_child(r, &c);
    read_controls(r);  // root controls
    for (auto& c : s->children) read_cam_tree(r, c);
    std::vector<Store*> stores;
    for (auto& c : s->children) collect_stores(c, &stores);
    require(r.one<int32_t>() == int32_t(stores.size()), "store count mismatch");
    // stores in collection order: four per MHA child, depth first
    {
      std::vector<Child*> mhas;
      std::function<void(Child&)> walk = [&](Child& c) {
        if (c.kind == kKindMha) mhas.push_back(&c);
        for (auto& ch : c.nested) walk(ch);
      };
      for (auto& c : s->children) walk(c);
      for (Child* m : mhas) {
        int32_t rows[4], cols[4];
        mha_store_shapes(*m, rows, cols);
        for (int i = 0; i < 4; ++i) read_store(r, m->store[i], rows[i], cols[i]);
      }
    }
    // Grid root: the cell metadata is read and checked before any layer is mounted,
    // so a malformed descriptor is rejected without device work.
    std::vector<int32_t> meta;
    if (s->root == 2) {
      int64_t n = 1;
      for (int32_t d : dims) {
        require(d > 0 && d <= 4096 && n <= 4096 / d, "invalid grid dimensions");
        n *= d;
      }
      require(n == count, "grid cell count mismatch");
      s->grid = welvet::architecture::new_grid(dims[0], dims[1], dims[2], dims[3]);
      meta.resize(6 * size_t(count));
      r.read(meta.data(), meta.size());
      for (int i = 0; i < count; ++i) {
        const int32_t* mc = meta.data() + 6 * size_t(i);
        const int kind = s->children[i].kind;
        if (kind == kKindNestedStack)
          throw CodedError(2, "nested Stack cells of a Grid root are not served by this library");
        require(!mc[0] || kind != kKindNone, "enabled grid cell has no operation");
        if (mc[1]) require(welvet::architecture::at(s->grid, mc[2], mc[3], mc[4], mc[5]) != nullptr,
                           "invalid remote link");
      }
    }
    require(r.left == 0, "trailing descriptor bytes");
    for (auto& c : s->children) mount_children(c);
    if (s->root == 2) {
      const auto hops = welvet::architecture::hop_order(s->grid);
      for (int i = 0; i < count; ++i) {
        Child& c = s->children[i];
        if (c.kind == kKindMha) {
          for (const auto& st : c.store) s->grid_stores.push_back(st);
          good(welvet::architecture::bind_mha(s->grid, hops[i].z, hops[i].y, hops[i].x, hops[i].l,
                                              std::move(c.layer)));
        }
        const int32_t* mc = meta.data() + 6 * size_t(i);
        auto& cell = s->grid.cells[i];
        cell.meta.is_disabled = mc[0] == 0;
        cell.is_remote_link = mc[1] != 0;
        cell.target_z = mc[2];
        cell.target_y = mc[3];
        cell.target_x = mc[4];
        cell.target_l = mc[5];
      }
      s->children.clear();
    }
    *out = s.release();
  });
}

welvet_status welvet_model_forward(welvet_model_session* s, const uint8_t* input, size_t size,
                                   welvet_metal_blob* out) {
  return guarded([&] {
    require(s && input && out, "invalid forward arguments");
    std::lock_guard<std::mutex> lock(s->mu);
    Reader r{input, size};
    TensorF32 x = read_tensor(r);
    require(r.left == 0, "trailing descriptor bytes");
    TensorF32 post;
    if (s->root == 0) {
      TensorF32 pre;
      good(stack_forward(s->children, x, &pre, &post));
    } else {
      welvet::runtime::forward::Result res;
      good(welvet::runtime::forward::volume_dense(s->grid, x, &res));
      post = std::move(res.output);
    }
    Writer w;
    write_tensor(w, post);
    to_blob(w, out);
  });
}

welvet_status welvet_model_forward_pair(welvet_model_session* s, const uint8_t* data, size_t size,
                                        welvet_metal_blob* out) {
  return guarded([&] {
    require(s && data && out, "invalid segment forward arguments");
    std::lock_guard<std::mutex> lock(s->mu);
    require(s->root != 2, "segment forward expects Stack or Parallel");
    Reader r{data, size};
    TensorF32 x = read_tensor(r);
    require(r.left == 0, "trailing descriptor bytes");
    TensorF32 pre, post;
    good(stack_forward(s->children, x, &pre, &post));
    Writer w;
    write_tensor(w, pre);
    write_tensor(w, post);
    to_blob(w, out);
  });
}

welvet_status welvet_model_export_weights(welvet_model_session* s, welvet_metal_blob* out) {
  return guarded([&] {
    require(s && out, "invalid export arguments");
    std::lock_guard<std::mutex> lock(s->mu);
    std::vector<Store*> stores;
    if (s->root == 2) {
      for (auto& st : s->grid_stores) stores.push_back(&st);
    } else {
      for (auto& c : s->children) collect_stores(c, &stores);
    }
    Writer w;
    w.one(kNws1);
    w.one(int32_t(stores.size()));
    for (Store* st : stores) write_store(w, *st);
    w.one(int32_t(0));  // no Mamba / GDN records
    to_blob(w, out);
  });
}

welvet_status welvet_model_train_credit(welvet_model_session*, int32_t, double, const uint8_t*, size_t) {
  return make_status(2, "model training is not served by this library (forward path)");
}
welvet_status welvet_model_dense_proxy(welvet_model_session*, int32_t, const uint8_t*, size_t,
                                       welvet_metal_blob* out) {
  if (out) *out = welvet_metal_blob{nullptr, 0};
  return make_status(2, "dense proxy is not served by this library (MHA models only)");
}
welvet_status welvet_model_backward(welvet_model_session*, const uint8_t*, size_t, welvet_metal_blob* out) {
  if (out) *out = welvet_metal_blob{nullptr, 0};
  return make_status(2, "model backward is not served by this library (forward path)");
}
welvet_status welvet_model_apply_sgd(welvet_model_session*, double, const uint8_t*, size_t) {
  return make_status(2, "model SGD is not served by this library (forward path)");
}
welvet_status welvet_model_train_mse(welvet_model_session*, int32_t, double, int32_t, const uint8_t*, size_t,
                                     double* loss) {
  if (loss) *loss = 0.0;
  return make_status(2, "model training is not served by this library (forward path)");
}
welvet_status welvet_model_sync(welvet_model_session*, int32_t) {
  return make_status(2, "CamSync is not served by this library (forward path)");
}

void welvet_model_release(welvet_model_session* s) { delete s; }

void welvet_metal_blob_free(welvet_metal_blob* b) {
  if (b) {
    std::free(b->data);
    b->data = nullptr;
    b->size = 0;
  }
}

}  // extern "C"

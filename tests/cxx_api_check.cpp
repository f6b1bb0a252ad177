// Host-side checks of the C++ layer / volume API (include/welvet/*.hpp) that need
// no GPU: the reference's validate() defaults and messages, the grid's hop order,
// coordinates and remote links, and the status answers of volume_dense and
// mha::forward before any device work. Built and run by tests/test_wire_tool.py;
// prints "ok" and exits 0, or prints the failed check and exits 1.
#include <cstdio>
#include <string>

#include "welvet/architecture.hpp"
#include "welvet/mha.hpp"
#include "welvet/runtime/forward.hpp"

#define CHECK(cond)                                              \
  do {                                                           \
    if (!(cond)) {                                               \
      std::printf("FAILED %s:%d %s\n", __FILE__, __LINE__, #cond); \
      return 1;                                                  \
    }                                                            \
  } while (0)

int main() {
  using namespace welvet;
  // validate(): defaults of src/layers/mha/mha.cpp:63-94
  mha::Config c = mha::decoder_causal(64, 4, 0);
  CHECK(mha::validate(&c).ok());
  CHECK(c.head_dim == 16 && c.num_kv_heads == 4 && c.max_seq_len == 512 && c.rope_theta == 10000.0);
  CHECK(c.mask == mha::MaskKind::Causal && c.causal && c.uses_rope() && !c.uses_alibi());
  CHECK(c.q_dim() == 64 && c.kv_dim() == 64 && c.heads_per_kv() == 1);
  CHECK(c.scale() == 0.25);
  mha::Config bad;
  Status st = mha::validate(&bad);
  CHECK(st.code == StatusCode::InvalidArgument && st.message == "mha: need DModel>0 and NumHeads>0");
  bad.d_model = 10;
  bad.num_heads = 3;
  st = mha::validate(&bad);
  CHECK(st.message == "mha: HeadDim unset and DModel%NumHeads!=0");
  bad.d_model = 12;
  bad.num_kv_heads = 2;
  st = mha::validate(&bad);
  CHECK(st.message == "mha: NumHeads not divisible by NumKVHeads");
  CHECK(mha::validate(nullptr).message == "mha: nil config");
  mha::Config un;
  un.d_model = 8;
  un.num_heads = 2;
  un.mask = mha::MaskKind::Unspecified;
  un.causal = false;
  CHECK(mha::validate(&un).ok() && un.mask == mha::MaskKind::Causal && un.causal);

  // grid: clamps, hop order z -> y -> x -> l, coordinates, links
  architecture::Grid g = architecture::new_grid(0, 2, 1, 2);
  CHECK(g.depth == 1 && g.rows == 2 && g.cols == 1 && g.layers_per_cell == 2 && g.cells.size() == 4);
  auto hops = architecture::hop_order(g);
  CHECK(hops.size() == 4 && hops[1] == (architecture::Coord{0, 0, 0, 1}) && hops[2] == (architecture::Coord{0, 1, 0, 0}));
  CHECK(architecture::index(g, 0, 1, 0, 1) == 3 && architecture::at(g, 0, 2, 0, 0) == nullptr);
  st = architecture::set_remote_link(g, 0, 1, 0, 0, 0, 0, 0, 1);
  CHECK(st.ok() && architecture::at(g, 0, 1, 0, 0)->is_remote_link);
  st = architecture::set_remote_link(g, 0, 0, 0, 0, 0, 5, 0, 0);
  CHECK(st.code == StatusCode::InvalidArgument && st.message == "architecture: bad target coord z=0 y=5 x=0 l=0");
  st = architecture::bind_mha(g, 1, 0, 0, 0, mha::Layer{});
  CHECK(st.message == "architecture: bad bind coord z=1 y=0 x=0 l=0");

  // volume_dense before any device work
  runtime::forward::Result res;
  TensorF32 x;
  st = runtime::forward::volume_dense(g, x, &res);
  CHECK(st.message == "runtime.forward: empty input");
  x.shape = {1, 2, 64};
  x.data.assign(128, 0.5f);
  st = runtime::forward::volume_dense(g, x, nullptr);
  CHECK(st.message == "runtime.forward: nil result");
  st = runtime::forward::volume_dense(g, x, &res);
  CHECK(st.message == "runtime.forward: no op at z=0 y=0 x=0 l=0");
  for (auto& cell : g.cells) cell.meta.is_disabled = true;
  st = runtime::forward::volume_dense(g, x, &res);
  CHECK(st.message == "runtime.forward: grid has no enabled cells with ops");

  // mha::forward argument answers (no mounted weights needed)
  mha::Layer layer;
  layer.cfg = mha::decoder_causal(64, 4, 0);
  TensorF32 pre, post;
  CHECK(mha::forward(layer, x, nullptr, &post).message == "mha: nil pre/post");
  layer.cfg.mode = mha::AttnMode::Cross;
  st = mha::forward(layer, x, &pre, &post);
  CHECK(st.code == StatusCode::Gap && st.message == "gap? mha forward: ModeCross not in baseline");
  layer.cfg.mode = mha::AttnMode::Self;
  CHECK(mha::forward(layer, x, &pre, &post).code == StatusCode::InvalidArgument);  // not mounted
  std::printf("ok\n");
  return 0;
}

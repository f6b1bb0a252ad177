#pragma once
// Single-cell volume API of the MHA path (reference include/welvet/architecture.hpp:
// Coord, OpKind, Cell, Grid, new_grid, index, at, hop_order, set_remote_link,
// bind_mha; src/architecture/grid.cpp). Same names, enum values and hop order
// (z, then y, then x, then l). A cell here holds an MHA layer or nothing: the other
// layer families of the reference's grid are not part of this library, and
// runtime::forward::cell answers code 3 (gap) for them.
#include <cstdint>
#include <vector>

#include "welvet/dtype.hpp"
#include "welvet/export.hpp"
#include "welvet/mha.hpp"
#include "welvet/status.hpp"

namespace welvet {

// Layer type ids (reference include/welvet/layer.hpp:10-34).
enum class LayerType : int32_t {
  Dense = 0, MultiHeadAttention = 1, SwiGLU = 2, RMSNorm = 3, CNN1 = 4, CNN2 = 5, CNN3 = 6, RNN = 7,
  LSTM = 8, LayerNorm = 9, ConvTransposed1D = 10, ConvTransposed2D = 11, ConvTransposed3D = 12,
  Embedding = 13, KMeans = 14, Softmax = 15, Parallel = 16, Sequential = 17, Residual = 18,
  Metacognition = 19, Mamba = 20, GDN = 21, Stack = 22,
};

struct LayerMeta {
  LayerType type = LayerType::Dense;
  DType dtype = DType::Float32;
  int input_height = 0;
  int output_height = 0;
  int z = 0, y = 0, x = 0, l = 0;
  bool is_disabled = false;
};

}  // namespace welvet

namespace welvet::architecture {

struct Coord {
  int z = 0, y = 0, x = 0, l = 0;
  bool operator==(const Coord& o) const { return z == o.z && y == o.y && x == o.x && l == o.l; }
};

enum class OpKind : int32_t {
  None = 0, Dense = 1, RMSNorm = 2, LayerNorm = 3, SwiGLU = 4, Softmax = 5, Embedding = 6, MHA = 7,
  CNN1 = 8, CNN2 = 9, CNN3 = 10, ConvT1 = 11, ConvT2 = 12, ConvT3 = 13, RNN = 14, LSTM = 15,
  Sequential = 16, Residual = 17, Mamba = 18, Stack = 19, Metacognition = 20, GDN = 21, KMeans = 22,
  Parallel = 23,
};

struct Cell {
  LayerMeta meta{};
  OpKind op_kind = OpKind::None;
  mha::Layer mha_op;

  bool is_remote_link = false;
  int target_z = 0, target_y = 0, target_x = 0, target_l = 0;
};

struct Grid {
  int depth = 1;
  int rows = 1;
  int cols = 1;
  int layers_per_cell = 1;
  std::vector<Cell> cells;
};

WELVET_CXX_API Grid new_grid(int depth, int rows, int cols, int layers_per_cell);
WELVET_CXX_API int index(const Grid& g, int z, int y, int x, int l);
WELVET_CXX_API Cell* at(Grid& g, int z, int y, int x, int l);
WELVET_CXX_API const Cell* at(const Grid& g, int z, int y, int x, int l);
inline int stack_layer_count(const Grid& g) { return g.depth * g.rows * g.cols * g.layers_per_cell; }
WELVET_CXX_API std::vector<Coord> hop_order(const Grid& g);
WELVET_CXX_API Status set_remote_link(Grid& g, int z, int y, int x, int l, int tz, int ty, int tx, int tl);
WELVET_CXX_API Status bind_mha(Grid& g, int z, int y, int x, int l, mha::Layer op);

}  // namespace welvet::architecture

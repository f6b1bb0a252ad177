#pragma once
// Volume forward over a grid of MHA cells (reference include/welvet/runtime/
// forward.hpp:10-24, src/runtime/forward.cpp:21-132): cells run in hop order,
// each cell's input is the previous cell's post (or, for a remote-link cell, the
// recorded post of its target), and the result keeps every step.
#include <vector>

#include "welvet/architecture.hpp"
#include "welvet/export.hpp"
#include "welvet/status.hpp"
#include "welvet/tensor.hpp"

namespace welvet::runtime::forward {

struct Step {
  architecture::Coord coord;
  TensorF32 input;
  TensorF32 pre;
  TensorF32 post;
};

struct Result {
  TensorF32 output;
  std::vector<Step> steps;
};

WELVET_CXX_API Status cell(architecture::Cell& cell, const TensorF32& in, TensorF32* pre, TensorF32* post);
WELVET_CXX_API Status volume_dense(architecture::Grid& g, const TensorF32& input, Result* out);

}  // namespace welvet::runtime::forward

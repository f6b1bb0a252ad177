#pragma once
// Host FP32 tensor of the C++ API (reference include/welvet/tensor.hpp:8-14).
#include <cstddef>
#include <cstdint>
#include <vector>

#include "welvet/export.hpp"

namespace welvet {

struct TensorF32 {
  std::vector<int64_t> shape;
  std::vector<float> data;

  WELVET_CXX_API static TensorF32 zeros(int64_t a, int64_t b);
  std::size_t numel() const { return data.size(); }
};

}  // namespace welvet

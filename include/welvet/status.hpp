#pragma once
// welvet::Status of the C++ API (reference include/welvet/status.hpp:8-30): the same
// codes as welvet_status in welvet_c.h — 0 ok, 1 invalid argument, 2 unsupported,
// 3 gap, 4 internal (CUDA / NCCL / device-side error).
#include <string>
#include <string_view>

namespace welvet {

enum class StatusCode { Ok = 0, InvalidArgument = 1, Unsupported = 2, Gap = 3, Internal = 4 };

struct Status {
  StatusCode code = StatusCode::Ok;
  std::string message;

  static Status Ok() { return {}; }
  static Status Err(StatusCode c, std::string_view msg) { return Status{c, std::string(msg)}; }
  static Status Gap(std::string_view what) { return Err(StatusCode::Gap, std::string("gap? ") + std::string(what)); }

  explicit operator bool() const { return code == StatusCode::Ok; }
  bool ok() const { return code == StatusCode::Ok; }
};

}  // namespace welvet

// Stand-in for <c10/util/Exception.h> used only when the reference's
// csrc/jit/Jit.cpp is compiled into the oracle library: TORCH_CHECK throws
// std::runtime_error so the reference's own checks still fire, without
// linking libc10.  Test infrastructure only.
#pragma once

#include <sstream>
#include <stdexcept>
#include <string>

namespace tvr_ref_shim {
inline void append(std::ostringstream&) {}
template <typename T, typename... Rest>
void append(std::ostringstream& o, const T& v, const Rest&... rest) {
  o << v;
  append(o, rest...);
}
template <typename... Args>
std::string message(const Args&... args) {
  std::ostringstream o;
  append(o, args...);
  return o.str();
}
}  // namespace tvr_ref_shim

#define TORCH_CHECK(cond, ...)                                                        \
  do {                                                                                \
    if (!(cond)) {                                                                    \
      throw std::runtime_error(::tvr_ref_shim::message("check failed: " #cond " ", \
                                                       ##__VA_ARGS__));               \
    }                                                                                 \
  } while (0)

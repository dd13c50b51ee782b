// Integer division by a divisor fixed for a launch, for the index arithmetic
// of the N-d elementwise, copy and selection kernels.
#pragma once

#include <cuda_runtime.h>

#include <cstdint>

namespace tvr {

// Division of n < 2^31 by a divisor d fixed for the launch, by multiplication:
// the round-up method of Granlund and Montgomery ("Division by Invariant
// Integers using Multiplication", PLDI 1994, section 4) with N = 32,
// l = ceil(log2 d), m = floor(2^32 (2^l - d) / d) + 1, q = (umulhi(n, m) + n) >> l.
// Exact for all n < 2^32 and 1 <= d < 2^31; a 64-bit divide per dimension
// per element otherwise dominates the index arithmetic of the N-d kernels.
struct FastDiv {
  uint32_t d = 1, m = 1, l = 0;
};

inline FastDiv make_fastdiv(uint32_t d) {
  FastDiv f;
  f.d = d;
  f.l = 0;
  while ((uint64_t(1) << f.l) < d) ++f.l;
  f.m = static_cast<uint32_t>((uint64_t(1) << 32) * ((uint64_t(1) << f.l) - d) / d + 1);
  return f;
}

__device__ __forceinline__ uint32_t fast_div(uint32_t n, const FastDiv& f) {
  return static_cast<uint32_t>((static_cast<uint64_t>(__umulhi(n, f.m)) + n) >> f.l);
}

}  // namespace tvr

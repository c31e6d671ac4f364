// Drop-in replacement for CAIRN's runtime/cairn_tensor.hpp on a B200 (sm_100a): the `mma_unordered` multiply that
// compiler/device/tensor.py:69-82 lowers to. c (row-major m x n, f32) += a (row-major m x k) * b (row-major k x n),
// a and b one storage float (f16, bf16, f8e4m3 or f8e5m2).
//
// Host programs keep the reference's host semantics exactly, since the host multiply is its own reference
// (runtime/cairn_tensor.hpp:26-41): for every output its old value, then its k products added in increasing p, each
// product and each sum rounded to f32. Device programs call libcairn_b200.so's tcgen05 multiply
// (cairn_b200_mma_<format>, include/cairn_b200.h) on the calling thread's synchronous lane instead of the WMMA tile
// kernel; the contract is unchanged (every product exact in f32, every output within (k + 1) * 2^-22 * (|c| +
// sum |a * b|) of the exact sum), and a violated guard traps as before. Link with -lcairn_b200.
#pragma once
#include <cstddef>
#include <cstdint>
#include <type_traits>
#include "cairn_float.hpp"

namespace cr::tensor {

// The call's extents against its views: c holds m * n, a holds m * k and b holds k * n elements, or the call traps.
inline void shape(std::size_t m, std::size_t n, std::size_t k, std::size_t c, std::size_t a, std::size_t b) noexcept {
  if(cr::mul<std::size_t>(m, n) != c || cr::mul<std::size_t>(m, k) != a || cr::mul<std::size_t>(k, n) != b) trap();
}

// The host multiply, in the reference's order: row by row, each a[i][p] widened once and its products with row p of
// b added across the row of c, so every output sees its products in increasing p after its old value.
template<class A> inline void reference(std::size_t m, std::size_t n, std::size_t k, float* c, const A* a,
                                        const A* b) noexcept {
  for(std::size_t i = 0; i < m; ++i) {
    float* row = c + i * n;
    for(std::size_t p = 0; p < k; ++p) {
      const float x = static_cast<float>(a[i * k + p]);
      const A* brow = b + p * n;
      for(std::size_t j = 0; j < n; ++j) row[j] = row[j] + x * static_cast<float>(brow[j]);
    }
  }
}

template<class A> inline void multiply(std::size_t m, std::size_t n, std::size_t k, float* c, std::size_t cn,
                                       const A* a, std::size_t an, const A* b, std::size_t bn) noexcept {
  shape(m, n, k, cn, an, bn);
  reference(m, n, k, c, a, b);
}

}  // namespace cr::tensor

#if defined(__CUDACC__)
#include "../../cairn_b200.h"
#include "cairn_gpu.hpp"

namespace cr::tensor {

// The storage float's entry in libcairn_b200.so.
template<class A> inline int b200_multiply(cudaStream_t s, std::size_t m, std::size_t n, std::size_t k, float* c,
                                           std::size_t cn, const A* a, std::size_t an, const A* b,
                                           std::size_t bn) noexcept {
  if constexpr(std::is_same_v<A, cr::bf16>)
    return cairn_b200_mma_bf16(s, m, n, k, c, cn, reinterpret_cast<const std::uint16_t*>(a), an,
                               reinterpret_cast<const std::uint16_t*>(b), bn);
  else if constexpr(std::is_same_v<A, cr::f16>)
    return cairn_b200_mma_f16(s, m, n, k, c, cn, reinterpret_cast<const std::uint16_t*>(a), an,
                              reinterpret_cast<const std::uint16_t*>(b), bn);
  else if constexpr(std::is_same_v<A, cr::f8e4m3>)
    return cairn_b200_mma_f8e4m3(s, m, n, k, c, cn, reinterpret_cast<const std::uint8_t*>(a), an,
                                 reinterpret_cast<const std::uint8_t*>(b), bn);
  else if constexpr(std::is_same_v<A, cr::f8e5m2>)
    return cairn_b200_mma_f8e5m2(s, m, n, k, c, cn, reinterpret_cast<const std::uint8_t*>(a), an,
                                 reinterpret_cast<const std::uint8_t*>(b), bn);
  else
    static_assert(sizeof(A) == 0, "mma_unordered takes f16, bf16, f8e4m3 or f8e5m2 operands");
}

// On the calling thread's execution context: the product runs on its synchronous lane, and the call returns once
// that lane has run it (or at the end of a held run), never by waiting for the whole device.
template<class A> inline void launch(gpu::Context& ctx, std::size_t m, std::size_t n, std::size_t k, float* c,
                                     std::size_t cn, const A* a, std::size_t an, const A* b, std::size_t bn) noexcept {
  shape(m, n, k, cn, an, bn);
  if(!m || !n) return;
  reuse::synchronous(ctx, [&](cudaStream_t s) {
    if(b200_multiply<A>(s, m, n, k, c, cn, a, an, b, bn) != CAIRN_B200_OK) trap();
  });
}

}  // namespace cr::tensor
#endif

// TEST INFRASTRUCTURE ONLY: C entry points over the CAIRN reference's own host path, compiled from the reference's
// header-only runtime where it lies (oracle/Makefile names the include directory). Nothing here restates an
// algorithm: each entry calls the reference's template exactly as the code cairnc emits for the matching CAIRN
// function calls it. The parity tests use it to pin oracle/cairn_oracle.c and to write tests/golden/, and bench.py's
// reference arm times it on the host cores. The cairn_b200 package never loads it.
//
//   ref_mma_<fmt>        cr::tensor::multiply<A> (runtime/cairn_tensor.hpp:37-41): the host lowering of
//                        mma_unordered (compiler/device/tensor.py:69-82), single-threaded.
//   ref_mma_bf16_pooled  the same reference loop, one lane per row of c on the reference's lane pool
//                        (cr::par::run, runtime/cairn_parallel.hpp:372-378): what a CAIRN program that splits a
//                        host multiply by rows runs, and the all-cores CPU baseline of the GEMM bench.
//   ref_gemm_f32_region  `parallel e in m*n { c[e] = c[e] + sum over p in order }` on the lane pool: the host
//                        f32 GEMM of BASELINE config 1 (mma_unordered refuses f32, compiler/device/tensor.py:49-50).
//   ref_sum_f32/_f64     cr::par::sum (runtime/cairn_sum.hpp:311-331): `reduce + parallel` over floats.
//   ref_sum_u64          cr::par::reduce (runtime/cairn_parallel.hpp:385-399) over cr::Sum<u64>
//                        (runtime/cairn_runtime.hpp:158-166): the checked sum, with its overflow flag returned
//                        instead of trapping.
//   ref_saxpy_f32        cr::par::run of out[i] = a * x[i] + y[i].
//   ref_scan_u32         cr::par::scan<false> (runtime/cairn_parallel.hpp:401-440) of `scan add_wrap parallel i
//                        in n yield x[i]` over u32: inclusive prefixes modulo 2^32, returning the total.
//   ref_runmax_i32       cr::par::scan<true> of `scan exclusive max` over i32 from the identity INT32_MIN.
//   ref_narrow_*/ref_widen_*  cr::fp::narrow and the storage floats' exact widening (runtime/cairn_float.hpp).
#include <cstddef>
#include <cstdint>
#include "cairn_tensor.hpp"
#include "cairn_sum.hpp"

namespace {
template<class A, class B> void mma(std::size_t m, std::size_t n, std::size_t k, float* c, const B* a, const B* b) {
  static_assert(sizeof(A) == sizeof(B));
  cr::tensor::multiply<A>(m, n, k, c, m * n, reinterpret_cast<const A*>(a), m * k, reinterpret_cast<const A*>(b),
                          k * n);
}
}  // namespace

extern "C" {

void ref_mma_bf16(std::size_t m, std::size_t n, std::size_t k, float* c, const std::uint16_t* a,
                  const std::uint16_t* b) { mma<cr::bf16>(m, n, k, c, a, b); }
void ref_mma_f16(std::size_t m, std::size_t n, std::size_t k, float* c, const std::uint16_t* a,
                 const std::uint16_t* b) { mma<cr::f16>(m, n, k, c, a, b); }
void ref_mma_f8e4m3(std::size_t m, std::size_t n, std::size_t k, float* c, const std::uint8_t* a,
                    const std::uint8_t* b) { mma<cr::f8e4m3>(m, n, k, c, a, b); }
void ref_mma_f8e5m2(std::size_t m, std::size_t n, std::size_t k, float* c, const std::uint8_t* a,
                    const std::uint8_t* b) { mma<cr::f8e5m2>(m, n, k, c, a, b); }

void ref_mma_bf16_pooled(std::size_t m, std::size_t n, std::size_t k, float* c, const std::uint16_t* a,
                         const std::uint16_t* b) {
  const auto* A = reinterpret_cast<const cr::bf16*>(a);
  const auto* B = reinterpret_cast<const cr::bf16*>(b);
  cr::par::run(m, [&](std::size_t i) noexcept { cr::tensor::reference<cr::bf16>(1, n, k, c + i * n, A + i * k, B); },
               n * k + 1);
}

void ref_gemm_f32_region(std::size_t m, std::size_t n, std::size_t k, float* c, const float* a, const float* b) {
  cr::par::run(m * n, [&](std::size_t e) noexcept {
    const std::size_t i = e / n, j = e % n;
    float acc = c[e];
    for(std::size_t p = 0; p < k; ++p) acc = acc + a[i * k + p] * b[p * n + j];
    c[e] = acc;
  }, k + 1);
}

float ref_sum_f32(std::size_t n, const float* x) {
  return cr::par::sum<float>(n, [x](std::size_t i) noexcept { return x[i]; });
}
double ref_sum_f64(std::size_t n, const double* x) {
  return cr::par::sum<double>(n, [x](std::size_t i) noexcept { return x[i]; });
}

std::uint64_t ref_sum_u64(std::size_t n, const std::uint64_t* x, int* overflow) {
  using S = cr::Sum<std::uint64_t>;
  const S total = cr::par::reduce<S>(n, S{}, [](S p, S q) noexcept { return p + q; },
                                     [x](std::size_t i) noexcept { return S(x[i]); });
  *overflow = total.over ? 1 : 0;
  return total.v;
}

void ref_saxpy_f32(std::size_t n, float* out, const float* x, const float* y, float a) {
  cr::par::run(n, [=](std::size_t i) noexcept { out[i] = a * x[i] + y[i]; });
}

std::uint32_t ref_scan_u32(std::size_t n, std::uint32_t* out, const std::uint32_t* x) {
  return cr::par::scan<false, std::uint32_t>(
      out, n, 0u, [](std::uint32_t p, std::uint32_t q) noexcept { return cr::add_wrap(p, q); },
      [x](std::size_t i) noexcept { return x[i]; });
}
std::int32_t ref_runmax_i32(std::size_t n, std::int32_t* out, const std::int32_t* x) {
  return cr::par::scan<true, std::int32_t>(
      out, n, std::int32_t(-2147483647 - 1), [](std::int32_t p, std::int32_t q) noexcept { return p < q ? q : p; },
      [x](std::size_t i) noexcept { return x[i]; });
}

std::uint16_t ref_narrow_bf16(double x) { return cr::fp::narrow<cr::bf16>(x).bits; }
std::uint16_t ref_narrow_f16(double x) { return cr::fp::narrow<cr::f16>(x).bits; }
float ref_widen_bf16(std::uint16_t b) { return static_cast<float>(cr::bf16{b}); }
float ref_widen_f16(std::uint16_t b) { return static_cast<float>(cr::f16{b}); }
float ref_widen_f8e4m3(std::uint8_t b) { return static_cast<float>(cr::f8e4m3{b}); }
float ref_widen_f8e5m2(std::uint8_t b) { return static_cast<float>(cr::f8e5m2{b}); }

// How many lanes the reference's pool runs (CAIRN_LANES, else the hardware's thread count).
std::size_t ref_lanes() { return cr::par::lanes::shared().lanes(); }

}  // extern "C"

// A CAIRN device library in the form cairnc emits it (compiler/lower/codegen.py:438-446 for the checked cf_ entries,
// compiler/lower/header.py:230-247 for the enqueued cq_ entries, compiler/lower/region_lowering.py:122-183 and
// compiler/device/tensor.py:69-82 for the bodies): every function's body calls only the runtime's templates,
// cr::gpu::run, cr::gpu::run_vector, cr::gpu::run_staged, cr::gpu::reduce_on, cr::gpu::scan_on, cr::gpu::compact_on and cr::tensor::launch. It is built against the CAIRN
// runtime headers with include/cairn_b200/runtime ahead of them on the include path (tests/dropin/build_emitted.py),
// so the same source runs on the B200 machine and libcairn_b200.so. Test input of tests/test_dropin_gpu.py. Built
// over the reference's headers alone, the same source runs the reference's own CUDA machine (its lane kernels, CUB
// collectors and WMMA multiply): the reference-on-B200 baseline bench.py times beside this project's kernels.
#include <cstddef>
#include <cstdint>
#include "cairn_runtime.hpp"
#include "cairn_float.hpp"
#include "cairn_gpu.hpp"
#include "cairn_cub.hpp"
#include "cairn_tensor.hpp"

namespace {
using Sum64 = cr::Sum<std::uint64_t>;

// pub fn saxpy(n, out: rw<f32>[n]@device, x: ro<f32>[n]@device, y: ro<f32>[n]@device, a: f32)
//   { parallel i in n { out[i] = a * x[i] + y[i]; } }
void ci_saxpy(std::size_t n, float* out, const float* x, const float* y, float a) {
  cr::gpu::run(cr::gpu::here(), n, [=] CR_DEVICE(std::size_t i) { out[i] = (a * x[i]) + y[i]; });
}
// the same region with `plan saxpy4 { vector 4; }`
void ci_saxpy4(std::size_t n, float* out, const float* x, const float* y, float a) {
  cr::gpu::run_vector<4>(
      cr::gpu::here(), n, cr::gpu::aligned<4>(out, x, y),
      [=] CR_DEVICE(std::size_t i) { out[i] = (a * x[i]) + y[i]; },
      [=] CR_DEVICE(std::size_t i) {
        const auto xv = cr::gpu::Chunk<float, 4>::load(x + i);
        const auto yv = cr::gpu::Chunk<float, 4>::load(y + i);
        cr::gpu::Chunk<float, 4> o;
        for(unsigned q = 0; q < 4; ++q) o[q] = (a * xv.v[q]) + yv.v[q];
        o.store(out + i);
      });
}
// pub fn dsum(n, x: ro<f32>[n]@device) -> f32 { let s = reduce + parallel i in n yield x[i]; return s; }
float ci_dsum(std::size_t n, const float* x) {
  return cr::gpu::reduce_on<float>(
      cr::gpu::here(), n, 0.0f, [] CR_DEVICE(float p, float q) { return static_cast<float>(p + q); },
      [=] CR_DEVICE(std::size_t i) { return x[i]; });
}
// pub fn usum(n, x: ro<u64>[n]@device) -> u64 { let s = reduce + parallel i in n yield x[i]; return s; }
std::uint64_t ci_usum(std::size_t n, const std::uint64_t* x) {
  return cr::gpu::reduce_on<Sum64>(
             cr::gpu::here(), n, Sum64{}, [] CR_DEVICE(Sum64 p, Sum64 q) { return p + q; },
             [=] CR_DEVICE(std::size_t i) { return Sum64(x[i]); })
      .checked();
}
// pub fn vmax(n, x: ro<i32>[n]@device) -> i32 { let s = reduce max parallel i in n yield x[i]; return s; }
std::int32_t ci_vmax(std::size_t n, const std::int32_t* x) {
  return cr::gpu::reduce_on<std::int32_t>(
      cr::gpu::here(), n, std::int32_t(-2147483647 - 1),
      [] CR_DEVICE(std::int32_t p, std::int32_t q) { return p < q ? q : p; },
      [=] CR_DEVICE(std::size_t i) { return x[i]; });
}
// pub fn gemm(m, n, k, c: rw<f32>[cn]@device, a: ro<bf16>[an]@device, b: ro<bf16>[bn]@device)
//   { mma_unordered(m, n, k, c, a, b); }
void ci_gemm(std::size_t m, std::size_t n, std::size_t k, float* c, std::size_t cn, const cr::bf16* a,
             std::size_t an, const cr::bf16* b, std::size_t bn) {
  cr::tensor::launch<cr::bf16>(cr::gpu::here(), m, n, k, c, cn, a, an, b, bn);
}
// pub fn prefix(n, out: rw<u64>[n]@device, x: ro<u64>[n]@device) -> u64
//   { let s = scan + parallel i in n yield x[i] into out; return s; }
std::uint64_t ci_prefix(std::size_t n, std::uint64_t* out, const std::uint64_t* x) {
  return cr::gpu::scan_on<false, Sum64>(
             cr::gpu::here(), out, n, Sum64{}, [] CR_DEVICE(Sum64 p, Sum64 q) { return p + q; },
             [=] CR_DEVICE(std::size_t i) { return Sum64(x[i]); })
      .checked();
}
// pub fn wprefix(n, out: rw<u32>[n]@device, x: ro<u32>[n]@device) -> u32
//   { let s = scan add_wrap parallel i in n yield x[i] into out; return s; }
std::uint32_t ci_wprefix(std::size_t n, std::uint32_t* out, const std::uint32_t* x) {
  return cr::gpu::scan_on<false, std::uint32_t>(
      cr::gpu::here(), out, n, 0u, [] CR_DEVICE(std::uint32_t p, std::uint32_t q) { return cr::add_wrap(p, q); },
      [=] CR_DEVICE(std::size_t i) { return x[i]; });
}
// pub fn runmax(n, out: rw<i32>[n]@device, x: ro<i32>[n]@device) -> i32
//   { let s = scan exclusive max parallel i in n yield x[i] into out; return s; }
std::int32_t ci_runmax(std::size_t n, std::int32_t* out, const std::int32_t* x) {
  return cr::gpu::scan_on<true, std::int32_t>(
      cr::gpu::here(), out, n, std::int32_t(-2147483647 - 1),
      [] CR_DEVICE(std::int32_t p, std::int32_t q) { return p < q ? q : p; },
      [=] CR_DEVICE(std::size_t i) { return x[i]; });
}
// pub fn fprefix(n, out: rw<f32>[n]@device, x: ro<f32>[n]@device) -> f32
//   { let s = scan + parallel i in n yield x[i] into out; return s; }
float ci_fprefix(std::size_t n, float* out, const float* x) {
  return cr::gpu::scan_on<false, float>(
      cr::gpu::here(), out, n, 0.0f, [] CR_DEVICE(float p, float q) { return static_cast<float>(p + q); },
      [=] CR_DEVICE(std::size_t i) { return x[i]; });
}
// pub fn positives(n, out: rw<f32>[n]@device, x: ro<f32>[n]@device) -> usize
//   { return compact parallel i in n where x[i] > 0.0 yield x[i] into out; }
std::size_t ci_positives(std::size_t n, float* out, const float* x) {
  return cr::gpu::compact_on(
      cr::gpu::here(), out, n, [=] CR_DEVICE(std::size_t i) { return x[i] > 0.0f; },
      [=] CR_DEVICE(std::size_t i) { return x[i]; });
}
// fn blur(n: usize, out: rw<f32>[n]@device, x: ro<f32>[n]@device) {
//   parallel i in n {
//     if i >= 2 && i + 2 < n { out[i] = x[i - 2] + x[i - 1] * 2.0 + x[i] * 3.0 + x[i + 1] + x[i + 2]; }
//     else { out[i] = x[i]; }
//   }
// }
// plan blur { stage 2; block 128; }   (compiler/plans/staging.py:95-122 emits the three lambdas this way)
void ci_blur(std::size_t n, float* out, const float* x) {
  cr::gpu::run_staged<2>(
      cr::gpu::here(), n,
      [=] CR_DEVICE(std::size_t cr_base, std::size_t cr_w, std::size_t cr_t, std::size_t cr_b,
                    unsigned char* cr_shared) {
        float* const cr_s_x = reinterpret_cast<float*>(cr_shared + 0);
        for(std::size_t cr_e = cr_t; cr_e < cr_w; cr_e += cr_b) {
          const std::size_t cr_g = cr_base + cr_e;  // element cr_g - 2, loaded only inside the array
          if(cr_g >= 2 && cr_g - 2 < n) cr_s_x[cr_e] = x[cr_g - 2];
        }
      },
      [=] CR_DEVICE(std::size_t v_i, std::size_t cr_base, std::size_t cr_w, unsigned char* cr_shared) {
        const float* const cr_s_x = reinterpret_cast<const float*>(cr_shared + 0);
        const std::size_t o = v_i - cr_base + 2;  // x[i + d] is cr_s_x[o + d]
        if(v_i >= 2 && v_i + 2 < n)
          out[v_i] = cr_s_x[o - 2] + cr_s_x[o - 1] * 2.0f + cr_s_x[o] * 3.0f + cr_s_x[o + 1] + cr_s_x[o + 2];
        else
          out[v_i] = cr_s_x[o];
      },
      [](std::size_t cr_w) { return cr::gpu::tile_bytes<float>(cr_w); }, 128);
}
#if defined(CAIRN_B200_MACHINE)
struct WrapAdd {
  CR_DEVICE std::uint32_t operator()(std::uint32_t p, std::uint32_t q) const { return cr::add_wrap(p, q); }
};
inline const std::uint32_t* x_none() { return nullptr; }
#endif
}  // namespace

extern "C" {
void cf_saxpy(std::size_t n, float* out, const float* x, const float* y, float a) noexcept {
  cr::view(out, n);
  cr::view(x, n);
  cr::view(y, n);
  ci_saxpy(n, out, x, y, a);
}
void cf_saxpy4(std::size_t n, float* out, const float* x, const float* y, float a) noexcept {
  cr::view(out, n);
  cr::view(x, n);
  cr::view(y, n);
  ci_saxpy4(n, out, x, y, a);
}
void cq_saxpy(void* stream, std::size_t n, float* out, const float* x, const float* y, float a) noexcept {
  cr::view(out, n);
  cr::view(x, n);
  cr::view(y, n);
  cr::gpu::Enqueued queued(stream);
  ci_saxpy(n, out, x, y, a);
}
float cf_dsum(std::size_t n, const float* x) noexcept {
  cr::view(x, n);
  return ci_dsum(n, x);
}
std::uint64_t cf_usum(std::size_t n, const std::uint64_t* x) noexcept {
  cr::view(x, n);
  return ci_usum(n, x);
}
std::int32_t cf_vmax(std::size_t n, const std::int32_t* x) noexcept {
  cr::view(x, n);
  return ci_vmax(n, x);
}
void cf_gemm(std::size_t m, std::size_t n, std::size_t k, std::size_t cn, float* c, std::size_t an,
             const std::uint16_t* a, std::size_t bn, const std::uint16_t* b) noexcept {
  const auto* A = reinterpret_cast<const cr::bf16*>(a);
  const auto* B = reinterpret_cast<const cr::bf16*>(b);
  cr::view(c, cn);
  cr::view(A, an);
  cr::view(B, bn);
  cr::disjoint(c, cn, A, an);
  cr::disjoint(c, cn, B, bn);
  ci_gemm(m, n, k, c, cn, A, an, B, bn);
}
void cq_gemm(void* stream, std::size_t m, std::size_t n, std::size_t k, std::size_t cn, float* c, std::size_t an,
             const std::uint16_t* a, std::size_t bn, const std::uint16_t* b) noexcept {
  const auto* A = reinterpret_cast<const cr::bf16*>(a);
  const auto* B = reinterpret_cast<const cr::bf16*>(b);
  cr::view(c, cn);
  cr::view(A, an);
  cr::view(B, bn);
  cr::disjoint(c, cn, A, an);
  cr::disjoint(c, cn, B, bn);
  cr::gpu::Enqueued queued(stream);
  ci_gemm(m, n, k, c, cn, A, an, B, bn);
}
std::uint64_t cf_prefix(std::size_t n, std::uint64_t* out, const std::uint64_t* x) noexcept {
  cr::view(out, n);
  cr::view(x, n);
  return ci_prefix(n, out, x);
}
std::uint32_t cf_wprefix(std::size_t n, std::uint32_t* out, const std::uint32_t* x) noexcept {
  cr::view(out, n);
  cr::view(x, n);
  return ci_wprefix(n, out, x);
}
std::int32_t cf_runmax(std::size_t n, std::int32_t* out, const std::int32_t* x) noexcept {
  cr::view(out, n);
  cr::view(x, n);
  return ci_runmax(n, out, x);
}
float cf_fprefix(std::size_t n, float* out, const float* x) noexcept {
  cr::view(out, n);
  cr::view(x, n);
  return ci_fprefix(n, out, x);
}
std::size_t cf_positives(std::size_t n, float* out, const float* x) noexcept {
  cr::view(out, n);
  cr::view(x, n);
  return ci_positives(n, out, x);
}
#if defined(CAIRN_B200_MACHINE)  // entries of the B200 machine's own scan (absent from the reference's machine)
// Not a cairnc entry: the machine's inclusive u64 scan with a zero wait for predecessors, so that blocks which find
// a predecessor unpublished take the look-back's escape (folding the inputs before their tile themselves).
void cf_prefix_escape(std::size_t n, std::uint64_t* out, const std::uint64_t* x) noexcept {
  std::size_t bytes = 0;
  cr::gpu::b200::scan<false, std::uint64_t>(nullptr, bytes, x, out, n, cr::gpu::b200::Plus{}, nullptr);
  void* temp = nullptr;
  cr::gpu::check(cudaMalloc(&temp, bytes));
  cr::gpu::b200::scan<false, std::uint64_t>(temp, bytes, x, out, n, cr::gpu::b200::Plus{}, nullptr, 0);
  cr::gpu::check(cudaStreamSynchronize(nullptr));
  cr::gpu::check(cudaFree(temp));
}
#endif
void cf_blur(std::size_t n, float* out, const float* x) noexcept {
  cr::view(out, n);
  cr::view(x, n);
  ci_blur(n, out, x);
}
// pub fn wscan(n, out: rw<u32>[n]@device, x: ro<u32>[n]@device)
//   { scan add_wrap parallel i in n yield x[i] into out; }   (no total: scan_into, enqueued on the caller's stream)
void cq_wscan(void* stream, std::size_t n, std::uint32_t* out, const std::uint32_t* x) noexcept {
  cr::view(out, n);
  cr::view(x, n);
  cr::gpu::Enqueued queued(stream);
  cr::gpu::scan_into<false, std::uint32_t>(
      cr::gpu::here(), out, n, 0u, [] CR_DEVICE(std::uint32_t p, std::uint32_t q) { return cr::add_wrap(p, q); },
      [=] CR_DEVICE(std::size_t i) { return x[i]; });
}
#if defined(CAIRN_B200_MACHINE)
// Not cairnc entries: the machine's inclusive u32 add_wrap scan kernel alone, on the caller's stream and scratch
// (b200_scan_u32_scratch bytes), so a bench can time the kernel without the context's copy pass.
std::size_t b200_scan_u32_scratch(std::size_t n) noexcept {
  std::size_t bytes = 0;
  cr::gpu::b200::scan<false, std::uint32_t>(nullptr, bytes, x_none(), static_cast<std::uint32_t*>(nullptr), n,
                                            WrapAdd{}, nullptr);
  return bytes;
}
void b200_scan_u32(void* stream, std::size_t n, std::uint32_t* out, const std::uint32_t* x, void* temp) noexcept {
  std::size_t bytes = b200_scan_u32_scratch(n);
  cr::gpu::b200::scan<false, std::uint32_t>(temp, bytes, x, out, n, WrapAdd{}, static_cast<cudaStream_t>(stream));
}
#endif
}

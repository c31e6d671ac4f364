// Entries of the B200 machine's scan that no CAIRN program emits, for tests/test_dropin_gpu.py and bench.py: the
// inclusive u64 scan with no wait for predecessors (every block that finds a predecessor unpublished takes the
// look-back's escape and folds the inputs before its tile itself), and the u32 add_wrap scan kernel alone on the
// caller's stream and scratch, so that a bench can time the kernel without the context's copy pass. Built over the
// drop-in headers by tests/dropin/build_emitted.py.
#include <cstddef>
#include <cstdint>
#include "cairn_runtime.hpp"
#include "cairn_gpu.hpp"
#include "cairn_cub.hpp"

namespace {
struct WrapAdd {
  CR_DEVICE std::uint32_t operator()(std::uint32_t p, std::uint32_t q) const { return cr::add_wrap(p, q); }
};
const std::uint32_t* no_input() { return nullptr; }
}  // namespace

extern "C" {
void cf_prefix_escape(std::size_t n, std::uint64_t* out, const std::uint64_t* x) noexcept {
  std::size_t bytes = 0;
  cr::gpu::b200::scan<false, std::uint64_t>(nullptr, bytes, x, out, n, cr::gpu::b200::Plus{}, nullptr);
  void* temp = nullptr;
  cr::gpu::check(cudaMalloc(&temp, bytes));
  cr::gpu::b200::scan<false, std::uint64_t>(temp, bytes, x, out, n, cr::gpu::b200::Plus{}, nullptr, 0);
  cr::gpu::check(cudaStreamSynchronize(nullptr));
  cr::gpu::check(cudaFree(temp));
}
std::size_t b200_scan_u32_scratch(std::size_t n) noexcept {
  std::size_t bytes = 0;
  cr::gpu::b200::scan<false, std::uint32_t>(nullptr, bytes, no_input(), static_cast<std::uint32_t*>(nullptr), n,
                                            WrapAdd{}, nullptr);
  return bytes;
}
void b200_scan_u32(void* stream, std::size_t n, std::uint32_t* out, const std::uint32_t* x, void* temp) noexcept {
  std::size_t bytes = b200_scan_u32_scratch(n);
  cr::gpu::b200::scan<false, std::uint32_t>(temp, bytes, x, out, n, WrapAdd{}, static_cast<cudaStream_t>(stream));
}
}

// Drop-in replacement for CAIRN's runtime/cairn_kernels.hpp on a B200 (sm_100a): the device side of every `parallel`
// region. It keeps the names, signatures and contracts generated code and runtime/cairn_exec.hpp rely on
// (cr::gpu::check, BLOCK / MAX_GRID / WARP, the lanes / chunks / staged_lanes kernels and the fire, fire_vector and
// fire_staged launchers; runtime/cairn_kernels.hpp:55-138): every index below n runs exactly once, on the caller's
// stream, without a wait, and a CUDA error aborts the process as the reference's guard does.
//
// What differs is the launch geometry. The reference sizes a region's grid at one thread per index, capped at
// 65,535 blocks, whatever the device. Here a region is a persistent grid-stride loop sized to the device: as many
// blocks as the SMs hold resident at once (the occupancy calculator's answer for this kernel and block, times the SM
// count), never more blocks than the region has work for, so every block strides over a long run of indices and the
// loop body is unrolled U times as the plan asks. A `plan vector W` region (chunks) moves W adjacent elements per
// access, which for f32 and W = 4 is the 16-byte access a B200 streams at full HBM bandwidth.
//
// Build a program with this directory ahead of the reference's runtime directory on the include path.
#pragma once
#include <cstddef>
#include <cstdio>
#include <cuda_runtime.h>
#include "cairn_runtime.hpp"
namespace cr::gpu {

inline void check(cudaError_t e) noexcept {
  if(e == cudaSuccess) return;
  std::fprintf(stderr, "cairn: cuda: %s\n", cudaGetErrorString(e));
  trap();
}

// The reference's constants, kept for runtime/cairn_reuse.hpp's static checks: a region's default block, the
// reference's grid cap (used here only as an upper bound), a warp.
constexpr unsigned BLOCK = 256, MAX_GRID = 65535, WARP = 32;

// The SM count of the current device, asked once per device.
inline unsigned sm_count() noexcept {
  static unsigned held[64] = {};
  int dev = 0;
  check(cudaGetDevice(&dev));
  if(dev < 0 || dev >= 64) return 148;
  if(!held[dev]) {
    int sms = 0;
    check(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev));
    held[dev] = unsigned(sms);
  }
  return held[dev];
}

template<unsigned U, class F> __global__ void lanes(std::size_t n, F body) {
  const std::size_t step = std::size_t(gridDim.x) * blockDim.x;
#pragma unroll U
  for(std::size_t i = blockIdx.x * std::size_t(blockDim.x) + threadIdx.x; i < n; i += step) body(i);
}

// The widest block a kernel can run (its registers may not allow the block a plan asked for), in whole warps.
template<class K> inline unsigned most(K kernel) noexcept {
  cudaFuncAttributes held{};
  check(cudaFuncGetAttributes(&held, kernel));
  return unsigned(held.maxThreadsPerBlock) / WARP * WARP;
}
template<unsigned U, class F> inline unsigned widest() noexcept {
  static const unsigned held = most(lanes<U, F>);
  return held;
}

// Blocks for a region of n indices with `each` indices per block-step: no more than the work needs, and no more
// than the device holds resident (persistent blocks), never more than the reference's cap.
template<class K> inline unsigned resident_grid(K kernel, unsigned block, std::size_t shared, std::size_t n,
                                                std::size_t each) noexcept {
  int per_sm = 0;
  check(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kernel, int(block), shared));
  std::size_t resident = std::size_t(per_sm > 0 ? per_sm : 1) * sm_count();
  const std::size_t needed = (n + each - 1) / each;
  std::size_t g = needed < resident ? needed : resident;
  if(g > MAX_GRID) g = MAX_GRID;
  return unsigned(g ? g : 1);
}

template<unsigned U = 1, class F>
inline void fire(std::size_t n, const F& body, cudaStream_t s, unsigned block = BLOCK, std::size_t per_lane = 1) noexcept {
  static_assert(std::is_trivially_copyable_v<F>, "a lane body crosses over as kernel arguments");
  if(!n) return;
  if(block > widest<U, F>()) block = widest<U, F>();
  lanes<U><<<resident_grid(lanes<U, F>, block, 0, n, std::size_t(block) * per_lane), block, 0, s>>>(n, body);
  check(cudaGetLastError());
}

// `plan f { vector W; }`: W adjacent indices per lane through one aligned chunk, the tail one at a time.
template<unsigned W, unsigned U, class F, class G> __global__ void chunks(std::size_t n, F scalar, G chunk) {
  const std::size_t step = std::size_t(gridDim.x) * blockDim.x * W;
#pragma unroll U
  for(std::size_t i = (blockIdx.x * std::size_t(blockDim.x) + threadIdx.x) * W; i < n; i += step) {
    if(n - i >= W) chunk(i);
    else for(std::size_t k = i; k < n; ++k) scalar(k);
  }
}
template<unsigned W, unsigned U, class F, class G>
inline void fire_vector(std::size_t n, F scalar, G chunk, cudaStream_t s, unsigned block, std::size_t per_lane) noexcept {
  static const unsigned held = most(chunks<W, U, F, G>);
  if(block > held) block = held;
  const unsigned grid = resident_grid(chunks<W, U, F, G>, block, 0, n, std::size_t(block) * per_lane * W);
  chunks<W, U><<<grid, block, 0, s>>>(n, scalar, chunk);
  check(cudaGetLastError());
}

// `plan f { stage R; }`: a block runs its indices tile by tile through shared memory, between two barriers every
// thread of the block reaches (runtime/cairn_exec.hpp's run_staged states the rule).
template<std::size_t R, unsigned U, class L, class F> __global__ void staged_lanes(std::size_t n, L load, F body) {
  extern __shared__ __align__(16) unsigned char cr_shared[];
  const std::size_t b = blockDim.x, w = b + 2 * R, t = threadIdx.x, step = std::size_t(gridDim.x) * b;
#pragma unroll U
  for(std::size_t base = blockIdx.x * b; base < n; base += step) {
    __syncthreads();
    load(base, w, t, b, cr_shared);
    __syncthreads();
    if(base + t < n) body(base + t, base, w, cr_shared);
  }
}
template<std::size_t R, unsigned U, class L, class F, class S>
inline void fire_staged(std::size_t n, L load, F body, S bytes, cudaStream_t s, unsigned block,
                        std::size_t per_lane) noexcept {
  static const unsigned held = most(staged_lanes<R, U, L, F>);
  if(block > held) block = held;
  const std::size_t shared = bytes(std::size_t(block) + 2 * R);
  if(shared > 48 * 1024)
    check(cudaFuncSetAttribute(staged_lanes<R, U, L, F>, cudaFuncAttributeMaxDynamicSharedMemorySize, int(shared)));
  const unsigned grid = resident_grid(staged_lanes<R, U, L, F>, block, shared, n, std::size_t(block) * per_lane);
  staged_lanes<R, U><<<grid, block, shared, s>>>(n, load, body);
  check(cudaGetLastError());
}

}  // namespace cr::gpu

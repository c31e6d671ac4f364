// Drop-in replacement for CAIRN's runtime/cairn_kernels.hpp on a B200 (sm_100a): the device side of a `parallel`
// region. Generated code and the reference's own headers name four things from this file: cr::gpu::check (a CUDA
// error ends the process, as every guard does: runtime/cairn_kernels.hpp:55-59, compiler/device/launches.py:67),
// and the constants BLOCK, MAX_GRID and WARP (runtime/cairn_reuse.hpp:28, cairn_coop.hpp:500, cairn_tensor.hpp:211).
// Everything else here is this project's: the region kernels and their launchers, which only this directory's
// cairn_gpu.hpp calls, as the B200 machine's `lanes`, `vector_lanes` and `staged_lanes` members.
//
// The contract each kernel keeps is the one runtime/cairn_exec.hpp states for run, run_vector and run_staged: every
// index below n runs its body exactly once, on the stream the caller names, and nothing waits. How a B200 runs them:
//
// * A region is a persistent grid. The launcher sizes it from the occupancy calculator for the kernel, its block
//   and its shared memory, times the SM count (148 on a B200): every block is resident from the start, and no more
//   blocks are launched than the region has tiles of work for. There is no 65,535-block cap to stride around.
// * The unit of work is a tile of U * block consecutive indices (U from the plan's `unroll`): thread t of the block
//   runs indices t, t + block, ... of each tile it is handed, so every step of the warp touches 32 consecutive
//   elements, and the U steps of a tile are unrolled without a bounds test. Blocks take tiles in rotation; the
//   last, partial tile goes to whichever block the rotation hands it to, with a test per index.
// * A `plan vector W` region runs its whole chunks the same way (one W-wide access per array per lane, 16 bytes for
//   f32 and W = 4), and the fewer than W indices past the last whole chunk run in parallel, one thread each.
// * A `plan stage R` region keeps two tiles of shared memory when they fit: while a block's lanes read one tile,
//   its threads have already loaded the next one into the other, so one barrier per tile separates the two, where a
//   single tile needs a barrier before its load and another after it.
//
// Why a plain region's body runs one index at a time per thread: the body is the program's lambda over raw
// pointers, and the compiler must assume that its store to out[i] may alias the next index's loads, so those loads
// cannot be issued early. A plain region's memory parallelism is therefore two to three loads in flight per
// thread, times the 2048 threads an SM holds; the 16-byte chunks of a vector region carry four times the bytes per
// load, which is what reaches HBM's bandwidth.
//
// Build a program with this directory ahead of the reference's runtime directory on the include path.
#pragma once
#include <atomic>
#include <cstddef>
#include <cstdio>
#include <mutex>
#include <type_traits>
#include <cuda_runtime.h>
#include "cairn_runtime.hpp"
namespace cr::gpu {

// A failed CUDA call aborts the process through the same trap as a failed guard.
inline void check(cudaError_t e) noexcept {
  if(e == cudaSuccess) return;
  std::fprintf(stderr, "cairn: cuda: %s: %s\n", cudaGetErrorName(e), cudaGetErrorString(e));
  trap();
}

// The default block of a region, the largest grid the reference's launches use (this machine's persistent grids
// stay far below it), and a warp.
constexpr unsigned BLOCK = 256, MAX_GRID = 65535, WARP = 32;

namespace b200 {

// The SM count of each device, asked once per device.
inline unsigned sm_count() noexcept {
  constexpr int DEVICES = 64;
  static unsigned sms[DEVICES];
  static std::once_flag asked[DEVICES];
  int dev = 0;
  check(cudaGetDevice(&dev));
  if(dev < 0 || dev >= DEVICES) trap();
  std::call_once(asked[dev], [dev] {
    int v = 0;
    check(cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev));
    sms[dev] = v > 0 ? unsigned(v) : 1u;
  });
  return sms[dev];
}

// What one kernel allows, asked once per kernel: its widest block in whole warps (its registers may not allow the
// block a plan asked for; the region then runs narrower blocks and computes the same).
template<class K> inline unsigned widest_block(K kernel) noexcept {
  cudaFuncAttributes a{};
  check(cudaFuncGetAttributes(&a, kernel));
  const unsigned w = unsigned(a.maxThreadsPerBlock) / WARP * WARP;
  return w ? w : WARP;
}

// Blocks of one kernel resident on the whole device for this block and shared memory. The occupancy calculator's
// answer is kept in `last`, which each launcher holds for its own kernel, for the last (block, shared memory) it was
// asked about, so a region launched again with the same plan asks nothing.
template<class K>
inline std::size_t resident_blocks(std::atomic<unsigned long long>& last, K kernel, unsigned block,
                                   std::size_t shared) noexcept {
  const unsigned long long key = (static_cast<unsigned long long>(block) << 40) |
                                 (static_cast<unsigned long long>(shared) << 8);
  const unsigned long long seen = last.load(std::memory_order_relaxed);
  unsigned per_sm = 0;
  if(seen != 0 && (seen & ~0xffull) == key) {
    per_sm = unsigned(seen & 0xffull);
  } else {
    int fit = 0;
    check(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&fit, kernel, int(block), shared));
    per_sm = fit > 0 ? (fit < 255 ? unsigned(fit) : 255u) : 1u;
    last.store(key | per_sm, std::memory_order_relaxed);  // block << 40 | shared << 8 | blocks per SM
  }
  return std::size_t(per_sm) * sm_count();
}

// The persistent grid: the device's resident blocks, fewer when the region has fewer tiles of work, or when the
// plan asked for about `per_lane` indices per thread over `indices` indices (a block covers block * per_lane).
inline unsigned persistent_grid(std::size_t resident, std::size_t tiles, std::size_t indices, unsigned block,
                                std::size_t per_lane) noexcept {
  const std::size_t each = std::size_t(block) * (per_lane ? per_lane : 1);
  std::size_t g = (indices + each - 1) / each;
  if(g > tiles) g = tiles;
  if(g > resident) g = resident;
  return unsigned(g ? g : 1);
}

// `parallel i in n`: tiles of U * blockDim.x indices.
template<unsigned U, class F> __global__ void region_lanes(std::size_t n, F body) {
  const std::size_t width = std::size_t(U) * blockDim.x, whole = n / width;
  std::size_t tile = blockIdx.x;
  for(; tile < whole; tile += gridDim.x) {
    const std::size_t first = tile * width + threadIdx.x;
#pragma unroll
    for(unsigned u = 0; u < U; ++u) body(first + std::size_t(u) * blockDim.x);
  }
  if(tile == whole)  // the rotation handed this block the partial tile
    for(std::size_t i = whole * width + threadIdx.x; i < n; i += blockDim.x) body(i);
}

template<unsigned U, class F>
inline void start_lanes(std::size_t n, const F& body, cudaStream_t s, unsigned block, std::size_t per_lane) noexcept {
  static_assert(U >= 1, "a plan unrolls at least once");
  static_assert(std::is_trivially_copyable_v<F>, "a lane body crosses over as kernel arguments");
  if(!n) return;
  static const unsigned most = widest_block(region_lanes<U, F>);
  static std::atomic<unsigned long long> fit{0};
  if(block > most) block = most;
  if(block < WARP) block = WARP;
  const std::size_t width = std::size_t(U) * block, tiles = (n + width - 1) / width;
  const unsigned grid =
      persistent_grid(resident_blocks(fit, region_lanes<U, F>, block, 0), tiles, n, block, per_lane);
  region_lanes<U><<<grid, block, 0, s>>>(n, body);
  check(cudaGetLastError());
}

// `plan f { vector W; }`: whole chunks of W indices from index 0 in tiles of U * blockDim.x chunks, then the
// n % W indices past them, one thread each.
template<unsigned W, unsigned U, class F, class G> __global__ void region_chunks(std::size_t n, F scalar, G chunk) {
  const std::size_t chunks = n / W, width = std::size_t(U) * blockDim.x, whole = chunks / width;
  std::size_t tile = blockIdx.x;
  for(; tile < whole; tile += gridDim.x) {
    const std::size_t first = tile * width + threadIdx.x;
#pragma unroll
    for(unsigned u = 0; u < U; ++u) chunk((first + std::size_t(u) * blockDim.x) * W);
  }
  if(tile == whole) {
    for(std::size_t c = whole * width + threadIdx.x; c < chunks; c += blockDim.x) chunk(c * W);
    const std::size_t rest = n - chunks * W;  // fewer than W <= 16 indices, and a block is at least a warp
    if(threadIdx.x < rest) scalar(chunks * W + threadIdx.x);
  }
}

template<unsigned W, unsigned U, class F, class G>
inline void start_chunks(std::size_t n, F scalar, G chunk, cudaStream_t s, unsigned block,
                         std::size_t per_lane) noexcept {
  static_assert(W >= 1 && W <= 16 && U >= 1, "a chunk is 1 to 16 indices");
  static_assert(std::is_trivially_copyable_v<F> && std::is_trivially_copyable_v<G>, "lanes cross as arguments");
  if(!n) return;
  static const unsigned most = widest_block(region_chunks<W, U, F, G>);
  static std::atomic<unsigned long long> fit{0};
  if(block > most) block = most;
  if(block < WARP) block = WARP;
  const std::size_t width = std::size_t(U) * block, tiles = (n / W + width - 1) / width + 1;
  const unsigned grid =
      persistent_grid(resident_blocks(fit, region_chunks<W, U, F, G>, block, 0), tiles, n / W + 1, block, per_lane);
  region_chunks<W, U><<<grid, block, 0, s>>>(n, scalar, chunk);
  check(cudaGetLastError());
}

// `plan f { stage R; }`: a tile covers blockDim.x indices from `base`; `load(base, w, t, b, tile)` fills the tile
// with the staged arrays' elements from base - R to base + b + R that lie inside them, and `body(i, base, w, tile)`
// runs index i reading them there (runtime/cairn_exec.hpp's run_staged). With `pair`, the block holds two tiles
// `stride` bytes apart and loads tile k + 1 into one while its lanes read tile k from the other; the barrier after
// the lanes both publishes the next tile and frees the one just read. Without it, one tile between two barriers.
// Every thread of a block reaches every barrier: the loop bounds depend on the block, never the thread.
template<std::size_t R, class L, class F>
__global__ void region_staged(std::size_t n, L load, F body, std::size_t stride, bool pair) {
  extern __shared__ __align__(128) unsigned char tiles_smem[];
  const std::size_t b = blockDim.x, w = b + 2 * R, t = threadIdx.x, tiles = (n + b - 1) / b;
  std::size_t tile = blockIdx.x;
  if(tile >= tiles) return;
  if(!pair) {
    for(; tile < tiles; tile += gridDim.x) {
      const std::size_t base = tile * b;
      __syncthreads();  // the lanes of the previous tile are done with it
      load(base, w, t, b, tiles_smem);
      __syncthreads();
      if(base + t < n) body(base + t, base, w, tiles_smem);
    }
    return;
  }
  unsigned char* held = tiles_smem;
  unsigned char* next_tile = tiles_smem + stride;
  load(tile * b, w, t, b, held);
  __syncthreads();
  for(;;) {
    const std::size_t next = tile + gridDim.x, base = tile * b;
    if(next < tiles) load(next * b, w, t, b, next_tile);
    if(base + t < n) body(base + t, base, w, held);
    __syncthreads();
    if(next >= tiles) break;
    tile = next;
    unsigned char* read = held;
    held = next_tile;
    next_tile = read;
  }
}

template<std::size_t R, unsigned U, class L, class F, class S>
inline void start_staged(std::size_t n, L load, F body, S bytes, cudaStream_t s, unsigned block,
                         std::size_t per_lane) noexcept {
  static_assert(std::is_trivially_copyable_v<L> && std::is_trivially_copyable_v<F>, "lanes cross as arguments");
  (void)U;  // a tile's barriers leave nothing to unroll
  if(!n) return;
  static const unsigned most = widest_block(region_staged<R, L, F>);
  static std::atomic<unsigned long long> fit{0};
  if(block > most) block = most;
  if(block < WARP) block = WARP;
  const std::size_t one = (bytes(std::size_t(block) + 2 * R) + 127) / 128 * 128;
  int optin = 0, dev = 0;
  check(cudaGetDevice(&dev));
  check(cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev));
  const bool pair = 2 * one <= std::size_t(optin);
  const std::size_t shared = pair ? 2 * one : one;
  if(shared > std::size_t(optin)) trap();  // a tile larger than any block's shared memory
  if(shared > 48 * 1024)
    check(cudaFuncSetAttribute(region_staged<R, L, F>, cudaFuncAttributeMaxDynamicSharedMemorySize, int(shared)));
  const std::size_t tiles = (n + block - 1) / block;
  const unsigned grid = persistent_grid(resident_blocks(fit, region_staged<R, L, F>, block, shared), tiles, n, block,
                                        per_lane);
  region_staged<R><<<grid, block, shared, s>>>(n, load, body, one, pair);
  check(cudaGetLastError());
}

}  // namespace b200
}  // namespace cr::gpu

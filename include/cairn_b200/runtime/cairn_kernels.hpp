// Drop-in replacement for CAIRN's runtime/cairn_kernels.hpp on a B200 (sm_100a): the device side of a `parallel`
// region. Generated code and the reference's own headers name four things from this file: cr::gpu::check (a CUDA
// error ends the process, as every guard does: runtime/cairn_kernels.hpp:55-59, compiler/device/launches.py:67),
// and the constants BLOCK, MAX_GRID and WARP (runtime/cairn_reuse.hpp:28, cairn_coop.hpp:500, cairn_tensor.hpp:211).
// Everything else here is this project's: the region kernels and their launchers, which only this directory's
// cairn_gpu.hpp calls, as the B200 machine's `lanes`, `vector_lanes` and `staged_lanes` members.
//
// The contract each kernel keeps is the one runtime/cairn_exec.hpp states for run, run_vector and run_staged: every
// index below n runs its body exactly once, on the stream the caller names, and nothing waits. The grid shapes are
// the ones that ran fastest on a B200 at n = 2^30 (f32 saxpy and a five-point blur, each shape against the others):
//
// * Plain region: a grid-stride loop in which each thread runs about LANE_INDICES = 64 indices (more if the plan's
//   per_lane asks), and never fewer blocks than the SMs hold resident while n has work for them; the whole strides
//   run without a bounds test and the plan's `unroll` unrolls them. Around 64 indices per thread ran fastest (about
//   4.96 TB/s for saxpy, 1-3 % above 9,472 or 131,072 blocks); a persistent grid of one resident wave ran 4 % slower,
//   because the SMs whose blocks fell behind finished last. A plain region cannot go much faster: the body is the
//   program's lambda over raw pointers, the compiler must assume its store to out[i] may alias the next index's
//   loads, so a thread has only this index's loads in flight, times the 2048 threads an SM holds.
// * `plan vector W`: one W-wide chunk per thread (per_lane chunks when the plan asks), a block per block-width of
//   chunks, and the fewer than W indices past the last whole chunk run by the last block, one thread each. For f32
//   and W = 4 each access is 16 bytes; this shape ran 7.1 TB/s for saxpy, where a grid-stride loop over 65,535
//   blocks ran 6.9 and a persistent grid 6.3.
// * `plan stage R`: one tile of shared memory per block, several block widths wide (plus the 2R halo), each thread
//   running the body at as many indices of it, and each block taking a run of consecutive tiles (STAGE_TILES block
//   widths' worth, or the plan's per_lane widths if more), between the two barriers run_staged's rule asks for. The
//   emitted load and lane bodies take the tile's width as an argument (compiler/plans/staging.py:85-120: the load
//   loops over it, the arrays' offsets and bytes follow it), so a tile may hold several block widths. For blocks of
//   128 or 256 threads a tile holds STAGE_WIDE = 2048 indices and the kernel is compiled for that block width, so the
//   load loop's trip count is known and every one of a thread's loads is in flight at once; other blocks take four
//   widths with the width known only at launch. Measured on a B200 for the blur (n = 2^30, blocks of 128): the
//   width known at launch, tiles of 1, 2, 3, 4, 5, 6 and 8 block widths ran 2.29, 2.09, 2.07, 3.10, 2.32, 2.34 and
//   2.40 TB/s; known where compiled, 4, 8, 16, 32 and 64 widths 2.98, 4.46, 4.93, 4.21 and 2.25, and 5.15-5.48 with
//   16 widths held to 32 registers (the reference's machine, one width: 2.17). Consecutive tiles share their halos in cache (a run of tiles per block ran 2.49 TB/s
//   against 1.69 with one tile per block, at one width). Two one-width tiles per block, loading the next while the
//   lanes read the current one, measured slower (2.31): the loads must land before their stores into the tile.
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

constexpr std::size_t LANE_INDICES = 64;  // indices per thread a plain region's grid aims at
constexpr std::size_t STAGE_TILES = 64;   // block widths of consecutive tiles per block of a staged region
constexpr std::size_t STAGE_WIDTHS = 4;   // block widths per staged tile, for a block width known only at launch
constexpr std::size_t STAGE_WIDE = 2048;  // indices per staged tile for blocks of 128 or 256 threads
constexpr std::size_t GRID_LIMIT = 0x7fffffff;

// The grid for `units` units of work (indices, chunks or tiles), `per` per thread or block as the caller counts
// them, in blocks of `each` units: no fewer blocks than the device holds resident when there are units for them,
// and past that a whole multiple of the SM count (every SM gets as many blocks: 65,564 blocks of a saxpy region ran
// 4.96 TB/s on a B200 where 65,535 ran 4.79).
inline unsigned region_grid(std::size_t units, std::size_t each, std::size_t per, std::size_t resident) noexcept {
  const std::size_t blocks = (units + each - 1) / each;  // one unit per thread (or tile per block)
  std::size_t g = (units + each * per - 1) / (each * per);
  const std::size_t least = blocks < resident ? blocks : resident;
  if(g <= least) {
    g = least;
  } else {
    const std::size_t sms = sm_count();
    g = (g + sms - 1) / sms * sms;
    if(g > blocks) g = blocks;
  }
  if(g > GRID_LIMIT) trap();  // the caller raises `per` first
  return unsigned(g ? g : 1);
}

// `parallel i in n`: thread (b, t) runs indices b * blockDim.x + t + k * stride, k = 0, 1, ...
template<unsigned U, class F> __global__ void region_lanes(std::size_t n, F body) {
  const std::size_t stride = std::size_t(gridDim.x) * blockDim.x;
  std::size_t i = std::size_t(blockIdx.x) * blockDim.x + threadIdx.x;
  const std::size_t whole = n / stride;  // strides in which every thread has an index
#pragma unroll U
  for(std::size_t k = 0; k < whole; ++k, i += stride) body(i);
  if(i < n) body(i);
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
  std::size_t per = per_lane > LANE_INDICES ? per_lane : LANE_INDICES;
  while((n + block * per - 1) / (block * per) > GRID_LIMIT) per *= 2;
  const unsigned grid = region_grid(n, block, per, resident_blocks(fit, region_lanes<U, F>, block, 0));
  region_lanes<U><<<grid, block, 0, s>>>(n, body);
  check(cudaGetLastError());
}

// `plan f { vector W; }`: block b runs chunks b * per * blockDim.x + t + k * blockDim.x, k < per; a chunk is W
// indices from index chunk * W. The last block also runs the n % W indices past the last whole chunk.
template<unsigned W, unsigned U, class F, class G>
__global__ void region_chunks(std::size_t n, std::size_t per, F scalar, G chunk) {
  const std::size_t chunks = n / W;
  std::size_t c = std::size_t(blockIdx.x) * per * blockDim.x + threadIdx.x;
#pragma unroll U
  for(std::size_t k = 0; k < per; ++k, c += blockDim.x)
    if(c < chunks) chunk(c * W);
  if(blockIdx.x == gridDim.x - 1 && threadIdx.x < n - chunks * W) scalar(chunks * W + threadIdx.x);
}

template<unsigned W, unsigned U, class F, class G>
inline void start_chunks(std::size_t n, F scalar, G chunk, cudaStream_t s, unsigned block,
                         std::size_t per_lane) noexcept {
  static_assert(W >= 1 && W <= 16 && U >= 1, "a chunk is 1 to 16 indices");
  static_assert(std::is_trivially_copyable_v<F> && std::is_trivially_copyable_v<G>, "lanes cross as arguments");
  if(!n) return;
  static const unsigned most = widest_block(region_chunks<W, U, F, G>);
  if(block > most) block = most;
  if(block < WARP) block = WARP;
  const std::size_t chunks = n / W;
  std::size_t per = per_lane ? per_lane : 1;
  while((chunks + block * per - 1) / (block * per) > GRID_LIMIT) per *= 2;
  const std::size_t g = (chunks + block * per - 1) / (block * per);
  region_chunks<W, U><<<unsigned(g ? g : 1), block, 0, s>>>(n, per, scalar, chunk);
  check(cudaGetLastError());
}

// `plan f { stage R; }`: a tile covers K block widths of indices from `base` (STAGE_WIDE / B for blocks of B = 128 or
// 256 threads, STAGE_WIDTHS for other blocks, or one where the wider tile would take more than 48 KB of shared
// memory); `load(base, w, t, b, tile)` fills the tile (w = K b + 2R) with the staged arrays' elements from base - R
// to base + K b + R that lie inside them, and `body(i, base, w, tile)` runs each index i of the tile reading them
// there, thread t at base + t, base + b + t, ... (runtime/cairn_exec.hpp's run_staged). Block b takes tiles
// b * span to b * span + span - 1. Every thread of a block reaches every barrier: the loop bounds depend on the
// block alone.
template<std::size_t R, std::size_t K, unsigned B, class L, class F>
__device__ __forceinline__ void staged_tiles(std::size_t n, std::size_t span, L& load, F& body) {
  extern __shared__ __align__(128) unsigned char tile_smem[];
  // B: the block width when it is known where the kernel is compiled (the launcher picks such a kernel only for
  // blocks of B threads), so that the load body's loop over the tile has a known trip count; 0: blockDim.x
  const std::size_t b = B ? B : blockDim.x, w = K * b + 2 * R, t = threadIdx.x, tiles = (n + K * b - 1) / (K * b);
  const std::size_t first = std::size_t(blockIdx.x) * span, last = first + span < tiles ? first + span : tiles;
#pragma unroll 1
  for(std::size_t tile = first; tile < last; ++tile) {
    const std::size_t base = tile * K * b;
    __syncthreads();  // the lanes of the previous tile are done with it
    load(base, w, t, b, tile_smem);
    __syncthreads();
#pragma unroll
    for(std::size_t k = 0; k < K; ++k)
      if(base + k * b + t < n) body(base + k * b + t, base, w, tile_smem);
  }
}
// The width known at launch.
template<std::size_t R, std::size_t K, class L, class F>
__global__ void region_staged(std::size_t n, std::size_t span, L load, F body) {
  staged_tiles<R, K, 0>(n, span, load, body);
}
// The width known where compiled, held to the registers that let an SM hold 2048 / B blocks of it (measured on a
// B200 for the blur at B = 128: 5.15 TB/s against 4.93 with the compiler's 39 registers, 12 blocks per SM).
template<std::size_t R, std::size_t K, unsigned B, class L, class F>
__global__ void __launch_bounds__(B, 2048 / B) region_staged_fixed(std::size_t n, std::size_t span, L load, F body) {
  staged_tiles<R, K, B>(n, span, load, body);
}

template<std::size_t R, unsigned U, class L, class F, class S>
inline void start_staged(std::size_t n, L load, F body, S bytes, cudaStream_t s, unsigned block,
                         std::size_t per_lane) noexcept {
  static_assert(std::is_trivially_copyable_v<L> && std::is_trivially_copyable_v<F>, "lanes cross as arguments");
  (void)U;  // a tile's barriers leave nothing to unroll
  if(!n) return;
  static const unsigned most = [] {  // the widest block both tile widths' kernels launch with
    const unsigned one = widest_block(region_staged<R, 1, L, F>);
    const unsigned wide = widest_block(region_staged<R, STAGE_WIDTHS, L, F>);
    return one < wide ? one : wide;
  }();
  if(block > most) block = most;
  if(block < WARP) block = WARP;
  auto launch = [&](auto kernel, std::size_t k, std::atomic<unsigned long long>& fit) {
    const std::size_t shared = bytes(k * block + 2 * R);
    if(shared > 48 * 1024)
      check(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, int(shared)));
    const std::size_t tiles = (n + k * block - 1) / (k * block);
    // a block's run: per_lane block widths (the plan's tiles per block) or STAGE_TILES widths, whichever is more
    const std::size_t asked = (per_lane + k - 1) / k;
    std::size_t span = asked > STAGE_TILES / k ? asked : STAGE_TILES / k;
    while((tiles + span - 1) / span > GRID_LIMIT) span *= 2;
    // a grid of at least the resident blocks (when there are tiles for them), each block `span` tiles or fewer
    const std::size_t resident = resident_blocks(fit, kernel, block, shared);
    const unsigned grid = region_grid(tiles, 1, span, resident);
    const std::size_t each = (tiles + grid - 1) / grid;
    kernel<<<grid, block, shared, s>>>(n, each, load, body);
    check(cudaGetLastError());
  };
  static std::atomic<unsigned long long> fit_128{0}, fit_256{0}, fit_wide{0}, fit_one{0};
  constexpr std::size_t LIMIT = 48 * 1024;
  if(block == 128 && bytes(STAGE_WIDE + 2 * R) <= LIMIT)
    launch(region_staged_fixed<R, STAGE_WIDE / 128, 128, L, F>, STAGE_WIDE / 128, fit_128);
  else if(block == 256 && bytes(STAGE_WIDE + 2 * R) <= LIMIT)
    launch(region_staged_fixed<R, STAGE_WIDE / 256, 256, L, F>, STAGE_WIDE / 256, fit_256);
  else if(bytes(STAGE_WIDTHS * block + 2 * R) <= LIMIT)
    launch(region_staged<R, STAGE_WIDTHS, L, F>, STAGE_WIDTHS, fit_wide);
  else
    launch(region_staged<R, 1, L, F>, 1, fit_one);
}

}  // namespace b200
}  // namespace cr::gpu

// Drop-in replacement for CAIRN's runtime/cairn_cub.hpp on a B200 (sm_100a): the machine's collectors, which the
// lowering includes only in a program with a device `reduce`, `scan` or `compact` (compiler/lower/region_lowering.py
// :7-36), and the older synchronous forms. Nothing here uses CUB (runtime/cairn_cub.hpp:14-25 calls DeviceReduce and
// DeviceScan).
//
// B200::reduce: one launch of a device-sized persistent grid. Each thread loads eight values of a tile, so eight loads
// per thread are in flight, before folding them in turn into its accumulators (eight for values of up to 4 bytes,
// four for wider ones); the accumulators fold pairwise, each warp folds by shuffles, the block's eight warp totals fold in warp 0, one
// partial per block goes to the scratch the context lends, and the last block to finish (an atomic ticket) folds
// the partials and stores the total. The order of the folds is fixed by n and the device; the operator must be
// associative and commutative, which every operator a device `reduce` admits is (+ over the checked Sum, add_wrap,
// *, min, max, &, |, ^).
//
// B200::inclusive_scan and exclusive_sum: one pass over the input with decoupled look-back (Merrill and Garland,
// "Single-pass Parallel Prefix Scan with Decoupled Look-back", NVIDIA technical report NVR-2016-002). Each block
// takes the next tile in launch order from an atomic counter, scans it in shared memory (coalesced rows in, each
// thread's contiguous segment in sequence, the segments' totals across the block), publishes its aggregate, looks
// back over its predecessors' published aggregates and inclusive prefixes, 32 tiles per step, until it meets an
// inclusive prefix, and publishes its own. The operator must be associative (commutativity is not assumed: every
// fold keeps the elements' order). Every wait for a predecessor is bounded; a block that waited longer than the
// limit folds the inputs before its tile itself, so the scan ends with the right answer whatever the scheduling.
#pragma once
#if defined(__CUDACC__)
#include <algorithm>
#include <cstdint>
#include <cstring>
#include <iterator>
#include <type_traits>
#include "cairn_gpu.hpp"
namespace cr::gpu {
namespace b200 {

constexpr unsigned FOLD_THREADS = 256;
constexpr unsigned FOLD_WARPS = FOLD_THREADS / 32;
// The grid: at most 128 blocks per SM (18,944 on a B200) for values of up to 8 bytes, 64 for wider ones, whose last
// block's fold of the partials reads twice the bytes per block.
template<class T> constexpr unsigned fold_blocks_per_sm() noexcept { return sizeof(T) <= 8 ? 128u : 64u; }
// Independent accumulators per thread: eight for values of up to 4 bytes, four for wider ones. Measured on a B200 at
// n = 2^30: an f32 fold with 8 ran 7.2-7.4 TB/s (4 or 16 no faster), a u64 fold over a 16-byte (value, flag)
// accumulator 7.4-7.5 with 4 and 7.0 with 8.
template<class T> constexpr unsigned fold_ways() noexcept { return sizeof(T) <= 4 ? 8u : 4u; }
// A thread's loads in flight per round, folded into its accumulators in turn: eight whatever the width. Measured on a
// B200 through the compiler-emitted checked u64 `reduce +` at n = 2^30 (16-byte accumulators): four loads a round
// 7.02 TB/s, eight 7.10, sixteen 7.10, eight with 64 blocks per SM 7.14 (CUB on the same box: 7.19); the f32 fold
// unchanged at 6.86-6.89.
constexpr unsigned FOLD_LOADS = 8;

inline std::size_t fold_partials_bytes(unsigned grid, std::size_t t_size) noexcept {
  return (std::size_t(grid) * t_size + 255) / 256 * 256;
}

// A value another block wrote, read past this SM's L1 (which does not see other SMs' writes).
template<class T> __device__ inline T read_fresh(const T* p) {
  T v;
  if constexpr(sizeof(T) % 4 == 0) {
    unsigned w[sizeof(T) / 4];
    const unsigned* src = reinterpret_cast<const unsigned*>(p);
#pragma unroll
    for(unsigned i = 0; i < sizeof(T) / 4; ++i) w[i] = __ldcg(src + i);
    std::memcpy(&v, w, sizeof(T));
  } else {
    unsigned char b[sizeof(T)];
    const volatile unsigned char* src = reinterpret_cast<const volatile unsigned char*>(p);
    for(unsigned i = 0; i < sizeof(T); ++i) b[i] = src[i];
    std::memcpy(&v, b, sizeof(T));
  }
  return v;
}

// The value `down` lanes above this one in the warp, moved a 32-bit word at a time (any trivially copyable T).
template<class T> __device__ inline T from_lane_above(const T& v, unsigned down) {
  constexpr unsigned WORDS = (sizeof(T) + 3) / 4;
  unsigned w[WORDS] = {};
  std::memcpy(w, &v, sizeof(T));
#pragma unroll
  for(unsigned i = 0; i < WORDS; ++i) w[i] = __shfl_down_sync(0xffffffffu, w[i], down);
  T r;
  std::memcpy(&r, w, sizeof(T));
  return r;
}

// A warp's fold of one value per lane: five shuffle steps, lane 0 holds the result.
template<class T, class Fold> __device__ inline T fold_warp(T v, Fold& fold) {
#pragma unroll
  for(unsigned down = 16; down; down >>= 1) v = fold(v, from_lane_above(v, down));
  return v;
}

// A block's fold of one value per thread: each warp by shuffles, then the eight warp totals by warp 0. Thread 0
// holds the result; every thread of the block must call it.
template<class T, class Fold> __device__ inline T fold_block(T v, Fold& fold, T identity, T* warp_totals) {
  v = fold_warp(v, fold);
  const unsigned lane = threadIdx.x % 32, warp = threadIdx.x / 32;
  if(lane == 0) warp_totals[warp] = v;
  __syncthreads();
  T r = identity;
  if(warp == 0) r = fold_warp(lane < FOLD_WARPS ? warp_totals[lane] : identity, fold);
  __syncthreads();  // warp_totals may be written again
  return r;
}

// The reduction: a persistent grid over tiles of L * FOLD_THREADS consecutive values, each thread loading its L values
// of a tile (coalesced: step k of a warp reads 32 consecutive values) before it folds them into its K accumulators in
// turn; the accumulators fold pairwise, the block folds by shuffles, one partial per block
// lands in the scratch, and the last block to arrive (an atomic ticket) folds the partials and stores the total.
// The order is fixed by n and the grid; every operator a device `reduce` admits is associative and commutative.
template<class T, class In, class Out, class Fold>
__global__ void __launch_bounds__(FOLD_THREADS)
    fold_kernel(In in, Out out, std::size_t n, Fold fold, T identity, T* partials, unsigned* ticket) {
  static_assert(alignof(T) <= 16, "a fold value fits the shared totals' alignment");
  constexpr unsigned K = fold_ways<T>(), L = FOLD_LOADS > K ? FOLD_LOADS : K;
  static_assert(L % K == 0, "each round's loads fold into the accumulators in turn");
  __shared__ __align__(16) unsigned char raw[FOLD_WARPS * sizeof(T)];
  __shared__ bool last;
  T* warp_totals = reinterpret_cast<T*>(raw);
  T acc[K];
#pragma unroll
  for(unsigned k = 0; k < K; ++k) acc[k] = identity;
  const std::size_t width = std::size_t(L) * FOLD_THREADS, whole = n / width;
  std::size_t tile = blockIdx.x;
#pragma unroll 1
  for(; tile < whole; tile += gridDim.x) {
    const std::size_t first = tile * width + threadIdx.x;
    T v[L];
#pragma unroll
    for(unsigned k = 0; k < L; ++k) v[k] = in[first + std::size_t(k) * FOLD_THREADS];
#pragma unroll
    for(unsigned k = 0; k < L; ++k) acc[k % K] = fold(acc[k % K], v[k]);
  }
  if(tile == whole)  // the partial tile, to the block the rotation hands it to
    for(std::size_t i = whole * width + threadIdx.x; i < n; i += FOLD_THREADS) acc[0] = fold(acc[0], in[i]);
#pragma unroll
  for(unsigned w = K / 2; w; w >>= 1)
#pragma unroll
    for(unsigned k = 0; k < w; ++k) acc[k] = fold(acc[k], acc[k + w]);
  const T mine = fold_block(acc[0], fold, identity, warp_totals);
  if(threadIdx.x == 0) {
    partials[blockIdx.x] = mine;
    __threadfence();
    last = atomicAdd(ticket, 1u) == gridDim.x - 1;
  }
  __syncthreads();
  if(!last) return;
  __threadfence();
  // the partials, K per thread at a time so that K reads are in flight
  const unsigned blocks = gridDim.x, rounds = blocks / (K * FOLD_THREADS);
  unsigned b = threadIdx.x;
#pragma unroll
  for(unsigned k = 0; k < K; ++k) acc[k] = identity;
#pragma unroll 1
  for(unsigned r = 0; r < rounds; ++r, b += K * FOLD_THREADS) {
    T v[K];
#pragma unroll
    for(unsigned k = 0; k < K; ++k) v[k] = read_fresh(partials + b + k * FOLD_THREADS);
#pragma unroll
    for(unsigned k = 0; k < K; ++k) acc[k] = fold(acc[k], v[k]);
  }
  T total = identity;
#pragma unroll
  for(unsigned k = 0; k < K; ++k) total = fold(total, acc[k]);
  for(; b < blocks; b += FOLD_THREADS) total = fold(total, read_fresh(partials + b));
  total = fold_block(total, fold, identity, warp_totals);
  if(threadIdx.x == 0) {
    *out = total;
    *ticket = 0u;
  }
}

// Blocks of one reduction: one per tile of n, at most fold_blocks_per_sm<T>() per SM. Measured on a B200 at n = 2^30
// (f32, 8 accumulators): 18,944 blocks ran 7.23 TB/s, 65,535 7.41 and one resident wave (1,184) 6.27; the grid
// stops at 18,944 so that the last block's fold of the partials stays a few microseconds.
template<class T> inline unsigned fold_grid(std::size_t n) noexcept {
  const std::size_t loads = FOLD_LOADS > fold_ways<T>() ? FOLD_LOADS : fold_ways<T>();
  const std::size_t width = loads * FOLD_THREADS, needed = (n + width - 1) / width;
  const std::size_t most = std::size_t(sm_count()) * fold_blocks_per_sm<T>();
  return unsigned(needed < most ? (needed ? needed : 1) : most);
}

// ---- scan ------------------------------------------------------------------------------------------------------

// A block scans a 64 KB tile held in shared memory (three blocks resident per SM). Eight worker warps load the tile
// in coalesced 32-element rows, then each thread scans its own contiguous segment of S elements in sequence
// (raking), the 256 segment totals are scanned across the block, and the workers write the rows out with their
// prefixes. A ninth warp starts the look-back over the predecessors as the tile starts, so it runs while the
// workers load and rake rather than after them.
constexpr unsigned SCAN_THREADS = 256;                   // the tile's workers: load, rake, write
constexpr unsigned SCAN_WARPS = SCAN_THREADS / 32;
constexpr unsigned SCAN_BLOCK = SCAN_THREADS + 32;       // and one more warp that looks back meanwhile
constexpr unsigned SCAN_BLOCKS_PER_SM = 3;
constexpr unsigned SCAN_LOAD_BATCH = 16;  // rows a warp loads per batch (two batches in flight)
constexpr std::uint64_t SCAN_WAIT_NS = 2000000000ull;  // how long a block waits for its predecessors

// Elements per thread's segment (and rows per warp): 64 KB of values per tile where the value allows, 16, 32 or 64
// (whole batches of SCAN_LOAD_BATCH rows).
template<class T> constexpr unsigned scan_segment() noexcept {
  constexpr std::size_t s = (64 * 1024) / (std::size_t(SCAN_THREADS) * sizeof(T));
  return s >= 64 ? 64u : s >= 32 ? 32u : 16u;
}
template<class T> constexpr std::size_t scan_tile() noexcept { return std::size_t(SCAN_THREADS) * scan_segment<T>(); }
// Shared memory holds element e at e + e / S: one pad per segment, so rows (32 consecutive elements) and segments
// (S consecutive elements, one per thread) are both read and written without bank conflicts.
template<class T> constexpr std::size_t scan_smem() noexcept {
  return (scan_tile<T>() + SCAN_THREADS) * sizeof(T) + SCAN_THREADS * sizeof(T) + SCAN_THREADS;
}
// The worker warps' own barrier (the look-back warp does not take part).
__device__ inline void workers_sync() { asm volatile("bar.sync 1, %0;" ::"n"(SCAN_THREADS) : "memory"); }
constexpr std::size_t round256(std::size_t b) noexcept { return (b + 255) / 256 * 256; }

// A value that may be absent (no identity is known to an inclusive scan).
template<class T> struct Part {
  T v;
  bool ok;
};

__device__ inline std::uint64_t globaltimer() {
  std::uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}
__device__ inline unsigned load_acquire(const unsigned* p) {
  unsigned v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ inline void store_release(unsigned* p, unsigned v) {
  asm volatile("st.release.gpu.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ inline unsigned long long load_acquire(const unsigned long long* p) {
  unsigned long long v;
  asm volatile("ld.acquire.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}
__device__ inline unsigned long long load_relaxed(const unsigned long long* p) {
  unsigned long long v;
  asm volatile("ld.relaxed.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}
__device__ inline void store_relaxed(unsigned long long* p, unsigned long long v) {
  asm volatile("st.relaxed.gpu.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}

// A warp shuffle of any trivially copyable value, a 32-bit word at a time; `move` shuffles one word.
template<class T, class Move> __device__ inline T shuffled(const T& v, Move move) {
  constexpr unsigned W = (sizeof(T) + 3) / 4;
  unsigned w[W] = {};
  std::memcpy(w, &v, sizeof(T));
#pragma unroll
  for(unsigned i = 0; i < W; ++i) w[i] = move(w[i]);
  T r;
  std::memcpy(&r, w, sizeof(T));
  return r;
}

// Tile states: 0 nothing yet, 1 its aggregate is published, 2 its inclusive prefix is published.
constexpr unsigned TILE_AGGREGATE = 1, TILE_PREFIX = 2;

// The tiles' published states and values. A value of four bytes or fewer shares one 64-bit word with its state (the
// state in the high half): one relaxed load gets both, and nothing else is read on the strength of it, so no fence
// is needed. A larger value sits in its own array (aggregate or inclusive prefix), written before the state word is
// released and read after it is acquired.
template<class T> struct TileStates {
  static constexpr bool PACKED = sizeof(T) <= 4;
  unsigned long long* words;  // PACKED
  unsigned* flags;            // otherwise
  T* aggregate;
  T* inclusive;
  __device__ void publish(std::size_t t, unsigned state, const T& v) const {
    if constexpr(PACKED) {
      unsigned bits = 0;
      std::memcpy(&bits, &v, sizeof(T));
      store_relaxed(words + t, (static_cast<unsigned long long>(state) << 32) | bits);
    } else {
      (state == TILE_PREFIX ? inclusive : aggregate)[t] = v;
      store_release(flags + t, state);
    }
  }
  // Tile t's state (0: not yet published) and, once published, its value.
  __device__ unsigned read(std::size_t t, T& v) const {
    if constexpr(PACKED) {
      const unsigned long long w = load_relaxed(words + t);
      const unsigned bits = static_cast<unsigned>(w);
      std::memcpy(&v, &bits, sizeof(T));
      return static_cast<unsigned>(w >> 32);
    } else {
      const unsigned f = load_acquire(flags + t);
      if(f) v = read_fresh(f == TILE_PREFIX ? inclusive + t : aggregate + t);
      return f;
    }
  }
};

// Lane 0's result: op over [begin, end) of the inputs, in order (the look-back's escape when a predecessor is late).
template<class T, class In, class Fold>
__device__ inline Part<T> fold_range_warp(In in, std::size_t begin, std::size_t end, Fold& fold, unsigned lane) {
  const std::size_t len = end - begin, per = (len + 31) / 32;
  const std::size_t lo = begin + std::min(len, per * lane), hi = begin + std::min(len, per * (lane + 1));
  Part<T> acc{T{}, false};
  for(std::size_t i = lo; i < hi; ++i) {
    const T x = T(in[i]);
    acc = acc.ok ? Part<T>{fold(acc.v, x), true} : Part<T>{x, true};
  }
#pragma unroll
  for(unsigned d = 1; d < 32; d <<= 1) {  // lane + d holds later elements
    const T o = shuffled(acc.v, [&](unsigned w) { return __shfl_down_sync(~0u, w, d); });
    const bool ook = __shfl_down_sync(~0u, acc.ok ? 1 : 0, d) && lane + d < 32;
    if(ook) acc = acc.ok ? Part<T>{fold(acc.v, o), true} : Part<T>{o, true};
  }
  return acc;
}

// Predecessors each lane of the looking-back warp reads per step (lane l reads the l-th nearest: one coalesced
// 256-byte read a step). Measured on a B200 at n = 2^30: 4 or 8 per lane read more lines per step at the frontier
// every look-back warp is reading, and ran slower.
constexpr unsigned LOOK_PER_LANE = 1;
// How long a looking-back lane sleeps between reads of a predecessor that has published nothing. Measured on a B200
// at n = 2^30 (u32 add_wrap, the kernel alone): 32 ns doubling to 128 ran 3973 GB/s, a fixed 512 ns 4375, 32 doubling
// to 1024 4293, to 2048 3796; starting the look-back only once the tile is loaded (3496) or raked (3415) was slower.
constexpr unsigned LOOK_PAUSE_NS = 512;

// Warp 0's look-back for tile t > 0: op over every element before the tile, in lane 0.
template<class T, class In, class Fold>
__device__ inline Part<T> look_back(In in, std::size_t t, std::size_t tile_elems, Fold& fold, const TileStates<T>& st,
                                    std::uint64_t wait_ns, unsigned lane) {
  constexpr int K = LOOK_PER_LANE;
  Part<T> run{T{}, false};
  long long end = static_cast<long long>(t) - 1;
  const std::uint64_t start = globaltimer();
  for(;;) {
    // lane l reads tiles end - K l - k for k = 0 (the newest) .. K - 1; before tile 0 nothing is missing
    T v[K];
    unsigned f[K];
#pragma unroll
    for(int k = 0; k < K; ++k) {
      const long long pred = end - K * static_cast<long long>(lane) - k;
      v[k] = T{};
      f[k] = pred >= 0 ? st.read(static_cast<std::size_t>(pred), v[k]) : TILE_PREFIX;
    }
    bool missing = false;
#pragma unroll
    for(int k = 0; k < K; ++k) {
      const long long pred = end - K * static_cast<long long>(lane) - k;
      // A lane whose predecessor has published nothing yet reads it again every LOOK_PAUSE_NS: about 444 blocks
      // (three per SM) look back at once, and polls any faster crowd L2 with reads of the lines being published.
      while(pred >= 0 && f[k] == 0) {
        if(globaltimer() - start > wait_ns) break;
        __nanosleep(LOOK_PAUSE_NS);
        f[k] = st.read(static_cast<std::size_t>(pred), v[k]);
      }
      missing = missing || f[k] == 0;
    }
    if(__any_sync(~0u, missing)) return fold_range_warp<T>(in, 0, t * tile_elems, fold, lane);
    int nearest = K;  // this lane's nearest predecessor holding a prefix (or standing before tile 0)
#pragma unroll
    for(int k = K - 1; k >= 0; --k)
      if(f[k] == TILE_PREFIX) nearest = k;
    const unsigned holders = __ballot_sync(~0u, nearest < K);
    const unsigned stop = holders ? __ffs(holders) - 1 : 31;  // the nearest lane holding one
    // this lane's share, oldest first: every tile newer than the nearest prefix in the window, and that prefix
    Part<T> mine{T{}, false};
    if(lane <= stop) {
      const int top = lane == stop ? nearest : K - 1;
#pragma unroll
      for(int k = K - 1; k >= 0; --k) {
        const long long pred = end - K * static_cast<long long>(lane) - k;
        if(k > top || pred < 0) continue;
        mine = mine.ok ? Part<T>{fold(mine.v, v[k]), true} : Part<T>{v[k], true};
      }
    }
    T w = mine.v;
    bool ok = mine.ok;
#pragma unroll
    for(unsigned d = 1; d < 32; d <<= 1) {  // lane + d holds earlier tiles
      const T o = shuffled(w, [&](unsigned x) { return __shfl_down_sync(~0u, x, d); });
      const bool ook = __shfl_down_sync(~0u, ok ? 1 : 0, d) && lane + d < 32;
      if(ook) {
        w = ok ? fold(o, w) : o;
        ok = true;
      }
    }
    if(ok) run = run.ok ? Part<T>{fold(w, run.v), true} : Part<T>{w, true};  // meaningful in lane 0
    if(holders) return run;
    end -= 32 * K;
  }
}

// One tile per block. Inclusive: out[i] = op over in[0..i]. Exclusive: out[0] = T{} and out[i] = op over in[0..i)
// (used for the exclusive sum, whose T{} is zero).
template<bool Exclusive, class T, class In, class Out, class Fold>
__global__ void __launch_bounds__(SCAN_BLOCK, SCAN_BLOCKS_PER_SM)
    scan_kernel(In in, Out out, std::size_t n, Fold fold, unsigned* next, TileStates<T> st, std::uint64_t wait_ns) {
  constexpr unsigned S = scan_segment<T>(), ROWS = S;  // each worker warp loads and writes S rows of 32
  constexpr std::size_t TILE = scan_tile<T>();
  extern __shared__ __align__(16) unsigned char scan_raw[];
  T* vals = reinterpret_cast<T*>(scan_raw);                    // the tile, element e at e + e / S
  T* seg = vals + TILE + SCAN_THREADS;                         // op over the tile before segment s, for each s
  bool* seg_ok = reinterpret_cast<bool*>(seg + SCAN_THREADS);  // whether seg[s] holds anything
  __shared__ unsigned tile_id;
  __shared__ __align__(16) unsigned char totals_raw[SCAN_WARPS * sizeof(T)];
  __shared__ __align__(16) unsigned char prior_raw[sizeof(T)];
  __shared__ bool prior_ok;
  T* totals = reinterpret_cast<T*>(totals_raw);
  T& prior = *reinterpret_cast<T*>(prior_raw);  // op over every tile before this one
  const unsigned warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  auto at = [](std::size_t e) { return e + e / S; };
  if(threadIdx.x == 0) tile_id = atomicAdd(next, 1u);  // tiles in the order blocks start: predecessors are running
  __syncthreads();
  const std::size_t t = tile_id, tile0 = t * TILE;
  const std::size_t valid = n - tile0 < TILE ? n - tile0 : TILE;  // elements of this tile inside the input
  const bool full = valid == TILE;

  if(warp == SCAN_WARPS) {  // the look-back warp: op over every tile before this one
    Part<T> p{T{}, false};
    if(t > 0) p = look_back<T>(in, t, TILE, fold, st, wait_ns, lane);
    if(lane == 0) {
      prior = p.v;
      prior_ok = p.ok;
    }
    __syncthreads();  // (1) the prefix is ready; the workers have published the tile's aggregate
    return;
  }

  // load: this warp's rows w S .. w S + S - 1, coalesced, a second batch in flight while one is stored
  {
    T y[2][SCAN_LOAD_BATCH];
    auto load = [&](T (&dst)[SCAN_LOAD_BATCH], unsigned r0) {
#pragma unroll
      for(unsigned r = 0; r < SCAN_LOAD_BATCH; ++r) {
        const std::size_t e = (std::size_t(warp) * ROWS + r0 + r) * 32 + lane;
        dst[r] = e < valid ? T(in[tile0 + e]) : T{};
      }
    };
    auto store = [&](const T (&src)[SCAN_LOAD_BATCH], unsigned r0) {
#pragma unroll
      for(unsigned r = 0; r < SCAN_LOAD_BATCH; ++r) vals[at((std::size_t(warp) * ROWS + r0 + r) * 32 + lane)] = src[r];
    };
    load(y[0], 0);
    if constexpr(ROWS == SCAN_LOAD_BATCH) {
      store(y[0], 0);
    } else {
      static_assert(ROWS % (2 * SCAN_LOAD_BATCH) == 0, "batches in pairs");
#pragma unroll 1
      for(unsigned r0 = 0; r0 < ROWS; r0 += 2 * SCAN_LOAD_BATCH) {
        load(y[1], r0 + SCAN_LOAD_BATCH);
        store(y[0], r0);
        if(r0 + 2 * SCAN_LOAD_BATCH < ROWS) load(y[0], r0 + 2 * SCAN_LOAD_BATCH);
        store(y[1], r0 + SCAN_LOAD_BATCH);
      }
    }
  }
  __syncwarp();  // a thread's segment (S elements: S / 32 of its warp's rows) holds only rows its own warp loaded

  // rake: this thread's segment, in order; its total
  const std::size_t s0 = std::size_t(threadIdx.x) * S;
  Part<T> mine{T{}, false};
  if(full) {
    T* v = vals + at(s0);  // a segment is contiguous in shared memory
    T acc = v[0];
#pragma unroll 16
    for(unsigned j = 1; j < S; ++j) v[j] = acc = fold(acc, v[j]);
    mine = Part<T>{acc, true};
  } else {
    for(unsigned j = 0; j < S && s0 + j < valid; ++j) {
      T& v = vals[at(s0 + j)];
      if(mine.ok) v = fold(mine.v, v);
      mine = Part<T>{v, true};
    }
  }
  // the segments before this one in the warp (an exclusive shuffle scan of the totals; lane - d holds earlier ones)
  Part<T> before{T{}, false};
  {
    T w = mine.v;
    bool ok = mine.ok;  // inclusive over lanes 0 .. lane
#pragma unroll
    for(unsigned d = 1; d < 32; d <<= 1) {
      const T o = shuffled(w, [&](unsigned x) { return __shfl_up_sync(~0u, x, d); });
      const bool ook = __shfl_up_sync(~0u, ok ? 1 : 0, d) && lane >= d;
      if(ook) {
        w = ok ? fold(o, w) : o;
        ok = true;
      }
    }
    const T ex = shuffled(w, [&](unsigned x) { return __shfl_up_sync(~0u, x, 1); });
    const bool ex_ok = __shfl_up_sync(~0u, ok ? 1 : 0, 1) && lane > 0;
    before = Part<T>{ex, ex_ok};
    if(lane == 31) totals[warp] = w;  // the warp's total (a warp with no valid element is never read)
  }
  workers_sync();  // every warp's total is in

  // the tile's aggregate, published at once for the tiles after this one
  Part<T> agg{T{}, false};
  if(threadIdx.x == 0) {
    for(unsigned w = 0; w < SCAN_WARPS; ++w)  // warp w's segments hold elements only if its first one does
      if(std::size_t(w) * 32 * S < valid) agg = agg.ok ? Part<T>{fold(agg.v, totals[w]), true} : Part<T>{totals[w], true};
    if(full && t > 0) st.publish(t, TILE_AGGREGATE, agg.v);
  }
  __syncthreads();  // (1) with the look-back warp: `prior` is known
  if(threadIdx.x == 0 && full) st.publish(t, TILE_PREFIX, prior_ok ? fold(prior, agg.v) : agg.v);

  // this segment's prefix: the tiles before, the warps before, the segments before in this warp
  {
    Part<T> q{prior, prior_ok};
    for(unsigned w = 0; w < warp; ++w) q = q.ok ? Part<T>{fold(q.v, totals[w]), true} : Part<T>{totals[w], true};
    if(before.ok) q = q.ok ? Part<T>{fold(q.v, before.v), true} : before;
    seg[threadIdx.x] = q.v;
    seg_ok[threadIdx.x] = q.ok;
  }
  workers_sync();

  // write: this warp's rows again, each element with its segment's prefix. A whole tile of an inclusive scan takes a
  // loop with no bounds test and 32-bit offsets (a tile holds at most 16,384 elements), which unrolls.
  if constexpr(!Exclusive) {
    if(full) {
#pragma unroll 8
      for(unsigned r = 0; r < ROWS; ++r) {
        const unsigned e = (warp * ROWS + r) * 32 + lane, s = e / S;
        const T v = vals[e + s];
        out[tile0 + e] = seg_ok[s] ? fold(seg[s], v) : v;
      }
      return;
    }
  }
  for(unsigned r = 0; r < ROWS; ++r) {
    const std::size_t e = (std::size_t(warp) * ROWS + r) * 32 + lane;
    if(e >= valid) break;
    if constexpr(Exclusive) {  // the inclusive prefix of the element before
      if(e == 0) {
        out[tile0] = prior_ok ? prior : T{};
      } else {
        const std::size_t p = e - 1, s = p / S;
        const T v = vals[at(p)];
        out[tile0 + e] = seg_ok[s] ? fold(seg[s], v) : v;
      }
    } else {
      const std::size_t s = e / S;
      const T v = vals[at(e)];
      out[tile0 + e] = seg_ok[s] ? fold(seg[s], v) : v;
    }
  }
}

// The scan's scratch: the tile counter, then one 64-bit state-and-value word per tile (values of four bytes or
// fewer), or one state word per tile and each tile's aggregate and inclusive prefix (larger values).
template<class T> inline std::size_t scan_tiles(std::size_t n) noexcept { return (n + scan_tile<T>() - 1) / scan_tile<T>(); }
template<class T> inline std::size_t scan_head_bytes(std::size_t n) noexcept {
  return 256 + round256(scan_tiles<T>(n) * (TileStates<T>::PACKED ? 8 : 4));
}
template<class T> inline std::size_t scan_scratch_bytes(std::size_t n) noexcept {
  return scan_head_bytes<T>(n) + (TileStates<T>::PACKED ? 0 : 2 * round256(scan_tiles<T>(n) * sizeof(T)));
}

template<bool Exclusive, class T, class In, class Out, class Fold>
void scan(void* temp, std::size_t& bytes, In in, Out out, std::size_t n, Fold fold, cudaStream_t s,
          std::uint64_t wait_ns = SCAN_WAIT_NS) noexcept {
  static_assert(std::is_trivially_copyable_v<T>, "a scanned value crosses lanes as words");
  if(temp == nullptr) {  // the context asks how much scratch the scan needs
    bytes = scan_scratch_bytes<T>(n);
    return;
  }
  if(!n) return;
  const std::size_t tiles = scan_tiles<T>(n);
  if(tiles > 0x7fffffffull) trap();
  char* base = static_cast<char*>(temp);
  const std::size_t head = scan_head_bytes<T>(n), cells = round256(tiles * sizeof(T));
  TileStates<T> st{};
  st.words = reinterpret_cast<unsigned long long*>(base + 256);
  st.flags = reinterpret_cast<unsigned*>(base + 256);
  st.aggregate = reinterpret_cast<T*>(base + head);
  st.inclusive = reinterpret_cast<T*>(base + head + cells);
  static const bool sized = [] {  // the tile's dynamic shared memory, above the 48 KB default
    check(cudaFuncSetAttribute(scan_kernel<Exclusive, T, In, Out, Fold>,
                               cudaFuncAttributeMaxDynamicSharedMemorySize, int(scan_smem<T>())));
    check(cudaFuncSetAttribute(scan_kernel<Exclusive, T, In, Out, Fold>,
                               cudaFuncAttributePreferredSharedMemoryCarveout, 100));  // room for three tiles
    return true;
  }();
  (void)sized;
  check(cudaMemsetAsync(base, 0, head, s));  // the counter and every tile's state start at zero
  scan_kernel<Exclusive, T><<<unsigned(tiles), SCAN_BLOCK, scan_smem<T>(), s>>>(
      in, out, n, fold, reinterpret_cast<unsigned*>(base), st, wait_ns);
  check(cudaGetLastError());
}

struct Plus {
  template<class T> __device__ T operator()(T a, T b) const { return static_cast<T>(a + b); }
};

}  // namespace b200

template<class In, class Out, class Fold, class T>
void B200::reduce(void* temp, std::size_t& bytes, In in, Out out, std::size_t n, Fold fold, T identity,
                  Stream s) noexcept {
  const unsigned grid = b200::fold_grid<T>(n);
  const std::size_t partials = b200::fold_partials_bytes(grid, sizeof(T));
  if(temp == nullptr) {  // the context asks how much scratch the reduction needs
    bytes = partials + 256;
    return;
  }
  T* cells = static_cast<T*>(temp);
  unsigned* ticket = reinterpret_cast<unsigned*>(static_cast<char*>(temp) + partials);
  check(cudaMemsetAsync(ticket, 0, sizeof(unsigned), s));  // arena scratch holds whatever its last user left
  b200::fold_kernel<T><<<grid, b200::FOLD_THREADS, 0, s>>>(in, out, n, fold, identity, cells, ticket);
  check(cudaGetLastError());
}
template<class In, class Out, class Fold>
void B200::inclusive_scan(void* temp, std::size_t& bytes, In in, Out out, Fold fold, std::size_t n,
                          Stream s) noexcept {
  b200::scan<false, typename std::iterator_traits<In>::value_type>(temp, bytes, in, out, n, fold, s);
}
// The offsets accumulate in the output's type (a count of selected elements can exceed the flags' type).
template<class In, class Out>
void B200::exclusive_sum(void* temp, std::size_t& bytes, In in, Out out, std::size_t n, Stream s) noexcept {
  b200::scan<true, typename std::iterator_traits<Out>::value_type>(temp, bytes, in, out, n, b200::Plus{}, s);
}

// The older synchronous collectors, kept for programs that still call them: each runs the context form of
// runtime/cairn_exec.hpp on the calling thread's context and then waits for the whole device, as they always did.
template<class T, class Op, class F> inline T reduce(std::size_t n, T identity, Op op, F value) noexcept {
  const T total = reduce_on(here(), n, identity, op, value);
  check(cudaDeviceSynchronize());
  return total;
}
template<bool Exclusive, class T, class R, class Op, class F>
inline T scan(R* out, std::size_t n, T identity, Op op, F value) noexcept {
  const T total = scan_on<Exclusive>(here(), out, n, identity, op, value);
  check(cudaDeviceSynchronize());
  return total;
}
template<class T, class P, class F>
inline std::size_t compact(T* out, std::size_t n, P pred, F value) noexcept {
  const std::size_t used = compact_on(here(), out, n, pred, value);
  check(cudaDeviceSynchronize());
  return used;
}
}  // namespace cr::gpu
#endif

// Drop-in replacement for CAIRN's runtime/cairn_cub.hpp on a B200 (sm_100a): the machine's collectors, which the
// lowering includes only in a program with a device `reduce`, `scan` or `compact` (compiler/lower/region_lowering.py
// :7-36), and the older synchronous forms. Nothing here uses CUB (runtime/cairn_cub.hpp:14-25 calls DeviceReduce and
// DeviceScan).
//
// B200::reduce: one launch of a device-sized persistent grid, each thread folding a grid-strided run of value(i) in
// registers, a shared-memory tree per block, one partial per block in the scratch the context lends, and the last
// block to finish (an atomic ticket) folding the partials and storing the total. The order of the folds is fixed by
// n and the device; the operator must be associative and commutative, which every operator a device `reduce` admits
// is (+ over the checked Sum, add_wrap, *, min, max, &, |, ^).
//
// B200::inclusive_scan and exclusive_sum: one pass over the input with decoupled look-back (Merrill and Garland,
// "Single-pass Parallel Prefix Scan with Decoupled Look-back", NVIDIA technical report NVR-2016-002). Each block
// takes the next tile in launch order from an atomic counter, scans it in registers (eight warps, each a contiguous
// run of 32-element rows: a shuffle scan per row, carried row to row), publishes the tile's aggregate, then looks
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

// Blocks of a reduction over n values on the current device: no more than the work needs, four per SM at most.
inline unsigned fold_grid(std::size_t n) noexcept {
  const std::size_t needed = (n + FOLD_THREADS - 1) / FOLD_THREADS;
  const std::size_t most = std::size_t(sm_count()) * 4;
  return unsigned(needed < most ? (needed ? needed : 1) : most);
}
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

// The block's fold of one value per thread, in thread order pairs; thread 0 holds it on return.
template<class T, class Fold> __device__ inline T fold_block(T v, Fold& fold, T* shared) {
  shared[threadIdx.x] = v;
  __syncthreads();
  for(unsigned w = FOLD_THREADS / 2; w; w >>= 1) {
    if(threadIdx.x < w) shared[threadIdx.x] = fold(shared[threadIdx.x], shared[threadIdx.x + w]);
    __syncthreads();
  }
  const T r = shared[0];
  __syncthreads();
  return r;
}

template<class T, class In, class Out, class Fold>
__global__ void __launch_bounds__(FOLD_THREADS)
    fold_kernel(In in, Out out, std::size_t n, Fold fold, T identity, T* partials, unsigned* ticket) {
  static_assert(alignof(T) <= 16, "a fold value fits the shared tree's alignment");
  __shared__ __align__(16) unsigned char raw[FOLD_THREADS * sizeof(T)];
  __shared__ bool last;
  T* shared = reinterpret_cast<T*>(raw);
  const std::size_t stride = std::size_t(gridDim.x) * FOLD_THREADS;
  T acc = identity;
  for(std::size_t i = blockIdx.x * std::size_t(FOLD_THREADS) + threadIdx.x; i < n; i += stride) acc = fold(acc, in[i]);
  acc = fold_block(acc, fold, shared);
  if(threadIdx.x == 0) {
    partials[blockIdx.x] = acc;
    __threadfence();
    last = atomicAdd(ticket, 1u) == gridDim.x - 1;
  }
  __syncthreads();
  if(!last) return;
  __threadfence();
  T total = identity;
  for(unsigned b = threadIdx.x; b < gridDim.x; b += FOLD_THREADS) total = fold(total, read_fresh(partials + b));
  total = fold_block(total, fold, shared);
  if(threadIdx.x == 0) {
    *out = total;
    *ticket = 0u;
  }
}

// ---- scan ------------------------------------------------------------------------------------------------------

constexpr unsigned SCAN_THREADS = 256;
constexpr unsigned SCAN_WARPS = SCAN_THREADS / 32;
constexpr std::uint64_t SCAN_WAIT_NS = 2000000000ull;  // how long a block waits for its predecessors

// Rows of 32 elements each warp scans: 64 bytes of values per lane.
template<class T> constexpr unsigned scan_rows() noexcept { return sizeof(T) <= 4 ? 16u : sizeof(T) <= 8 ? 8u : 4u; }
template<class T> constexpr std::size_t scan_tile() noexcept { return std::size_t(SCAN_THREADS) * scan_rows<T>(); }
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

// Warp 0's look-back for tile t > 0: op over every element before the tile, in lane 0.
template<class T, class In, class Fold>
__device__ inline Part<T> look_back(In in, std::size_t t, std::size_t tile_elems, Fold& fold, const unsigned* flags,
                                    const T* aggregate, const T* inclusive, std::uint64_t wait_ns, unsigned lane) {
  Part<T> run{T{}, false};
  long long end = static_cast<long long>(t) - 1;
  const std::uint64_t start = globaltimer();
  for(;;) {
    const long long pred = end - static_cast<long long>(lane);
    unsigned f = TILE_PREFIX;  // before tile 0 nothing is missing
    if(pred >= 0) {
      while((f = load_acquire(flags + pred)) == 0)
        if(globaltimer() - start > wait_ns) break;
    }
    if(__any_sync(~0u, f == 0)) return fold_range_warp<T>(in, 0, t * tile_elems, fold, lane);
    T v = T{};
    if(pred >= 0) v = read_fresh(f == TILE_PREFIX ? inclusive + pred : aggregate + pred);
    const unsigned prefixes = __ballot_sync(~0u, f == TILE_PREFIX);
    const unsigned stop = prefixes ? __ffs(prefixes) - 1 : 31;  // the nearest predecessor holding a prefix
    bool ok = pred >= 0 && lane <= stop;
#pragma unroll
    for(unsigned d = 1; d < 32; d <<= 1) {  // lane + d holds earlier tiles
      const T o = shuffled(v, [&](unsigned w) { return __shfl_down_sync(~0u, w, d); });
      const bool ook = __shfl_down_sync(~0u, ok ? 1 : 0, d) && lane + d < 32;
      if(ook) {
        v = ok ? fold(o, v) : o;
        ok = true;
      }
    }
    if(ok) run = run.ok ? Part<T>{fold(v, run.v), true} : Part<T>{v, true};  // meaningful in lane 0
    if(prefixes) return run;
    end -= 32;
  }
}

// One tile per block. Inclusive: out[i] = op over in[0..i]. Exclusive: out[0] = T{} and out[i] = op over in[0..i)
// (used for the exclusive sum, whose T{} is zero).
template<bool Exclusive, class T, class In, class Out, class Fold>
__global__ void __launch_bounds__(SCAN_THREADS)
    scan_kernel(In in, Out out, std::size_t n, Fold fold, unsigned* next, unsigned* flags, T* aggregate,
                T* inclusive, std::uint64_t wait_ns) {
  constexpr unsigned ROWS = scan_rows<T>();
  constexpr std::size_t TILE = scan_tile<T>(), RUN = std::size_t(32) * ROWS;
  __shared__ unsigned tile_id;
  __shared__ __align__(16) unsigned char totals_raw[SCAN_WARPS * sizeof(T)];
  __shared__ __align__(16) unsigned char prefix_raw[(SCAN_WARPS + 1) * sizeof(T)];
  __shared__ bool prefix_ok[SCAN_WARPS + 1];
  T* totals = reinterpret_cast<T*>(totals_raw);
  T* prefix = reinterpret_cast<T*>(prefix_raw);  // [w]: op over the tile's warps before w; [SCAN_WARPS]: the tile's
  const unsigned warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  if(threadIdx.x == 0) tile_id = atomicAdd(next, 1u);  // tiles in the order blocks start: predecessors are running
  __syncthreads();
  const std::size_t t = tile_id, tile0 = t * TILE, run0 = tile0 + warp * RUN;

  T y[ROWS];
#pragma unroll
  for(unsigned r = 0; r < ROWS; ++r) {
    const std::size_t i = run0 + r * 32 + lane;
    y[r] = i < n ? T(in[i]) : T{};
  }
  T carry{};
#pragma unroll
  for(unsigned r = 0; r < ROWS; ++r) {
    const bool valid = run0 + r * 32 + lane < n;
#pragma unroll
    for(unsigned d = 1; d < 32; d <<= 1) {
      const T o = shuffled(y[r], [&](unsigned w) { return __shfl_up_sync(~0u, w, d); });
      if(lane >= d && valid) y[r] = fold(o, y[r]);
    }
    if(r > 0 && valid) y[r] = fold(carry, y[r]);
    carry = shuffled(y[r], [&](unsigned w) { return __shfl_sync(~0u, w, 31); });
  }
  if(lane == 0) totals[warp] = carry;
  __syncthreads();

  if(warp == 0) {
    const bool full = tile0 + TILE <= n;
    Part<T> agg{T{}, false};
    if(lane == 0) {
      for(unsigned w = 0; w < SCAN_WARPS; ++w) {
        prefix[w] = agg.v;
        prefix_ok[w] = agg.ok;
        // a run the input ends inside (or before) is the last that holds elements: its total is not needed
        if(tile0 + (w + 1) * RUN <= n)
          agg = agg.ok ? Part<T>{fold(agg.v, totals[w]), true} : Part<T>{totals[w], true};
      }
      if(full) {
        if(t == 0) {
          inclusive[0] = agg.v;
          store_release(flags, TILE_PREFIX);
        } else {
          aggregate[t] = agg.v;
          store_release(flags + t, TILE_AGGREGATE);
        }
      }
    }
    Part<T> before{T{}, false};
    if(t > 0) before = look_back<T>(in, t, TILE, fold, flags, aggregate, inclusive, wait_ns, lane);
    if(lane == 0) {
      if(full && t > 0) {
        inclusive[t] = before.ok ? fold(before.v, agg.v) : agg.v;
        store_release(flags + t, TILE_PREFIX);
      }
      prefix[SCAN_WARPS] = before.v;
      prefix_ok[SCAN_WARPS] = before.ok;
    }
  }
  __syncthreads();

  // op over everything before this warp's run, then into each element
  Part<T> q{prefix[SCAN_WARPS], prefix_ok[SCAN_WARPS]};
  if(prefix_ok[warp]) q = q.ok ? Part<T>{fold(q.v, prefix[warp]), true} : Part<T>{prefix[warp], true};
  if(q.ok) {
#pragma unroll
    for(unsigned r = 0; r < ROWS; ++r)
      if(run0 + r * 32 + lane < n) y[r] = fold(q.v, y[r]);
  }
#pragma unroll
  for(unsigned r = 0; r < ROWS; ++r) {
    const std::size_t i = run0 + r * 32 + lane;
    if constexpr(Exclusive) {
      const T up = shuffled(y[r], [&](unsigned w) { return __shfl_up_sync(~0u, w, 1); });
      const T last = shuffled(r ? y[r - 1] : y[0], [&](unsigned w) { return __shfl_sync(~0u, w, 31); });
      if(i < n) out[i] = lane ? up : (r ? last : (q.ok ? q.v : T{}));
    } else {
      if(i < n) out[i] = y[r];
    }
  }
}

// The scan's scratch: the tile counter, one state word per tile, then each tile's aggregate and inclusive prefix.
template<class T> inline std::size_t scan_scratch_bytes(std::size_t n) noexcept {
  const std::size_t tiles = (n + scan_tile<T>() - 1) / scan_tile<T>();
  return 256 + round256(tiles * 4) + 2 * round256(tiles * sizeof(T));
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
  const std::size_t tiles = (n + scan_tile<T>() - 1) / scan_tile<T>();
  if(tiles > 0x7fffffffull) trap();
  char* base = static_cast<char*>(temp);
  const std::size_t head = 256 + round256(tiles * 4), cells = round256(tiles * sizeof(T));
  unsigned* next = reinterpret_cast<unsigned*>(base);
  unsigned* flags = reinterpret_cast<unsigned*>(base + 256);
  T* aggregate = reinterpret_cast<T*>(base + head);
  T* inclusive = reinterpret_cast<T*>(base + head + cells);
  check(cudaMemsetAsync(base, 0, head, s));  // the counter and every tile's state start at zero
  scan_kernel<Exclusive, T><<<unsigned(tiles), SCAN_THREADS, 0, s>>>(in, out, n, fold, next, flags, aggregate,
                                                                     inclusive, wait_ns);
  check(cudaGetLastError());
}

struct Plus {
  template<class T> __device__ T operator()(T a, T b) const { return static_cast<T>(a + b); }
};

}  // namespace b200

template<class In, class Out, class Fold, class T>
void B200::reduce(void* temp, std::size_t& bytes, In in, Out out, std::size_t n, Fold fold, T identity,
                  Stream s) noexcept {
  const unsigned grid = b200::fold_grid(n);
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

// Drop-in replacement for CAIRN's runtime/cairn_cub.hpp on a B200 (sm_100a): the machine's collectors, which the
// lowering includes only in a program with a device `reduce`, `scan` or `compact` (compiler/lower/region_lowering.py
// :7-36), and the older synchronous forms.
//
// B200::reduce is this project's kernel, not CUB's DeviceReduce (runtime/cairn_cub.hpp:14-17): one launch of a
// device-sized persistent grid, each thread folding a grid-strided run of value(i) in registers, a shared-memory
// tree per block, one partial per block in the scratch the context lends, and the last block to finish (an atomic
// ticket) folding the partials and storing the total. The order of the folds is fixed by n and the device; the
// operator must be associative and commutative, which every operator a device `reduce` admits is (+ over the
// checked Sum, add_wrap, *, min, max, &, |, ^). The scans stay on CUB (the next step on this path).
#pragma once
#if defined(__CUDACC__)
#include <cstring>
#include <cub/device/device_scan.cuh>
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
  check(cub::DeviceScan::InclusiveScan(temp, bytes, in, out, fold, n, s));
}
template<class In, class Out>
void B200::exclusive_sum(void* temp, std::size_t& bytes, In in, Out out, std::size_t n, Stream s) noexcept {
  check(cub::DeviceScan::ExclusiveSum(temp, bytes, in, out, n, s));
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

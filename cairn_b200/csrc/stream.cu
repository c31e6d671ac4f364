// The bandwidth-bound half of the hot path: the `parallel` saxpy region and the `reduce +` collectors over f32 and
// u64, rebuilt for sm_100a.
//
// The reference runs a `parallel` region as one index per thread in a grid of at most 65535 blocks of 256 threads,
// scalar 4-byte accesses (runtime/cairn_kernels.hpp:69-96), and a device `reduce +` through CUB's DeviceReduce with
// temporaries from the context's arena (runtime/cairn_reuse.hpp:346-372, runtime/cairn_cub.hpp:14-17). Here:
//   - saxpy: one 16-byte vector of each operand per thread, in 1024-thread blocks, a block per 4096 elements, with
//     streaming cache hints (each byte is touched once). Measured on a B200 at n = 2^30 over random values (all-zero
//     inputs stream faster and mislead): 7.2 TB/s, where two resident 512-thread blocks per SM striding over four
//     vectors per step ran 6.1-6.3: with short blocks the SMs finish together;
//   - the reductions fold each thread's terms into registers, then a warp shuffle tree, a shared-memory tree across
//     the block's 16 warps, one partial per block in scratch, and the last block to finish (an atomic ticket, no
//     spin-wait) folds the partials in block order and writes the total. One launch, deterministic for a given n
//     and device: every thread's terms and every tree are fixed by (n, grid). Each reduction's grid is the one that
//     ran fastest at n = 2^30 (random values) among 2 to 64 blocks per SM: 8 per SM for the f32 sum (6.8 TB/s; its
//     double-double additions keep two 512-thread blocks resident), 32 for the u64 sum (7.4), 2 for the loss (6.8).
//   - f32 terms are added in f64, which holds every f32 term exactly; the total is rounded to f32 once.
//   - u64 terms carry cr::Sum's sticky overflow flag (runtime/cairn_runtime.hpp:158-166) through every fold.
#include <cstdint>
#include <cstring>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include "gemm.h"
#include "ptx.cuh"

namespace cb {

int sum_f32_grid(int sms) { return 8 * sms; }
int sum_u64_grid(int sms) { return 32 * sms; }
int mse_grid(int sms) { return 2 * sms; }
// The ticket (256 bytes, zero between launches), then one 32-byte partial per block of the widest reduction grid.
std::size_t reduce_scratch_bytes(int sms) { return 256 + static_cast<std::size_t>(sum_u64_grid(sms)) * 32; }

namespace {

constexpr int T = STREAM_THREADS;
constexpr int WARPS = T / 32;
constexpr int UNROLL = 4;
constexpr int SAXPY_THREADS = 1024;

// The ticket sits at the start of the scratch and the partials after it, wherever each launch's grid ends.
unsigned int* ticket_of(void* scratch) { return static_cast<unsigned int*>(scratch); }
template <class P> P* partials_of(void* scratch) { return reinterpret_cast<P*>(static_cast<char*>(scratch) + 256); }

__device__ __forceinline__ float saxpy1(float a, float x, float y) { return __fadd_rn(__fmul_rn(a, x), y); }

// out may equal x or y: each vector is read before the same vector is written. One vector per thread, a block per
// 4096 elements (the launcher refuses an n whose grid would not fit, past 2^43 elements); the last block also runs
// the n % 4 elements past the last whole vector. A grid-stride loop over the same grid measured 12 % slower.
__global__ void __launch_bounds__(SAXPY_THREADS)
    saxpy_vec_kernel(std::size_t n, float* out, const float* x, const float* y, float a) {
  const std::size_t n4 = n / 4, i = static_cast<std::size_t>(blockIdx.x) * SAXPY_THREADS + threadIdx.x;
  if (i < n4) {
    const float4 xv = __ldcs(reinterpret_cast<const float4*>(x) + i);
    const float4 yv = __ldcs(reinterpret_cast<const float4*>(y) + i);
    __stcs(reinterpret_cast<float4*>(out) + i, make_float4(saxpy1(a, xv.x, yv.x), saxpy1(a, xv.y, yv.y),
                                                         saxpy1(a, xv.z, yv.z), saxpy1(a, xv.w, yv.w)));
  }
  if (blockIdx.x == gridDim.x - 1 && threadIdx.x < n - n4 * 4) {
    const std::size_t j = n4 * 4 + threadIdx.x;
    out[j] = saxpy1(a, x[j], y[j]);
  }
}

// Views off 16 bytes: 4-byte accesses, about 64 per thread (the grid-stride shape a plain region runs fastest in).
__global__ void __launch_bounds__(256)
    saxpy_scalar_kernel(std::size_t n, float* out, const float* x, const float* y, float a) {
  const std::size_t stride = static_cast<std::size_t>(gridDim.x) * blockDim.x;
  for (std::size_t i = static_cast<std::size_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n; i += stride)
    out[i] = saxpy1(a, x[i], y[i]);
}

// ---- f32 sum --------------------------------------------------------------------------------------------------
// The host's `reduce + parallel` over f32 is the exact sum rounded once (runtime/cairn_sum.hpp:1-17). The device
// keeps that answer: each thread runs four double-double accumulators (s, c), where Knuth's TwoSum adds a term to s
// and moves the rounding error, exactly, into c; the trees combine double-doubles the same way, and the total is
// rounded to f32 from the double-double with the tie decided by its low part. A term that is an infinity or a NaN
// leaves a non-finite s or c, and only such a term does (finite f32 terms cannot overflow f64); such a thread looks
// at its terms again for the flags cr::sum::result reads (runtime/cairn_sum.hpp:186-195). OTHER marks a term that is
// not -0.0: an exact zero total is -0.0 only when every term was.
enum : unsigned { SUM_NAN = 1, SUM_PINF = 2, SUM_NINF = 4, SUM_OTHER = 8, SUM_SOME = 16 };

struct DD {
  double s, c;
};
struct Partial {  // one block's part, in scratch (32 bytes)
  double s, c;
  unsigned flags, pad[3];
};

__device__ __forceinline__ void two_sum_into(double& s, double& c, double x) {
  const double t = __dadd_rn(s, x);
  const double z = __dsub_rn(t, s);
  c = __dadd_rn(c, __dadd_rn(__dsub_rn(s, __dsub_rn(t, z)), __dsub_rn(x, z)));
  s = t;
}
__device__ __forceinline__ DD dd_add(DD p, DD q) {
  double s = p.s, c = __dadd_rn(p.c, q.c);
  two_sum_into(s, c, q.s);
  return {s, c};
}
__device__ __forceinline__ DD warp_dd(DD v) {
#pragma unroll
  for (int off = 16; off; off >>= 1) {
    DD o;
    o.s = __shfl_xor_sync(0xffffffffu, v.s, off);
    o.c = __shfl_xor_sync(0xffffffffu, v.c, off);
    v = dd_add(v, o);
  }
  return v;
}
__device__ __forceinline__ unsigned warp_or(unsigned f) {
#pragma unroll
  for (int off = 16; off; off >>= 1) f |= __shfl_xor_sync(0xffffffffu, f, off);
  return f;
}
// The block's double-double and flags, held by every thread of warp 0 on return.
__device__ __forceinline__ void block_dd(DD& v, unsigned& flags, DD* sv, unsigned* sf) {
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  v = warp_dd(v);
  flags = warp_or(flags);
  if (lane == 0) {
    sv[warp] = v;
    sf[warp] = flags;
  }
  __syncthreads();
  if (warp == 0) {
    v = lane < WARPS ? sv[lane] : DD{-0.0, -0.0};
    flags = lane < WARPS ? sf[lane] : 0u;
    v = warp_dd(v);
    flags = warp_or(flags);
  }
  __syncthreads();
}

// The f32 nearest (ties to even) to the exact value hi + lo, where hi = RN(hi + lo) in f64.
__device__ float round_dd_f32(double hi, double lo) {
  const float f = __double2float_rn(hi);
  if (lo == 0.0) return f;
  if (isinf(f)) {  // hi is at or past the overflow threshold: only the threshold itself can still go back down
    const double threshold = 3.4028235677973366e38;  // FLT_MAX + 2^103, the midpoint to 2^128
    return (fabs(hi) == threshold && ((lo < 0.0) == (hi > 0.0))) ? copysignf(3.4028234663852886e38f, f) : f;
  }
  const double fd = static_cast<double>(f);
  if (fd == hi) return f;  // |lo| is below half an f64 ulp of hi, far below half an f32 ulp
  const float g = hi > fd ? nextafterf(f, INFINITY) : nextafterf(f, -INFINITY);
  const double gd = static_cast<double>(g);
  if (__dsub_rn(hi, fd) == __dsub_rn(gd, hi)) return ((lo > 0.0) == (gd > fd)) ? g : f;  // hi is the midpoint
  return f;
}

template <bool VEC, class F>
__device__ __forceinline__ void for_terms(std::size_t n, const float* x, F&& term) {
  const std::size_t stride = static_cast<std::size_t>(gridDim.x) * T;
  std::size_t i = static_cast<std::size_t>(blockIdx.x) * T + threadIdx.x;
  if constexpr (VEC) {
    const std::size_t n4 = n / 4;
    const float4* x4 = reinterpret_cast<const float4*>(x);
    for (; i + (UNROLL - 1) * stride < n4; i += UNROLL * stride) {
      float4 v[UNROLL];
#pragma unroll
      for (int u = 0; u < UNROLL; ++u) v[u] = __ldcs(x4 + i + u * stride);
#pragma unroll
      for (int u = 0; u < UNROLL; ++u) {
        term(0, v[u].x);
        term(1, v[u].y);
        term(2, v[u].z);
        term(3, v[u].w);
      }
    }
    for (; i < n4; i += stride) {
      const float4 v = __ldcs(x4 + i);
      term(0, v.x);
      term(1, v.y);
      term(2, v.z);
      term(3, v.w);
    }
    i = n4 * 4 + static_cast<std::size_t>(blockIdx.x) * T + threadIdx.x;
  }
  for (; i < n; i += stride) term(0, __ldcs(x + i));
}

template <bool VEC>
__global__ void __launch_bounds__(T, 2) sum_f32_kernel(std::size_t n, const float* x, float* out_f32,
                                                      double* out_f64, Partial* partials, unsigned int* ticket) {
  __shared__ DD sv[WARPS];
  __shared__ unsigned sf[WARPS];
  __shared__ bool last;
  // -0.0 is the identity of IEEE addition: a chain that only ever adds -0.0 terms stays -0.0.
  double s[4] = {-0.0, -0.0, -0.0, -0.0}, c[4] = {-0.0, -0.0, -0.0, -0.0};
  for_terms<VEC>(n, x, [&](int q, float v) { two_sum_into(s[q], c[q], static_cast<double>(v)); });
  unsigned flags = 0;
  bool special = false;
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    special |= !isfinite(s[q]) || !isfinite(c[q]);
    if (__double_as_longlong(s[q]) != static_cast<long long>(0x8000000000000000ull)) flags |= SUM_OTHER;
  }
  DD v = dd_add(dd_add(DD{s[0], c[0]}, DD{s[1], c[1]}), dd_add(DD{s[2], c[2]}, DD{s[3], c[3]}));
  if (special) {  // an infinity or a NaN among this thread's terms: read them again for the flags
    for_terms<VEC>(n, x, [&](int, float t) {
      const unsigned u = __float_as_uint(t);
      if ((u & 0x7f800000u) == 0x7f800000u) flags |= (u & 0x7fffffu) ? SUM_NAN : ((u >> 31) ? SUM_NINF : SUM_PINF);
    });
    v = DD{0.0, 0.0};
  }
  block_dd(v, flags, sv, sf);
  if (threadIdx.x == 0) {
    partials[blockIdx.x].s = v.s;
    partials[blockIdx.x].c = v.c;
    partials[blockIdx.x].flags = flags;
    __threadfence();
    last = atomicAdd(ticket, 1u) == gridDim.x - 1;
  }
  __syncthreads();
  if (!last) return;
  __threadfence();
  DD t{-0.0, -0.0};
  unsigned tf = 0;
  for (unsigned int b = threadIdx.x; b < gridDim.x; b += T) {
    t = dd_add(t, DD{__ldcg(&partials[b].s), __ldcg(&partials[b].c)});
    tf |= __ldcg(&partials[b].flags);
  }
  block_dd(t, tf, sv, sf);
  if (threadIdx.x == 0) {
    // hi + lo = s + c exactly, with hi = RN(s + c) (TwoSum: s and c may be of either size after cancellation)
    const double hi = __dadd_rn(t.s, t.c);
    const double z = __dsub_rn(hi, t.s);
    const double lo = __dadd_rn(__dsub_rn(t.s, __dsub_rn(hi, z)), __dsub_rn(t.c, z));
    float r;
    if ((tf & SUM_NAN) || ((tf & SUM_PINF) && (tf & SUM_NINF))) r = __uint_as_float(0x7fc00000u);
    else if (tf & SUM_PINF) r = __uint_as_float(0x7f800000u);
    else if (tf & SUM_NINF) r = __uint_as_float(0xff800000u);
    else if (hi == 0.0) r = (tf & SUM_OTHER) ? 0.0f : -0.0f;
    else r = round_dd_f32(hi, lo);
    if (out_f32) out_f32[0] = r;
    if (out_f64) {  // the unrounded part for a sharded sum: hi, lo and the flags (SUM_SOME: n > 0)
      out_f64[0] = hi;
      out_f64[1] = lo;
      out_f64[2] = static_cast<double>(tf | SUM_SOME);
    }
    *ticket = 0u;  // ready for the next launch that uses this scratch
  }
}

// The sharded sum's last step, on the device: the ranks' parts (hi, lo, flags; cairn_b200_sum_f32_partial) added as
// double-doubles in rank order and rounded once, as the single-device kernel rounds its blocks' total.
__global__ void combine_f32_parts_kernel(const double* parts, int count, float* out) {
  if (threadIdx.x != 0 || blockIdx.x != 0) return;
  DD t{-0.0, -0.0};
  unsigned tf = 0;
  for (int p = 0; p < count; ++p) {
    t = dd_add(t, DD{parts[3 * p], parts[3 * p + 1]});
    tf |= static_cast<unsigned>(parts[3 * p + 2]);
  }
  const double hi = __dadd_rn(t.s, t.c);
  const double z = __dsub_rn(hi, t.s);
  const double lo = __dadd_rn(__dsub_rn(t.s, __dsub_rn(hi, z)), __dsub_rn(t.c, z));
  float r;
  if ((tf & SUM_NAN) || ((tf & SUM_PINF) && (tf & SUM_NINF))) r = __uint_as_float(0x7fc00000u);
  else if (tf & SUM_PINF) r = __uint_as_float(0x7f800000u);
  else if (tf & SUM_NINF) r = __uint_as_float(0xff800000u);
  else if (hi == 0.0) r = ((tf & SUM_SOME) && !(tf & SUM_OTHER)) ? -0.0f : 0.0f;
  else r = round_dd_f32(hi, lo);
  *out = r;
}

// ---- the MLP's loss head: mean-squared error and its gradient in one pass ------------------------------------------
__device__ __forceinline__ double block_sum_f64(double v, double* shared) {
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
#pragma unroll
  for (int off = 16; off; off >>= 1) v += __shfl_xor_sync(0xffffffffu, v, off);
  if (lane == 0) shared[warp] = v;
  __syncthreads();
  double t = 0.0;
  if (warp == 0) {
    t = lane < WARPS ? shared[lane] : 0.0;
#pragma unroll
    for (int off = 16; off; off >>= 1) t += __shfl_xor_sync(0xffffffffu, t, off);
  }
  __syncthreads();
  return t;
}

// VEC: y and t start on 16 bytes and dy on 8, so four elements move per float4 load and 8-byte store, UNROLL vectors
// of each operand in flight per thread (the saxpy kernel's shape); the last n % 4 elements run in block 0.
template <bool VEC>
__global__ void __launch_bounds__(T, 2) mse_grad_kernel(std::size_t n, const float* y, const float* t,
                                                       __nv_bfloat16* dy, float scale, float* loss,
                                                       Partial* partials, unsigned int* ticket) {
  __shared__ double shared[WARPS];
  __shared__ bool last;
  const std::size_t stride = static_cast<std::size_t>(gridDim.x) * T;
  double acc = 0.0;  // each term d^2 is exact in f64: a product of two f32
  std::size_t i = static_cast<std::size_t>(blockIdx.x) * T + threadIdx.x;
  if constexpr (VEC) {
    const std::size_t n4 = n / 4;
    const float4* y4 = reinterpret_cast<const float4*>(y);
    const float4* t4 = reinterpret_cast<const float4*>(t);
    uint2* d4 = reinterpret_cast<uint2*>(dy);
    auto one = [&](std::size_t v, const float4& yv, const float4& tv) {
      const float d0 = __fsub_rn(yv.x, tv.x), d1 = __fsub_rn(yv.y, tv.y), d2 = __fsub_rn(yv.z, tv.z),
                  d3 = __fsub_rn(yv.w, tv.w);
      __stcs(d4 + v, make_uint2(bf16x2_bits(__fmul_rn(d0, scale), __fmul_rn(d1, scale)),
                                bf16x2_bits(__fmul_rn(d2, scale), __fmul_rn(d3, scale))));
      acc += static_cast<double>(d0) * static_cast<double>(d0);
      acc += static_cast<double>(d1) * static_cast<double>(d1);
      acc += static_cast<double>(d2) * static_cast<double>(d2);
      acc += static_cast<double>(d3) * static_cast<double>(d3);
    };
    for (; i + (UNROLL - 1) * stride < n4; i += UNROLL * stride) {
      float4 yv[UNROLL], tv[UNROLL];
#pragma unroll
      for (int u = 0; u < UNROLL; ++u) {
        yv[u] = __ldcs(y4 + i + u * stride);
        tv[u] = __ldcs(t4 + i + u * stride);
      }
#pragma unroll
      for (int u = 0; u < UNROLL; ++u) one(i + u * stride, yv[u], tv[u]);
    }
    for (; i < n4; i += stride) one(i, __ldcs(y4 + i), __ldcs(t4 + i));
    if (blockIdx.x == 0 && threadIdx.x < n - n4 * 4) {
      const std::size_t j = n4 * 4 + threadIdx.x;
      const float d = __fsub_rn(y[j], t[j]);
      dy[j] = __float2bfloat16_rn(__fmul_rn(d, scale));
      acc += static_cast<double>(d) * static_cast<double>(d);
    }
  } else {
    for (; i < n; i += stride) {
      const float d = __fsub_rn(__ldcs(y + i), __ldcs(t + i));
      dy[i] = __float2bfloat16_rn(__fmul_rn(d, scale));
      acc += static_cast<double>(d) * static_cast<double>(d);
    }
  }
  const double s = block_sum_f64(acc, shared);
  if (threadIdx.x == 0) {
    partials[blockIdx.x].s = s;
    __threadfence();
    last = atomicAdd(ticket, 1u) == gridDim.x - 1;
  }
  __syncthreads();
  if (!last) return;
  __threadfence();
  double total = 0.0;
  for (unsigned int b = threadIdx.x; b < gridDim.x; b += T) total += __ldcg(&partials[b].s);
  total = block_sum_f64(total, shared);
  if (threadIdx.x == 0) {
    *loss = __double2float_rn(total / static_cast<double>(n));
    *ticket = 0u;
  }
}

// ---- u64 checked sum --------------------------------------------------------------------------------------------
struct SumU64 {
  unsigned long long v;
  unsigned int over;
};
__device__ __forceinline__ SumU64 fold(SumU64 p, SumU64 q) {
  const unsigned long long s = p.v + q.v;
  return {s, p.over | q.over | (s < p.v ? 1u : 0u)};
}
__device__ __forceinline__ SumU64 warp_fold(SumU64 s) {
#pragma unroll
  for (int off = 16; off; off >>= 1) {
    SumU64 o;
    o.v = __shfl_xor_sync(0xffffffffu, s.v, off);
    o.over = __shfl_xor_sync(0xffffffffu, s.over, off);
    s = fold(s, o);
  }
  return s;
}
__device__ __forceinline__ SumU64 block_fold(SumU64 s, SumU64* shared) {
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  s = warp_fold(s);
  if (lane == 0) shared[warp] = s;
  __syncthreads();
  SumU64 t{0ull, 0u};
  if (warp == 0) {
    if (lane < WARPS) t = shared[lane];
    t = warp_fold(t);
  }
  __syncthreads();
  return t;
}
__device__ __forceinline__ void add_term(SumU64& s, unsigned long long x) {
  s.v += x;
  s.over |= s.v < x ? 1u : 0u;
}

template <bool VEC>
__global__ void __launch_bounds__(T, 2) sum_u64_kernel(std::size_t n, const unsigned long long* x,
                                                      unsigned long long* out, unsigned int* overflow,
                                                      SumU64* partials, unsigned int* ticket) {
  __shared__ SumU64 shared[WARPS];
  __shared__ bool last;
  const std::size_t stride = static_cast<std::size_t>(gridDim.x) * T;
  std::size_t i = static_cast<std::size_t>(blockIdx.x) * T + threadIdx.x;
  SumU64 s0{0ull, 0u}, s1{0ull, 0u};
  if constexpr (VEC) {
    const std::size_t n2 = n / 2;
    const ulonglong2* x2 = reinterpret_cast<const ulonglong2*>(x);
    for (; i + (UNROLL - 1) * stride < n2; i += UNROLL * stride) {
      ulonglong2 v[UNROLL];
#pragma unroll
      for (int u = 0; u < UNROLL; ++u) v[u] = __ldcs(x2 + i + u * stride);
#pragma unroll
      for (int u = 0; u < UNROLL; ++u) {
        add_term(s0, v[u].x);
        add_term(s1, v[u].y);
      }
    }
    for (; i < n2; i += stride) {
      const ulonglong2 v = __ldcs(x2 + i);
      add_term(s0, v.x);
      add_term(s1, v.y);
    }
    i = n2 * 2 + static_cast<std::size_t>(blockIdx.x) * T + threadIdx.x;
  }
  for (; i < n; i += stride) add_term(s0, __ldcs(x + i));
  SumU64 s = block_fold(fold(s0, s1), shared);
  if (threadIdx.x == 0) {
    partials[blockIdx.x] = s;
    __threadfence();
    last = atomicAdd(ticket, 1u) == gridDim.x - 1;
  }
  __syncthreads();
  if (!last) return;
  __threadfence();
  SumU64 t{0ull, 0u};
  for (unsigned int b = threadIdx.x; b < gridDim.x; b += T) {
    SumU64 p;
    p.v = __ldcg(&partials[b].v);
    p.over = __ldcg(&partials[b].over);
    t = fold(t, p);
  }
  t = block_fold(t, shared);
  if (threadIdx.x == 0) {
    *out = t.v;
    *overflow = t.over;
    *ticket = 0u;
  }
}

bool aligned16(const void* p) { return (reinterpret_cast<std::uintptr_t>(p) & 15u) == 0; }

}  // namespace

cudaError_t saxpy_f32_launch(std::size_t n, float* out, const float* x, const float* y, float a, cudaStream_t s,
                             int sms) {
  if (!n) return cudaSuccess;
  constexpr std::size_t MAX_BLOCKS = 0x7fffffff;
  if (aligned16(out) && aligned16(x) && aligned16(y)) {
    const std::size_t blocks = (n / 4 + SAXPY_THREADS - 1) / SAXPY_THREADS;
    if (blocks > MAX_BLOCKS) return cudaErrorInvalidValue;
    saxpy_vec_kernel<<<static_cast<unsigned>(blocks ? blocks : 1), SAXPY_THREADS, 0, s>>>(n, out, x, y, a);
  } else {  // about 64 indices per thread, in whole multiples of the SM count
    const std::size_t per_wave = static_cast<std::size_t>(sms), want = (n + 256 * 64 - 1) / (256 * 64),
                      least = per_wave * 8, most = (n + 255) / 256;
    std::size_t blocks = (want > least ? want : least + per_wave - 1) / per_wave * per_wave;
    if (blocks > most) blocks = most;
    saxpy_scalar_kernel<<<static_cast<unsigned>(blocks < MAX_BLOCKS ? blocks : MAX_BLOCKS), 256, 0, s>>>(n, out, x,
                                                                                                          y, a);
  }
  return cudaGetLastError();
}

cudaError_t sum_f32_launch(std::size_t n, const float* x, float* out_f32, double* out_f64, void* scratch,
                           cudaStream_t s, int sms) {
  if (!n) {  // the empty sum is +0.0 (cr::sum::result with n == 0), and its part is (0, 0, no flags)
    if (out_f32) {
      const cudaError_t e = cudaMemsetAsync(out_f32, 0, sizeof(float), s);
      if (e != cudaSuccess) return e;
    }
    if (out_f64) return cudaMemsetAsync(out_f64, 0, 3 * sizeof(double), s);
    return cudaSuccess;
  }
  const int grid = sum_f32_grid(sms);
  Partial* partials = partials_of<Partial>(scratch);
  unsigned int* ticket = ticket_of(scratch);
  if (aligned16(x)) sum_f32_kernel<true><<<grid, T, 0, s>>>(n, x, out_f32, out_f64, partials, ticket);
  else sum_f32_kernel<false><<<grid, T, 0, s>>>(n, x, out_f32, out_f64, partials, ticket);
  return cudaGetLastError();
}

cudaError_t combine_f32_parts_launch(const double* parts, int count, float* out, cudaStream_t s) {
  combine_f32_parts_kernel<<<1, 32, 0, s>>>(parts, count, out);
  return cudaGetLastError();
}

cudaError_t mse_grad_launch(std::size_t n, const float* y, const float* t, std::uint16_t* dy, float scale,
                            float* loss, void* scratch, cudaStream_t s, int sms) {
  if (!n) return cudaMemsetAsync(loss, 0, sizeof(float), s);
  const int grid = mse_grid(sms);
  Partial* partials = partials_of<Partial>(scratch);
  unsigned int* ticket = ticket_of(scratch);
  auto* d = reinterpret_cast<__nv_bfloat16*>(dy);
  if (aligned16(y) && aligned16(t) && (reinterpret_cast<std::uintptr_t>(dy) & 7u) == 0)
    mse_grad_kernel<true><<<grid, T, 0, s>>>(n, y, t, d, scale, loss, partials, ticket);
  else
    mse_grad_kernel<false><<<grid, T, 0, s>>>(n, y, t, d, scale, loss, partials, ticket);
  return cudaGetLastError();
}

cudaError_t sum_u64_launch(std::size_t n, const std::uint64_t* x, std::uint64_t* out, std::uint32_t* overflow,
                           void* scratch, cudaStream_t s, int sms) {
  if (!n) {
    cudaError_t e = cudaMemsetAsync(out, 0, sizeof(std::uint64_t), s);
    if (e == cudaSuccess) e = cudaMemsetAsync(overflow, 0, sizeof(std::uint32_t), s);
    return e;
  }
  const int grid = sum_u64_grid(sms);
  SumU64* partials = partials_of<SumU64>(scratch);
  unsigned int* ticket = ticket_of(scratch);
  const auto* xx = reinterpret_cast<const unsigned long long*>(x);
  auto* oo = reinterpret_cast<unsigned long long*>(out);
  if (aligned16(x)) sum_u64_kernel<true><<<grid, T, 0, s>>>(n, xx, oo, overflow, partials, ticket);
  else sum_u64_kernel<false><<<grid, T, 0, s>>>(n, xx, oo, overflow, partials, ticket);
  return cudaGetLastError();
}

// The watchdog self-test: one thread waits, through the same bounded mbarrier wait every kernel here uses, on a
// barrier that nothing arrives at. The wait gives up after WAIT_LIMIT_NS, records FAULT_WATCHDOG and returns.
__global__ void watchdog_kernel(std::uint32_t* fault) {
  __shared__ __align__(8) std::uint64_t never;
  __shared__ std::uint32_t abort_flag;
  if (threadIdx.x == 0) {
    mbar_init(&never, 1);
    abort_flag = 0u;
    fence_barrier_init();
  }
  __syncthreads();
  if (threadIdx.x == 0) mbar_wait(&never, 0u, &abort_flag, fault, FAULT_WATCHDOG);
}

// Clock marks: each block's first thread writes its SM's cycle counter (%clock64) and the global nanosecond timer
// into the SM's slot (%smid), so that two marks on a stream bracket the work between them: cycles over nanoseconds
// per SM is that SM's average clock over the interval. Enough blocks that every SM holds at least one.
__global__ void clock_marks_kernel(unsigned long long* slots, unsigned count) {
  if (threadIdx.x != 0) return;
  unsigned smid;
  asm volatile("mov.u32 %0, %%smid;" : "=r"(smid));
  if (smid >= count) return;
  long long cycles;
  asm volatile("mov.u64 %0, %%clock64;" : "=l"(cycles));
  slots[2 * smid] = static_cast<unsigned long long>(cycles);
  slots[2 * smid + 1] = globaltimer();
}

cudaError_t clock_marks_launch(cudaStream_t s, unsigned long long* slots, unsigned count, int sms) {
  clock_marks_kernel<<<4 * sms, 32, 0, s>>>(slots, count);
  return cudaGetLastError();
}

cudaError_t watchdog_launch(cudaStream_t s, std::uint32_t* fault) {
  watchdog_kernel<<<1, 32, 0, s>>>(fault);
  return cudaGetLastError();
}

}  // namespace cb

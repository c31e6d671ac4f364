// The dense multiply of CAIRN's tensor runtime, rebuilt for sm_100a.
//
// What it computes (the mma_unordered contract, runtime/cairn_tensor.hpp:1-6 and docs/numerics.md "The tensor-core
// multiply"): C (m x n, f32) += A (m x k) * B (k x n) over one storage float, each product exact in f32 and each
// output the f32 sum of its old value and its k products in an order the hardware picks. Beside it, the same product
// with either operand transposed (the backward of a dense layer: dX = dY * W^T, dW = X^T * dY) and with a fused
// epilogue (C = act(A * B + bias) cast to bf16, or C = A * B stored as f32).
//
// How (one persistent CTA per SM, 192 threads, 6 warps):
//   warp 0, one lane   TMA producer: for each output tile and each 128-byte slice of k, loads the A tile (128 rows)
//                      and the B tile (BN columns) into a ring of shared-memory stages, 128-byte swizzled, and
//                      arms the stage's "full" mbarrier with the byte count.
//   warp 1             allocates the tile accumulators in tensor memory (2 x BN columns of 128 lanes, double
//                      buffered); one lane issues tcgen05.mma (M=128, N=BN, 32 bytes of k per instruction) from
//                      the stage's shared-memory descriptors, commits each stage back to its "empty" mbarrier, and
//                      commits each finished accumulator to its "tmem full" mbarrier.
//   warps 2-5          epilogue: each warp owns 32 TMEM lanes (rows); it drains the accumulator 32 columns at a time
//                      with tcgen05.ld, frees the accumulator for the next tile, and writes the tile to global
//                      memory with the requested epilogue (C += acc, C = acc, or bf16(act(acc + bias))).
// Tiles are visited in groups of 8 column blocks so a wave of 148 CTAs shares A rows and B columns in L2.
//
// Operands are read straight from the caller's row-major arrays through TMA tensor maps; TMA zero-fills past the
// edges, so any m, n, k works as long as the rows start on 16 bytes (the tensor-map rule). Shapes that break it, and
// k == 0, run the SIMT tile kernel at the end of this file, which computes the same products.
#include <atomic>
#include <cstdint>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <type_traits>
#include <utility>
#include <vector>
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include "gemm.h"
#include "ptx.cuh"

namespace cb {

// ---------------------------------------------------------------------------------------------------------------
// Formats
// ---------------------------------------------------------------------------------------------------------------
template <int FMT> struct Fmt;
template <> struct Fmt<FMT_BF16> { static constexpr int bytes = 2, kind = KIND_F16, code = 1; };
template <> struct Fmt<FMT_F16> { static constexpr int bytes = 2, kind = KIND_F16, code = 0; };
template <> struct Fmt<FMT_E4M3> { static constexpr int bytes = 1, kind = KIND_F8F6F4, code = 0; };
template <> struct Fmt<FMT_E5M2> { static constexpr int bytes = 1, kind = KIND_F8F6F4, code = 1; };
template <> struct Fmt<FMT_TF32> { static constexpr int bytes = 4, kind = KIND_TF32, code = 2; };

struct TcParams {
  int m, n, k;
  int a_mn;       // A is stored k x m (the transposed operand): M-major in shared memory
  int b_k;        // B is stored n x k (the transposed operand): K-major in shared memory
  int out_kind;   // OUT_ACC_F32, OUT_STORE_F32 or OUT_BF16
  void* out;
  const float* bias;
  int act;
  const std::uint16_t* mask;  // OUT_BF16 only: keep an output where this m x n bf16 array is > 0, else 0
  int mask_vec;               // mask starts on 16 bytes (its rows then do too whenever vec holds)
  int tma_store;              // pair kernel: chunks leave through TMA stores (1), TMA reduce-adds into C (2), or
                              // TMA stores of bf16 outputs masked by the mask's tiles, which come in by TMA (3)
  int vec;        // every output row starts on 16 bytes and holds whole 16-byte groups
  std::uint32_t* fault;
  int streamk;            // split the tiles' k-blocks evenly over the pairs (pair kernel only)
  float* ws;              // stream-K partials: two slots per CTA of every pair
  std::uint32_t* flags;   // stream-K grid barrier: the count of CTAs that have written their partials
  std::uint32_t epoch;    // the count's value when this launch starts
};

constexpr int BM = 128;              // rows of a tile: the MMA's M, one TMEM lane per row
constexpr int SLICE = 128;           // bytes of k per stage: one 128-byte swizzle row
constexpr int A_STAGE = BM * SLICE;  // 16 KiB
constexpr int GROUP_N = 8;           // column blocks per rasterization group

template <int BN> struct Shape {
  static constexpr int B_STAGE = BN * SLICE;
  static constexpr int STAGES = (200 * 1024) / (A_STAGE + B_STAGE);
  static constexpr int TMEM_COLS = 2 * BN;  // two accumulators
  static constexpr int SMEM = 1024 + STAGES * (A_STAGE + B_STAGE) + 256;
  static_assert(TMEM_COLS == 256 || TMEM_COLS == 512, "TMEM allocations are powers of two");
};

__device__ __forceinline__ void tile_of(int t, int num_m, int num_n, int& mb, int& nb) {
  const int per_group = num_m * GROUP_N;
  const int g = t / per_group;
  const int first = g * GROUP_N;
  const int width = min(GROUP_N, num_n - first);
  const int r = t - g * per_group;
  mb = r / width;
  nb = first + r % width;
}

// Waits out copies or MMAs still in flight on the exit path, ignoring the abort flag but still bounded.
__device__ __noinline__ void drain_wait(std::uint64_t* bar, std::uint32_t parity, std::uint32_t* fault) {
  const std::uint64_t start = globaltimer();
  while (!mbar_test(bar, parity)) {
    if (globaltimer() - start > WAIT_LIMIT_NS) {
      atomicOr(fault, static_cast<std::uint32_t>(FAULT_DRAIN));
      return;
    }
  }
}

template <int FMT>
__device__ __forceinline__ void store_chunk(const TcParams& p, int row, int col, const std::uint32_t (&r)[32]) {
  if (row >= p.m) return;
  if (p.out_kind == OUT_BF16) {
    float v[32], bias[32];
    if (p.bias == nullptr) {  // zeros, added all the same (-0 becomes +0 as in the biased forms)
#pragma unroll
      for (int j = 0; j < 32; ++j) bias[j] = 0.0f;
    } else {
#pragma unroll
      for (int j = 0; j < 32; ++j) bias[j] = col + j < p.n ? __ldg(p.bias + col + j) : 0.0f;
    }
#pragma unroll
    for (int j = 0; j < 32; ++j) {
      float x = __fadd_rn(__uint_as_float(r[j]), bias[j]);
      if (p.act == ACT_RELU) x = x < 0.0f ? 0.0f : x;
      v[j] = x;
    }
    if (p.mask != nullptr) {  // the ReLU's backward: the gradient passes where the forward's output was positive
      const std::uint16_t* mrow = p.mask + static_cast<std::size_t>(row) * p.n + col;
#pragma unroll
      for (int j = 0; j < 32; ++j)
        if (col + j < p.n && !(__uint_as_float(static_cast<std::uint32_t>(__ldg(mrow + j)) << 16) > 0.0f)) v[j] = 0.0f;
    }
    __nv_bfloat16* dst = static_cast<__nv_bfloat16*>(p.out) + static_cast<std::size_t>(row) * p.n + col;
    if (p.vec && col + 32 <= p.n) {
      uint4* d4 = reinterpret_cast<uint4*>(dst);
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        uint4 w;
        __nv_bfloat162 h0 = __floats2bfloat162_rn(v[8 * q + 0], v[8 * q + 1]);
        __nv_bfloat162 h1 = __floats2bfloat162_rn(v[8 * q + 2], v[8 * q + 3]);
        __nv_bfloat162 h2 = __floats2bfloat162_rn(v[8 * q + 4], v[8 * q + 5]);
        __nv_bfloat162 h3 = __floats2bfloat162_rn(v[8 * q + 6], v[8 * q + 7]);
        std::memcpy(&w.x, &h0, 4);
        std::memcpy(&w.y, &h1, 4);
        std::memcpy(&w.z, &h2, 4);
        std::memcpy(&w.w, &h3, 4);
        d4[q] = w;
      }
    } else {
#pragma unroll
      for (int j = 0; j < 32; ++j)
        if (col + j < p.n) dst[j] = __float2bfloat16_rn(v[j]);
    }
  } else {
    float* dst = static_cast<float*>(p.out) + static_cast<std::size_t>(row) * p.n + col;
    const bool acc = p.out_kind == OUT_ACC_F32;
    if (p.vec && col + 32 <= p.n) {
      float4* d4 = reinterpret_cast<float4*>(dst);
#pragma unroll
      for (int q = 0; q < 8; ++q) {
        float4 o = make_float4(__uint_as_float(r[4 * q]), __uint_as_float(r[4 * q + 1]), __uint_as_float(r[4 * q + 2]),
                               __uint_as_float(r[4 * q + 3]));
        if (acc) {
          const float4 old = d4[q];
          o.x = __fadd_rn(old.x, o.x);
          o.y = __fadd_rn(old.y, o.y);
          o.z = __fadd_rn(old.z, o.z);
          o.w = __fadd_rn(old.w, o.w);
        }
        d4[q] = o;
      }
    } else {
#pragma unroll
      for (int j = 0; j < 32; ++j)
        if (col + j < p.n) dst[j] = acc ? __fadd_rn(dst[j], __uint_as_float(r[j])) : __uint_as_float(r[j]);
    }
  }
}

template <int FMT, int BN>
__global__ void __launch_bounds__(192, 1)
    tc_gemm_kernel(const __grid_constant__ CUtensorMap tm_a, const __grid_constant__ CUtensorMap tm_b,
                   const TcParams p) {
  using F = Fmt<FMT>;
  using S = Shape<BN>;
  constexpr int STAGES = S::STAGES;
  constexpr int CH = SLICE / F::bytes;              // elements per 128-byte row: the k of a stage, the width of a chunk
  constexpr int MMA_K_BYTES = 32;                   // every kind consumes 32 bytes of k per instruction
  constexpr int MMA_K_ROWS = MMA_K_BYTES / F::bytes;  // ... which is this many k rows of an M/N-major tile
  constexpr std::uint32_t STAGE_BYTES = A_STAGE + S::B_STAGE;

  extern __shared__ std::uint8_t smem_raw[];
  std::uint8_t* base = reinterpret_cast<std::uint8_t*>((reinterpret_cast<std::uintptr_t>(smem_raw) + 1023) &
                                                       ~static_cast<std::uintptr_t>(1023));
  std::uint8_t* a_smem = base;
  std::uint8_t* b_smem = base + STAGES * A_STAGE;
  std::uint64_t* bars = reinterpret_cast<std::uint64_t*>(b_smem + STAGES * S::B_STAGE);
  std::uint64_t* full = bars;
  std::uint64_t* empty = bars + STAGES;
  std::uint64_t* tfull = bars + 2 * STAGES;
  std::uint64_t* tempty = tfull + 2;
  std::uint64_t* drain = tempty + 2;
  std::uint32_t* tmem_slot = reinterpret_cast<std::uint32_t*>(drain + 1);
  volatile std::uint32_t* abort_flag = tmem_slot + 1;

  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int num_m = (p.m + BM - 1) / BM, num_n = (p.n + BN - 1) / BN;
  const int tiles = num_m * num_n;
  const int num_kb = (p.k + CH - 1) / CH;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&tfull[a], 1);
      mbar_init(&tempty[a], 4);
    }
    mbar_init(drain, 1);
    *abort_flag = 0u;
    fence_barrier_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, S::TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const std::uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      tma_prefetch_desc(&tm_a);
      tma_prefetch_desc(&tm_b);
      std::uint32_t stage = 0, phase = 0;
      std::uint32_t issued = 0, parity_of = 0;  // per stage: ever loaded, and the parity of its last load
      for (int t = blockIdx.x; t < tiles; t += gridDim.x) {
        int mb, nb;
        tile_of(t, num_m, num_n, mb, nb);
        const int m0 = mb * BM, n0 = nb * BN;
        for (int kb = 0; kb < num_kb; ++kb) {
          if (!mbar_wait(&empty[stage], phase ^ 1u, abort_flag, p.fault, FAULT_WAIT_EMPTY)) goto producer_done;
          mbar_arrive_expect_tx(&full[stage], STAGE_BYTES);
          issued |= 1u << stage;
          parity_of = (parity_of & ~(1u << stage)) | (phase << stage);
          const std::uint32_t a_dst = smem_u32(a_smem + stage * A_STAGE);
          const std::uint32_t b_dst = smem_u32(b_smem + stage * S::B_STAGE);
          const int k0 = kb * CH;
          if (!p.a_mn) {
            tma_load_2d(a_dst, &tm_a, &full[stage], k0, m0);
          } else {
#pragma unroll
            for (int c = 0; c < BM / CH; ++c) tma_load_2d(a_dst + c * CH * SLICE, &tm_a, &full[stage], m0 + c * CH, k0);
          }
          if (p.b_k) {
            tma_load_2d(b_dst, &tm_b, &full[stage], k0, n0);
          } else {
#pragma unroll
            for (int c = 0; c < BN / CH; ++c) tma_load_2d(b_dst + c * CH * SLICE, &tm_b, &full[stage], n0 + c * CH, k0);
          }
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
    producer_done:
      if (*abort_flag) {
        for (int s = 0; s < STAGES; ++s)
          if (issued & (1u << s)) drain_wait(&full[s], (parity_of >> s) & 1u, p.fault);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      const std::uint32_t idesc =
          idesc_make(F::code, F::code, p.a_mn != 0, p.b_k == 0, static_cast<std::uint32_t>(BM), BN);
      // Leading/stride byte offsets: a K-major tile is rows of 128 bytes, 8-row swizzle atoms 1024 bytes apart; an
      // M/N-major tile is CH-element chunks of SLICE rows each (chunk stride CH * SLICE bytes), 8 k rows per atom.
      const std::uint32_t a_lbo = p.a_mn ? CH * SLICE : 16u, b_lbo = p.b_k ? 16u : CH * SLICE;
      // An M/N-major tf32 tile uses 4-row atoms (512 bytes apart); everything else 8-row atoms (1024 bytes apart).
      constexpr bool MN32 = F::bytes == 4;
      const std::uint32_t a_layout = (MN32 && p.a_mn) ? LAYOUT_SW128_32B : LAYOUT_SW128;
      const std::uint32_t b_layout = (MN32 && !p.b_k) ? LAYOUT_SW128_32B : LAYOUT_SW128;
      const std::uint32_t a_sbo = a_layout == LAYOUT_SW128_32B ? 512u : 1024u;
      const std::uint32_t b_sbo = b_layout == LAYOUT_SW128_32B ? 512u : 1024u;
      std::uint32_t stage = 0, phase = 0, it = 0;
      for (int t = blockIdx.x; t < tiles; t += gridDim.x, ++it) {
        const std::uint32_t acc = it & 1u, acc_phase = (it >> 1) & 1u;
        if (!mbar_wait(&tempty[acc], acc_phase ^ 1u, abort_flag, p.fault, FAULT_WAIT_TEMPTY)) goto mma_done;
        tc_fence_after();
        const std::uint32_t d_tmem = tmem_base + acc * BN;
        for (int kb = 0; kb < num_kb; ++kb) {
          if (!mbar_wait(&full[stage], phase, abort_flag, p.fault, FAULT_WAIT_FULL)) goto mma_done;
          tc_fence_after();
          const std::uint32_t a_addr = smem_u32(a_smem + stage * A_STAGE);
          const std::uint32_t b_addr = smem_u32(b_smem + stage * S::B_STAGE);
#pragma unroll
          for (int kk = 0; kk < SLICE / MMA_K_BYTES; ++kk) {
            const std::uint32_t a_off = p.a_mn ? kk * (MMA_K_ROWS / 8) * 1024 : kk * MMA_K_BYTES;
            const std::uint32_t b_off = p.b_k ? kk * MMA_K_BYTES : kk * (MMA_K_ROWS / 8) * 1024;
            const std::uint64_t a_desc = sdesc(a_addr + a_off, a_lbo, a_sbo, a_layout);
            const std::uint64_t b_desc = sdesc(b_addr + b_off, b_lbo, b_sbo, b_layout);
            umma<F::kind>(d_tmem, a_desc, b_desc, idesc, (kb | kk) != 0 ? 1u : 0u);
          }
          tc_commit(&empty[stage]);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
        tc_commit(&tfull[acc]);
      }
    mma_done:
      // Every MMA this thread issued completes before the accumulators are released.
      tc_commit(drain);
      drain_wait(drain, 0u, p.fault);
    }
    __syncwarp();
  } else {
    const int quarter = warp & 3;  // TMEM lanes a warp may read: 32 * (warp id % 4) .. + 31
    std::uint32_t it = 0;
    for (int t = blockIdx.x; t < tiles; t += gridDim.x, ++it) {
      const std::uint32_t acc = it & 1u, acc_phase = (it >> 1) & 1u;
      if (!mbar_wait(&tfull[acc], acc_phase, abort_flag, p.fault, FAULT_WAIT_TFULL)) break;
      tc_fence_after();
      int mb, nb;
      tile_of(t, num_m, num_n, mb, nb);
      const int row = mb * BM + quarter * 32 + lane;
      const std::uint32_t t_row = tmem_base + (static_cast<std::uint32_t>(quarter * 32) << 16) + acc * BN;
#pragma unroll 1
      for (int c = 0; c < BN; c += 32) {
        std::uint32_t r[32];
        tmem_ld_32x32b_x32(t_row + c, r);
        tmem_wait_ld();
        if (c + 32 == BN) {  // the whole accumulator is in registers: hand it back to the MMA issuer
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(&tempty[acc]);
        }
        store_chunk<FMT>(p, row, nb * BN + c, r);
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, S::TMEM_COLS);
  }
}

// ---------------------------------------------------------------------------------------------------------------
// The staged epilogue store (the pair kernel's): a warp's 32 rows x 32 columns go through a 32 x 80-byte buffer of
// its own in shared memory. Written by rows (thread t = row t, 64 bytes: the 16-byte padding spreads the 32 rows'
// writes over every bank) and read back by row segments (4 threads per row, 8 rows per instruction), so every global
// store instruction writes 8 whole 64-byte row segments instead of touching 32 rows with 16 bytes each. f32 outputs
// go through in two 16-column halves.
// ---------------------------------------------------------------------------------------------------------------
constexpr int STAGE_PITCH = 80;                  // bytes per staged row: 64 of data, 16 of padding
constexpr int STAGE_BYTES = 32 * STAGE_PITCH;    // one warp's buffer

// Asks L2 for the line-aligned span of row `row` of an m x n row-major array (es bytes an element) covering columns
// [c_begin, c_end) that an epilogue warp will read while it drains: the ReLU-gradient mask, or the old C of the
// accumulate form. Issued before the tile's accumulator is ready, so the drain (which the next tile's MMAs wait for
// when the accumulator is single) finds those lines in L2 instead of waiting on DRAM. Every address stays inside the
// array: the span starts at or after the row's first byte and ends before its column c_end.
__device__ __forceinline__ void prefetch_row_span(const void* base, int es, const TcParams& p, int row, int c_begin,
                                                  int c_end) {
  if (row >= p.m) return;
  const int end = c_end < p.n ? c_end : p.n;
  if (c_begin >= end) return;
  const char* first = static_cast<const char*>(base) + static_cast<std::size_t>(row) * p.n * es;
  const std::size_t stop = static_cast<std::size_t>(end) * es;
  for (std::size_t off = (static_cast<std::size_t>(c_begin) * es) & ~static_cast<std::size_t>(127); off < stop;
       off += 128)
    asm volatile("prefetch.global.L2 [%0];" ::"l"(first + off));
}

// The ReLU's backward on two packed bf16 outputs: each 16-bit half of `out2` stays where the matching half of
// `mask2` (bf16 bits of the forward's output) is > 0 and becomes +0 elsewhere. A bf16 value is > 0 exactly when its
// bits, read as an unsigned 16-bit number, lie in [0x0001, 0x7f80] (positive subnormals up to +inf; +0, every
// negative value and NaN fall outside), so this is the same test as the float comparison, and zeroing after the
// rounding gives the bits that rounding a zeroed value does.
__device__ __forceinline__ std::uint32_t keep_where_positive(std::uint32_t out2, std::uint32_t mask2) {
  std::uint32_t kept = 0;
  if ((mask2 & 0xffffu) - 1u < 0x7f80u) kept |= out2 & 0xffffu;
  if ((mask2 >> 16) - 1u < 0x7f80u) kept |= out2 & 0xffff0000u;
  return kept;
}

// bias_s: the chunk's 32 bias values staged in shared memory (16-byte aligned), or null to read them from p.bias.
__device__ __forceinline__ void epilogue_values(const TcParams& p, int row, int col, const std::uint32_t (&r)[32],
                                                float (&v)[32], bool apply_mask, const float* bias_s) {
  float bias[32];
  if (bias_s != nullptr) {
#pragma unroll
    for (int q = 0; q < 8; ++q) {
      const float4 b = reinterpret_cast<const float4*>(bias_s)[q];
      bias[4 * q] = b.x;
      bias[4 * q + 1] = b.y;
      bias[4 * q + 2] = b.z;
      bias[4 * q + 3] = b.w;
    }
  } else if (p.bias == nullptr) {
    // No bias: zeros, added all the same (x + 0 turns -0 into +0, as the biased forms' arithmetic does). Tested
    // before any per-element branch, which costs the drain several hundred cycles per chunk for loads never made.
#pragma unroll
    for (int j = 0; j < 32; ++j) bias[j] = 0.0f;
  } else if (col + 32 <= p.n && (reinterpret_cast<std::uintptr_t>(p.bias + col) & 15u) == 0) {
    const float4* b4 = reinterpret_cast<const float4*>(p.bias + col);
#pragma unroll
    for (int q = 0; q < 8; ++q) {
      const float4 b = __ldg(b4 + q);
      bias[4 * q] = b.x;
      bias[4 * q + 1] = b.y;
      bias[4 * q + 2] = b.z;
      bias[4 * q + 3] = b.w;
    }
  } else {
#pragma unroll
    for (int j = 0; j < 32; ++j) bias[j] = col + j < p.n ? __ldg(p.bias + col + j) : 0.0f;
  }
#pragma unroll
  for (int j = 0; j < 32; ++j) {
    float x = __fadd_rn(__uint_as_float(r[j]), bias[j]);
    if (p.act == ACT_RELU) x = x < 0.0f ? 0.0f : x;
    v[j] = x;
  }
  if (apply_mask && p.mask != nullptr && row < p.m) {
    const std::uint16_t* mrow = p.mask + static_cast<std::size_t>(row) * p.n + col;
#pragma unroll
    for (int j = 0; j < 32; ++j)
      if (col + j < p.n && !(__uint_as_float(static_cast<std::uint32_t>(__ldg(mrow + j)) << 16) > 0.0f)) v[j] = 0.0f;
  }
}

// Stores the warp's 32 x 32 chunk whose first row is row0 (this thread holds row row0 + lane) at column col, through
// the warp's staging rows, so each write-back pass moves 8 rows x 64 bytes.
// LOADS = false, for epilogues that read no memory (the double-buffered drain): bias, ReLU and the mask (read per
//   element, should one be given) over all 32 values at once, then bf16 packing; f32 goes through in two 16-column
//   halves.
// LOADS = true, for epilogues that read memory (the single-buffered drain, whose registers allow it): bf16 values are
//   formed eight at a time (bias, ReLU, per-element mask) straight into the staging row, so few are live beside
//   the chunk; with 16-byte rows the ReLU-gradient mask is instead read at write-back, one coalesced 16-byte load
//   per 8 outputs, and the accumulate form's old values likewise, a half's four at once. Both kinds of load are
//   issued together before the first store: a load after a store to the output could not be moved above it,
//   which would serialise the passes on the load's latency.
// The TMA mask path's per-warp state: the warp's mbarrier for its mask tiles, the parity of the next, and the abort
// flag its bounded wait watches.
struct MaskTiles {
  const CUtensorMap* map;
  std::uint64_t* bar;
  std::uint32_t phase;
  volatile std::uint32_t* abort_flag;
};

// A bf16 chunk with no mask through the output's tensor map (the plain TMA-store path of store_chunk_staged, below):
// the warp forms its values, writes them once, 64-byte swizzled (row r's 16-byte group q at r 64 + 16 (q ^ ((r >> 1)
// & 3)), which spreads each quarter-warp's writes over all 32 banks), into its buffer once the previous chunk's store
// has read it, and one lane hands the buffer to a TMA store, which clips rows and columns outside the output. The
// drain calls it from a loop of its own: a loop body that carries every output path is several times larger, and
// was measured 1-1.5 % slower on the products that take this path.
__device__ __forceinline__ void store_chunk_bf16_tma(const TcParams& p, int row0, int col, const std::uint32_t (&r)[32],
                                                     std::uint8_t* stage, int lane, const float* bias_s,
                                                     const CUtensorMap* tm_c) {
  if (lane == 0) bulk_wait_read();
  float v[32];
  epilogue_values(p, row0 + lane, col, r, v, false, bias_s);
  __syncwarp();
  std::uint8_t* mine = stage + lane * 64;
#pragma unroll
  for (int q = 0; q < 4; ++q)
    *reinterpret_cast<uint4*>(mine + 16 * (q ^ ((lane >> 1) & 3))) =
        make_uint4(bf16x2_bits(v[8 * q + 0], v[8 * q + 1]), bf16x2_bits(v[8 * q + 2], v[8 * q + 3]),
                   bf16x2_bits(v[8 * q + 4], v[8 * q + 5]), bf16x2_bits(v[8 * q + 6], v[8 * q + 7]));
  fence_proxy_async_shared();
  __syncwarp();
  if (lane == 0) {
    tma_store_2d(tm_c, smem_u32(stage), col, row0);
    bulk_commit();
  }
}

// An f32 chunk through the output's tensor map, a 16-column half (32 rows of 64 bytes, swizzled as above) at a time.
// The accumulate form (C += A B, p.tma_store == 2) hands each half to a TMA reduce-add: L2 adds it to C element by
// element, each sum rounded once to nearest, as old + acc rounded in the epilogue would be; one tile owns each
// element, so each is added once. Like store_chunk_bf16_tma, the drain runs it in a loop of its own.
__device__ __forceinline__ void store_chunk_f32_tma(const TcParams& p, int row0, int col, const std::uint32_t (&r)[32],
                                                    std::uint8_t* stage, int lane, const CUtensorMap* tm_c) {
  std::uint8_t* mine = stage + lane * 64;
#pragma unroll
  for (int half = 0; half < 2; ++half) {
    if (lane == 0) bulk_wait_read();
    __syncwarp();
#pragma unroll
    for (int q = 0; q < 4; ++q)
      *reinterpret_cast<float4*>(mine + 16 * (q ^ ((lane >> 1) & 3))) =
          make_float4(__uint_as_float(r[16 * half + 4 * q]), __uint_as_float(r[16 * half + 4 * q + 1]),
                      __uint_as_float(r[16 * half + 4 * q + 2]), __uint_as_float(r[16 * half + 4 * q + 3]));
    fence_proxy_async_shared();
    __syncwarp();
    if (lane == 0) {
      if (p.tma_store == 2)
        tma_reduce_add_2d(tm_c, smem_u32(stage), col + 16 * half, row0);
      else
        tma_store_2d(tm_c, smem_u32(stage), col + 16 * half, row0);
      bulk_commit();
    }
  }
}

template <bool LOADS, bool MASKED>
__device__ __forceinline__ void store_chunk_staged(const TcParams& p, int row0, int col, const std::uint32_t (&r)[32],
                                                   std::uint8_t* stage, int lane, const float* bias_s,
                                                   const CUtensorMap* tm_c, MaskTiles& mt) {
  const int seg = lane & 3, sub = lane >> 2;  // read-back: 4 threads per row (16 bytes each), 8 rows per pass
  if constexpr (!LOADS) {
    if (p.out_kind == OUT_BF16 && p.tma_store) {
      if constexpr (!MASKED) {
        store_chunk_bf16_tma(p, row0, col, r, stage, lane, bias_s, tm_c);
      } else {
        // Under the ReLU-gradient mask (mode 3) the chunk leaves as store_chunk_bf16_tma's does, and lane 0 first
        // asks TMA for the chunk's 32 x 32 mask tile into the buffer, laid out as the output will be, as soon as the
        // previous chunk's store has read the buffer; the warp forms its values meanwhile, then each thread masks its
        // own row in place (keep_where_positive, the same test as the per-element one) before the store.
        if (lane == 0) {
          bulk_wait_read();
          mbar_arrive_expect_tx(mt.bar, 32 * 64);
          tma_load_2d(smem_u32(stage), mt.map, mt.bar, col, row0);
        }
        float v[32];
        epilogue_values(p, row0 + lane, col, r, v, false, bias_s);
        __syncwarp();
        mbar_wait(mt.bar, mt.phase, mt.abort_flag, p.fault, FAULT_WAIT_MASK);
        mt.phase ^= 1u;
        std::uint8_t* mine = stage + lane * 64;
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          uint4* slot = reinterpret_cast<uint4*>(mine + 16 * (q ^ ((lane >> 1) & 3)));
          const uint4 mk = *slot;
          *slot = make_uint4(keep_where_positive(bf16x2_bits(v[8 * q + 0], v[8 * q + 1]), mk.x),
                             keep_where_positive(bf16x2_bits(v[8 * q + 2], v[8 * q + 3]), mk.y),
                             keep_where_positive(bf16x2_bits(v[8 * q + 4], v[8 * q + 5]), mk.z),
                             keep_where_positive(bf16x2_bits(v[8 * q + 6], v[8 * q + 7]), mk.w));
        }
        fence_proxy_async_shared();
        __syncwarp();
        if (lane == 0) {
          tma_store_2d(tm_c, smem_u32(stage), col, row0);
          bulk_commit();
        }
      }
      return;
    }
    if ((p.out_kind == OUT_STORE_F32 || p.out_kind == OUT_ACC_F32) && p.tma_store) {
      store_chunk_f32_tma(p, row0, col, r, stage, lane, tm_c);
      return;
    }
  }
  if (p.out_kind == OUT_BF16) {
    const bool late_mask = LOADS && p.mask != nullptr && p.vec && p.mask_vec;
    uint4* mine = reinterpret_cast<uint4*>(stage + lane * STAGE_PITCH);
    if constexpr (!LOADS) {
      float v[32];
      epilogue_values(p, row0 + lane, col, r, v, true, bias_s);
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        uint4 w;
        __nv_bfloat162 h0 = __floats2bfloat162_rn(v[8 * q + 0], v[8 * q + 1]);
        __nv_bfloat162 h1 = __floats2bfloat162_rn(v[8 * q + 2], v[8 * q + 3]);
        __nv_bfloat162 h2 = __floats2bfloat162_rn(v[8 * q + 4], v[8 * q + 5]);
        __nv_bfloat162 h3 = __floats2bfloat162_rn(v[8 * q + 6], v[8 * q + 7]);
        std::memcpy(&w.x, &h0, 4);
        std::memcpy(&w.y, &h1, 4);
        std::memcpy(&w.z, &h2, 4);
        std::memcpy(&w.w, &h3, 4);
        mine[q] = w;
      }
    } else {
      const int row = row0 + lane;
      const std::uint16_t* mrow = (!late_mask && p.mask != nullptr && row < p.m)
                                      ? p.mask + static_cast<std::size_t>(row) * p.n + col
                                      : nullptr;
      const bool bias_vec =
          p.bias != nullptr && col + 32 <= p.n && (reinterpret_cast<std::uintptr_t>(p.bias + col) & 15u) == 0;
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        float b[8];
        if (bias_s != nullptr || bias_vec) {
          const float4* src = bias_s != nullptr ? reinterpret_cast<const float4*>(bias_s)
                                                : reinterpret_cast<const float4*>(p.bias + col);
          const float4 b0 = bias_s != nullptr ? src[2 * q] : __ldg(src + 2 * q);
          const float4 b1 = bias_s != nullptr ? src[2 * q + 1] : __ldg(src + 2 * q + 1);
          b[0] = b0.x, b[1] = b0.y, b[2] = b0.z, b[3] = b0.w, b[4] = b1.x, b[5] = b1.y, b[6] = b1.z, b[7] = b1.w;
        } else if (p.bias == nullptr) {
#pragma unroll
          for (int j = 0; j < 8; ++j) b[j] = 0.0f;
        } else {
#pragma unroll
          for (int j = 0; j < 8; ++j) {
            const int c = col + 8 * q + j;
            b[j] = c < p.n ? __ldg(p.bias + c) : 0.0f;
          }
        }
        std::uint32_t packed[4];
#pragma unroll
        for (int j = 0; j < 8; j += 2) {
          float x0 = __fadd_rn(__uint_as_float(r[8 * q + j]), b[j]);
          float x1 = __fadd_rn(__uint_as_float(r[8 * q + j + 1]), b[j + 1]);
          if (p.act == ACT_RELU) {
            x0 = x0 < 0.0f ? 0.0f : x0;
            x1 = x1 < 0.0f ? 0.0f : x1;
          }
          if (mrow != nullptr) {  // the ReLU's backward: the gradient passes where the forward's output was positive
            const int c = col + 8 * q + j;
            if (c < p.n && !(__uint_as_float(static_cast<std::uint32_t>(__ldg(mrow + 8 * q + j)) << 16) > 0.0f))
              x0 = 0.0f;
            if (c + 1 < p.n &&
                !(__uint_as_float(static_cast<std::uint32_t>(__ldg(mrow + 8 * q + j + 1)) << 16) > 0.0f))
              x1 = 0.0f;
          }
          const __nv_bfloat162 h = __floats2bfloat162_rn(x0, x1);
          std::memcpy(&packed[j / 2], &h, 4);
        }
        mine[q] = make_uint4(packed[0], packed[1], packed[2], packed[3]);
      }
    }
    uint4 mk[4];
    if (late_mask) {
#pragma unroll
      for (int pass = 0; pass < 4; ++pass) {
        const int mr = row0 + pass * 8 + sub, c0 = col + seg * 8;
        mk[pass] = (mr < p.m && c0 + 8 <= p.n)
                       ? __ldg(reinterpret_cast<const uint4*>(p.mask + static_cast<std::size_t>(mr) * p.n + c0))
                       : make_uint4(0u, 0u, 0u, 0u);
      }
    }
    __syncwarp();
#pragma unroll
    for (int pass = 0; pass < 4; ++pass) {
      const int rr = pass * 8 + sub, orow = row0 + rr, c0 = col + seg * 8;
      uint4 w = *reinterpret_cast<const uint4*>(stage + rr * STAGE_PITCH + seg * 16);
      if (orow < p.m) {
        __nv_bfloat16* dst = static_cast<__nv_bfloat16*>(p.out) + static_cast<std::size_t>(orow) * p.n + c0;
        if (p.vec && c0 + 8 <= p.n) {
          if (late_mask) {
            w.x = keep_where_positive(w.x, mk[pass].x);
            w.y = keep_where_positive(w.y, mk[pass].y);
            w.z = keep_where_positive(w.z, mk[pass].z);
            w.w = keep_where_positive(w.w, mk[pass].w);
          }
          *reinterpret_cast<uint4*>(dst) = w;
        } else {
          const std::uint16_t* h = reinterpret_cast<const std::uint16_t*>(&w);
#pragma unroll
          for (int j = 0; j < 8; ++j)
            if (c0 + j < p.n) reinterpret_cast<std::uint16_t*>(dst)[j] = h[j];
        }
      }
    }
    __syncwarp();
  } else {
    const bool acc = p.out_kind == OUT_ACC_F32;
    const bool batch_old = LOADS && acc && p.vec;
#pragma unroll
    for (int half = 0; half < 2; ++half) {
      float4* mine = reinterpret_cast<float4*>(stage + lane * STAGE_PITCH);
#pragma unroll
      for (int q = 0; q < 4; ++q)
        mine[q] = make_float4(__uint_as_float(r[16 * half + 4 * q]), __uint_as_float(r[16 * half + 4 * q + 1]),
                              __uint_as_float(r[16 * half + 4 * q + 2]), __uint_as_float(r[16 * half + 4 * q + 3]));
      float4 old[4];
      if (batch_old) {
#pragma unroll
        for (int pass = 0; pass < 4; ++pass) {
          const int orow = row0 + pass * 8 + sub, c0 = col + 16 * half + seg * 4;
          old[pass] = (orow < p.m && c0 + 4 <= p.n)
                          ? *reinterpret_cast<const float4*>(static_cast<const float*>(p.out) +
                                                             static_cast<std::size_t>(orow) * p.n + c0)
                          : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
        }
      }
      __syncwarp();
#pragma unroll
      for (int pass = 0; pass < 4; ++pass) {
        const int rr = pass * 8 + sub, orow = row0 + rr, c0 = col + 16 * half + seg * 4;
        float4 w = *reinterpret_cast<const float4*>(stage + rr * STAGE_PITCH + seg * 16);
        if (orow < p.m) {
          float* dst = static_cast<float*>(p.out) + static_cast<std::size_t>(orow) * p.n + c0;
          if (p.vec && c0 + 4 <= p.n) {
            if (acc) {
              const float4 o = batch_old ? old[pass] : *reinterpret_cast<const float4*>(dst);
              w.x = __fadd_rn(o.x, w.x);
              w.y = __fadd_rn(o.y, w.y);
              w.z = __fadd_rn(o.z, w.z);
              w.w = __fadd_rn(o.w, w.w);
            }
            *reinterpret_cast<float4*>(dst) = w;
          } else {
            const float e[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
            for (int j = 0; j < 4; ++j)
              if (c0 + j < p.n) dst[j] = acc ? __fadd_rn(dst[j], e[j]) : e[j];
          }
        }
      }
      __syncwarp();
    }
  }
}

// ---------------------------------------------------------------------------------------------------------------
// A pair's work, as segments (tile, first k-block, end k-block). Data-parallel: whole tiles pair, pair + pairs, ...
// Stream-K: the tiles x k-blocks units cut into `pairs` contiguous ranges of equal length, so every pair does the
// same amount of MMA work however the tile count divides. A range that starts inside a tile begins with that
// tile's later k-blocks (a contributor: it publishes an f32 partial); one that ends inside a tile ends with that
// tile's first k-blocks (the finisher: it adds the contributors' partials and writes the tile). A pair contributes at
// most once, first, and finishes at most once, last, so a finisher waits only for work its contributors did at the
// start of the launch.
// ---------------------------------------------------------------------------------------------------------------
// Where a 32 x 32 block of a split tile's partial sum sits in a CTA's workspace slot, in float4 units: block (w, ci)
// of epilogue warp w, chunk ci, holds 8 rows of 32 float4 (row e: values 4e .. 4e + 3 of every lane), so each warp
// store and load covers 512 contiguous bytes.
__device__ __forceinline__ std::size_t partial_cell(int w, int ci, int chunks) {
  return static_cast<std::size_t>(w * chunks + ci) * 256;
}

// One output tile of the pair kernel: rows [256 mb, 256 mb + 256) and `units` blocks of 128 columns from column n0.
struct TileSpec {
  int mb, n0, units;
};

// A planned cover of the output (mixed tile widths; the host's planner, pair_tiles_plan): each pair's tiles listed in
// turn, packed as band << 16 | first 128-column unit << 3 | units. Unplanned launches cover the output uniformly with
// tiles of G * 256 columns in the order tile_of gives.
constexpr int PLAN_MAX_PAIRS = 128, PLAN_MAX_TILES = 512;
struct PairTiles {
  int planned;
  std::uint16_t first[PLAN_MAX_PAIRS + 1];  // pair q's tiles are tile[first[q]] .. tile[first[q + 1] - 1]
  std::uint32_t tile[PLAN_MAX_TILES];
};

struct PairWork {
  long long u, u_end;  // stream-K: this pair's units
  int t, tiles, pairs, num_kb, num_m, num_n, tile_n;
  bool sk;
  const PairTiles* plan;
  int q, q_end;  // planned: this pair's entries of the table
  __device__ PairWork(int pair, int pairs_, int num_m_, int num_n_, int tile_n_, int num_kb_, bool streamk,
                      const PairTiles* plan_)
      : t(pair), tiles(num_m_ * num_n_), pairs(pairs_), num_kb(num_kb_), num_m(num_m_), num_n(num_n_),
        tile_n(tile_n_), sk(streamk), plan(plan_), q(0), q_end(0) {
    const long long units = static_cast<long long>(tiles) * num_kb_;
    u = units * pair / pairs_;
    u_end = units * (pair + 1) / pairs_;
    if (plan->planned) {
      q = plan->first[pair];
      q_end = plan->first[pair + 1];
    }
  }
  __device__ bool next(TileSpec& ts, int& kb0, int& kb1) {
    int tile;
    if (plan->planned) {
      if (q >= q_end) return false;
      const std::uint32_t e = plan->tile[q++];
      ts = {static_cast<int>(e >> 16), static_cast<int>((e >> 3) & 0x1fffu) * 128, static_cast<int>(e & 7u)};
      kb0 = 0;
      kb1 = num_kb;
      return true;
    }
    if (!sk) {
      if (t >= tiles) return false;
      tile = t;
      kb0 = 0;
      kb1 = num_kb;
      t += pairs;
    } else {
      if (u >= u_end) return false;
      tile = static_cast<int>(u / num_kb);
      kb0 = static_cast<int>(u % num_kb);
      const long long left = u_end - u;
      kb1 = left < num_kb - kb0 ? kb0 + static_cast<int>(left) : num_kb;
      u += kb1 - kb0;
    }
    int nb;
    tile_of(tile, num_m, num_n, ts.mb, nb);
    ts.n0 = nb * tile_n;
    ts.units = tile_n / 128;
    return true;
  }
  // The first unit of pair q's range.
  __device__ long long start_of(int qq) const {
    return static_cast<long long>(tiles) * num_kb * qq / pairs;
  }
};

// ---------------------------------------------------------------------------------------------------------------
// The two-SM multiply: a cluster of two CTAs (a pair) computes a 256 x (256 G) tile with tcgen05.mma.cta_group::2,
// G = 1 or 2 column groups of 256. Each CTA stages its own half of the operands at the same shared-memory offsets:
// rows [128 r, 128 r + 128) of the tile's A, and in each column group g the columns [256 g + 128 r, + 128) of B,
// for pair rank r. The leader (rank 0) issues one pair MMA per column group and 32-byte k step; each MMA reads both
// CTAs' halves and accumulates rows 128 r .. 128 r + 127, 256 columns, into rank r's tensor memory.
//   Why two shapes: a 256 x 256 pair step (G = 1) moves 64 KB per 128-byte k slice per pair, about 18 TB/s from L2
//   at the tensor pipe's full rate, near the 20-24 TB/s a B200's L2 delivers to the SMs; it measured about 1.3
//   PFLOP/s. A 256 x 512 tile (G = 2) reads A once for both column groups, 25 % fewer bytes per flop (about 13.7
//   TB/s at full rate), at the price of a single accumulator (512 TMEM columns) whose drain the next tile waits for;
//   G = 1 keeps two accumulators and hides the drain. Eight epilogue warps (two per TMEM lane quarter, each draining
//   half the columns) keep that drain short.
//   Both CTAs' TMA loads count their bytes on the leader's "full" barrier; the leader's commits arrive on the
//   "empty" and "tmem full" barriers of both CTAs (one plain commit per CTA); every epilogue warp of the pair
//   arrives on the leader's "tmem empty" barrier.
// ---------------------------------------------------------------------------------------------------------------
constexpr int PAIR_BN = 256;  // columns per MMA (and per column group); each CTA stages half of each group

template <int G> struct PairShape {
  static constexpr int B_HALF = G * (PAIR_BN / 2) * SLICE;         // 16 KiB per column group
  static constexpr int STAGES = (200 * 1024) / (A_STAGE + B_HALF);  // 6 (G = 1) or 4 (G = 2)
  static constexpr int ACCS = G == 1 ? 2 : 1;                       // accumulators in TMEM
  static constexpr int TMEM_COLS = 512;
  static constexpr int EPI_WARPS = 8;                               // two warps per TMEM lane quarter
  static constexpr int THREADS = 64 + 32 * EPI_WARPS;
  static constexpr int TILE_N = G * PAIR_BN;
  static constexpr int BIAS_BYTES = 1024;  // an epilogue warp's staged bias: up to 256 columns of f32
  static constexpr int SMEM = 1024 + STAGES * (A_STAGE + B_HALF) + 1024 + EPI_WARPS * (STAGE_BYTES + BIAS_BYTES);
};

// EPI: 0 an epilogue that reads no memory (its chunks leave by TMA stores or reduce-adds, or the threads' stores);
// 1 one that reads memory through the threads' loads (the mask or old C off the tensor-map rules); 2 bf16 under the
// ReLU-gradient mask, whose tiles come in by TMA. Each is its own instantiation, so each gets its own registers.
template <int FMT, int G, int EPI>
__global__ void __launch_bounds__(PairShape<G>::THREADS, 1)
    tc_gemm_pair_kernel(const __grid_constant__ CUtensorMap tm_a, const __grid_constant__ CUtensorMap tm_b,
                        const __grid_constant__ CUtensorMap tm_c, const __grid_constant__ CUtensorMap tm_m,
                        const TcParams p, const __grid_constant__ PairTiles plan) {
  using F = Fmt<FMT>;
  using S = PairShape<G>;
  constexpr bool READS = EPI == 1;
  constexpr bool MASKED = EPI == 2;
  constexpr int STAGES = S::STAGES;
  constexpr int CH = SLICE / F::bytes;
  constexpr int MMA_K_BYTES = 32;
  constexpr int MMA_K_ROWS = MMA_K_BYTES / F::bytes;
  constexpr int HALF = PAIR_BN / 2;               // rows of A, and columns of B per group, each CTA stages
  constexpr int GROUP_BYTES = HALF * SLICE;       // one column group's half in a stage
  constexpr int UNIT_BYTES = (HALF / 2) * SLICE;  // a CTA's share of one 128-column unit of B in a stage

  extern __shared__ std::uint8_t smem_raw[];
  std::uint8_t* base = reinterpret_cast<std::uint8_t*>((reinterpret_cast<std::uintptr_t>(smem_raw) + 1023) &
                                                       ~static_cast<std::uintptr_t>(1023));
  std::uint8_t* a_smem = base;
  std::uint8_t* b_smem = base + STAGES * A_STAGE;
  std::uint64_t* bars = reinterpret_cast<std::uint64_t*>(b_smem + STAGES * S::B_HALF);
  std::uint64_t* full = bars;
  std::uint64_t* empty = bars + STAGES;
  std::uint64_t* tfull = bars + 2 * STAGES;
  std::uint64_t* tempty = tfull + 2;
  std::uint64_t* drain = tempty + 2;
  std::uint64_t* published = drain + 1;  // every epilogue warp of this CTA has written its stream-K partial
  std::uint64_t* mask_bars = published + 1;  // one per epilogue warp: its mask tiles' TMA loads (mode 3)
  std::uint32_t* tmem_slot = reinterpret_cast<std::uint32_t*>(mask_bars + S::EPI_WARPS);
  volatile std::uint32_t* abort_flag = tmem_slot + 1;
  // EPI_WARPS buffers of STAGE_BYTES, from 1024 bytes past the barriers: each starts on 512 bytes (STAGE_BYTES is a
  // multiple), as a TMA store's 64-byte-swizzled source must.
  std::uint8_t* epi_stage = reinterpret_cast<std::uint8_t*>(bars) + 1024;
  float* epi_bias = reinterpret_cast<float*>(epi_stage + S::EPI_WARPS * STAGE_BYTES);  // EPI_WARPS x BIAS_BYTES

  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const std::uint32_t rank = cluster_rank();
  const int pair = blockIdx.x / 2, pairs = gridDim.x / 2;
  const int num_m = (p.m + 2 * HALF - 1) / (2 * HALF), num_n = (p.n + S::TILE_N - 1) / S::TILE_N;
  const int tiles = num_m * num_n;
  const int num_kb = (p.k + CH - 1) / CH;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&tfull[a], 1);
      mbar_init(&tempty[a], 2 * S::EPI_WARPS);
    }
    mbar_init(drain, 1);
    mbar_init(published, S::EPI_WARPS);
    for (int w = 0; w < S::EPI_WARPS; ++w) mbar_init(&mask_bars[w], 1);
    *abort_flag = 0u;
    fence_barrier_init();
  }
  if (warp == 1) {
    tmem_alloc_pair(tmem_slot, S::TMEM_COLS);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  cluster_sync();  // both CTAs' barriers exist before either side's copies or arrivals reach them
  tc_fence_after();
  const std::uint32_t tmem_base = *tmem_slot;
  // Launched as a programmatic dependent, this CTA may have started on an SM the product before it on the stream has
  // left while that product still runs: the set-up above touches only this CTA's shared and tensor memory and its
  // parameters, and no thread reads or writes global memory until that product has completed. The next product may
  // then start its own set-up wherever an SM comes free.
  griddep_launch_dependents();
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tm_a);
    tma_prefetch_desc(&tm_b);
  }
  griddep_wait();

  if (warp == 0) {
    if (lane == 0) {
      std::uint32_t stage = 0, phase = 0;
      PairWork work(pair, pairs, num_m, num_n, S::TILE_N, num_kb, p.streamk != 0, &plan);
      TileSpec ts;
      int kb_begin, kb_end;
      while (work.next(ts, kb_begin, kb_end)) {
        const int m0 = ts.mb * 2 * HALF + static_cast<int>(rank) * HALF;  // this CTA's rows of A
        const int n_tile = ts.n0;
        const int u0 = ts.units < 2 ? ts.units : 2, u1 = ts.units - u0;  // units of the two column groups
        const std::uint32_t stage_bytes = 2u * (A_STAGE + static_cast<std::uint32_t>(ts.units) * UNIT_BYTES);
        for (int kb = kb_begin; kb < kb_end; ++kb) {
          if (!mbar_wait(&empty[stage], phase ^ 1u, abort_flag, p.fault, FAULT_WAIT_EMPTY)) goto producer_done;
          const std::uint32_t leader_full = cluster_addr(&full[stage], 0);
          if (rank == 0) mbar_arrive_expect_tx(&full[stage], stage_bytes);
          const std::uint32_t a_dst = smem_u32(a_smem + stage * A_STAGE);
          const std::uint32_t b_dst = smem_u32(b_smem + stage * S::B_HALF);
          const int k0 = kb * CH;
          if (!p.a_mn) {
            tma_load_2d_pair(a_dst, &tm_a, leader_full, k0, m0);
          } else {
#pragma unroll
            for (int c = 0; c < HALF / CH; ++c)
              tma_load_2d_pair(a_dst + c * CH * SLICE, &tm_a, leader_full, m0 + c * CH, k0);
          }
#pragma unroll
          for (int g = 0; g < G; ++g) {
            const int ug = g == 0 ? u0 : u1;
            if (ug == 0) continue;
            // this CTA's columns of group g: the group's first or second half (64 ug columns each)
            const int n0 = n_tile + g * PAIR_BN + static_cast<int>(rank) * (HALF / 2) * ug;
            const std::uint32_t dst = b_dst + g * GROUP_BYTES;
            if (p.b_k) {  // K-major B: one box of 64 rows (B's columns) per unit
              for (int u = 0; u < ug; ++u)
                tma_load_2d_pair(dst + u * UNIT_BYTES, &tm_b, leader_full, k0, n0 + u * (HALF / 2));
            } else {
              for (int c = 0; c < (HALF / 2) * ug / CH; ++c)
                tma_load_2d_pair(dst + c * CH * SLICE, &tm_b, leader_full, n0 + c * CH, k0);
            }
          }
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
    producer_done:;
    }
    __syncwarp();
  } else if (warp == 1) {
    if (lane == 0 && rank == 0) {
      const std::uint32_t idesc_full =
          idesc_make(F::code, F::code, p.a_mn != 0, p.b_k == 0, static_cast<std::uint32_t>(2 * HALF), PAIR_BN);
      const std::uint32_t idesc_half =
          idesc_make(F::code, F::code, p.a_mn != 0, p.b_k == 0, static_cast<std::uint32_t>(2 * HALF), PAIR_BN / 2);
      constexpr bool MN32 = F::bytes == 4;
      const std::uint32_t a_layout = (MN32 && p.a_mn) ? LAYOUT_SW128_32B : LAYOUT_SW128;
      const std::uint32_t b_layout = (MN32 && !p.b_k) ? LAYOUT_SW128_32B : LAYOUT_SW128;
      const std::uint32_t a_sbo = a_layout == LAYOUT_SW128_32B ? 512u : 1024u;
      const std::uint32_t b_sbo = b_layout == LAYOUT_SW128_32B ? 512u : 1024u;
      const std::uint32_t a_lbo = p.a_mn ? CH * SLICE : 16u, b_lbo = p.b_k ? 16u : CH * SLICE;
      std::uint32_t stage = 0, phase = 0, it = 0;
      PairWork work(pair, pairs, num_m, num_n, S::TILE_N, num_kb, p.streamk != 0, &plan);
      TileSpec ts;
      int kb_begin, kb_end;
      for (; work.next(ts, kb_begin, kb_end); ++it) {
        const int u0 = ts.units < 2 ? ts.units : 2, u1 = ts.units - u0;
        const std::uint32_t idesc0 = u0 == 2 ? idesc_full : idesc_half, idesc1 = u1 == 2 ? idesc_full : idesc_half;
        const std::uint32_t acc = S::ACCS == 2 ? (it & 1u) : 0u;
        const std::uint32_t acc_phase = S::ACCS == 2 ? ((it >> 1) & 1u) : (it & 1u);
        if (!mbar_wait(&tempty[acc], acc_phase ^ 1u, abort_flag, p.fault, FAULT_WAIT_TEMPTY)) goto mma_done;
        tc_fence_after();
        const std::uint32_t d_tmem = tmem_base + acc * PAIR_BN;
        for (int kb = kb_begin; kb < kb_end; ++kb) {
          if (!mbar_wait(&full[stage], phase, abort_flag, p.fault, FAULT_WAIT_FULL)) goto mma_done;
          tc_fence_after();
          const std::uint32_t a_addr = smem_u32(a_smem + stage * A_STAGE);
          const std::uint32_t b_addr = smem_u32(b_smem + stage * S::B_HALF);
#pragma unroll
          for (int kk = 0; kk < SLICE / MMA_K_BYTES; ++kk) {
            const std::uint32_t a_off = p.a_mn ? kk * (MMA_K_ROWS / 8) * 1024 : kk * MMA_K_BYTES;
            const std::uint32_t b_off = p.b_k ? kk * MMA_K_BYTES : kk * (MMA_K_ROWS / 8) * 1024;
            const std::uint64_t a_desc = sdesc(a_addr + a_off, a_lbo, a_sbo, a_layout);
            const std::uint32_t accumulate = (kb != kb_begin || kk != 0) ? 1u : 0u;
            umma_pair<F::kind>(d_tmem, a_desc, sdesc(b_addr + b_off, b_lbo, b_sbo, b_layout), idesc0, accumulate);
            if (G == 2 && u1 != 0)
              umma_pair<F::kind>(d_tmem + PAIR_BN, a_desc, sdesc(b_addr + GROUP_BYTES + b_off, b_lbo, b_sbo, b_layout),
                                 idesc1, accumulate);
          }
          tc_commit_pair(cluster_addr(&empty[stage], 0));
          tc_commit_pair(cluster_addr(&empty[stage], 1));
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
        tc_commit_pair(cluster_addr(&tfull[acc], 0));
        tc_commit_pair(cluster_addr(&tfull[acc], 1));
      }
    mma_done:
      tc_commit_pair(cluster_addr(drain, 0));
      drain_wait(drain, 0u, p.fault);
    }
    __syncwarp();
  } else {
    const int quarter = warp & 3;                       // TMEM lanes 32 * (warp id % 4) .. + 31
    const int ew = warp - 2;                            // epilogue warp 0..EPI_WARPS-1
    constexpr int CHUNKS = S::TILE_N / 64;              // chunks per warp of a uniform tile (the stream-K slots)
    constexpr std::size_t SLOT = static_cast<std::size_t>(S::EPI_WARPS) * CHUNKS * 32 * 32;  // floats per slot
    std::uint8_t* stage = epi_stage + ew * STAGE_BYTES;
    MaskTiles mt{&tm_m, &mask_bars[ew], 0u, abort_flag};
    std::uint32_t it = 0;
    PairWork work(pair, pairs, num_m, num_n, S::TILE_N, num_kb, p.streamk != 0, &plan);
    TileSpec ts;
    int kb_begin, kb_end;
    for (; work.next(ts, kb_begin, kb_end); ++it) {
      const std::uint32_t acc = S::ACCS == 2 ? (it & 1u) : 0u;
      const std::uint32_t acc_phase = S::ACCS == 2 ? ((it >> 1) & 1u) : (it & 1u);
      // each of the two warps on a lane quarter drains half the tile's columns, 32 at a time
      const int cols_per_warp = ts.units * 64, chunks = ts.units * 2;
      const int col0 = (ew / 4) * cols_per_warp;
      const int row0 = ts.mb * 2 * HALF + static_cast<int>(rank) * HALF + quarter * 32;
      const int c_first = ts.n0 + col0;  // this warp's first output column of the tile
      // The tile's bias for this warp's columns, staged in shared memory while the MMAs run: read from global
      // memory chunk by chunk during the drain, each chunk's bias waited on L2 (shared memory leaves L1 little room),
      // and the next tile's MMAs wait for the drain. (The drain of the tile before has finished with the buffer.)
      float* bias_s = p.bias != nullptr ? epi_bias + ew * (S::BIAS_BYTES / 4) : nullptr;
      if (bias_s != nullptr) {
        for (int i = lane; i < cols_per_warp; i += 32) {
          const int c = c_first + i;
          bias_s[i] = c < p.n ? __ldg(p.bias + c) : 0.0f;
        }
        __syncwarp();
      }
      if constexpr (READS || MASKED) {
        if (p.mask != nullptr)
          prefetch_row_span(p.mask, 2, p, row0 + lane, c_first, c_first + cols_per_warp);
        else if (p.out_kind == OUT_ACC_F32 && kb_begin == 0 && kb_end == num_kb)
          prefetch_row_span(p.out, 4, p, row0 + lane, c_first, c_first + cols_per_warp);
      }
      if (!mbar_wait(&tfull[acc], acc_phase, abort_flag, p.fault, FAULT_WAIT_TFULL)) break;
      tc_fence_after();
      const std::uint32_t t_row = tmem_base + (static_cast<std::uint32_t>(quarter * 32) << 16) + acc * PAIR_BN;
      // A segment holding part of a tile's k-blocks leaves its raw f32 sum in one of this CTA's two slots (slot 0
      // for the pair's first segment, slot 1 for its last); the fix-up after the grid barrier adds the parts.
      const bool split = kb_begin > 0 || kb_end < num_kb;
      float* slot = p.ws + static_cast<std::size_t>(2 * (2 * pair + static_cast<int>(rank)) + (it ? 1 : 0)) * SLOT;
      // Writes chunk ci (in r) to its destination: the tile's columns, or this segment's workspace slot.
      auto emit = [&](int ci, const std::uint32_t (&r)[32]) {
        if (split) {
          float4* dst = reinterpret_cast<float4*>(slot) + partial_cell(ew, ci, CHUNKS) + lane;
#pragma unroll
          for (int q = 0; q < 8; ++q)
            __stcg(dst + q * 32, make_float4(__uint_as_float(r[4 * q]), __uint_as_float(r[4 * q + 1]),
                                             __uint_as_float(r[4 * q + 2]), __uint_as_float(r[4 * q + 3])));
        } else {
          store_chunk_staged<READS, MASKED>(p, row0, c_first + ci * 32, r, stage, lane,
                                    bias_s != nullptr ? bias_s + ci * 32 : nullptr, &tm_c, mt);
        }
      };
      if constexpr (READS || MASKED) {
        // An epilogue that reads memory (the ReLU-gradient mask, or the old outputs of the accumulate form) keeps
        // those loads in flight rather than the TMEM loads: single-buffered, so its registers hold a chunk's loads.
#pragma unroll 1
        for (int ci = 0; ci < chunks; ++ci) {
          std::uint32_t r[32];
          tmem_ld_32x32b_x32(t_row + col0 + ci * 32, r);
          tmem_wait_ld(r);
          if (ci + 1 == chunks) {  // this warp's part of the accumulator is in registers
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive_cluster(cluster_addr(&tempty[acc], 0));
          }
          emit(ci, r);
        }
      } else {
        // Otherwise the drain is double-buffered: a TMEM load takes several hundred cycles to reach the registers,
        // so each chunk's load is issued before the chunk ahead of it is written out. The accumulator goes back to
        // the MMA issuer once the last chunk's load has landed. `chunks` is even (twice the tile's units). Outputs
        // that leave by plain TMA stores (bf16) or TMA stores and reduce-adds (f32) run the loop with their own
        // compact chunk bodies.
        auto drain_chunks = [&](auto&& put) {
          std::uint32_t ra[32], rb[32];
          tmem_ld_32x32b_x32(t_row + col0, ra);
#pragma unroll 1
          for (int ci = 0; ci < chunks; ci += 2) {
            tmem_wait_ld(ra);
            tmem_ld_32x32b_x32(t_row + col0 + (ci + 1) * 32, rb);
            put(ci, ra);
            tmem_wait_ld(rb);
            if (ci + 2 < chunks) {
              tmem_ld_32x32b_x32(t_row + col0 + (ci + 2) * 32, ra);
            } else {  // this warp's part of the accumulator is in registers
              tc_fence_before();
              __syncwarp();
              if (lane == 0) mbar_arrive_cluster(cluster_addr(&tempty[acc], 0));
            }
            put(ci + 1, rb);
          }
        };
        if (p.out_kind == OUT_BF16 && p.tma_store == 1 && !split) {
          drain_chunks([&](int ci, const std::uint32_t(&r)[32]) {
            store_chunk_bf16_tma(p, row0, c_first + ci * 32, r, stage, lane,
                                 bias_s != nullptr ? bias_s + ci * 32 : nullptr, &tm_c);
          });
        } else if (p.out_kind != OUT_BF16 && p.tma_store != 0 && !split) {
          drain_chunks([&](int ci, const std::uint32_t(&r)[32]) {
            store_chunk_f32_tma(p, row0, c_first + ci * 32, r, stage, lane, &tm_c);
          });
        } else {
          drain_chunks(emit);
        }
      }
    }
    if (p.streamk) {
      // The grid barrier: once every CTA's epilogue warps have written their partials, each CTA adds one arrival to
      // the workspace's counter; the fix-up starts when all gridDim.x arrivals of this launch are in (the host
      // passes the count before it as p.epoch). All CTAs are resident, so the wait ends; it is bounded all the same.
      __threadfence();
      __syncwarp();
      if (lane == 0) mbar_arrive(published);
      if (ew == 0 && lane == 0) {
        mbar_wait(published, 0u, abort_flag, p.fault, FAULT_WAIT_PEER);
        __threadfence();
        atomicAdd(p.flags, 1u);
      }
      if (lane == 0) {
        const std::uint32_t target = p.epoch + gridDim.x;
        const std::uint64_t start = globaltimer();
        while (static_cast<int>(ld_acquire_gpu(p.flags) - target) < 0) {
          if (*abort_flag) break;
          if (globaltimer() - start > WAIT_LIMIT_NS) {
            atomicOr(p.fault, static_cast<std::uint32_t>(FAULT_WAIT_PEER));
            *abort_flag = 1u;
            break;
          }
        }
      }
      __syncwarp();
      // The fix-up: the grid's epilogue warps take (tile, rank, 32 x 32 block) items in turn. A tile that one pair
      // computed whole was stored already; a split tile's block is the sum of its parts in pair order, then the
      // epilogue.
      const long long units = static_cast<long long>(tiles) * num_kb;
      const int per_rank = S::EPI_WARPS * CHUNKS, per_tile = 2 * per_rank;
      const int items = tiles * per_tile;
      for (int item = blockIdx.x * S::EPI_WARPS + ew; item < items && !*abort_flag;
           item += gridDim.x * S::EPI_WARPS) {
        const int tt = item / per_tile, rr = (item % per_tile) / per_rank, wc = item % per_rank;
        const int w = wc / CHUNKS, ci = wc % CHUNKS;
        const long long lo = static_cast<long long>(tt) * num_kb, hi = lo + num_kb;
        int q = static_cast<int>(lo * pairs / units);  // the pair whose range holds k-block 0 of the tile
        while (q + 1 < pairs && work.start_of(q + 1) <= lo) ++q;
        while (q > 0 && work.start_of(q) > lo) --q;
        if (work.start_of(q + 1) >= hi) continue;  // one pair's range holds the whole tile
        std::uint32_t r[32];
        for (int qq = q; qq < pairs && work.start_of(qq) < hi; ++qq) {
          const int which = work.start_of(qq) >= lo ? 0 : 1;  // the tile is this pair's first segment, or its last
          const float* part = p.ws + static_cast<std::size_t>(2 * (2 * qq + rr) + which) * SLOT;
          const float4* src = reinterpret_cast<const float4*>(part) + partial_cell(w, ci, CHUNKS) + lane;
#pragma unroll
          for (int e = 0; e < 8; ++e) {
            const float4 v = __ldcg(src + e * 32);
            if (qq == q) {
              r[4 * e] = __float_as_uint(v.x);
              r[4 * e + 1] = __float_as_uint(v.y);
              r[4 * e + 2] = __float_as_uint(v.z);
              r[4 * e + 3] = __float_as_uint(v.w);
            } else {
              r[4 * e] = __float_as_uint(__fadd_rn(__uint_as_float(r[4 * e]), v.x));
              r[4 * e + 1] = __float_as_uint(__fadd_rn(__uint_as_float(r[4 * e + 1]), v.y));
              r[4 * e + 2] = __float_as_uint(__fadd_rn(__uint_as_float(r[4 * e + 2]), v.z));
              r[4 * e + 3] = __float_as_uint(__fadd_rn(__uint_as_float(r[4 * e + 3]), v.w));
            }
          }
        }
        int mb, nb;
        tile_of(tt, num_m, num_n, mb, nb);
        const int w_quarter = (w + 2) & 3;  // epilogue warp w is warp w + 2: its TMEM lane quarter
        store_chunk_staged<READS, MASKED>(p, mb * 2 * HALF + rr * HALF + w_quarter * 32,
                                  nb * S::TILE_N + (w / 4) * (S::TILE_N / 2) + ci * 32, r, stage, lane, nullptr,
                                  &tm_c, mt);
      }
    }
    if (p.tma_store && lane == 0) bulk_wait();  // this warp's TMA stores are complete before the CTA ends
  }

  tc_fence_before();
  cluster_sync();  // every pair MMA has landed in both CTAs' TMEM and every remote arrival is done
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc_pair(tmem_base, S::TMEM_COLS);
  }
}

// ---------------------------------------------------------------------------------------------------------------
// The SIMT tile kernel: shapes the tensor maps cannot describe (a row not on 16 bytes), and k == 0. 64 x 64 tiles,
// 256 threads of 4 x 4 outputs, k in steps of 16 staged through shared memory as f32 (every storage float widens to
// f32 exactly; tf32 operands are used at full f32 precision here).
// ---------------------------------------------------------------------------------------------------------------
template <int FMT> __device__ __forceinline__ float widen(const void* base, std::size_t i);
template <> __device__ __forceinline__ float widen<FMT_BF16>(const void* b, std::size_t i) {
  return __uint_as_float(static_cast<std::uint32_t>(static_cast<const std::uint16_t*>(b)[i]) << 16);
}
template <> __device__ __forceinline__ float widen<FMT_F16>(const void* b, std::size_t i) {
  return __half2float(__ushort_as_half(static_cast<const std::uint16_t*>(b)[i]));
}
__device__ __forceinline__ float widen_small(std::uint32_t bits, int E, int M, bool has_inf) {
  const std::uint32_t sign = (bits >> (E + M)) & 1u, e = (bits >> M) & ((1u << E) - 1u), f = bits & ((1u << M) - 1u);
  const std::uint32_t top = (1u << E) - 1u;
  const int bias = (1 << (E - 1)) - 1;
  float v;
  if (e == top && (has_inf || f == (1u << M) - 1u)) v = (has_inf && f == 0) ? __int_as_float(0x7f800000) : __int_as_float(0x7fc00000);
  else if (e == 0) v = scalbnf(static_cast<float>(f), 1 - bias - M);
  else v = scalbnf(static_cast<float>((1u << M) | f), static_cast<int>(e) - bias - M);
  return sign ? -v : v;
}
template <> __device__ __forceinline__ float widen<FMT_E4M3>(const void* b, std::size_t i) {
  return widen_small(static_cast<const std::uint8_t*>(b)[i], 4, 3, false);
}
template <> __device__ __forceinline__ float widen<FMT_E5M2>(const void* b, std::size_t i) {
  return widen_small(static_cast<const std::uint8_t*>(b)[i], 5, 2, true);
}
template <> __device__ __forceinline__ float widen<FMT_TF32>(const void* b, std::size_t i) {
  return static_cast<const float*>(b)[i];
}

template <int FMT>
__global__ void __launch_bounds__(256) simt_gemm_kernel(const void* a, const void* b, const TcParams p) {
  __shared__ float as[16][64 + 1];
  __shared__ float bs[16][64 + 1];
  const int tiles_n = (p.n + 63) / 64;
  const int tiles = ((p.m + 63) / 64) * tiles_n;
  const int tx = threadIdx.x % 16, ty = threadIdx.x / 16;
  for (int t = blockIdx.x; t < tiles; t += gridDim.x) {
    const int m0 = (t / tiles_n) * 64, n0 = (t % tiles_n) * 64;
    float acc[4][4];
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
      for (int j = 0; j < 4; ++j) acc[i][j] = 0.0f;
    for (int k0 = 0; k0 < p.k; k0 += 16) {
      for (int e = threadIdx.x; e < 64 * 16; e += 256) {
        const int i = e / 16, q = e % 16;  // A(i, q)
        const int r = m0 + i, kk = k0 + q;
        as[q][i] = (r < p.m && kk < p.k)
                       ? widen<FMT>(a, p.a_mn ? static_cast<std::size_t>(kk) * p.m + r
                                              : static_cast<std::size_t>(r) * p.k + kk)
                       : 0.0f;
        const int j = e % 64, q2 = e / 64;  // B(q2, j)
        const int cidx = n0 + j, kk2 = k0 + q2;
        bs[q2][j] = (cidx < p.n && kk2 < p.k)
                        ? widen<FMT>(b, p.b_k ? static_cast<std::size_t>(cidx) * p.k + kk2
                                              : static_cast<std::size_t>(kk2) * p.n + cidx)
                        : 0.0f;
      }
      __syncthreads();
#pragma unroll
      for (int q = 0; q < 16; ++q) {
        float x[4], y[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) x[i] = as[q][ty * 4 + i];
#pragma unroll
        for (int j = 0; j < 4; ++j) y[j] = bs[q][tx * 4 + j];
#pragma unroll
        for (int i = 0; i < 4; ++i)
#pragma unroll
          for (int j = 0; j < 4; ++j) acc[i][j] = __fadd_rn(acc[i][j], __fmul_rn(x[i], y[j]));
      }
      __syncthreads();
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int row = m0 + ty * 4 + i;
      if (row >= p.m) continue;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int col = n0 + tx * 4 + j;
        if (col >= p.n) continue;
        const std::size_t o = static_cast<std::size_t>(row) * p.n + col;
        if (p.out_kind == OUT_BF16) {
          float v = __fadd_rn(acc[i][j], p.bias ? p.bias[col] : 0.0f);
          if (p.act == ACT_RELU) v = v < 0.0f ? 0.0f : v;
          if (p.mask != nullptr && !(__uint_as_float(static_cast<std::uint32_t>(p.mask[o]) << 16) > 0.0f)) v = 0.0f;
          static_cast<__nv_bfloat16*>(p.out)[o] = __float2bfloat16_rn(v);
        } else if (p.out_kind == OUT_ACC_F32) {
          float* c = static_cast<float*>(p.out);
          c[o] = __fadd_rn(c[o], acc[i][j]);
        } else {
          static_cast<float*>(p.out)[o] = acc[i][j];
        }
      }
    }
  }
}

// ---------------------------------------------------------------------------------------------------------------
// Host side
// ---------------------------------------------------------------------------------------------------------------
namespace {

using EncodeTiled = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                 const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                 CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiled encoder() {
  static EncodeTiled fn = []() -> EncodeTiled {
    void* f = nullptr;
    cudaDriverEntryPointQueryResult q{};
    if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &f, 12000, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess)
      return nullptr;
    return reinterpret_cast<EncodeTiled>(f);
  }();
  return fn;
}

CUtensorMapDataType map_type(int fmt) {
  switch (fmt) {
    case FMT_BF16: return CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
    case FMT_F16: return CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
    case FMT_TF32: return CU_TENSOR_MAP_DATA_TYPE_FLOAT32;
    default: return CU_TENSOR_MAP_DATA_TYPE_UINT8;
  }
}

// A 2-D row-major array of `rows` rows of `cols` elements, read in boxes of box_cols x box_rows with 128-byte rows,
// swizzled as the MMA will read the tile: 32-byte atoms for an M/N-major 32-bit operand, 16-byte atoms otherwise.
bool encode(CUtensorMap* map, int fmt, const void* base, std::uint64_t cols, std::uint64_t rows, int esize,
            std::uint32_t box_cols, std::uint32_t box_rows, bool mn_major) {
  EncodeTiled fn = encoder();
  if (!fn) return false;
  const cuuint64_t dims[2] = {cols, rows};
  const cuuint64_t strides[1] = {cols * static_cast<cuuint64_t>(esize)};
  const cuuint32_t box[2] = {box_cols, box_rows};
  const cuuint32_t estr[2] = {1, 1};
  const CUtensorMapSwizzle swizzle =
      (mn_major && esize == 4) ? CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B : CU_TENSOR_MAP_SWIZZLE_128B;
  return fn(map, map_type(fmt), 2, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
            swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

int esize_of(int fmt) { return fmt == FMT_TF32 ? 4 : (fmt == FMT_E4M3 || fmt == FMT_E5M2) ? 1 : 2; }

// The pair kernel's output as the target of TMA stores: boxes of 32 rows of 64 bytes (a bf16 epilogue chunk, or
// half of an f32 one), 64-byte swizzled. Needs the output on 16 bytes and rows of whole 16-byte groups.
bool encode_out(CUtensorMap* map, void* out, std::uint64_t n, std::uint64_t m, bool f32) {
  EncodeTiled fn = encoder();
  if (!fn) return false;
  const cuuint64_t dims[2] = {n, m};
  const cuuint64_t strides[1] = {n * (f32 ? 4 : 2)};
  const cuuint32_t box[2] = {f32 ? 16u : 32u, 32};
  const cuuint32_t estr[2] = {1, 1};
  return fn(map, f32 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, out, dims, strides, box,
            estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_64B, CU_TENSOR_MAP_L2_PROMOTION_NONE,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

bool aligned16(const void* p) { return (reinterpret_cast<std::uintptr_t>(p) & 15u) == 0; }

// Which tile runs: 0 the one-SM 128 x BN tile, 1 the pair's 256 x 256, 2 the pair's 256 x 512. The pair tiles pay
// off once both extents fill them, 256 x 512 wherever n allows it. CAIRN_B200_PAIR=0, 1 or 2 pins the choice for
// measuring the kernels against each other (whichever runs computes the whole product).
int pair_path(const GemmArgs& g) {
  static const int pinned = [] {
    const char* v = std::getenv("CAIRN_B200_PAIR");
    return (v && v[0] >= '0' && v[0] <= '2') ? v[0] - '0' : -1;
  }();
  if (g.m < 256 || g.n < 256) return 0;
  if (pinned >= 0) return pinned;
  return g.n >= 512 ? 2 : 1;
}

// How the pair kernel covers `tiles` tiles of `num_kb` k-blocks with at most `most` resident pairs. Data-parallel
// (each pair takes whole tiles in turn) unless the tiles would leave most pairs idle while each has a long k loop:
// then stream-K spreads the k-blocks of all tiles evenly over more pairs, at least STREAMK_MIN_KB each, and the pairs
// that share a tile add their partial sums through a workspace. Measured on a B200 (4096^3 bf16): with as many tiles
// as pairs or more, splitting k costs more than the last wave's idle pairs do (DRAM reads 161 MB against 78 MB, L2
// hits 70 % against 79 %: pairs that share a panel no longer read it at the same time), so it is not used there.
// CAIRN_B200_STREAMK=0 or 1 pins the choice (1 splits whenever there is more than one pair).
constexpr int STREAMK_MIN_KB = 32;
struct PairPlan {
  int pairs;
  bool streamk;
};
PairPlan pair_plan(int tiles, int num_kb, int resident, int sms) {
  static const int pinned = [] {
    const char* v = std::getenv("CAIRN_B200_STREAMK");
    return (v && (v[0] == '0' || v[0] == '1')) ? v[0] - '0' : -1;
  }();
  const int most = resident > 0 ? resident : sms / 2;
  const PairPlan dp{tiles < most ? tiles : most, false};
  const bool want = pinned >= 0 ? pinned == 1 : (2 * tiles <= most && num_kb >= 2 * STREAMK_MIN_KB);
  if (!want || resident <= 0) return dp;  // stream-K's finishing pairs wait for the others: all must be resident
  const long long units = static_cast<long long>(tiles) * num_kb;
  long long pairs = units / STREAMK_MIN_KB;
  pairs = pairs > tiles ? pairs : tiles;
  pairs = pairs < most ? pairs : most;
  if (pairs < 2) return dp;
  return PairPlan{static_cast<int>(pairs), true};
}

// ---- mixed-width tiles --------------------------------------------------------------------------------------------
// The uniform cover (tiles of 256 x 512) leaves pairs idle in the last wave whenever the tile count is not near a
// multiple of the pairs: 4096^3 has 128 tiles for 74 pairs, a second wave of 54 tiles in which 20 pairs wait, so the
// product takes two tile-times for 1.73 tile-times of work. The planner covers each 256-row band with tiles of four
// and three 128-column units (512 and 384 columns: every band of at least six units splits so), choosing per band how
// many of each so that, dealt largest first to the least loaded pair, the most loaded pair holds as few units as
// possible: for 4096^3, 74 tiles of 512 and 72 of 384 columns, seven units on every pair but two, where the uniform
// cover puts eight on 54 of them. Tile widths are whole 64-column TMA boxes of B per CTA (B row-major: boxes of 64
// columns; B transposed: boxes of 64 of its rows), so the plan is for 16-bit operands in either layout; other shapes
// and formats keep the uniform cover. Kept per shape.
struct PlannedShape {
  std::uint64_t m, n;
  int pairs;
  bool ok;
  PairTiles tiles;
};

// Units of the most loaded pair when tiles of 4 units (`fours`) and 3 units (`threes`) are dealt largest first to
// the least loaded of `pairs` pairs.
int lpt_makespan(long long fours, long long threes, int pairs) {
  std::vector<int> load(static_cast<std::size_t>(pairs), 0);
  auto deal = [&](long long count, int size) {
    for (long long i = 0; i < count; ++i) {
      std::size_t best = 0;
      for (std::size_t q = 1; q < load.size(); ++q)
        if (load[q] < load[best]) best = q;
      load[best] += size;
    }
  };
  deal(fours, 4);
  deal(threes, 3);
  int most = 0;
  for (int v : load) most = v > most ? v : most;
  return most;
}

bool plan_pair_tiles(const GemmArgs& g, int pairs, PairTiles* out) {
  if ((g.fmt != FMT_BF16 && g.fmt != FMT_F16) || pairs < 2 || pairs > PLAN_MAX_PAIRS) return false;
  const long long num_m = static_cast<long long>((g.m + 255) / 256), units = static_cast<long long>((g.n + 127) / 128);
  if (units < 6 || units > 8191 || num_m > 65535) return false;
  const long long uniform_tiles = num_m * ((units + 3) / 4);
  if (uniform_tiles < pairs || uniform_tiles > PLAN_MAX_TILES) return false;
  const long long uniform = (uniform_tiles + pairs - 1) / pairs * 4;  // units on the most loaded pair
  std::vector<std::pair<long long, long long>> ways;                // (fours, threes) covering one band
  for (long long a = units / 4; a >= 0; --a)
    if ((units - 4 * a) % 3 == 0) ways.push_back({a, (units - 4 * a) / 3});
  long long best = uniform, best_tiles = 0, best_x = 0;
  std::size_t best_i = 0, best_j = 0;
  for (std::size_t i = 0; i < ways.size(); ++i)
    for (std::size_t j = i; j < ways.size(); ++j)
      for (long long x = 0; x <= num_m; ++x) {  // x bands split the first way, the rest the second
        const long long fours = x * ways[i].first + (num_m - x) * ways[j].first;
        const long long threes = x * ways[i].second + (num_m - x) * ways[j].second;
        if (fours + threes > PLAN_MAX_TILES) continue;
        const long long span = lpt_makespan(fours, threes, pairs);
        if (span < best || (span == best && best_tiles && fours + threes < best_tiles)) {
          best = span, best_tiles = fours + threes, best_i = i, best_j = j, best_x = x;
        }
        if (i == j) break;  // one way for every band: x does not matter
      }
  if (!best_tiles || best * 20 > uniform * 19) return false;  // keep the uniform cover unless 5 % or more is saved
  // Lay the tiles out band by band (the band's four-unit tiles, then its three-unit ones), then deal them as above:
  // all four-unit tiles in band order, then all three-unit ones, each to the least loaded pair.
  std::vector<std::uint32_t> fours_list, threes_list;
  for (long long band = 0; band < num_m; ++band) {
    const auto& w = band < best_x ? ways[best_i] : ways[best_j];
    long long unit = 0;
    for (long long a = 0; a < w.first; ++a, unit += 4)
      fours_list.push_back(static_cast<std::uint32_t>(band << 16 | unit << 3 | 4));
    for (long long b = 0; b < w.second; ++b, unit += 3)
      threes_list.push_back(static_cast<std::uint32_t>(band << 16 | unit << 3 | 3));
  }
  std::vector<int> load(static_cast<std::size_t>(pairs), 0);
  std::vector<std::vector<std::uint32_t>> mine(static_cast<std::size_t>(pairs));
  for (const auto* list : {&fours_list, &threes_list})
    for (std::uint32_t e : *list) {
      std::size_t q = 0;
      for (std::size_t r = 1; r < load.size(); ++r)
        if (load[r] < load[q]) q = r;
      load[q] += static_cast<int>(e & 7u);
      mine[q].push_back(e);
    }
  std::memset(out, 0, sizeof(*out));
  out->planned = 1;
  int k = 0;
  for (int q = 0; q < pairs; ++q) {
    out->first[q] = static_cast<std::uint16_t>(k);
    for (std::uint32_t e : mine[static_cast<std::size_t>(q)]) out->tile[k++] = e;
  }
  out->first[pairs] = static_cast<std::uint16_t>(k);
  return true;
}

// The plan for (g, pairs), made once per shape: false when the uniform cover stands. CAIRN_B200_PLAN=0 keeps the
// uniform cover (for measuring the two against each other).
bool pair_tiles_plan(const GemmArgs& g, int pairs, PairTiles* out) {
  static const bool on = [] {
    const char* v = std::getenv("CAIRN_B200_PLAN");
    return !(v && v[0] == '0');
  }();
  if (!on || (g.fmt != FMT_BF16 && g.fmt != FMT_F16)) return false;
  static std::mutex mu;
  static std::vector<PlannedShape> cache;
  std::lock_guard<std::mutex> hold(mu);
  for (const auto& c : cache)
    if (c.m == g.m && c.n == g.n && c.pairs == pairs) {
      if (c.ok) *out = c.tiles;
      return c.ok;
    }
  PlannedShape made{g.m, g.n, pairs, false, {}};
  made.ok = plan_pair_tiles(g, pairs, &made.tiles);
  if (cache.size() < 64) cache.push_back(made);
  if (made.ok) *out = made.tiles;
  return made.ok;
}

template <int FMT, int BN>
cudaError_t launch_tc(const GemmArgs& g, const TcParams& p, cudaStream_t stream, int sms) {
  using S = Shape<BN>;
  constexpr int CH = SLICE / Fmt<FMT>::bytes;
  const int es = Fmt<FMT>::bytes;
  CUtensorMap ta, tb;
  const bool ok_a = g.trans_a ? encode(&ta, FMT, g.a, g.m, g.k, es, CH, CH, true)
                              : encode(&ta, FMT, g.a, g.k, g.m, es, CH, BM, false);
  const bool ok_b = g.trans_b ? encode(&tb, FMT, g.b, g.k, g.n, es, CH, BN, false)
                              : encode(&tb, FMT, g.b, g.n, g.k, es, CH, CH, true);
  if (!ok_a || !ok_b) return cudaErrorInvalidValue;
  // The shared-memory opt-in is a property of the kernel on each device: set once per device before its first launch.
  static std::atomic<std::uint64_t> configured{0};
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  const std::uint64_t bit = 1ull << (dev & 63);
  if (!(configured.load(std::memory_order_acquire) & bit)) {
    e = cudaFuncSetAttribute(tc_gemm_kernel<FMT, BN>, cudaFuncAttributeMaxDynamicSharedMemorySize, S::SMEM);
    if (e != cudaSuccess) return e;
    configured.fetch_or(bit, std::memory_order_acq_rel);
  }
  const int tiles = ((p.m + BM - 1) / BM) * ((p.n + BN - 1) / BN);
  const int grid = tiles < sms ? tiles : sms;
  tc_gemm_kernel<FMT, BN><<<grid, 192, S::SMEM, stream>>>(ta, tb, p);
  return cudaGetLastError();
}

// The pair kernel's dynamic shared memory, set once per device and instantiation before its first launch.
template <int FMT, int G, int EPI> cudaError_t configure_pair() {
  static std::atomic<std::uint64_t> configured{0};
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  const std::uint64_t bit = 1ull << (dev & 63);
  if (configured.load(std::memory_order_acquire) & bit) return cudaSuccess;
  e = cudaFuncSetAttribute(tc_gemm_pair_kernel<FMT, G, EPI>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           PairShape<G>::SMEM);
  if (e != cudaSuccess) return e;
  configured.fetch_or(bit, std::memory_order_acq_rel);
  return cudaSuccess;
}

// How many pairs (two-CTA clusters) of the G-group kernel the device holds at once: clusters must fit inside one
// GPC, so this can be below sms / 2. Every storage format's instantiation has the same shared memory and threads,
// so the bf16 one answers for all. Cached per device; 0 when the query fails (stream-K is then not used, since its
// finishing CTAs wait for the others and so need them all resident).
template <int G> int resident_pairs(int sms) {
  static std::atomic<int> cached[64] = {};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return 0;
  const int known = cached[dev & 63].load(std::memory_order_acquire);
  if (known) return known;
  if (configure_pair<FMT_BF16, G, 0>() != cudaSuccess) return 0;
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(sms, 1, 1);
  cfg.blockDim = dim3(PairShape<G>::THREADS, 1, 1);
  cfg.dynamicSmemBytes = PairShape<G>::SMEM;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  int clusters = 0;
  if (cudaOccupancyMaxActiveClusters(&clusters, tc_gemm_pair_kernel<FMT_BF16, G, 0>, &cfg) != cudaSuccess ||
      clusters <= 0) {
    cudaGetLastError();  // leave no sticky error behind for the launch to report
    return 0;
  }
  const int pairs = clusters < sms / 2 ? clusters : sms / 2;
  cached[dev & 63].store(pairs, std::memory_order_release);
  return pairs;
}

template <int FMT, int G>
cudaError_t launch_pair(const GemmArgs& g, const TcParams& p, cudaStream_t stream, int sms) {
  using S = PairShape<G>;
  constexpr int CH = SLICE / Fmt<FMT>::bytes;
  constexpr int HALF = PAIR_BN / 2;
  const int es = Fmt<FMT>::bytes;
  CUtensorMap ta, tb;
  const bool ok_a = g.trans_a ? encode(&ta, FMT, g.a, g.m, g.k, es, CH, CH, true)
                              : encode(&ta, FMT, g.a, g.k, g.m, es, CH, HALF, false);
  // K-major B (stored n x k) comes in boxes of 64 of its rows, one per 128-column unit's half, so that tiles of any
  // width take it.
  const bool ok_b = g.trans_b ? encode(&tb, FMT, g.b, g.k, g.n, es, CH, HALF / 2, false)
                              : encode(&tb, FMT, g.b, g.n, g.k, es, CH, CH, true);
  if (!ok_a || !ok_b) return cudaErrorInvalidValue;
  // Outputs leave through TMA stores where the output's tensor map allows (bf16, f32 stored, f32 accumulated as a TMA
  // reduce-add into C, and bf16 under the ReLU-gradient mask, whose tiles come in by TMA). Epilogues off the
  // tensor-map rules that read memory (the mask, the accumulate form's old C) run their own instantiation, whose drain
  // keeps those loads in flight; the others keep the double-buffered TMEM drain. CAIRN_B200_TMA_STORE=0 keeps the
  // threads' own stores and loads (for measuring one against the other).
  static const bool tma_store_on = [] {
    const char* v = std::getenv("CAIRN_B200_TMA_STORE");
    return !(v && v[0] == '0');
  }();
  CUtensorMap tc, tm;
  std::memset(&tc, 0, sizeof(tc));
  std::memset(&tm, 0, sizeof(tm));
  const bool f32_out = g.out_kind != OUT_BF16;
  const bool tma_ok = tma_store_on && p.vec && encode_out(&tc, g.out, g.n, g.m, f32_out) &&
                      (p.mask == nullptr ||
                       (p.mask_vec && encode_out(&tm, const_cast<std::uint16_t*>(g.mask), g.n, g.m, false)));
  const int tma_store = !tma_ok ? 0 : p.mask != nullptr ? 3 : g.out_kind == OUT_ACC_F32 ? 2 : 1;
  const bool reads = !tma_ok && (p.mask != nullptr || p.out_kind == OUT_ACC_F32);
  const int epi = tma_store == 3 ? 2 : reads ? 1 : 0;
  cudaError_t e = epi == 2 ? configure_pair<FMT, G, 2>() : epi == 1 ? configure_pair<FMT, G, 1>()
                                                                  : configure_pair<FMT, G, 0>();
  if (e != cudaSuccess) return e;
  const int tiles = ((p.m + 2 * HALF - 1) / (2 * HALF)) * ((p.n + S::TILE_N - 1) / S::TILE_N);
  const int num_kb = (p.k + CH - 1) / CH;
  PairPlan plan = pair_plan(tiles, num_kb, resident_pairs<G>(sms), sms);
  if (plan.streamk && g.ws == nullptr) plan = pair_plan(tiles, num_kb, 0, sms);  // no workspace: data-parallel
  int pairs = plan.pairs;
  // Mixed-width tiles where the uniform cover's last wave leaves pairs idle (data-parallel G = 2 launches only).
  static thread_local PairTiles cover;
  cover.planned = 0;
  if (G == 2 && !plan.streamk) {
    const int resident = resident_pairs<G>(sms);
    if (resident > 0 && pair_tiles_plan(g, resident, &cover)) pairs = resident;
  }
  TcParams q = p;
  q.streamk = plan.streamk;
  q.flags = static_cast<std::uint32_t*>(g.ws);  // the workspace: the barrier's arrival counter, then the slots
  q.ws = g.ws ? reinterpret_cast<float*>(static_cast<char*>(g.ws) + 256) : nullptr;
  q.epoch = g.epoch;
  q.tma_store = tma_store;
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(2 * pairs, 1, 1);
  cfg.blockDim = dim3(S::THREADS, 1, 1);
  cfg.dynamicSmemBytes = S::SMEM;
  cfg.stream = stream;
  // A programmatic dependent launch: the kernel's set-up may overlap the tail of the grid before it on the stream (it
  // waits for that grid before touching global memory). CAIRN_B200_PDL=0 launches it plainly (for measuring).
  static const bool pdl_on = [] {
    const char* v = std::getenv("CAIRN_B200_PDL");
    return !(v && v[0] == '0');
  }();
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl_on ? 2 : 1;
  e = epi == 2   ? cudaLaunchKernelEx(&cfg, tc_gemm_pair_kernel<FMT, G, 2>, ta, tb, tc, tm, q, cover)
      : epi == 1 ? cudaLaunchKernelEx(&cfg, tc_gemm_pair_kernel<FMT, G, 1>, ta, tb, tc, tm, q, cover)
                 : cudaLaunchKernelEx(&cfg, tc_gemm_pair_kernel<FMT, G, 0>, ta, tb, tc, tm, q, cover);
  if (e != cudaSuccess) return e;
  return cudaGetLastError();
}

template <int FMT> cudaError_t launch_simt(const GemmArgs& g, const TcParams& p, cudaStream_t stream, int sms) {
  const int tiles = ((p.m + 63) / 64) * ((p.n + 63) / 64);
  const int grid = tiles < sms * 8 ? tiles : sms * 8;
  simt_gemm_kernel<FMT><<<grid, 256, 0, stream>>>(g.a, g.b, p);
  return cudaGetLastError();
}

template <int FMT> cudaError_t dispatch(const GemmArgs& g, const TcParams& p, cudaStream_t s, int sms, bool tc) {
  if (!tc) return launch_simt<FMT>(g, p, s, sms);
  switch (pair_path(g)) {
    case 1: return launch_pair<FMT, 1>(g, p, s, sms);
    case 2: return launch_pair<FMT, 2>(g, p, s, sms);
    default: break;
  }
  if (p.n > 128) return launch_tc<FMT, 256>(g, p, s, sms);
  return launch_tc<FMT, 128>(g, p, s, sms);
}

}  // namespace

// Whether the tensor-core path can read the operands through TMA: 16-byte aligned bases and row strides, extents
// that fit the tensor map, and at least one slice of k.
bool tensor_path_ok(const GemmArgs& g) {
  const std::uint64_t es = static_cast<std::uint64_t>(esize_of(g.fmt));
  if (g.k == 0 || g.m == 0 || g.n == 0) return false;
  if (!aligned16(g.a) || !aligned16(g.b)) return false;
  const std::uint64_t a_row = (g.trans_a ? g.m : g.k) * es, b_row = (g.trans_b ? g.k : g.n) * es;
  if (a_row % 16 || b_row % 16) return false;
  const std::uint64_t lim = 1ull << 31;
  return g.m < lim && g.n < lim && g.k < lim;
}

std::size_t gemm_workspace_bytes(const GemmArgs& g, int sms, std::uint32_t* arrivals) {
  *arrivals = 0;
  if (!tensor_path_ok(g)) return 0;
  const int G = pair_path(g);
  if (G == 0) return 0;
  const int tile_n = G * PAIR_BN;
  const std::uint64_t tiles64 = ((g.m + 255) / 256) * ((g.n + tile_n - 1) / tile_n);
  const std::uint64_t ch = SLICE / esize_of(g.fmt);
  const PairPlan plan = pair_plan(static_cast<int>(tiles64), static_cast<int>((g.k + ch - 1) / ch),
                                  G == 1 ? resident_pairs<1>(sms) : resident_pairs<2>(sms), sms);
  if (!plan.streamk) return 0;
  *arrivals = 2u * static_cast<std::uint32_t>(plan.pairs);
  // the arrival counter (256 bytes), then two slots per CTA of EPI_WARPS x (tile_n / 64) blocks of 32 x 32 floats
  const std::size_t slot = static_cast<std::size_t>(8) * (tile_n / 64) * 32 * 32 * sizeof(float);
  return 256 + static_cast<std::size_t>(plan.pairs) * 2 * 2 * slot;
}

cudaError_t gemm_launch(const GemmArgs& g, cudaStream_t stream, int sms, std::uint32_t* fault) {
  TcParams p{};
  p.m = static_cast<int>(g.m);
  p.n = static_cast<int>(g.n);
  p.k = static_cast<int>(g.k);
  p.a_mn = g.trans_a;
  p.b_k = g.trans_b;
  p.out_kind = g.out_kind;
  p.out = g.out;
  p.bias = g.bias;
  p.act = g.act;
  p.mask = g.mask;
  p.mask_vec = g.mask != nullptr && aligned16(g.mask);
  p.fault = fault;
  const std::uint64_t out_es = g.out_kind == OUT_BF16 ? 2 : 4;
  p.vec = aligned16(g.out) && (g.n * out_es) % 16 == 0;
  const bool tc = tensor_path_ok(g);
  switch (g.fmt) {
    case FMT_BF16: return dispatch<FMT_BF16>(g, p, stream, sms, tc);
    case FMT_F16: return dispatch<FMT_F16>(g, p, stream, sms, tc);
    case FMT_E4M3: return dispatch<FMT_E4M3>(g, p, stream, sms, tc);
    case FMT_E5M2: return dispatch<FMT_E5M2>(g, p, stream, sms, tc);
    case FMT_TF32: return dispatch<FMT_TF32>(g, p, stream, sms, tc);
    default: return cudaErrorInvalidValue;
  }
}

}  // namespace cb

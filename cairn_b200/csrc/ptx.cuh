// Thin inline-PTX wrappers for the sm_100a features the kernels use: mbarriers with bounded waits, TMA tensor loads,
// and the tcgen05 family (TMEM allocation, UMMA issue, commit, TMEM loads). Every wait in this library is bounded:
// after WAIT_LIMIT_NS of polling it records a fault in the kernel's fault word, raises the block's abort flag, and
// returns false, so a kernel whose partner never arrives ends with an error status instead of hanging the GPU.
#pragma once
#include <cstdint>
#include <cstring>
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>

namespace cb {

// How long a device-side wait polls before it gives up (2 s of %globaltimer).
constexpr std::uint64_t WAIT_LIMIT_NS = 2000000000ull;

// Fault codes a kernel ORs into its fault word. The host maps any nonzero word to CAIRN_B200_ERR_TIMEOUT.
enum Fault : std::uint32_t {
  FAULT_WAIT_FULL = 1u << 0,    // the MMA issuer waited for a stage's TMA load
  FAULT_WAIT_EMPTY = 1u << 1,   // the producer waited for a stage to be consumed
  FAULT_WAIT_TFULL = 1u << 2,   // an epilogue warp waited for an accumulator
  FAULT_WAIT_TEMPTY = 1u << 3,  // the MMA issuer waited for an accumulator to be drained
  FAULT_DRAIN = 1u << 4,        // the exit path waited for copies or MMAs still in flight
  FAULT_WAIT_PEER = 1u << 5,    // a stream-K CTA waited at the grid barrier for the others' partials
  FAULT_WATCHDOG = 1u << 6,     // the watchdog self-test's wait (on a barrier nothing completes) ran out
  FAULT_WAIT_MASK = 1u << 7,    // an epilogue warp waited for its ReLU-gradient mask tile's TMA load
};

// Two floats rounded to bf16 (to nearest even) and packed, `lo` at the lower address.
__device__ __forceinline__ std::uint32_t bf16x2_bits(float lo, float hi) {
  const __nv_bfloat162 h = __floats2bfloat162_rn(lo, hi);
  std::uint32_t u;
  std::memcpy(&u, &h, 4);
  return u;
}

// A flag another CTA raises: read with acquire ordering at GPU scope, raised with release ordering.
__device__ __forceinline__ std::uint32_t ld_acquire_gpu(const std::uint32_t* p) {
  std::uint32_t v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void st_release_gpu(std::uint32_t* p, std::uint32_t v) {
  asm volatile("st.release.gpu.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
// A barrier among `count` threads of the block (a multiple of 32) on hardware barrier `id` (1..15).
__device__ __forceinline__ void named_barrier(std::uint32_t id, std::uint32_t count) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(count) : "memory");
}

__device__ __forceinline__ std::uint64_t globaltimer() {
  std::uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ std::uint32_t smem_u32(const void* p) {
  return static_cast<std::uint32_t>(__cvta_generic_to_shared(p));
}

// ---------------------------------------------------------------------------------------------------------------
// mbarrier
// ---------------------------------------------------------------------------------------------------------------
__device__ __forceinline__ void mbar_init(std::uint64_t* bar, std::uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
// Makes initialised barriers visible to the async proxy (TMA, tcgen05) before any thread uses them.
__device__ __forceinline__ void fence_barrier_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(std::uint64_t* bar, std::uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes) : "memory");
}
__device__ __forceinline__ void mbar_arrive(std::uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
// True once the phase of parity `parity` has completed.
__device__ __forceinline__ bool mbar_test(std::uint64_t* bar, std::uint32_t parity) {
  std::uint32_t done;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.b32 %0, 1, 0, p;\n\t}"
      : "=r"(done)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return done != 0;
}

// The slow half of a bounded wait: polls until the phase completes, the block's abort flag rises, or the limit
// passes (then records `fault`, raises the flag and gives up).
__device__ __noinline__ inline bool mbar_wait_slow(std::uint64_t* bar, std::uint32_t parity,
                                                   volatile std::uint32_t* abort_flag, std::uint32_t* fault_word,
                                                   std::uint32_t fault) {
  const std::uint64_t start = globaltimer();
  for (std::uint32_t spin = 1;; ++spin) {
    if (mbar_test(bar, parity)) return true;
    if ((spin & 63u) == 0) {
      if (*abort_flag) return false;
      if (globaltimer() - start > WAIT_LIMIT_NS) {
        atomicOr(fault_word, fault);
        *abort_flag = 1u;
        __threadfence_block();
        return false;
      }
    }
  }
}
__device__ __forceinline__ bool mbar_wait(std::uint64_t* bar, std::uint32_t parity, volatile std::uint32_t* abort_flag,
                                          std::uint32_t* fault_word, std::uint32_t fault) {
  if (mbar_test(bar, parity)) return true;
  return mbar_wait_slow(bar, parity, abort_flag, fault_word, fault);
}

// ---------------------------------------------------------------------------------------------------------------
// TMA (bulk tensor copies, global -> shared, completion counted on an mbarrier). Every copy lands in one CTA only.
// ---------------------------------------------------------------------------------------------------------------
__device__ __forceinline__ void tma_prefetch_desc(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<std::uint64_t>(map)) : "memory");
}
__device__ __forceinline__ void tma_load_2d(std::uint32_t dst, const CUtensorMap* map, std::uint64_t* bar,
                                            std::int32_t x, std::int32_t y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], [%2];" ::"r"(
          dst),
      "l"(reinterpret_cast<std::uint64_t>(map)), "r"(smem_u32(bar)), "r"(x), "r"(y)
      : "memory");
}

// ---------------------------------------------------------------------------------------------------------------
// tcgen05: tensor memory and the 5th-generation MMA (single-CTA group)
// ---------------------------------------------------------------------------------------------------------------
// Warp-wide: allocates `cols` TMEM columns and writes their base address to the shared slot.
__device__ __forceinline__ void tmem_alloc(std::uint32_t* slot, std::uint32_t cols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(slot)), "r"(cols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(std::uint32_t taddr, std::uint32_t cols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(cols) : "memory");
}
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
// Arrives once on `bar` when every tcgen05 operation this thread issued before it has completed.
__device__ __forceinline__ void tc_commit(std::uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}

// The MMA kinds this library issues.
enum MmaKind : int { KIND_F16 = 0, KIND_TF32 = 1, KIND_F8F6F4 = 2 };

// D[tmem] (+)= A[smem desc] * B[smem desc]; `accumulate` 0 overwrites D.
template <int KIND>
__device__ __forceinline__ void umma(std::uint32_t d_tmem, std::uint64_t a_desc, std::uint64_t b_desc,
                                     std::uint32_t idesc, std::uint32_t accumulate) {
  if constexpr (KIND == KIND_F16) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
        "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate));
  } else if constexpr (KIND == KIND_TF32) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
        "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate));
  } else {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f8f6f4 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
        "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate));
  }
}

// 32 TMEM lanes x 32 consecutive 32-bit columns: lane i of the warp receives TMEM lane (base lane + i), columns
// [col, col + 32) in r[0..31]. Warp-collective; follow with tmem_wait_ld before reading r.
__device__ __forceinline__ void tmem_ld_32x32b_x32(std::uint32_t taddr, std::uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
      "%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]),
        "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
        "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
}
__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }
// The same wait, naming the registers a tcgen05.ld filled: the compiler then schedules no read of r before it.
__device__ __forceinline__ void tmem_wait_ld(std::uint32_t (&r)[32]) {
  asm volatile("tcgen05.wait::ld.sync.aligned;"
               : "+r"(r[0]), "+r"(r[1]), "+r"(r[2]), "+r"(r[3]), "+r"(r[4]), "+r"(r[5]), "+r"(r[6]), "+r"(r[7]),
                 "+r"(r[8]), "+r"(r[9]), "+r"(r[10]), "+r"(r[11]), "+r"(r[12]), "+r"(r[13]), "+r"(r[14]), "+r"(r[15]),
                 "+r"(r[16]), "+r"(r[17]), "+r"(r[18]), "+r"(r[19]), "+r"(r[20]), "+r"(r[21]), "+r"(r[22]),
                 "+r"(r[23]), "+r"(r[24]), "+r"(r[25]), "+r"(r[26]), "+r"(r[27]), "+r"(r[28]), "+r"(r[29]),
                 "+r"(r[30]), "+r"(r[31])
               :
               : "memory");
}

// ---------------------------------------------------------------------------------------------------------------
// Programmatic dependent launch. A grid launched with cudaLaunchAttributeProgrammaticStreamSerialization may start
// while the grid before it on the stream is still running, once every CTA of that grid has issued
// griddep_launch_dependents (or exited). griddep_wait blocks until the grid before has completed and its memory
// operations are visible; without the launch attribute both are no-ops.
// ---------------------------------------------------------------------------------------------------------------
__device__ __forceinline__ void griddep_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void griddep_launch_dependents() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// ---------------------------------------------------------------------------------------------------------------
// CTA pairs (a cluster of 2): the two-SM MMA (cta_group::2). Every copy and every arrival targets one CTA.
// ---------------------------------------------------------------------------------------------------------------
__device__ __forceinline__ std::uint32_t cluster_rank() {
  std::uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
// All threads of both CTAs; orders the release of everything before it against everything after it.
__device__ __forceinline__ void cluster_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;" ::: "memory");
  asm volatile("barrier.cluster.wait.acquire.aligned;" ::: "memory");
}
// The shared::cluster address of this CTA's shared-memory object `p` as it lies in CTA `rank` of the cluster.
__device__ __forceinline__ std::uint32_t cluster_addr(const void* p, std::uint32_t rank) {
  std::uint32_t out;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(out) : "r"(smem_u32(p)), "r"(rank));
  return out;
}
// One arrival on an mbarrier anywhere in the cluster.
__device__ __forceinline__ void mbar_arrive_cluster(std::uint32_t cluster_bar) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(cluster_bar) : "memory");
}
// A TMA load into this CTA's shared memory whose completed bytes count on `cluster_bar`, an mbarrier of either CTA
// of the pair.
__device__ __forceinline__ void tma_load_2d_pair(std::uint32_t dst, const CUtensorMap* map, std::uint32_t cluster_bar,
                                                 std::int32_t x, std::int32_t y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], "
      "[%2];" ::"r"(dst),
      "l"(reinterpret_cast<std::uint64_t>(map)), "r"(cluster_bar), "r"(x), "r"(y)
      : "memory");
}
// TMA store of a box from this CTA's shared memory into the tensor at (x, y), in the thread's bulk group; elements
// outside the tensor's extents are not written. Shared-memory writes made through the generic proxy must be fenced
// (fence_proxy_async_shared) before the store reads them.
__device__ __forceinline__ void tma_store_2d(const CUtensorMap* map, std::uint32_t src, std::int32_t x, std::int32_t y) {
  asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%2, %3}], [%1];" ::"l"(
                   reinterpret_cast<std::uint64_t>(map)),
               "r"(src), "r"(x), "r"(y)
               : "memory");
}
// The same box added element by element into the tensor (f32 add, rounded to nearest), in the thread's bulk group.
__device__ __forceinline__ void tma_reduce_add_2d(const CUtensorMap* map, std::uint32_t src, std::int32_t x,
                                                  std::int32_t y) {
  asm volatile("cp.reduce.async.bulk.tensor.2d.global.shared::cta.add.bulk_group [%0, {%2, %3}], [%1];" ::"l"(
                   reinterpret_cast<std::uint64_t>(map)),
               "r"(src), "r"(x), "r"(y)
               : "memory");
}
__device__ __forceinline__ void bulk_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
// Waits until every committed bulk store of this thread has read its shared-memory source (the buffer is free).
__device__ __forceinline__ void bulk_wait_read() { asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory"); }
// Waits until every committed bulk store of this thread has completed.
__device__ __forceinline__ void bulk_wait() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }
__device__ __forceinline__ void fence_proxy_async_shared() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}
__device__ __forceinline__ void tmem_alloc_pair(std::uint32_t* slot, std::uint32_t cols) {
  asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(slot)), "r"(cols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish_pair() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc_pair(std::uint32_t taddr, std::uint32_t cols) {
  asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(cols) : "memory");
}
// Arrives once on `cluster_bar` (either CTA of the pair) when every pair MMA this thread issued has completed.
__device__ __forceinline__ void tc_commit_pair(std::uint32_t cluster_bar) {
  asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(cluster_bar)
               : "memory");
}
// The pair MMA: D (128 lanes of each CTA's TMEM) (+)= A (each CTA's half of the rows) * B (each CTA's half of the
// columns), both halves at the same shared-memory offsets the descriptors name.
template <int KIND>
__device__ __forceinline__ void umma_pair(std::uint32_t d_tmem, std::uint64_t a_desc, std::uint64_t b_desc,
                                          std::uint32_t idesc, std::uint32_t accumulate) {
  if constexpr (KIND == KIND_F16) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
        "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate));
  } else if constexpr (KIND == KIND_TF32) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::2.kind::tf32 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
        "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate));
  } else {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::2.kind::f8f6f4 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
        "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate));
  }
}

// ---------------------------------------------------------------------------------------------------------------
// UMMA descriptors (the sm_100 shared-memory matrix descriptor and the kind::f16/tf32/f8f6f4 instruction descriptor)
// ---------------------------------------------------------------------------------------------------------------
// Shared-memory layouts of the operand tiles: 128-byte rows, swizzled in 16-byte units over 8-row atoms (SW128), or
// in 32-byte units over 4-row atoms (SW128_32B: the one layout UMMA reads an M/N-major 32-bit operand from).
enum SmemLayout : std::uint32_t { LAYOUT_SW128 = 2, LAYOUT_SW128_32B = 1 };

// Shared-memory matrix descriptor: start address, leading- and stride-dimension byte offsets (all in 16-byte
// units), version 1 (sm_100) at bit 46, layout type at bits 61-63. Every tile starts on a 1024-byte boundary, a
// whole number of swizzle atoms, so the base-offset field stays 0.
__device__ __forceinline__ std::uint64_t sdesc(std::uint32_t saddr, std::uint32_t lbo_bytes, std::uint32_t sbo_bytes,
                                               std::uint32_t layout) {
  std::uint64_t d = 0;
  d |= static_cast<std::uint64_t>((saddr >> 4) & 0x3fffu);
  d |= static_cast<std::uint64_t>((lbo_bytes >> 4) & 0x3fffu) << 16;
  d |= static_cast<std::uint64_t>((sbo_bytes >> 4) & 0x3fffu) << 32;
  d |= 1ull << 46;
  d |= static_cast<std::uint64_t>(layout) << 61;
  return d;
}

// Instruction descriptor: D format f32 (bits 4-5 = 1), A and B formats (bits 7-9, 10-12), A/B major-ness (bit 15:
// A is MN-major, bit 16: B is MN-major), N >> 3 (bits 17-22), M >> 4 (bits 24-28).
__host__ __device__ constexpr std::uint32_t idesc_make(std::uint32_t a_fmt, std::uint32_t b_fmt, bool a_mn, bool b_mn,
                                                       std::uint32_t m, std::uint32_t n) {
  return (1u << 4) | (a_fmt << 7) | (b_fmt << 10) | (static_cast<std::uint32_t>(a_mn) << 15) |
         (static_cast<std::uint32_t>(b_mn) << 16) | ((n >> 3) << 17) | ((m >> 4) << 24);
}

}  // namespace cb

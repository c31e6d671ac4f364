// Drop-in replacement for CAIRN's runtime/cairn_gpu.hpp on a B200 (sm_100a): the machine that the reference's
// execution contexts (runtime/cairn_reuse.hpp) and device operations (runtime/cairn_exec.hpp) are written for.
// Generated code includes this header by name (compiler/lower/codegen.py:46); placed ahead of the reference's
// runtime directory on the include path, it is picked up with no change to the emitted source.
//
// What the reference's headers require of a machine is its concept: the type names Stream and Event, and members
// that make and destroy streams and events, order one stream after an event, wait for a stream or an event, answer
// whether a stream is capturing, allocate and release, zero and copy, run the three kinds of region, and run the
// collectors (runtime/cairn_gpu.hpp:47-125 lists them). Those names and signatures are interface and are kept. The
// machine behind them is this project's:
//
// * Regions run on cairn_kernels.hpp's persistent, device-sized grids.
// * The collectors (reduce, inclusive_scan, exclusive_sum) are cairn_cub.hpp's own kernels, not CUB's.
// * Stream-ordered allocations (alloc_async, which a context created with Allocation::stream_ordered grows its arena
//   through) come from a memory pool this machine keeps per device, whose release threshold is unbounded: memory a
//   context frees in stream order stays in the pool for its next growth instead of going back to the driver at the
//   next synchronization, and the pool is the machine's alone, so no other user of the default pool is affected.
// * Every member is one CUDA call on the stream it is given; nothing here waits for the whole device, and only
//   make_stream makes a stream. Streams are ordered after the legacy default stream, as the reference's are, so
//   work a caller queued there earlier runs first.
//
// The reference's header also kept an older synchronous API beside the machine (launch, launch_vector,
// launch_staged, copy, Ticket and its launch_async / copy_async forms, runtime/cairn_gpu.hpp:128-224); its own
// comment says generated code no longer calls it, and this header does not provide it.
#pragma once
// Marks a program built over these headers (the B200 machine) rather than over the reference's own.
#define CAIRN_B200_MACHINE 1
#if !defined(CAIRN_EMULATE)
#include <cstddef>
#include <cstdint>
#include <mutex>
#include <cuda_runtime.h>
#include "cairn_kernels.hpp"
#include "cairn_reuse.hpp"
#include "cairn_runtime.hpp"
namespace cr::gpu {
// cairn_reuse.hpp keeps its own copies of the launch defaults; a region planned against one must run with the other.
static_assert(BLOCK == reuse::BLOCK && MAX_GRID == reuse::MAX_GRID && WARP == reuse::WARP);
using reuse::Binary;
using reuse::Dir;
using reuse::Indexed;
using reuse::plain;
using reuse::Where;

namespace b200 {

// A release made while the process exits can find the CUDA runtime already unloaded (a thread's context may be
// destroyed after it); nothing is left to release then, and that is not a failure.
inline void let_go(cudaError_t e) noexcept {
  if(e != cudaErrorCudartUnloading) check(e);
}

inline cudaMemcpyKind crossing(Dir d) noexcept {
  switch(d) {
    case Dir::h2d: return cudaMemcpyHostToDevice;
    case Dir::d2h: return cudaMemcpyDeviceToHost;
    case Dir::d2d: return cudaMemcpyDeviceToDevice;
    case Dir::h2h: return cudaMemcpyHostToHost;
  }
  trap();
  return cudaMemcpyDefault;
}

// The machine's stream-ordered pool on the current device, made on first use. Device memory, unbounded release
// threshold (the pool keeps what is freed into it until the process ends).
inline cudaMemPool_t arena_pool() noexcept {
  constexpr int DEVICES = 64;
  static cudaMemPool_t pools[DEVICES];
  static std::once_flag made[DEVICES];
  int dev = 0;
  check(cudaGetDevice(&dev));
  if(dev < 0 || dev >= DEVICES) trap();
  std::call_once(made[dev], [dev] {
    cudaMemPoolProps props{};
    props.allocType = cudaMemAllocationTypePinned;
    props.location.type = cudaMemLocationTypeDevice;
    props.location.id = dev;
    check(cudaMemPoolCreate(&pools[dev], &props));
    std::uint64_t keep = ~std::uint64_t(0);
    check(cudaMemPoolSetAttribute(pools[dev], cudaMemPoolAttrReleaseThreshold, &keep));
  });
  return pools[dev];
}

}  // namespace b200

// The B200 as the machine of an execution context.
struct B200 {
  using Stream = cudaStream_t;
  using Event = cudaEvent_t;

  // Streams and events.
  Stream make_stream() noexcept {
    Stream s = nullptr;
    check(cudaStreamCreateWithFlags(&s, cudaStreamDefault));
    return s;
  }
  void destroy_stream(Stream s) noexcept { b200::let_go(cudaStreamDestroy(s)); }
  Event make_event() noexcept {
    Event e = nullptr;
    check(cudaEventCreateWithFlags(&e, cudaEventDisableTiming));
    return e;
  }
  void destroy_event(Event e) noexcept { b200::let_go(cudaEventDestroy(e)); }
  void record(Event e, Stream s) noexcept { check(cudaEventRecord(e, s)); }
  void wait_event(Stream s, Event e) noexcept { check(cudaStreamWaitEvent(s, e, 0)); }
  // A stream's handle is its address, which asks CUDA nothing and so is safe inside a graph capture; its id is
  // CUDA's, unique for the life of the process; capturing says whether a capture is recording the stream.
  unsigned long long handle(Stream s) noexcept {
    return static_cast<unsigned long long>(reinterpret_cast<std::uintptr_t>(s));
  }
  unsigned long long stream_id(Stream s) noexcept {
    unsigned long long id = 0;
    check(cudaStreamGetId(s, &id));
    return id;
  }
  bool capturing(Stream s, unsigned long long* id) noexcept {
    cudaStreamCaptureStatus status = cudaStreamCaptureStatusNone;
    check(cudaStreamGetCaptureInfo(s, &status, id));
    return status != cudaStreamCaptureStatusNone;
  }
  void sync_stream(Stream s) noexcept { check(cudaStreamSynchronize(s)); }
  void sync_event(Event e) noexcept { b200::let_go(cudaEventSynchronize(e)); }

  // Memory. alloc/free hold a context's arena; the _async pair takes it from the machine's pool in stream order;
  // allocate/release hold a scoped owner's storage where it asked to live.
  void* alloc(std::size_t bytes) noexcept {
    void* p = nullptr;
    check(cudaMalloc(&p, bytes));
    return p;
  }
  void free(void* p) noexcept { b200::let_go(cudaFree(p)); }
  void* alloc_async(std::size_t bytes, Stream s) noexcept {
    void* p = nullptr;
    check(cudaMallocFromPoolAsync(&p, bytes, b200::arena_pool(), s));
    return p;
  }
  void free_async(void* p, Stream s) noexcept { check(cudaFreeAsync(p, s)); }
  void* allocate(Where where, std::size_t bytes) noexcept {
    void* p = nullptr;
    switch(where) {
      case Where::device: check(cudaMalloc(&p, bytes)); break;
      case Where::pinned: check(cudaMallocHost(&p, bytes)); break;
      case Where::unified: check(cudaMallocManaged(&p, bytes)); break;
    }
    return p;
  }
  void release(Where where, void* p) noexcept { check(where == Where::pinned ? cudaFreeHost(p) : cudaFree(p)); }
  void zero(void* p, std::size_t bytes, Stream s) noexcept { check(cudaMemsetAsync(p, 0, bytes, s)); }
  void copy(void* dst, const void* src, std::size_t bytes, Dir d, Stream s) noexcept {
    check(cudaMemcpyAsync(dst, src, bytes, b200::crossing(d), s));
  }

  // Regions (cairn_kernels.hpp).
  template<unsigned U, class F>
  void lanes(std::size_t n, const F& body, Stream s, unsigned block, std::size_t per_lane) noexcept {
    b200::start_lanes<U>(n, body, s, block, per_lane);
  }
  template<unsigned W, unsigned U, class F, class G>
  void vector_lanes(std::size_t n, F scalar, G chunk, Stream s, unsigned block, std::size_t per_lane) noexcept {
    b200::start_chunks<W, U>(n, scalar, chunk, s, block, per_lane);
  }
  template<std::size_t R, unsigned U, class L, class F, class S>
  void staged_lanes(std::size_t n, L load, F body, S bytes, Stream s, unsigned block, std::size_t per_lane) noexcept {
    b200::start_staged<R, U>(n, load, body, bytes, s, block, per_lane);
  }

  // Collectors, defined in cairn_cub.hpp, which the lowering includes only in a program with a device reduce, scan
  // or compact. Called with a null `temp`, each only answers how many bytes of scratch it needs.
  template<class In, class Out, class Fold, class T>
  void reduce(void* temp, std::size_t& bytes, In in, Out out, std::size_t n, Fold fold, T identity, Stream s) noexcept;
  template<class In, class Out, class Fold>
  void inclusive_scan(void* temp, std::size_t& bytes, In in, Out out, Fold fold, std::size_t n, Stream s) noexcept;
  template<class In, class Out>
  void exclusive_sum(void* temp, std::size_t& bytes, In in, Out out, std::size_t n, Stream s) noexcept;
};
using Machine = B200;
}  // namespace cr::gpu

#include "cairn_exec.hpp"
#endif

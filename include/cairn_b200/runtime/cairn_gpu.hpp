// Drop-in replacement for CAIRN's runtime/cairn_gpu.hpp on a B200 (sm_100a): the machine that the execution
// contexts of runtime/cairn_reuse.hpp and the operations of runtime/cairn_exec.hpp run on, and the older
// synchronous entry points beside it. Generated code includes this header by name (compiler/lower/codegen.py:46);
// placed ahead of the reference's runtime directory on the include path, it is picked up with no source change.
//
// The machine keeps every member the context and the operations call (runtime/cairn_gpu.hpp:47-125), each one CUDA
// call as before: streams, events, allocation, copies, and the region launchers, which now come from this
// directory's cairn_kernels.hpp (persistent, device-sized grids). Its `reduce` is this project's own kernel instead
// of CUB's, and so are its scans (defined in this directory's cairn_cub.hpp).
#pragma once
// Marks a program built over these headers (the B200 machine) rather than over the reference's own.
#define CAIRN_B200_MACHINE 1
#if !defined(CAIRN_EMULATE)
#include <cstdio>
#include <cstring>
#include <cuda_runtime.h>
#include <iterator>
#include "cairn_kernels.hpp"
#include "cairn_reuse.hpp"
#include "cairn_runtime.hpp"
namespace cr::gpu {
static_assert(BLOCK == reuse::BLOCK && MAX_GRID == reuse::MAX_GRID && WARP == reuse::WARP);

// At process exit a context may outlive the CUDA runtime; its releases then have nothing left to release.
inline void released(cudaError_t e) noexcept {
  if(e != cudaErrorCudartUnloading) check(e);
}
template<class T> inline std::size_t bytes(std::size_t n) noexcept { return reuse::span<T>(n); }
using reuse::aligned;
using reuse::ALIGN;
using reuse::Binary;
using reuse::Dir;
using reuse::Indexed;
using reuse::plain;
using reuse::Where;

inline cudaMemcpyKind kind(Dir d) noexcept {
  if(d == Dir::h2d) return cudaMemcpyHostToDevice;
  if(d == Dir::d2h) return cudaMemcpyDeviceToHost;
  if(d == Dir::d2d) return cudaMemcpyDeviceToDevice;
  return cudaMemcpyHostToHost;
}

// The B200 as the machine of an execution context. Nothing here waits for the whole device; only make_stream makes a
// stream; only the alloc / allocate members allocate.
struct B200 {
  using Stream = cudaStream_t;
  using Event = cudaEvent_t;
  Stream make_stream() noexcept {
    cudaStream_t s = nullptr;
    check(cudaStreamCreate(&s));
    return s;
  }
  void destroy_stream(Stream s) noexcept { released(cudaStreamDestroy(s)); }
  Event make_event() noexcept {
    cudaEvent_t e = nullptr;
    check(cudaEventCreateWithFlags(&e, cudaEventDisableTiming));
    return e;
  }
  void destroy_event(Event e) noexcept { released(cudaEventDestroy(e)); }
  void record(Event e, Stream s) noexcept { check(cudaEventRecord(e, s)); }
  void wait_event(Stream s, Event e) noexcept { check(cudaStreamWaitEvent(s, e, 0)); }
  unsigned long long handle(Stream s) noexcept { return reinterpret_cast<std::uintptr_t>(s); }
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
  void sync_event(Event e) noexcept { released(cudaEventSynchronize(e)); }
  void* alloc(std::size_t b) noexcept {
    void* p = nullptr;
    check(cudaMalloc(&p, b));
    return p;
  }
  void free(void* p) noexcept { released(cudaFree(p)); }
  void* alloc_async(std::size_t b, Stream s) noexcept {
    void* p = nullptr;
    check(cudaMallocAsync(&p, b, s));
    return p;
  }
  void free_async(void* p, Stream s) noexcept { check(cudaFreeAsync(p, s)); }
  void* allocate(Where w, std::size_t b) noexcept {
    void* p = nullptr;
    if(w == Where::device) check(cudaMalloc(&p, b));
    else if(w == Where::pinned) check(cudaMallocHost(&p, b));
    else check(cudaMallocManaged(&p, b));
    return p;
  }
  void release(Where w, void* p) noexcept { check(w == Where::pinned ? cudaFreeHost(p) : cudaFree(p)); }
  void zero(void* p, std::size_t b, Stream s) noexcept { check(cudaMemsetAsync(p, 0, b, s)); }
  void copy(void* dst, const void* src, std::size_t b, Dir d, Stream s) noexcept {
    check(cudaMemcpyAsync(dst, src, b, kind(d), s));
  }
  template<unsigned U, class F>
  void lanes(std::size_t n, const F& body, Stream s, unsigned block, std::size_t per_lane) noexcept {
    fire<U>(n, body, s, block, per_lane);
  }
  template<unsigned W, unsigned U, class F, class G>
  void vector_lanes(std::size_t n, F scalar, G chunk, Stream s, unsigned block, std::size_t per_lane) noexcept {
    fire_vector<W, U>(n, scalar, chunk, s, block, per_lane);
  }
  template<std::size_t R, unsigned U, class L, class F, class S>
  void staged_lanes(std::size_t n, L load, F body, S bytes, Stream s, unsigned block, std::size_t per_lane) noexcept {
    fire_staged<R, U>(n, load, body, bytes, s, block, per_lane);
  }
  // Defined in cairn_cub.hpp (included only by programs with a device collector). With a null `temp` each says how
  // many bytes of scratch it needs.
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

namespace cr::gpu {

// The older synchronous entry points: the legacy default stream, then a wait for the whole device.
template<class T> inline void copy(T* dst, const T* src, std::size_t n, Dir d) noexcept {
  if(n) check(cudaMemcpy(dst, src, bytes<T>(n), kind(d)));
}
template<unsigned U = 1, class F>
inline void launch(std::size_t n, F body, unsigned block = BLOCK, std::size_t per_lane = 1) noexcept {
  fire<U>(n, body, nullptr, block, per_lane);
  check(cudaDeviceSynchronize());
}
template<unsigned W, unsigned U = 1, class F, class G>
inline void launch_vector(std::size_t n, bool whole, F scalar, G chunk, unsigned block = BLOCK,
                          std::size_t per_lane = 1) noexcept {
  if(!whole) return launch<U>(n, scalar, block, per_lane);
  if(!n) return;
  fire_vector<W, U>(n, scalar, chunk, nullptr, block, per_lane);
  check(cudaDeviceSynchronize());
}
template<std::size_t R, unsigned U = 1, class L, class F, class S>
inline void launch_staged(std::size_t n, L load, F body, S bytes, unsigned block = BLOCK,
                          std::size_t per_lane = 1) noexcept {
  if(!n) return;
  fire_staged<R, U>(n, load, body, bytes, nullptr, block, per_lane);
  check(cudaDeviceSynchronize());
}

// A ticket: one stream and one event, consumed by exactly one wait; dropping it unwaited traps.
class Ticket final {
  cudaStream_t s_ = nullptr;
  cudaEvent_t e_ = nullptr;
public:
  Ticket() noexcept {
    check(cudaStreamCreate(&s_));
    check(cudaEventCreateWithFlags(&e_, cudaEventDisableTiming));
  }
  Ticket(Ticket&& o) noexcept : s_(o.s_), e_(o.e_) { o.s_ = nullptr; o.e_ = nullptr; }
  Ticket(const Ticket&) = delete;
  Ticket& operator=(const Ticket&) = delete;
  Ticket& operator=(Ticket&&) = delete;
  ~Ticket() noexcept { if(s_) trap(); }
  cudaStream_t stream() const noexcept { return s_; }
  cudaEvent_t mark() const noexcept {
    check(cudaEventRecord(e_, s_));
    return e_;
  }
  void follow(const Ticket& dep) const noexcept {
    check(cudaEventRecord(dep.e_, dep.s_));
    check(cudaStreamWaitEvent(s_, dep.e_, 0));
  }
  void wait() && noexcept { finish(); }
  void finish() noexcept {
    check(cudaStreamSynchronize(s_));
    check(cudaEventDestroy(e_));
    check(cudaStreamDestroy(s_));
    s_ = nullptr;
    e_ = nullptr;
  }
};
inline void wait(Ticket&& t) noexcept { t.finish(); }
template<class F, class... After> inline Ticket launch_async(std::size_t n, F body, const After&... after) noexcept {
  Ticket t;
  (t.follow(after), ...);
  fire(n, body, t.stream());
  return t;
}
template<class F> inline Ticket launch_after(const Ticket& dep, std::size_t n, F body) noexcept {
  Ticket t;
  t.follow(dep);
  fire(n, body, t.stream());
  return t;
}
template<class T, class... After>
inline Ticket copy_async(T* dst, const T* src, std::size_t n, Dir d, const After&... after) noexcept {
  Ticket t;
  (t.follow(after), ...);
  if(n) check(cudaMemcpyAsync(dst, src, bytes<T>(n), kind(d), t.stream()));
  return t;
}
template<class T>
inline Ticket copy_after(const Ticket& dep, T* dst, const T* src, std::size_t n, Dir d) noexcept {
  Ticket t;
  t.follow(dep);
  if(n) check(cudaMemcpyAsync(dst, src, bytes<T>(n), kind(d), t.stream()));
  return t;
}
}  // namespace cr::gpu
#endif

// The C ABI of libcairn_b200.so (include/cairn_b200.h): argument checks with the reference's guard semantics turned
// into statuses, the per-device state (SM count, fault word) and the per-thread scratch arena.
//
// The reference keeps one execution context per host thread (runtime/cairn_exec.hpp:30-33) whose scratch arena is
// handed from one user to the next "ordered after its last one on the device, never by stopping the host"
// (runtime/cairn_reuse.hpp:188-211): the next user's stream waits on an event the previous user recorded. The arena
// here does the same, per thread and per device; it is allocated at its first use and never grows (the streaming
// reductions need a fixed amount: one 16-byte cell per block plus a ticket).
#include <cmath>
#include <cstdint>
#include <cstring>
#include <limits>
#include <mutex>
#include <vector>
#include <cuda_runtime.h>
#include "../../include/cairn_b200.h"
#include "gemm.h"

namespace cb {

// Fault word of this library's kernels on each device: a kernel whose bounded wait ran out ORs a code into it.
__device__ std::uint32_t g_fault_word;

namespace {

constexpr int MAX_DEVICES = 64;

struct Device {
  bool ready = false;
  int status = CAIRN_B200_OK;
  int sms = 0;
  std::uint32_t* fault = nullptr;
};

std::mutex g_devices_mutex;
Device g_devices[MAX_DEVICES];

// The current device's state, made on first use: it must be an sm_100 part (compute capability 10.x).
const Device* current(int* status) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= MAX_DEVICES) {
    *status = CAIRN_B200_ERR_DEVICE;
    return nullptr;
  }
  std::lock_guard<std::mutex> hold(g_devices_mutex);
  Device& d = g_devices[dev];
  if (!d.ready) {
    cudaDeviceProp prop{};
    d.status = CAIRN_B200_OK;
    if (cudaGetDeviceProperties(&prop, dev) != cudaSuccess) d.status = CAIRN_B200_ERR_CUDA;
    else if (prop.major != 10) d.status = CAIRN_B200_ERR_DEVICE;
    else {
      d.sms = prop.multiProcessorCount;
      if (cudaGetSymbolAddress(reinterpret_cast<void**>(&d.fault), g_fault_word) != cudaSuccess)
        d.status = CAIRN_B200_ERR_CUDA;
    }
    d.ready = true;
  }
  if (d.status != CAIRN_B200_OK) {
    *status = d.status;
    return nullptr;
  }
  *status = CAIRN_B200_OK;
  return &d;
}

// One thread's scratch on one device, lent to one operation at a time and ordered between streams by an event.
struct Scratch {
  void* ptr = nullptr;
  std::size_t bytes = 0;
  cudaEvent_t last{};
  bool used = false;
};
struct Arena {
  Scratch slot[MAX_DEVICES];
  Scratch gemm[MAX_DEVICES];           // the multiply's stream-K workspace, grown to the largest request
  std::uint32_t arrivals[MAX_DEVICES] = {};  // grid-barrier arrivals every launch on gemm[d] has added so far
  ~Arena() {
    for (Scratch* set : {slot, gemm})
      for (int d = 0; d < MAX_DEVICES; ++d) {
        if (set[d].ptr) cudaFree(set[d].ptr);  // errors at process exit (runtime already unloaded) are ignored
        if (set[d].last) cudaEventDestroy(set[d].last);
      }
  }
};
thread_local Arena t_arena;

// Lends the thread's scratch on the current device for work queued on `stream` after it.
int acquire(const Device& d, cudaStream_t stream, void** out) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return CAIRN_B200_ERR_CUDA;
  Scratch& s = t_arena.slot[dev];
  if (!s.ptr) {
    const std::size_t bytes = reduce_scratch_bytes(d.sms) + 256;
    if (cudaMalloc(&s.ptr, bytes) != cudaSuccess) return CAIRN_B200_ERR_CUDA;
    if (cudaMemset(s.ptr, 0, bytes) != cudaSuccess) return CAIRN_B200_ERR_CUDA;
    if (cudaEventCreateWithFlags(&s.last, cudaEventDisableTiming) != cudaSuccess) return CAIRN_B200_ERR_CUDA;
    s.bytes = bytes;
  }
  if (s.used && cudaStreamWaitEvent(stream, s.last, 0) != cudaSuccess) return CAIRN_B200_ERR_CUDA;
  *out = s.ptr;
  return CAIRN_B200_OK;
}
int release(cudaStream_t stream) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return CAIRN_B200_ERR_CUDA;
  Scratch& s = t_arena.slot[dev];
  if (cudaEventRecord(s.last, stream) != cudaSuccess) return CAIRN_B200_ERR_CUDA;
  s.used = true;
  return CAIRN_B200_OK;
}
// Lends the thread's multiply workspace on the current device, grown to `bytes` if it is smaller (the growth waits
// for the workspace's last user, frees it and allocates a zeroed one: its arrival counter must start at zero).
// Ordered after its previous user's stream like the reduction scratch. `base` is the counter's value when the
// launch starts: the arrivals of every earlier launch on this workspace.
int acquire_gemm(cudaStream_t stream, std::size_t bytes, void** out, std::uint32_t* base) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return CAIRN_B200_ERR_CUDA;
  Scratch& s = t_arena.gemm[dev];
  if (!s.last && cudaEventCreateWithFlags(&s.last, cudaEventDisableTiming) != cudaSuccess) return CAIRN_B200_ERR_CUDA;
  if (s.bytes < bytes) {
    if (s.used && cudaEventSynchronize(s.last) != cudaSuccess) return CAIRN_B200_ERR_CUDA;
    if (s.ptr) cudaFree(s.ptr);
    s.ptr = nullptr;
    s.bytes = 0;
    s.used = false;
    if (cudaMalloc(&s.ptr, bytes) != cudaSuccess) return CAIRN_B200_ERR_CUDA;
    if (cudaMemset(s.ptr, 0, bytes) != cudaSuccess) return CAIRN_B200_ERR_CUDA;
    s.bytes = bytes;
    t_arena.arrivals[dev] = 0;
  }
  if (s.used && cudaStreamWaitEvent(stream, s.last, 0) != cudaSuccess) return CAIRN_B200_ERR_CUDA;
  *out = s.ptr;
  *base = t_arena.arrivals[dev];
  return CAIRN_B200_OK;
}
// After a launch on the workspace: the next user follows it, and its arrivals (when it was launched) are counted.
int release_gemm(cudaStream_t stream, std::uint32_t added) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return CAIRN_B200_ERR_CUDA;
  Scratch& s = t_arena.gemm[dev];
  t_arena.arrivals[dev] += added;  // wraps modulo 2^32, as the kernel's comparison does
  if (cudaEventRecord(s.last, stream) != cudaSuccess) return CAIRN_B200_ERR_CUDA;
  s.used = true;
  return CAIRN_B200_OK;
}

// The cell after the reduction scratch that a _host entry reduces into before copying it back.
void* result_cell(const Device& d, void* scratch) {
  return static_cast<char*>(scratch) + reduce_scratch_bytes(d.sms);
}

// ---- guards (cr::view, cr::disjoint, cr::tensor::shape) ----------------------------------------------------------
bool view_ok(const void* p, std::size_t n, std::size_t size, std::size_t align) {
  if (n == 0) return true;
  if (p == nullptr || reinterpret_cast<std::uintptr_t>(p) % align) return false;
  if (n > SIZE_MAX / size) return false;
  return reinterpret_cast<std::uintptr_t>(p) <= UINTPTR_MAX - n * size;
}
bool overlaps(const void* a, std::size_t abytes, const void* b, std::size_t bbytes) {
  if (!abytes || !bbytes) return false;
  const auto x = reinterpret_cast<std::uintptr_t>(a), y = reinterpret_cast<std::uintptr_t>(b);
  return x < y + bbytes && y < x + abytes;
}
bool mul_ok(std::size_t a, std::size_t b, std::size_t* r) { return !__builtin_mul_overflow(a, b, r); }

int cuda_status(cudaError_t e) { return e == cudaSuccess ? CAIRN_B200_OK : CAIRN_B200_ERR_CUDA; }

std::size_t format_bytes(int fmt) {
  switch (fmt) {
    case FMT_BF16:
    case FMT_F16: return 2;
    case FMT_E4M3:
    case FMT_E5M2: return 1;
    case FMT_TF32: return 4;
    default: return 0;
  }
}

int gemm_entry(cudaStream_t stream, int fmt, std::size_t m, std::size_t n, std::size_t k, const void* a, int trans_a,
               const void* b, int trans_b, void* out, int out_kind, const float* bias, int act,
               const std::uint16_t* mask = nullptr) {
  const std::size_t es = format_bytes(fmt);
  if (!es || (out_kind != OUT_ACC_F32 && out_kind != OUT_STORE_F32 && out_kind != OUT_BF16) ||
      (act != ACT_NONE && act != ACT_RELU) || (trans_a != 0 && trans_a != 1) || (trans_b != 0 && trans_b != 1))
    return CAIRN_B200_ERR_ARG;
  std::size_t mn, mk, kn;
  if (!mul_ok(m, n, &mn) || !mul_ok(m, k, &mk) || !mul_ok(k, n, &kn)) return CAIRN_B200_ERR_SHAPE;
  const std::size_t oes = out_kind == OUT_BF16 ? 2 : 4;
  if (!view_ok(a, mk, es, es) || !view_ok(b, kn, es, es) || !view_ok(out, mn, oes, oes)) return CAIRN_B200_ERR_VIEW;
  const bool biased = out_kind == OUT_BF16 && bias != nullptr;
  if (biased && !view_ok(bias, n, 4, 4)) return CAIRN_B200_ERR_VIEW;
  if (mask && (out_kind != OUT_BF16 || !view_ok(mask, mn, 2, 2))) return CAIRN_B200_ERR_VIEW;
  if (overlaps(out, mn * oes, a, mk * es) || overlaps(out, mn * oes, b, kn * es) ||
      (biased && overlaps(out, mn * oes, bias, n * 4)) || (mask && overlaps(out, mn * oes, mask, mn * 2)))
    return CAIRN_B200_ERR_OVERLAP;
  if (!m || !n) return CAIRN_B200_OK;
  if (!k && out_kind == OUT_ACC_F32) return CAIRN_B200_OK;  // no products: every output keeps its old value
  int status;
  const Device* d = current(&status);
  if (!d) return status;
  GemmArgs g{fmt, m, n, k, a, trans_a, b, trans_b, out, out_kind, biased ? bias : nullptr, act, mask, nullptr, 0};
  std::uint32_t arrivals = 0;
  const std::size_t ws_bytes = gemm_workspace_bytes(g, d->sms, &arrivals);
  if (ws_bytes == 0) return cuda_status(gemm_launch(g, stream, d->sms, d->fault));
  if ((status = acquire_gemm(stream, ws_bytes, &g.ws, &g.epoch)) != CAIRN_B200_OK) return status;
  const cudaError_t e = gemm_launch(g, stream, d->sms, d->fault);
  const int r = release_gemm(stream, e == cudaSuccess ? arrivals : 0u);
  return e != cudaSuccess ? CAIRN_B200_ERR_CUDA : r;
}

int mma_entry(void* stream, int fmt, std::size_t m, std::size_t n, std::size_t k, float* c, std::size_t cn,
              const void* a, std::size_t an, const void* b, std::size_t bn) {
  const std::size_t es = format_bytes(fmt);
  // cr::view and cr::disjoint on the cf_ entry's views (compiler/lower/codegen.py:438-446), then
  // cr::tensor::shape (runtime/cairn_tensor.hpp:22-24).
  if (!view_ok(c, cn, 4, 4) || !view_ok(a, an, es, es) || !view_ok(b, bn, es, es)) return CAIRN_B200_ERR_VIEW;
  if (overlaps(c, cn * 4, a, an * es) || overlaps(c, cn * 4, b, bn * es)) return CAIRN_B200_ERR_OVERLAP;
  std::size_t mn, mk, kn;
  if (!mul_ok(m, n, &mn) || !mul_ok(m, k, &mk) || !mul_ok(k, n, &kn) || mn != cn || mk != an || kn != bn)
    return CAIRN_B200_ERR_SHAPE;
  return gemm_entry(static_cast<cudaStream_t>(stream), fmt, m, n, k, a, 0, b, 0, c, OUT_ACC_F32, nullptr, ACT_NONE);
}


// ---- combining the parts of a sharded f32 sum (host) -------------------------------------------------------------
// Each part is (hi, lo, flags) from cairn_b200_sum_f32_partial. The parts' values are added as an exact expansion
// (Shewchuk's grow-expansion of TwoSums: nonoverlapping components whose sum is the exact total), and the total is
// rounded once to f32 with the flags' special values, as on the device.
void two_sum(double a, double b, double& s, double& e) {
  s = a + b;
  const double z = s - a;
  e = (a - (s - z)) + (b - z);
}
float round_f32(double hi, double lo) {
  const float f = static_cast<float>(hi);
  if (lo == 0.0) return f;
  if (std::isinf(f)) {
    const double threshold = 3.4028235677973366e38;
    return (std::fabs(hi) == threshold && ((lo < 0.0) == (hi > 0.0))) ? std::copysign(3.4028234663852886e38f, f) : f;
  }
  const double fd = f;
  if (fd == hi) return f;
  const float g = hi > fd ? std::nextafter(f, INFINITY) : std::nextafter(f, -INFINITY);
  const double gd = g;
  if (hi - fd == gd - hi) return ((lo > 0.0) == (gd > fd)) ? g : f;
  return f;
}
float combine_parts(const double* parts, std::size_t count) {
  std::vector<double> e;
  unsigned flags = 0;
  for (std::size_t p = 0; p < count; ++p) {
    flags |= static_cast<unsigned>(parts[3 * p + 2]);
    for (int h = 0; h < 2; ++h) {
      double q = parts[3 * p + h];
      std::vector<double> next;
      for (double c : e) {
        double s, err;
        two_sum(q, c, s, err);
        if (err != 0.0) next.push_back(err);
        q = s;
      }
      next.push_back(q);
      e.swap(next);
    }
  }
  if ((flags & 1u) || ((flags & 2u) && (flags & 4u))) return std::numeric_limits<float>::quiet_NaN();
  if (flags & 2u) return INFINITY;
  if (flags & 4u) return -INFINITY;
  // the largest component last; fold the rest into (hi, lo) from the top
  double hi = 0.0, lo = 0.0;
  for (double c : e) {
    double s, err;
    two_sum(hi, c, s, err);
    hi = s;
    lo += err;
  }
  double s, err;
  two_sum(hi, lo, s, err);
  if (s == 0.0) return ((flags & 16u) && !(flags & 8u)) ? -0.0f : 0.0f;  // -0.0 only when every term was -0.0
  return round_f32(s, err);
}

int fault_status() {
  int status;
  const Device* d = current(&status);
  if (!d) return status;
  std::uint32_t word = 0;
  if (cudaMemcpy(&word, d->fault, sizeof word, cudaMemcpyDeviceToHost) != cudaSuccess) return CAIRN_B200_ERR_CUDA;
  if (!word) return CAIRN_B200_OK;
  const std::uint32_t zero = 0;
  if (cudaMemcpy(d->fault, &zero, sizeof zero, cudaMemcpyHostToDevice) != cudaSuccess) return CAIRN_B200_ERR_CUDA;
  return CAIRN_B200_ERR_TIMEOUT;
}

}  // namespace
}  // namespace cb

using namespace cb;

extern "C" {

int cairn_b200_mma_bf16(void* stream, size_t m, size_t n, size_t k, float* c, size_t cn, const uint16_t* a,
                        size_t an, const uint16_t* b, size_t bn) {
  return mma_entry(stream, FMT_BF16, m, n, k, c, cn, a, an, b, bn);
}
int cairn_b200_mma_f16(void* stream, size_t m, size_t n, size_t k, float* c, size_t cn, const uint16_t* a,
                       size_t an, const uint16_t* b, size_t bn) {
  return mma_entry(stream, FMT_F16, m, n, k, c, cn, a, an, b, bn);
}
int cairn_b200_mma_f8e4m3(void* stream, size_t m, size_t n, size_t k, float* c, size_t cn, const uint8_t* a,
                          size_t an, const uint8_t* b, size_t bn) {
  return mma_entry(stream, FMT_E4M3, m, n, k, c, cn, a, an, b, bn);
}
int cairn_b200_mma_f8e5m2(void* stream, size_t m, size_t n, size_t k, float* c, size_t cn, const uint8_t* a,
                          size_t an, const uint8_t* b, size_t bn) {
  return mma_entry(stream, FMT_E5M2, m, n, k, c, cn, a, an, b, bn);
}
int cairn_b200_mma_tf32(void* stream, size_t m, size_t n, size_t k, float* c, size_t cn, const float* a, size_t an,
                        const float* b, size_t bn) {
  return mma_entry(stream, FMT_TF32, m, n, k, c, cn, a, an, b, bn);
}

int cairn_b200_gemm(void* stream, int format, size_t m, size_t n, size_t k, const void* a, int trans_a,
                    const void* b, int trans_b, void* out, int out_kind, const float* bias, int act) {
  return gemm_entry(static_cast<cudaStream_t>(stream), format, m, n, k, a, trans_a, b, trans_b, out, out_kind, bias,
                    act);
}

int cairn_b200_gemm_relu_grad(void* stream, int format, size_t m, size_t n, size_t k, const void* a, int trans_a,
                              const void* b, int trans_b, uint16_t* out, const uint16_t* mask) {
  if (!mask) return CAIRN_B200_ERR_VIEW;
  return gemm_entry(static_cast<cudaStream_t>(stream), format, m, n, k, a, trans_a, b, trans_b, out, OUT_BF16, nullptr,
                    ACT_NONE, mask);
}

int cairn_b200_mse_grad(void* stream, size_t n, const float* y, const float* t, uint16_t* dy, float* loss) {
  if (!view_ok(y, n, 4, 4) || !view_ok(t, n, 4, 4) || !view_ok(dy, n, 2, 2) || !view_ok(loss, 1, 4, 4))
    return CAIRN_B200_ERR_VIEW;
  if (overlaps(dy, n * 2, y, n * 4) || overlaps(dy, n * 2, t, n * 4) || overlaps(loss, 4, dy, n * 2) ||
      overlaps(loss, 4, y, n * 4) || overlaps(loss, 4, t, n * 4))
    return CAIRN_B200_ERR_OVERLAP;
  int status;
  const Device* d = current(&status);
  if (!d) return status;
  const cudaStream_t s = static_cast<cudaStream_t>(stream);
  void* scratch = nullptr;
  if ((status = acquire(*d, s, &scratch)) != CAIRN_B200_OK) return status;
  const float scale = n ? 2.0f / static_cast<float>(n) : 0.0f;
  const cudaError_t e = mse_grad_launch(n, y, t, dy, scale, loss, scratch, s, d->sms);
  const int r = release(s);
  return e != cudaSuccess ? CAIRN_B200_ERR_CUDA : r;
}

int cairn_b200_saxpy_f32(void* stream, size_t n, float* out, const float* x, const float* y, float a) {
  if (!view_ok(out, n, 4, 4) || !view_ok(x, n, 4, 4) || !view_ok(y, n, 4, 4)) return CAIRN_B200_ERR_VIEW;
  // A lane reads its own x[i] and y[i] before it writes out[i], so out may be x or y; any other overlap races.
  if ((out != x && overlaps(out, n * 4, x, n * 4)) || (out != y && overlaps(out, n * 4, y, n * 4)))
    return CAIRN_B200_ERR_OVERLAP;
  if (!n) return CAIRN_B200_OK;
  int status;
  const Device* d = current(&status);
  if (!d) return status;
  return cuda_status(saxpy_f32_launch(n, out, x, y, a, static_cast<cudaStream_t>(stream), d->sms));
}

static int sum_f32_common(void* stream, size_t n, const float* x, float* out32, double* out64) {
  if (!view_ok(x, n, 4, 4)) return CAIRN_B200_ERR_VIEW;
  if (out32 && !view_ok(out32, 1, 4, 4)) return CAIRN_B200_ERR_VIEW;
  if (out64 && !view_ok(out64, 3, 8, 8)) return CAIRN_B200_ERR_VIEW;
  if ((out32 && overlaps(out32, 4, x, n * 4)) || (out64 && overlaps(out64, 24, x, n * 4)))
    return CAIRN_B200_ERR_OVERLAP;
  int status;
  const Device* d = current(&status);
  if (!d) return status;
  const cudaStream_t s = static_cast<cudaStream_t>(stream);
  void* scratch = nullptr;
  if ((status = acquire(*d, s, &scratch)) != CAIRN_B200_OK) return status;
  const cudaError_t e = sum_f32_launch(n, x, out32, out64, scratch, s, d->sms);
  const int r = release(s);
  return e != cudaSuccess ? CAIRN_B200_ERR_CUDA : r;
}

int cairn_b200_sum_f32(void* stream, size_t n, const float* x, float* out) {
  if (!out) return CAIRN_B200_ERR_VIEW;
  return sum_f32_common(stream, n, x, out, nullptr);
}
int cairn_b200_sum_f32_partial(void* stream, size_t n, const float* x, double* out) {
  if (!out) return CAIRN_B200_ERR_VIEW;
  return sum_f32_common(stream, n, x, nullptr, out);
}

int cairn_b200_sum_f32_host(void* stream, size_t n, const float* x, float* result) {
  if (!result || !view_ok(x, n, 4, 4)) return CAIRN_B200_ERR_VIEW;
  int status;
  const Device* d = current(&status);
  if (!d) return status;
  const cudaStream_t s = static_cast<cudaStream_t>(stream);
  void* scratch = nullptr;
  if ((status = acquire(*d, s, &scratch)) != CAIRN_B200_OK) return status;
  float* cell = static_cast<float*>(result_cell(*d, scratch));
  cudaError_t e = sum_f32_launch(n, x, cell, nullptr, scratch, s, d->sms);
  float host = 0.0f;
  if (e == cudaSuccess) e = cudaMemcpyAsync(&host, cell, sizeof host, cudaMemcpyDeviceToHost, s);
  const int r = release(s);
  if (e != cudaSuccess) return CAIRN_B200_ERR_CUDA;
  if (r != CAIRN_B200_OK) return r;
  if ((status = cairn_b200_stream_status(stream)) != CAIRN_B200_OK) return status;
  *result = host;
  return CAIRN_B200_OK;
}

int cairn_b200_sum_u64(void* stream, size_t n, const uint64_t* x, uint64_t* out, uint32_t* overflow) {
  if (!view_ok(x, n, 8, 8) || !view_ok(out, 1, 8, 8) || !view_ok(overflow, 1, 4, 4)) return CAIRN_B200_ERR_VIEW;
  if (overlaps(out, 8, x, n * 8) || overlaps(overflow, 4, x, n * 8) || overlaps(out, 8, overflow, 4))
    return CAIRN_B200_ERR_OVERLAP;
  int status;
  const Device* d = current(&status);
  if (!d) return status;
  const cudaStream_t s = static_cast<cudaStream_t>(stream);
  void* scratch = nullptr;
  if ((status = acquire(*d, s, &scratch)) != CAIRN_B200_OK) return status;
  const cudaError_t e = sum_u64_launch(n, x, out, overflow, scratch, s, d->sms);
  const int r = release(s);
  return e != cudaSuccess ? CAIRN_B200_ERR_CUDA : r;
}

int cairn_b200_sum_u64_host(void* stream, size_t n, const uint64_t* x, uint64_t* result, int* overflow) {
  if (!result || !overflow || !view_ok(x, n, 8, 8)) return CAIRN_B200_ERR_VIEW;
  int status;
  const Device* d = current(&status);
  if (!d) return status;
  const cudaStream_t s = static_cast<cudaStream_t>(stream);
  void* scratch = nullptr;
  if ((status = acquire(*d, s, &scratch)) != CAIRN_B200_OK) return status;
  char* cell = static_cast<char*>(result_cell(*d, scratch));
  auto* total = reinterpret_cast<std::uint64_t*>(cell);
  auto* flag = reinterpret_cast<std::uint32_t*>(cell + 8);
  cudaError_t e = sum_u64_launch(n, x, total, flag, scratch, s, d->sms);
  std::uint64_t host[2] = {0, 0};
  if (e == cudaSuccess) e = cudaMemcpyAsync(host, cell, 16, cudaMemcpyDeviceToHost, s);
  const int r = release(s);
  if (e != cudaSuccess) return CAIRN_B200_ERR_CUDA;
  if (r != CAIRN_B200_OK) return r;
  if ((status = cairn_b200_stream_status(stream)) != CAIRN_B200_OK) return status;
  *result = host[0];
  *overflow = static_cast<int>(host[1] & 0xffffffffu) != 0;
  return *overflow ? CAIRN_B200_ERR_OVERFLOW : CAIRN_B200_OK;
}

int cairn_b200_sum_f32_combine(const double* parts, size_t count, float* result) {
  if (!result || !view_ok(parts, count * 3, 8, 8)) return CAIRN_B200_ERR_VIEW;
  *result = combine_parts(parts, count);
  return CAIRN_B200_OK;
}

int cairn_b200_sum_f32_combine_device(void* stream, const double* parts, size_t count, float* out) {
  if (!view_ok(parts, count * 3, 8, 8) || !view_ok(out, 1, 4, 4) || count > 1u << 20) return CAIRN_B200_ERR_VIEW;
  int status;
  const Device* d = current(&status);
  if (!d) return status;
  return cuda_status(combine_f32_parts_launch(parts, static_cast<int>(count), out, static_cast<cudaStream_t>(stream)));
}

int cairn_b200_watchdog_selftest(void* stream) {
  int status;
  const Device* d = current(&status);
  if (!d) return status;
  if ((status = cairn_b200_stream_status(stream)) != CAIRN_B200_OK) return status;  // start from a clear fault word
  if (watchdog_launch(static_cast<cudaStream_t>(stream), d->fault) != cudaSuccess) return CAIRN_B200_ERR_CUDA;
  status = cairn_b200_stream_status(stream);
  if (status == CAIRN_B200_ERR_TIMEOUT) return CAIRN_B200_OK;  // the wait gave up, and its fault came back
  return status == CAIRN_B200_OK ? CAIRN_B200_ERR_DEVICE : status;
}

int cairn_b200_stream_status(void* stream) {
  const cudaError_t e = cudaStreamSynchronize(static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return CAIRN_B200_ERR_CUDA;
  return fault_status();
}

const char* cairn_b200_status_string(int status) {
  switch (status) {
    case CAIRN_B200_OK: return "ok";
    case CAIRN_B200_ERR_SHAPE: return "the extents disagree with the views";
    case CAIRN_B200_ERR_VIEW: return "a view is null, misaligned or wraps the address space";
    case CAIRN_B200_ERR_OVERLAP: return "the output overlaps an input";
    case CAIRN_B200_ERR_OVERFLOW: return "a checked unsigned sum overflowed";
    case CAIRN_B200_ERR_CUDA: return "a CUDA call failed";
    case CAIRN_B200_ERR_TIMEOUT: return "a device-side wait ran out its bound";
    case CAIRN_B200_ERR_ARG: return "an argument is outside the entry's domain";
    case CAIRN_B200_ERR_DEVICE: return "the current device is not an sm_100 part";
    case CAIRN_B200_ERR_SCRATCH: return "the launch needs more partial cells than the static scratch array holds";
    default: return "unknown status";
  }
}

int cairn_b200_clock_marks(void* stream, unsigned long long* slots, size_t count) {
  int status;
  const Device* d = current(&status);
  if (!d) return status;
  if (count == 0 || slots == nullptr || (reinterpret_cast<std::uintptr_t>(slots) & 7u) != 0) return CAIRN_B200_ERR_VIEW;
  if (count > 0xffffffffu) return CAIRN_B200_ERR_ARG;
  return clock_marks_launch(static_cast<cudaStream_t>(stream), slots, static_cast<unsigned>(count), d->sms) ==
                 cudaSuccess
             ? CAIRN_B200_OK
             : CAIRN_B200_ERR_CUDA;
}

int cairn_b200_sm_count(void) {
  int status;
  const Device* d = current(&status);
  return d ? d->sms : -status;
}

int cairn_b200_version(void) { return 100; }

}  // extern "C"

// cairn_b200_sum_f32_noalloc: the f32 `reduce +` for callers that cannot allocate device memory.
//
// The ordinary entry (cairn_b200_sum_f32) takes its scratch, one 32-byte partial per block plus a ticket, from a
// per-thread arena it allocates with cudaMalloc on the first call on each device. Some callers cannot let a library
// do that: a serving process whose device memory is fully reserved up front by its own allocator, so a cudaMalloc at
// an arbitrary point fails or fragments it; a real-time loop that cannot afford the implicit device-wide
// synchronization a cudaMalloc may cause; code that must not change the process's device-memory footprint after
// start-up. This entry runs the same kernel over a fixed scratch array compiled into the library instead, and
// allocates nothing, ever.
//
// The array is a file-scope static __device__ object of STATIC_SCRATCH_BYTES: every GPU that loads the library holds
// it until the process exits. Its size is stated by the largest grid it serves, STATIC_MAX_BLOCKS blocks (a 148-SM
// B200 launches 1184); a device whose launch would need more partial cells is refused with
// CAIRN_B200_ERR_SCRATCH and nothing is queued.
//
// In host code the array's name is only a host-side stand-in, not a device address, so the first call on each device
// (with that device current) looks its device address up with cudaGetSymbolAddress and keeps it. Make that first call
// before any stream capture begins. Every call on a device shares the one array, which keeps the last call's
// contents: the ticket that must start at zero is cleared on the caller's stream before each launch, and the partials
// are written before they are read. Calls whose work can overlap on the GPU (two streams, or two threads) race on the
// array and give wrong totals; the caller must order them, for example on one stream.
#include <cstdint>
#include <mutex>
#include <cuda_runtime.h>
#include "../../include/cairn_b200.h"
#include "gemm.h"

namespace cb {
namespace {

constexpr int STATIC_MAX_BLOCKS = 2048;                                     // partial cells the array holds
constexpr std::size_t STATIC_SCRATCH_BYTES = 256 + STATIC_MAX_BLOCKS * 32;  // the ticket, then the cells
static __device__ __align__(256) unsigned char g_static_scratch[STATIC_SCRATCH_BYTES];

constexpr int MAX_DEVICES = 64;
struct StaticScratch {
  bool ready = false;
  int status = CAIRN_B200_OK;
  int sms = 0;
  unsigned char* ptr = nullptr;  // the array's device address on this device
};
std::mutex g_static_mutex;
StaticScratch g_static[MAX_DEVICES];

// Once per device, with the device current: its SM count and the array's device address. Only a definite answer
// is kept (the address, or a device that is not an sm_100 part); a CUDA call that failed, for example because the
// first call came during a stream capture, leaves the device unresolved, and the next call asks again.
const StaticScratch* static_scratch(int* status) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= MAX_DEVICES) {
    *status = CAIRN_B200_ERR_DEVICE;
    return nullptr;
  }
  std::lock_guard<std::mutex> hold(g_static_mutex);
  StaticScratch& s = g_static[dev];
  if (!s.ready) {
    int major = 0, sms = 0;
    if (cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev) != cudaSuccess ||
        cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) {
      cudaGetLastError();
      *status = CAIRN_B200_ERR_CUDA;
      return nullptr;
    }
    if (major != 10) {
      s.status = CAIRN_B200_ERR_DEVICE;
    } else {
      void* p = nullptr;
      const cudaError_t e = cudaGetSymbolAddress(&p, g_static_scratch);
      if (e != cudaSuccess || p == nullptr) {
        cudaGetLastError();
        *status = CAIRN_B200_ERR_CUDA;
        return nullptr;
      }
      s.sms = sms;
      s.ptr = static_cast<unsigned char*>(p);
      s.status = CAIRN_B200_OK;
    }
    s.ready = true;
  }
  *status = s.status;
  return s.status == CAIRN_B200_OK ? &s : nullptr;
}

bool view_ok(const void* p, std::size_t n, std::size_t size) {
  if (n == 0) return true;
  if (p == nullptr || reinterpret_cast<std::uintptr_t>(p) % size) return false;
  return n <= SIZE_MAX / size && reinterpret_cast<std::uintptr_t>(p) <= UINTPTR_MAX - n * size;
}

}  // namespace
}  // namespace cb

extern "C" int cairn_b200_sum_f32_noalloc(void* stream, size_t n, const float* x, float* out) {
  using namespace cb;
  if (!out || !view_ok(x, n, 4) || !view_ok(out, 1, 4)) return CAIRN_B200_ERR_VIEW;
  const auto xa = reinterpret_cast<std::uintptr_t>(x), oa = reinterpret_cast<std::uintptr_t>(out);
  if (n && oa < xa + n * 4 && xa < oa + 4) return CAIRN_B200_ERR_OVERLAP;
  int status;
  const StaticScratch* s = static_scratch(&status);
  if (!s) return status;
  const int grid = sum_f32_grid(s->sms);
  if (grid > STATIC_MAX_BLOCKS) return CAIRN_B200_ERR_SCRATCH;
  const cudaStream_t st = static_cast<cudaStream_t>(stream);
  // The ticket, at the start of the array, must read zero when the kernel starts.
  if (n && cudaMemsetAsync(s->ptr, 0, sizeof(unsigned int), st) != cudaSuccess) return CAIRN_B200_ERR_CUDA;
  return sum_f32_launch(n, x, out, nullptr, s->ptr, st, s->sms) == cudaSuccess ? CAIRN_B200_OK : CAIRN_B200_ERR_CUDA;
}

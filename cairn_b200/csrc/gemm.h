// Internal interface between the C ABI (abi.cu) and the kernels (gemm.cu, stream.cu).
#pragma once
#include <cstddef>
#include <cstdint>
#include <cuda_runtime.h>

namespace cb {

// The same values as enum cairn_b200_format / cairn_b200_out / cairn_b200_act in include/cairn_b200.h.
enum : int { FMT_BF16 = 0, FMT_F16 = 1, FMT_E4M3 = 2, FMT_E5M2 = 3, FMT_TF32 = 4 };
enum : int { OUT_ACC_F32 = 0, OUT_STORE_F32 = 1, OUT_BF16 = 2 };
enum : int { ACT_NONE = 0, ACT_RELU = 1 };

struct GemmArgs {
  int fmt;
  std::uint64_t m, n, k;
  const void* a;
  int trans_a;
  const void* b;
  int trans_b;
  void* out;
  int out_kind;
  const float* bias;
  int act;
  const std::uint16_t* mask;  // OUT_BF16: zero the outputs where this bf16 m x n array is not > 0 (may be null)
  // Stream-K workspace, filled in by gemm_launch's caller when gemm_workspace_bytes asks for one: a grid barrier's
  // arrival counter (zero when the workspace was allocated) and the split tiles' f32 partials; `epoch` is the count
  // of arrivals every earlier launch on this workspace added.
  void* ws;
  std::uint32_t epoch;
};

// Bytes of stream-K workspace the product needs on a device with `sms` SMs (0: no tile is split); the flags sit at
// the end, and a fresh workspace must hold zeros there.
// The stream-K workspace a launch of g needs (0: none), and how many arrivals it adds to the workspace's counter.
std::size_t gemm_workspace_bytes(const GemmArgs& g, int sms, std::uint32_t* arrivals);

// True when the tensor-core path reads both operands through TMA (otherwise the SIMT tile kernel runs).
bool tensor_path_ok(const GemmArgs& g);
// Queues the product on `stream`; `sms` is the device's SM count, `fault` its fault word.
cudaError_t gemm_launch(const GemmArgs& g, cudaStream_t stream, int sms, std::uint32_t* fault);

// Streaming kernels (stream.cu). A reduction's scratch (reduce_scratch_bytes) starts with its ticket, one counter
// that must be zero before the launch and is zero again after it, followed 256 bytes in by one 32-byte cell per
// block of the launch's grid.
constexpr int STREAM_THREADS = 512;
int sum_f32_grid(int sms);  // blocks of each reduction's launch (STREAM_THREADS each)
int sum_u64_grid(int sms);
int mse_grid(int sms);
std::size_t reduce_scratch_bytes(int sms);
cudaError_t saxpy_f32_launch(std::size_t n, float* out, const float* x, const float* y, float a, cudaStream_t s,
                             int sms);
cudaError_t sum_f32_launch(std::size_t n, const float* x, float* out_f32, double* out_f64, void* scratch,
                           cudaStream_t s, int sms);
cudaError_t combine_f32_parts_launch(const double* parts, int count, float* out, cudaStream_t s);
cudaError_t watchdog_launch(cudaStream_t s, std::uint32_t* fault);
cudaError_t clock_marks_launch(cudaStream_t s, unsigned long long* slots, unsigned count, int sms);
// out (bf16, n) = (y - t) * scale rounded to nearest-even, and the f64 sum of (y - t)^2 into `partials` (one
// 32-byte cell per block, then the ticket); the last block writes loss[0] = f32(sum / n).
cudaError_t mse_grad_launch(std::size_t n, const float* y, const float* t, std::uint16_t* dy, float scale,
                            float* loss, void* scratch, cudaStream_t s, int sms);
cudaError_t sum_u64_launch(std::size_t n, const std::uint64_t* x, std::uint64_t* out, std::uint32_t* overflow,
                           void* scratch, cudaStream_t s, int sms);

}  // namespace cb

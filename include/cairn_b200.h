/* cairn_b200: the B200 (sm_100a) execution layer of CAIRN's data-parallel hot path, as a flat C ABI.
 *
 * Every entry point is C, takes plain pointers and sizes, and returns an int status (CAIRN_B200_OK = 0). Unless its
 * name ends in _host, an entry only queues work on `stream` (a cudaStream_t the caller owns; NULL is the legacy
 * default stream) and returns: it never waits, allocates on the call path after its first use on a device, or
 * creates streams, like the reference's enqueued `cq_NAME(stream, ...)` entries (compiler/lower/header.py:237-247,
 * runtime/cairn_exec.hpp:56-67). Device pointers are the caller's; the library owns only a small per-thread,
 * per-device scratch arena that it orders between streams with an event, as the reference's execution context does
 * (runtime/cairn_reuse.hpp:188-211).
 *
 * Where the reference traps on a violated guard (cr::trap, runtime/cairn_runtime.hpp:59-70), these entries return a
 * status and queue nothing. A device-side wait that runs out its bound (2 s) records a fault that
 * cairn_b200_stream_status reports; no kernel in this library traps.
 *
 * Citations name files of the CAIRN source tree (src/cairn/...).
 */
#ifndef CAIRN_B200_H
#define CAIRN_B200_H
#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

enum cairn_b200_status {
  CAIRN_B200_OK = 0,
  CAIRN_B200_ERR_SHAPE = 1,    /* extents disagree with the views: cr::tensor::shape traps, runtime/cairn_tensor.hpp:22-24 */
  CAIRN_B200_ERR_VIEW = 2,     /* a null or misaligned view: cr::view traps, runtime/cairn_runtime.hpp:194-200 */
  CAIRN_B200_ERR_OVERLAP = 3,  /* the output overlaps an input: cr::disjoint traps, runtime/cairn_runtime.hpp:201-205 */
  CAIRN_B200_ERR_OVERFLOW = 4, /* a checked unsigned sum did not fit: cr::Sum::checked traps, runtime/cairn_runtime.hpp:165 */
  CAIRN_B200_ERR_CUDA = 5,     /* a CUDA call failed: cr::gpu::check aborts, runtime/cairn_kernels.hpp:55-59 */
  CAIRN_B200_ERR_TIMEOUT = 6,  /* a device-side wait ran out its bound (no reference counterpart: it traps nowhere) */
  CAIRN_B200_ERR_ARG = 7,      /* an argument outside the entry's domain (unknown format, activation, ...) */
  CAIRN_B200_ERR_DEVICE = 8,   /* no sm_100 device is current */
  CAIRN_B200_ERR_SCRATCH = 9   /* the launch needs more than a fixed scratch array holds (cairn_b200_sum_f32_noalloc) */
};

/* Storage formats of the multiply's operands (runtime/cairn_float.hpp:160-167), and f32 read as tf32. */
enum cairn_b200_format {
  CAIRN_B200_BF16 = 0,
  CAIRN_B200_F16 = 1,
  CAIRN_B200_F8E4M3 = 2,
  CAIRN_B200_F8E5M2 = 3,
  CAIRN_B200_TF32 = 4
};

/* What the multiply does with its f32 accumulator. */
enum cairn_b200_out {
  CAIRN_B200_OUT_ACC_F32 = 0,   /* c (f32) += acc: the mma_unordered contract */
  CAIRN_B200_OUT_STORE_F32 = 1, /* c (f32) = acc */
  CAIRN_B200_OUT_BF16 = 2       /* out (bf16) = act(acc + bias[j]), rounded to nearest-even */
};

enum cairn_b200_act { CAIRN_B200_ACT_NONE = 0, CAIRN_B200_ACT_RELU = 1 };

/* ---- the multiply ---------------------------------------------------------------------------------------------
 * cr::tensor::launch<A>(ctx, m, n, k, c, cn, a, an, b, bn), runtime/cairn_tensor.hpp:206-221 (the device lowering
 * of mma_unordered, compiler/device/tensor.py:69-82): c (row-major m x n f32) += a (row-major m x k) * b (row-major
 * k x n), one storage float. cn, an and bn are the views' extents, checked against m*n, m*k and k*n
 * (cairn_tensor.hpp:22-24); c must not overlap a or b (the cf_ entry checks, compiler/lower/codegen.py:438-446).
 * The contract is the reference's: every product exact in f32, every output its old value plus its k products in
 * an order the hardware picks, within (k + 1) * 2^-22 * (|c| + sum |a*b|) of the exact sum. */
int cairn_b200_mma_bf16(void* stream, size_t m, size_t n, size_t k, float* c, size_t cn, const uint16_t* a,
                        size_t an, const uint16_t* b, size_t bn);
int cairn_b200_mma_f16(void* stream, size_t m, size_t n, size_t k, float* c, size_t cn, const uint16_t* a,
                       size_t an, const uint16_t* b, size_t bn);
int cairn_b200_mma_f8e4m3(void* stream, size_t m, size_t n, size_t k, float* c, size_t cn, const uint8_t* a,
                          size_t an, const uint8_t* b, size_t bn);
int cairn_b200_mma_f8e5m2(void* stream, size_t m, size_t n, size_t k, float* c, size_t cn, const uint8_t* a,
                          size_t an, const uint8_t* b, size_t bn);
/* The same over f32 operands read as tf32 by the tensor cores. The reference refuses f32 operands to
 * mma_unordered (E-MMA, compiler/device/tensor.py:49-50) and runs f32 products as `parallel` regions on the host
 * lane pool; this is their device form, with tf32 products (relative error about 2^-10 per product). */
int cairn_b200_mma_tf32(void* stream, size_t m, size_t n, size_t k, float* c, size_t cn, const float* a, size_t an,
                        const float* b, size_t bn);

/* The general product behind the entries above and the backward of a dense layer (the dX = dY W^T and dW = X^T dY
 * that derive grad writes as loops, compiler/derive/gradients.py:1-11): op(A) is a (m x k, row-major) or, with
 * trans_a, the transpose of a stored k x m; op(B) is b (k x n) or, with trans_b, the transpose of b stored n x k.
 * `out_kind` picks the epilogue (enum cairn_b200_out); `bias` (n floats, may be NULL) and `act` apply to
 * CAIRN_B200_OUT_BF16 only. `out` is f32 (m x n) or bf16 (m x n). */
int cairn_b200_gemm(void* stream, int format, size_t m, size_t n, size_t k, const void* a, int trans_a,
                    const void* b, int trans_b, void* out, int out_kind, const float* bias, int act);

/* The backward of a ReLU layer fused into its gradient product: out (bf16, m x n) = op(A) * op(B) rounded to bf16
 * where mask[i][j] (bf16, m x n: the layer's forward output) is > 0, and 0 elsewhere; derive grad's chain rule
 * through `relu` (compiler/derive/gradients.py) applied in the product's epilogue. */
int cairn_b200_gemm_relu_grad(void* stream, int format, size_t m, size_t n, size_t k, const void* a, int trans_a,
                              const void* b, int trans_b, uint16_t* out, const uint16_t* mask);

/* Mean-squared-error loss and its gradient over n f32 pairs (the MLP step's head): dy[i] = bf16((y[i] - t[i]) *
 * (2 / n)) and *loss = f32(sum (y[i] - t[i])^2 / n), the sum in f64; loss is a device f32. */
int cairn_b200_mse_grad(void* stream, size_t n, const float* y, const float* t, uint16_t* dy, float* loss);

/* ---- parallel regions -----------------------------------------------------------------------------------------
 * cr::gpu::run(ctx, n, [=](size_t i) { out[i] = a * x[i] + y[i]; }), runtime/cairn_exec.hpp:103-108 with the lane
 * kernel of runtime/cairn_kernels.hpp:69-96: every i below n once, a * x[i] and the sum each rounded to f32 (the
 * device build is --fmad=false, projects/toolchain.py:197-200). out may equal x or y (a lane reads its own
 * element before it writes it); otherwise the three must not overlap. */
int cairn_b200_saxpy_f32(void* stream, size_t n, float* out, const float* x, const float* y, float a);

/* ---- reductions -------------------------------------------------------------------------------------------------
 * `reduce + parallel i in n yield x[i]` over a device view of f32 (runtime/cairn_exec.hpp:163-180 reduce_on /
 * reduce_into, runtime/cairn_reuse.hpp:346-428), with the host's answer: the exact sum of the terms rounded once to
 * nearest-even, as cr::par::sum gives it (runtime/cairn_sum.hpp:311-331), where the reference's device path folds
 * f32 in an unspecified order. Each thread carries double-double (TwoSum) accumulators, combined the same way in a
 * fixed order for a given n and device; the double-double total is rounded to f32 with its low part deciding ties.
 * NaN, infinities and the sign of an exact zero follow cr::sum::result (cairn_sum.hpp:186-195).
 *   _f32          writes the total to *out, a device f32
 *   _f32_partial  writes the unrounded part to out[0..2], device doubles: out[0] + out[1] is the part's value as a
 *                 double-double and out[2] its flags (1 NaN, 2 +inf, 4 -inf, 8 a term other than -0.0, 16 n > 0); one rank's
 *                 part of a sharded sum
 *   _f32_host     writes the total to *result in host memory and waits for the stream (the reduce_on form)
 *   _f32_combine  host only: the f32 total of `count` parts (3 doubles each, host memory), added exactly and rounded
 *                 once, as the host's cr::par::sum rounds the exact total of all the ranks' terms
 *   _f32_combine_device  the same on `stream` from parts in device memory (after an all-gather of the ranks' parts),
 *                 the parts added as double-doubles in rank order; the total lands in *out, a device f32 */
int cairn_b200_sum_f32(void* stream, size_t n, const float* x, float* out);
int cairn_b200_sum_f32_partial(void* stream, size_t n, const float* x, double* out);
int cairn_b200_sum_f32_host(void* stream, size_t n, const float* x, float* result);
int cairn_b200_sum_f32_combine(const double* parts, size_t count, float* result);
int cairn_b200_sum_f32_combine_device(void* stream, const double* parts, size_t count, float* out);

/* `reduce + parallel` over u64 with the checked sum cr::Sum<u64> (runtime/cairn_runtime.hpp:158-166): the total
 * modulo 2^64 and a sticky overflow flag that is 1 exactly when the true total does not fit. *out and *overflow are
 * device memory (a u64 and a u32). The _host form waits and returns CAIRN_B200_ERR_OVERFLOW where the reference's
 * .checked() would trap, with the wrapped total still written. */
int cairn_b200_sum_u64(void* stream, size_t n, const uint64_t* x, uint64_t* out, uint32_t* overflow);
int cairn_b200_sum_u64_host(void* stream, size_t n, const uint64_t* x, uint64_t* result, int* overflow);

/* The f32 sum of cairn_b200_sum_f32 for callers that cannot allocate device memory: no reference counterpart (the
 * reference's reductions always take their temporaries from the context's arena). A serving process whose device
 * memory is reserved up front by its own allocator, or a loop that cannot afford a cudaMalloc's implicit
 * synchronization, calls this form: it runs the same kernel over a scratch array compiled into the library
 * (65,536 bytes of partials for at most 2048 blocks, plus the ticket; every GPU that loads the library holds it until
 * exit), and never calls cudaMalloc, cudaFree or an allocating library routine. A device whose launch would need more
 * than 2048 blocks gets CAIRN_B200_ERR_SCRATCH (a 148-SM B200 launches 1184). The first call on each device looks up the array's device address;
 * make it before any stream capture. All calls share the array: calls whose work overlaps on the GPU race, so order
 * them (one stream). Same result bits as cairn_b200_sum_f32. */
int cairn_b200_sum_f32_noalloc(void* stream, size_t n, const float* x, float* out);

/* ---- status ----------------------------------------------------------------------------------------------------
 * Waits for `stream`, then reports a CUDA error or a device-side fault recorded by this library's kernels on the
 * current device since the last call (and clears the fault). The synchronous half of a cf_ entry
 * (runtime/cairn_reuse.hpp:125-141 give_back waits on the lane's stream). */
int cairn_b200_stream_status(void* stream);
const char* cairn_b200_status_string(int status);
/* The device watchdog's self-test, synchronous on `stream`: one block waits, through the bounded wait every kernel
 * of this library uses, on a shared-memory barrier that nothing completes; the wait gives up after its 2 s limit
 * and records a fault, which this call reads back and clears. Returns CAIRN_B200_OK when all of that happened (the
 * context stays usable), CAIRN_B200_ERR_DEVICE when no fault came back, or the failing status. No reference
 * counterpart: the reference's device guards trap and poison the context (runtime/cairn_kernels.hpp:33-59). */
int cairn_b200_watchdog_selftest(void* stream);
/* Clock marks, queued on `stream`: for each SM that runs one of the entry's blocks, slots[2 * smid] = its cycle
 * counter (%clock64) and slots[2 * smid + 1] = the global nanosecond timer (%globaltimer), for smid < count (device
 * memory, 2 * count 8-byte slots; SMs without a block keep what the slots held). Two marks bracket the work queued
 * between them: an SM's cycles over nanoseconds is its average clock over that work. No reference counterpart: a
 * measurement aid (bench.py reports the SM clock inside its timed region with it). */
int cairn_b200_clock_marks(void* stream, unsigned long long* slots, size_t count);
/* The number of SMs of the current device the kernels size their grids for, or a negative status. */
int cairn_b200_sm_count(void);
/* The ABI version: major * 10000 + minor * 100 + patch. */
int cairn_b200_version(void);

#ifdef __cplusplus
}
#endif
#endif /* CAIRN_B200_H */

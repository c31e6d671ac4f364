/* TEST INFRASTRUCTURE ONLY: the CPU oracle for the cairn_b200 parity tests.
 *
 * A plain-C restatement of what CAIRN's host path computes on its data-parallel hot path. Only tests/, the smoke
 * check of __graft_entry__.py and the CPU-baseline leg of bench.py load it, and only as the checker; nothing in the
 * cairn_b200 package calls it. Every function cites the reference file:line (paths inside the CAIRN source tree)
 * whose behaviour it restates. The arithmetic is written from the stated semantics, not from the reference's code:
 *
 *   - oracle_mma_*        cr::tensor::reference, runtime/cairn_tensor.hpp:28-35: for every output its old value,
 *                         then its k products added in increasing p, each product and each partial sum rounded to
 *                         f32 (no contraction: projects/toolchain.py builds with -ffp-contract=off).
 *   - oracle_sum_f32      cr::par::sum<float>, runtime/cairn_sum.hpp:311-331 and docs/numerics.md "Parallel float
 *                         sums": the exact sum of the terms rounded once to nearest-even, with the special-value rules
 *                         of cr::sum::result (cairn_sum.hpp:186-195). Restated here as an integer count of 2^-149.
 *   - oracle_sum_u64      cr::Sum<u64> folded in index order (runtime/cairn_runtime.hpp:158-166, and
 *                         cr::par::reduce, runtime/cairn_parallel.hpp:385-399): the wrapped total and a sticky
 *                         overflow flag that is set exactly when the true total does not fit.
 *   - oracle_saxpy_f32    cr::gpu::run / cr::par::run of out[i] = a * x[i] + y[i] (runtime/cairn_exec.hpp:103-108,
 *                         cairn_parallel.hpp:372-378): two roundings, no fused multiply-add.
 *   - oracle_scan_u32     cr::par::scan<false> (runtime/cairn_parallel.hpp:401-440) of add_wrap over u32: the
 *                         inclusive prefixes modulo 2^32 in index order, and the total.
 *   - oracle_runmax_i32   cr::par::scan<true> of max over i32: out[0] = INT32_MIN, out[i] = max(x[0..i)), and the
 *                         total max(x[0..n)).
 *   - oracle_bias_act     the fused epilogue this project adds beside the multiply (the reference has none,
 *                         cairn_tensor.hpp:189-193 only stores the f32 accumulator): bf16(act(f32(acc + bias[j]))).
 *   - oracle_gemm_t16     the transposed products the derive-grad backward of a dense layer forms
 *                         (compiler/derive/gradients.py:1-11): dX += dY * W^T and dW += X^T * dY, each output a
 *                         sequential f32 sum in increasing p after its old value.
 *   - oracle_mlp_step     BASELINE config 3's 2-layer MLP forward + MSE + backward from those loops.
 */
#include <math.h>
#include <stdint.h>
#include <stddef.h>
#include <string.h>

/* ---------------------------------------------------------------------------------------------------------------
 * Storage floats (runtime/cairn_float.hpp:11-24,160-167): bf16 = (8,7) with infinities, f16 = (5,10) with
 * infinities, f8e4m3 = (4,3) OCP without infinities (only S.1111.111 is NaN), f8e5m2 = (5,2) with infinities.
 * Every value of each is exactly an f32, so decoding is exact.
 * ------------------------------------------------------------------------------------------------------------- */
static float from_bits32(uint32_t u) { float f; memcpy(&f, &u, 4); return f; }
static uint32_t bits32(float f) { uint32_t u; memcpy(&u, &f, 4); return u; }

/* A small-float pattern with E exponent bits and M fraction bits, decoded exactly. */
static float decode_small(uint32_t bits, int E, int M, int has_inf) {
  const uint32_t sign = (bits >> (E + M)) & 1u;
  const uint32_t e = (bits >> M) & ((1u << E) - 1u);
  const uint32_t f = bits & ((1u << M) - 1u);
  const uint32_t top = (1u << E) - 1u;
  const int bias = (1 << (E - 1)) - 1;
  float v;
  if (e == top && (has_inf || f == (1u << M) - 1u)) {
    v = (has_inf && f == 0) ? INFINITY : NAN;
  } else if (e == 0) {
    v = ldexpf((float)f, 1 - bias - M);  /* subnormal: f * 2^(1 - bias - M), exact */
  } else {
    v = ldexpf((float)((1u << M) | f), (int)e - bias - M);
  }
  return sign ? -v : v;
}

float oracle_bf16_to_f32(uint16_t b) { return from_bits32((uint32_t)b << 16); }
float oracle_f16_to_f32(uint16_t b) { return decode_small(b, 5, 10, 1); }
float oracle_e4m3_to_f32(uint8_t b) { return decode_small(b, 4, 3, 0); }
float oracle_e5m2_to_f32(uint8_t b) { return decode_small(b, 5, 2, 1); }

/* f32 -> bf16, round to nearest with ties to even; a NaN becomes the quiet NaN of its sign. */
uint16_t oracle_f32_to_bf16(float x) {
  uint32_t u = bits32(x);
  if ((u & 0x7fffffffu) > 0x7f800000u) return (uint16_t)(((u >> 16) & 0x8000u) | 0x7fc0u);
  const uint32_t lsb = (u >> 16) & 1u;
  u += 0x7fffu + lsb;
  return (uint16_t)(u >> 16);
}

/* ---------------------------------------------------------------------------------------------------------------
 * The multiply: cr::tensor::reference (runtime/cairn_tensor.hpp:28-35) over each storage format. Row-major c (m x n),
 * a (m x k), b (k x n). The volatile stores pin each rounding to f32 whatever the compiler's flags.
 * ------------------------------------------------------------------------------------------------------------- */
#define MMA_BODY(DECODE)                                                              \
  for (size_t i = 0; i < m; ++i)                                                      \
    for (size_t p = 0; p < k; ++p) {                                                  \
      const float x = DECODE(a[i * k + p]);                                           \
      for (size_t j = 0; j < n; ++j) {                                                \
        volatile float prod = x * DECODE(b[p * n + j]);                               \
        volatile float sum = c[i * n + j] + prod;                                     \
        c[i * n + j] = sum;                                                           \
      }                                                                               \
    }

void oracle_mma_bf16(size_t m, size_t n, size_t k, float* c, const uint16_t* a, const uint16_t* b) {
  MMA_BODY(oracle_bf16_to_f32)
}
void oracle_mma_f16(size_t m, size_t n, size_t k, float* c, const uint16_t* a, const uint16_t* b) {
  MMA_BODY(oracle_f16_to_f32)
}
void oracle_mma_e4m3(size_t m, size_t n, size_t k, float* c, const uint8_t* a, const uint8_t* b) {
  MMA_BODY(oracle_e4m3_to_f32)
}
void oracle_mma_e5m2(size_t m, size_t n, size_t k, float* c, const uint8_t* a, const uint8_t* b) {
  MMA_BODY(oracle_e5m2_to_f32)
}
#define IDENT(x) (x)
/* The f32 multiply as a CAIRN `parallel e in m*n` region with an in-order p loop: the host form of config 1
 * (mma_unordered refuses f32 operands, compiler/device/tensor.py:49-50). Same order as the storage-float loop. */
void oracle_mma_f32(size_t m, size_t n, size_t k, float* c, const float* a, const float* b) { MMA_BODY(IDENT) }

/* Only rows [r0, r1) of the bf16 multiply: the sampled-row check of large products. */
void oracle_mma_bf16_rows(size_t m, size_t n, size_t k, size_t r0, size_t r1, float* c_rows, const uint16_t* a,
                          const uint16_t* b) {
  (void)m;
  for (size_t i = r0; i < r1; ++i)
    for (size_t p = 0; p < k; ++p) {
      const float x = oracle_bf16_to_f32(a[i * k + p]);
      float* row = c_rows + (i - r0) * n;
      for (size_t j = 0; j < n; ++j) {
        volatile float prod = x * oracle_bf16_to_f32(b[p * n + j]);
        volatile float sum = row[j] + prod;
        row[j] = sum;
      }
    }
}

/* General f32-accumulating product over 16-bit storage floats with either operand transposed, for the backward GEMMs:
 * c[i][j] (row-major m x n) += sum over p in increasing order of A(i,p) * B(p,j), where A(i,p) is a[i*k+p] (a is
 * m x k) or, transposed, a[p*m+i] (a is k x m); B(p,j) is b[p*n+j] (b is k x n) or, transposed, b[j*k+p] (b is
 * n x k). `fmt` 0 = bf16, 1 = f16. */
void oracle_gemm_t16(size_t m, size_t n, size_t k, float* c, const uint16_t* a, const uint16_t* b, int trans_a,
                     int trans_b, int fmt) {
  for (size_t i = 0; i < m; ++i)
    for (size_t j = 0; j < n; ++j) {
      float acc = c[i * n + j];
      for (size_t p = 0; p < k; ++p) {
        const uint16_t ab = trans_a ? a[p * m + i] : a[i * k + p];
        const uint16_t bb = trans_b ? b[j * k + p] : b[p * n + j];
        const float x = fmt ? oracle_f16_to_f32(ab) : oracle_bf16_to_f32(ab);
        const float y = fmt ? oracle_f16_to_f32(bb) : oracle_bf16_to_f32(bb);
        volatile float prod = x * y;
        volatile float sum = acc + prod;
        acc = sum;
      }
      c[i * n + j] = acc;
    }
}

/* The fused epilogue: out[i][j] = bf16(act(f32(acc[i][j] + bias[j]))), act 0 = identity, 1 = ReLU. A null bias adds
 * nothing. ReLU keeps NaN (max(NaN, 0) is taken as NaN, as the device's comparison form does). */
void oracle_bias_act(size_t m, size_t n, const float* acc, const float* bias, int act, uint16_t* out) {
  for (size_t i = 0; i < m; ++i)
    for (size_t j = 0; j < n; ++j) {
      volatile float v = acc[i * n + j] + (bias ? bias[j] : 0.0f);
      float w = v;
      if (act == 1 && w < 0.0f) w = 0.0f;
      out[i * n + j] = oracle_f32_to_bf16(w);
    }
}

/* ---------------------------------------------------------------------------------------------------------------
 * The exact f32 sum, rounded once (cr::par::sum<float>, runtime/cairn_sum.hpp:311-331). Every finite f32 is an
 * integer multiple of 2^-149, at most (2^24 - 1) * 2^253 of them, so the exact total of up to 2^60 terms is a
 * signed integer below 2^338 in units of 2^-149: six 64-bit limbs in two's complement hold it.
 * ------------------------------------------------------------------------------------------------------------- */
#define LIMBS 6
typedef struct { uint64_t w[LIMBS]; } Wide;

static void wide_add_shifted(Wide* t, uint64_t mag, int shift, int negative) {
  /* t += (negative ? -1 : 1) * mag * 2^shift, mag < 2^25, shift <= 253 */
  uint64_t part[LIMBS] = {0};
  const int k = shift >> 6, s = shift & 63;
  part[k] = mag << s;
  if (s && k + 1 < LIMBS) part[k + 1] = mag >> (64 - s);
  if (negative) { /* two's complement of part */
    uint64_t carry = 1;
    for (int j = 0; j < LIMBS; ++j) {
      const uint64_t v = ~part[j] + carry;
      carry = (carry && v == 0) ? 1 : 0;
      part[j] = v;
    }
  }
  uint64_t carry = 0;
  for (int j = 0; j < LIMBS; ++j) {
    const uint64_t x = t->w[j], y = part[j];
    const uint64_t s1 = x + y;
    const uint64_t c1 = s1 < x;
    const uint64_t s2 = s1 + carry;
    const uint64_t c2 = s2 < s1;
    t->w[j] = s2;
    carry = c1 | c2;
  }
}

static int wide_bit(const Wide* t, int i) { return (int)((t->w[i >> 6] >> (i & 63)) & 1u); }

/* Round the magnitude held in t (non-negative, nonzero) to an f32 pattern without sign, ties to even. */
static uint32_t wide_round_f32(const Wide* t) {
  int lead = -1;
  for (int j = LIMBS - 1; j >= 0 && lead < 0; --j)
    if (t->w[j]) lead = 64 * j + 63 - __builtin_clzll(t->w[j]);
  int q = lead - 23 > 0 ? lead - 23 : 0; /* index of the result's last bit; 0 is 2^-149, the least subnormal */
  uint64_t mant = 0;
  for (int i = lead; i >= q; --i) mant = (mant << 1) | (uint64_t)wide_bit(t, i);
  if (q > 0) {
    const int guard = wide_bit(t, q - 1);
    int sticky = 0;
    for (int i = q - 2; i >= 0 && !sticky; --i) sticky = wide_bit(t, i);
    if (guard && (sticky || (mant & 1u))) ++mant;
    if (mant >> 24) { mant >>= 1; ++q; }
  }
  if (mant < (1u << 23)) return (uint32_t)mant; /* subnormal (q == 0) */
  const int biased = q + 1;                       /* value = mant * 2^(q-149) = 1.f * 2^(q-126) */
  if (biased >= 255) return 0x7f800000u;
  return ((uint32_t)biased << 23) | ((uint32_t)mant & 0x7fffffu);
}

float oracle_sum_f32(size_t n, const float* x) {
  Wide t;
  memset(&t, 0, sizeof t);
  int nan = 0, pinf = 0, ninf = 0, other = 0;
  for (size_t i = 0; i < n; ++i) {
    const uint32_t u = bits32(x[i]);
    if (u != 0x80000000u) other = 1;
    const uint32_t e = (u >> 23) & 0xffu, f = u & 0x7fffffu;
    if (e == 0xffu) {
      if (f) nan = 1;
      else if (u >> 31) ninf = 1;
      else pinf = 1;
      continue;
    }
    const uint64_t mag = e ? (f | 0x800000u) : f;
    if (!mag) continue;
    const int shift = e ? (int)e - 1 : 0; /* value = mag * 2^(shift - 149) */
    wide_add_shifted(&t, mag, shift, (int)(u >> 31));
  }
  if (nan || (pinf && ninf)) return from_bits32(0x7fc00000u);
  if (pinf) return INFINITY;
  if (ninf) return -INFINITY;
  const int negative = (int)(t.w[LIMBS - 1] >> 63);
  int zero = 1;
  for (int j = 0; j < LIMBS; ++j) zero &= t.w[j] == 0;
  if (zero) return from_bits32((n && !other) ? 0x80000000u : 0u);
  if (negative) { /* magnitude */
    uint64_t carry = 1;
    for (int j = 0; j < LIMBS; ++j) {
      const uint64_t v = ~t.w[j] + carry;
      carry = (carry && v == 0) ? 1 : 0;
      t.w[j] = v;
    }
  }
  return from_bits32(wide_round_f32(&t) | ((uint32_t)negative << 31));
}

/* cr::Sum<u64> folded in index order: the wrapped total, and whether any partial sum wrapped. */
uint64_t oracle_sum_u64(size_t n, const uint64_t* x, int* overflow) {
  uint64_t s = 0;
  int over = 0;
  for (size_t i = 0; i < n; ++i) {
    const uint64_t t = s + x[i];
    over |= t < s;
    s = t;
  }
  *overflow = over;
  return s;
}

/* out[i] = f32(f32(a * x[i]) + y[i]) */
uint32_t oracle_scan_u32(size_t n, uint32_t* out, const uint32_t* x) {
  uint32_t acc = 0;
  for (size_t i = 0; i < n; ++i) out[i] = acc = acc + x[i];
  return acc;
}

int32_t oracle_runmax_i32(size_t n, int32_t* out, const int32_t* x) {
  int32_t acc = INT32_MIN;
  for (size_t i = 0; i < n; ++i) {
    out[i] = acc;
    if (x[i] > acc) acc = x[i];
  }
  return acc;
}

void oracle_saxpy_f32(size_t n, float* out, const float* x, const float* y, float a) {
  for (size_t i = 0; i < n; ++i) {
    volatile float p = a * x[i];
    volatile float s = p + y[i];
    out[i] = s;
  }
}

/* ---------------------------------------------------------------------------------------------------------------
 * The 2-layer MLP step of BASELINE config 3 (forward, MSE loss, backward), with the bf16 storage of the device path
 * (H, dY, dH in bf16; Y and the weight and input gradients in f32). The backward of each dense layer is the loop
 * derive grad writes for `out[i][j] = sum_p x[i][p] * w[p][j]` (compiler/derive/gradients.py:1-11; the expanded
 * form re-runs the forward, then for each output e = (i, j) in order adds d_out[e] * w[p][j] into d_x[i][p] and
 * x[i][p] * d_out[e] into d_w[p][j] for p in order): d_x = d_out * w^T and d_w = x^T * d_out, every sum sequential in
 * f32. ReLU's backward passes d where the forward's output is positive. Loss = sum (y - t)^2 / n in f64, rounded;
 * dY = bf16((y - t) * (2 / n)).
 * ------------------------------------------------------------------------------------------------------------- */
void oracle_mlp_step(size_t B, size_t D, size_t Hd, size_t O, const uint16_t* X, const uint16_t* W1,
                     const uint16_t* W2, const float* T, uint16_t* H, float* Y, uint16_t* dY, float* loss,
                     float* dW2, uint16_t* dH, float* dW1, float* dX) {
  for (size_t b = 0; b < B; ++b)
    for (size_t h = 0; h < Hd; ++h) {
      float s = 0.0f;
      for (size_t d = 0; d < D; ++d) {
        volatile float prod = oracle_bf16_to_f32(X[b * D + d]) * oracle_bf16_to_f32(W1[d * Hd + h]);
        volatile float sum = s + prod;
        s = sum;
      }
      H[b * Hd + h] = oracle_f32_to_bf16(s < 0.0f ? 0.0f : s);
    }
  for (size_t b = 0; b < B; ++b)
    for (size_t o = 0; o < O; ++o) {
      float s = 0.0f;
      for (size_t h = 0; h < Hd; ++h) {
        volatile float prod = oracle_bf16_to_f32(H[b * Hd + h]) * oracle_bf16_to_f32(W2[h * O + o]);
        volatile float sum = s + prod;
        s = sum;
      }
      Y[b * O + o] = s;
    }
  const size_t n = B * O;
  const float scale = 2.0f / (float)n;
  double acc = 0.0;
  for (size_t i = 0; i < n; ++i) {
    volatile float d = Y[i] - T[i];
    volatile float g = d * scale;
    dY[i] = oracle_f32_to_bf16(g);
    acc += (double)d * (double)d;
  }
  *loss = (float)(acc / (double)n);
  /* layer 2's backward: dH_acc = dY * W2^T, dW2 = H^T * dY (sequential sums in increasing index) */
  for (size_t h = 0; h < Hd; ++h)
    for (size_t o = 0; o < O; ++o) {
      float s = 0.0f;
      for (size_t b = 0; b < B; ++b) {
        volatile float prod = oracle_bf16_to_f32(H[b * Hd + h]) * oracle_bf16_to_f32(dY[b * O + o]);
        volatile float sum = s + prod;
        s = sum;
      }
      dW2[h * O + o] = s;
    }
  for (size_t b = 0; b < B; ++b)
    for (size_t h = 0; h < Hd; ++h) {
      float s = 0.0f;
      for (size_t o = 0; o < O; ++o) {
        volatile float prod = oracle_bf16_to_f32(dY[b * O + o]) * oracle_bf16_to_f32(W2[h * O + o]);
        volatile float sum = s + prod;
        s = sum;
      }
      dH[b * Hd + h] = oracle_bf16_to_f32(H[b * Hd + h]) > 0.0f ? oracle_f32_to_bf16(s) : 0;
    }
  /* layer 1's backward: dX = dH * W1^T, dW1 = X^T * dH */
  for (size_t d = 0; d < D; ++d)
    for (size_t h = 0; h < Hd; ++h) {
      float s = 0.0f;
      for (size_t b = 0; b < B; ++b) {
        volatile float prod = oracle_bf16_to_f32(X[b * D + d]) * oracle_bf16_to_f32(dH[b * Hd + h]);
        volatile float sum = s + prod;
        s = sum;
      }
      dW1[d * Hd + h] = s;
    }
  for (size_t b = 0; b < B; ++b)
    for (size_t d = 0; d < D; ++d) {
      float s = 0.0f;
      for (size_t h = 0; h < Hd; ++h) {
        volatile float prod = oracle_bf16_to_f32(dH[b * Hd + h]) * oracle_bf16_to_f32(W1[d * Hd + h]);
        volatile float sum = s + prod;
        s = sum;
      }
      dX[b * D + d] = s;
    }
}

/*
 * awq_oracle.c — CPU restatement of the reference's AWQ arithmetic.
 *
 * TEST INFRASTRUCTURE ONLY (see awq_oracle.h). Built with -ffp-contract=off so
 * that every multiply and add rounds separately, as the restated formulas say.
 */
#include "awq_oracle.h"

#include <math.h>
#include <string.h>

#ifdef _OPENMP
#include <omp.h>
#endif

/* Logical column -> packed nibble, AWQ order: awq_kernel_gemm.rs:809
 * (AWQ_REVERSE_ORDER) and the shifts of unpack_u32_to_i4_0_4/_4_8 (:10-30). */
static const int kAwqReverseOrder[8] = {0, 4, 1, 5, 2, 6, 3, 7};

uint32_t awqo_nibble(uint32_t packed, int c, int order) {
  int lane = order == 0 ? kAwqReverseOrder[c & 7] : (c & 7); /* awq_kernel.rs:14 */
  return (packed >> (4 * lane)) & 0xFu;
}

/* ---------------------------------------------------------------- rounding */

/* Round a double to a binary format with `p` significand bits (incl. the
 * implicit one), minimum normal exponent emin, maximum finite value maxv.
 * Round to nearest, ties to even (nearbyint in the default mode). */
static double round_to_format(double a, int p, int emin, double maxv) {
  if (isnan(a) || isinf(a) || a == 0.0) return a;
  double s = a < 0 ? -1.0 : 1.0;
  double m = fabs(a);
  int e;
  frexp(m, &e); /* m = f * 2^e, f in [0.5, 1) -> exponent of leading bit e-1 */
  int lead = e - 1;
  if (lead < emin) lead = emin; /* subnormal: fixed quantum */
  double quantum = ldexp(1.0, lead - (p - 1));
  double r = nearbyint(m / quantum) * quantum;
  /* overflow: values at or above max + half-ulp round to infinity */
  if (r > maxv) return s * INFINITY;
  return s * r;
}

static double round_f16(double a) { return round_to_format(a, 11, -14, 65504.0); }
static double round_bf16(double a) {
  return round_to_format(a, 8, -126, 3.3895313892515355e38);
}
static double round_f32(double a) { return (double)(float)a; }

static double round_dt(double a, int dtype) {
  switch (dtype) {
    case 1: return round_f16(a);
    case 2: return round_bf16(a);
    default: return round_f32(a);
  }
}

float awqo_f16_to_f32(uint16_t h) {
  uint32_t sign = (uint32_t)(h >> 15) & 1u;
  uint32_t exp = (uint32_t)(h >> 10) & 0x1Fu;
  uint32_t man = (uint32_t)h & 0x3FFu;
  double v;
  if (exp == 0) {
    v = ldexp((double)man, -24);
  } else if (exp == 31) {
    v = man ? NAN : INFINITY;
  } else {
    v = ldexp((double)(man | 0x400u), (int)exp - 25);
  }
  return (float)(sign ? -v : v);
}

static uint16_t f16_bits_of_exact(double v) {
  /* v is exactly representable in binary16 (or inf/nan) */
  uint16_t sign = signbit(v) ? 0x8000u : 0u;
  double m = fabs(v);
  if (isnan(v)) return (uint16_t)(sign | 0x7E00u);
  if (isinf(v)) return (uint16_t)(sign | 0x7C00u);
  if (m == 0.0) return sign;
  if (m < ldexp(1.0, -14)) { /* subnormal */
    uint32_t man = (uint32_t)ldexp(m, 24);
    return (uint16_t)(sign | man);
  }
  int e;
  double f = frexp(m, &e); /* m = f*2^e, f in [0.5,1) */
  uint32_t exp = (uint32_t)(e - 1 + 15);
  uint32_t man = (uint32_t)(ldexp(f, 11)) & 0x3FFu;
  return (uint16_t)(sign | (exp << 10) | man);
}

uint16_t awqo_f64_to_f16(double d) { return f16_bits_of_exact(round_f16(d)); }
uint16_t awqo_f32_to_f16(float f) { return awqo_f64_to_f16((double)f); }

float awqo_bf16_to_f32(uint16_t h) {
  uint32_t u = (uint32_t)h << 16;
  float f;
  memcpy(&f, &u, 4);
  return f;
}

uint16_t awqo_f64_to_bf16(double d) {
  if (isnan(d)) return 0x7FC0u;
  float f = (float)round_bf16(d); /* exact in f32 */
  uint32_t u;
  memcpy(&u, &f, 4);
  return (uint16_t)(u >> 16);
}

uint16_t awqo_f32_to_bf16(float f) { return awqo_f64_to_bf16((double)f); }

double awqo_load(const void* p, size_t i, int dtype) {
  switch (dtype) {
    case 1: return (double)awqo_f16_to_f32(((const uint16_t*)p)[i]);
    case 2: return (double)awqo_bf16_to_f32(((const uint16_t*)p)[i]);
    default: return (double)((const float*)p)[i];
  }
}

static void store_dt(void* p, size_t i, double v, int dtype) {
  switch (dtype) {
    case 1: ((uint16_t*)p)[i] = awqo_f64_to_f16(v); break;
    case 2: ((uint16_t*)p)[i] = awqo_f64_to_bf16(v); break;
    default: ((float*)p)[i] = (float)v; break;
  }
}

int awqo_max_threads(void) {
#ifdef _OPENMP
  return omp_get_max_threads();
#else
  return 1;
#endif
}

/* -------------------------------------------------------------- dequantize */

/* dequantize_awq_symmetric (awq_kernel.rs:38-60): one rounding of the product
 * (the difference of two small integers is exact in every F). */
static double deq_value(const uint32_t* qw, const uint32_t* qz, const void* sc,
                        size_t k, size_t n, size_t N, size_t g, int dtype,
                        int order) {
  size_t npk = N / 8;
  size_t grp = k / g;
  double q = (double)awqo_nibble(qw[k * npk + n / 8], (int)(n % 8), order);
  double z = (double)awqo_nibble(qz[grp * npk + n / 8], (int)(n % 8), order);
  double s = awqo_load(sc, grp * N + n, dtype);
  return round_dt((q - z) * s, dtype);
}

void awqo_dequant(const uint32_t* qw, const uint32_t* qz, const void* sc,
                  void* out, size_t K, size_t N, size_t g, int dtype, int order) {
  long long kk;
#pragma omp parallel for schedule(static)
  for (kk = 0; kk < (long long)K; ++kk) {
    for (size_t n = 0; n < N; ++n) {
      double v = deq_value(qw, qz, sc, (size_t)kk, n, N, g, dtype, order);
      store_dt(out, (size_t)kk * N + n, v, dtype);
    }
  }
}

/* -------------------------------------------------------------------- GEMM */

/* Reference numerics, f32: float operations, contraction disabled. Per
 * output: w = (q - z) * s rounded once, acc = acc + x * w (product and sum
 * each rounded), k ascending from acc = 0 -- the reference's F = f32 path.
 * Laid out for the host's vector units: one task owns 128 columns (16 packed
 * words) of one row; the 8 columns of a word are one 8-lane vector, unpacked
 * with the nibble order's shift table. Lanes are independent outputs, so the
 * operations and their order per output are those of a plain scalar loop. */
static const int kShiftAwq[8] = {0, 16, 4, 20, 8, 24, 12, 28};
static const int kShiftNat[8] = {0, 4, 8, 12, 16, 20, 24, 28};

typedef uint32_t v8u __attribute__((vector_size(32)));
typedef float v8f __attribute__((vector_size(32)));

static inline void f32_block(const float* x, const uint32_t* qw,
                             const uint32_t* qz, const float* sc,
                             const float* bias, float* out, size_t m, size_t K,
                             size_t N, size_t g, size_t j0, size_t nw,
                             const int* sh) {
  const size_t npk = N / 8;
  const v8u shv = {(uint32_t)sh[0], (uint32_t)sh[1], (uint32_t)sh[2], (uint32_t)sh[3],
                   (uint32_t)sh[4], (uint32_t)sh[5], (uint32_t)sh[6], (uint32_t)sh[7]};
  const v8u mask = {15u, 15u, 15u, 15u, 15u, 15u, 15u, 15u};
  v8f acc[16];
  for (size_t j = 0; j < 16; ++j) acc[j] = (v8f){0, 0, 0, 0, 0, 0, 0, 0};
  for (size_t k0 = 0; k0 < K; k0 += g) {
    const size_t grp = k0 / g;
    const size_t k1 = k0 + g < K ? k0 + g : K;
    v8f zf[16], sf[16];
    for (size_t j = 0; j < nw; ++j) {
      const uint32_t b = qz[grp * npk + j0 + j];
      const v8u bz = {b, b, b, b, b, b, b, b};
      zf[j] = __builtin_convertvector((bz >> shv) & mask, v8f);
      memcpy(&sf[j], sc + grp * N + 8 * (j0 + j), sizeof(v8f));
    }
    for (size_t k = k0; k < k1; ++k) {
      const float xs = x[m * K + k];
      const v8f xv = {xs, xs, xs, xs, xs, xs, xs, xs};
      const uint32_t* wq = qw + k * npk + j0;
      for (size_t j = 0; j < nw; ++j) {
        const uint32_t a = wq[j];
        const v8u av = {a, a, a, a, a, a, a, a};
        const v8f q = __builtin_convertvector((av >> shv) & mask, v8f);
        const v8f w = (q - zf[j]) * sf[j];   /* (q - z) exact, one rounding of * s */
        acc[j] = acc[j] + xv * w;            /* product and sum rounded separately */
      }
    }
  }
  for (size_t j = 0; j < nw; ++j) {
    float v[8];
    memcpy(v, &acc[j], sizeof(v));
    for (int c = 0; c < 8; ++c) {
      float r = v[c];
      if (bias) r = r + bias[8 * (j0 + j) + (size_t)c];
      out[m * N + 8 * (j0 + j) + (size_t)c] = r;
    }
  }
}

static void gemm_ref_f32(const float* x, const uint32_t* qw, const uint32_t* qz,
                         const float* sc, const float* bias, float* out,
                         size_t M, size_t K, size_t N, size_t g, int order,
                         int nthreads) {
  const size_t npk = N / 8;
  const size_t WB = 16; /* packed words (128 columns) per task */
  const long long nblocks = (long long)((npk + WB - 1) / WB);
  const int* sh = order == 0 ? kShiftAwq : kShiftNat;
  long long task;
#pragma omp parallel for schedule(dynamic, 1) num_threads(nthreads > 0 ? nthreads : awqo_max_threads())
  for (task = 0; task < nblocks * (long long)M; ++task) {
    const size_t m = (size_t)(task / nblocks);
    const size_t j0 = (size_t)(task % nblocks) * WB;
    const size_t nw = j0 + WB < npk ? WB : npk - j0;
    if (order == 0) {
      f32_block(x, qw, qz, sc, bias, out, m, K, N, g, j0, nw, kShiftAwq);
    } else {
      f32_block(x, qw, qz, sc, bias, out, m, K, N, g, j0, nw, kShiftNat);
    }
  }
  (void)sh;
}

/* Reference numerics in a 16-bit F: each operation computed exactly in
 * double, then rounded to F once. */
static void gemm_ref_16(const uint16_t* x, const uint32_t* qw,
                        const uint32_t* qz, const uint16_t* sc,
                        const uint16_t* bias, uint16_t* out, size_t M, size_t K,
                        size_t N, size_t g, int dtype, int order, int nthreads) {
  long long task;
#pragma omp parallel for schedule(dynamic, 16) num_threads(nthreads > 0 ? nthreads : awqo_max_threads())
  for (task = 0; task < (long long)(M * N); ++task) {
    size_t m = (size_t)task / N;
    size_t n = (size_t)task % N;
    double acc = 0.0;
    for (size_t k = 0; k < K; ++k) {
      double w = deq_value(qw, qz, sc, k, n, N, g, dtype, order);
      double xv = awqo_load(x, m * K + k, dtype);
      double prod = round_dt(xv * w, dtype);
      acc = round_dt(acc + prod, dtype);
    }
    if (bias) acc = round_dt(acc + awqo_load(bias, n, dtype), dtype);
    store_dt(out, m * N + n, acc, dtype);
  }
}

void awqo_gemm_ref(const void* x, const uint32_t* qw, const uint32_t* qz,
                   const void* sc, const void* bias, void* out, size_t M,
                   size_t K, size_t N, size_t g, int dtype, int order,
                   int nthreads) {
  if (dtype == 0) {
    gemm_ref_f32((const float*)x, qw, qz, (const float*)sc, (const float*)bias,
                 (float*)out, M, K, N, g, order, nthreads);
  } else {
    gemm_ref_16((const uint16_t*)x, qw, qz, (const uint16_t*)sc,
                (const uint16_t*)bias, (uint16_t*)out, M, K, N, g, dtype, order,
                nthreads);
  }
}

void awqo_gemm_f64(const void* x, const uint32_t* qw, const uint32_t* qz,
                   const void* sc, const void* bias, double* out, size_t M,
                   size_t K, size_t N, size_t g, int dtype, int order,
                   int deq_round, int nthreads) {
  size_t npk = N / 8;
  const size_t NB = 256;
  long long nblocks = (long long)((N + NB - 1) / NB);
  long long task;
#pragma omp parallel for schedule(dynamic, 1) num_threads(nthreads > 0 ? nthreads : awqo_max_threads())
  for (task = 0; task < nblocks * (long long)M; ++task) {
    size_t m = (size_t)(task / nblocks);
    size_t n0 = (size_t)(task % nblocks) * NB;
    size_t n1 = n0 + NB < N ? n0 + NB : N;
    double acc[256];
    for (size_t n = n0; n < n1; ++n) acc[n - n0] = 0.0;
    for (size_t k = 0; k < K; ++k) {
      size_t grp = k / g;
      double xv = awqo_load(x, m * K + k, dtype);
      for (size_t n = n0; n < n1; ++n) {
        double w;
        if (deq_round) {
          w = deq_value(qw, qz, sc, k, n, N, g, dtype, order);
        } else {
          double q = (double)awqo_nibble(qw[k * npk + n / 8], (int)(n % 8), order);
          double z = (double)awqo_nibble(qz[grp * npk + n / 8], (int)(n % 8), order);
          w = (q - z) * awqo_load(sc, grp * N + n, dtype);
        }
        acc[n - n0] += xv * w;
      }
    }
    for (size_t n = n0; n < n1; ++n) {
      double v = acc[n - n0];
      if (bias) v += awqo_load(bias, n, dtype);
      out[m * N + n] = v;
    }
  }
}

/*
 * awq_oracle.h — CPU restatement of the reference's AWQ arithmetic.
 *
 * TEST INFRASTRUCTURE ONLY. Only tests/, __graft_entry__.smoke() and the
 * cpu_baseline leg of bench.py may load this library, and only as the checker
 * or the timed CPU baseline. The product (libcube_awq.so and the
 * cube_awq_b200 package) never calls it.
 *
 * Restated from joshuawm/cube-awq (paths relative to that project):
 *   - nibble unpack, AWQ order:     src/kernel/awq_kernel_gemm.rs:10-30, :809-811
 *   - nibble unpack, natural order: src/kernel/awq_kernel.rs:9-19
 *   - dequantize (q - z) * s in F:  src/kernel/awq_kernel.rs:38-60
 *   - fused GEMM numerics in F:     src/kernel/awq_kernel_gemm.rs:346-399, :555-605
 *     (per output: acc starts at 0, k strictly ascending, acc += x * deq)
 *   - golden CPU references:        awq_kernel_gemm.rs:793-829,
 *                                   src/modules/awq_gemm.rs:344-383,
 *                                   src/modules/awq_dequantize.rs:169-180
 *   - bias added after the sum:     src/modules/awq_gemm.rs:225-228
 *
 * dtype codes: 0 = f32, 1 = f16, 2 = bf16 (same as cawq_dtype).
 * order codes: 0 = AWQ, 1 = natural (same as cawq_order).
 */
#ifndef AWQ_ORACLE_H_
#define AWQ_ORACLE_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Nibble of logical column c (0..7) of a packed word. */
uint32_t awqo_nibble(uint32_t packed, int c, int order);

/* IEEE binary16 / bfloat16 conversions (round to nearest even). */
float awqo_f16_to_f32(uint16_t h);
uint16_t awqo_f32_to_f16(float f);
uint16_t awqo_f64_to_f16(double d);
float awqo_bf16_to_f32(uint16_t h);
uint16_t awqo_f32_to_bf16(float f);
uint16_t awqo_f64_to_bf16(double d);

/* Element `i` of a buffer of `dtype` as a double (exact). */
double awqo_load(const void* p, size_t i, int dtype);

/* out[k, n] = (q - z) * s rounded once to `dtype` (awq_kernel.rs:59). */
void awqo_dequant(const uint32_t* qw, const uint32_t* qz, const void* sc,
                  void* out, size_t K, size_t N, size_t g, int dtype, int order);

/*
 * The reference's own numerics: every operation in F (dtype), one rounding
 * per operation, no fused multiply-add:
 *   w   = round_F(round_F(q - z) * s)
 *   acc = round_F(acc + round_F(x * w))   for k = 0, 1, ..., K-1
 *   out = round_F(acc + bias)             (when bias != NULL)
 * out has `dtype`. Threads: OpenMP over columns (0 = all).
 */
void awqo_gemm_ref(const void* x, const uint32_t* qw, const uint32_t* qz,
                   const void* sc, const void* bias, void* out, size_t M,
                   size_t K, size_t N, size_t g, int dtype, int order,
                   int nthreads);

/*
 * Exact-accumulation oracle: out (double) = sum_k x * w (+ bias) in double.
 * deq_round = 1: w rounded to F as the reference dequantizes it;
 * deq_round = 0: w = (q - z) * s exactly.
 */
void awqo_gemm_f64(const void* x, const uint32_t* qw, const uint32_t* qz,
                   const void* sc, const void* bias, double* out, size_t M,
                   size_t K, size_t N, size_t g, int dtype, int order,
                   int deq_round, int nthreads);

/* Number of OpenMP threads the library would use for nthreads = 0. */
int awqo_max_threads(void);

#ifdef __cplusplus
}
#endif

#endif /* AWQ_ORACLE_H_ */

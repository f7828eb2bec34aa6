// cawq_generic.cuh — CUDA-core fused AWQ GEMM for any shape the reference's
// rules accept (sm_100a). It is the planner's choice when neither the decode
// nor the tensor-core kernel covers a problem (a group size that is not a
// multiple of 16, unaligned buffers, ...). It follows gemm_awq
// (src/kernel/awq_kernel_gemm.rs:181-439) closely: each weight is dequantized
// in F, w = round_F((q - z) * s), and each output accumulates x * w over k in
// ascending order, here in fp32.
#pragma once

#include "cawq_common.cuh"

namespace cawq {

constexpr int kGenericCols = 128;  // threads (= columns) per CTA
constexpr int kGenericRows = 8;    // rows of x per CTA

template <int DT, int ODT, int ORDER>
__global__ void __launch_bounds__(kGenericCols)
    generic_gemm_kernel(const typename DType<DT>::T* __restrict__ x,
                        const uint32_t* __restrict__ qw, const uint32_t* __restrict__ qz,
                        const typename DType<DT>::T* __restrict__ sc,
                        const typename DType<DT>::T* __restrict__ bias,
                        const OutMap<typename DType<ODT>::T> om, uint32_t rows, uint32_t k,
                        uint32_t n, uint32_t g) {
  const uint32_t col = blockIdx.x * kGenericCols + threadIdx.x;
  const uint32_t r0 = blockIdx.y * kGenericRows;
  if (col >= n) return;
  const uint32_t npk = n / 8;
  const uint32_t p = col / 8;
  const int sh = 4 * nibble_of_col(static_cast<int>(col % 8), ORDER);
  float acc[kGenericRows];
#pragma unroll
  for (int r = 0; r < kGenericRows; ++r) acc[r] = 0.f;
  const uint32_t nr = min(static_cast<uint32_t>(kGenericRows), rows - r0);

  for (uint32_t kk = 0; kk < k;) {
    const uint32_t grp = kk / g;
    const uint32_t kend = min(k, (grp + 1) * g);
    const float s = DType<DT>::to_f32(sc[(size_t)grp * n + col]);
    const float z = static_cast<float>((__ldg(qz + (size_t)grp * npk + p) >> sh) & 15u);
    for (; kk < kend; ++kk) {
      const float q = static_cast<float>((__ldg(qw + (size_t)kk * npk + p) >> sh) & 15u);
      // dequantized weight in F, as the reference computes it
      const float w = DType<DT>::to_f32(DType<DT>::from_f32(__fmul_rn(q - z, s)));
#pragma unroll
      for (int r = 0; r < kGenericRows; ++r) {
        if (static_cast<uint32_t>(r) < nr) {
          const float xv = DType<DT>::to_f32(x[(size_t)(r0 + r) * k + kk]);
          acc[r] = fmaf(xv, w, acc[r]);
        }
      }
    }
  }
  const float b = bias ? DType<DT>::to_f32(bias[col]) : 0.f;
#pragma unroll
  for (int r = 0; r < kGenericRows; ++r) {
    if (static_cast<uint32_t>(r) < nr) {
      *om.at(r0 + r, col) = DType<ODT>::from_f32(acc[r] + b);
    }
  }
}

bool generic_supports(const GemmProblem& p) {
  return p.rows > 0 && p.k > 0 && p.n % 8 == 0 && p.g > 0 && p.k % p.g == 0 &&
         p.rows <= 65535ull * kGenericRows && p.k < (1ull << 31) && p.n < (1ull << 31) &&
         p.ld_out < (1ull << 31);
}

template <int DT, int ODT, int ORDER>
static cudaError_t launch_generic_t(const GemmProblem& p) {
  using T = typename DType<DT>::T;
  using OT = typename DType<ODT>::T;
  dim3 grid(static_cast<uint32_t>((p.n + kGenericCols - 1) / kGenericCols),
            static_cast<uint32_t>((p.rows + kGenericRows - 1) / kGenericRows));
  generic_gemm_kernel<DT, ODT, ORDER><<<grid, kGenericCols, 0, p.stream>>>(
      static_cast<const T*>(p.x), p.qw, p.qz, static_cast<const T*>(p.sc),
      static_cast<const T*>(p.bias), out_map<OT>(p), static_cast<uint32_t>(p.rows),
      static_cast<uint32_t>(p.k), static_cast<uint32_t>(p.n), static_cast<uint32_t>(p.g));
  return cudaGetLastError();
}

template <int DT, int ODT>
static cudaError_t launch_generic_o(const GemmProblem& p) {
  return p.order == kOrderNatural ? launch_generic_t<DT, ODT, kOrderNatural>(p)
                                  : launch_generic_t<DT, ODT, kOrderAwq>(p);
}

cudaError_t launch_generic(const GemmProblem& p) {
  if (p.dtype == kF32) return launch_generic_o<kF32, kF32>(p);
  if (p.dtype == kF16) {
    return p.out_dtype == kF32 ? launch_generic_o<kF16, kF32>(p) : launch_generic_o<kF16, kF16>(p);
  }
  return p.out_dtype == kF32 ? launch_generic_o<kBF16, kF32>(p) : launch_generic_o<kBF16, kBF16>(p);
}

}  // namespace cawq

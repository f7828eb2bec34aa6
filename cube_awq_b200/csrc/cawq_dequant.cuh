// cawq_dequant.cuh — standalone AWQ dequantize kernel (sm_100a).
//
// out[k, n] = (q[k, n] - z[k / g, n]) * s[k / g, n], rounded once to F.
// Replaces dequantize_awq_symmetric (src/kernel/awq_kernel.rs:23-61) and its
// launcher dequantize_native (:63-111). The reference maps one thread to four
// packed words; here one thread owns one packed word (8 outputs) per visit so a
// warp's stores cover one contiguous span, and a grid-stride loop over rows
// keeps every SM busy for any K.
//
// Bit exactness: q - z is an exact small integer in every F; its product with
// s is exact in f32 when s is f16/bf16 (at most 4 + 11 significant bits), so
// one conversion to F rounds once, like the reference's multiply in F.
#pragma once

#include "cawq_common.cuh"

namespace cawq {

// Rows handled per loop pass: their packed words are loaded before any is
// used, so a thread keeps kDqRows loads in flight.
constexpr int kDqRows = 4;

template <int DT, int ORDER, bool VEC>
__global__ void __launch_bounds__(256)
    dequant_kernel(const uint32_t* __restrict__ qw, const uint32_t* __restrict__ qz,
                   const typename DType<DT>::T* __restrict__ sc,
                   typename DType<DT>::T* __restrict__ out, uint32_t k, uint32_t npk,
                   uint32_t g) {
  using T = typename DType<DT>::T;
  const uint32_t n = npk * 8;
  const uint32_t ystep = gridDim.y;
  for (uint32_t row0 = blockIdx.y; row0 < k; row0 += kDqRows * ystep) {
    for (uint32_t p = blockIdx.x * blockDim.x + threadIdx.x; p < npk; p += gridDim.x * blockDim.x) {
      uint32_t qv[kDqRows];
#pragma unroll
      for (int i = 0; i < kDqRows; ++i) {
        const uint32_t row = row0 + i * ystep;
        qv[i] = row < k ? ldg_nc_u32(qw + (size_t)row * npk + p) : 0u;
      }
#pragma unroll
      for (int i = 0; i < kDqRows; ++i) {
        const uint32_t row = row0 + i * ystep;
        if (row >= k) break;
        const uint32_t grp = row / g;
        const uint32_t q = qv[i];
        const uint32_t z = __ldg(qz + (size_t)grp * npk + p);
        const T* srow = sc + (size_t)grp * n + (size_t)p * 8;
        float s[8];
        if constexpr (VEC && DT == kF32) {
          const float4 s0 = __ldg(reinterpret_cast<const float4*>(srow));
          const float4 s1 = __ldg(reinterpret_cast<const float4*>(srow) + 1);
          s[0] = s0.x; s[1] = s0.y; s[2] = s0.z; s[3] = s0.w;
          s[4] = s1.x; s[5] = s1.y; s[6] = s1.z; s[7] = s1.w;
        } else if constexpr (VEC) {
          const uint4 raw = __ldg(reinterpret_cast<const uint4*>(srow));
          const T* h = reinterpret_cast<const T*>(&raw);
#pragma unroll
          for (int c = 0; c < 8; ++c) s[c] = DType<DT>::to_f32(h[c]);
        } else {
#pragma unroll
          for (int c = 0; c < 8; ++c) s[c] = DType<DT>::to_f32(srow[c]);
        }
        float v[8];
#pragma unroll
        for (int c = 0; c < 8; ++c) {
          const int sh = 4 * nibble_of_col(c, ORDER);
          const int d = static_cast<int>((q >> sh) & 15u) - static_cast<int>((z >> sh) & 15u);
          v[c] = __fmul_rn(static_cast<float>(d), s[c]);
        }
        T* orow = out + (size_t)row * n + (size_t)p * 8;
        if constexpr (VEC && DT == kF32) {
          uint4 a, b;
          a.x = __float_as_uint(v[0]); a.y = __float_as_uint(v[1]);
          a.z = __float_as_uint(v[2]); a.w = __float_as_uint(v[3]);
          b.x = __float_as_uint(v[4]); b.y = __float_as_uint(v[5]);
          b.z = __float_as_uint(v[6]); b.w = __float_as_uint(v[7]);
          stg_cs_v4(orow, a);
          stg_cs_v4(orow + 4, b);
        } else if constexpr (VEC) {
          uint4 a;
          T* h = reinterpret_cast<T*>(&a);
#pragma unroll
          for (int c = 0; c < 8; ++c) h[c] = DType<DT>::from_f32(v[c]);
          stg_cs_v4(orow, a);
        } else {
#pragma unroll
          for (int c = 0; c < 8; ++c) orow[c] = DType<DT>::from_f32(v[c]);
        }
      }
    }
  }
}

template <int DT, int ORDER, bool VEC>
static cudaError_t launch_dequant_t(const uint32_t* qw, const uint32_t* qz, const void* sc,
                                    void* out, size_t k, size_t n, size_t g, cudaStream_t stream,
                                    int sm_count) {
  using T = typename DType<DT>::T;
  const uint32_t npk = static_cast<uint32_t>(n / 8);
  dim3 block(256);
  const uint32_t gx = (npk + 255) / 256;
  // 8 resident CTAs of 256 threads per SM (a full SM) cover the grid.
  uint32_t gy = static_cast<uint32_t>(sm_count) * 8u / gx;
  if (gy < 1) gy = 1;
  if (gy > k) gy = static_cast<uint32_t>(k);
  if (gy > 65535) gy = 65535;
  dim3 grid(gx, gy);
  dequant_kernel<DT, ORDER, VEC><<<grid, block, 0, stream>>>(
      qw, qz, static_cast<const T*>(sc), static_cast<T*>(out), static_cast<uint32_t>(k), npk,
      static_cast<uint32_t>(g));
  return cudaGetLastError();
}

cudaError_t launch_dequant(const uint32_t* qw, const uint32_t* qz, const void* sc, void* out,
                           size_t k, size_t n, size_t g, int dtype, int order,
                           cudaStream_t stream, int sm_count) {
  // 16-byte vectors need 16-byte aligned scale rows and output rows.
  const bool vec = (reinterpret_cast<uintptr_t>(sc) % 16 == 0) &&
                   (reinterpret_cast<uintptr_t>(out) % 16 == 0);
#define CAWQ_DQ(DT, OR)                                                                        \
  return vec ? launch_dequant_t<DT, OR, true>(qw, qz, sc, out, k, n, g, stream, sm_count)    \
             : launch_dequant_t<DT, OR, false>(qw, qz, sc, out, k, n, g, stream, sm_count)
  if (order == kOrderNatural) {
    if (dtype == kF32) { CAWQ_DQ(kF32, kOrderNatural); }
    if (dtype == kF16) { CAWQ_DQ(kF16, kOrderNatural); }
    CAWQ_DQ(kBF16, kOrderNatural);
  }
  if (dtype == kF32) { CAWQ_DQ(kF32, kOrderAwq); }
  if (dtype == kF16) { CAWQ_DQ(kF16, kOrderAwq); }
  CAWQ_DQ(kBF16, kOrderAwq);
#undef CAWQ_DQ
}

}  // namespace cawq

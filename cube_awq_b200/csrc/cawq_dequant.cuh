// cawq_dequant.cuh — standalone AWQ dequantize kernel (sm_100a).
//
// out[k, n] = (q[k, n] - z[k / g, n]) * s[k / g, n], rounded once to F.
// Replaces dequantize_awq_symmetric (src/kernel/awq_kernel.rs:23-61) and its
// launcher dequantize_native (:63-111). The reference maps one thread to four
// packed words; here one thread owns one packed word column (8 outputs per
// row) so that a warp's loads and stores of a row are each one contiguous
// span, and the group's zero and scales are reused across the tile's rows.
//
// Bit exactness: q - z is an exact small integer in every F. For f16 / bf16
// it is formed as (m + q) - (m + z) on packed pairs (magic-number unpack, exact)
// and multiplied by s in F, one rounding; for f32, (float)(q - z) * s, one
// rounding: in both cases the reference's multiply in F.
#pragma once

#include "cawq_common.cuh"

namespace cawq {

// One thread owns one packed word column (8 outputs per row) of a tile of
// kDqThreads words x `rows` rows: a warp's loads of a row are one 128-byte
// line and its stores one contiguous 512-byte (16-bit F) or 1 KiB (f32, as
// 256-bit stores) span. The zero word and the 8 scales of a group stay in
// registers while the tile's rows of that group stream through, and
// kDqInflight rows' words are loaded before any is used. Tiles are small
// enough that every SM holds several CTAs, and many enough (several waves)
// that a late CTA costs little.
constexpr int kDqThreads = 128;
constexpr int kDqInflight = 8;

__device__ __forceinline__ uint32_t ldg_stream_u32(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.global.nc.L1::no_allocate.u32 %0, [%1];" : "=r"(v) : "l"(p));
  return v;
}

__device__ __forceinline__ void stg_cs_v8(void* p, const float (&v)[8]) {
  asm volatile("st.global.cs.v8.f32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8};" ::"l"(p), "f"(v[0]),
               "f"(v[1]), "f"(v[2]), "f"(v[3]), "f"(v[4]), "f"(v[5]), "f"(v[6]), "f"(v[7])
               : "memory");
}

// VEC: scale and output rows 16-byte aligned (vector loads and stores);
// W8 (f32): the output also 32-byte aligned (one 256-bit store per word).
template <int DT, int ORDER, bool VEC, bool W8 = false>
__global__ void __launch_bounds__(kDqThreads)
    dequant_kernel(const uint32_t* __restrict__ qw, const uint32_t* __restrict__ qz,
                   const typename DType<DT>::T* __restrict__ sc,
                   typename DType<DT>::T* __restrict__ out, uint32_t k, uint32_t npk,
                   uint32_t g, uint32_t rows) {
  using T = typename DType<DT>::T;
  const uint32_t n = npk * 8;
  const uint32_t p = blockIdx.x * kDqThreads + threadIdx.x;
  if (p >= npk) return;
  const uint32_t row0 = blockIdx.y * rows;
  const uint32_t row1 = min(row0 + rows, k);
  uint32_t cur = 0xFFFFFFFFu;  // group whose zero word and scales are loaded
  uint32_t z = 0;
  float s[8];
  [[maybe_unused]] uint32_t zp[4], sp[4];  // 16-bit F: (m + z) and s as packed pairs
  for (uint32_t r0 = row0; r0 < row1; r0 += kDqInflight) {
    uint32_t qv[kDqInflight];
#pragma unroll
    for (int i = 0; i < kDqInflight; ++i) {
      const uint32_t row = r0 + i;
      qv[i] = row < row1 ? ldg_stream_u32(qw + (size_t)row * npk + p) : 0u;
    }
#pragma unroll
    for (int i = 0; i < kDqInflight; ++i) {
      const uint32_t row = r0 + i;
      if (row >= row1) break;
      const uint32_t grp = row / g;
      if (grp != cur) {
        cur = grp;
        z = __ldg(qz + (size_t)grp * npk + p);
        const T* srow = sc + (size_t)grp * n + (size_t)p * 8;
        if constexpr (DT != kF32) {
          pf_pairs<DT, ORDER>(z, zp);
          if constexpr (VEC) {
            const uint4 raw = __ldg(reinterpret_cast<const uint4*>(srow));
            sp[0] = raw.x; sp[1] = raw.y; sp[2] = raw.z; sp[3] = raw.w;
          } else {
            const uint16_t* h = reinterpret_cast<const uint16_t*>(srow);
#pragma unroll
            for (int c = 0; c < 4; ++c)
              sp[c] = (uint32_t)__ldg(h + 2 * c) | ((uint32_t)__ldg(h + 2 * c + 1) << 16);
          }
        } else if constexpr (VEC) {
          const float4 s0 = __ldg(reinterpret_cast<const float4*>(srow));
          const float4 s1 = __ldg(reinterpret_cast<const float4*>(srow) + 1);
          s[0] = s0.x; s[1] = s0.y; s[2] = s0.z; s[3] = s0.w;
          s[4] = s1.x; s[5] = s1.y; s[6] = s1.z; s[7] = s1.w;
        } else {
#pragma unroll
          for (int c = 0; c < 8; ++c) s[c] = srow[c];
        }
      }
      const uint32_t q = qv[i];
      T* orow = out + (size_t)row * n + (size_t)p * 8;
      if constexpr (DT != kF32) {
        // 16-bit F: (m + q) - (m + z) = q - z exactly, then one rounding of
        // the product with s, two columns per instruction
        using H = PfHalf2<DT>;
        uint32_t t[4];
        pf_pairs<DT, ORDER>(q, t);
        uint4 v;
        v.x = H::mul(H::sub(t[0], zp[0]), sp[0]);
        v.y = H::mul(H::sub(t[1], zp[1]), sp[1]);
        v.z = H::mul(H::sub(t[2], zp[2]), sp[2]);
        v.w = H::mul(H::sub(t[3], zp[3]), sp[3]);
        if constexpr (VEC) {
          stg_cs_v4(orow, v);
        } else {
          const uint32_t w4[4] = {v.x, v.y, v.z, v.w};
          uint16_t* o16 = reinterpret_cast<uint16_t*>(orow);
#pragma unroll
          for (int c = 0; c < 4; ++c) {
            o16[2 * c] = static_cast<uint16_t>(w4[c] & 0xFFFFu);
            o16[2 * c + 1] = static_cast<uint16_t>(w4[c] >> 16);
          }
        }
      } else {
        float v[8];
#pragma unroll
        for (int c = 0; c < 8; ++c) {
          const int sh = 4 * nibble_of_col(c, ORDER);
          const int d = static_cast<int>((q >> sh) & 15u) - static_cast<int>((z >> sh) & 15u);
          v[c] = __fmul_rn(static_cast<float>(d), s[c]);  // (q - z) exact, one rounding of * s
        }
        if constexpr (VEC && W8) {
          stg_cs_v8(orow, v);
        } else if constexpr (VEC) {
          stg_cs_v4(orow, make_uint4(__float_as_uint(v[0]), __float_as_uint(v[1]),
                                     __float_as_uint(v[2]), __float_as_uint(v[3])));
          stg_cs_v4(orow + 4, make_uint4(__float_as_uint(v[4]), __float_as_uint(v[5]),
                                         __float_as_uint(v[6]), __float_as_uint(v[7])));
        } else {
#pragma unroll
          for (int c = 0; c < 8; ++c) orow[c] = v[c];
        }
      }
    }
  }
}

template <int DT, int ORDER, bool VEC, bool W8 = false>
static cudaError_t launch_dequant_t(const uint32_t* qw, const uint32_t* qz, const void* sc,
                                    void* out, size_t k, size_t n, size_t g, cudaStream_t stream,
                                    int sm_count) {
  using T = typename DType<DT>::T;
  const uint32_t npk = static_cast<uint32_t>(n / 8);
  const uint32_t gx = (npk + kDqThreads - 1) / kDqThreads;
  // Rows per tile: the tallest of 64 / 32 / 16 / 8 that still gives about
  // four waves of 16 CTAs per SM (shorter tiles for small matrices); more
  // when K would need more than 65535 tiles.
  const size_t target = static_cast<size_t>(sm_count > 0 ? sm_count : 148) * 16 * 4;
  size_t rows = 64;
  while (rows > 8 && (size_t)gx * ((k + rows - 1) / rows) < target) rows >>= 1;
  if ((k + rows - 1) / rows > 65535) rows = (k + 65534) / 65535;
  dim3 grid(gx, static_cast<uint32_t>((k + rows - 1) / rows));
  dequant_kernel<DT, ORDER, VEC, W8><<<grid, kDqThreads, 0, stream>>>(
      qw, qz, static_cast<const T*>(sc), static_cast<T*>(out), static_cast<uint32_t>(k), npk,
      static_cast<uint32_t>(g), static_cast<uint32_t>(rows));
  return cudaGetLastError();
}

cudaError_t launch_dequant(const uint32_t* qw, const uint32_t* qz, const void* sc, void* out,
                           size_t k, size_t n, size_t g, int dtype, int order,
                           cudaStream_t stream, int sm_count) {
  // 16-byte vectors need 16-byte aligned scale rows and output rows; the
  // 256-bit f32 stores a 32-byte aligned output.
  const bool vec = (reinterpret_cast<uintptr_t>(sc) % 16 == 0) &&
                   (reinterpret_cast<uintptr_t>(out) % 16 == 0);
  const bool w8 = vec && reinterpret_cast<uintptr_t>(out) % 32 == 0;
#define CAWQ_DQ(DT, OR)                                                                        \
  return vec ? launch_dequant_t<DT, OR, true>(qw, qz, sc, out, k, n, g, stream, sm_count)    \
             : launch_dequant_t<DT, OR, false>(qw, qz, sc, out, k, n, g, stream, sm_count)
#define CAWQ_DQ32(OR)                                                                          \
  return w8 ? launch_dequant_t<kF32, OR, true, true>(qw, qz, sc, out, k, n, g, stream,        \
                                                     sm_count)                                \
            : vec ? launch_dequant_t<kF32, OR, true>(qw, qz, sc, out, k, n, g, stream, sm_count) \
                  : launch_dequant_t<kF32, OR, false>(qw, qz, sc, out, k, n, g, stream, sm_count)
  if (order == kOrderNatural) {
    if (dtype == kF32) { CAWQ_DQ32(kOrderNatural); }
    if (dtype == kF16) { CAWQ_DQ(kF16, kOrderNatural); }
    CAWQ_DQ(kBF16, kOrderNatural);
  }
  if (dtype == kF32) { CAWQ_DQ32(kOrderAwq); }
  if (dtype == kF16) { CAWQ_DQ(kF16, kOrderAwq); }
  CAWQ_DQ(kBF16, kOrderAwq);
#undef CAWQ_DQ32
#undef CAWQ_DQ
}

}  // namespace cawq

// cawq_decode.cuh — small-M (decode) fused AWQ GEMM for sm_100a.
//
// Y[rows, N] = X[rows, K] · ((Q - Z) · S)[K, N], rows <= 16.
// Replaces gemm_awq_decode (src/kernel/awq_kernel_gemm.rs:445-624), which the
// reference launches for M <= DECODE_M_THRESHOLD = 8 (:81, :691).
//
// The work is bound by HBM bandwidth on the packed weights (0.5 byte per
// weight). On B200 that leaves about three issue slots per weight, so the
// kernel turns nibbles into tensor-core operands with two instructions per
// pair of weights and lets mma.sync accumulate in fp32:
//
//   * Tiles. A CTA owns 128 output columns (16 packed words per k row) and a
//     slice of K. A cluster of `split` CTAs shares one column tile and splits
//     K; their partial sums are added through distributed shared memory, so
//     no global scratch is needed.
//   * Loads. Each warp streams its own k range through a ring of TMA stages:
//     a 64-row x 16-word weight box (64-byte swizzle) and the matching
//     64-column slice of X (128-byte swizzle), both landing on one mbarrier.
//   * Operands. The MMA is swapped: A = W^T (16 output columns x 16 k),
//     B = X^T (16 k x 8 rows of X). Two packed words from k rows r, r' are
//     byte-interleaved (prmt) so one lop3 yields the f16 pair
//     (1024 + q[r], 1024 + q[r']) of one column; the high nibble is taken in
//     place as 1024 + 16 q. bf16 (and f32 inputs, split into bf16 hi + lo)
//     use 128 + q with a shift. No per-weight subtraction or scaling.
//   * Group fold. Within a quantization group, sum_k x (c + q) is accumulated
//     by the MMA; when the group ends each output adds
//         s' * (D - c' * sum_k x)      (c' = offset + zero, s' = scale)
//     in fp32. This equals sum_k x (q - z) s up to fp32 rounding.
//
// Arithmetic differs from the reference in rounding only: the reference
// rounds (q - z) * s and every partial sum to F; here the weight is exact and
// the sum is fp32 (see the tolerance of the parity tests).
#pragma once

#include "cawq_common.cuh"

namespace cawq {

constexpr int kDecTileCols = 128;  // output columns per CTA
constexpr int kDecTileWords = 16;  // packed words per k row in a CTA tile
constexpr int kDecStageRows = 64;  // k rows per TMA stage (4 MMA steps)
constexpr int kDecMaxWarps = 8;
constexpr int kDecMaxStages = 4;

template <int DT, int MT>
struct DecodeLayout {
  using T = typename DType<DT>::T;
  static constexpr int XB = 8 * MT;                               // X rows per tile
  static constexpr int kXBytes = XB * kDecStageRows * (int)sizeof(T);
  static constexpr int kWBytes = kDecStageRows * kDecTileWords * 4;  // 4096
  static constexpr int kSlot = kXBytes + kWBytes;                  // multiple of 1024
  static constexpr int kRedBytes = kDecMaxWarps * XB * kDecTileCols * 4;
  static size_t smem_bytes(int warps, int stages) {
    size_t ring = (size_t)warps * stages * kSlot;
    size_t red = (size_t)warps * XB * kDecTileCols * 4;
    size_t body = ring > red ? ring : red;
    return 1024 /* alignment slack */ + body + (size_t)warps * stages * 8;
  }
};

// Physical k row (0..15 within a 16-row step) that lane quad position t uses
// for fragment slot i (0..3). Chosen so the four rows a half-warp reads fall
// in four different bank groups under the 64-byte swizzle.
__device__ __forceinline__ int dec_row(int t, int i) {
  const int base = (i & 1) * 2 + (i >> 1) * 8;  // {0, 2, 8, 10}
  return base + (t & 1) + 4 * (t >> 1);
}

// prmt selectors: bytes (b of word a, b of word b) -> result bytes 0 and 2.
__device__ __forceinline__ uint32_t dec_sel(int b) {
  return static_cast<uint32_t>(b | (b << 4) | ((4 + b) << 8) | ((4 + b) << 12));
}

template <int DT, int ODT, int ORDER, int MT>
__global__ void __launch_bounds__(kDecMaxWarps * 32)
    decode_kernel(const __grid_constant__ CUtensorMap tm_w, const __grid_constant__ CUtensorMap tm_x,
                  const uint32_t* __restrict__ qz, const typename DType<DT>::T* __restrict__ sc,
                  const typename DType<DT>::T* __restrict__ bias,
                  typename DType<ODT>::T* __restrict__ out, uint32_t rows, uint32_t k, uint32_t n,
                  uint32_t g, uint32_t ld_out, uint32_t split, uint32_t nstage_ring) {
  using L = DecodeLayout<DT, MT>;
  using T = typename DType<DT>::T;
  constexpr bool kF16Mma = (DT == kF16);
  constexpr int XB = L::XB;

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = smem_raw + ((1024 - (smem_u32(smem_raw) & 1023)) & 1023);

  const int nwarps = blockDim.x >> 5;
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int gq = lane >> 2;
  const int t = lane & 3;

  const uint32_t rank = split > 1 ? cluster_ctarank() : 0u;
  const uint32_t tile = blockIdx.x / split;
  const uint32_t p0 = tile * kDecTileWords;
  const uint32_t npk = n >> 3;
  const uint32_t steps = k >> 4;
  const uint32_t nst_total = (steps + 3) >> 2;
  const uint32_t c_beg = (uint32_t)((uint64_t)nst_total * rank / split);
  const uint32_t c_end = (uint32_t)((uint64_t)nst_total * (rank + 1) / split);
  const uint32_t w_beg = c_beg + (c_end - c_beg) * warp / nwarps;
  const uint32_t w_end = c_beg + (c_end - c_beg) * (warp + 1) / nwarps;
  const int nst = static_cast<int>(w_end - w_beg);
  const int NS = static_cast<int>(nstage_ring);

  const size_t ring_bytes = (size_t)nwarps * NS * L::kSlot;
  const size_t red_bytes = (size_t)nwarps * XB * kDecTileCols * 4;
  uint8_t* ring = smem + (size_t)warp * NS * L::kSlot;
  uint64_t* bars =
      reinterpret_cast<uint64_t*>(smem + (ring_bytes > red_bytes ? ring_bytes : red_bytes)) +
      warp * NS;

  auto issue = [&](int j) {
    const int slot = j % NS;
    uint8_t* dst = ring + (size_t)slot * L::kSlot;
    const int kr = static_cast<int>((w_beg + j) * kDecStageRows);
    mbar_arrive_expect_tx(&bars[slot], L::kSlot);
    if constexpr (DT == kF32) {
      tma_load_2d(dst, &tm_x, kr, 0, &bars[slot]);
      tma_load_2d(dst + XB * 128, &tm_x, kr + 32, 0, &bars[slot]);
    } else {
      tma_load_2d(dst, &tm_x, kr, 0, &bars[slot]);
    }
    tma_load_2d(dst + L::kXBytes, &tm_w, static_cast<int>(p0), kr, &bars[slot]);
  };

  if (lane == 0) {
    for (int s = 0; s < NS; ++s) mbar_init(&bars[s], 1);
    fence_mbarrier_init();
    fence_proxy_async_smem();
    for (int j = 0; j < NS && j < nst; ++j) issue(j);
  }
  __syncwarp();

  float D[MT][8][4];
  float tot[MT][8][4];
#pragma unroll
  for (int m = 0; m < MT; ++m)
#pragma unroll
    for (int j = 0; j < 8; ++j)
#pragma unroll
      for (int e = 0; e < 4; ++e) D[m][j][e] = tot[m][j][e] = 0.f;
  float xacc[MT];
#pragma unroll
  for (int m = 0; m < MT; ++m) xacc[m] = 0.f;

  // scale / zero of the current group for this lane's 16 columns
  const uint32_t pc = p0 + 2 * gq;
  const bool col_valid = pc < npk;
  float s_reg[16];
  uint32_t z_reg[2];
  auto load_sz = [&](uint32_t grp) {
    if (col_valid) {
      const uint2 zz = __ldg(reinterpret_cast<const uint2*>(qz + (size_t)grp * npk + pc));
      z_reg[0] = zz.x;
      z_reg[1] = zz.y;
      const T* sp = sc + (size_t)grp * n + (size_t)pc * 8;
      if constexpr (DT == kF32) {
#pragma unroll
        for (int v = 0; v < 4; ++v) {
          const float4 f = __ldg(reinterpret_cast<const float4*>(sp) + v);
          s_reg[4 * v + 0] = f.x; s_reg[4 * v + 1] = f.y;
          s_reg[4 * v + 2] = f.z; s_reg[4 * v + 3] = f.w;
        }
      } else {
#pragma unroll
        for (int v = 0; v < 2; ++v) {
          const uint4 raw = __ldg(reinterpret_cast<const uint4*>(sp) + v);
          const T* h = reinterpret_cast<const T*>(&raw);
#pragma unroll
          for (int c = 0; c < 8; ++c) s_reg[8 * v + c] = DType<DT>::to_f32(h[c]);
        }
      }
    } else {
      z_reg[0] = z_reg[1] = 0u;
#pragma unroll
      for (int c = 0; c < 16; ++c) s_reg[c] = 0.f;
    }
  };

  auto fold = [&]() {
    float X[MT][2];
#pragma unroll
    for (int m = 0; m < MT; ++m) {
      float v = xacc[m];
      v += __shfl_xor_sync(0xffffffffu, v, 1);
      v += __shfl_xor_sync(0xffffffffu, v, 2);
      X[m][0] = __shfl_sync(0xffffffffu, v, (2 * t) * 4);
      X[m][1] = __shfl_sync(0xffffffffu, v, (2 * t + 1) * 4);
      xacc[m] = 0.f;
    }
#pragma unroll
    for (int u = 0; u < 2; ++u) {
#pragma unroll
      for (int b = 0; b < 4; ++b) {
        const int j = u * 4 + b;
        const float zl = static_cast<float>((z_reg[u] >> (8 * b)) & 15u);
        const float zh = static_cast<float>((z_reg[u] >> (8 * b + 4)) & 15u);
        const float sl = s_reg[u * 8 + col_of_nibble(2 * b, ORDER)];
        float sh = s_reg[u * 8 + col_of_nibble(2 * b + 1, ORDER)];
        float cl, ch;
        if constexpr (kF16Mma) {
          cl = 1024.f + zl;
          ch = 1024.f + 16.f * zh;
          sh *= 0.0625f;
        } else {
          cl = 128.f + zl;
          ch = 128.f + zh;
        }
#pragma unroll
        for (int m = 0; m < MT; ++m) {
          tot[m][j][0] = fmaf(sl, fmaf(-cl, X[m][0], D[m][j][0]), tot[m][j][0]);
          tot[m][j][1] = fmaf(sl, fmaf(-cl, X[m][1], D[m][j][1]), tot[m][j][1]);
          tot[m][j][2] = fmaf(sh, fmaf(-ch, X[m][0], D[m][j][2]), tot[m][j][2]);
          tot[m][j][3] = fmaf(sh, fmaf(-ch, X[m][1], D[m][j][3]), tot[m][j][3]);
          D[m][j][0] = D[m][j][1] = D[m][j][2] = D[m][j][3] = 0.f;
        }
      }
    }
  };

  bool ok = true;
  int cur_grp = -1;
  if (nst > 0) {
    cur_grp = static_cast<int>((w_beg * kDecStageRows) / g);
    load_sz(static_cast<uint32_t>(cur_grp));
  }

  for (int j = 0; j < nst; ++j) {
    const int slot = j % NS;
    if (ok) ok = mbar_wait_bounded(&bars[slot], static_cast<uint32_t>((j / NS) & 1));
    ok = __all_sync(0xffffffffu, ok);  // keep the warp convergent for the shuffles
    const uint32_t xbase = smem_u32(ring + (size_t)slot * L::kSlot);
    const uint32_t wbase = xbase + L::kXBytes;
    const uint32_t stage = w_beg + j;
#pragma unroll 1
    for (int s = 0; s < 4; ++s) {
      const uint32_t step = stage * 4 + s;
      if (!ok || step >= steps) break;
      const int grp = static_cast<int>((step * 16) / g);
      if (grp != cur_grp) {
        fold();
        cur_grp = grp;
        load_sz(static_cast<uint32_t>(grp));
      }
      // ---- weights: rows dec_row(t, i) of this step, words 2gq, 2gq+1
      uint32_t wv[4][2];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int r = s * 16 + dec_row(t, i);
        const uint32_t addr = wbase + r * 64 + ((((gq >> 1) ^ ((r >> 1) & 3))) << 4) + ((gq & 1) << 3);
        asm volatile("ld.shared.v2.u32 {%0,%1}, [%2];"
                     : "=r"(wv[i][0]), "=r"(wv[i][1])
                     : "r"(addr));
      }
      // ---- X^T fragments for rows 8m + gq
      uint32_t bh[MT][2], bl[MT][2];
#pragma unroll
      for (int m = 0; m < MT; ++m) {
        const int xr = 8 * m + gq;
        float xv[4];
        uint16_t raw16[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const int kk = s * 16 + dec_row(t, i);
          if constexpr (DT == kF32) {
            const int h = kk >> 5, kq = kk & 31;
            const uint32_t a = xbase + h * XB * 128 + xr * 128 + (((kq >> 2) ^ (xr & 7)) << 4) + ((kq & 3) << 2);
            asm volatile("ld.shared.f32 %0, [%1];" : "=f"(xv[i]) : "r"(a));
          } else {
            const uint32_t a = xbase + xr * 128 + (((kk >> 3) ^ (xr & 7)) << 4) + ((kk & 7) << 1);
            asm volatile("ld.shared.u16 %0, [%1];" : "=h"(raw16[i]) : "r"(a));
          }
        }
        if constexpr (DT == kF32) {
          float hs = 0.f;
#pragma unroll
          for (int pr = 0; pr < 2; ++pr) {
            const __nv_bfloat162 hi = __floats2bfloat162_rn(xv[2 * pr], xv[2 * pr + 1]);
            const float h0 = __low2float(hi), h1 = __high2float(hi);
            const __nv_bfloat162 lo = __floats2bfloat162_rn(xv[2 * pr] - h0, xv[2 * pr + 1] - h1);
            bh[m][pr] = *reinterpret_cast<const uint32_t*>(&hi);
            bl[m][pr] = *reinterpret_cast<const uint32_t*>(&lo);
            hs += (h0 + __low2float(lo)) + (h1 + __high2float(lo));
          }
          xacc[m] += hs;
        } else {
          bh[m][0] = static_cast<uint32_t>(raw16[0]) | (static_cast<uint32_t>(raw16[1]) << 16);
          bh[m][1] = static_cast<uint32_t>(raw16[2]) | (static_cast<uint32_t>(raw16[3]) << 16);
          float hs = 0.f;
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            if constexpr (DT == kF16) {
              hs += __half2float(__ushort_as_half(raw16[i]));
            } else {
              hs += __bfloat162float(__ushort_as_bfloat16(raw16[i]));
            }
          }
          xacc[m] += hs;
        }
      }
      // ---- dequantize into A fragments and multiply
#pragma unroll
      for (int u = 0; u < 2; ++u) {
#pragma unroll
        for (int b = 0; b < 4; ++b) {
          const uint32_t p01 = prmt(wv[0][u], wv[1][u], dec_sel(b));
          const uint32_t p23 = prmt(wv[2][u], wv[3][u], dec_sel(b));
          uint32_t a0, a1, a2, a3;
          if constexpr (kF16Mma) {
            a0 = lop3_and_or(p01, 0x000F000Fu, 0x64006400u);
            a1 = lop3_and_or(p01, 0x00F000F0u, 0x64006400u);
            a2 = lop3_and_or(p23, 0x000F000Fu, 0x64006400u);
            a3 = lop3_and_or(p23, 0x00F000F0u, 0x64006400u);
          } else {
            a0 = lop3_and_or(p01, 0x000F000Fu, 0x43004300u);
            a1 = lop3_and_or(p01 >> 4, 0x000F000Fu, 0x43004300u);
            a2 = lop3_and_or(p23, 0x000F000Fu, 0x43004300u);
            a3 = lop3_and_or(p23 >> 4, 0x000F000Fu, 0x43004300u);
          }
#pragma unroll
          for (int m = 0; m < MT; ++m) {
            mma_16816<!kF16Mma>(D[m][u * 4 + b], a0, a1, a2, a3, bh[m][0], bh[m][1]);
            if constexpr (DT == kF32) {
              mma_16816<true>(D[m][u * 4 + b], a0, a1, a2, a3, bl[m][0], bl[m][1]);
            }
          }
        }
      }
    }
    __syncwarp();
    if (lane == 0 && ok && j + NS < nst) {
      fence_proxy_async_smem();
      issue(j + NS);
    }
    __syncwarp();
  }
  if (cur_grp >= 0) fold();

  // ---- reduction: warps of this CTA, then the CTAs of the cluster
  __syncthreads();
  float* red = reinterpret_cast<float*>(smem);  // [nwarps][XB][128], reuses the ring
#pragma unroll
  for (int m = 0; m < MT; ++m) {
#pragma unroll
    for (int u = 0; u < 2; ++u) {
#pragma unroll
      for (int b = 0; b < 4; ++b) {
        const int j = u * 4 + b;
        const int cl = (2 * gq + u) * 8 + col_of_nibble(2 * b, ORDER);
        const int ch = (2 * gq + u) * 8 + col_of_nibble(2 * b + 1, ORDER);
        float* r0 = red + ((size_t)warp * XB + 8 * m + 2 * t) * kDecTileCols;
        float* r1 = r0 + kDecTileCols;
        r0[cl] = tot[m][j][0];
        r1[cl] = tot[m][j][1];
        r0[ch] = tot[m][j][2];
        r1[ch] = tot[m][j][3];
      }
    }
  }
  __syncthreads();
  const int rows_eff = static_cast<int>(rows < (uint32_t)XB ? rows : (uint32_t)XB);
  for (int idx = threadIdx.x; idx < rows_eff * kDecTileCols; idx += blockDim.x) {
    const int b = idx / kDecTileCols, c = idx % kDecTileCols;
    float v = 0.f;
    for (int w = 0; w < nwarps; ++w) v += red[((size_t)w * XB + b) * kDecTileCols + c];
    red[(size_t)b * kDecTileCols + c] = v;
  }
  if (split > 1) {
    cluster_sync_all();
  } else {
    __syncthreads();
  }
  const int cbeg = static_cast<int>(kDecTileCols * rank / split);
  const int cend = static_cast<int>(kDecTileCols * (rank + 1) / split);
  const int ncols = cend - cbeg;
  for (int idx = threadIdx.x; idx < rows_eff * ncols; idx += blockDim.x) {
    const int b = idx / ncols, c = cbeg + idx % ncols;
    const uint32_t col = p0 * 8 + c;
    float v = 0.f;
    if (split > 1) {
      const uint32_t a = smem_u32(red + (size_t)b * kDecTileCols + c);
      for (uint32_t q = 0; q < split; ++q) v += ld_shared_cluster_f32(map_shared_rank(a, q));
    } else {
      v = red[(size_t)b * kDecTileCols + c];
    }
    if (col < n) {
      if (bias) v += DType<DT>::to_f32(bias[col]);
      out[(size_t)b * ld_out + col] = DType<ODT>::from_f32(v);
    }
  }
  if (split > 1) cluster_sync_all();
}

// ------------------------------------------------------------------ host
static bool encode_2d(CUtensorMap* map, CUtensorMapDataType dt, const void* base, uint64_t inner,
                      uint64_t outer, uint64_t row_bytes, uint32_t box_inner, uint32_t box_outer,
                      CUtensorMapSwizzle swz) {
  EncodeTiledFn fn = encode_tiled_fn();
  if (!fn) return false;
  const uint64_t dims[2] = {inner, outer};
  const uint64_t strides[1] = {row_bytes};
  const uint32_t box[2] = {box_inner, box_outer};
  const uint32_t estr[2] = {1, 1};
  const int r = fn(map, static_cast<int>(dt), 2, const_cast<void*>(base), dims, strides, box, estr,
                   static_cast<int>(CU_TENSOR_MAP_INTERLEAVE_NONE), static_cast<int>(swz),
                   static_cast<int>(CU_TENSOR_MAP_L2_PROMOTION_L2_256B),
                   static_cast<int>(CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE));
  return r == 0;
}

static int decode_mt(size_t rows) { return rows <= 8 ? 1 : 2; }

bool decode_supports(const GemmProblem& p, const cawq_plan& plan, const DeviceInfo& dev) {
  if (p.rows == 0 || p.rows > 16) return false;
  if (p.k % 16 != 0 || p.g % 16 != 0 || p.k % p.g != 0 || p.n % 32 != 0) return false;
  if (p.k >= (1ull << 31) || p.n >= (1ull << 31) || p.ld_out >= (1ull << 31)) return false;
  const uintptr_t ax = reinterpret_cast<uintptr_t>(p.x), aw = reinterpret_cast<uintptr_t>(p.qw);
  const uintptr_t az = reinterpret_cast<uintptr_t>(p.qz), as = reinterpret_cast<uintptr_t>(p.sc);
  if (ax % 16 || aw % 16 || az % 8 || as % 16) return false;
  if (plan.split < 1 || plan.split > 16 || (plan.split & (plan.split - 1))) return false;
  if (plan.warps < 1 || plan.warps > kDecMaxWarps) return false;
  if (plan.stages < 1 || plan.stages > kDecMaxStages) return false;
  const size_t tiles = (p.n + kDecTileCols - 1) / kDecTileCols;
  if (tiles * plan.split >= (1ull << 31)) return false;
  size_t smem = 0;
  if (p.dtype == kF32) {
    smem = decode_mt(p.rows) == 1 ? DecodeLayout<kF32, 1>::smem_bytes(plan.warps, plan.stages)
                                  : DecodeLayout<kF32, 2>::smem_bytes(plan.warps, plan.stages);
  } else {
    smem = decode_mt(p.rows) == 1 ? DecodeLayout<kF16, 1>::smem_bytes(plan.warps, plan.stages)
                                  : DecodeLayout<kF16, 2>::smem_bytes(plan.warps, plan.stages);
  }
  return smem <= dev.smem_optin && dev.cc_major == 10;
}

template <int DT, int ODT, int ORDER, int MT>
static cudaError_t launch_decode_t(const GemmProblem& p, const cawq_plan& plan) {
  using L = DecodeLayout<DT, MT>;
  using T = typename DType<DT>::T;
  using OT = typename DType<ODT>::T;
  CUtensorMap tm_w, tm_x;
  const uint64_t npk = p.n / 8;
  if (!encode_2d(&tm_w, CU_TENSOR_MAP_DATA_TYPE_UINT32, p.qw, npk, p.k, npk * 4, kDecTileWords,
                 kDecStageRows, CU_TENSOR_MAP_SWIZZLE_64B)) {
    return cudaErrorInvalidValue;
  }
  const CUtensorMapDataType xdt = DT == kF32   ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32
                                  : DT == kF16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16
                                               : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
  const uint32_t xbox = DT == kF32 ? 32 : 64;  // 128-byte rows for the 128B swizzle
  if (!encode_2d(&tm_x, xdt, p.x, p.k, p.rows, p.k * sizeof(T), xbox, L::XB,
                 CU_TENSOR_MAP_SWIZZLE_128B)) {
    return cudaErrorInvalidValue;
  }
  auto kern = decode_kernel<DT, ODT, ORDER, MT>;
  const size_t smem = L::smem_bytes(plan.warps, plan.stages);
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       static_cast<int>(smem));
  if (e != cudaSuccess) return e;
  if (plan.split > 8) {
    e = cudaFuncSetAttribute(kern, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
    if (e != cudaSuccess) return e;
  }
  const uint32_t tiles = static_cast<uint32_t>((p.n + kDecTileCols - 1) / kDecTileCols);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(tiles * plan.split);
  cfg.blockDim = dim3(plan.warps * 32);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = p.stream;
  cudaLaunchAttribute attr[1];
  if (plan.split > 1) {
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = plan.split;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
  }
  return cudaLaunchKernelEx(&cfg, kern, tm_w, tm_x, p.qz, static_cast<const T*>(p.sc),
                            static_cast<const T*>(p.bias), static_cast<OT*>(p.out),
                            static_cast<uint32_t>(p.rows), static_cast<uint32_t>(p.k),
                            static_cast<uint32_t>(p.n), static_cast<uint32_t>(p.g),
                            static_cast<uint32_t>(p.ld_out), static_cast<uint32_t>(plan.split),
                            static_cast<uint32_t>(plan.stages));
}

template <int DT, int ODT, int ORDER>
static cudaError_t launch_decode_m(const GemmProblem& p, const cawq_plan& plan) {
  return decode_mt(p.rows) == 1 ? launch_decode_t<DT, ODT, ORDER, 1>(p, plan)
                                : launch_decode_t<DT, ODT, ORDER, 2>(p, plan);
}

template <int DT, int ODT>
static cudaError_t launch_decode_o(const GemmProblem& p, const cawq_plan& plan) {
  return p.order == kOrderNatural ? launch_decode_m<DT, ODT, kOrderNatural>(p, plan)
                                  : launch_decode_m<DT, ODT, kOrderAwq>(p, plan);
}

cudaError_t launch_decode(const GemmProblem& p, const cawq_plan& plan, const DeviceInfo&) {
  if (p.dtype == kF32) return launch_decode_o<kF32, kF32>(p, plan);
  if (p.dtype == kF16) {
    return p.out_dtype == kF32 ? launch_decode_o<kF16, kF32>(p, plan)
                               : launch_decode_o<kF16, kF16>(p, plan);
  }
  return p.out_dtype == kF32 ? launch_decode_o<kBF16, kF32>(p, plan)
                             : launch_decode_o<kBF16, kBF16>(p, plan);
}

cawq_plan decode_default_plan(const GemmProblem& p, const DeviceInfo& dev) {
  cawq_plan plan = {};
  plan.path = CAWQ_PATH_DECODE;
  plan.warps = 8;
  plan.stages = 2;
  const size_t tiles = (p.n + kDecTileCols - 1) / kDecTileCols;
  const size_t nst_total = (p.k / 16 + 3) / 4;
  const size_t target = static_cast<size_t>(dev.sm_count > 0 ? dev.sm_count : 148) * 2;
  int split = 1;
  while (split < 16 && tiles * split < target && nst_total >= (size_t)split * 2 * plan.warps) split *= 2;
  while (plan.warps > 4 && nst_total < (size_t)split * plan.warps) plan.warps /= 2;
  plan.split = split;
  return plan;
}

void decode_candidates(const GemmProblem& p, const DeviceInfo& dev, cawq_plan* out, int* count,
                       int max_count) {
  int c = 0;
  for (int split = 1; split <= 16; split *= 2) {
    for (int warps = 4; warps <= 8; warps *= 2) {
      for (int stages = 2; stages <= 4; stages *= 2) {
        cawq_plan pl = {};
        pl.path = CAWQ_PATH_DECODE;
        pl.split = split;
        pl.warps = warps;
        pl.stages = stages;
        const size_t nst_total = (p.k / 16 + 3) / 4;
        if (nst_total < (size_t)split * warps) continue;  // idle warps
        if (!decode_supports(p, pl, dev)) continue;
        if (c < max_count) out[c++] = pl;
      }
    }
  }
  *count = c;
}

}  // namespace cawq

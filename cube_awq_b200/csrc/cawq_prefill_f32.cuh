// cawq_prefill_f32.cuh — large-M fused AWQ GEMM with f32 activations and
// scales on tcgen05 tensor cores (sm_100a).
//
// Y[M, N] = X[M, K] · ((Q - Z) · S)[K, N], F = f32: the reference's gemm_awq
// with F = f32 (src/kernel/awq_kernel_gemm.rs:181-439), the precision its own
// tests use. The tensor cores take 16-bit operands, so the f32 arithmetic is
// arranged so that nothing is lost where it matters:
//
//   * B = (q - z), a small integer, is exact in bf16: the weights enter the
//     MMA without rounding and the scale is not applied there;
//   * X = hi + lo with hi = x truncated to bf16 and lo = bf16(x - hi), so
//     |x - hi - lo| <= 2^-16 |x|; two MMAs (hi·B + lo·B) per k step;
//   * each quantization group accumulates in its own fp32 TMEM buffer (two,
//     used in turn), and the epilogue warps add s[g, n] · D_g into a running
//     fp32 sum kept in TMEM while the tensor core fills the other buffer:
//     Y = sum_g s_g · (sum_{k in g} x (q - z)).
//
// The result differs from the reference's sequential f32 sum by rounding
// only: every product is exact but for the 2^-16 split of x, and the sums are
// fp32 (the parity tests bound it against the exact fp64 oracle at the north
// star's 1e-3 · ||ref||_inf).
//
// CTA tile 128 x BN (BN = 256 when the grid fills the GPU, else 128), 64-row
// k stages; 15 + S warps (S = 4 X-split warps for BN = 256, 8 for 128):
//   warp 0      TMA producer of the f32 X ring (two 32-column boxes a stage);
//   warp 1      allocates 512 TMEM columns (two 128-column group slots, the
//               running sum) and issues tcgen05.mma.cta_group::1.kind::f16
//               (bf16, M=128, N=128, K=16) per 128-column block;
//   warp 2      TMA producer of the packed weights + zero row (W ring) and,
//               at each group's first stage, of the group's scale row;
//   next S      split each X stage into the hi / lo bf16 A tiles (K-major,
//               128-byte swizzle): every column tile converts its own rows of
//               X, so a wider tile spends this work on more columns;
//   next 4      turn the packed stage into the exact (q - z) bf16 B tile
//               (MN-major, 128-byte swizzle);
//   last 8      per group: running += s · D_g (tcgen05.ld / st), two warps per
//               TMEM lane quarter; after the last group, add the bias and
//               store the rows. This fold is what paces the kernel: without
//               it a 64-row stage of a 128 x 256 tile took 1.1 us, with it
//               1.44 us.
// Group slots: block h (128 columns) of group g accumulates in TMEM slot
// (g · BN/128 + h) mod 2. With BN = 128 the two slots double-buffer whole
// groups; with BN = 256 block 0 of the next group waits only for block 0 of
// this one to be read, so reading block 1 overlaps the next MMAs.
#pragma once

#include "cawq_common.cuh"
#include "cawq_prefill.cuh"

namespace cawq {

constexpr int kP32BM = 128;
constexpr int kP32BK = 64;
// X-split warps: a 128-column tile splits the same X stage for half the
// MMA work of a 256-column one, so it gets twice the warps; the 256-column
// tile's fewer threads leave the epilogue registers for 32-column TMEM
// chunks (at 23 warps those spill and 16-column chunks are used).
// Measured per 64-row stage at M = 2048: 128-column tiles 1.05 us with 8
// split warps against 1.13 us with 4; 256-column tiles 1.44 us with 4 split
// warps and 32-column chunks against 1.54 us with 8 and 16.
__host__ __device__ constexpr int p32_split_warps(int bn) { return bn == 256 ? 4 : 8; }
__host__ __device__ constexpr int p32_chunk_cols(int bn) { return bn == 256 ? 32 : 16; }
// group-epilogue warps (a multiple of 4: whole TMEM lane quarters)
__host__ __device__ constexpr int p32_epi_warps(int bn) { return 8; }
__host__ __device__ constexpr int p32_threads(int bn) {
  return (7 + p32_split_warps(bn) + p32_epi_warps(bn)) * 32;
}

template <int BN>
struct P32Layout {
  static constexpr int kNB = BN / 128;                // 128-column MMA blocks
  static constexpr int kXSt = 2, kASt = BN == 256 ? 2 : 3, kWSt = BN == 256 ? 3 : 4, kBSt = 2;
  static constexpr int kX = kP32BM * kP32BK * 4;      // 32768: f32 X, two 128-B boxes
  static constexpr int kA = kP32BM * kP32BK * 2;      // 16384: one bf16 A tile (hi or lo)
  static constexpr int kB = kP32BK * BN * 2;          // bf16 B tile
  static constexpr int kWords = BN / 8;               // packed words per k row
  static constexpr int kW = kP32BK * kWords * 4;      // packed words, BN / 2 bytes a row
  static constexpr int kZ = kWords * 4;               // the stage's zero row
  static constexpr int kWSlot = (kW + kZ + 255) / 256 * 256;
  static constexpr int kS = BN * 4;                   // a group's scale row
  static constexpr size_t kOffA = (size_t)kX * kXSt;
  static constexpr size_t kOffB = kOffA + (size_t)2 * kA * kASt;
  static constexpr size_t kOffW = kOffB + (size_t)kB * kBSt;
  static constexpr size_t kOffS = kOffW + (size_t)kWSlot * kWSt;
  static constexpr size_t kOffBars = kOffS + (size_t)kS * 2;
  static constexpr size_t kSmem = 1024 + kOffBars + 512;
};

// 32 lanes x 32 fp32 columns -> registers, without the wait (the caller
// issues tcgen05.wait::ld before using them).
__device__ __forceinline__ void tmem_ld_32x32b_x32_nowait(uint32_t taddr, float (&v)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=f"(v[0]), "=f"(v[1]), "=f"(v[2]), "=f"(v[3]), "=f"(v[4]), "=f"(v[5]), "=f"(v[6]),
        "=f"(v[7]), "=f"(v[8]), "=f"(v[9]), "=f"(v[10]), "=f"(v[11]), "=f"(v[12]), "=f"(v[13]),
        "=f"(v[14]), "=f"(v[15]), "=f"(v[16]), "=f"(v[17]), "=f"(v[18]), "=f"(v[19]),
        "=f"(v[20]), "=f"(v[21]), "=f"(v[22]), "=f"(v[23]), "=f"(v[24]), "=f"(v[25]),
        "=f"(v[26]), "=f"(v[27]), "=f"(v[28]), "=f"(v[29]), "=f"(v[30]), "=f"(v[31])
      : "r"(taddr)
      : "memory");
}

// 32 lanes x 32 fp32 columns <- registers, without the wait (the caller
// issues tcgen05.wait::st before the columns are read again).
__device__ __forceinline__ void tmem_st_32x32b_x32_nowait(uint32_t taddr, const float (&v)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], "
      "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
      "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
      "f"(v[0]), "f"(v[1]), "f"(v[2]), "f"(v[3]), "f"(v[4]), "f"(v[5]), "f"(v[6]), "f"(v[7]),
      "f"(v[8]), "f"(v[9]), "f"(v[10]), "f"(v[11]), "f"(v[12]), "f"(v[13]), "f"(v[14]),
      "f"(v[15]), "f"(v[16]), "f"(v[17]), "f"(v[18]), "f"(v[19]), "f"(v[20]), "f"(v[21]),
      "f"(v[22]), "f"(v[23]), "f"(v[24]), "f"(v[25]), "f"(v[26]), "f"(v[27]), "f"(v[28]),
      "f"(v[29]), "f"(v[30]), "f"(v[31])
      : "memory");
}

// 32 lanes x 16 fp32 columns <-> registers, without the waits.
__device__ __forceinline__ void tmem_ld_32x32b_x16_nowait(uint32_t taddr, float (&v)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=f"(v[0]), "=f"(v[1]), "=f"(v[2]), "=f"(v[3]), "=f"(v[4]), "=f"(v[5]), "=f"(v[6]),
        "=f"(v[7]), "=f"(v[8]), "=f"(v[9]), "=f"(v[10]), "=f"(v[11]), "=f"(v[12]), "=f"(v[13]),
        "=f"(v[14]), "=f"(v[15])
      : "r"(taddr)
      : "memory");
}

__device__ __forceinline__ void tmem_st_32x32b_x16_nowait(uint32_t taddr, const float (&v)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], "
      "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};" ::"r"(taddr),
      "f"(v[0]), "f"(v[1]), "f"(v[2]), "f"(v[3]), "f"(v[4]), "f"(v[5]), "f"(v[6]), "f"(v[7]),
      "f"(v[8]), "f"(v[9]), "f"(v[10]), "f"(v[11]), "f"(v[12]), "f"(v[13]), "f"(v[14]),
      "f"(v[15])
      : "memory");
}

template <int W>
__device__ __forceinline__ void tmem_ld_cols_nowait(uint32_t taddr, float (&v)[W]) {
  if constexpr (W == 32) tmem_ld_32x32b_x32_nowait(taddr, v);
  else tmem_ld_32x32b_x16_nowait(taddr, v);
}
template <int W>
__device__ __forceinline__ void tmem_st_cols_nowait(uint32_t taddr, const float (&v)[W]) {
  if constexpr (W == 32) tmem_st_32x32b_x32_nowait(taddr, v);
  else tmem_st_32x32b_x16_nowait(taddr, v);
}

// x (f32 pair) -> (hi, lo) bf16 pairs: hi = x with its low 16 bits cleared
// (exact), lo = x - hi (exact in f32) rounded to bf16.
__device__ __forceinline__ void split_bf16x2(float x0, float x1, uint32_t& hi, uint32_t& lo) {
  const uint32_t u0 = __float_as_uint(x0), u1 = __float_as_uint(x1);
  hi = prmt(u0, u1, 0x7632u);
  // (x0, x1) - (hi0, hi1) as one packed f32x2 subtraction
  const uint64_t xv = (uint64_t)u0 | ((uint64_t)u1 << 32);
  const uint64_t hv = xv & 0xFFFF0000FFFF0000ull;
  uint64_t rv;
  asm("sub.rn.f32x2 %0, %1, %2;" : "=l"(rv) : "l"(xv), "l"(hv));
  const __nv_bfloat162 l = __floats2bfloat162_rn(__uint_as_float((uint32_t)rv),
                                                 __uint_as_float((uint32_t)(rv >> 32)));
  lo = *reinterpret_cast<const uint32_t*>(&l);
}

template <int ORDER, int BN>
__global__ void __launch_bounds__(p32_threads(BN), 1)
    prefill_f32_kernel(const __grid_constant__ CUtensorMap tm_x,
                       const __grid_constant__ CUtensorMap tm_w,
                       const __grid_constant__ CUtensorMap tm_s,
                       const __grid_constant__ CUtensorMap tm_z, const float* __restrict__ bias,
                       const OutMap<float> om, uint32_t rows, uint32_t k, uint32_t n, uint32_t g) {
  using L = P32Layout<BN>;
  constexpr int NB = L::kNB;
  constexpr int kP32SplitWarps = p32_split_warps(BN);
  constexpr int kP32EpiWarps = p32_epi_warps(BN);
  constexpr int kParts = kP32EpiWarps / 4;  // epilogue warps per TMEM lane quarter
  constexpr int kPartCols = 128 / kParts;   // columns of a block per epilogue warp
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = smem_raw + ((1024 - (smem_u32(smem_raw) & 1023)) & 1023);
  uint64_t* xfull = reinterpret_cast<uint64_t*>(smem + L::kOffBars);
  uint64_t* xempty = xfull + L::kXSt;
  uint64_t* afull = xempty + L::kXSt;
  uint64_t* aempty = afull + L::kASt;
  uint64_t* wfull = aempty + L::kASt;
  uint64_t* wempty = wfull + L::kWSt;
  uint64_t* bfull = wempty + L::kWSt;
  uint64_t* bempty = bfull + L::kBSt;
  uint64_t* dfull = bempty + L::kBSt;  // [2] a block's group sum is in TMEM slot [i]
  uint64_t* dempty = dfull + 2;        // [2] the epilogue has read slot [i]
  uint64_t* sfull = dempty + 2;        // [2] the group's scale row landed
  uint64_t* sempty = sfull + 2;        // [2] the epilogue is done with it
  uint64_t* drain_bar = sempty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain_bar + 1);
  __shared__ int s_x_issued, s_w_issued;
  bool role_ok = true;

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t n0 = blockIdx.x * BN;
  const uint32_t m0 = blockIdx.y * kP32BM;
  const int KT = static_cast<int>(k / kP32BK);
  const int spg = static_cast<int>(g / kP32BK);  // stages per group (g % 64 == 0)
  const int NG = KT / spg;

  auto x_slot = [&](int s) { return smem + (size_t)s * L::kX; };
  auto a_slot = [&](int s) { return smem + L::kOffA + (size_t)s * 2 * L::kA; };
  auto b_slot = [&](int s) { return smem + L::kOffB + (size_t)s * L::kB; };
  auto w_slot = [&](int s) { return smem + L::kOffW + (size_t)s * L::kWSlot; };
  auto s_slot = [&](int b) { return reinterpret_cast<const float*>(smem + L::kOffS + (size_t)b * L::kS); };

  if (threadIdx.x == 0) {
    for (int s = 0; s < L::kXSt; ++s) {
      mbar_init(&xfull[s], 1);
      mbar_init(&xempty[s], 32 * kP32SplitWarps);
    }
    for (int s = 0; s < L::kASt; ++s) {
      mbar_init(&afull[s], 32 * kP32SplitWarps);
      mbar_init(&aempty[s], 1);
    }
    for (int s = 0; s < L::kWSt; ++s) {
      mbar_init(&wfull[s], 1);
      mbar_init(&wempty[s], 128);
    }
    for (int s = 0; s < L::kBSt; ++s) {
      mbar_init(&bfull[s], 128);
      mbar_init(&bempty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&dfull[b], 1);
      mbar_init(&dempty[b], 32 * kP32EpiWarps);  // every epilogue warp reads each slot
      mbar_init(&sfull[b], 1);
      mbar_init(&sempty[b], 32 * kP32EpiWarps);
    }
    mbar_init(drain_bar, 1);
    fence_mbarrier_init();
    fence_proxy_async_smem();
    tma_prefetch_desc(&tm_x);
    tma_prefetch_desc(&tm_w);
  }
  if (warp == 1) tmem_alloc(tmem_slot, 512);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  pdl_launch_dependents();

  if (warp == 0) {
    // ------------------------------------------------- X ring producer
    if (lane == 0) {
      bool ok = true;
      int issued = 0;
      pdl_wait();  // X may be the previous kernel's output
      for (int i = 0; i < KT && ok; ++i) {
        const int s = i % L::kXSt, u = i / L::kXSt;
        if (u > 0) ok = mbar_wait_bounded(&xempty[s], (uint32_t)((u - 1) & 1));
        if (!ok) break;
        mbar_arrive_expect_tx(&xfull[s], L::kX);
        tma_load_2d(x_slot(s), &tm_x, i * kP32BK, static_cast<int>(m0), &xfull[s]);
        tma_load_2d(x_slot(s) + L::kX / 2, &tm_x, i * kP32BK + 32, static_cast<int>(m0),
                    &xfull[s]);
        issued = i + 1;
      }
      s_x_issued = issued;
      role_ok = ok;
    }
    __syncwarp();
  } else if (warp == 2) {
    // ---------------------------------- W ring + group scale producer
    if (lane == 0) {
      bool ok = true;
      int issued = 0;
      for (int i = 0; i < KT && ok; ++i) {
        const int s = i % L::kWSt, u = i / L::kWSt;
        const int grp = i / spg;
        if (i % spg == 0) {
          const int b = grp & 1;
          if (grp >= 2) ok = mbar_wait_bounded(&sempty[b], (uint32_t)(((grp >> 1) - 1) & 1));
          if (!ok) break;
          mbar_arrive_expect_tx(&sfull[b], L::kS);
          tma_load_2d(smem + L::kOffS + (size_t)b * L::kS, &tm_s, static_cast<int>(n0), grp,
                      &sfull[b]);
        }
        if (u > 0) ok = mbar_wait_bounded(&wempty[s], (uint32_t)((u - 1) & 1));
        if (!ok) break;
        mbar_arrive_expect_tx(&wfull[s], L::kW + L::kZ);
        tma_load_2d(w_slot(s), &tm_w, static_cast<int>(n0 / 8), i * kP32BK, &wfull[s]);
        tma_load_2d(w_slot(s) + L::kW, &tm_z, static_cast<int>(n0 / 8), grp, &wfull[s]);
        issued = i + 1;
      }
      s_w_issued = issued;
      role_ok = ok;
    }
    __syncwarp();
  } else if (warp == 1) {
    // ------------------------------------------------------- MMA issuer
    if (lane == 0) {
      // per k step one N = 128 MMA per 128-column block, block 0 first: at a
      // group's first stage block 0 waits only for the epilogue to have read
      // block 0 of the previous group, and at its last stage block 0's sum is
      // handed to the epilogue before block 1's last MMAs complete
      constexpr uint32_t idesc = umma_idesc_f16(true, kP32BM, 128);
      bool ok = true;
      for (int kt = 0; kt < KT && ok; ++kt) {
        const int grp = kt / spg;
        const bool first = kt % spg == 0, last = kt % spg == spg - 1;
        const int sa = kt % L::kASt, ua = kt / L::kASt;
        const int sb = kt % L::kBSt, ub = kt / L::kBSt;
        ok = mbar_wait_bounded(&afull[sa], (uint32_t)(ua & 1)) &&
             mbar_wait_bounded(&bfull[sb], (uint32_t)(ub & 1));
        if (!ok) break;
        tc_fence_after();
        const uint32_t ahi = smem_u32(a_slot(sa)), alo = ahi + L::kA;
        const uint32_t ba = smem_u32(b_slot(sb));
#pragma unroll
        for (int h = 0; h < NB; ++h) {
          const int use = grp * NB + h, slot = use & 1;
          // the slot's previous group must have been read by the epilogue
          if (first && use >= 2) {
            ok = mbar_wait_bounded(&dempty[slot], (uint32_t)(((use >> 1) - 1) & 1));
            if (!ok) break;
            tc_fence_after();
          }
          const uint32_t d = tmem + (uint32_t)slot * 128;
#pragma unroll
          for (int j = 0; j < kP32BK / 16; ++j) {
            // columns [128 h, 128 h + 128): 64-column atoms 2h and 2h + 1
            const uint64_t bd = umma_desc_sw128(ba + 16384 * h + 2048 * j, 8192, 1024);
            umma_f16(d, umma_desc_sw128(ahi + 32 * j, 16, 1024), bd, idesc,
                     (first && j == 0) ? 0u : 1u);
            umma_f16(d, umma_desc_sw128(alo + 32 * j, 16, 1024), bd, idesc, 1u);
          }
          if (last) umma_commit(&dfull[slot]);
        }
        if (!ok) break;
        umma_commit(&aempty[sa]);
        umma_commit(&bempty[sb]);
      }
      if (!ok) {
        umma_commit(drain_bar);  // wait (bounded) for the MMAs already issued
        mbar_wait_bounded(drain_bar, 0u);
      }
      role_ok = ok;
    }
    __syncwarp();
  } else if (warp >= 3 && warp < 3 + kP32SplitWarps) {
    // ------------------------------------------ X split into hi / lo
    constexpr int kSplitThreads = 32 * kP32SplitWarps;
    const int t = threadIdx.x - 96;
    bool ok = true;
    for (int kt = 0; kt < KT; ++kt) {
      const int sx = kt % L::kXSt, ux = kt / L::kXSt;
      const int sa = kt % L::kASt, ua = kt / L::kASt;
      if (ok) ok = mbar_wait_bounded(&xfull[sx], (uint32_t)(ux & 1));
      if (ok && ua > 0) ok = mbar_wait_bounded(&aempty[sa], (uint32_t)((ua - 1) & 1));
      if (ok) {
        const uint8_t* xs = x_slot(sx);
        uint8_t* ah = a_slot(sa);
        uint8_t* al = ah + L::kA;
        // 128 rows x 8 chunks of 8 k; item i: row i >> 3, chunk i & 7
#pragma unroll 2
        for (int it = 0; it < 1024 / kSplitThreads; ++it) {
          const int i = t + kSplitThreads * it;
          const int r = i >> 3, c8 = i & 7, r7 = r & 7;
          // f32 source: box c8 >> 2 (k 0-31 / 32-63), 16-byte chunks 2 (c8 & 3)
          // and + 1 of row r, 128-byte swizzled
          const uint8_t* srow = xs + (c8 >> 2) * (L::kX / 2) + r * 128;
          const int cc = (c8 & 3) * 2;
          const float4 a = *reinterpret_cast<const float4*>(srow + ((cc ^ r7) << 4));
          const float4 b = *reinterpret_cast<const float4*>(srow + (((cc + 1) ^ r7) << 4));
          uint4 hi, lo;
          split_bf16x2(a.x, a.y, hi.x, lo.x);
          split_bf16x2(a.z, a.w, hi.y, lo.y);
          split_bf16x2(b.x, b.y, hi.z, lo.z);
          split_bf16x2(b.z, b.w, hi.w, lo.w);
          const int off = r * 128 + ((c8 ^ r7) << 4);
          *reinterpret_cast<uint4*>(ah + off) = hi;
          *reinterpret_cast<uint4*>(al + off) = lo;
        }
      }
      mbar_arrive(&xempty[sx]);  // after the reads above
      fence_proxy_async_smem();
      mbar_arrive(&afull[sa]);
    }
    role_ok = ok;
  } else if (warp >= 3 + kP32SplitWarps && warp < 7 + kP32SplitWarps) {
    // ------------------------------------------- dequantize: B = q - z
    constexpr int kWords = L::kWords;         // packed words per k row (16 / 32)
    constexpr int kRowsPer = kWords / 2;      // k rows per thread and stage (8 / 16)
    constexpr int kRowStep = 128 / kWords;    // between a thread's rows (8 / 4)
    const int t = threadIdx.x - 32 * (3 + kP32SplitWarps);  // 0..127
    const int w = t % kWords;                 // packed word of the row (8 columns)
    const int r0 = t / kWords;                // rows r0 + kRowStep i
    const int a = w >> 3, l = w & 7;          // 64-column atom, 16-byte chunk in it
    bool ok = true;
    for (int kt = 0; kt < KT; ++kt) {
      const int sw = kt % L::kWSt, uw = kt / L::kWSt;
      const int sb = kt % L::kBSt, ub = kt / L::kBSt;
      if (ok) ok = mbar_wait_bounded(&wfull[sw], (uint32_t)(uw & 1));
      if (ok && ub > 0) ok = mbar_wait_bounded(&bempty[sb], (uint32_t)((ub - 1) & 1));
      if (ok) {
        const uint8_t* ws = w_slot(sw);
        uint8_t* bs = b_slot(sb);
        uint32_t zp[4];
        pf_pairs<kBF16, ORDER>(reinterpret_cast<const uint32_t*>(ws + L::kW)[w], zp);
        uint32_t qv[kRowsPer];
#pragma unroll
        for (int i = 0; i < kRowsPer; ++i)
          qv[i] = reinterpret_cast<const uint32_t*>(ws)[(r0 + kRowStep * i) * kWords + w];
#pragma unroll
        for (int i = 0; i < kRowsPer; ++i) {
          const int r = r0 + kRowStep * i, r7 = r & 7;
          uint32_t tq[4];
          pf_pairs<kBF16, ORDER>(qv[i], tq);
          uint4 v;  // (128 + q) - (128 + z) = q - z, exact
          v.x = PfHalf2<kBF16>::sub(tq[0], zp[0]);
          v.y = PfHalf2<kBF16>::sub(tq[1], zp[1]);
          v.z = PfHalf2<kBF16>::sub(tq[2], zp[2]);
          v.w = PfHalf2<kBF16>::sub(tq[3], zp[3]);
          *reinterpret_cast<uint4*>(bs + a * 8192 + (r >> 3) * 1024 + r7 * 128 +
                                    ((l ^ r7) << 4)) = v;
        }
      }
      mbar_arrive(&wempty[sw]);  // after the values above were consumed
      fence_proxy_async_smem();
      mbar_arrive(&bfull[sb]);
    }
    role_ok = ok;
  } else {
    // ------------------------------------------------ group epilogue
    // kParts warps per TMEM lane quarter; warp part p takes columns
    // [kPartCols p, kPartCols (p + 1)) of every 128-column block, blocks in
    // order, so block 0's slot is free for the next group while block 1 is
    // being read
    const int lq = warp & 3;  // TMEM lane quarter this warp may access
    const int part = (warp - 7 - kP32SplitWarps) >> 2;  // 0 .. kParts - 1
    const uint32_t row_t = (uint32_t)(32 * lq);
    bool ok = true;
    for (int grp = 0; grp < NG; ++grp) {
      const int b = grp & 1;
      const bool last = grp == NG - 1;
      if (ok) ok = mbar_wait_bounded(&sfull[b], (uint32_t)((grp >> 1) & 1));
      for (int h = 0; h < NB; ++h) {
        const int use = grp * NB + h, slot = use & 1;
        if (ok) ok = mbar_wait_bounded(&dfull[slot], (uint32_t)((use >> 1) & 1));
        ok = __all_sync(0xffffffffu, ok);  // tcgen05.ld / st are warp-collective
        if (!ok) {
          mbar_arrive(&dempty[slot]);
          continue;
        }
        tc_fence_after();
        const int cb = 128 * h + kPartCols * part;  // first tile column of this warp
        const float* sc = s_slot(b) + cb;
        const uint32_t dbuf = tmem + (uint32_t)(slot * 128 + kPartCols * part) + (row_t << 16);
        const uint32_t run = tmem + 256 + (uint32_t)cb + (row_t << 16);
        // Chunks of kCW columns (two kCW-register arrays live at a time).
        // Per chunk one wait for both loads; the running-sum stores are
        // waited for once, at the group's end, and the slot is released to
        // the MMA as soon as its last chunk has been read.
        constexpr int kCW = p32_chunk_cols(BN);
#pragma unroll 1
        for (int c = 0; c < kPartCols / kCW; ++c) {
          float d[kCW], acc[kCW];
          tmem_ld_cols_nowait<kCW>(dbuf + kCW * c, d);
          if (grp > 0) tmem_ld_cols_nowait<kCW>(run + kCW * c, acc);
          asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
          if (c == kPartCols / kCW - 1) {
            tc_fence_before();
            mbar_arrive(&dempty[slot]);
          }
          if (grp == 0) {
#pragma unroll
            for (int i = 0; i < kCW; ++i) acc[i] = 0.f;
          }
#pragma unroll
          for (int i = 0; i < kCW; i += 4) {
            const float4 s4 = *reinterpret_cast<const float4*>(sc + kCW * c + i);
            acc[i] = fmaf(s4.x, d[i], acc[i]);
            acc[i + 1] = fmaf(s4.y, d[i + 1], acc[i + 1]);
            acc[i + 2] = fmaf(s4.z, d[i + 2], acc[i + 2]);
            acc[i + 3] = fmaf(s4.w, d[i + 3], acc[i + 3]);
          }
          if (!last) {
            tmem_st_cols_nowait<kCW>(run + kCW * c, acc);
          } else {
            const uint32_t row = m0 + row_t + lane, col0 = n0 + cb + kCW * c;
            if (row < rows && col0 < n) {
              if (bias) {
#pragma unroll
                for (int i = 0; i < kCW; ++i) acc[i] += bias[col0 + i];
              }
              // the chunk lies in one output (its boundaries are multiples of 32)
              float* o = om.at(row, col0);
              if ((reinterpret_cast<uintptr_t>(o) & 15) == 0) {
#pragma unroll
                for (int i = 0; i < kCW; i += 4)
                  *reinterpret_cast<float4*>(o + i) =
                      make_float4(acc[i], acc[i + 1], acc[i + 2], acc[i + 3]);
              } else {
#pragma unroll
                for (int i = 0; i < kCW; ++i) o[i] = acc[i];
              }
            }
          }
        }
      }
      // the running sums must be in place before the next group reads them
      if (ok) asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
      mbar_arrive(&sempty[b]);
    }
    role_ok = ok;
  }

  // No copy this CTA issued may still be writing its shared memory when it
  // exits: after a failed (timed-out) run, wait (bounded) for the last
  // stage issued into each ring slot.
  if (__syncthreads_or(role_ok ? 0 : 1) && threadIdx.x == 0) {
    const int xi = s_x_issued, wi = s_w_issued;
    for (int j = xi > L::kXSt ? xi - L::kXSt : 0; j < xi; ++j)
      mbar_wait_bounded(&xfull[j % L::kXSt], (uint32_t)((j / L::kXSt) & 1));
    for (int j = wi > L::kWSt ? wi - L::kWSt : 0; j < wi; ++j)
      mbar_wait_bounded(&wfull[j % L::kWSt], (uint32_t)((j / L::kWSt) & 1));
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

// ------------------------------------------------------------------ host
// plan.tile_n: 128 or 256 columns per CTA tile; 0 = 256 when those tiles
// alone fill the GPU (one tile per SM), else 128.
int prefill_f32_tile_n(const GemmProblem& p, const cawq_plan& plan, const DeviceInfo& dev) {
  if (plan.tile_n == 128 || plan.tile_n == 256) return plan.tile_n;
  const size_t sms = static_cast<size_t>(dev.sm_count > 0 ? dev.sm_count : 148);
  const size_t tiles256 = ((p.n + 255) / 256) * ((p.rows + kP32BM - 1) / kP32BM);
  return tiles256 >= sms ? 256 : 128;
}

bool prefill_f32_supports(const GemmProblem& p, const cawq_plan& plan, const DeviceInfo& dev) {
  if (plan.split > 1 || p.epi != 0 || p.nrep > 0) return false;
  if (plan.tile_n != 0 && plan.tile_n != 128 && plan.tile_n != 256) return false;
  if (p.dtype != kF32 || p.out_dtype != kF32) return false;
  const size_t need = prefill_f32_tile_n(p, plan, dev) == 256 ? P32Layout<256>::kSmem : P32Layout<128>::kSmem;
  if (dev.cc_major != 10 || dev.smem_optin < need) return false;
  if (p.rows == 0 || p.k % kP32BK != 0 || p.g % kP32BK != 0 || p.k % p.g != 0 || p.n % 32 != 0)
    return false;
  if (p.k >= (1ull << 31) || p.n >= (1ull << 31) || p.rows >= (1ull << 31) ||
      p.ld_out >= (1ull << 31))
    return false;
  if ((p.rows + kP32BM - 1) / kP32BM > 65535) return false;
  const uintptr_t ax = reinterpret_cast<uintptr_t>(p.x), aw = reinterpret_cast<uintptr_t>(p.qw);
  const uintptr_t az = reinterpret_cast<uintptr_t>(p.qz), as = reinterpret_cast<uintptr_t>(p.sc);
  return ax % 16 == 0 && aw % 16 == 0 && az % 16 == 0 && as % 16 == 0;
}

template <int ORDER, int BN>
static cudaError_t launch_prefill_f32_t(const GemmProblem& p, bool pdl) {
  using L = P32Layout<BN>;
  CUtensorMap tx, tw, ts, tz;
  const uint64_t npk = p.n / 8, groups = p.k / p.g;
  if (!pf_encode(&tx, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, p.x, p.k, p.rows, p.k * 4, 32, kP32BM,
                 CU_TENSOR_MAP_SWIZZLE_128B) ||
      !pf_encode(&tw, CU_TENSOR_MAP_DATA_TYPE_UINT32, p.qw, npk, p.k, npk * 4, BN / 8, kP32BK,
                 CU_TENSOR_MAP_SWIZZLE_NONE) ||
      !pf_encode(&ts, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, p.sc, p.n, groups, p.n * 4, BN, 1,
                 CU_TENSOR_MAP_SWIZZLE_NONE) ||
      !pf_encode(&tz, CU_TENSOR_MAP_DATA_TYPE_UINT32, p.qz, npk, groups, npk * 4, BN / 8, 1,
                 CU_TENSOR_MAP_SWIZZLE_NONE)) {
    return cudaErrorInvalidValue;
  }
  auto kern = prefill_f32_kernel<ORDER, BN>;
  static bool attr_set = false;  // per instantiation
  if (!attr_set) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         static_cast<int>(L::kSmem));
    if (e != cudaSuccess) return e;
    attr_set = true;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<uint32_t>((p.n + BN - 1) / BN),
                     static_cast<uint32_t>((p.rows + kP32BM - 1) / kP32BM), 1);
  cfg.blockDim = dim3(p32_threads(BN));
  cfg.dynamicSmemBytes = L::kSmem;
  cfg.stream = p.stream;
  cudaLaunchAttribute attr[1];
  int na = 0;
  if (pdl) {
    attr[na].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[na].val.programmaticStreamSerializationAllowed = 1;
    ++na;
  }
  cfg.attrs = attr;
  cfg.numAttrs = na;
  return cudaLaunchKernelEx(&cfg, kern, tx, tw, ts, tz, static_cast<const float*>(p.bias),
                            out_map<float>(p), static_cast<uint32_t>(p.rows),
                            static_cast<uint32_t>(p.k), static_cast<uint32_t>(p.n),
                            static_cast<uint32_t>(p.g));
}

cudaError_t launch_prefill_f32(const GemmProblem& p, const cawq_plan& plan, const DeviceInfo& dev) {
  const int bn = prefill_f32_tile_n(p, plan, dev);
  const size_t ctas = ((p.n + bn - 1) / bn) * ((p.rows + kP32BM - 1) / kP32BM);
  const size_t sms = static_cast<size_t>(dev.sm_count > 0 ? dev.sm_count : 148);
  const bool pdl = plan.reserved[0] == 0 && ctas <= sms;
  if (bn == 256)
    return p.order == kOrderNatural ? launch_prefill_f32_t<kOrderNatural, 256>(p, pdl)
                                    : launch_prefill_f32_t<kOrderAwq, 256>(p, pdl);
  return p.order == kOrderNatural ? launch_prefill_f32_t<kOrderNatural, 128>(p, pdl)
                                  : launch_prefill_f32_t<kOrderAwq, 128>(p, pdl);
}

}  // namespace cawq

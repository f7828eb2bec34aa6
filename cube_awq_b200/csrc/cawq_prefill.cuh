// cawq_prefill.cuh — large-M fused AWQ GEMM on tcgen05 tensor cores (sm_100a).
//
// Y[M, N] = X[M, K] · ((Q - Z) · S)[K, N] for f16 / bf16 activations.
// Replaces gemm_awq (src/kernel/awq_kernel_gemm.rs:181-439), the reference's
// M > 8 kernel, which computes on CUDA cores with scalar FMA.
//
// One CTA computes a 256 x 256 output tile as two 128-row halves that share
// every dequantized B stage (two M=128 MMAs per k step into two TMEM
// accumulators, all 512 columns): dequantizing, not the tensor core, is the
// cost of this kernel, and this spends it once per 256 rows. K advances in
// 64-row stages through three shared-memory rings:
//   X ring (3 x 32 KB)  X tile 256 x 64, 128B swizzle, K-major; loaded by TMA,
//                       freed by the MMA;
//   W ring (4 x 9 KB)   packed weight tile 64 x 32 words (128B swizzle) and
//                       the stage's scale and zero rows; loaded by TMA, freed
//                       by the dequantize warps once they have used it;
//   B ring (2 x 32 KB)  the dequantized B operand (MN-major, 128B swizzle);
//                       written by the dequantize warps, freed by the MMA.
// Warp roles (96 + 32 * kPfDqWarps threads):
//   warp 0     TMA producer of the X ring;
//   warp 1     allocates 512 TMEM columns; one thread issues
//              tcgen05.mma.cta_group::1.kind::f16 (M=128, N=256, K=16) x 8
//              per stage and commits each stage back to the X and B rings;
//   warp 2     TMA producer of the W ring;
//   warps 3.. dequantize the packed stage into the B operand: per packed
//              word, lop3 makes (1024 + q) f16 pairs of adjacent columns,
//              then (q - z) * s is formed in F exactly as the reference does
//              (one rounding), and 16 bytes land in the canonical MN-major
//              128B-swizzled layout. After the last stage they read the fp32
//              accumulator from TMEM (tcgen05.ld), add bias and store.
//
// The weights therefore enter the MMA bit-identical to the reference's
// dequantized values; the products are exact and the sum is fp32.
#pragma once

#include <mutex>

#include "cawq_common.cuh"

namespace cawq {

constexpr int kPfBN = 256;
constexpr int kPfBK = 64;
constexpr int kPfXStages = 3;
constexpr int kPfWStages = 4;
constexpr int kPfBStages = 2;
// dequant / epilogue warps: 16 for 128-row tiles (their stage has a quarter
// of the MMA work, so dequantization paces the loop), 8 for 256-row tiles
// (their registers would not fit 16)
__host__ __device__ constexpr int pf_dq_warps(int halves) { return halves == 1 ? 16 : 8; }
// 128-row tiles: the dequantize warps form two groups that take alternate
// k stages, so two stages are dequantized at once. A stage's wait / load /
// convert / store / fence / arrive chain is latency bound: with one group the
// stage cadence stayed the same whether 8 or 16 warps shared each stage.
__host__ __device__ constexpr int pf_dq_groups(int halves) { return halves == 1 ? 2 : 1; }
__host__ __device__ constexpr int pf_threads(int halves) {
  return 96 + 32 * pf_dq_warps(halves);  // + X producer, MMA, W producer
}
constexpr int kPfMaxSplit = 8;                      // CTAs of a cluster splitting K

// HALVES = 128-row MMA halves per CTA tile (1 or 2)
template <int HALVES>
struct PrefillLayout {
  static constexpr int kBM = 128 * HALVES;
  // ring depths: 128-row tiles stream more weight bytes per unit of MMA work,
  // so they keep more packed stages in flight and one more dequantized stage
  static constexpr int kXSt = kPfXStages;
  static constexpr int kWSt = HALVES == 1 ? 8 : kPfWStages;
  static constexpr int kBSt = HALVES == 1 ? 3 : kPfBStages;
  static constexpr int kX = kBM * kPfBK * 2;        // 16 KB per half
  static constexpr int kB = kPfBK * kPfBN * 2;      // 32768
  static constexpr int kW = kPfBK * kPfBN / 8 * 4;  // 8192
  static constexpr int kS = kPfBN * 2;              // 512
  static constexpr int kZ = kPfBN / 8 * 4;          // 128
  static constexpr int kWSlot = ((kW + kS + kZ) + 1023) / 1024 * 1024;
  static constexpr size_t kOffB = (size_t)kX * kXSt;
  static constexpr size_t kOffW = kOffB + (size_t)kB * kBSt;
  static constexpr size_t kOffBars = kOffW + (size_t)kWSlot * kWSt;
  static constexpr int kBars = 1024;  // barriers + TMEM slot
  static constexpr size_t kSmem = 1024 + kOffBars + kBars;
};

// ------------------------------------------------------- tcgen05 helpers
__device__ __forceinline__ uint64_t umma_desc_sw128(uint32_t saddr, uint32_t lbo, uint32_t sbo) {
  uint64_t d = 0;
  d |= (uint64_t)((saddr & 0x3FFFFu) >> 4);
  d |= (uint64_t)((lbo >> 4) & 0x3FFFu) << 16;
  d |= (uint64_t)((sbo >> 4) & 0x3FFFu) << 32;
  d |= 1ull << 46;  // descriptor version for sm_100
  d |= 2ull << 61;  // SWIZZLE_128B
  return d;
}

// kind::f16 instruction descriptor: fp32 accumulate, A K-major, B MN-major.
__host__ __device__ constexpr uint32_t umma_idesc_f16(bool bf16, int m, int n) {
  return (1u << 4) | ((bf16 ? 1u : 0u) << 7) | ((bf16 ? 1u : 0u) << 10) | (0u << 15) |
         (1u << 16) | ((uint32_t)(n >> 3) << 17) | ((uint32_t)(m >> 4) << 24);
}

__device__ __forceinline__ void umma_f16(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc,
                                         uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}"
      ::"r"(tmem_d), "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

__device__ __forceinline__ void umma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                   smem_u32(bar))
               : "memory");
}

__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

__device__ __forceinline__ void tmem_alloc(uint32_t* slot, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                   smem_u32(slot)),
               "r"(ncols)
               : "memory");
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
               : "memory");
}

// 32 lanes x 32 consecutive fp32 columns -> 32 registers per thread.
__device__ __forceinline__ void tmem_ld_32x32b_x32(uint32_t taddr, float (&v)[32]) {
  uint32_t r[32];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]),
        "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]),
        "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}

// EPI 1: gate / up columns interleaved in 128-column blocks, so each 256-column
// tile holds 128 gate columns and their 128 up columns; the epilogue writes
// silu(gate) * up (bias, if any, added to both first) to output columns
// [n0 / 2, n0 / 2 + 128) of an [rows, n / 2] output.
template <int DT, int ODT, int ORDER, int HALVES, int EPI = 0>
__global__ void __launch_bounds__(pf_threads(HALVES), 1)
    prefill_kernel(const __grid_constant__ CUtensorMap tm_x, const __grid_constant__ CUtensorMap tm_w,
                   const __grid_constant__ CUtensorMap tm_s, const __grid_constant__ CUtensorMap tm_z,
                   const typename DType<DT>::T* __restrict__ bias,
                   const OutMap<typename DType<ODT>::T> om, uint32_t rows, uint32_t k, uint32_t n,
                   uint32_t g, uint32_t split) {
  using L = PrefillLayout<HALVES>;
  constexpr int BM = L::kBM;
  constexpr int kPfDqWarps = pf_dq_warps(HALVES);
  constexpr int kDqGroups = pf_dq_groups(HALVES);
  constexpr int kGrpWarps = kPfDqWarps / kDqGroups;  // dequantize warps per stage
  constexpr int kPasses = 16 / kGrpWarps;            // 4-row sets per warp and stage
  constexpr uint32_t kTmemCols = HALVES * kPfBN;
  using H = PfHalf2<DT>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = smem_raw + ((1024 - (smem_u32(smem_raw) & 1023)) & 1023);
  uint64_t* full_x = reinterpret_cast<uint64_t*>(smem + L::kOffBars);
  uint64_t* empty_x = full_x + L::kXSt;
  uint64_t* full_w = empty_x + L::kXSt;
  uint64_t* empty_w = full_w + L::kWSt;
  uint64_t* bready = empty_w + L::kWSt;
  uint64_t* bempty = bready + L::kBSt;
  uint64_t* acc_full = bempty + L::kBSt;
  uint64_t* drain_bar = acc_full + 1;  // the MMA thread's own MMAs, on a failed run
  uint64_t* recv_bar = drain_bar + 1;  // split K: the peers' partial sums have landed
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(recv_bar + 1);
  __shared__ int s_x_issued, s_w_issued;  // stages each producer issued
  bool role_ok = true;

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t n0 = blockIdx.x * kPfBN;
  const uint32_t m0 = blockIdx.y * BM;
  // split K: the `split` CTAs of a cluster (along z) share one output tile;
  // CTA `rank` runs k-stages [kt0, kt0 + KTL)
  const uint32_t rank = split > 1 ? cluster_ctarank() : 0u;
  const int KT = static_cast<int>(k / kPfBK);
  const int kt0 = static_cast<int>((uint64_t)KT * rank / split);
  const int KTL = static_cast<int>((uint64_t)KT * (rank + 1) / split) - kt0;
  // Split K: the tile's valid rows are dealt out to the CTAs of the cluster,
  // rpo each (the last ones may get fewer or none); CTA q sums rows
  // [q rpo, q rpo + own_rows).
  // (128-row tiles). 256-row tiles: BM / split rows each, the CTA's own part
  // summed straight from TMEM (their receive buffer would not fit).
  const int vrows = min(BM, static_cast<int>(rows) - static_cast<int>(m0));
  const int rpo = HALVES == 1 ? (vrows + static_cast<int>(split) - 1) / static_cast<int>(split)
                              : BM / static_cast<int>(split);
  const int own_rows =
      HALVES == 1 ? max(0, min(rpo, vrows - static_cast<int>(rank) * rpo)) : rpo;

  auto x_slot = [&](int s) { return smem + (size_t)s * L::kX; };
  auto b_slot = [&](int s) { return smem + L::kOffB + (size_t)s * L::kB; };
  auto w_slot = [&](int s) { return smem + L::kOffW + (size_t)s * L::kWSlot; };

  if (threadIdx.x == 0) {
    for (int s = 0; s < L::kXSt; ++s) {
      mbar_init(&full_x[s], 1);
      mbar_init(&empty_x[s], 1);
    }
    for (int s = 0; s < L::kWSt; ++s) {
      mbar_init(&full_w[s], 1);
      mbar_init(&empty_w[s], 32 * kGrpWarps);
    }
    for (int s = 0; s < L::kBSt; ++s) {
      mbar_init(&bready[s], 32 * kGrpWarps);
      mbar_init(&bempty[s], 1);
    }
    mbar_init(acc_full, 1);
    mbar_init(drain_bar, 1);
    mbar_init(recv_bar, 1);
    if (split > 1) mbar_arrive_expect_tx(recv_bar, (split - 1) * own_rows * kPfBN * 4);
    fence_mbarrier_init();
    fence_proxy_async_smem();
    tma_prefetch_desc(&tm_x);
    tma_prefetch_desc(&tm_w);
  }
  if (warp == 1) tmem_alloc(tmem_slot, kTmemCols);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  // The next kernel of the stream may launch now and set itself up while
  // this one runs; it reads this kernel's output only after its own
  // griddepcontrol.wait, which waits for this whole grid.
  pdl_launch_dependents();

  if (warp == 0) {
    // ------------------------------------------------- X ring producer
    if (lane == 0) {
      bool ok = true;
      int issued = 0;
      // X may be the previous kernel's output: wait for that grid (the
      // weights, scales and zeros are loaded by warp 2 without waiting). The
      // epilogue's stores come after every X stage, so they also follow the
      // previous grid, which may still have been reading this output.
      pdl_wait();
      for (int i = 0; i < KTL && ok; ++i) {
        const int s = i % L::kXSt, u = i / L::kXSt;
        if (u > 0) ok = mbar_wait_bounded(&empty_x[s], (uint32_t)((u - 1) & 1));
        if (!ok) break;
        mbar_arrive_expect_tx(&full_x[s], L::kX);
        tma_load_2d(x_slot(s), &tm_x, (kt0 + i) * kPfBK, static_cast<int>(m0), &full_x[s]);
        issued = i + 1;
      }
      s_x_issued = issued;
      role_ok = ok;
    }
    __syncwarp();
  } else if (warp == 2) {
    // ------------------------------------------------- W ring producer
    if (lane == 0) {
      bool ok = true;
      int issued = 0;
      for (int i = 0; i < KTL && ok; ++i) {
        const int kt = kt0 + i;
        const int s = i % L::kWSt, u = i / L::kWSt;
        if (u > 0) ok = mbar_wait_bounded(&empty_w[s], (uint32_t)((u - 1) & 1));
        if (!ok) break;
        uint8_t* b = w_slot(s);
        const int grp = static_cast<int>((uint32_t)kt * kPfBK / g);
        mbar_arrive_expect_tx(&full_w[s], L::kW + L::kS + L::kZ);
        tma_load_2d(b, &tm_w, static_cast<int>(n0 / 8), kt * kPfBK, &full_w[s]);
        tma_load_2d(b + L::kW, &tm_s, static_cast<int>(n0), grp, &full_w[s]);
        tma_load_2d(b + L::kW + L::kS, &tm_z, static_cast<int>(n0 / 8), grp, &full_w[s]);
        issued = i + 1;
      }
      s_w_issued = issued;
      role_ok = ok;
    }
    __syncwarp();
  } else if (warp == 1) {
    // ------------------------------------------------------- MMA issuer
    if (lane == 0) {
      constexpr uint32_t idesc = umma_idesc_f16(DT == kBF16, 128, kPfBN);
      bool ok = true;
      for (int kt = 0; kt < KTL && ok; ++kt) {
        const int sx = kt % L::kXSt, ux = kt / L::kXSt;
        const int sb = kt % L::kBSt, ub = kt / L::kBSt;
        ok = mbar_wait_bounded(&full_x[sx], (uint32_t)(ux & 1)) &&
             mbar_wait_bounded(&bready[sb], (uint32_t)(ub & 1));
        if (!ok) break;
        tc_fence_after();
        const uint32_t xa = smem_u32(x_slot(sx));
        const uint32_t ba = smem_u32(b_slot(sb));
#pragma unroll
        for (int j = 0; j < kPfBK / 16; ++j) {
          const uint64_t bd = umma_desc_sw128(ba + 2048 * j, 8192, 1024);
#pragma unroll
          for (int h = 0; h < HALVES; ++h) {
            const uint64_t ad = umma_desc_sw128(xa + h * (L::kX / HALVES) + 32 * j, 16, 1024);
            umma_f16(tmem + h * kPfBN, ad, bd, idesc, (kt > 0 || j > 0) ? 1u : 0u);
          }
        }
        umma_commit(&empty_x[sx]);
        umma_commit(&bempty[sb]);
      }
      if (ok) {
        umma_commit(acc_full);
      } else {
        // wait (bounded) for the MMAs already issued before giving up
        umma_commit(drain_bar);
        mbar_wait_bounded(drain_bar, 0u);
      }
      role_ok = ok;
    }
    __syncwarp();
  } else {
    // ------------------------------------------- dequant, then epilogue
    const int dw = warp - 3;
    const int gw = dw % kGrpWarps;  // warp within its group
    const int q4 = lane >> 3;       // quarter of the warp -> row offset 2*q4
    const int l = lane & 7;         // packed word l + 8a, a = 0..3
    bool ok = true;
    for (int kt = dw / kGrpWarps; kt < KTL; kt += kDqGroups) {
      const int sw = kt % L::kWSt, uw = kt / L::kWSt;
      const int sb = kt % L::kBSt, ub = kt / L::kBSt;
      if (ok) ok = mbar_wait_bounded(&full_w[sw], (uint32_t)(uw & 1));
      if (ok && ub > 0) ok = mbar_wait_bounded(&bempty[sb], (uint32_t)((ub - 1) & 1));
      if (ok) {
        uint8_t* bsm = b_slot(sb);
        const uint8_t* wsm = w_slot(sw);
        const uint8_t* srow = wsm + L::kW;
        const uint32_t* zrow = reinterpret_cast<const uint32_t*>(srow + L::kS);
        uint32_t sp[4][4], zp[4][4];
#pragma unroll
        for (int a = 0; a < 4; ++a) {
          const int w = l + 8 * a;
          const uint4 sv = *reinterpret_cast<const uint4*>(srow + w * 16);
          sp[a][0] = sv.x; sp[a][1] = sv.y; sp[a][2] = sv.z; sp[a][3] = sv.w;
          pf_pairs<DT, ORDER>(zrow[w], zp[a]);
        }
        // 16 row sets of 4 rows (8-row atom x parity), dealt to the group
        uint32_t qv[kPasses][4];
#pragma unroll
        for (int pass = 0; pass < kPasses; ++pass) {
          const int sidx = kGrpWarps * pass + gw;
          const int row = (sidx >> 1) * 8 + (sidx & 1) + 2 * q4;  // 0..63
          const int r8 = row & 7;
#pragma unroll
          for (int a = 0; a < 4; ++a) {
            const int w = l + 8 * a;
            qv[pass][a] = *reinterpret_cast<const uint32_t*>(wsm + row * 128 +
                                                             (((w >> 2) ^ r8) << 4) + ((w & 3) << 2));
          }
        }
#pragma unroll
        for (int pass = 0; pass < kPasses; ++pass) {
          const int sidx = kGrpWarps * pass + gw;
          const int row = (sidx >> 1) * 8 + (sidx & 1) + 2 * q4;
          const int r8 = row & 7;
#pragma unroll
          for (int a = 0; a < 4; ++a) {
            uint32_t t[4];
            pf_pairs<DT, ORDER>(qv[pass][a], t);
            uint4 v;
            v.x = H::mul(H::sub(t[0], zp[a][0]), sp[a][0]);
            v.y = H::mul(H::sub(t[1], zp[a][1]), sp[a][1]);
            v.z = H::mul(H::sub(t[2], zp[a][2]), sp[a][2]);
            v.w = H::mul(H::sub(t[3], zp[a][3]), sp[a][3]);
            *reinterpret_cast<uint4*>(bsm + a * 8192 + (row >> 3) * 1024 + r8 * 128 +
                                      ((l ^ r8) << 4)) = v;
          }
        }
        // Only now may the producer refill the W slot: an mbarrier arrive
        // does not wait for shared-memory loads still in flight, so it must
        // follow the instructions that consume them (else the next TMA write
        // can overtake a read).
        mbar_arrive(&empty_w[sw]);
      } else {
        mbar_arrive(&empty_w[sw]);
      }
      fence_proxy_async_smem();
      mbar_arrive(&bready[sb]);
    }
    // ---- accumulators complete
    if (ok) ok = mbar_wait_bounded(acc_full, 0u);
    ok = __all_sync(0xffffffffu, ok);  // tcgen05.ld is warp-collective
    role_ok = ok;
    tc_fence_after();
  }

  // Split K: past this barrier every CTA of the cluster has finished its main
  // loop (MMAs complete), so its rings may receive the peers' partial sums.
  if (split > 1) {
    cluster_arrive_release();
    cluster_wait_acquire();
  }

  if (warp >= 3) {
    // ---- epilogue: TMEM -> registers (-> peers) -> global
    const int dw = warp - 3;
    const int lq = warp & 3;  // TMEM lane quarter this warp may access
    // the warps of one lane quarter split the 32-column chunks of the tile
    // (8 per 128-row half)
    constexpr int kChunks = HALVES * 8 / (kPfDqWarps / 4);
    const int part = dw >> 2;
    const bool ok = role_ok;
    auto store = [&](uint32_t row, uint32_t col0, float (&v)[32]) {
      if (row >= rows || col0 >= n) return;
      if (bias) {
#pragma unroll
        for (int i = 0; i < 32; ++i) v[i] += DType<DT>::to_f32(bias[col0 + i]);
      }
      typename DType<ODT>::T* o = om.at(row, col0);  // the chunk lies in one output
      constexpr bool kRep = EPI == 2;  // also store to the replicas
      if constexpr (ODT == kF32) {
        if ((reinterpret_cast<uintptr_t>(o) & 15) == 0) {
#pragma unroll
          for (int i = 0; i < 32; i += 4)
            om.template put<kRep>(o + i, make_float4(v[i], v[i + 1], v[i + 2], v[i + 3]));
        } else {
#pragma unroll
          for (int i = 0; i < 32; ++i) om.template put<kRep>(o + i, v[i]);
        }
      } else {
        using OT = typename DType<ODT>::T;
        if ((reinterpret_cast<uintptr_t>(o) & 15) == 0) {
#pragma unroll
          for (int i = 0; i < 32; i += 8) {
            uint4 pk;
            OT* hp = reinterpret_cast<OT*>(&pk);
#pragma unroll
            for (int e = 0; e < 8; ++e) hp[e] = DType<ODT>::from_f32(v[i + e]);
            om.template put<kRep>(o + i, pk);
          }
        } else {
#pragma unroll
          for (int i = 0; i < 32; ++i) om.template put<kRep>(o + i, DType<ODT>::from_f32(v[i]));
        }
      }
    };
    // EPI 1: weight columns gcol (gate) and gcol + 128 (up) of tile n0 ->
    // output column (n0 / 2) + (gcol - n0), written 32 at a time
    auto store_silu = [&](uint32_t row, uint32_t gcol, float (&v)[32], float (&u)[32]) {
      if (row >= rows || gcol >= n) return;
      const uint32_t ocol = n0 / 2 + (gcol - n0);
#pragma unroll
      for (int i = 0; i < 32; ++i) {
        float gv = v[i], uv = u[i];
        if (bias) {
          gv += DType<DT>::to_f32(bias[gcol + i]);
          uv += DType<DT>::to_f32(bias[gcol + 128 + i]);
        }
        v[i] = silu_mul(gv, uv);
      }
      using OT = typename DType<ODT>::T;
      OT* o = om.p0 + (size_t)row * om.ld0 + ocol;
      // 16-byte stores: a lane owns one row, so 2-byte stores would reach L2
      // as 16 partial writes of each 32-byte sector
      if ((reinterpret_cast<uintptr_t>(o) & 15) == 0) {
#pragma unroll
        for (int i = 0; i < 32; i += 8) {
          uint4 pk;
          OT* hp = reinterpret_cast<OT*>(&pk);
#pragma unroll
          for (int e = 0; e < 8; ++e) hp[e] = DType<ODT>::from_f32(v[i + e]);
          *reinterpret_cast<uint4*>(o + i) = pk;
        }
      } else {
#pragma unroll
        for (int i = 0; i < 32; ++i) o[i] = DType<ODT>::from_f32(v[i]);
      }
    };
    if (split == 1) {
      if (ok && EPI != 1) {
#pragma unroll 1
        for (int cc = part * kChunks; cc < (part + 1) * kChunks; ++cc) {
          const int h = cc >> 3, c = cc & 7;
          float v[32];
          tmem_ld_32x32b_x32(tmem + ((uint32_t)(32 * lq) << 16) + h * kPfBN + 32 * c, v);
          store(m0 + 128 * h + 32 * lq + lane, n0 + 32 * c, v);
        }
      } else if (ok) {
        // gate chunk c (columns 32c) with its up chunk (128 + 32c)
        constexpr int kGate = HALVES * 4 / (kPfDqWarps / 4);
#pragma unroll 1
        for (int gc = part * kGate; gc < (part + 1) * kGate; ++gc) {
          const int h = gc >> 2, c = gc & 3;
          float v[32], u[32];
          tmem_ld_32x32b_x32(tmem + ((uint32_t)(32 * lq) << 16) + h * kPfBN + 32 * c, v);
          tmem_ld_32x32b_x32(tmem + ((uint32_t)(32 * lq) << 16) + h * kPfBN + 128 + 32 * c, u);
          store_silu(m0 + 128 * h + 32 * lq + lane, n0 + 32 * c, v, u);
        }
      }
    } else {
      if constexpr (HALVES == 1) {
      // Every CTA writes each valid row of its partial sums into slot [its
      // rank] of the receive buffer [source][rpo rows][256 columns] of the
      // row's owner (st.async to distributed shared memory for the peers,
      // counted on their recv_bar; plain stores for its own rows), which
      // reuses the rings. A lane writes one row, so the 16-byte chunk c of
      // row r sits at c ^ (r & 7): the 8 rows of a store land in 8 different
      // bank groups. After the peers' bytes have landed and the epilogue
      // warps have met, all of them sum the owned rows over the slots in rank
      // order (deterministic) and store them.
      float* recv = reinterpret_cast<float*>(smem);
      const uint32_t bar_local = smem_u32(recv_bar);
      if (ok) {
#pragma unroll 1
        for (int cc = part * kChunks; cc < (part + 1) * kChunks; ++cc) {
          const int h = cc >> 3, c = cc & 7;
          const int r = 128 * h + 32 * lq + lane;  // tile row
          if (128 * h + 32 * lq >= vrows) continue;  // no valid row in this warp's quarter
          float v[32];
          tmem_ld_32x32b_x32(tmem + ((uint32_t)(32 * lq) << 16) + h * kPfBN + 32 * c, v);
          if (r >= vrows) continue;
          const uint32_t q = static_cast<uint32_t>(r / rpo);
          const int lr = r - (int)q * rpo;  // row inside the owner's slot
          float* dst = recv + ((size_t)rank * rpo + lr) * kPfBN + 32 * c;
          const int sw = lr & 7;
          if (q == rank) {
#pragma unroll
            for (int i = 0; i < 8; ++i)
              *reinterpret_cast<float4*>(dst + 4 * (i ^ sw)) =
                  make_float4(v[4 * i], v[4 * i + 1], v[4 * i + 2], v[4 * i + 3]);
          } else {
            const uint32_t ra = map_shared_rank(smem_u32(dst), q);
            const uint32_t rb = map_shared_rank(bar_local, q);
#pragma unroll
            for (int i = 0; i < 8; ++i)
              st_async_v4(ra + 16 * (i ^ sw), v[4 * i], v[4 * i + 1], v[4 * i + 2], v[4 * i + 3], rb);
          }
        }
      }
      const bool got = mbar_wait_bounded(recv_bar, 0u);
      named_bar_sync(1, 32 * kPfDqWarps);  // this CTA's own rows are in place
      if (ok && got && EPI == 1) {
        // owned rows x 32 gate column quads (each with its up quad)
        const int tid = threadIdx.x - 96;
        for (int idx = tid; idx < own_rows * (kPfBN / 8); idx += 32 * kPfDqWarps) {
          const int i = idx / (kPfBN / 8), c4 = idx - i * (kPfBN / 8);
          float4 ga = make_float4(0.f, 0.f, 0.f, 0.f), ua = ga;
          const int pg = c4 ^ (i & 7), pu = (c4 + 32) ^ (i & 7);
          for (uint32_t src = 0; src < split; ++src) {
            const float* rowp = recv + ((size_t)src * rpo + i) * kPfBN;
            const float4 f = *reinterpret_cast<const float4*>(rowp + 4 * pg);
            const float4 e = *reinterpret_cast<const float4*>(rowp + 4 * pu);
            ga.x += f.x; ga.y += f.y; ga.z += f.z; ga.w += f.w;
            ua.x += e.x; ua.y += e.y; ua.z += e.z; ua.w += e.w;
          }
          const uint32_t row = m0 + rank * rpo + i;
          const uint32_t gcol = n0 + 4 * c4;
          if (row < rows && gcol < n) {
            const float gv[4] = {ga.x, ga.y, ga.z, ga.w}, uv[4] = {ua.x, ua.y, ua.z, ua.w};
            typename DType<ODT>::T* o = om.p0 + (size_t)row * om.ld0 + n0 / 2 + 4 * c4;
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              float g1 = gv[e], u1 = uv[e];
              if (bias) {
                g1 += DType<DT>::to_f32(bias[gcol + e]);
                u1 += DType<DT>::to_f32(bias[gcol + 128 + e]);
              }
              o[e] = DType<ODT>::from_f32(silu_mul(g1, u1));
            }
          }
        }
      } else if (ok && got) {
        // owned rows x 64 column quads, spread over the epilogue threads
        const int tid = threadIdx.x - 96;
        for (int idx = tid; idx < own_rows * (kPfBN / 4); idx += 32 * kPfDqWarps) {
          const int i = idx / (kPfBN / 4), c4 = idx - i * (kPfBN / 4);
          float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
          const int pc4 = c4 ^ (i & 7);  // swizzled chunk of row i
          for (uint32_t src = 0; src < split; ++src) {
            const float4 f = *reinterpret_cast<const float4*>(
                recv + ((size_t)src * rpo + i) * kPfBN + 4 * pc4);
            acc.x += f.x; acc.y += f.y; acc.z += f.z; acc.w += f.w;
          }
          const uint32_t row = m0 + rank * rpo + i;
          const uint32_t col = n0 + 4 * c4;
          if (row < rows && col < n) {
            float v4[4] = {acc.x, acc.y, acc.z, acc.w};
            typename DType<ODT>::T* o = om.at(row, col);  // the quad lies in one output
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              if (col + e < n) {
                float vv = v4[e];
                if (bias) vv += DType<DT>::to_f32(bias[col + e]);
                om.template put<EPI == 2>(o + e, DType<ODT>::from_f32(vv));
              }
            }
          }
        }
      }
      } else {
      // CTA q owns tile rows [q rpo, (q+1) rpo). Each CTA sends the rows it
      // does not own to their owner (st.async into the owner's receive
      // buffer [source slot][row][256 columns], which reuses its rings;
      // counted on the owner's recv_bar), then sums its own rows over all
      // CTAs in rank order (its own part read again from TMEM).
      float* recv = reinterpret_cast<float*>(smem);
      const uint32_t bar_local = smem_u32(recv_bar);
      if (ok) {
#pragma unroll 1
        for (int cc = part * kChunks; cc < (part + 1) * kChunks; ++cc) {
          const int h = cc >> 3, c = cc & 7;
          const int r = 128 * h + 32 * lq + lane;  // tile row
          const uint32_t q = static_cast<uint32_t>(r / rpo);
          float v[32];
          tmem_ld_32x32b_x32(tmem + ((uint32_t)(32 * lq) << 16) + h * kPfBN + 32 * c, v);
          if (q != rank) {
            const uint32_t slot_idx = rank < q ? rank : rank - 1;
            const float* dst =
                recv + ((size_t)slot_idx * rpo + (r - (int)q * rpo)) * kPfBN + 32 * c;
            const uint32_t ra = map_shared_rank(smem_u32(dst), q);
            const uint32_t rb = map_shared_rank(bar_local, q);
#pragma unroll
            for (int i = 0; i < 32; i += 4) st_async_v4(ra + 4 * i, v[i], v[i + 1], v[i + 2], v[i + 3], rb);
          }
        }
      }
      const bool got = mbar_wait_bounded(recv_bar, 0u);
      if (ok && __all_sync(0xffffffffu, got)) {
#pragma unroll 1
        for (int cc = part * kChunks; cc < (part + 1) * kChunks; ++cc) {
          const int h = cc >> 3, c = cc & 7;
          const int r = 128 * h + 32 * lq + lane;
          float v[32];
          tmem_ld_32x32b_x32(tmem + ((uint32_t)(32 * lq) << 16) + h * kPfBN + 32 * c, v);
          if (static_cast<uint32_t>(r / rpo) != rank) continue;
          float acc[32];
#pragma unroll
          for (int i = 0; i < 32; ++i) acc[i] = 0.f;
          for (uint32_t src = 0; src < split; ++src) {
            if (src == rank) {
#pragma unroll
              for (int i = 0; i < 32; ++i) acc[i] += v[i];
            } else {
              const uint32_t slot_idx = src < rank ? src : src - 1;
              const float4* sp4 = reinterpret_cast<const float4*>(
                  recv + ((size_t)slot_idx * rpo + (r - (int)rank * rpo)) * kPfBN + 32 * c);
#pragma unroll
              for (int i = 0; i < 8; ++i) {
                const float4 f = sp4[i];
                acc[4 * i] += f.x;
                acc[4 * i + 1] += f.y;
                acc[4 * i + 2] += f.z;
                acc[4 * i + 3] += f.w;
              }
            }
          }
          store(m0 + r, n0 + 32 * c, acc);
        }
      }
      }
    }
  }
  // No copy this CTA issued may still be writing its shared memory when it
  // exits: after a failed (timed-out) run, wait (bounded) for the last
  // stage issued into each ring slot.
  if (__syncthreads_or(role_ok ? 0 : 1) && threadIdx.x == 0) {
    const int xi = s_x_issued, wi = s_w_issued;
    for (int j = xi > L::kXSt ? xi - L::kXSt : 0; j < xi; ++j)
      mbar_wait_bounded(&full_x[j % L::kXSt], (uint32_t)((j / L::kXSt) & 1));
    for (int j = wi > L::kWSt ? wi - L::kWSt : 0; j < wi; ++j)
      mbar_wait_bounded(&full_w[j % L::kWSt], (uint32_t)((j / L::kWSt) & 1));
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
}

// ------------------------------------------------------------------ host
static bool pf_encode(CUtensorMap* map, CUtensorMapDataType dt, const void* base, uint64_t inner,
                      uint64_t outer, uint64_t row_bytes, uint32_t box_inner, uint32_t box_outer,
                      CUtensorMapSwizzle swz) {
  return encode_tiled_2d(map, static_cast<int>(dt), base, inner, outer, row_bytes, box_inner,
                         box_outer, static_cast<int>(swz));
}

// plan.warps = 128-row MMA halves per tile (1 or 2), plan.split = CTAs of a
// cluster splitting K (1, 2, 4, 8; at most 4 with 2 halves, whose receive
// buffers would not fit the rings otherwise).
static int pf_halves(const cawq_plan& plan) { return plan.warps == 1 ? 1 : 2; }

static size_t pf_smem(int halves) {
  return halves == 1 ? PrefillLayout<1>::kSmem : PrefillLayout<2>::kSmem;
}

bool prefill_supports(const GemmProblem& p, const cawq_plan& plan, const DeviceInfo& dev) {
  if (p.dtype == kF32) {  // the f32 kernel (128 x 128 / 256 tiles), no split
    return (plan.warps == 0 || plan.warps == 1) && prefill_f32_supports(p, plan, dev);
  }
  if (plan.warps == 4) return prefill_tw_supports(p, plan, dev);
  const int halves = pf_halves(plan);
  if (plan.warps != 0 && plan.warps != 1 && plan.warps != 2) return false;
  const int split = plan.split < 1 ? 1 : plan.split;
  if (split > kPfMaxSplit || (split & (split - 1)) || (halves == 2 && split > 4)) return false;
  if (dev.cc_major != 10 || dev.smem_optin < pf_smem(halves)) return false;
  if (p.dtype != kF16 && p.dtype != kBF16) return false;
  if (p.rows == 0 || p.k % kPfBK != 0 || p.g % kPfBK != 0 || p.k % p.g != 0 || p.n % 32 != 0)
    return false;
  if ((size_t)split > p.k / kPfBK) return false;
  if (p.k >= (1ull << 31) || p.n >= (1ull << 31) || p.rows >= (1ull << 31) ||
      p.ld_out >= (1ull << 31))
    return false;
  if ((p.rows + 128 * halves - 1) / (128 * halves) > 65535) return false;
  // SiLU-gated epilogue: whole 256-column gate/up tiles, AWQ order, output in
  // the input dtype; 256-row tiles only without split K
  if (p.epi == 1 && (p.n % kPfBN != 0 || p.order != kOrderAwq || p.out_dtype != p.dtype ||
                     (halves == 2 && split > 1)))
    return false;
  // replicated output (tensor-parallel push): plain epilogue, one output
  // range, AWQ order
  if (p.nrep > 0 && (p.epi != 0 || p.out_k || p.order != kOrderAwq)) return false;
  const uintptr_t ax = reinterpret_cast<uintptr_t>(p.x), aw = reinterpret_cast<uintptr_t>(p.qw);
  const uintptr_t az = reinterpret_cast<uintptr_t>(p.qz), as = reinterpret_cast<uintptr_t>(p.sc);
  return ax % 16 == 0 && aw % 16 == 0 && az % 16 == 0 && as % 16 == 0;
}

template <int DT, int ODT, int ORDER, int HALVES, int EPI = 0>
static cudaError_t launch_prefill_t(const GemmProblem& p, int split, bool pdl) {
  using T = typename DType<DT>::T;
  using OT = typename DType<ODT>::T;
  using L = PrefillLayout<HALVES>;
  const CUtensorMapDataType xdt =
      DT == kF16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
  CUtensorMap tx, tw, ts, tz;
  const uint64_t npk = p.n / 8, groups = p.k / p.g;
  if (!pf_encode(&tx, xdt, p.x, p.k, p.rows, p.k * 2, kPfBK, L::kBM, CU_TENSOR_MAP_SWIZZLE_128B) ||
      !pf_encode(&tw, CU_TENSOR_MAP_DATA_TYPE_UINT32, p.qw, npk, p.k, npk * 4, kPfBN / 8, kPfBK,
                 CU_TENSOR_MAP_SWIZZLE_128B) ||
      !pf_encode(&ts, xdt, p.sc, p.n, groups, p.n * 2, kPfBN, 1, CU_TENSOR_MAP_SWIZZLE_NONE) ||
      !pf_encode(&tz, CU_TENSOR_MAP_DATA_TYPE_UINT32, p.qz, npk, groups, npk * 4, kPfBN / 8, 1,
                 CU_TENSOR_MAP_SWIZZLE_NONE)) {
    return cudaErrorInvalidValue;
  }
  auto kern = prefill_kernel<DT, ODT, ORDER, HALVES, EPI>;
  static bool attr_set = false;  // per instantiation
  if (!attr_set) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         static_cast<int>(L::kSmem));
    if (e != cudaSuccess) return e;
    attr_set = true;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<uint32_t>((p.n + kPfBN - 1) / kPfBN),
                     static_cast<uint32_t>((p.rows + L::kBM - 1) / L::kBM),
                     static_cast<uint32_t>(split));
  cfg.blockDim = dim3(pf_threads(L::kBM / 128));
  cfg.dynamicSmemBytes = L::kSmem;
  cfg.stream = p.stream;
  cudaLaunchAttribute attr[2];
  int na = 0;
  if (split > 1) {
    attr[na].id = cudaLaunchAttributeClusterDimension;
    attr[na].val.clusterDim.x = 1;
    attr[na].val.clusterDim.y = 1;
    attr[na].val.clusterDim.z = static_cast<unsigned>(split);
    ++na;
  }
  // programmatic dependent launch (plan.reserved[0] = 1 turns it off): the
  // prologue and the weight loads overlap the previous kernel's tail
  if (pdl) {
    attr[na].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[na].val.programmaticStreamSerializationAllowed = 1;
    ++na;
  }
  cfg.attrs = attr;
  cfg.numAttrs = na;
  return cudaLaunchKernelEx(&cfg, kern, tx, tw, ts, tz, static_cast<const T*>(p.bias),
                            out_map<OT>(p), static_cast<uint32_t>(p.rows),
                            static_cast<uint32_t>(p.k), static_cast<uint32_t>(p.n),
                            static_cast<uint32_t>(p.g), static_cast<uint32_t>(split));
}

template <int DT, int ODT>
static cudaError_t launch_prefill_o(const GemmProblem& p, int halves, int split, bool pdl) {
  if (p.nrep > 0) {  // EPI 2: plain epilogue, each store also to the replicas
    return halves == 1 ? launch_prefill_t<DT, ODT, kOrderAwq, 1, 2>(p, split, pdl)
                       : launch_prefill_t<DT, ODT, kOrderAwq, 2, 2>(p, split, pdl);
  }
  if constexpr (DT == ODT) {
    if (p.epi == 1) {
      return halves == 1 ? launch_prefill_t<DT, ODT, kOrderAwq, 1, 1>(p, split, pdl)
                         : launch_prefill_t<DT, ODT, kOrderAwq, 2, 1>(p, split, pdl);
    }
  }
  if (halves == 1) {
    return p.order == kOrderNatural ? launch_prefill_t<DT, ODT, kOrderNatural, 1>(p, split, pdl)
                                    : launch_prefill_t<DT, ODT, kOrderAwq, 1>(p, split, pdl);
  }
  return p.order == kOrderNatural ? launch_prefill_t<DT, ODT, kOrderNatural, 2>(p, split, pdl)
                                  : launch_prefill_t<DT, ODT, kOrderAwq, 2>(p, split, pdl);
}

cudaError_t launch_prefill(const GemmProblem& p, const cawq_plan& plan, const DeviceInfo& dev) {
  if (p.dtype == kF32) return launch_prefill_f32(p, plan, dev);
  if (plan.warps == 4) return launch_prefill_tw(p, plan, dev);
  const int halves = pf_halves(plan);
  const int split = plan.split < 1 ? 1 : plan.split;
  // Programmatic dependent launch for grids of one wave, whose ~14-26 us of
  // fixed cost per tile it partly hides (Qwen2-7B layer: M = 64 105 -> 98 us,
  // M = 256 164 -> 156 us); with several waves it hides little and measured
  // within noise, so those launch plainly.
  const size_t ctas = ((p.n + kPfBN - 1) / kPfBN) *
                      ((p.rows + 128 * (size_t)halves - 1) / (128 * (size_t)halves)) * split;
  const size_t sms = static_cast<size_t>(dev.sm_count > 0 ? dev.sm_count : 148);
  const bool pdl = plan.reserved[0] == 0 && ctas <= sms;
  if (p.dtype == kF16) {
    return p.out_dtype == kF32 ? launch_prefill_o<kF16, kF32>(p, halves, split, pdl)
                               : launch_prefill_o<kF16, kF16>(p, halves, split, pdl);
  }
  if (p.dtype == kBF16) {
    return p.out_dtype == kF32 ? launch_prefill_o<kBF16, kF32>(p, halves, split, pdl)
                               : launch_prefill_o<kBF16, kBF16>(p, halves, split, pdl);
  }
  return cudaErrorNotSupported;
}

// Clusters of `split` CTAs (one per SM: the tile's shared memory) that can be
// resident at once on the current device, from the occupancy calculator;
// cached per (device, tile height, split). 0 if the query fails.
template <int HALVES>
static int pf_max_active_clusters(int device, int split) {
  static std::mutex mu;
  static int cache[64][4] = {};  // [device][log2 split - 1], 0 = not yet asked
  int lg = 0;
  while ((2 << lg) < split) ++lg;
  if (device < 0 || device >= 64 || lg > 3) return 0;
  std::lock_guard<std::mutex> lk(mu);
  if (cache[device][lg] != 0) return cache[device][lg] > 0 ? cache[device][lg] : 0;
  using L = PrefillLayout<HALVES>;
  auto kern = prefill_kernel<kF16, kF16, kOrderAwq, HALVES>;
  int n = 0;
  if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           static_cast<int>(L::kSmem)) == cudaSuccess) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(1, 1, static_cast<unsigned>(split));
    cfg.blockDim = dim3(pf_threads(HALVES));
    cfg.dynamicSmemBytes = L::kSmem;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 1;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = static_cast<unsigned>(split);
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    if (cudaOccupancyMaxActiveClusters(&n, kern, &cfg) != cudaSuccess) {
      (void)cudaGetLastError();
      n = 0;
    }
  } else {
    (void)cudaGetLastError();
  }
  cache[device][lg] = n > 0 ? n : -1;
  return n;
}

// One 128-row half up to 128 rows, else two; split K over a cluster while the
// tiles alone would leave more than half of the SMs idle.
cawq_plan prefill_default_plan(const GemmProblem& p, const DeviceInfo& dev) {
  cawq_plan pl = {};
  pl.path = CAWQ_PATH_PREFILL;
  pl.tile_n = kPfBN;
  pl.stages = kPfBStages;
  pl.warps = p.rows <= 128 ? 1 : 2;
  if (p.dtype == kF32) {  // the f32 kernel: 128 x 128 or 128 x 256 tiles, no split
    pl.warps = 1;
    pl.split = 1;
    pl.tile_n = 0;
    pl.tile_n = prefill_f32_tile_n(p, pl, dev);
    return pl;
  }
  const size_t sms = static_cast<size_t>(dev.sm_count > 0 ? dev.sm_count : 148);
  const size_t kt = p.k / kPfBK;
  auto split_for = [&](int warps) {
    const size_t bm = 128 * (size_t)warps;
    const size_t tiles = ((p.n + kPfBN - 1) / kPfBN) * ((p.rows + bm - 1) / bm);
    const int max_split = warps == 1 ? kPfMaxSplit : 4;
    int split = 1;
    while (split < max_split && tiles * split * 2 <= sms && kt >= (size_t)split * 2 * 4) split *= 2;
    // all clusters in one wave: a cluster needs `split` SMs of one GPC at
    // once, and a tile count above what fits leaves the last clusters for a
    // second wave (measured: Qwen2 qkv at M = 64, 18 clusters of 8 -> 24 us,
    // of 4 -> 17 us)
    while (split > 1) {
      const int act = warps == 1 ? pf_max_active_clusters<1>(dev.device, split)
                                 : pf_max_active_clusters<2>(dev.device, split);
      if (act <= 0 || tiles <= (size_t)act) break;
      split /= 2;
    }
    return split;
  };
  if (p.rows > 128) {
    // 256-row tiles (two MMA halves sharing each dequantized stage) or
    // 128-row tiles with more split K, whichever a cost model measured on
    // B200 puts first (Qwen2-7B and Llama-2-7B linears at M = 192-512, every
    // tile height and split): a launch takes waves x (fixed + 0.53 us per
    // 64-row stage of the CTA's K share), the fixed part ~26 us for 256-row
    // tiles (8 dequant / epilogue warps for twice the rows) and ~14 us for
    // 128-row tiles, plus ~4 us for the 256-row tile's split-K hand-off. The
    // model picked the measured best, or one within a few percent, in every
    // case swept; at large M the 256-row tiles always win (the fixed part is
    // paid by half as many tiles).
    const size_t ntiles = (p.n + kPfBN - 1) / kPfBN;
    double best = 1e300;
    int best_w = 2, best_s = 1;
    for (int warps : {2, 1}) {
      for (int sp : {1, 2, 4, 8}) {
        if (warps == 2 && sp > 4) continue;
        if (sp > 1 && kt < (size_t)sp * 8) continue;
        if (p.epi == 1 && warps == 2 && sp > 1) continue;
        const size_t tiles = ntiles * ((p.rows + 128 * (size_t)warps - 1) / (128 * (size_t)warps));
        const int act = sp == 1 ? static_cast<int>(sms)
                                : (warps == 1 ? pf_max_active_clusters<1>(dev.device, sp)
                                              : pf_max_active_clusters<2>(dev.device, sp));
        if (act <= 0) continue;
        const size_t waves = (tiles + act - 1) / act;
        const size_t stages = (kt + sp - 1) / sp;
        const double t = waves * ((warps == 2 ? 26.0 : 14.0) + 0.53 * stages) +
                         (warps == 2 && sp > 1 ? 4.0 : 0.0);
        if (t < best) {
          best = t;
          best_w = warps;
          best_s = sp;
        }
      }
    }
    pl.warps = best_w;
    pl.split = best_s;
    return pl;
  }
  int split = split_for(pl.warps);
  if (p.epi == 1 && pl.warps == 2 && split > 1) {
    // the 256-row tile's split-K hand-off has no SiLU epilogue: 128-row
    // tiles with their own split instead
    pl.warps = 1;
    split = split_for(1);
  }
  pl.split = split;
  return pl;
}

void prefill_candidates(const GemmProblem& p, const DeviceInfo& dev, cawq_plan* out, int* count,
                        int max_count) {
  int c = 0;
  if (p.dtype == kF32) {
    for (int tn : {128, 256}) {
      cawq_plan pl = {};
      pl.path = CAWQ_PATH_PREFILL;
      pl.tile_n = tn;
      pl.stages = kPfBStages;
      pl.warps = 1;
      pl.split = 1;
      if (prefill_supports(p, pl, dev) && c < max_count) out[c++] = pl;
    }
    *count = c;
    return;
  }
  for (int halves : {1, 2}) {
    for (int split : {1, 2, 4, 8}) {
      cawq_plan pl = {};
      pl.path = CAWQ_PATH_PREFILL;
      pl.tile_n = kPfBN;
      pl.stages = kPfBStages;
      pl.warps = halves;
      pl.split = split;
      if (prefill_supports(p, pl, dev) && c < max_count) out[c++] = pl;
    }
  }
  // the weights-in-tensor-memory tile (rows <= 128): 256 / 512 columns
  for (int tn : {256, 512}) {
    for (int split : {1, 2, 4, 8}) {
      cawq_plan pl = {};
      pl.path = CAWQ_PATH_PREFILL;
      pl.warps = 4;
      pl.tile_n = tn;
      pl.split = split;
      if (prefill_supports(p, pl, dev) && c < max_count) out[c++] = pl;
    }
  }
  *count = c;
}

}  // namespace cawq

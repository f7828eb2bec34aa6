// cawq_prefill_tw.cuh — mid-M fused AWQ GEMM with the dequantized weights as
// the tcgen05 A operand in tensor memory (sm_100a).
//
// Y[M, N] = X[M, K] · ((Q - Z) · S)[K, N] for f16 / bf16 activations and
// M <= 128, the range between the decode kernel (M <= 16) and the prefill
// kernel's 128 / 256-row X tiles. Like the prefill kernel it replaces the
// reference's gemm_awq (src/kernel/awq_kernel_gemm.rs:181-439) and
// dequantizes exactly as the reference does ((q - z) * s rounded once to F).
//
// The product is computed transposed, D[n][m] = sum_k W[k][n] X[m][k]: one
// UMMA has M = 128 weight columns and N = M' rows of X (M rounded up to 16).
// The weights, the large operand, go from the dequantize warps' registers
// straight into tensor memory (tcgen05.st) and the MMA reads them from there
// (A operand in TMEM); only the packed weights (half a byte per weight) and
// the X tile pass through shared memory. The prefill kernel writes every
// dequantized 16-bit B tile to shared memory and the MMA reads it back, four
// bytes of shared-memory traffic per weight on top of the packed load, which
// at M <= 128 kept its stages well below the weight-streaming rate.
//
// CTA: NB 128-column blocks of weight columns (NB = 2: 256 columns, NB = 4:
// 512 columns for M <= 64), every row of X, and a K slice (split K over a
// cluster of up to 8 CTAs along z). A CTA streams its packed weights at about
// one 64-row TMA box per 0.45 us whatever the box's width (measured on B200:
// 16 GB/s with one 128-byte row per k, 33 / 58 GB/s with two / four boxes side
// by side), so with one CTA per SM the weight stream per SM grows with the
// columns a CTA covers: NB = 4 loads two 128-byte boxes side by side per
// k row. Rings:
//   X (4 x M' x 128 B, 64 k per stage, TMA, 128-byte swizzle, K-major): the B
//     operand, freed by the MMA;
//   W (plan.stages x 9-10 KB, TMA): 128 / NB k rows x NB / 2 packed weight
//     boxes of 32 words (128-byte swizzle), the stage's scale and zero rows;
//     freed by the dequantize warps;
//   A (4 x 64 TMEM columns): the dequantized weights of a W stage, NB blocks
//     of 64 / NB columns (128 / NB k as 16-bit pairs) x 128 lanes, freed by
//     the MMA.
// TMEM: the accumulators D (NB x M' fp32 columns) from column 0, the A ring
// from column 256 (512 columns, one CTA per SM).
// Warps: 0 X producer, 1 TMEM allocation + MMA issue, 2 W producer, 3..18
// dequantize, then run the epilogue. Warp w may only touch TMEM lanes
// 32 (w % 4) .. + 31, so the 16 dequantize warps are four per lane quarter:
// block b = j % NB of stages kt = j / NB (mod 4 / NB) (j = (w - 3) / 4).
//
// Dequantize. ldmatrix.x4.trans gives a lane, per register, one 16-bit
// element (4 nibbles = 4 weight columns) of two consecutive k rows. The
// matrices' row addresses are k = 16 jb + 4 (r >> 1) + 2 h + (r & 1) (h =
// matrix parity), so lane t (e = t >> 2, p = t & 3) holds the k pair
// (16 jb + 4p + 2h, +1): column 8 jb + 2p + h of an A block, which is where
// tcgen05.st.16x256b puts that lane's registers. Nibble c of element e goes
// to lane 8c + e of the warp's quarter (two stores, lane bases 0 and 16), so
// TMEM lane l of quarter q of block b holds weight column
//   n = 128 b + 32 q + 8 ((l & 7) >> 1) + col_of_nibble(4 (l & 1) + (l >> 3))
// (e = l & 7, c = l >> 3). Per pair: one lop3 (m + q[k], m + q[k + 1]), one
// packed subtract of (m + z) and one packed multiply by s: (q - z) * s
// rounded once in F, the reference's dequantized weight; the sum is fp32.
//
// Split K: after a cluster barrier every CTA reads its accumulators in
// 16-column chunks and sends each group of 4 X rows to that group's owner
// (rows are dealt out in runs of rpo, a multiple of 4), into the owner's
// receive buffer recv[source][block][lane][rpo] fp32 (st.async, 16 bytes,
// counted on the owner's mbarrier; plain stores for its own rows). The
// owner sums the slots in rank order (deterministic), adds the bias and
// stores.
//
// Every wait is bounded (2 s); on a timeout the kernel sets bit 0 of the
// device error word, stops issuing, waits (bounded) for what it issued,
// frees its TMEM and returns.
#pragma once

#include "cawq_common.cuh"

namespace cawq {

constexpr int kTwXK = 64;       // k rows per X stage
constexpr int kTwXSt = 4;       // X stages
constexpr int kTwWStMax = 16;   // packed W stages (plan.stages; 6 by default)
constexpr int kTwWStDefault = 6;
constexpr int kTwASt = 4;       // dequantized A stages in TMEM
constexpr int kTwDqWarps = 16;  // dequantize / epilogue warps
constexpr int kTwThreads = 96 + 32 * kTwDqWarps;
constexpr int kTwMaxSplit = 8;
constexpr int kTwACol = 256;  // first TMEM column of the A ring

template <int NB>
struct TwLayout {
  static constexpr int kBN = 128 * NB;              // weight columns per CTA
  static constexpr int kKA = 128 / NB;              // k rows per W / A stage
  static constexpr int kMaxRows = 256 / NB;         // D: NB x M' <= 256 columns
  static constexpr int kW = kKA * kBN / 8 * 4;      // 8192
  static constexpr int kS = kBN * 2;
  static constexpr int kZ = kBN / 8 * 4;
  static constexpr int kWSlot = ((kW + kS + kZ) + 1023) / 1024 * 1024;
  // X rows of the MMA (M rounded up to 16)
  static __host__ __device__ uint32_t nx(uint32_t rows) { return (rows + 15) / 16 * 16; }
  // rows each CTA of a split-K cluster owns: a multiple of 4
  static __host__ __device__ uint32_t rpo(uint32_t rows, uint32_t split) {
    return ((rows + split - 1) / split + 3) / 4 * 4;
  }
  static __host__ __device__ size_t x_bytes(uint32_t nx) { return (size_t)nx * kTwXK * 2; }
  static __host__ __device__ size_t off_w(uint32_t nx) { return x_bytes(nx) * kTwXSt; }
  static __host__ __device__ size_t ring_bytes(uint32_t nx, uint32_t nw) {
    return off_w(nx) + (size_t)kWSlot * nw;
  }
  static __host__ __device__ size_t recv_bytes(uint32_t rows, uint32_t split) {
    return split > 1 ? (size_t)split * NB * 128 * rpo(rows, split) * 4 : 0;
  }
  static __host__ __device__ size_t off_bars(uint32_t rows, uint32_t split, uint32_t nw) {
    const size_t a = ring_bytes(nx(rows), nw), b = recv_bytes(rows, split);
    return ((a > b ? a : b) + 15) / 16 * 16;
  }
  static constexpr int kBars = 512;  // mbarriers + TMEM slot
  static __host__ __device__ size_t smem(uint32_t rows, uint32_t split, uint32_t nw) {
    return 1024 + off_bars(rows, split, nw) + kBars;
  }
};

// kind::f16 instruction descriptor with both operands K-major (A in TMEM,
// B = X rows in shared memory), fp32 accumulate.
__host__ __device__ constexpr uint32_t tw_idesc(bool bf16, uint32_t n) {
  return (1u << 4) | ((bf16 ? 1u : 0u) << 7) | ((bf16 ? 1u : 0u) << 10) | ((n >> 3) << 17) |
         ((128u >> 4) << 24);
}

// D[tmem_d] (+)= A[tmem_a] · B[bdesc]: A from tensor memory.
__device__ __forceinline__ void umma_f16_tmem_a(uint32_t tmem_d, uint32_t tmem_a, uint64_t bdesc,
                                                uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}"
      ::"r"(tmem_d), "r"(tmem_a), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// 16 lanes x 256 bits, four times along the columns: lane t holds, per
// repetition j, (lane t/4, column 8j + 2(t%4)), (same lane, + 1),
// (lane t/4 + 8, column 8j + 2(t%4)), (same lane, + 1).
__device__ __forceinline__ void tmem_st_16x256b_x4(uint32_t taddr, const uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.16x256b.x4.b32 [%0], "
      "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]),
      "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]),
      "r"(r[15])
      : "memory");
}

__device__ __forceinline__ void tmem_st_16x256b_x2(uint32_t taddr, const uint32_t (&r)[8]) {
  asm volatile("tcgen05.st.sync.aligned.16x256b.x2.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8};" ::"r"(taddr),
               "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7])
               : "memory");
}

__device__ __forceinline__ void tmem_wait_st() {
  asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}

// 32 lanes x 16 consecutive fp32 columns -> 16 registers per thread.
__device__ __forceinline__ void tmem_ld_32x32b_x16(uint32_t taddr, float (&v)[16]) {
  uint32_t r[16];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}

// Weight column (inside the CTA's 256) held by TMEM lane `lane` (0..31) of
// quarter q of block b.
template <int ORDER>
__device__ __forceinline__ uint32_t tw_col_of_lane(int b, int q, int lane) {
  const int e = lane & 7, c = lane >> 3;
  return static_cast<uint32_t>(128 * b + 32 * q + 8 * (e >> 1) +
                               col_of_nibble(4 * (e & 1) + c, ORDER));
}

template <int DT, int ODT, int ORDER, int NB>
__global__ void __launch_bounds__(kTwThreads, 1)
    prefill_tw_kernel(const __grid_constant__ CUtensorMap tm_x,
                      const __grid_constant__ CUtensorMap tm_w,
                      const __grid_constant__ CUtensorMap tm_s,
                      const __grid_constant__ CUtensorMap tm_z,
                      const typename DType<DT>::T* __restrict__ bias,
                      const OutMap<typename DType<ODT>::T> om, uint32_t rows, uint32_t k,
                      uint32_t n, uint32_t g, uint32_t split, uint32_t nw) {
  using L = TwLayout<NB>;
  using H = PfHalf2<DT>;
  constexpr int KA = L::kKA;        // k rows per W / A stage
  constexpr int NJB = KA / 16;      // 16-k MMA steps per stage
  constexpr int XPS = kTwXK / KA;   // W / A stages per X stage
  constexpr int G = 4 / NB;         // dequantize groups (stages in flight)
  constexpr uint32_t kTmemCols = 512;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = smem_raw + ((1024 - (smem_u32(smem_raw) & 1023)) & 1023);
  const uint32_t NX = L::nx(rows);
  const int NW = static_cast<int>(nw);  // W ring depth
  uint64_t* full_x = reinterpret_cast<uint64_t*>(smem + L::off_bars(rows, split, nw));
  uint64_t* empty_x = full_x + kTwXSt;
  uint64_t* full_w = empty_x + kTwXSt;
  uint64_t* empty_w = full_w + kTwWStMax;
  uint64_t* afull = empty_w + kTwWStMax;
  uint64_t* aempty = afull + kTwASt;
  uint64_t* acc_full = aempty + kTwASt;
  uint64_t* drain_bar = acc_full + 1;
  uint64_t* recv_bar = drain_bar + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(recv_bar + 1);
  __shared__ int s_x_issued, s_w_issued;
  bool role_ok = true;

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t n0 = blockIdx.x * L::kBN;
  const uint32_t rank = split > 1 ? cluster_ctarank() : 0u;
  // K is dealt out to the CTAs of a cluster in whole X stages (64 k)
  const int XT = static_cast<int>(k / kTwXK);
  const int xt0 = static_cast<int>((uint64_t)XT * rank / split);
  const int XTL = static_cast<int>((uint64_t)XT * (rank + 1) / split) - xt0;
  const int kt0 = xt0 * XPS, KTL = XTL * XPS;  // W / A stages
  // split K: rows [q rpo, q rpo + rpo) belong to CTA q; groups of 4 rows
  // below round_up(rows, 4) travel
  const uint32_t rpo = L::rpo(rows, split);
  const uint32_t rows4 = (rows + 3) / 4 * 4;
  const uint32_t own_lo = rank * rpo;
  const uint32_t own4 = own_lo < rows4 ? min(rpo, rows4 - own_lo) : 0u;

  auto x_slot = [&](int s) { return smem + (size_t)s * L::x_bytes(NX); };
  auto w_slot = [&](int s) { return smem + L::off_w(NX) + (size_t)s * L::kWSlot; };

  if (threadIdx.x == 0) {
    for (int s = 0; s < kTwXSt; ++s) {
      mbar_init(&full_x[s], 1);
      mbar_init(&empty_x[s], 1);
    }
    for (int s = 0; s < NW; ++s) {
      mbar_init(&full_w[s], 1);
      mbar_init(&empty_w[s], 4 * NB * 32);  // the warps of the stage's group
    }
    for (int s = 0; s < kTwASt; ++s) {
      mbar_init(&afull[s], 4 * NB * 32);
      mbar_init(&aempty[s], 1);
    }
    mbar_init(acc_full, 1);
    mbar_init(drain_bar, 1);
    mbar_init(recv_bar, 1);
    if (split > 1) mbar_arrive_expect_tx(recv_bar, (split - 1) * (uint32_t)NB * 128u * own4 * 4u);
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
  // The next kernel of the stream may launch now; it reads this kernel's
  // output only after its own griddepcontrol.wait (this whole grid).
  pdl_launch_dependents();

  if (warp == 0) {
    // ------------------------------------------------- X ring producer
    if (lane == 0) {
      bool ok = true;
      int issued = 0;
      // X may be the previous kernel's output; the epilogue's stores follow
      // every X stage, so they also wait for the previous grid.
      pdl_wait();
      const uint32_t xb = static_cast<uint32_t>(L::x_bytes(NX));
      for (int i = 0; i < XTL && ok; ++i) {
        const int s = i % kTwXSt, u = i / kTwXSt;
        if (u > 0) ok = mbar_wait_bounded(&empty_x[s], (uint32_t)((u - 1) & 1));
        if (!ok) break;
        mbar_arrive_expect_tx(&full_x[s], xb);
        tma_load_2d(x_slot(s), &tm_x, (xt0 + i) * kTwXK, 0, &full_x[s]);
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
        const int s = i % NW, u = i / NW;
        if (u > 0) ok = mbar_wait_bounded(&empty_w[s], (uint32_t)((u - 1) & 1));
        if (!ok) break;
        uint8_t* b = w_slot(s);
        const int grp = static_cast<int>((uint32_t)kt * KA / g);
        mbar_arrive_expect_tx(&full_w[s], L::kW + L::kS + L::kZ);
        // NB / 2 boxes of 32 words side by side: one 64-row box costs the
        // same time whatever its width, so wider k rows stream faster
#pragma unroll
        for (int h = 0; h < NB / 2; ++h) {
          tma_load_2d(b + h * (KA * 128), &tm_w, static_cast<int>(n0 / 8 + 32 * h), kt * KA,
                      &full_w[s]);
          tma_load_2d(b + L::kW + h * 512, &tm_s, static_cast<int>(n0 + 256 * h), grp, &full_w[s]);
        }
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
      const uint32_t idesc = tw_idesc(DT == kBF16, NX);
      bool ok = true;
      int sx = 0, sa = 0, sub = 0;
      uint32_t px = 0, pa = 0;  // phase parities of the X and A slots
      for (int kt = 0; kt < KTL && ok; ++kt) {
        if (sub == 0) ok = mbar_wait_bounded(&full_x[sx], px);
        ok = ok && mbar_wait_bounded(&afull[sa], pa);
        if (!ok) break;
        tc_fence_after();
        const uint32_t xa = smem_u32(x_slot(sx)) + 2 * KA * sub;  // this stage's k in the X row
#pragma unroll
        for (int j = 0; j < NJB; ++j) {
          const uint64_t bd = umma_desc_sw128(xa + 32 * j, 16, 1024);
#pragma unroll
          for (int b = 0; b < NB; ++b) {
            umma_f16_tmem_a(tmem + b * NX, tmem + kTwACol + 64 * sa + (KA / 2) * b + 8 * j, bd,
                            idesc, (kt > 0 || j > 0) ? 1u : 0u);
          }
        }
        umma_commit(&aempty[sa]);
        if (++sa == kTwASt) { sa = 0; pa ^= 1u; }
        if (++sub == XPS) {
          umma_commit(&empty_x[sx]);
          sub = 0;
          if (++sx == kTwXSt) { sx = 0; px ^= 1u; }
        }
      }
      if (ok) {
        umma_commit(acc_full);
      } else {
        umma_commit(drain_bar);
        mbar_wait_bounded(drain_bar, 0u);
      }
      role_ok = ok;
    }
    __syncwarp();
  } else {
    // ----------------------------------------------------- dequantize
    const int dw = warp - 3;
    const int q = warp & 3;        // TMEM lane quarter of this warp
    const int jq = dw >> 2;        // 0..3 among the quarter's warps
    const int blk = jq % NB;       // 128-column block
    const int gi = jq / NB;        // group: stages kt = gi (mod G)
    const int ch = 4 * blk + q;    // 16-byte chunk of the k row: 32 weight columns
    const int e = lane >> 2;
    const int wi = 4 * ch + (e >> 1);  // packed word of this lane's 4 columns
    int ncol[4];
#pragma unroll
    for (int c = 0; c < 4; ++c) ncol[c] = 8 * wi + col_of_nibble(4 * (e & 1) + c, ORDER);
    // ldmatrix row address offsets: lane L supplies row r of matrix mi; the
    // chunk lies in box ch / 8 at position ch % 8 of its 128-byte rows
    uint32_t ldoff[NJB / 2];
    {
      const int mi = lane >> 3, r = lane & 7;
      const int bx = ch >> 3, cx = ch & 7;
#pragma unroll
      for (int x = 0; x < NJB / 2; ++x) {
        const int kk = 16 * (2 * x + (mi >> 1)) + 4 * (r >> 1) + 2 * (mi & 1) + (r & 1);
        ldoff[x] = static_cast<uint32_t>(bx * (KA * 128) + kk * 128 + ((cx ^ (kk & 7)) << 4));
      }
    }
    const uint32_t lane_base = static_cast<uint32_t>(32 * q) << 16;
    bool ok = true;
    // this group's W and A slots and phase parities, advanced by G per stage
    int sw = gi % NW, sa = gi % kTwASt;
    uint32_t pw = 0, pa = 0;
    bool first_use = true;  // an A slot's first use needs no wait for the MMA
    for (int kt = gi; kt < KTL; kt += G) {
      if (ok) ok = mbar_wait_bounded(&full_w[sw], pw);
      if (ok && !first_use) ok = mbar_wait_bounded(&aempty[sa], pa ^ 1u);
      ok = __all_sync(0xffffffffu, ok);  // tcgen05.st is warp-collective
      if (ok) {
        tc_fence_after();
        const uint8_t* wsm = w_slot(sw);
        const uint16_t* srow = reinterpret_cast<const uint16_t*>(wsm + L::kW);
        const uint32_t zw = *reinterpret_cast<const uint32_t*>(wsm + L::kW + L::kS + 4 * wi);
        uint32_t zp[4], sp[4];
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          const uint32_t z = (zw >> (4 * (4 * (e & 1) + c))) & 15u;
          zp[c] = (H::kMagic | (z << 16)) | z;  // (m + z, m + z)
          const uint32_t sb = srow[ncol[c]];
          sp[c] = sb | (sb << 16);
        }
        uint32_t R[NJB / 2][4];
#pragma unroll
        for (int x = 0; x < NJB / 2; ++x)
          ldmatrix_x4_trans(smem_u32(wsm) + ldoff[x], R[x][0], R[x][1], R[x][2], R[x][3]);
        uint32_t st0[4 * NJB], st1[4 * NJB];
#pragma unroll
        for (int jb = 0; jb < NJB; ++jb) {
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            const uint32_t reg = R[jb >> 1][2 * (jb & 1) + h];
#pragma unroll
            for (int c = 0; c < 4; ++c) {
              const uint32_t pr = lop3_and_or(c ? (reg >> (4 * c)) : reg, 0x000F000Fu, H::kMagic);
              const uint32_t wv = H::mul(H::sub(pr, zp[c]), sp[c]);
              // store 0: nibbles 0 (lane e) and 1 (lane e + 8); store 1: 2, 3
              uint32_t* dst = c < 2 ? st0 : st1;
              dst[4 * jb + 2 * (c & 1) + h] = wv;
            }
          }
        }
        const uint32_t acol = tmem + kTwACol + 64 * sa + (KA / 2) * blk;
        if constexpr (NJB == 4) {
          tmem_st_16x256b_x4(acol + lane_base, st0);
          tmem_st_16x256b_x4(acol + lane_base + (16u << 16), st1);
        } else {
          tmem_st_16x256b_x2(acol + lane_base, st0);
          tmem_st_16x256b_x2(acol + lane_base + (16u << 16), st1);
        }
        tmem_wait_st();
      }
      // the W slot's values are consumed (the stores above used them)
      mbar_arrive(&empty_w[sw]);
      tc_fence_before();
      mbar_arrive(&afull[sa]);
      sw += G;
      if (sw >= NW) { sw -= NW; pw ^= 1u; }
      sa += G;
      if (sa >= kTwASt) { sa -= kTwASt; pa ^= 1u; first_use = false; }
    }
    // ---- accumulators complete
    if (ok) ok = mbar_wait_bounded(acc_full, 0u);
    ok = __all_sync(0xffffffffu, ok);  // tcgen05.ld is warp-collective
    role_ok = ok;
    tc_fence_after();
  }

  // Split K: past this barrier every CTA of the cluster has finished its main
  // loop, so its rings may receive the peers' partial sums.
  if (split > 1) {
    cluster_arrive_release();
    cluster_wait_acquire();
  }

  if (warp >= 3) {
    // ---- epilogue: TMEM -> registers (-> owners) -> global
    const int dw = warp - 3;
    const int q = warp & 3;
    const int jq = dw >> 2;
    const bool ok = role_ok;
    const uint32_t lane_base = static_cast<uint32_t>(32 * q) << 16;
    const int nchunk = static_cast<int>(NX / 16);  // 16-column chunks per block
    auto put = [&](uint32_t row, uint32_t col, float v) {
      if (bias) v += DType<DT>::to_f32(bias[col]);
      om.template put<false>(om.at(row, col), DType<ODT>::from_f32(v));
    };
    if (split == 1) {
      if (ok) {
#pragma unroll 1
        for (int u = jq; u < NB * nchunk; u += 4) {
          const int b = u % NB, cc = u / NB;
          float v[16];
          tmem_ld_32x32b_x16(tmem + lane_base + b * NX + 16 * cc, v);
          const uint32_t col = n0 + tw_col_of_lane<ORDER>(b, q, lane);
          if (col < n) {
#pragma unroll
            for (int i = 0; i < 16; ++i) {
              const uint32_t row = 16 * cc + i;
              if (row < rows) put(row, col, v[i]);
            }
          }
        }
      }
    } else {
      // recv[src][b][lane 0..127][rpo] fp32
      float* recv = reinterpret_cast<float*>(smem);
      const uint32_t bar_local = smem_u32(recv_bar);
      if (ok) {
#pragma unroll 1
        for (int u = jq; u < NB * nchunk; u += 4) {
          const int b = u % NB, cc = u / NB;
          if (static_cast<uint32_t>(16 * cc) >= rows4) continue;
          float v[16];
          tmem_ld_32x32b_x16(tmem + lane_base + b * NX + 16 * cc, v);
#pragma unroll
          for (int i4 = 0; i4 < 4; ++i4) {
            const uint32_t r0 = 16 * cc + 4 * i4;  // first row of the group
            if (r0 >= rows4) continue;
            const uint32_t o = r0 / rpo;
            float* dst =
                recv + (((size_t)rank * NB + b) * 128 + 32 * q + lane) * rpo + (r0 - o * rpo);
            if (o == rank) {
              *reinterpret_cast<float4*>(dst) =
                  make_float4(v[4 * i4], v[4 * i4 + 1], v[4 * i4 + 2], v[4 * i4 + 3]);
            } else {
              st_async_v4(map_shared_rank(smem_u32(dst), o), v[4 * i4], v[4 * i4 + 1],
                          v[4 * i4 + 2], v[4 * i4 + 3], map_shared_rank(bar_local, o));
            }
          }
        }
      }
      const bool got = mbar_wait_bounded(recv_bar, 0u);
      named_bar_sync(1, 32 * kTwDqWarps);  // this CTA's own groups are in place
      if (ok && got) {
        // the warps of a quarter: block jq % NB, every G-th group of 4 rows
        const int b = jq % NB;
        const uint32_t col = n0 + tw_col_of_lane<ORDER>(b, q, lane);
        for (uint32_t i4 = (uint32_t)(jq / NB) * 4; i4 < own4; i4 += 4 * G) {
          float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
          for (uint32_t src = 0; src < split; ++src) {
            const float4 f = *reinterpret_cast<const float4*>(
                recv + (((size_t)src * NB + b) * 128 + 32 * q + lane) * rpo + i4);
            acc.x += f.x; acc.y += f.y; acc.z += f.z; acc.w += f.w;
          }
          if (col < n) {
            const float a4[4] = {acc.x, acc.y, acc.z, acc.w};
#pragma unroll
            for (int t = 0; t < 4; ++t) {
              const uint32_t row = own_lo + i4 + t;
              if (row < rows) put(row, col, a4[t]);
            }
          }
        }
      }
    }
  }
  // No copy this CTA issued may still be writing its shared memory when it
  // exits: after a failed (timed-out) run, wait (bounded) for the last stage
  // issued into each ring slot.
  if (__syncthreads_or(role_ok ? 0 : 1) && threadIdx.x == 0) {
    const int xi = s_x_issued, wi = s_w_issued;
    for (int j = xi > kTwXSt ? xi - kTwXSt : 0; j < xi; ++j)
      mbar_wait_bounded(&full_x[j % kTwXSt], (uint32_t)((j / kTwXSt) & 1));
    for (int j = wi > NW ? wi - NW : 0; j < wi; ++j)
      mbar_wait_bounded(&full_w[j % NW], (uint32_t)((j / NW) & 1));
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
}

// ------------------------------------------------------------------ host
// plan.tile_n = 512 selects NB = 4 (rows <= 64), else NB = 2 (rows <= 128).
static int tw_nb(const cawq_plan& plan) { return plan.tile_n == 512 ? 4 : 2; }

template <int NB>
static size_t tw_smem(const GemmProblem& p, int split, int nw) {
  return TwLayout<NB>::smem(static_cast<uint32_t>(p.rows), static_cast<uint32_t>(split),
                            static_cast<uint32_t>(nw));
}

bool prefill_tw_supports(const GemmProblem& p, const cawq_plan& plan, const DeviceInfo& dev) {
  const int split = plan.split < 1 ? 1 : plan.split;
  const int nb = tw_nb(plan);
  if (plan.tile_n != 0 && plan.tile_n != 256 && plan.tile_n != 512) return false;
  if (split > kTwMaxSplit || (split & (split - 1))) return false;
  if (dev.cc_major != 10) return false;
  if (p.dtype != kF16 && p.dtype != kBF16) return false;
  if (p.rows == 0 || p.rows > (size_t)(256 / nb)) return false;
  if (p.k % kTwXK != 0 || p.g % kTwXK != 0 || p.k % p.g != 0 || p.n % 32 != 0) return false;
  if ((size_t)split > p.k / kTwXK) return false;
  if (p.k >= (1ull << 31) || p.n >= (1ull << 31) || p.ld_out >= (1ull << 31)) return false;
  if (p.epi != 0 || p.nrep > 0) return false;  // plain epilogue (one or three outputs)
  const int nw = plan.stages == 0 ? kTwWStDefault : plan.stages;
  if (nw < 4 / nb || nw > kTwWStMax) return false;
  if (dev.smem_optin < (nb == 4 ? tw_smem<4>(p, split, nw) : tw_smem<2>(p, split, nw)))
    return false;
  const uintptr_t ax = reinterpret_cast<uintptr_t>(p.x), aw = reinterpret_cast<uintptr_t>(p.qw);
  const uintptr_t az = reinterpret_cast<uintptr_t>(p.qz), as = reinterpret_cast<uintptr_t>(p.sc);
  return ax % 16 == 0 && aw % 16 == 0 && az % 16 == 0 && as % 16 == 0;
}

template <int DT, int ODT, int ORDER, int NB>
static cudaError_t launch_prefill_tw_t(const GemmProblem& p, int split, int nw, bool pdl) {
  using T = typename DType<DT>::T;
  using OT = typename DType<ODT>::T;
  using L = TwLayout<NB>;
  const CUtensorMapDataType xdt =
      DT == kF16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
  const uint32_t rows = static_cast<uint32_t>(p.rows);
  const uint32_t nx = L::nx(rows);
  CUtensorMap tx, tw, ts, tz;
  const uint64_t npk = p.n / 8, groups = p.k / p.g;
  if (!pf_encode(&tx, xdt, p.x, p.k, p.rows, p.k * 2, kTwXK, nx, CU_TENSOR_MAP_SWIZZLE_128B) ||
      !pf_encode(&tw, CU_TENSOR_MAP_DATA_TYPE_UINT32, p.qw, npk, p.k, npk * 4, 32, L::kKA,
                 CU_TENSOR_MAP_SWIZZLE_128B) ||
      !pf_encode(&ts, xdt, p.sc, p.n, groups, p.n * 2, 256, 1, CU_TENSOR_MAP_SWIZZLE_NONE) ||
      !pf_encode(&tz, CU_TENSOR_MAP_DATA_TYPE_UINT32, p.qz, npk, groups, npk * 4, L::kBN / 8, 1,
                 CU_TENSOR_MAP_SWIZZLE_NONE)) {
    return cudaErrorInvalidValue;
  }
  auto kern = prefill_tw_kernel<DT, ODT, ORDER, NB>;
  const size_t smem = L::smem(rows, static_cast<uint32_t>(split), static_cast<uint32_t>(nw));
  static size_t attr_smem = 0;  // per instantiation: the largest size set so far
  if (smem > attr_smem) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         static_cast<int>(smem));
    if (e != cudaSuccess) return e;
    attr_smem = smem;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<uint32_t>((p.n + L::kBN - 1) / L::kBN), 1,
                     static_cast<uint32_t>(split));
  cfg.blockDim = dim3(kTwThreads);
  cfg.dynamicSmemBytes = smem;
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
  if (pdl) {
    attr[na].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[na].val.programmaticStreamSerializationAllowed = 1;
    ++na;
  }
  cfg.attrs = attr;
  cfg.numAttrs = na;
  return cudaLaunchKernelEx(&cfg, kern, tx, tw, ts, tz, static_cast<const T*>(p.bias),
                            out_map<OT>(p), rows, static_cast<uint32_t>(p.k),
                            static_cast<uint32_t>(p.n), static_cast<uint32_t>(p.g),
                            static_cast<uint32_t>(split), static_cast<uint32_t>(nw));
}

template <int DT, int ODT, int NB>
static cudaError_t launch_prefill_tw_o(const GemmProblem& p, int split, int nw, bool pdl) {
  return p.order == kOrderNatural
             ? launch_prefill_tw_t<DT, ODT, kOrderNatural, NB>(p, split, nw, pdl)
             : launch_prefill_tw_t<DT, ODT, kOrderAwq, NB>(p, split, nw, pdl);
}

template <int DT, int ODT>
static cudaError_t launch_prefill_tw_nb(const GemmProblem& p, int nb, int split, int nw, bool pdl) {
  return nb == 4 ? launch_prefill_tw_o<DT, ODT, 4>(p, split, nw, pdl)
                 : launch_prefill_tw_o<DT, ODT, 2>(p, split, nw, pdl);
}

cudaError_t launch_prefill_tw(const GemmProblem& p, const cawq_plan& plan, const DeviceInfo& dev) {
  const int split = plan.split < 1 ? 1 : plan.split;
  const int nb = tw_nb(plan);
  const size_t ctas = ((p.n + 128 * nb - 1) / (128 * nb)) * (size_t)split;
  const size_t sms = static_cast<size_t>(dev.sm_count > 0 ? dev.sm_count : 148);
  const bool pdl = plan.reserved[0] == 0 && ctas <= sms;
  const int nw = plan.stages == 0 ? kTwWStDefault : plan.stages;
  if (p.dtype == kF16) {
    return p.out_dtype == kF32 ? launch_prefill_tw_nb<kF16, kF32>(p, nb, split, nw, pdl)
                               : launch_prefill_tw_nb<kF16, kF16>(p, nb, split, nw, pdl);
  }
  if (p.dtype == kBF16) {
    return p.out_dtype == kF32 ? launch_prefill_tw_nb<kBF16, kF32>(p, nb, split, nw, pdl)
                               : launch_prefill_tw_nb<kBF16, kBF16>(p, nb, split, nw, pdl);
  }
  return cudaErrorNotSupported;
}

}  // namespace cawq

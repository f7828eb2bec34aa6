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
//   * Tiles. A CTA owns a band of `strips` x 128 output columns and a slice
//     of K. Each strip is handled by two consumer warps, one per 64-column half
//     (one packed word per lane). A cluster of `split` CTAs shares one band and
//     splits K; partial sums are added across the cluster through distributed
//     shared memory, so no global scratch is needed.
//   * Loads. One producer warp streams 64-row stages through a TMA ring: one
//     128-byte-row weight box (128-byte swizzle) per pair of strips, back to
//     back, so every k row is requested as one contiguous run, plus the scale
//     and zero rows of the
//     stage's groups (bulk copies) and the matching slice of X (128-byte
//     swizzle). Weights, scales and zeros do not depend on the previous kernel
//     in the stream, so they are requested before griddepcontrol.wait; X
//     after it (programmatic dependent launch).
//   * Operands. The MMA is swapped: A = W^T (16 output columns x 16 k),
//     B = X^T (16 k x 8 rows of X). Two packed words from k rows r, r' are
//     byte-interleaved (prmt) so one lop3 yields the f16 pair
//     (1024 + q[r], 1024 + q[r']) of one column; the high nibble is taken in
//     place as 1024 + 16 q. bf16 (and f32 inputs, split into bf16 hi + lo)
//     use 128 + q with a shift. No per-weight subtraction or scaling.
//   * Group fold. Within a quantization group, sum_k x (c + q) is accumulated
//     by the MMA, and sum_k x by one more MMA with an all-ones A. When the
//     group ends each output adds
//         s' * (D - c' * sum_k x)      (c' = offset + zero, s' = scale)
//     in fp32. This equals sum_k x (q - z) s up to fp32 rounding.
//
// Arithmetic differs from the reference in rounding only: the reference
// rounds (q - z) * s and every partial sum to F; here the weight is exact and
// the sum is fp32 (see the tolerance of the parity tests).
#pragma once

#include "cawq_common.cuh"

namespace cawq {

constexpr int kDecTileCols = 128;  // output columns per strip (consumer warp)
constexpr int kDecTileWords = 16;  // packed words per k row in a strip
constexpr int kDecBoxWords = 32;   // packed words per k row in a weight box (2 strips)
constexpr int kDecStageRows = 64;  // k rows per TMA stage (4 MMA steps)
constexpr int kDecMaxWarps = 8;
constexpr int kDecMaxStages = 8;

// Shared-memory layout of one ring slot:
//   [X tile: XB rows x 64 k, 128B swizzle][W: strips/2 x 64 rows x 128 B, 128B swizzle]
//   [S: gps rows x band columns, F][Z: gps rows x band/8 words]
// gps = quantization groups a 64-row stage can touch.
template <int DT, int MT>
struct DecodeLayout {
  using T = typename DType<DT>::T;
  static constexpr int XB = 8 * MT;
  static constexpr int kXBytes = XB * kDecStageRows * (int)sizeof(T);
  static constexpr int kWBytes = kDecStageRows * kDecTileWords * 4;  // 4096 per strip
  // groups a 64-row window starting at a multiple of 64 can touch (g % 16 == 0)
  static __host__ __device__ int gps(uint32_t g) {
    if (64 % g == 0) return (int)(64 / g);
    if (g % 64 == 0) return 1;
    return (int)(64 / g) + 2;
  }
  static __host__ __device__ size_t s_off(int strips) {
    return (size_t)kXBytes + (size_t)strips * kWBytes;
  }
  static __host__ __device__ size_t s_row_bytes(int strips) {
    return (size_t)strips * kDecTileCols * sizeof(T);
  }
  static __host__ __device__ size_t z_off(int strips, uint32_t g) {
    return s_off(strips) + gps(g) * s_row_bytes(strips);
  }
  static __host__ __device__ size_t z_row_bytes(int strips) {
    return (size_t)strips * kDecTileWords * 4;
  }
  static __host__ __device__ size_t slot_bytes(int strips, uint32_t g) {
    const size_t raw = z_off(strips, g) + gps(g) * z_row_bytes(strips);
    return (raw + 1023) / 1024 * 1024;
  }
  // split-K receive buffer: [source rank][XB rows][band columns / split] fp32
  static __host__ __device__ size_t recv_bytes(int strips) {
    return (size_t)XB * strips * kDecTileCols * 4;
  }
  static size_t smem_bytes(int strips, int stages, uint32_t g) {
    return 1024 /* alignment slack */ + slot_bytes(strips, g) * stages + recv_bytes(strips) +
           (size_t)(2 * stages + 1) * 8;
  }
};

// Consumer warps per CTA (strips x 2 halves), bounded by the register file:
// about 80 registers per thread for 8-row X tiles, 128 for 16.
__host__ __device__ constexpr int dec_max_consumers(int mt) { return mt == 1 ? 16 : 8; }

// Physical k row (0..15 within a 16-row step) that lane quad position t uses
// for fragment slot i (0..3). The four rows one load instruction touches,
// {2t + (i & 1) + 8 (i >> 1)}, differ in bits 1-2, so under the 128-byte
// swizzle their 32-byte column pieces land in four different bank groups;
// and the k pairs of one fragment register, (2t, 2t+1) and (2t+8, 2t+9), are
// adjacent, so X^T fragments are single 32-bit loads.
__device__ __forceinline__ int dec_row(int t, int i) { return 2 * t + (i & 1) + 8 * (i >> 1); }

// prmt selectors: bytes (b of word a, b of word b) -> result bytes 0 and 2.
__device__ __forceinline__ uint32_t dec_sel(int b) {
  return static_cast<uint32_t>(b | (b << 4) | ((4 + b) << 8) | ((4 + b) << 12));
}

template <int DT, int ODT, int ORDER, int MT, bool GA>
__global__ void __launch_bounds__(dec_max_consumers(MT) * 32 + 32, 1)
    decode_kernel(const __grid_constant__ CUtensorMap tm_w, const __grid_constant__ CUtensorMap tm_x,
                  const uint32_t* __restrict__ qz, const typename DType<DT>::T* __restrict__ sc,
                  const typename DType<DT>::T* __restrict__ bias,
                  typename DType<ODT>::T* __restrict__ out, uint32_t rows, uint32_t k, uint32_t n,
                  uint32_t g, uint32_t ld_out, uint32_t split, uint32_t nstage_ring,
                  uint32_t strips_u) {
  using L = DecodeLayout<DT, MT>;
  using T = typename DType<DT>::T;
  constexpr bool kF16Mma = (DT == kF16);
  constexpr int XB = L::XB;
  // A operand of the "ones" MMA: sum_k x[b][k] for every row b of X comes out
  // of the tensor core with the same accumulation as the weight MMAs.
  constexpr uint32_t kOnes = kF16Mma ? 0x3C003C00u : 0x3F803F80u;

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = smem_raw + ((1024 - (smem_u32(smem_raw) & 1023)) & 1023);

  const int strips = static_cast<int>(strips_u);
  const int consumers = 2 * strips;  // warps 0..consumers-1; the producer follows
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int gq = lane >> 2;
  const int t = lane & 3;

  const uint32_t rank = split > 1 ? cluster_ctarank() : 0u;
  const uint32_t band = blockIdx.x / split;
  const uint32_t pband = band * strips * kDecTileWords;  // first packed column of the band
  const uint32_t npk = n >> 3;
  const uint32_t steps = k >> 4;
  const uint32_t nst_total = (steps + 3) >> 2;
  const uint32_t c_beg = (uint32_t)((uint64_t)nst_total * rank / split);
  const uint32_t c_end = (uint32_t)((uint64_t)nst_total * (rank + 1) / split);
  const int nst = static_cast<int>(c_end - c_beg);
  const uint32_t end_step = c_end * 4 < steps ? c_end * 4 : steps;
  const int NS = static_cast<int>(nstage_ring);
  const size_t slot = L::slot_bytes(strips, g);
  const int gps = L::gps(g);

  const size_t ring_bytes = slot * NS;
  float* recv = reinterpret_cast<float*>(smem + ring_bytes);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + ring_bytes + L::recv_bytes(strips));
  uint64_t* empty = full + NS;
  uint64_t* recv_bar = empty + NS;  // the peers' partial sums have landed
  const uint32_t rows_eff = rows < (uint32_t)XB ? rows : (uint32_t)XB;
  const uint32_t bcols = static_cast<uint32_t>(strips * kDecTileCols);
  const uint32_t ncols = bcols / split;  // columns of the band this CTA sums (multiple of 8)

  if (threadIdx.x == 0) {
    for (int s = 0; s < NS; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], static_cast<uint32_t>(consumers));
    }
    mbar_init(recv_bar, 1);
    if (split > 1) mbar_arrive_expect_tx(recv_bar, (split - 1) * rows_eff * ncols * 4);
    fence_mbarrier_init();
  }
  __syncthreads();
  // Peers push into this CTA's receive buffer only after every CTA of the
  // cluster has passed this point (the matching wait precedes the pushes).
  if (split > 1) cluster_arrive_release();
  // The next kernel in the stream may launch now: its CTAs take SMs as they
  // free up and prefetch their weights; they read this kernel's output only
  // after griddepcontrol.wait, which waits for this whole grid.
  pdl_launch_dependents();
  __shared__ int s_issued;  // stages whose copies the producer issued

  bool ok = true;
  if (warp == consumers) {
    // ------------------------------------------------------ TMA producer
    if (lane == 0) {
      // valid columns of the band (the bulk copies must stay inside a row)
      const uint32_t bcol0 = pband * 8;
      const uint32_t vcols = min((uint32_t)(strips * kDecTileCols), n - min(n, bcol0));
      const uint32_t ngroups = k / g;
      const uint32_t tx = static_cast<uint32_t>(L::kXBytes + strips * L::kWBytes) +
                          (uint32_t)gps * (vcols * (uint32_t)sizeof(T) + vcols / 2);
      auto issue_weights = [&](int j) {
        const int sl = j % NS;
        uint8_t* dst = smem + sl * slot;
        const int kr = static_cast<int>((c_beg + j) * kDecStageRows);
        mbar_arrive_expect_tx(&full[sl], tx);
        for (int b = 0; b < strips / 2; ++b) {
          tma_load_2d(dst + L::kXBytes + 2 * b * L::kWBytes, &tm_w,
                      static_cast<int>(pband + b * kDecBoxWords), kr, &full[sl]);
        }
        const uint32_t g0 = (uint32_t)kr / g;
        for (int r = 0; r < gps; ++r) {
          // rows past the last group repeat it; the fold never reads them
          const uint32_t grp = min(g0 + r, ngroups - 1);
          if (vcols) {
            bulk_load_1d(dst + L::s_off(strips) + r * L::s_row_bytes(strips),
                         sc + (size_t)grp * n + bcol0, vcols * sizeof(T), &full[sl]);
            bulk_load_1d(dst + L::z_off(strips, g) + r * L::z_row_bytes(strips),
                         qz + (size_t)grp * npk + pband, vcols / 2, &full[sl]);
          }
        }
      };
      auto issue_x = [&](int j) {
        const int sl = j % NS;
        uint8_t* dst = smem + sl * slot;
        const int kr = static_cast<int>((c_beg + j) * kDecStageRows);
        if constexpr (DT == kF32) {
          tma_load_2d(dst, &tm_x, kr, 0, &full[sl]);
          tma_load_2d(dst + XB * 128, &tm_x, kr + 32, 0, &full[sl]);
        } else {
          tma_load_2d(dst, &tm_x, kr, 0, &full[sl]);
        }
      };
      const int pro = NS < nst ? NS : nst;
      for (int j = 0; j < pro; ++j) issue_weights(j);  // independent of earlier kernels
      pdl_wait();                                       // X may be the previous kernel's output
      for (int j = 0; j < pro; ++j) issue_x(j);
      int issued = pro;
      for (int j = pro; j < nst && ok; ++j) {
        const int sl = j % NS;
        ok = mbar_wait_bounded(&empty[sl], static_cast<uint32_t>(((j / NS) - 1) & 1));
        if (!ok) break;
        issue_weights(j);
        issue_x(j);
        issued = j + 1;
      }
      s_issued = issued;
    }
    __syncwarp();
  }

  float tot[MT][4][4];
#pragma unroll
  for (int m = 0; m < MT; ++m)
#pragma unroll
    for (int j = 0; j < 4; ++j)
#pragma unroll
      for (int e = 0; e < 4; ++e) tot[m][j][e] = 0.f;

  // this warp's strip and 64-column half
  const int strip = warp % strips;
  const int half = (warp / strips) & 1;
  const int word = 8 * half + gq;  // packed word of this lane inside the strip

  if (warp < consumers) {
    // -------------------------------------------------------- consumers
    uint32_t woff[4];  // weight rows dec_row(t, i) of a step, this lane's word
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int r = dec_row(t, i);
      const int bw = 16 * (strip & 1) + word;  // word inside the 128-byte box row
      woff[i] = L::kXBytes + (strip >> 1) * 2 * L::kWBytes + r * 128 +
                ((((bw >> 2) ^ (r & 7))) << 4) + ((bw & 3) << 2);
    }
    // X^T fragments. 16-bit X: one ldmatrix.x4 per 8-row block of X loads the
    // fragments of two steps; lane L gives the address of row 8m + (L & 7),
    // 16-byte k chunk 4p + (L >> 3) of step pair p, under the tile's 128-byte
    // swizzle. f32 X: each k pair is loaded directly and split into bf16 hi/lo.
    uint32_t xrow[MT];    // byte offset of row 8m + gq (f32 X)
    uint32_t x7[MT];      // its swizzle phase
    uint32_t xld[MT][2];  // ldmatrix row addresses, step pairs 0 and 1 (16-bit X)
#pragma unroll
    for (int m = 0; m < MT; ++m) {
      const int xr = 8 * m + gq;
      xrow[m] = xr * 128;
      x7[m] = static_cast<uint32_t>(xr & 7);
      const int lr = lane & 7, li = lane >> 3;
#pragma unroll
      for (int p = 0; p < 2; ++p)
        xld[m][p] = static_cast<uint32_t>((8 * m + lr) * 128 + (((4 * p + li) ^ lr) << 4));
    }
    // scales of this lane's 8 columns and its zero word inside the stage rows
    const uint32_t s_lane = (uint32_t)(strip * kDecTileCols + 8 * word) * (uint32_t)sizeof(T);
    const uint32_t z_lane = (uint32_t)(strip * kDecTileWords + word) * 4;

    float D[MT][4][4];
    float Dx[MT][4];  // sum_k x over the current group (ones MMA)
#pragma unroll
    for (int m = 0; m < MT; ++m) {
#pragma unroll
      for (int j = 0; j < 4; ++j)
#pragma unroll
        for (int e = 0; e < 4; ++e) D[m][j][e] = 0.f;
#pragma unroll
      for (int e = 0; e < 4; ++e) Dx[m][e] = 0.f;
    }

    // tot += s' * (D - c' * sum_k x) with this group's scales / zeros from the
    // stage's shared-memory rows (see the file comment). c' = offset + zero is
    // built by the same magic-number lop3 as the weights: for f16 the lo
    // nibble gives 1024 + z and the hi nibble, in place, 1024 + 16 z; for
    // bf16 both give 128 + z. With `clear` the accumulators restart at 0;
    // else the next group's first MMA overwrites them.
    auto fold = [&](const uint8_t* srow, const uint8_t* zrow, auto clear_tag) {
      constexpr bool kClear = decltype(clear_tag)::value;
      float s_reg[8];
      if constexpr (DT == kF32) {
#pragma unroll
        for (int v = 0; v < 2; ++v) {
          const float4 f = *reinterpret_cast<const float4*>(srow + s_lane + 16 * v);
          s_reg[4 * v + 0] = f.x; s_reg[4 * v + 1] = f.y;
          s_reg[4 * v + 2] = f.z; s_reg[4 * v + 3] = f.w;
        }
      } else {
        const uint4 raw = *reinterpret_cast<const uint4*>(srow + s_lane);
        const T* h = reinterpret_cast<const T*>(&raw);
#pragma unroll
        for (int c = 0; c < 8; ++c) s_reg[c] = DType<DT>::to_f32(h[c]);
      }
      const uint32_t zw = *reinterpret_cast<const uint32_t*>(zrow + z_lane);
      float cz[8];  // c' of nibble p of zw
      if constexpr (kF16Mma) {
        const uint32_t z8 = zw >> 8;
        const uint32_t q[4] = {lop3_and_or(zw, 0x000F000Fu, 0x64006400u),   // nibbles 0, 4
                               lop3_and_or(zw, 0x00F000F0u, 0x64006400u),   // 1, 5 (x16)
                               lop3_and_or(z8, 0x000F000Fu, 0x64006400u),   // 2, 6
                               lop3_and_or(z8, 0x00F000F0u, 0x64006400u)};  // 3, 7 (x16)
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&q[i]));
          cz[i] = f.x;
          cz[i + 4] = f.y;
        }
      } else {
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const uint32_t q = lop3_and_or(zw >> (4 * i), 0x000F000Fu, 0x43004300u);
          cz[i] = __uint_as_float(q << 16);             // nibble i
          cz[i + 4] = __uint_as_float(q & 0xFFFF0000u);  // nibble i + 4
        }
      }
#pragma unroll
      for (int b = 0; b < 4; ++b) {
        const float sl = s_reg[col_of_nibble(2 * b, ORDER)];
        float sh = s_reg[col_of_nibble(2 * b + 1, ORDER)];
        if constexpr (kF16Mma) sh *= 0.0625f;  // the hi nibble entered the MMA as 16 q
        const float cl = cz[2 * b], ch = cz[2 * b + 1];
#pragma unroll
        for (int m = 0; m < MT; ++m) {
          tot[m][b][0] = fmaf(sl, fmaf(-cl, Dx[m][0], D[m][b][0]), tot[m][b][0]);
          tot[m][b][1] = fmaf(sl, fmaf(-cl, Dx[m][1], D[m][b][1]), tot[m][b][1]);
          tot[m][b][2] = fmaf(sh, fmaf(-ch, Dx[m][0], D[m][b][2]), tot[m][b][2]);
          tot[m][b][3] = fmaf(sh, fmaf(-ch, Dx[m][1], D[m][b][3]), tot[m][b][3]);
          if constexpr (kClear) D[m][b][0] = D[m][b][1] = D[m][b][2] = D[m][b][3] = 0.f;
        }
      }
      if constexpr (kClear) {
#pragma unroll
        for (int m = 0; m < MT; ++m)
#pragma unroll
          for (int e = 0; e < 4; ++e) Dx[m][e] = 0.f;
      }
    };

    // D += A B, or D = A B when the tag says this is a group's first step
    auto mma = [&](float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                   uint32_t b0, uint32_t b1, auto zero_tag) {
      if constexpr (decltype(zero_tag)::value) {
        mma_16816_c0<!kF16Mma>(d, a0, a1, a2, a3, b0, b1);
      } else {
        mma_16816<!kF16Mma>(d, a0, a1, a2, a3, b0, b1);
      }
    };

    // f32 X: the step's fragments, as bf16 hi and lo parts
    auto x_frags_f32 = [&](const uint8_t* sbase, int s, uint32_t (&bh)[MT][2],
                           uint32_t (&bl)[MT][2]) {
#pragma unroll
      for (int m = 0; m < MT; ++m) {
#pragma unroll
        for (int h2 = 0; h2 < 2; ++h2) {
          // two 32-k boxes; k = 16s + 8h2 + 2t lies in box s >> 1
          const uint32_t ch2 = (uint32_t)(4 * (s & 1) + 2 * h2 + (t >> 1));
          const float2 xv = *reinterpret_cast<const float2*>(
              sbase + (s >> 1) * XB * 128 + xrow[m] + ((ch2 ^ x7[m]) << 4) + 8 * (t & 1));
          const __nv_bfloat162 hi = __floats2bfloat162_rn(xv.x, xv.y);
          const __nv_bfloat162 lo =
              __floats2bfloat162_rn(xv.x - __low2float(hi), xv.y - __high2float(hi));
          bh[m][h2] = *reinterpret_cast<const uint32_t*>(&hi);
          bl[m][h2] = *reinterpret_cast<const uint32_t*>(&lo);
        }
      }
    };

    // one 16-row step with X^T fragments bh (and the bf16 lo parts bl of f32 X):
    // the ones MMA, dequantize and multiply
    auto step_mma = [&](const uint8_t* sbase, int s, const uint32_t (&bh)[MT][2],
                        const uint32_t (&bl)[MT][2], auto zero_tag) {
      uint32_t wv[4];
#pragma unroll
      for (int i = 0; i < 4; ++i)
        wv[i] = *reinterpret_cast<const uint32_t*>(sbase + woff[i] + s * 2048);
#pragma unroll
      for (int m = 0; m < MT; ++m) {
        mma(Dx[m], kOnes, kOnes, kOnes, kOnes, bh[m][0], bh[m][1], zero_tag);
        if constexpr (DT == kF32)
          mma_16816<true>(Dx[m], kOnes, kOnes, kOnes, kOnes, bl[m][0], bl[m][1]);
      }
#pragma unroll
      for (int b = 0; b < 4; ++b) {
        const uint32_t p01 = prmt(wv[0], wv[1], dec_sel(b));
        const uint32_t p23 = prmt(wv[2], wv[3], dec_sel(b));
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
          mma(D[m][b], a0, a1, a2, a3, bh[m][0], bh[m][1], zero_tag);
          if constexpr (DT == kF32) mma_16816<true>(D[m][b], a0, a1, a2, a3, bl[m][0], bl[m][1]);
        }
      }
    };

    // the four steps of a stage (the first one restarts the accumulators if
    // zero_tag says a group starts here)
    auto stage_mma = [&](const uint8_t* sbase, auto zero_tag) {
      using NoZero = std::integral_constant<bool, false>;
      uint32_t bh[MT][2], bl[MT][2];
      [[maybe_unused]] uint32_t bh2[MT][2];
      if constexpr (DT == kF32) {
        x_frags_f32(sbase, 0, bh, bl);
        step_mma(sbase, 0, bh, bl, zero_tag);
#pragma unroll
        for (int st = 1; st < 4; ++st) {
          x_frags_f32(sbase, st, bh, bl);
          step_mma(sbase, st, bh, bl, NoZero{});
        }
      } else {
#pragma unroll
        for (int p = 0; p < 2; ++p) {
#pragma unroll
          for (int m = 0; m < MT; ++m)
            ldmatrix_x4(smem_u32(sbase) + xld[m][p], bh[m][0], bh[m][1], bh2[m][0], bh2[m][1]);
          if (p == 0) {
            step_mma(sbase, 0, bh, bl, zero_tag);
          } else {
            step_mma(sbase, 2, bh, bl, NoZero{});
          }
          step_mma(sbase, 2 * p + 1, bh2, bl, NoZero{});
        }
      }
    };

    int sl = 0;
    uint32_t par = 0;
    if constexpr (GA) {
      // g is a multiple of 64: groups end on stage boundaries, so the four
      // steps of a stage run without any branch and the fold (if any) follows.
      const uint32_t spgs = g / kDecStageRows;  // stages per group
      uint32_t in_grp = c_beg % spgs;           // stage index inside its group
      for (int j = 0; j < nst; ++j) {
        if (ok) ok = mbar_wait_bounded(&full[sl], par);
        ok = __all_sync(0xffffffffu, ok);  // keep the warp convergent
        if (!ok) break;
        const uint8_t* sbase = smem + sl * slot;
        // a group's first stage (not the CTA's first: D starts at 0 there)
        if (in_grp == 0 && j > 0) {
          stage_mma(sbase, std::integral_constant<bool, true>{});
        } else {
          stage_mma(sbase, std::integral_constant<bool, false>{});
        }
        if (++in_grp == spgs || j + 1 == nst) {
          fold(sbase + L::s_off(strips), sbase + L::z_off(strips, g),
               std::integral_constant<bool, false>{});
          in_grp = 0;
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[sl]);
        if (++sl == NS) {
          sl = 0;
          par ^= 1u;
        }
      }
    } else {
      // any g % 16 == 0: group boundaries tracked per step, without division
      using NoZero = std::integral_constant<bool, false>;
      const uint32_t spg = g >> 4;  // 16-row steps per quantization group
      uint32_t grp = (c_beg * 4) / spg;
      uint32_t grp_end = (grp + 1) * spg;  // first step of the next group
      for (int j = 0; j < nst; ++j) {
        if (ok) ok = mbar_wait_bounded(&full[sl], par);
        ok = __all_sync(0xffffffffu, ok);
        if (!ok) break;
        const uint8_t* sbase = smem + sl * slot;
        const uint32_t stage = c_beg + j;
        uint32_t bh[MT][2], bl[MT][2];
        [[maybe_unused]] uint32_t bh2[MT][2];
#pragma unroll
        for (int st = 0; st < 4; ++st) {
          const uint32_t step = stage * 4 + st;
          if (step >= end_step) break;
          if constexpr (DT == kF32) {
            x_frags_f32(sbase, st, bh, bl);
            step_mma(sbase, st, bh, bl, NoZero{});
          } else {
            if ((st & 1) == 0) {
#pragma unroll
              for (int m = 0; m < MT; ++m)
                ldmatrix_x4(smem_u32(sbase) + xld[m][st >> 1], bh[m][0], bh[m][1], bh2[m][0],
                            bh2[m][1]);
              step_mma(sbase, st, bh, bl, NoZero{});
            } else {
              step_mma(sbase, st, bh2, bl, NoZero{});
            }
          }
          const uint32_t next = step + 1;
          if (next >= end_step || next >= grp_end) {
            const uint32_t r = grp - stage * kDecStageRows / g;  // scale row in this stage
            fold(sbase + L::s_off(strips) + r * L::s_row_bytes(strips),
                 sbase + L::z_off(strips, g) + r * L::z_row_bytes(strips),
                 std::integral_constant<bool, true>{});
            grp += 1;
            grp_end += spg;
          }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[sl]);
        if (++sl == NS) {
          sl = 0;
          par ^= 1u;
        }
      }
    }
  }

  // Before exiting, no copy this CTA issued may still be writing its shared
  // memory. Normally every issued stage has been consumed; after a timed-out
  // wait, wait (bounded) for the last stage issued into each slot.
  auto drain = [&]() {
    if (!__syncthreads_or(ok ? 0 : 1)) return;
    if (threadIdx.x == 0) {
      const int issued = s_issued;
      for (int j = issued > NS ? issued - NS : 0; j < issued; ++j)
        mbar_wait_bounded(&full[j % NS], static_cast<uint32_t>((j / NS) & 1));
    }
    __syncthreads();
  };

  // ---- split-K sums. CTA q of the cluster owns columns [q ncols, (q+1) ncols)
  // of the band: every CTA stores its partial sums of those columns into
  // slot [its rank] of q's receive buffer (st.async to distributed shared
  // memory, counted on q's recv_bar), then sums its own columns over the
  // slots in rank order. One wait, no cluster-wide barrier at the end.
  if (split == 1) {
    if (warp < consumers) {
#pragma unroll
      for (int m = 0; m < MT; ++m) {
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          const uint32_t row = static_cast<uint32_t>(8 * m + 2 * t + e);
          if (row >= rows_eff) continue;
#pragma unroll
          for (int b = 0; b < 4; ++b) {
#pragma unroll
            for (int hi = 0; hi < 2; ++hi) {
              const uint32_t col = pband * 8 + strip * kDecTileCols + 8 * word +
                                   col_of_nibble(2 * b + hi, ORDER);
              if (col < n) {
                float v = tot[m][b][2 * hi + e];
                if (bias) v += DType<DT>::to_f32(bias[col]);
                out[(size_t)row * ld_out + col] = DType<ODT>::from_f32(v);
              }
            }
          }
        }
      }
    }
    drain();
    return;
  }
  cluster_wait_acquire();  // every peer's recv_bar is initialised
  if (warp < consumers) {
    const uint32_t bar_local = smem_u32(recv_bar);
#pragma unroll
    for (int m = 0; m < MT; ++m) {
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const uint32_t row = static_cast<uint32_t>(8 * m + 2 * t + e);
        if (row >= rows_eff) continue;
        float v[8];  // this lane's 8 consecutive columns, natural order
#pragma unroll
        for (int b = 0; b < 4; ++b) {
          v[col_of_nibble(2 * b, ORDER)] = tot[m][b][e];
          v[col_of_nibble(2 * b + 1, ORDER)] = tot[m][b][2 + e];
        }
        const uint32_t col8 = static_cast<uint32_t>(strip * kDecTileCols + 8 * word);
        const uint32_t q = col8 / ncols;
        float* dst = recv + ((size_t)rank * XB + row) * ncols + (col8 - q * ncols);
        if (q == rank) {
          reinterpret_cast<float4*>(dst)[0] = make_float4(v[0], v[1], v[2], v[3]);
          reinterpret_cast<float4*>(dst)[1] = make_float4(v[4], v[5], v[6], v[7]);
        } else {
          const uint32_t ra = map_shared_rank(smem_u32(dst), q);
          const uint32_t rb = map_shared_rank(bar_local, q);
          st_async_v4(ra, v[0], v[1], v[2], v[3], rb);
          st_async_v4(ra + 16, v[4], v[5], v[6], v[7], rb);
        }
      }
    }
  }
  // the peers' bytes (bounded wait), and this CTA's own stores
  if (!mbar_wait_bounded(recv_bar, 0u)) ok = false;
  __syncthreads();
  for (uint32_t idx = threadIdx.x; idx < rows_eff * ncols; idx += blockDim.x) {
    const uint32_t row = idx / ncols, c = idx - row * ncols;
    const uint32_t col = pband * 8 + rank * ncols + c;
    float v = 0.f;
    for (uint32_t src = 0; src < split; ++src) v += recv[((size_t)src * XB + row) * ncols + c];
    if (col < n) {
      if (bias) v += DType<DT>::to_f32(bias[col]);
      out[(size_t)row * ld_out + col] = DType<ODT>::from_f32(v);
    }
  }
  drain();
}

// ------------------------------------------------------------------ host
static bool encode_2d(CUtensorMap* map, CUtensorMapDataType dt, const void* base, uint64_t inner,
                      uint64_t outer, uint64_t row_bytes, uint32_t box_inner, uint32_t box_outer,
                      CUtensorMapSwizzle swz) {
  return encode_tiled_2d(map, static_cast<int>(dt), base, inner, outer, row_bytes, box_inner,
                         box_outer, static_cast<int>(swz));
}

static int decode_mt(size_t rows) { return rows <= 8 ? 1 : 2; }

static size_t decode_smem(const GemmProblem& p, const cawq_plan& plan) {
  const uint32_t g = static_cast<uint32_t>(p.g);
  const bool mt1 = decode_mt(p.rows) == 1;
  if (p.dtype == kF32) {
    return mt1 ? DecodeLayout<kF32, 1>::smem_bytes(plan.warps, plan.stages, g)
               : DecodeLayout<kF32, 2>::smem_bytes(plan.warps, plan.stages, g);
  }
  return mt1 ? DecodeLayout<kF16, 1>::smem_bytes(plan.warps, plan.stages, g)
             : DecodeLayout<kF16, 2>::smem_bytes(plan.warps, plan.stages, g);
}

bool decode_supports(const GemmProblem& p, const cawq_plan& plan, const DeviceInfo& dev) {
  if (p.rows == 0 || p.rows > 16) return false;
  if (p.k % 16 != 0 || p.g % 16 != 0 || p.k % p.g != 0 || p.n % 32 != 0) return false;
  if (p.k >= (1ull << 31) || p.n >= (1ull << 31) || p.ld_out >= (1ull << 31)) return false;
  const uintptr_t ax = reinterpret_cast<uintptr_t>(p.x), aw = reinterpret_cast<uintptr_t>(p.qw);
  const uintptr_t az = reinterpret_cast<uintptr_t>(p.qz), as = reinterpret_cast<uintptr_t>(p.sc);
  if (ax % 16 || aw % 16 || az % 16 || as % 16) return false;
  if (plan.split < 1 || plan.split > 16 || (plan.split & (plan.split - 1))) return false;
  if (plan.tile_n > 1) return false;
  if (plan.warps < 2 || (plan.warps & 1) || 2 * plan.warps > dec_max_consumers(decode_mt(p.rows)))
    return false;
  if (plan.stages < 1 || plan.stages > kDecMaxStages) return false;
  const size_t bands =
      (p.n + (size_t)kDecTileCols * plan.warps - 1) / ((size_t)kDecTileCols * plan.warps);
  if (bands * plan.split >= (1ull << 31)) return false;
  return decode_smem(p, plan) <= dev.smem_optin && dev.cc_major == 10;
}

template <int DT, int ODT, int ORDER, int MT, bool GA>
static cudaError_t launch_decode_t(const GemmProblem& p, const cawq_plan& plan) {
  using L = DecodeLayout<DT, MT>;
  using T = typename DType<DT>::T;
  using OT = typename DType<ODT>::T;
  CUtensorMap tm_w, tm_x;
  const uint64_t npk = p.n / 8;
  if (!encode_2d(&tm_w, CU_TENSOR_MAP_DATA_TYPE_UINT32, p.qw, npk, p.k, npk * 4, kDecBoxWords,
                 kDecStageRows, CU_TENSOR_MAP_SWIZZLE_128B)) {
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
  auto kern = decode_kernel<DT, ODT, ORDER, MT, GA>;
  const size_t smem = decode_smem(p, plan);
  // function attributes are per process; set each once (a repeat is harmless)
  static size_t smem_set = 0;
  static bool nonportable_set = false;
  cudaError_t e;
  if (smem > smem_set) {
    e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             static_cast<int>(smem));
    if (e != cudaSuccess) return e;
    smem_set = smem;
  }
  if (plan.split > 8 && !nonportable_set) {
    e = cudaFuncSetAttribute(kern, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
    if (e != cudaSuccess) return e;
    nonportable_set = true;
  }
  const uint32_t bands = static_cast<uint32_t>(
      (p.n + (size_t)kDecTileCols * plan.warps - 1) / ((size_t)kDecTileCols * plan.warps));
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(bands * plan.split);
  cfg.blockDim = dim3((2 * plan.warps + 1) * 32);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = p.stream;
  cudaLaunchAttribute attr[2];
  int na = 0;
  if (plan.split > 1) {
    attr[na].id = cudaLaunchAttributeClusterDimension;
    attr[na].val.clusterDim.x = plan.split;
    attr[na].val.clusterDim.y = 1;
    attr[na].val.clusterDim.z = 1;
    ++na;
  }
  // Let this kernel's prologue (barrier set-up, weight loads) overlap the
  // tail of the previous kernel in the stream; X is read only after
  // griddepcontrol.wait. plan.reserved[0] = 1 launches without the overlap.
  if (plan.reserved[0] == 0) {
    attr[na].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[na].val.programmaticStreamSerializationAllowed = 1;
    ++na;
  }
  cfg.attrs = attr;
  cfg.numAttrs = na;
  return cudaLaunchKernelEx(&cfg, kern, tm_w, tm_x, p.qz, static_cast<const T*>(p.sc),
                            static_cast<const T*>(p.bias), static_cast<OT*>(p.out),
                            static_cast<uint32_t>(p.rows), static_cast<uint32_t>(p.k),
                            static_cast<uint32_t>(p.n), static_cast<uint32_t>(p.g),
                            static_cast<uint32_t>(p.ld_out), static_cast<uint32_t>(plan.split),
                            static_cast<uint32_t>(plan.stages), static_cast<uint32_t>(plan.warps));
}

template <int DT, int ODT, int ORDER>
static cudaError_t launch_decode_m(const GemmProblem& p, const cawq_plan& plan) {
  const bool ga = p.g % kDecStageRows == 0;  // groups end on stage boundaries
  if (decode_mt(p.rows) == 1) {
    return ga ? launch_decode_t<DT, ODT, ORDER, 1, true>(p, plan)
              : launch_decode_t<DT, ODT, ORDER, 1, false>(p, plan);
  }
  return ga ? launch_decode_t<DT, ODT, ORDER, 2, true>(p, plan)
            : launch_decode_t<DT, ODT, ORDER, 2, false>(p, plan);
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

// plan.warps = 128-column strips per CTA (two consumer warps each),
// plan.split = CTAs of a cluster splitting K, plan.stages = depth of the TMA ring.
cawq_plan decode_default_plan(const GemmProblem& p, const DeviceInfo& dev) {
  // Measured on B200 over chains of cold launches (Llama-2-7B shapes): two
  // strips per CTA, K split until there are about two CTAs per SM, and a
  // 6-stage ring once a CTA has more than 8 stages (4 below).
  cawq_plan plan = {};
  plan.path = CAWQ_PATH_DECODE;
  plan.warps = 2;
  const size_t sms = static_cast<size_t>(dev.sm_count > 0 ? dev.sm_count : 148);
  const size_t bands = (p.n + 2 * kDecTileCols - 1) / (2 * kDecTileCols);
  const size_t nst_total = (p.k / 16 + 3) / 4;
  int split = 1;
  while (split < 16 && bands * split < 2 * sms && nst_total >= (size_t)split * 8) split *= 2;
  plan.split = split;
  const size_t per_cta = (nst_total + split - 1) / split;
  plan.stages = per_cta > 8 ? 6 : (per_cta >= 4 ? 4 : (per_cta >= 2 ? 2 : 1));
  while (plan.stages > 1 && !decode_supports(p, plan, dev)) --plan.stages;
  return plan;
}

void decode_candidates(const GemmProblem& p, const DeviceInfo& dev, cawq_plan* out, int* count,
                       int max_count) {
  int c = 0;
  const size_t nst_total = (p.k / 16 + 3) / 4;
  for (int split = 2; split <= 16; split *= 2) {
    if (nst_total < (size_t)split) break;
    for (int warps : {2, 4, 6, 8}) {
      for (int stages : {2, 3, 4, 6}) {
        cawq_plan pl = {};
        pl.path = CAWQ_PATH_DECODE;
        pl.split = split;
        pl.warps = warps;
        pl.stages = stages;
        if (!decode_supports(p, pl, dev)) continue;
        if (c < max_count) out[c++] = pl;
      }
    }
  }
  *count = c;
}

}  // namespace cawq

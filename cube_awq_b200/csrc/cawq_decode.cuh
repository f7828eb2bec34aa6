// cawq_decode.cuh — small-M (decode) fused AWQ GEMM for sm_100a.
//
// Y[rows, N] = X[rows, K] · ((Q - Z) · S)[K, N], rows <= 16.
// Replaces gemm_awq_decode (src/kernel/awq_kernel_gemm.rs:445-624), which the
// reference launches for M <= DECODE_M_THRESHOLD = 8 (:81, :691).
//
// The work is bound by HBM bandwidth on the packed weights (0.5 byte per
// weight). On B200 that leaves about three issue slots per weight, so the
// kernel turns nibbles into tensor-core operands with little more than one
// instruction per pair of weights and lets mma.sync accumulate in fp32:
//
//   * Tiles. A CTA owns a band of `strips` x 128 output columns and a slice
//     of K. Each strip is handled by two consumer warps, one per 64-column half
//     (a lane holds 4 nibbles of 2 packed words). A cluster of `split` CTAs shares one band and
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
//     B = X^T (16 k x 8 rows of X). One ldmatrix.x4.trans per 16-row step
//     gives each lane, per register, one 16-bit element (4 nibbles = 4
//     columns) of two consecutive k rows: exactly the k pair an A-fragment
//     register holds. One lop3 per register and nibble then yields the f16
//     pair (1024 + q[k], 1024 + q[k + 1]): nibbles 0 and 2 as 1024 + q,
//     nibbles 1 and 3 in place as 1024 + 16 q, nibbles 2 and 3 after one
//     8-bit shift of the register. bf16 (and f32 inputs,
//     split into bf16 hi + lo) use 128 + q after a shift per nibble. No
//     per-weight subtraction or scaling.
//   * Group fold. Within a quantization group, sum_k x (c + q) is accumulated
//     by the MMA, and sum_k x by one more MMA with an all-ones A. When the
//     group ends each output adds
//         s' * (D - c' * sum_k x)      (c' = offset + zero, s' = scale)
//     in fp32. This equals sum_k x (q - z) s up to fp32 rounding.
//
// Arithmetic differs from the reference in rounding only: the reference
// rounds (q - z) * s and every partial sum to F; here the weight is exact and
// the sum is fp32 (see the tolerance of the parity tests).
//
// Integer path (plan.reserved[2] = 1; rows <= 4, 16-bit X, g % 64 == 0): an
// extra warp turns each stage's X rows into exact 16-bit fixed point (a
// power-of-two scale per row and stage, split into a signed high and an
// unsigned low byte) laid out as int8 B fragments; the weights enter
// mma.sync m16n8k32 as u8 nibbles (one AND per 4 weights: byte b of a
// transposed ldmatrix register is nibble 2 (b & 1) (+1) of k row b >> 1, and
// B spreads X over two column variants). Products accumulate exactly in
// int32; the fold applies 1 / scale per stage and s (acc - z sum x) per group.
#pragma once

#include "cawq_common.cuh"

namespace cawq {

constexpr int kDecTileCols = 128;  // output columns per strip (consumer warp)
constexpr int kDecTileWords = 16;  // packed words per k row in a strip
constexpr int kDecBoxWords = 32;   // packed words per k row in a weight box (2 strips)
constexpr int kDecStageRows = 64;  // k rows per TMA stage (4 MMA steps)
constexpr int kDecMaxWarps = 8;
constexpr int kDecMaxStages = 8;
// integer path (rows <= 4): B-fragment table and X row info per stage
constexpr int kDecI8MaxRows = 4;
constexpr int kDecI8BTable = 4 * 32 * 16;
constexpr int kDecI8RowInfo = kDecI8MaxRows * 8;
constexpr int kDecI8BSlots = 2;  // B-fragment tables in flight (their own small ring)
constexpr int kDecI8BSlot = kDecI8BTable + kDecI8RowInfo;
constexpr int kDecI8MaxStrips = 4;

// Shared-memory layout of one ring slot:
//   [X tile: XB rows x 64 k, 128B swizzle][W: strips/2 x 64 rows x 128 B, 128B swizzle]
//   [S: gps rows x band columns, F][Z: gps rows x band/8 words]
// gps = quantization groups a 64-row stage can touch.
// Columns of a band each CTA of a split-K cluster sums: the band's 8-column
// words dealt out in equal slices, rounded up (the last slice is shorter
// when split does not divide the words).
__host__ __device__ constexpr uint32_t dec_ncols(uint32_t bcols, uint32_t split) {
  return (bcols / 8 + split - 1) / split * 8;
}

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
  // split-K receive buffer: [source rank][XB rows][dec_ncols] fp32
  static __host__ __device__ size_t recv_bytes(int strips, uint32_t split) {
    return (size_t)XB * split * dec_ncols(static_cast<uint32_t>(strips * kDecTileCols), split) * 4;
  }
  // integer path: after the receive buffer, kDecI8BSlots tables of the
  // stage's B fragments (4 steps x 32 lanes x 16 bytes) and, per X row,
  // {1 / scale, sum(x_int) / scale}
  static size_t smem_bytes(int strips, int stages, uint32_t g, uint32_t split, bool i8 = false) {
    return 1024 /* alignment slack */ + slot_bytes(strips, g) * stages +
           recv_bytes(strips, split) +
           (i8 ? (size_t)kDecI8BSlots * kDecI8BSlot : 0) +
           (size_t)((i8 ? 3 : 2) * stages + (i8 ? 2 * kDecI8BSlots : 0) + 1) * 8;
  }
};

// Consumer warps per CTA (strips x 2 halves), bounded by the register file:
// about 80 registers per thread for 8-row X tiles, 128 for 16.
__host__ __device__ constexpr int dec_max_consumers(int mt) { return mt == 1 ? 16 : 8; }

// The integer path runs at most kDecI8MaxStrips strips and keeps 3 CTAs per
// SM within the register file.
// EPI 1: gate / up columns interleaved in 128-column blocks (strips 2j and
// 2j + 1 of a band are a gate block and its up block); the kernel writes
// silu(gate) * up (bias, if any, added to both first) to an [rows, n / 2]
// output, column (band column base) / 2 + pair index.
//
// PK (f32 X, rows <= 4): the hi and lo bf16 parts of X row j go to B columns
// 2j and 2j + 1 of one MMA instead of two MMAs over columns j; the fold works
// column by column as before, and the two columns of a row are added once,
// after the last group.
template <int DT, int ODT, int ORDER, int MT, bool GA, bool I8, int EPI = 0, bool PK = false>
__global__ void __launch_bounds__(I8 ? (2 * kDecI8MaxStrips + 2) * 32
                                     : dec_max_consumers(MT) * 32 + 32,
                                  I8 ? 3 : 1)
    decode_kernel(const __grid_constant__ CUtensorMap tm_w, const __grid_constant__ CUtensorMap tm_x,
                  const uint32_t* __restrict__ qz, const typename DType<DT>::T* __restrict__ sc,
                  const typename DType<DT>::T* __restrict__ bias,
                  const OutMap<typename DType<ODT>::T> om, uint32_t rows, uint32_t k, uint32_t n,
                  uint32_t g, uint32_t split, uint32_t nstage_ring,
                  uint32_t strips_u, uint32_t pf_stages) {
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
  // warps 0..consumers-1; then the producer; on the integer path the X
  // preparation warp last
  const int consumers = 2 * strips;
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
  uint8_t* btabs = smem + ring_bytes + L::recv_bytes(strips, split);  // integer path: B tables
  uint64_t* full = reinterpret_cast<uint64_t*>(
      btabs + (I8 ? (size_t)kDecI8BSlots * kDecI8BSlot : 0));
  uint64_t* empty = full + NS;
  uint64_t* xfull = empty + NS;              // integer path: the stage's X tile has landed
  uint64_t* bfull = xfull + NS;              // integer path: B table ready / free
  uint64_t* bempty = bfull + kDecI8BSlots;
  uint64_t* recv_bar = I8 ? bempty + kDecI8BSlots : empty + NS;  // peers' partial sums landed
  const uint32_t rows_eff = rows < (uint32_t)XB ? rows : (uint32_t)XB;
  const uint32_t bcols = static_cast<uint32_t>(strips * kDecTileCols);
  // CTA q of the cluster sums the band's columns [q ncols, q ncols + own):
  // slices of whole 8-column words, the last one shorter when split does not
  // divide the band's words
  const uint32_t ncols = dec_ncols(bcols, split);
  const uint32_t own = rank * ncols < bcols ? min(ncols, bcols - rank * ncols) : 0u;
  __shared__ int s_issued;  // stages whose copies the producer lanes issued

  if (threadIdx.x == 0) {
    s_issued = 0;
    for (int s = 0; s < NS; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], static_cast<uint32_t>(consumers + (I8 ? 1 : 0)));
      if constexpr (I8) mbar_init(&xfull[s], 1);
    }
    if constexpr (I8) {
      for (int b = 0; b < kDecI8BSlots; ++b) {
        mbar_init(&bfull[b], 1);
        mbar_init(&bempty[b], static_cast<uint32_t>(consumers));
      }
    }
    mbar_init(recv_bar, 1);
    if (split > 1) mbar_arrive_expect_tx(recv_bar, (split - 1) * rows_eff * own * 4);
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

  bool ok = true;
  if (warp == consumers) {
    // ------------------------------------------------------ TMA producer
    // Up to four lanes issue the stages round robin (stage j by lane j mod
    // np): a thread that issues every stage lands about one 64-row weight box
    // per 0.45-0.5 us, two threads about one per 0.31-0.35 us (measured on
    // B200), and with a stage's four or five copies four lanes gained again in
    // the decode chain. A lane waits for its stage's slot by phase parity,
    // which is only unambiguous while it is at most one phase ahead of the
    // slot: with at least np slots each lane has waited for its own previous
    // stage's release first (consumers release in order), so it is.
    const int np = NS >= 4 ? 4 : NS >= 2 ? 2 : 1;  // issuing lanes (<= ring slots)
    if (lane < np) {
      // valid columns of the band (the bulk copies must stay inside a row)
      const uint32_t bcol0 = pband * 8;
      const uint32_t vcols = min((uint32_t)(strips * kDecTileCols), n - min(n, bcol0));
      const uint32_t ngroups = k / g;
      // integer path: X has its own barrier, so that its preparation does not
      // wait for the stage's weights
      const uint32_t tx = static_cast<uint32_t>((I8 ? 0 : L::kXBytes) + strips * L::kWBytes) +
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
        } else if constexpr (I8) {
          mbar_arrive_expect_tx(&xfull[sl], static_cast<uint32_t>(L::kXBytes));
          tma_load_2d(dst, &tm_x, kr, 0, &xfull[sl]);
        } else {
          tma_load_2d(dst, &tm_x, kr, 0, &full[sl]);
        }
      };
      // stages past the ring: weights, scales and zeros prefetched into L2 only
      auto prefetch_weights = [&](int j) {
        const int kr = static_cast<int>((c_beg + j) * kDecStageRows);
        for (int b = 0; b < strips / 2; ++b)
          tma_prefetch_l2_2d(&tm_w, static_cast<int>(pband + b * kDecBoxWords), kr);
        const uint32_t g0 = (uint32_t)kr / g;
        for (int r = 0; r < gps && vcols; ++r) {
          const uint32_t grp = min(g0 + r, ngroups - 1);
          bulk_prefetch_l2(sc + (size_t)grp * n + bcol0, vcols * sizeof(T));
          bulk_prefetch_l2(qz + (size_t)grp * npk + pband, vcols / 2);
        }
      };
      const int pro = NS < nst ? NS : nst;
      for (int j = lane; j < pro; j += np) issue_weights(j);  // independent of earlier kernels
      if (lane == 0) {
        const int pf_end = (int)min((uint32_t)nst, (uint32_t)pro + pf_stages);
        for (int j = pro; j < pf_end; ++j) prefetch_weights(j);
      }
      pdl_wait();                                       // X may be the previous kernel's output
      for (int j = lane; j < pro; j += np) issue_x(j);
      int issued = pro;
      // this lane's stages: the first j >= pro with j = lane (mod np)
      for (int j = pro + ((lane - pro) % np + np) % np; j < nst && ok; j += np) {
        const int sl = j % NS;
        ok = mbar_wait_bounded(&empty[sl], static_cast<uint32_t>(((j / NS) - 1) & 1));
        if (!ok) break;
        issue_weights(j);
        issue_x(j);
        issued = j + 1;
      }
      // the drain after a failed run waits for the last stages either lane issued
      atomicMax(&s_issued, issued);
    }
    __syncwarp();
  }

  if constexpr (I8) {
    if (warp == consumers + 1) {
      // --------------------------------------------------- X preparation
      // Per stage, each X row (rows <= 4) becomes 16-bit fixed point with a
      // power-of-two scale: |x| < 2^(e+1) over the row's 64 values, so
      // x * 2^(14 - e) rounds into [-2^15, 2^15). The integer splits into a
      // signed high byte and an unsigned low byte (x_int = 256 hi + lo), each
      // the B operand of one integer MMA. Consumer lane (gq, t) reads B column
      // gq = (X row gq >> 1, variant gq & 1): per 16-row step st, word b0 holds
      // the digits of k rows 16 st + 2t, +1 at bytes (variant, variant + 2),
      // b1 those of 16 st + 8 + 2t, +1. Lane L here converts exactly the k
      // pair (2L, 2L + 1) of every live row, i.e. step L >> 3, word
      // (L >> 2) & 1, t = L & 3, and writes it for both variants. The words of
      // the other B columns stay zero (the tables are cleared once). Row r
      // also gets {1 / scale, sum(x_int) / scale}.
      for (int b = 0; b < kDecI8BSlots; ++b) {
        uint4* tab = reinterpret_cast<uint4*>(btabs + (size_t)b * kDecI8BSlot);
        for (int i = lane; i < kDecI8BTable / 16; i += 32) tab[i] = make_uint4(0u, 0u, 0u, 0u);
      }
      __syncwarp();
      const int st_l = lane >> 3;            // 16-row step of this lane's k pair
      const int wsel = (lane >> 2) & 1;      // b0 (0) or b1 (1)
      const int tl = lane & 3;               // t of the consumer lanes served
      const int chunk = lane >> 2;           // 16-byte chunk of the X row (k = 2 lane)
      for (int j = 0; j < nst && ok; ++j) {
        const int sl = j % NS;
        const int bs = j % kDecI8BSlots;
        ok = mbar_wait_bounded(&xfull[sl], static_cast<uint32_t>((j / NS) & 1));
        // the consumers are done with the table this slot held two stages ago
        if (ok && j >= kDecI8BSlots)
          ok = mbar_wait_bounded(&bempty[bs], static_cast<uint32_t>(((j / kDecI8BSlots) - 1) & 1));
        ok = __all_sync(0xffffffffu, ok);
        if (!ok) break;
        const uint8_t* sbase = smem + sl * slot;
        uint8_t* tbase = btabs + (size_t)bs * kDecI8BSlot;
        uint32_t* tab32 = reinterpret_cast<uint32_t*>(tbase);
        float2* info = reinterpret_cast<float2*>(tbase + kDecI8BTable);
        for (int r = 0; r < (int)rows_eff; ++r) {
          const uint32_t w = *reinterpret_cast<const uint32_t*>(
              sbase + r * 128 + ((chunk ^ (r & 7)) << 4) + ((lane & 3) << 2));
          const T* h = reinterpret_cast<const T*>(&w);
          const float x0 = DType<DT>::to_f32(h[0]), x1 = DType<DT>::to_f32(h[1]);
          float mx = fmaxf(fabsf(x0), fabsf(x1));
#pragma unroll
          for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
          // e = floor(log2 mx) from the exponent field (0 and subnormals give a
          // tiny e, clamped so that both scales stay normal floats)
          const int e = max(static_cast<int>((__float_as_uint(mx) >> 23) & 0xFFu) - 127, -100);
          const float scale = __uint_as_float(static_cast<uint32_t>(127 + 14 - e) << 23);
          const float inv = __uint_as_float(static_cast<uint32_t>(127 - 14 + e) << 23);
          const int i0 = min(__float2int_rn(x0 * scale), 32767);
          const int i1 = min(__float2int_rn(x1 * scale), 32767);
          int sum = i0 + i1;
#pragma unroll
          for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
          const uint32_t hi = prmt(static_cast<uint32_t>(i0), static_cast<uint32_t>(i1), 0x0501u) &
                              0x00FF00FFu;  // high bytes of k, k + 1 at bytes 0, 2
          const uint32_t lo = prmt(static_cast<uint32_t>(i0), static_cast<uint32_t>(i1), 0x0400u) &
                              0x00FF00FFu;  // low bytes
#pragma unroll
          for (int v = 0; v < 2; ++v) {
            const int cl = 4 * (2 * r + v) + tl;  // consumer lane served
            uint32_t* ent = tab32 + ((size_t)st_l * 32 + cl) * 4;
            ent[wsel] = hi << (8 * v);
            ent[2 + wsel] = lo << (8 * v);
          }
          if (lane == 0) info[r] = make_float2(inv, static_cast<float>(sum) * inv);
        }
        __syncwarp();
        if (lane == 0) {
          mbar_arrive(&bfull[bs]);
          mbar_arrive(&empty[sl]);
        }
      }
    }
  }

  float tot[MT][4][4];
#pragma unroll
  for (int m = 0; m < MT; ++m)
#pragma unroll
    for (int j = 0; j < 4; ++j)
#pragma unroll
      for (int e = 0; e < 4; ++e) tot[m][j][e] = 0.f;

  // this warp's strip and 64-column half; the lane's two packed words inside
  // the strip (element gq of the warp's 16-byte chunks A and B) and which four
  // nibbles of them it holds (npar 0: nibbles 0-3, npar 1: nibbles 4-7)
  const int strip = warp % strips;
  const int half = (warp / strips) & 1;
  const int wA = 8 * half + (gq >> 1);
  const int wB = wA + 4;
  const int npar = gq & 1;
  int oword = 0;               // the word whose 8 columns this lane writes
  float outv[MT][2][8] = {};   // its sums, rows 8m + 2t + e, column order

  if (warp < consumers) {
    // -------------------------------------------------------- consumers
    // Weights: one ldmatrix.x4.trans per 16-row step. Lane L supplies row
    // L & 7 of matrix L >> 3 (matrices 0 / 1: k rows 0-7 of chunks A / B,
    // 2 / 3: rows 8-15); the 128-byte swizzle moves chunk c of box row r to
    // c ^ (r & 7), which spreads each matrix over all banks.
    uint32_t wld;
    {
      const int mi = lane >> 3, r8 = lane & 7;
      const int chunk = 4 * (strip & 1) + 2 * half + (mi & 1);  // 16-byte chunk in the box row
      wld = L::kXBytes + (strip >> 1) * 2 * L::kWBytes + (8 * (mi >> 1) + r8) * 128 +
            ((chunk ^ r8) << 4);
    }
    // scales of words wA / wB and their zero words inside the stage rows
    const uint32_t s_off[2] = {(uint32_t)(strip * kDecTileCols + 8 * wA) * (uint32_t)sizeof(T),
                               (uint32_t)(strip * kDecTileCols + 8 * wB) * (uint32_t)sizeof(T)};
    const uint32_t z_off[2] = {(uint32_t)(strip * kDecTileWords + wA) * 4,
                               (uint32_t)(strip * kDecTileWords + wB) * 4};

    // this group's 8 scales (s') and zero terms (c') of the lane's columns:
    // nibble 4 npar + n of words wA (slot 0) and wB (slot 1); `zmul` scales
    // the zero of odd nibbles n (their weights entered the MMA as 16 q)
    auto group_scales = [&](const uint8_t* srow, float (&sc)[2][4], float div_odd) {
#pragma unroll
      for (int q = 0; q < 2; ++q) {
        float s8[8];  // the word's 8 scales, column order
        if constexpr (DT == kF32) {
#pragma unroll
          for (int v = 0; v < 2; ++v) {
            const float4 f = *reinterpret_cast<const float4*>(srow + s_off[q] + 16 * v);
            s8[4 * v + 0] = f.x; s8[4 * v + 1] = f.y;
            s8[4 * v + 2] = f.z; s8[4 * v + 3] = f.w;
          }
        } else {
          const uint4 raw = *reinterpret_cast<const uint4*>(srow + s_off[q]);
          const T* h = reinterpret_cast<const T*>(&raw);
#pragma unroll
          for (int c = 0; c < 8; ++c) s8[c] = DType<DT>::to_f32(h[c]);
        }
#pragma unroll
        for (int n = 0; n < 4; ++n) {
          const float s0 = s8[col_of_nibble(n, ORDER)], s1 = s8[col_of_nibble(4 + n, ORDER)];
          sc[q][n] = (npar ? s1 : s0) * ((n & 1) ? div_odd : 1.f);
        }
      }
    };
    // the two zero words, each shifted to the lane's 4 nibbles, packed as
    // (slot 0 | slot 1 << 16)
    auto group_zeros = [&](const uint8_t* zrow) {
      const uint32_t za = *reinterpret_cast<const uint32_t*>(zrow + z_off[0]) >> (16 * npar);
      const uint32_t zb = *reinterpret_cast<const uint32_t*>(zrow + z_off[1]) >> (16 * npar);
      return prmt(za, zb, 0x5410u);
    };

    if constexpr (I8) {
      // ------------------------------------------- consumers, integer path
      // Per 16-row step, nibble masks 0x0F / 0xF0 turn the same ldmatrix.trans
      // registers into u8 A fragments: byte b of a register is nibble 2 (b & 1)
      // (mask 0x0F; nibble 2 (b & 1) + 1 as 16 q with 0xF0) of element gq at k
      // row 2t + (b >> 1), which matches the B fragment's (k row, variant)
      // bytes. D column 2t + v is X row t, column variant v: nibble 2 v + mask
      // of the slot's element. Per stage: D (exact int32, high and low byte
      // MMAs) / scale accumulates per column; per group: tot += s' (acc - z'
      // * sum_k x).
      using Zero = std::integral_constant<bool, true>;
      using NoZero = std::integral_constant<bool, false>;
      float acc[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};  // [slot][n]
      float xs = 0.f;  // sum over the group's stages of sum(x_int) / scale, X row t
      float ti[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};   // [slot][n]
      auto imma = [&](int (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                      uint32_t b0, uint32_t b1, auto zero_tag, auto signed_tag) {
        constexpr bool kZero = decltype(zero_tag)::value;
        constexpr bool kSigned = decltype(signed_tag)::value;
        if constexpr (kZero && kSigned) {
          asm("mma.sync.aligned.m16n8k32.row.col.s32.u8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
              "{%8,%9}, {%10,%10,%10,%10};"
              : "=r"(d[0]), "=r"(d[1]), "=r"(d[2]), "=r"(d[3])
              : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1), "r"(0));
        } else if constexpr (kZero) {
          asm("mma.sync.aligned.m16n8k32.row.col.s32.u8.u8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
              "{%8,%9}, {%10,%10,%10,%10};"
              : "=r"(d[0]), "=r"(d[1]), "=r"(d[2]), "=r"(d[3])
              : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1), "r"(0));
        } else if constexpr (kSigned) {
          asm("mma.sync.aligned.m16n8k32.row.col.s32.u8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
              "{%8,%9}, {%0,%1,%2,%3};"
              : "+r"(d[0]), "+r"(d[1]), "+r"(d[2]), "+r"(d[3])
              : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
        } else {
          asm("mma.sync.aligned.m16n8k32.row.col.s32.u8.u8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
              "{%8,%9}, {%0,%1,%2,%3};"
              : "+r"(d[0]), "+r"(d[1]), "+r"(d[2]), "+r"(d[3])
              : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
        }
      };
      auto fold_i8 = [&](const uint8_t* sbase) {
        float sc[2][4];
        group_scales(sbase + L::s_off(strips), sc, 0.0625f);
        const uint32_t zz = group_zeros(sbase + L::z_off(strips, g));
#pragma unroll
        for (int q = 0; q < 2; ++q) {
#pragma unroll
          for (int n = 0; n < 4; ++n) {
            const float z = static_cast<float>((zz >> (16 * q + 4 * n)) & 15u) * ((n & 1) ? 16.f : 1.f);
            ti[q][n] = fmaf(sc[q][n], fmaf(-z, xs, acc[q][n]), ti[q][n]);
            acc[q][n] = 0.f;
          }
        }
        xs = 0.f;
      };
      int sl = 0;
      uint32_t par = 0;
      const uint32_t spgs = g / kDecStageRows;  // stages per group (g % 64 == 0 here)
      uint32_t in_grp = c_beg % spgs;
      for (int j = 0; j < nst; ++j) {
        const int bs = j % kDecI8BSlots;
        if (ok) ok = mbar_wait_bounded(&full[sl], par);
        if (ok) ok = mbar_wait_bounded(&bfull[bs], static_cast<uint32_t>((j / kDecI8BSlots) & 1));
        ok = __all_sync(0xffffffffu, ok);
        if (!ok) break;
        const uint8_t* sbase = smem + sl * slot;
        const uint8_t* tbase = btabs + (size_t)bs * kDecI8BSlot;
        int Dh[2][4], Dl[2][4];  // [mask][fragment]: high / low byte products
#pragma unroll
        for (int st = 0; st < 4; ++st) {
          uint32_t R[4];
          ldmatrix_x4_trans(smem_u32(sbase) + wld + st * 2048, R[0], R[1], R[2], R[3]);
          const uint4 bt = *reinterpret_cast<const uint4*>(tbase + st * 512 + lane * 16);
#pragma unroll
          for (int mk = 0; mk < 2; ++mk) {
            const uint32_t msk = mk ? 0xF0F0F0F0u : 0x0F0F0F0Fu;
            const uint32_t a0 = R[0] & msk, a1 = R[1] & msk, a2 = R[2] & msk, a3 = R[3] & msk;
            if (st == 0) {
              imma(Dh[mk], a0, a1, a2, a3, bt.x, bt.y, Zero{}, Zero{});
              imma(Dl[mk], a0, a1, a2, a3, bt.z, bt.w, Zero{}, NoZero{});
            } else {
              imma(Dh[mk], a0, a1, a2, a3, bt.x, bt.y, NoZero{}, Zero{});
              imma(Dl[mk], a0, a1, a2, a3, bt.z, bt.w, NoZero{}, NoZero{});
            }
          }
        }
        const float2 ri = *reinterpret_cast<const float2*>(tbase + kDecI8BTable + t * 8);
        xs += ri.y;
#pragma unroll
        for (int mk = 0; mk < 2; ++mk) {
#pragma unroll
          for (int f = 0; f < 4; ++f) {
            // fragment f: slot f >> 1, variant f & 1 -> element nibble 2 (f & 1) + mk
            const float val = static_cast<float>(Dh[mk][f] * 256 + Dl[mk][f]);
            acc[f >> 1][2 * (f & 1) + mk] = fmaf(val, ri.x, acc[f >> 1][2 * (f & 1) + mk]);
          }
        }
        if (++in_grp == spgs || j + 1 == nst) {
          fold_i8(sbase);
          in_grp = 0;
        }
        __syncwarp();
        if (lane == 0) {
          mbar_arrive(&empty[sl]);
          mbar_arrive(&bempty[bs]);
        }
        if (++sl == NS) {
          sl = 0;
          par ^= 1u;
        }
      }
      // exchange with lane gq ^ 1 so that each lane has all 8 columns of one
      // word (X row t)
      oword = npar ? wB : wA;
      float lo[4], hi[4];
#pragma unroll
      for (int n = 0; n < 4; ++n) {
        const float keep = npar ? ti[1][n] : ti[0][n];
        const float send = npar ? ti[0][n] : ti[1][n];
        const float recv = __shfl_xor_sync(0xffffffffu, send, 4);
        lo[n] = npar ? recv : keep;
        hi[n] = npar ? keep : recv;
      }
#pragma unroll
      for (int n = 0; n < 4; ++n) {
        outv[0][0][col_of_nibble(n, ORDER)] = lo[n];
        outv[0][0][col_of_nibble(4 + n, ORDER)] = hi[n];
      }
    } else {
    // X^T fragments. 16-bit X: one ldmatrix.x4 per 8-row block of X loads the
    // fragments of two steps; lane L gives the address of row 8m + (L & 7),
    // 16-byte k chunk 4p + (L >> 3) of step pair p, under the tile's 128-byte
    // swizzle. f32 X: each k pair is loaded directly and split into bf16 hi/lo.
    uint32_t xrow[MT];    // byte offset of row 8m + gq (f32 X)
    uint32_t x7[MT];      // its swizzle phase
    uint32_t xld[MT][2];  // ldmatrix row addresses, step pairs 0 and 1 (16-bit X)
#pragma unroll
    for (int m = 0; m < MT; ++m) {
      const int xr = PK ? (gq >> 1) : 8 * m + gq;  // PK: B column gq holds row gq / 2
      xrow[m] = xr * 128;
      x7[m] = static_cast<uint32_t>(xr & 7);
      const int lr = lane & 7, li = lane >> 3;
#pragma unroll
      for (int p = 0; p < 2; ++p)
        xld[m][p] = static_cast<uint32_t>((8 * m + lr) * 128 + (((4 * p + li) ^ lr) << 4));
    }

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
    // stage's shared-memory rows (see the file comment), for the lane's 8
    // columns: nibble 4 npar + n of words wA (slot 0) and wB (slot 1). c' =
    // offset + zero is built by the same magic-number lop3 as the weights: for
    // f16 nibbles n = 0, 2 give 1024 + z and n = 1, 3, in place, 1024 + 16 z
    // (their weights entered the MMA as 16 q); for bf16 every nibble gives
    // 128 + z. With `clear` the accumulators restart at 0; else the next
    // group's first MMA overwrites them.
    auto fold = [&](const uint8_t* srow, const uint8_t* zrow, auto clear_tag) {
      constexpr bool kClear = decltype(clear_tag)::value;
      float sc[2][4];  // [slot][n] scale of nibble 4 npar + n
#pragma unroll
      for (int q = 0; q < 2; ++q) {
        float s8[8];  // the word's 8 scales, column order
        if constexpr (DT == kF32) {
#pragma unroll
          for (int v = 0; v < 2; ++v) {
            const float4 f = *reinterpret_cast<const float4*>(srow + s_off[q] + 16 * v);
            s8[4 * v + 0] = f.x; s8[4 * v + 1] = f.y;
            s8[4 * v + 2] = f.z; s8[4 * v + 3] = f.w;
          }
        } else {
          const uint4 raw = *reinterpret_cast<const uint4*>(srow + s_off[q]);
          const T* h = reinterpret_cast<const T*>(&raw);
#pragma unroll
          for (int c = 0; c < 8; ++c) s8[c] = DType<DT>::to_f32(h[c]);
        }
#pragma unroll
        for (int n = 0; n < 4; ++n) {
          const float s0 = s8[col_of_nibble(n, ORDER)], s1 = s8[col_of_nibble(4 + n, ORDER)];
          sc[q][n] = npar ? s1 : s0;
          if constexpr (kF16Mma) {
            if (n & 1) sc[q][n] *= 0.0625f;  // the nibble entered the MMA as 16 q
          }
        }
      }
      // the two zero words, each shifted to the lane's 4 nibbles, packed as
      // (slot 0 | slot 1 << 16): one lop3 gives c' of both slots
      const uint32_t za = *reinterpret_cast<const uint32_t*>(zrow + z_off[0]) >> (16 * npar);
      const uint32_t zb = *reinterpret_cast<const uint32_t*>(zrow + z_off[1]) >> (16 * npar);
      const uint32_t zz = prmt(za, zb, 0x5410u);
      float cz[2][4];
#pragma unroll
      for (int n = 0; n < 4; ++n) {
        if constexpr (kF16Mma) {
          const uint32_t src = n < 2 ? zz : (zz >> 8);
          const uint32_t q = lop3_and_or(src, (n & 1) ? 0x00F000F0u : 0x000F000Fu, 0x64006400u);
          const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&q));
          cz[0][n] = f.x;
          cz[1][n] = f.y;
        } else {
          const uint32_t q = lop3_and_or(zz >> (4 * n), 0x000F000Fu, 0x43004300u);
          cz[0][n] = __uint_as_float(q << 16);
          cz[1][n] = __uint_as_float(q & 0xFFFF0000u);
        }
      }
#pragma unroll
      for (int n = 0; n < 4; ++n) {
#pragma unroll
        for (int m = 0; m < MT; ++m) {
          tot[m][n][0] = fmaf(sc[0][n], fmaf(-cz[0][n], Dx[m][0], D[m][n][0]), tot[m][n][0]);
          tot[m][n][1] = fmaf(sc[0][n], fmaf(-cz[0][n], Dx[m][1], D[m][n][1]), tot[m][n][1]);
          tot[m][n][2] = fmaf(sc[1][n], fmaf(-cz[1][n], Dx[m][0], D[m][n][2]), tot[m][n][2]);
          tot[m][n][3] = fmaf(sc[1][n], fmaf(-cz[1][n], Dx[m][1], D[m][n][3]), tot[m][n][3]);
          if constexpr (kClear) D[m][n][0] = D[m][n][1] = D[m][n][2] = D[m][n][3] = 0.f;
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
          if constexpr (PK) {  // column gq: the hi part of row gq / 2, or its lo part
            bh[m][h2] = (gq & 1) ? *reinterpret_cast<const uint32_t*>(&lo)
                                 : *reinterpret_cast<const uint32_t*>(&hi);
          } else {
            bh[m][h2] = *reinterpret_cast<const uint32_t*>(&hi);
            bl[m][h2] = *reinterpret_cast<const uint32_t*>(&lo);
          }
        }
      }
    };

    // one 16-row step with X^T fragments bh (and the bf16 lo parts bl of f32 X):
    // the ones MMA, dequantize and multiply. R[0..3] hold, per lane, element
    // gq of chunks A / B at k rows (2t, 2t + 1) and (2t + 8, 2t + 9): nibble n
    // of each half is column n of the lane's slot, so one lop3 per register
    // and nibble gives the f16 pair (magic + q[k], magic + q[k + 1]), the A
    // fragment of MMA n.
    auto step_mma = [&](const uint8_t* sbase, int s, const uint32_t (&bh)[MT][2],
                        const uint32_t (&bl)[MT][2], auto zero_tag) {
      uint32_t R[4];
      ldmatrix_x4_trans(smem_u32(sbase) + wld + s * 2048, R[0], R[1], R[2], R[3]);
#pragma unroll
      for (int m = 0; m < MT; ++m) {
        mma(Dx[m], kOnes, kOnes, kOnes, kOnes, bh[m][0], bh[m][1], zero_tag);
        if constexpr (DT == kF32 && !PK)
          mma_16816<true>(Dx[m], kOnes, kOnes, kOnes, kOnes, bl[m][0], bl[m][1]);
      }
      [[maybe_unused]] uint32_t Rh[4];
      if constexpr (kF16Mma) {
#pragma unroll
        for (int i = 0; i < 4; ++i) Rh[i] = R[i] >> 8;
      }
#pragma unroll
      for (int n = 0; n < 4; ++n) {
        uint32_t a[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          if constexpr (kF16Mma) {
            // nibbles 0, 1 in place (1024 + q, 1024 + 16 q); 2, 3 after >> 8
            a[i] = lop3_and_or(n < 2 ? R[i] : Rh[i], (n & 1) ? 0x00F000F0u : 0x000F000Fu,
                               0x64006400u);
          } else {
            a[i] = lop3_and_or(n ? (R[i] >> (4 * n)) : R[i], 0x000F000Fu, 0x43004300u);
          }
        }
#pragma unroll
        for (int m = 0; m < MT; ++m) {
          mma(D[m][n], a[0], a[1], a[2], a[3], bh[m][0], bh[m][1], zero_tag);
          if constexpr (DT == kF32 && !PK)
            mma_16816<true>(D[m][n], a[0], a[1], a[2], a[3], bl[m][0], bl[m][1]);
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

    if constexpr (PK) {  // columns 2t (hi) + 2t + 1 (lo) = row t
#pragma unroll
      for (int n = 0; n < 4; ++n) {
        tot[0][n][0] += tot[0][n][1];
        tot[0][n][2] += tot[0][n][3];
      }
    }
    // Lanes gq and gq ^ 1 hold the two nibble halves of words wA and wB: swap
    // one slot so that each lane has all 8 columns of one word.
    oword = npar ? wB : wA;
#pragma unroll
    for (int m = 0; m < MT; ++m) {
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        float lo[4], hi[4];  // nibbles 0-3 and 4-7 of oword
#pragma unroll
        for (int n = 0; n < 4; ++n) {
          const float keep = npar ? tot[m][n][2 + e] : tot[m][n][e];
          const float send = npar ? tot[m][n][e] : tot[m][n][2 + e];
          const float recv = __shfl_xor_sync(0xffffffffu, send, 4);
          lo[n] = npar ? recv : keep;
          hi[n] = npar ? keep : recv;
        }
#pragma unroll
        for (int n = 0; n < 4; ++n) {
          outv[m][e][col_of_nibble(n, ORDER)] = lo[n];
          outv[m][e][col_of_nibble(4 + n, ORDER)] = hi[n];
        }
      }
    }
    }  // f16 / bf16 tensor path
  }

  // Before exiting, no copy this CTA issued may still be writing its shared
  // memory. Normally every issued stage has been consumed; after a timed-out
  // wait, wait (bounded) for the last stage issued into each slot.
  auto drain = [&]() {
    if (!__syncthreads_or(ok ? 0 : 1)) return;
    if (threadIdx.x == 0) {
      const int issued = s_issued;
      for (int j = issued > NS ? issued - NS : 0; j < issued; ++j) {
        mbar_wait_bounded(&full[j % NS], static_cast<uint32_t>((j / NS) & 1));
        if constexpr (I8) mbar_wait_bounded(&xfull[j % NS], static_cast<uint32_t>((j / NS) & 1));
      }
    }
    __syncthreads();
  };

  // ---- split-K sums. CTA q of the cluster owns columns [q ncols, (q+1) ncols)
  // of the band: every CTA stores its partial sums of those columns into
  // slot [its rank] of q's receive buffer (st.async to distributed shared
  // memory, counted on q's recv_bar), then sums its own columns over the
  // slots in rank order. One wait, no cluster-wide barrier at the end.
  // SiLU-gated output of pair index pi of this band from its gate / up sums
  auto store_pair = [&](uint32_t row, uint32_t pi, float gv, float uv) {
    const uint32_t wcol = pband * 8 + (pi / 128) * 256 + (pi & 127u);  // gate weight column
    if (wcol >= n) return;
    if (bias) {
      gv += DType<DT>::to_f32(bias[wcol]);
      uv += DType<DT>::to_f32(bias[wcol + 128]);
    }
    om.p0[(size_t)row * om.ld0 + pband * 4 + pi] = DType<ODT>::from_f32(silu_mul(gv, uv));
  };
  if (split == 1 && EPI == 1) {
    // the band's sums meet in the receive buffer (unused without split K):
    // [row][band column], then the consumer threads pair gate with up
    if (warp < consumers) {
#pragma unroll
      for (int m = 0; m < MT; ++m) {
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          const uint32_t row = static_cast<uint32_t>(8 * m + 2 * t + e);
          if (row >= rows_eff) continue;
          float* dst = recv + (size_t)row * bcols + strip * kDecTileCols + 8 * oword;
          reinterpret_cast<float4*>(dst)[0] =
              make_float4(outv[m][e][0], outv[m][e][1], outv[m][e][2], outv[m][e][3]);
          reinterpret_cast<float4*>(dst)[1] =
              make_float4(outv[m][e][4], outv[m][e][5], outv[m][e][6], outv[m][e][7]);
        }
      }
      named_bar_sync(1, 32 * consumers);
      const uint32_t npairs = bcols / 2;
      for (uint32_t idx = threadIdx.x; idx < rows_eff * npairs; idx += 32 * consumers) {
        const uint32_t row = idx / npairs, pi = idx - row * npairs;
        const uint32_t gb = (pi / 128) * 256 + (pi & 127u);  // band column of the gate
        store_pair(row, pi, recv[(size_t)row * bcols + gb], recv[(size_t)row * bcols + gb + 128]);
      }
    }
    drain();
    return;
  }
  if (split == 1) {
    if (warp < consumers) {
#pragma unroll
      for (int m = 0; m < MT; ++m) {
#pragma unroll
        for (int e = 0; e < (I8 || PK ? 1 : 2); ++e) {
          // integer and packed paths: lane row t; else rows 8m + 2t + e
          const uint32_t row = static_cast<uint32_t>(I8 || PK ? t : 8 * m + 2 * t + e);
          if (row >= rows_eff) continue;
#pragma unroll
          for (int c = 0; c < 8; ++c) {
            const uint32_t col = pband * 8 + strip * kDecTileCols + 8 * oword + c;
            if (col < n) {
              float v = outv[m][e][c];
              if (bias) v += DType<DT>::to_f32(bias[col]);
              om.template put<EPI == 2>(om.at(row, col), DType<ODT>::from_f32(v));
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
      for (int e = 0; e < (I8 || PK ? 1 : 2); ++e) {
        const uint32_t row = static_cast<uint32_t>(I8 || PK ? t : 8 * m + 2 * t + e);
        if (row >= rows_eff) continue;
        const float* v = outv[m][e];  // this lane's 8 consecutive columns
        const uint32_t col8 = static_cast<uint32_t>(strip * kDecTileCols + 8 * oword);
        // owner and place in its slot: plain, column slices of the band;
        // EPI 1, slices of the band's gate / up pairs (gate part, then up part)
        uint32_t q, pos;
        if constexpr (EPI == 1) {
          const uint32_t npair = ncols / 2;
          const uint32_t w = col8 & 255u;
          const uint32_t pi = (col8 / 256) * 128 + (w & 127u);
          q = pi / npair;
          pos = (pi - q * npair) + (w >= 128 ? npair : 0u);
        } else {
          q = col8 / ncols;
          pos = col8 - q * ncols;
        }
        float* dst = recv + ((size_t)rank * XB + row) * ncols + pos;
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
  if constexpr (EPI == 1) {
    const uint32_t npair = ncols / 2;
    for (uint32_t idx = threadIdx.x; idx < rows_eff * npair; idx += blockDim.x) {
      const uint32_t row = idx / npair, p = idx - row * npair;
      float gv = 0.f, uv = 0.f;
      for (uint32_t src = 0; src < split; ++src) {
        const float* rp = recv + ((size_t)src * XB + row) * ncols;
        gv += rp[p];
        uv += rp[p + npair];
      }
      store_pair(row, rank * npair + p, gv, uv);
    }
  } else {
    for (uint32_t idx = threadIdx.x; idx < rows_eff * own; idx += blockDim.x) {
      const uint32_t row = idx / own, c = idx - row * own;
      const uint32_t col = pband * 8 + rank * ncols + c;
      float v = 0.f;
      for (uint32_t src = 0; src < split; ++src) v += recv[((size_t)src * XB + row) * ncols + c];
      if (col < n) {
        if (bias) v += DType<DT>::to_f32(bias[col]);
        om.template put<EPI == 2>(om.at(row, col), DType<ODT>::from_f32(v));
      }
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

// plan.reserved[2] = 1 selects the integer tensor path (int8 MMA on exact
// 16-bit fixed-point X) where it applies: rows <= 4, 16-bit X, groups that
// are whole 64-row stages. Off by default: its larger stage slots and extra
// warp hold fewer CTAs per SM, which costs more than its faster inner loop
// gains in chains of dependent launches.
static bool decode_use_i8(const GemmProblem& p, const cawq_plan& plan) {
  return plan.reserved[2] == 1 && p.epi == 0 && p.nrep == 0 &&
         p.rows <= (size_t)kDecI8MaxRows && p.dtype != kF32 &&
         p.g % kDecStageRows == 0 && plan.warps <= kDecI8MaxStrips;
}

static size_t decode_smem(const GemmProblem& p, const cawq_plan& plan) {
  const uint32_t g = static_cast<uint32_t>(p.g);
  const bool mt1 = decode_mt(p.rows) == 1;
  const bool i8 = decode_use_i8(p, plan);
  const uint32_t sp = plan.split < 1 ? 1u : static_cast<uint32_t>(plan.split);
  if (p.dtype == kF32) {
    return mt1 ? DecodeLayout<kF32, 1>::smem_bytes(plan.warps, plan.stages, g, sp)
               : DecodeLayout<kF32, 2>::smem_bytes(plan.warps, plan.stages, g, sp);
  }
  return mt1 ? DecodeLayout<kF16, 1>::smem_bytes(plan.warps, plan.stages, g, sp, i8)
             : DecodeLayout<kF16, 2>::smem_bytes(plan.warps, plan.stages, g, sp);
}

bool decode_supports(const GemmProblem& p, const cawq_plan& plan, const DeviceInfo& dev) {
  if (p.rows == 0 || p.rows > 16) return false;
  if (p.k % 16 != 0 || p.g % 16 != 0 || p.k % p.g != 0 || p.n % 32 != 0) return false;
  if (p.k >= (1ull << 31) || p.n >= (1ull << 31) || p.ld_out >= (1ull << 31)) return false;
  const uintptr_t ax = reinterpret_cast<uintptr_t>(p.x), aw = reinterpret_cast<uintptr_t>(p.qw);
  const uintptr_t az = reinterpret_cast<uintptr_t>(p.qz), as = reinterpret_cast<uintptr_t>(p.sc);
  if (ax % 16 || aw % 16 || az % 16 || as % 16) return false;
  if (plan.split < 1 || plan.split > 16) return false;
  // any cluster size for the plain epilogue; powers of two for the SiLU one
  if (p.epi == 1 && (plan.split & (plan.split - 1))) return false;
  if (plan.tile_n > 1) return false;
  if (plan.warps < 2 || (plan.warps & 1) || 2 * plan.warps > dec_max_consumers(decode_mt(p.rows)))
    return false;
  if (plan.stages < 1 || plan.stages > kDecMaxStages) return false;
  if (plan.reserved[2] < 0 || plan.reserved[2] > 1) return false;
  // SiLU-gated epilogue: whole 256-column gate / up blocks, AWQ order, output
  // in the input dtype
  if (p.epi == 1 && (p.n % 256 != 0 || p.order != kOrderAwq || p.out_dtype != p.dtype))
    return false;
  // replicated output (tensor-parallel push): plain epilogue, one output
  // range, f16 / bf16 activations, AWQ order
  if (p.nrep > 0 && (p.epi != 0 || p.out_k || p.dtype == kF32 || p.order != kOrderAwq))
    return false;
  const size_t bands =
      (p.n + (size_t)kDecTileCols * plan.warps - 1) / ((size_t)kDecTileCols * plan.warps);
  if (bands * plan.split >= (1ull << 31)) return false;
  return decode_smem(p, plan) <= dev.smem_optin && dev.cc_major == 10;
}

template <int DT, int ODT, int ORDER, int MT, bool GA, bool I8, int EPI = 0, bool PK = false>
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
  auto kern = decode_kernel<DT, ODT, ORDER, MT, GA, I8, EPI, PK>;
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
  cfg.blockDim = dim3((2 * plan.warps + (I8 ? 2 : 1)) * 32);
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
                            static_cast<const T*>(p.bias), out_map<OT>(p),
                            static_cast<uint32_t>(p.rows), static_cast<uint32_t>(p.k),
                            static_cast<uint32_t>(p.n), static_cast<uint32_t>(p.g),
                            static_cast<uint32_t>(plan.split),
                            static_cast<uint32_t>(plan.stages), static_cast<uint32_t>(plan.warps),
                            static_cast<uint32_t>(plan.reserved[1] > 0 ? plan.reserved[1] : 0));
}

template <int DT, int ODT, int ORDER>
static cudaError_t launch_decode_m(const GemmProblem& p, const cawq_plan& plan) {
  const bool ga = p.g % kDecStageRows == 0;  // groups end on stage boundaries
  if (p.nrep > 0) {
    // EPI 2: the plain epilogue, each element also stored to the replicas
    if constexpr (DT != kF32 && ORDER == kOrderAwq) {
      if (decode_mt(p.rows) == 1) {
        return ga ? launch_decode_t<DT, ODT, ORDER, 1, true, false, 2>(p, plan)
                  : launch_decode_t<DT, ODT, ORDER, 1, false, false, 2>(p, plan);
      }
      return ga ? launch_decode_t<DT, ODT, ORDER, 2, true, false, 2>(p, plan)
                : launch_decode_t<DT, ODT, ORDER, 2, false, false, 2>(p, plan);
    }
    return cudaErrorInvalidValue;
  }
  if constexpr (DT == ODT && ORDER == kOrderAwq) {
    if (p.epi == 1) {
      if (decode_mt(p.rows) == 1) {
        return ga ? launch_decode_t<DT, ODT, ORDER, 1, true, false, 1>(p, plan)
                  : launch_decode_t<DT, ODT, ORDER, 1, false, false, 1>(p, plan);
      }
      return ga ? launch_decode_t<DT, ODT, ORDER, 2, true, false, 1>(p, plan)
                : launch_decode_t<DT, ODT, ORDER, 2, false, false, 1>(p, plan);
    }
  }
  if constexpr (DT != kF32) {
    if (decode_use_i8(p, plan)) return launch_decode_t<DT, ODT, ORDER, 1, true, true>(p, plan);
  } else {
    if (p.rows <= 4) {  // hi / lo of X in the columns of one MMA
      return ga ? launch_decode_t<DT, ODT, ORDER, 1, true, false, 0, true>(p, plan)
                : launch_decode_t<DT, ODT, ORDER, 1, false, false, 0, true>(p, plan);
    }
  }
  if (decode_mt(p.rows) == 1) {
    return ga ? launch_decode_t<DT, ODT, ORDER, 1, true, false>(p, plan)
              : launch_decode_t<DT, ODT, ORDER, 1, false, false>(p, plan);
  }
  return ga ? launch_decode_t<DT, ODT, ORDER, 2, true, false>(p, plan)
            : launch_decode_t<DT, ODT, ORDER, 2, false, false>(p, plan);
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
  // (at least 3 stages per CTA after the doubling: short-K narrow layers,
  // e.g. Qwen2-7B o_proj / qkv, measured fastest at split 16 with 3.5 stages)
  while (split < 16 && bands * split < 2 * sms && nst_total >= (size_t)split * 6) split *= 2;
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

// cawq_tp.cuh — helper kernels of the tensor-parallel layers:
//   * interleave_columns: turns the rank-major result of an all-gather of
//     column shards, src[world][rows][n/world], back into the row-major
//     output dst[rows][n];
//   * rowpar_finish: out[rows][n] = F(partial + bias) after the fp32
//     all-reduce of a row-parallel layer (the bias is added once, after the
//     full sum, as the single-device layer does);
//   * interleave_gate_up: the block-interleaved gate / up column order of
//     the SiLU-gated GEMM, from the plain [gate | up] layout;
//   * p2p_*_finish: the signal / wait / gather or reduce step that follows a
//     GEMM whose epilogue pushed its output into the other ranks' buffers.
#pragma once

#include <mutex>

#include "cawq_common.cuh"

namespace cawq {

template <typename V>
__global__ void __launch_bounds__(256)
    interleave_columns_kernel(const V* __restrict__ src, V* __restrict__ dst, size_t rows,
                              size_t shard_v, int world) {
  // shard_v: vectors of type V per shard row; dst row has world * shard_v vectors
  const size_t total = rows * shard_v * world;
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < total;
       i += (size_t)gridDim.x * blockDim.x) {
    const size_t row = i / (shard_v * world);
    const size_t rem = i - row * shard_v * world;
    const size_t r = rem / shard_v;
    const size_t c = rem - r * shard_v;
    dst[i] = src[(r * rows + row) * shard_v + c];
  }
}

cudaError_t launch_interleave_columns(const void* src, void* dst, size_t rows, size_t n, int world,
                                      size_t elem, cudaStream_t stream) {
  const size_t shard_bytes = n / world * elem;
  const bool v16 = shard_bytes % 16 == 0 && reinterpret_cast<uintptr_t>(src) % 16 == 0 &&
                   reinterpret_cast<uintptr_t>(dst) % 16 == 0;
  const size_t total_bytes = rows * n * elem;
  const size_t vec = v16 ? 16 : elem;
  size_t blocks = (total_bytes / vec + 255) / 256;
  if (blocks > 4096) blocks = 4096;
  if (blocks < 1) blocks = 1;
  if (v16) {
    interleave_columns_kernel<uint4><<<(unsigned)blocks, 256, 0, stream>>>(
        static_cast<const uint4*>(src), static_cast<uint4*>(dst), rows, shard_bytes / 16, world);
  } else if (elem == 4) {
    interleave_columns_kernel<uint32_t><<<(unsigned)blocks, 256, 0, stream>>>(
        static_cast<const uint32_t*>(src), static_cast<uint32_t*>(dst), rows, shard_bytes / 4,
        world);
  } else {
    interleave_columns_kernel<uint16_t><<<(unsigned)blocks, 256, 0, stream>>>(
        static_cast<const uint16_t*>(src), static_cast<uint16_t*>(dst), rows, shard_bytes / 2,
        world);
  }
  return cudaGetLastError();
}

template <int DT>
__global__ void __launch_bounds__(256)
    rowpar_finish_kernel(const float* __restrict__ partial, const typename DType<DT>::T* bias,
                         typename DType<DT>::T* out, size_t rows, size_t n) {
  const size_t total = rows * n;
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < total;
       i += (size_t)gridDim.x * blockDim.x) {
    float v = partial[i];
    if (bias) v += DType<DT>::to_f32(bias[i % n]);
    out[i] = DType<DT>::from_f32(v);
  }
}

cudaError_t launch_rowpar_finish(const float* partial, const void* bias, void* out, size_t rows,
                                 size_t n, int dtype, cudaStream_t stream) {
  size_t blocks = (rows * n + 255) / 256;
  if (blocks > 4096) blocks = 4096;
  if (blocks < 1) blocks = 1;
  const unsigned b = static_cast<unsigned>(blocks);
  if (dtype == kF32) {
    rowpar_finish_kernel<kF32><<<b, 256, 0, stream>>>(partial, static_cast<const float*>(bias),
                                                      static_cast<float*>(out), rows, n);
  } else if (dtype == kF16) {
    rowpar_finish_kernel<kF16><<<b, 256, 0, stream>>>(partial, static_cast<const __half*>(bias),
                                                      static_cast<__half*>(out), rows, n);
  } else {
    rowpar_finish_kernel<kBF16><<<b, 256, 0, stream>>>(
        partial, static_cast<const __nv_bfloat16*>(bias), static_cast<__nv_bfloat16*>(out), rows,
        n);
  }
  return cudaGetLastError();
}

// [gate | up] (width_e elements each per row) -> blocks of block_e elements
// alternating gate, up, gate, ... (the column order of cawq_gemm_silu_mul).
template <typename V>
__global__ void __launch_bounds__(256)
    interleave_gate_up_kernel(const V* __restrict__ src, V* __restrict__ dst, size_t rows,
                              size_t width_e, size_t block_e) {
  const size_t row_e = 2 * width_e;
  const size_t total = rows * row_e;
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < total;
       i += (size_t)gridDim.x * blockDim.x) {
    const size_t r = i / row_e, c = i - r * row_e;  // destination element
    const size_t j = c / (2 * block_e), w = c - j * 2 * block_e;
    const size_t half = w / block_e, e = w - half * block_e;
    dst[i] = src[r * row_e + half * width_e + j * block_e + e];
  }
}

cudaError_t launch_interleave_gate_up(const void* src, void* dst, size_t rows, size_t width_e,
                                      size_t block_e, size_t elem, cudaStream_t stream) {
  const size_t total = rows * 2 * width_e;
  size_t blocks = (total + 255) / 256;
  if (blocks > 65535 * 16) blocks = 65535 * 16;
  if (blocks == 0) return cudaSuccess;
  if (elem == 4) {
    interleave_gate_up_kernel<uint32_t><<<(unsigned)blocks, 256, 0, stream>>>(
        static_cast<const uint32_t*>(src), static_cast<uint32_t*>(dst), rows, width_e, block_e);
  } else {
    interleave_gate_up_kernel<uint16_t><<<(unsigned)blocks, 256, 0, stream>>>(
        static_cast<const uint16_t*>(src), static_cast<uint16_t*>(dst), rows, width_e, block_e);
  }
  return cudaGetLastError();
}

// ------------------------------------------- fused tensor-parallel push
// Every block publishes the epoch to each peer (a repeated store of the same
// value is harmless), then one thread per block waits, bounded, for every
// peer's epoch in this rank's own flag words. The data the flags cover was
// written by the previous kernel of the stream (the GEMM's replicated
// epilogue), which has completed when this kernel starts; the system-scope
// fence and release store publish it, the acquire load and the block barrier
// make it visible to the block's readers. On timeout: bit 1 of the device
// error word, and the block does nothing more.
// flags[j] by selects, so the kernel parameter is not copied to local memory
__device__ __forceinline__ uint32_t* p2p_flags(const P2PSync& s, int j) {
  uint32_t* p = s.flags[0];
#pragma unroll
  for (int i = 1; i < kP2PMaxWorld; ++i)
    if (j == i) p = s.flags[i];
  return p;
}

__device__ __forceinline__ bool p2p_signal_and_wait(const P2PSync& s) {
  __shared__ int ok;
  if (threadIdx.x < static_cast<unsigned>(s.world) && threadIdx.x != static_cast<unsigned>(s.rank)) {
    __threadfence_system();
    uint32_t* f = p2p_flags(s, threadIdx.x) + s.fofs + s.rank;
    asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(f), "r"(s.epoch) : "memory");
  }
  if (threadIdx.x == 0) {
    int good = 1;
    const uint64_t t0 = globaltimer_ns();
    for (int j = 0; j < s.world && good; ++j) {
      if (j == s.rank) continue;
      const uint32_t* f = p2p_flags(s, s.rank) + s.fofs + j;
      for (uint32_t it = 0;; ++it) {
        uint32_t v;
        asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(f) : "memory");
        if (static_cast<int32_t>(v - s.epoch) >= 0) break;
        if ((it & 15u) == 15u && globaltimer_ns() - t0 > s.timeout_ns) {
          atomicOr(&g_cawq_device_error, 2u);
          good = 0;
          break;
        }
      }
    }
    ok = good;
  }
  __syncthreads();
  return ok != 0;
}

template <typename V>
__global__ void __launch_bounds__(256)
    p2p_colpar_finish_kernel(const P2PSync s, const V* __restrict__ slot, V* __restrict__ out,
                             size_t rows, size_t nv, size_t ldv) {
  if (!p2p_signal_and_wait(s)) return;
  const size_t total = rows * nv;
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < total;
       i += (size_t)gridDim.x * blockDim.x) {
    const size_t r = i / nv, c = i - r * nv;
    out[r * ldv + c] = __ldcg(slot + i);  // L2: peers wrote it
  }
}

template <int DT>
__global__ void __launch_bounds__(256)
    p2p_rowpar_finish_kernel(const P2PSync s, const float* __restrict__ slot,
                             const typename DType<DT>::T* __restrict__ bias,
                             typename DType<DT>::T* __restrict__ out, size_t rows, size_t n) {
  if (!p2p_signal_and_wait(s)) return;
  const size_t quads = rows * n / 4;  // n % 4 == 0
  const size_t plane = rows * n;
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < quads;
       i += (size_t)gridDim.x * blockDim.x) {
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int j = 0; j < s.world; ++j) {  // rank order: the same sum on every rank
      const float4 f = __ldcg(reinterpret_cast<const float4*>(slot + j * plane) + i);
      acc.x += f.x; acc.y += f.y; acc.z += f.z; acc.w += f.w;
    }
    const size_t e0 = 4 * i, c = e0 % n;
    const float v[4] = {acc.x, acc.y, acc.z, acc.w};
#pragma unroll
    for (int e = 0; e < 4; ++e)
      out[e0 + e] = DType<DT>::from_f32(v[e] + (bias ? DType<DT>::to_f32(bias[c + e]) : 0.f));
  }
}

// ------------------------------------- fused tensor-parallel, large outputs
// For large outputs the GEMM writes only into this rank's own buffer (stores
// over NVLink inside the epilogue stall it), and separate kernels after it
// push the data to the peers: plain 16-byte stores, which are posted, so the
// links stay busy (reading the peers' buffers instead reached about half the
// rate). A peer's slot is not overwritten while the peer still reads it: this
// rank writes slot (epoch & 1) again only two epochs later, after waiting for
// the peer's flag of the epoch in between, which the peer publishes only in a
// later kernel of its stream than its reads.

__device__ __forceinline__ const uint8_t* p2p_base(const P2PSync& s, int j) {
  return reinterpret_cast<const uint8_t*>(p2p_flags(s, j));
}

// Copies, for every row, the column chunks of the other ranks (chunk o =
// vectors [o cwv, (o+1) cwv) of a row of nv 16-byte vectors) from this
// rank's buffer at byte offset `off` (dense [rows, nv], where the other
// ranks pushed them) into out (same layout). Four loads in flight per thread.
__device__ __forceinline__ void p2p_copy_other_chunks(const P2PSync& s, size_t off,
                                                      uint4* __restrict__ out, size_t rows,
                                                      size_t nv) {
  constexpr int kU = 4;
  const size_t cwv = nv / s.world;      // 16-byte vectors per chunk row
  const size_t per_row = nv - cwv;      // outside the own chunk
  const size_t total = rows * per_row;
  const size_t own0 = (size_t)s.rank * cwv;
  const uint4* src = reinterpret_cast<const uint4*>(p2p_base(s, s.rank) + off);
  const size_t stride = (size_t)gridDim.x * blockDim.x;
  for (size_t i0 = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i0 < total; i0 += kU * stride) {
    uint4 v[kU];
    size_t at[kU];
#pragma unroll
    for (int u = 0; u < kU; ++u) {
      const size_t i = i0 + u * stride;
      at[u] = ~static_cast<size_t>(0);
      if (i < total) {
        const size_t r = i / per_row;
        size_t c = i - r * per_row;
        if (c >= own0) c += cwv;
        at[u] = r * nv + c;
        v[u] = __ldcg(src + at[u]);  // L2: peers wrote it
      }
    }
#pragma unroll
    for (int u = 0; u < kU; ++u)
      if (at[u] != ~static_cast<size_t>(0)) out[at[u]] = v[u];
  }
}

// Column-parallel all-gather of large outputs, step 1 (no flags; the GEMM
// before it has completed and wrote this rank's columns into its own slot,
// dense [rows, nv] at byte offset `off`, and into out): copy this rank's
// chunk of every row into the same place of every other rank's slot. Stores
// over NVLink are posted, so the links stay busy without the round trip a
// peer load waits for; four vectors in flight per thread.
__global__ void __launch_bounds__(256)
    p2p_colpar_push_kernel(const P2PSync s, size_t off, size_t rows, size_t nv) {
  constexpr int kU = 4;
  const size_t cwv = nv / s.world;
  const size_t total = rows * cwv;
  const size_t own0 = (size_t)s.rank * cwv;
  const uint4* src = reinterpret_cast<const uint4*>(p2p_base(s, s.rank) + off);
  const size_t stride = (size_t)gridDim.x * blockDim.x;
  for (size_t i0 = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i0 < total; i0 += kU * stride) {
    uint4 v[kU];
    size_t at[kU];
#pragma unroll
    for (int u = 0; u < kU; ++u) {
      const size_t i = i0 + u * stride;
      at[u] = ~static_cast<size_t>(0);
      if (i < total) {
        const size_t r = i / cwv;
        at[u] = r * nv + own0 + (i - r * cwv);
        v[u] = __ldcg(src + at[u]);
      }
    }
    for (int j = 0; j < s.world; ++j) {
      if (j == s.rank) continue;
      uint4* dst = reinterpret_cast<uint4*>(const_cast<uint8_t*>(p2p_base(s, j)) + off);
#pragma unroll
      for (int u = 0; u < kU; ++u)
        if (at[u] != ~static_cast<size_t>(0)) dst[at[u]] = v[u];  // over NVLink
    }
  }
}

// Step 2 (flags): every rank's chunk is in this rank's slot; copy the other
// ranks' chunks into out (this rank's own is there already).
__global__ void __launch_bounds__(256)
    p2p_colpar_gather_kernel(const P2PSync s, size_t off, uint4* __restrict__ out, size_t rows,
                             size_t nv) {
  if (!p2p_signal_and_wait(s)) return;
  p2p_copy_other_chunks(s, off, out, rows, nv);
}

// Row-parallel reduce-scatter, written by the ranks that own the data: every
// rank's fp32 partial [rows, n] is in its own slot (byte offset `off`),
// followed by a receive region recv[world][rows][n / world] (byte offset
// recv_off) and a gather region [rows, n] of F (byte offset gath_off).
//
// Step 1 (no flags; the GEMM before it has completed): copy column chunk o
// (n / world columns) of this rank's partial into recv[rank] of rank o, for
// every o != rank: stores over NVLink, four 16-byte vectors in flight per
// thread. Stores are posted, so the links stay busy without the round trip
// a peer load waits for.
__global__ void __launch_bounds__(256)
    p2p_rowpar_scatter_kernel(const P2PSync s, size_t off, size_t recv_off, size_t rows,
                              size_t n) {
  constexpr int kU = 4;
  const size_t cw = n / s.world;
  const size_t cwv = cw / 4;               // float4 vectors per chunk row
  const size_t per_row = (n - cw) / 4;     // vectors outside the own chunk
  const size_t total = rows * per_row;
  const size_t own0 = (size_t)s.rank * cwv;
  const float4* part = reinterpret_cast<const float4*>(p2p_base(s, s.rank) + off);
  const size_t stride = (size_t)gridDim.x * blockDim.x;
  for (size_t i0 = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i0 < total; i0 += kU * stride) {
    float4 v[kU];
    size_t src[kU];
#pragma unroll
    for (int u = 0; u < kU; ++u) {
      const size_t i = i0 + u * stride;
      src[u] = ~static_cast<size_t>(0);
      if (i < total) {
        const size_t r = i / per_row;
        size_t c = i - r * per_row;
        if (c >= own0) c += cwv;
        src[u] = r * (n / 4) + c;
        v[u] = __ldcg(part + src[u]);
      }
    }
#pragma unroll
    for (int u = 0; u < kU; ++u) {
      if (src[u] == ~static_cast<size_t>(0)) continue;
      const size_t r = src[u] / (n / 4), c = src[u] - r * (n / 4);
      const int o = static_cast<int>(c / cwv);
      float4* dst = reinterpret_cast<float4*>(const_cast<uint8_t*>(p2p_base(s, o)) + recv_off) +
                    ((size_t)s.rank * rows + r) * cwv + (c - (size_t)o * cwv);
      *dst = v[u];  // over NVLink
    }
  }
}

// Step 2 (flag set A: every rank's step 1 is done): sum column chunk `rank`
// over the world partials in rank order (this rank's from its partial, the
// others' from its receive region), add the bias once, cast, and write the
// chunk to out and into every other rank's gather region.
template <int DT>
__global__ void __launch_bounds__(256)
    p2p_rowpar_reduce_kernel(const P2PSync s, size_t off, size_t recv_off, size_t gath_off,
                             const typename DType<DT>::T* __restrict__ bias,
                             typename DType<DT>::T* __restrict__ out, size_t rows, size_t n) {
  using T = typename DType<DT>::T;
  if (!p2p_signal_and_wait(s)) return;
  const size_t cw = n / s.world, c0 = (size_t)s.rank * cw;
  const size_t per_row = cw / 8;  // 8 columns per item (cw % 32 == 0)
  const size_t oct = rows * per_row;
  const uint8_t* own = p2p_base(s, s.rank);
  const float* part = reinterpret_cast<const float*>(own + off);
  const float* recv = reinterpret_cast<const float*>(own + recv_off);
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < oct;
       i += (size_t)gridDim.x * blockDim.x) {
    const size_t r = i / per_row, cl = (i - r * per_row) * 8;  // column inside the chunk
    float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    for (int j = 0; j < s.world; ++j) {  // rank order: the same sum on every rank
      const float* src = j == s.rank ? part + r * n + c0 + cl
                                     : recv + ((size_t)j * rows + r) * cw + cl;
      const float4 a = __ldcg(reinterpret_cast<const float4*>(src));  // L2: peers wrote it
      const float4 b = __ldcg(reinterpret_cast<const float4*>(src) + 1);
      acc[0] += a.x; acc[1] += a.y; acc[2] += a.z; acc[3] += a.w;
      acc[4] += b.x; acc[5] += b.y; acc[6] += b.z; acc[7] += b.w;
    }
    uint4 v;
    T* h = reinterpret_cast<T*>(&v);
#pragma unroll
    for (int e = 0; e < 8; ++e)
      h[e] = DType<DT>::from_f32(acc[e] + (bias ? DType<DT>::to_f32(bias[c0 + cl + e]) : 0.f));
    const size_t at = r * n + c0 + cl;
    *reinterpret_cast<uint4*>(out + at) = v;
    for (int j = 0; j < s.world; ++j) {
      if (j == s.rank) continue;
      T* g = reinterpret_cast<T*>(const_cast<uint8_t*>(p2p_base(s, j)) + gath_off);
      *reinterpret_cast<uint4*>(g + at) = v;  // over NVLink
    }
  }
}

// Step 3 (flag set B: every rank's step 2 is done): the other chunks are in
// this rank's gather region; copy them to out.
template <int DT>
__global__ void __launch_bounds__(256)
    p2p_rowpar_gather_kernel(const P2PSync s, size_t gath_off,
                             typename DType<DT>::T* __restrict__ out, size_t rows, size_t n) {
  if (!p2p_signal_and_wait(s)) return;
  p2p_copy_other_chunks(s, gath_off, reinterpret_cast<uint4*>(out), rows, n / 8);
}

static unsigned p2p_blocks(size_t work) {
  size_t b = (work + 255) / 256;
  if (b > 148 * 4) b = 148 * 4;  // all blocks resident: each one waits
  return static_cast<unsigned>(b < 1 ? 1 : b);
}

cudaError_t launch_p2p_colpar_finish(const P2PSync& s, const void* slot, void* out, size_t rows,
                                     size_t n, size_t ld_out, int dtype, cudaStream_t stream) {
  const size_t es = dtype == kF32 ? 4 : 2;
  const bool v16 = (n * es) % 16 == 0 && (ld_out * es) % 16 == 0 &&
                   reinterpret_cast<uintptr_t>(slot) % 16 == 0 &&
                   reinterpret_cast<uintptr_t>(out) % 16 == 0;
  if (v16) {
    const size_t nv = n * es / 16;
    p2p_colpar_finish_kernel<uint4><<<p2p_blocks(rows * nv), 256, 0, stream>>>(
        s, static_cast<const uint4*>(slot), static_cast<uint4*>(out), rows, nv, ld_out * es / 16);
  } else if (es == 4) {
    p2p_colpar_finish_kernel<uint32_t><<<p2p_blocks(rows * n), 256, 0, stream>>>(
        s, static_cast<const uint32_t*>(slot), static_cast<uint32_t*>(out), rows, n, ld_out);
  } else {
    p2p_colpar_finish_kernel<uint16_t><<<p2p_blocks(rows * n), 256, 0, stream>>>(
        s, static_cast<const uint16_t*>(slot), static_cast<uint16_t*>(out), rows, n, ld_out);
  }
  return cudaGetLastError();
}

cudaError_t launch_p2p_rowpar_finish(const P2PSync& s, const float* slot, const void* bias,
                                     void* out, size_t rows, size_t n, int dtype,
                                     cudaStream_t stream) {
  const unsigned b = p2p_blocks(rows * n / 4);
  if (dtype == kF32) {
    p2p_rowpar_finish_kernel<kF32><<<b, 256, 0, stream>>>(
        s, slot, static_cast<const float*>(bias), static_cast<float*>(out), rows, n);
  } else if (dtype == kF16) {
    p2p_rowpar_finish_kernel<kF16><<<b, 256, 0, stream>>>(
        s, slot, static_cast<const __half*>(bias), static_cast<__half*>(out), rows, n);
  } else {
    p2p_rowpar_finish_kernel<kBF16><<<b, 256, 0, stream>>>(
        s, slot, static_cast<const __nv_bfloat16*>(bias), static_cast<__nv_bfloat16*>(out), rows,
        n);
  }
  return cudaGetLastError();
}

cudaError_t launch_p2p_colpar_push(const P2PSync& s, size_t off, void* out, size_t rows,
                                   size_t n, int dtype, cudaStream_t stream) {
  const size_t es = dtype == kF32 ? 4 : 2;
  const size_t nv = n * es / 16;
  p2p_colpar_push_kernel<<<p2p_blocks(rows * (nv / s.world) / 4), 256, 0, stream>>>(s, off, rows,
                                                                                  nv);
  p2p_colpar_gather_kernel<<<p2p_blocks(rows * (nv - nv / s.world)), 256, 0, stream>>>(
      s, off, static_cast<uint4*>(out), rows, nv);
  return cudaGetLastError();
}

cudaError_t launch_p2p_rowpar_rs(const P2PSync& sa, const P2PSync& sb, size_t off,
                                 size_t recv_off, size_t gath_off, const void* bias, void* out,
                                 size_t rows, size_t n, int dtype, cudaStream_t stream) {
  const size_t cw = n / sa.world;
  const unsigned b0 = p2p_blocks(rows * (n - cw) / 16);
  const unsigned b1 = p2p_blocks(rows * cw / 8);
  const unsigned b2 = p2p_blocks(rows * (n - cw) / 8);
  p2p_rowpar_scatter_kernel<<<b0, 256, 0, stream>>>(sa, off, recv_off, rows, n);
  if (dtype == kF16) {
    p2p_rowpar_reduce_kernel<kF16><<<b1, 256, 0, stream>>>(
        sa, off, recv_off, gath_off, static_cast<const __half*>(bias), static_cast<__half*>(out),
        rows, n);
    p2p_rowpar_gather_kernel<kF16><<<b2, 256, 0, stream>>>(sb, gath_off,
                                                           static_cast<__half*>(out), rows, n);
  } else {
    p2p_rowpar_reduce_kernel<kBF16><<<b1, 256, 0, stream>>>(
        sa, off, recv_off, gath_off, static_cast<const __nv_bfloat16*>(bias),
        static_cast<__nv_bfloat16*>(out), rows, n);
    p2p_rowpar_gather_kernel<kBF16><<<b2, 256, 0, stream>>>(
        sb, gath_off, static_cast<__nv_bfloat16*>(out), rows, n);
  }
  return cudaGetLastError();
}

// Fixed-size fp32 scratch of cawq_gemm_rowpar_noalloc: one per device,
// loaded with the module image, so the call allocates nothing. In host code
// `g_rowpar_scratch` is only a handle for the runtime, not a device address:
// the address comes from cudaGetSymbolAddress below.
static __device__ __align__(256) float g_rowpar_scratch[CAWQ_ROWPAR_SCRATCH_FLOATS];

cudaError_t rowpar_static_scratch(float** ptr) {
  // Set-up on the first call per device: cudaGetSymbolAddress with that
  // device current (the caller's current device, the communicator's), its
  // status checked, the address kept for every later call on that device
  // for the life of the process (a device reset, which would move the
  // array, is not supported with this entry point).
  constexpr int kMaxDevices = 64;
  static std::mutex mu;
  static float* cached[kMaxDevices] = {};
  int dev = -1;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 0 || dev >= kMaxDevices) return cudaErrorInvalidDevice;
  std::lock_guard<std::mutex> lk(mu);
  if (!cached[dev]) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_rowpar_scratch);
    if (e != cudaSuccess) return e;
    cached[dev] = static_cast<float*>(p);
  }
  *ptr = cached[dev];
  return cudaSuccess;
}

}  // namespace cawq

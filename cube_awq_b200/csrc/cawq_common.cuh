// cawq_common.cuh — device helpers shared by the sm_100a kernels of
// libcube_awq.so: dtype traits, nibble order tables, PTX wrappers (mbarrier,
// TMA, mma.sync, cluster shared memory) and the bounded-wait error word.
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <type_traits>

#include "cawq_internal.h"

namespace cawq {

// ---------------------------------------------------------------- dtypes
template <int DT> struct DType;
template <> struct DType<kF32> {
  using T = float;
  static __device__ __forceinline__ float to_f32(T v) { return v; }
  static __device__ __forceinline__ T from_f32(float v) { return v; }
};
template <> struct DType<kF16> {
  using T = __half;
  static __device__ __forceinline__ float to_f32(T v) { return __half2float(v); }
  static __device__ __forceinline__ T from_f32(float v) { return __float2half_rn(v); }
};
template <> struct DType<kBF16> {
  using T = __nv_bfloat16;
  static __device__ __forceinline__ float to_f32(T v) { return __bfloat162float(v); }
  static __device__ __forceinline__ T from_f32(float v) { return __float2bfloat16_rn(v); }
};

__device__ __forceinline__ float load_as_f32(const void* p, size_t i, int dt) {
  if (dt == kF32) return static_cast<const float*>(p)[i];
  if (dt == kF16) return __half2float(static_cast<const __half*>(p)[i]);
  return __bfloat162float(static_cast<const __nv_bfloat16*>(p)[i]);
}

__device__ __forceinline__ void store_from_f32(void* p, size_t i, float v, int dt) {
  if (dt == kF32) {
    static_cast<float*>(p)[i] = v;
  } else if (dt == kF16) {
    static_cast<__half*>(p)[i] = __float2half_rn(v);
  } else {
    static_cast<__nv_bfloat16*>(p)[i] = __float2bfloat16_rn(v);
  }
}

// ------------------------------------------------------ nibble ordering
// Nibble that holds logical column c (0..7) of a packed word.
//   AWQ order (awq_kernel_gemm.rs:10-30): [0,4,1,5,2,6,3,7]
//   natural (awq_kernel.rs:9-19): c
__device__ __forceinline__ int nibble_of_col(int c, int order) {
  return order == kOrderAwq ? ((c & 1) * 4 + (c >> 1)) : c;
}
// Logical column stored in nibble p (inverse of nibble_of_col).
//   AWQ: AWQ_ORDER = [0,2,4,6,1,3,5,7] (awq_gemm.rs:248)
__host__ __device__ __forceinline__ int col_of_nibble(int p, int order) {
  return order == kOrderAwq ? ((p & 3) * 2 + (p >> 2)) : p;
}

// --------------------------------------------------------- bit helpers
__device__ __forceinline__ uint32_t lop3_and_or(uint32_t a, uint32_t mask, uint32_t magic) {
  uint32_t d;
  // (a & mask) | magic  ->  immLut 0xEA
  asm("lop3.b32 %0, %1, %2, %3, 0xEA;" : "=r"(d) : "r"(a), "r"(mask), "r"(magic));
  return d;
}

__device__ __forceinline__ uint32_t prmt(uint32_t a, uint32_t b, uint32_t sel) {
  uint32_t d;
  asm("prmt.b32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(sel));
  return d;
}

// ------------------------------------------------- device error word
// Bit 0: a bounded wait (mbarrier / cluster) gave up. Host reads it through
// cawq_device_error(). Defined here: only cawq_kernels.cu includes this file.
__device__ uint32_t g_cawq_device_error = 0;

__device__ __forceinline__ uint64_t globaltimer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
  return t;
}

// ------------------------------------------------------------ mbarrier
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}

__device__ __forceinline__ void fence_mbarrier_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
               "r"(bytes)
               : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Waits for phase `parity` of `bar` to complete, for at most kWaitLimitNs.
// On timeout it records bit 0 in the device error word and returns false; the
// caller then skips its work but still takes every barrier it would have.
constexpr uint64_t kWaitLimitNs = 2000000000ull;  // 2 s

__device__ __forceinline__ bool mbar_wait_bounded(uint64_t* bar, uint32_t parity) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = globaltimer_ns();
  for (uint32_t it = 0;; ++it) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((it & 63u) == 63u && globaltimer_ns() - t0 > kWaitLimitNs) {
      atomicOr(&g_cawq_device_error, 1u);
      return false;
    }
  }
}

// ----------------------------------------------------------------- TMA
// 2-D tiled bulk tensor load into this CTA's shared memory, completion on an
// mbarrier (no multicast). c0 is the inner (contiguous) coordinate.
__device__ __forceinline__ void tma_load_2d(void* smem_dst, const CUtensorMap* map, int c0, int c1,
                                            uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cta.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3}], [%4];" ::"r"(smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(smem_u32(bar))
      : "memory");
}

// 1-D bulk copy global -> this CTA's shared memory (16-byte aligned, size a
// multiple of 16), completion on an mbarrier.
__device__ __forceinline__ void bulk_load_1d(void* smem_dst, const void* src, uint32_t bytes,
                                             uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cta.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_u32(smem_dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

// Barrier among `count` threads (a multiple of 32) of the CTA on named
// barrier `id` (1..15; 0 is __syncthreads).
__device__ __forceinline__ void named_bar_sync(uint32_t id, uint32_t count) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(count) : "memory");
}

// Address of output element (row, col): columns [0, c1) live in p0 (row
// stride ld0), [c1, c2) in p1 and [c2, n) in p2 (the q / k / v outputs of a
// fused qkv projection); a single output has c1 = c2 = 0xFFFFFFFF. Fields,
// not arrays, so the choice compiles to selects on kernel parameters.
template <typename OT>
struct OutMap {
  OT* p0;
  OT* p1;
  OT* p2;
  uint32_t ld0, ld1, ld2, c1, c2;
  // replicas of a single-range output (peer buffers): rep[i] + (a - p0)
  OT* rep[7];
  uint32_t nrep;
  __device__ __forceinline__ OT* at(uint32_t row, uint32_t col) const {
    if (col < c1) return p0 + (size_t)row * ld0 + col;
    if (col < c2) return p1 + (size_t)row * ld1 + (col - c1);
    return p2 + (size_t)row * ld2 + (col - c2);
  }
  // stores v at `a` (an address from at()) and, with REP, at every replica
  template <bool REP, typename V>
  __device__ __forceinline__ void put(OT* a, const V& v) const {
    *reinterpret_cast<V*>(a) = v;
    if constexpr (REP) {
      const size_t off = static_cast<size_t>(a - p0);
#pragma unroll
      for (int i = 0; i < 7; ++i)
        if (static_cast<uint32_t>(i) < nrep) *reinterpret_cast<V*>(rep[i] + off) = v;
    }
  }
};

template <typename OT>
inline OutMap<OT> out_map(const GemmProblem& p) {
  OutMap<OT> m;
  m.p0 = static_cast<OT*>(p.out);
  m.ld0 = static_cast<uint32_t>(p.ld_out);
  if (p.out_k) {
    m.p1 = static_cast<OT*>(p.out_k);
    m.p2 = static_cast<OT*>(p.out_v);
    m.ld1 = static_cast<uint32_t>(p.ld_k);
    m.ld2 = static_cast<uint32_t>(p.ld_v);
    m.c1 = static_cast<uint32_t>(p.col_k);
    m.c2 = static_cast<uint32_t>(p.col_v);
  } else {
    m.p1 = m.p2 = m.p0;
    m.ld1 = m.ld2 = m.ld0;
    m.c1 = m.c2 = 0xFFFFFFFFu;
  }
  for (int i = 0; i < 7; ++i) m.rep[i] = static_cast<OT*>(p.rep[i]);
  m.nrep = static_cast<uint32_t>(p.nrep);
  return m;
}

// silu(g) * u, the gate of a gated MLP, with the fast-math intrinsics
// (exp and divide; a few ulp in fp32, far below the f16 / bf16 output's
// rounding). A gate below about -88 makes the denominator infinite and the
// result 0, its limit.
__device__ __forceinline__ float silu_mul(float g, float u) {
  return __fdividef(g, 1.f + __expf(-g)) * u;
}

// Prefetches into L2 (no shared memory, no completion): one 2-D tensor box,
// or a 1-D byte range (16-byte aligned, size a multiple of 16).
__device__ __forceinline__ void tma_prefetch_l2_2d(const CUtensorMap* map, int c0, int c1) {
  asm volatile("cp.async.bulk.prefetch.tensor.2d.L2.global.tile [%0, {%1, %2}];" ::"l"(
                   reinterpret_cast<uint64_t>(map)),
               "r"(c0), "r"(c1)
               : "memory");
}
__device__ __forceinline__ void bulk_prefetch_l2(const void* src, uint32_t bytes) {
  asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(src), "r"(bytes) : "memory");
}

// Programmatic dependent launch: wait for the preceding grid's results /
// allow the next grid in the stream to start its prologue.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_launch_dependents() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

__device__ __forceinline__ void tma_prefetch_desc(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

// ------------------------------------------------------------- cluster
__device__ __forceinline__ uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}

__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::
                   : "memory");
}

// Split cluster barrier: arrive (release) early, wait (acquire) where needed.
__device__ __forceinline__ void cluster_arrive_release() {
  asm volatile("barrier.cluster.arrive.release.aligned;" ::: "memory");
}
__device__ __forceinline__ void cluster_wait_acquire() {
  asm volatile("barrier.cluster.wait.acquire.aligned;" ::: "memory");
}

// 16-byte store into another CTA's shared memory; its mbarrier `remote_bar`
// (same cluster) counts the bytes on arrival.
__device__ __forceinline__ void st_async_v4(uint32_t remote_addr, float a, float b, float c,
                                            float d, uint32_t remote_bar) {
  asm volatile(
      "st.async.shared::cluster.mbarrier::complete_tx::bytes.v4.f32 [%0], {%1, %2, %3, %4}, [%5];"
      ::"r"(remote_addr), "f"(a), "f"(b), "f"(c), "f"(d), "r"(remote_bar)
      : "memory");
}

// Address of the same shared variable in CTA `rank` of this cluster.
__device__ __forceinline__ uint32_t map_shared_rank(uint32_t local_addr, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(local_addr), "r"(rank));
  return r;
}

__device__ __forceinline__ float ld_shared_cluster_f32(uint32_t addr) {
  float v;
  asm volatile("ld.shared::cluster.f32 %0, [%1];" : "=f"(v) : "r"(addr) : "memory");
  return v;
}

// ------------------------------------------------------------- mma.sync
// D(16x8, f32) += A(16x16) * B(16x8), A/B 16-bit (f16 or bf16).
template <bool kBF16>
__device__ __forceinline__ void mma_16816(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2,
                                          uint32_t a3, uint32_t b0, uint32_t b1) {
  if constexpr (kBF16) {
    asm(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 "
        "{%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
  } else {
    asm(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 "
        "{%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
  }
}

// D(16x8, f32) = A(16x16) * B(16x8): a fresh accumulator (C = 0).
template <bool kBF16>
__device__ __forceinline__ void mma_16816_c0(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2,
                                             uint32_t a3, uint32_t b0, uint32_t b1) {
  const float z = 0.f;
  if constexpr (kBF16) {
    asm(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 "
        "{%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%10,%10,%10,%10};"
        : "=f"(d[0]), "=f"(d[1]), "=f"(d[2]), "=f"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1), "f"(z));
  } else {
    asm(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 "
        "{%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%10,%10,%10,%10};"
        : "=f"(d[0]), "=f"(d[1]), "=f"(d[2]), "=f"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1), "f"(z));
  }
}

// Four 8x8 b16 matrices from shared memory: lane L supplies the address of
// row L & 7 of matrix L >> 3; each lane receives its 32-bit piece of each.
__device__ __forceinline__ void ldmatrix_x4(uint32_t saddr, uint32_t& r0, uint32_t& r1,
                                            uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(saddr)
               : "memory");
}

// The same four matrices transposed: lane (g, t) = (L >> 2, L & 3) receives,
// per matrix, element g of rows 2t (low half) and 2t + 1 (high half).
__device__ __forceinline__ void ldmatrix_x4_trans(uint32_t saddr, uint32_t& r0, uint32_t& r1,
                                                  uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(saddr)
               : "memory");
}

// ------------------------------------------------------- global access
// ------------------------------------------------- packed 16-bit dequant
// Magic-number unpack shared by the prefill and dequantize kernels: a nibble
// q masked into the mantissa of the magic value m gives m + q exactly (f16:
// m = 1024, bf16: m = 128), so (m + q) - (m + z) = q - z exactly and one
// multiply by s rounds once, as the reference's (q - z) * s in F does.
template <int DT>
struct PfHalf2;
template <>
struct PfHalf2<kF16> {
  static constexpr uint32_t kMagic = 0x64006400u;  // f16 1024
  static __device__ __forceinline__ uint32_t sub(uint32_t a, uint32_t b) {
    __half2 r = __hsub2(*reinterpret_cast<const __half2*>(&a), *reinterpret_cast<const __half2*>(&b));
    return *reinterpret_cast<uint32_t*>(&r);
  }
  static __device__ __forceinline__ uint32_t mul(uint32_t a, uint32_t b) {
    __half2 r = __hmul2(*reinterpret_cast<const __half2*>(&a), *reinterpret_cast<const __half2*>(&b));
    return *reinterpret_cast<uint32_t*>(&r);
  }
};
template <>
struct PfHalf2<kBF16> {
  static constexpr uint32_t kMagic = 0x43004300u;  // bf16 128
  static __device__ __forceinline__ uint32_t sub(uint32_t a, uint32_t b) {
    __nv_bfloat162 r = __hsub2(*reinterpret_cast<const __nv_bfloat162*>(&a),
                               *reinterpret_cast<const __nv_bfloat162*>(&b));
    return *reinterpret_cast<uint32_t*>(&r);
  }
  static __device__ __forceinline__ uint32_t mul(uint32_t a, uint32_t b) {
    __nv_bfloat162 r = __hmul2(*reinterpret_cast<const __nv_bfloat162*>(&a),
                               *reinterpret_cast<const __nv_bfloat162*>(&b));
    return *reinterpret_cast<uint32_t*>(&r);
  }
};

// Four (1024 + nibble) pairs of adjacent logical columns of one packed word.
template <int DT, int ORDER>
__device__ __forceinline__ void pf_pairs(uint32_t q, uint32_t (&t)[4]) {
  constexpr uint32_t M = PfHalf2<DT>::kMagic;
  if constexpr (ORDER == kOrderAwq) {
    // logical (2i, 2i+1) live in nibbles (i, i+4)
    t[0] = lop3_and_or(q, 0x000F000Fu, M);
    t[1] = lop3_and_or(q >> 4, 0x000F000Fu, M);
    t[2] = lop3_and_or(q >> 8, 0x000F000Fu, M);
    t[3] = lop3_and_or(q >> 12, 0x000F000Fu, M);
  } else {
    // logical (2i, 2i+1) live in nibbles (2i, 2i+1) = both halves of byte i
    const uint32_t q4 = q >> 4;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const uint32_t sel = (uint32_t)(i | (i << 4) | ((4 + i) << 8) | ((4 + i) << 12));
      t[i] = lop3_and_or(prmt(q, q4, sel), 0x000F000Fu, M);
    }
  }
}

__device__ __forceinline__ uint32_t ldg_nc_u32(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.global.nc.u32 %0, [%1];" : "=r"(v) : "l"(p));
  return v;
}

__device__ __forceinline__ void stg_cs_v4(void* p, uint4 v) {
  asm volatile("st.global.cs.v4.u32 [%0], {%1,%2,%3,%4};" ::"l"(p), "r"(v.x), "r"(v.y), "r"(v.z),
               "r"(v.w)
               : "memory");
}

}  // namespace cawq

// cawq_internal.h — declarations shared by the translation units of
// libcube_awq.so (host side). Not part of the public C ABI.
#pragma once

#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

#include <string>

#include "cube_awq.h"

namespace cawq {

enum { kF32 = CAWQ_F32, kF16 = CAWQ_F16, kBF16 = CAWQ_BF16 };
enum { kOrderAwq = CAWQ_ORDER_AWQ, kOrderNatural = CAWQ_ORDER_NATURAL };

inline size_t dtype_size(int dt) { return dt == kF32 ? 4 : 2; }

// One fused GEMM call after validation.
struct GemmProblem {
  const void* x;         // [rows, k] dtype
  const uint32_t* qw;    // [k, n/8]
  const uint32_t* qz;    // [k/g, n/8]
  const void* sc;        // [k/g, n] dtype
  const void* bias;      // [n] dtype or nullptr
  void* out;             // [rows, ld_out] out_dtype
  size_t rows, k, n, g, ld_out;
  int dtype, out_dtype, order;
  cudaStream_t stream;
  // epilogue: 0 = plain; 1 = SiLU-gated product of block-interleaved gate/up
  // columns (128-column blocks: gate, up, gate, ...): out [rows, n / 2]
  int epi = 0;
  // column split of the output (qkv projection): columns [0, col_k) go to
  // `out` (row stride ld_out), [col_k, col_v) to out_k (ld_k), [col_v, n) to
  // out_v (ld_v); out_k == nullptr: one output. col_k and col_v are multiples
  // of 32, so no 32-column store chunk straddles two outputs.
  void* out_k = nullptr;
  void* out_v = nullptr;
  size_t ld_k = 0, ld_v = 0, col_k = 0, col_v = 0;
  // replicas of the (single-range) output: every element is also stored at
  // the same offset from rep[i] as from `out` — other GPUs' buffers, mapped
  // into this process (the push of a fused tensor-parallel collective).
  // Decode and prefill kernels, f16 / bf16 activations, AWQ order only.
  void* rep[7] = {};
  int nrep = 0;
};

// Thread-local error message (cawq_last_error).
void set_error(const std::string& msg);
cawq_status fail(cawq_status st, const std::string& msg);
cawq_status cuda_fail(cudaError_t e, const char* where);

// Device properties cached per device.
struct DeviceInfo {
  int device = -1;
  int sm_count = 0;
  int cc_major = 0, cc_minor = 0;
  size_t smem_optin = 0;
};
cawq_status current_device_info(DeviceInfo* info);

// Driver entry point for cuTensorMapEncodeTiled (resolved through the runtime,
// so the library needs no -lcuda).
typedef int (*EncodeTiledFn)(void*, int, uint32_t, void*, const uint64_t*, const uint64_t*,
                             const uint32_t*, const uint32_t*, int, int, int, int);
EncodeTiledFn encode_tiled_fn();

// cuTensorMapEncodeTiled of a 2-D row-major tensor into the 128-byte map at
// `map` (no interleave, L2 promotion 256 B, no OOB fill), through a small
// per-thread cache keyed by every argument (a hit yields the identical map).
bool encode_tiled_2d(void* map, int cu_dtype, const void* base, uint64_t inner, uint64_t outer,
                     uint64_t row_bytes, uint32_t box_inner, uint32_t box_outer, int cu_swizzle);

// ---------------------------------------------------------- launchers
// Each returns cudaSuccess or the launch error. `supports` functions say
// whether a plan can run a problem (shape, dtype and alignment).
bool generic_supports(const GemmProblem& p);
cudaError_t launch_generic(const GemmProblem& p);

bool decode_supports(const GemmProblem& p, const cawq_plan& plan, const DeviceInfo& dev);
cudaError_t launch_decode(const GemmProblem& p, const cawq_plan& plan, const DeviceInfo& dev);
void decode_candidates(const GemmProblem& p, const DeviceInfo& dev, cawq_plan* out, int* count,
                       int max_count);
cawq_plan decode_default_plan(const GemmProblem& p, const DeviceInfo& dev);

bool prefill_supports(const GemmProblem& p, const cawq_plan& plan, const DeviceInfo& dev);
// f32 activations and scales on the tensor cores (cawq_prefill_f32.cuh);
// prefill_supports / launch_prefill hand f32 problems to these
bool prefill_f32_supports(const GemmProblem& p, const cawq_plan& plan, const DeviceInfo& dev);
// CTA tile width of the f32 kernel for this plan (128 or 256)
int prefill_f32_tile_n(const GemmProblem& p, const cawq_plan& plan, const DeviceInfo& dev);
cudaError_t launch_prefill_f32(const GemmProblem& p, const cawq_plan& plan,
                               const DeviceInfo& dev);
cudaError_t launch_prefill(const GemmProblem& p, const cawq_plan& plan, const DeviceInfo& dev);
// prefill_supports / launch_prefill hand plans with warps == 4 (weights as the
// MMA's A operand in tensor memory, rows <= 128) to these
bool prefill_tw_supports(const GemmProblem& p, const cawq_plan& plan, const DeviceInfo& dev);
cudaError_t launch_prefill_tw(const GemmProblem& p, const cawq_plan& plan, const DeviceInfo& dev);
void prefill_candidates(const GemmProblem& p, const DeviceInfo& dev, cawq_plan* out, int* count,
                        int max_count);
cawq_plan prefill_default_plan(const GemmProblem& p, const DeviceInfo& dev);

cudaError_t launch_dequant(const uint32_t* qw, const uint32_t* qz, const void* sc, void* out,
                           size_t k, size_t n, size_t g, int dtype, int order,
                           cudaStream_t stream, int sm_count);

cudaError_t launch_interleave_gate_up(const void* src, void* dst, size_t rows, size_t width_e,
                                      size_t block_e, size_t elem, cudaStream_t stream);
cudaError_t launch_interleave_columns(const void* src, void* dst, size_t rows, size_t n,
                                      int world, size_t elem, cudaStream_t stream);
cudaError_t launch_rowpar_finish(const float* partial, const void* bias, void* out, size_t rows,
                                 size_t n, int dtype, cudaStream_t stream);
// Fused tensor-parallel push: every rank's peer buffer starts with a flag
// word per rank. flags[j] is rank j's flag array as mapped in this process
// (flags[rank] = this rank's own). Rank r publishes `epoch` in word r of
// every peer's array once its pushed data is complete, then waits until word
// j of its own array holds `epoch` for every peer j (at most timeout_ns).
constexpr int kP2PMaxWorld = 8;
struct P2PSync {
  uint32_t* flags[kP2PMaxWorld];
  int world, rank;
  uint32_t epoch;
  uint64_t timeout_ns;
  int fofs = 0;  // first flag word of the set this exchange uses (0 or 8)
};
// After the push of a column-parallel GEMM: signal, wait, then copy the
// gathered [rows, n] result (dense in `slot`) to out (row stride ld_out).
cudaError_t launch_p2p_colpar_finish(const P2PSync& s, const void* slot, void* out, size_t rows,
                                     size_t n, size_t ld_out, int dtype, cudaStream_t stream);
// Exchanges for large outputs (the GEMM wrote only this rank's own buffer).
// Column-parallel: push this rank's columns of its slot (dense [rows, n] at
// byte offset off) into every other rank's slot; flag exchange; copy the
// other ranks' columns from the own slot into out (row stride n, 16-byte
// aligned, n * sizeof(F) % (16 * world) == 0).
cudaError_t launch_p2p_colpar_push(const P2PSync& s, size_t off, void* out, size_t rows,
                                   size_t n, int dtype, cudaStream_t stream);
// Row-parallel reduce-scatter + all-gather after the local GEMM wrote its
// fp32 partial [rows, n] at byte offset off of this rank's buffer: push the
// other ranks' column chunks into their receive regions (recv_off:
// [world][rows][n / world] fp32); flag set A, sum the own chunk in rank
// order (+ bias, cast) into out and push it into the other ranks' gather
// regions (gath_off: [rows, n] of F); flag set B, copy the other chunks from
// the own gather region into out. dtype f16 / bf16, n % (32 world) == 0.
cudaError_t launch_p2p_rowpar_rs(const P2PSync& sa, const P2PSync& sb, size_t off,
                                 size_t recv_off, size_t gath_off, const void* bias, void* out,
                                 size_t rows, size_t n, int dtype, cudaStream_t stream);
// After the push of a row-parallel GEMM's fp32 partials into slot[world][rows][n]:
// signal, wait, then out = sum over ranks (in rank order) + bias, cast to dtype.
cudaError_t launch_p2p_rowpar_finish(const P2PSync& s, const float* slot, const void* bias,
                                     void* out, size_t rows, size_t n, int dtype,
                                     cudaStream_t stream);

// Device address of the current device's static row-parallel scratch
// (CAWQ_ROWPAR_SCRATCH_FLOATS floats).
cudaError_t rowpar_static_scratch(float** ptr);

cudaError_t read_device_error(uint32_t* word, int reset);

}  // namespace cawq

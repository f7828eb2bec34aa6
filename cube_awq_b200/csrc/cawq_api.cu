// cawq_api.cu — the extern "C" entry points of libcube_awq.so (host code):
// argument checks with the reference's messages, the planner / autotuner, and
// dispatch to the sm_100a kernels in cawq_kernels.cu.
#include <cuda.h>
#include <cuda_runtime.h>
#include <dlfcn.h>
#include <nccl.h>

#include <algorithm>
#include <chrono>
#include <cstdarg>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <map>
#include <mutex>
#include <string>
#include <thread>
#include <tuple>
#include <vector>

#include "cawq_internal.h"

#define CAWQ_API extern "C" __attribute__((visibility("default")))

namespace cawq {

// ------------------------------------------------------------- errors
static thread_local std::string g_last_error;

void set_error(const std::string& msg) { g_last_error = msg; }

cawq_status fail(cawq_status st, const std::string& msg) {
  g_last_error = msg;
  return st;
}

cawq_status cuda_fail(cudaError_t e, const char* where) {
  std::string m = std::string("CUDA error in ") + where + ": " + cudaGetErrorName(e) + " (" +
                  cudaGetErrorString(e) + ")";
  return fail(CAWQ_ERR_CUDA, m);
}

static std::string fmt(const char* f, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, f);
  vsnprintf(buf, sizeof(buf), f, ap);
  va_end(ap);
  return buf;
}

// ------------------------------------------------------------- device
static std::mutex g_dev_mu;
static std::map<int, DeviceInfo> g_dev_cache;

cawq_status current_device_info(DeviceInfo* info) {
  int dev = -1;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
  {
    std::lock_guard<std::mutex> lk(g_dev_mu);
    auto it = g_dev_cache.find(dev);
    if (it != g_dev_cache.end()) {
      *info = it->second;
      return CAWQ_OK;
    }
  }
  DeviceInfo d;
  d.device = dev;
  int v = 0;
  if ((e = cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev)) != cudaSuccess)
    return cuda_fail(e, "cudaDeviceGetAttribute");
  d.sm_count = v;
  cudaDeviceGetAttribute(&d.cc_major, cudaDevAttrComputeCapabilityMajor, dev);
  cudaDeviceGetAttribute(&d.cc_minor, cudaDevAttrComputeCapabilityMinor, dev);
  cudaDeviceGetAttribute(&v, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
  d.smem_optin = static_cast<size_t>(v);
  {
    std::lock_guard<std::mutex> lk(g_dev_mu);
    g_dev_cache[dev] = d;
  }
  *info = d;
  return CAWQ_OK;
}

static cawq_status require_sm100(DeviceInfo* dev) {
  cawq_status st = current_device_info(dev);
  if (st != CAWQ_OK) return st;
  if (dev->cc_major != 10) {
    return fail(CAWQ_ERR_UNSUPPORTED,
                fmt("libcube_awq.so has sm_100a code only; device %d is sm_%d%d", dev->device,
                    dev->cc_major, dev->cc_minor));
  }
  return CAWQ_OK;
}

EncodeTiledFn encode_tiled_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess) {
      fn = reinterpret_cast<EncodeTiledFn>(p);
    }
  });
  return fn;
}

// ------------------------------------------------------- tensor maps
namespace {
struct TensorMapEntry {
  const void* base = nullptr;
  uint64_t inner = 0, outer = 0, row_bytes = 0;
  uint32_t box_inner = 0, box_outer = 0;
  int dt = -1, swz = -1;
  alignas(64) CUtensorMap map;
};
constexpr int kTensorMapCache = 64;
thread_local TensorMapEntry t_maps[kTensorMapCache];
}  // namespace

bool encode_tiled_2d(void* map, int cu_dtype, const void* base, uint64_t inner, uint64_t outer,
                     uint64_t row_bytes, uint32_t box_inner, uint32_t box_outer, int cu_swizzle) {
  const uint64_t h = (reinterpret_cast<uintptr_t>(base) >> 8) ^ (inner * 0x9E3779B97F4A7C15ull) ^
                     (outer << 7) ^ ((uint64_t)box_outer << 3) ^ (uint64_t)cu_dtype;
  TensorMapEntry& e = t_maps[(h ^ (h >> 29)) % kTensorMapCache];
  if (e.base == base && e.inner == inner && e.outer == outer && e.row_bytes == row_bytes &&
      e.box_inner == box_inner && e.box_outer == box_outer && e.dt == cu_dtype &&
      e.swz == cu_swizzle) {
    std::memcpy(map, &e.map, sizeof(CUtensorMap));
    return true;
  }
  EncodeTiledFn fn = encode_tiled_fn();
  if (!fn) return false;
  const uint64_t dims[2] = {inner, outer};
  const uint64_t strides[1] = {row_bytes};
  const uint32_t box[2] = {box_inner, box_outer};
  const uint32_t estr[2] = {1, 1};
  const int r = fn(map, cu_dtype, 2, const_cast<void*>(base), dims, strides, box, estr,
                   static_cast<int>(CU_TENSOR_MAP_INTERLEAVE_NONE), cu_swizzle,
                   static_cast<int>(CU_TENSOR_MAP_L2_PROMOTION_L2_256B),
                   static_cast<int>(CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE));
  if (r != 0) return false;
  e.base = base;
  e.inner = inner;
  e.outer = outer;
  e.row_bytes = row_bytes;
  e.box_inner = box_inner;
  e.box_outer = box_outer;
  e.dt = cu_dtype;
  e.swz = cu_swizzle;
  std::memcpy(&e.map, map, sizeof(CUtensorMap));
  return true;
}

// --------------------------------------------------- reference rules
static bool multiple_of(size_t a, size_t b) { return b == 0 ? a == 0 : a % b == 0; }

// validate_launch_params_impl (awq_kernel_gemm.rs:89-158), same order and text.
static cawq_status validate_impl(const cawq_shape_config& s, size_t group_size,
                                 size_t rows_per_thread, size_t n_lines_per_thread) {
  auto bad = [](const char* m) { return fail(CAWQ_ERR_INVALID_SHAPE, m); };
  if (!(s.m > 0)) return bad("m must be > 0");
  if (!(s.line_size > 0)) return bad("line_size must be > 0");
  if (!(s.tile_m > 0)) return bad("m_tile_size must be > 0");
  if (!(s.tile_n > 0)) return bad("n_tile_size must be > 0");
  if (!(s.inner_k > 0)) return bad("inner_k_size must be > 0");
  if (!(group_size > 0)) return bad("group_size must be > 0");
  if (!multiple_of(s.k, s.line_size)) return bad("k must be divisible by line_size");
  if (!multiple_of(s.n, s.line_size)) return bad("n must be divisible by line_size");
  if (!multiple_of(s.inner_k, s.line_size)) return bad("inner_k_size must be divisible by line_size");
  if (!multiple_of(s.n, s.tile_n)) return bad("n must be divisible by n_tile_size");
  if (!multiple_of(s.k, s.inner_k)) return bad("k must be divisible by inner_k_size");
  if (!multiple_of(s.tile_n, s.line_size * 8))
    return bad("n_tile_size must be divisible by line_size*8");
  if (!multiple_of(s.n, s.line_size * 8)) return bad("n must be divisible by line_size*8");
  if (!multiple_of(s.k, group_size)) return bad("k must be divisible by group_size");
  if (!(group_size >= s.inner_k && multiple_of(group_size, s.inner_k)))
    return bad("fast path requires group_size >= inner_k_size and divisible by inner_k_size");
  if (!(s.m_valid <= s.m)) return bad("m_valid must be <= m");
  if (!multiple_of(s.tile_n, s.line_size * n_lines_per_thread))
    return bad("tile_n must be divisible by line_size * N_LINES_PER_THREAD");
  if (!multiple_of(s.tile_m, rows_per_thread))
    return bad("m_tile_size must be divisible by ROWS_PER_THREAD");
  return CAWQ_OK;
}

// ROWS_PER_THREAD / N_LINES_PER_THREAD of awq_kernel_gemm.rs:84-87
static cawq_status validate_prefill(const cawq_shape_config& s, size_t g) {
  return validate_impl(s, g, 2, 2);
}
static cawq_status validate_decode(const cawq_shape_config& s, size_t g) {
  return validate_impl(s, g, 1, 4);
}

constexpr size_t kDecodeMThreshold = 8;  // DECODE_M_THRESHOLD, awq_kernel_gemm.rs:81

// AWQ_GEMM_FORCE_TILE_M (awq_gemm.rs:20-28): read once, accepted values 8|16|32.
static size_t forced_tile_m() {
  static size_t forced = [] {
    const char* raw = std::getenv("AWQ_GEMM_FORCE_TILE_M");
    if (!raw) return (size_t)0;
    char* end = nullptr;
    unsigned long v = std::strtoul(raw, &end, 10);
    while (end && (*end == ' ' || *end == '\t' || *end == '\n')) ++end;
    if (end == raw || (end && *end != '\0')) return (size_t)0;
    return (v == 8 || v == 16 || v == 32) ? (size_t)v : (size_t)0;
  }();
  return forced;
}

size_t select_tile_m(size_t m) {
  if (size_t f = forced_tile_m()) return f;
  if (m <= kDecodeMThreshold) return 8;  // DECODE_TILE_M
  if (m <= 16) return 16;                // TILE_M_SMALL
  return 32;                             // TILE_M_LARGE
}

size_t select_tile_n(size_t n) {
  if (n >= 128 && n % 128 == 0) return 128;
  if (n >= 64 && n % 64 == 0) return 64;
  return 32;
}

// K tile the module validates with. The reference uses INNER_K = 64
// (awq_gemm.rs:16); its own module tests also run group_size 32
// (awq_gemm.rs:408-503), which needs a 32-row K tile, so the K tile here is
// the largest of 64, 32, 16, 8, 4 that divides the group size.
static size_t module_inner_k(size_t g) {
  for (size_t t : {64, 32, 16, 8, 4}) {
    if (g % t == 0) return t;
  }
  return 64;
}

// Rules of AWQGEMMLinearConfig::build (awq_gemm.rs:77-95) that apply to a
// forward call, then the kernel rules with the module's tiles.
static cawq_status validate_module(size_t rows, size_t k, size_t n, size_t g) {
  auto bad = [](const std::string& m) { return fail(CAWQ_ERR_INVALID_SHAPE, m); };
  if (!(g > 0)) return bad("group_size must be > 0");
  if (n % 8 != 0) return bad("d_output must be divisible by 8");
  if (n % 32 != 0) return bad("d_output must be divisible by TILE_N (32)");
  if (k % g != 0) return bad("d_input must be divisible by group_size");
  cawq_shape_config s = {rows, k, n, select_tile_m(rows), select_tile_n(n), module_inner_k(g), 4,
                         rows};
  return rows <= kDecodeMThreshold ? validate_decode(s, g) : validate_prefill(s, g);
}

// --------------------------------------------------------- plan cache
using PlanKey = std::tuple<size_t, size_t, size_t, size_t, int>;
static std::mutex g_plan_mu;
static std::map<PlanKey, cawq_plan> g_plan_cache;

static int forced_path() {
  static int forced = [] {
    const char* raw = std::getenv("CUBE_AWQ_FORCE_PATH");
    if (!raw) return 0;
    if (!std::strcmp(raw, "decode")) return (int)CAWQ_PATH_DECODE;
    if (!std::strcmp(raw, "prefill")) return (int)CAWQ_PATH_PREFILL;
    if (!std::strcmp(raw, "generic")) return (int)CAWQ_PATH_GENERIC;
    return 0;
  }();
  return forced;
}

static bool plan_supports(const GemmProblem& p, const cawq_plan& plan, const DeviceInfo& dev) {
  switch (plan.path) {
    case CAWQ_PATH_DECODE: return decode_supports(p, plan, dev);
    case CAWQ_PATH_PREFILL: return prefill_supports(p, plan, dev);
    case CAWQ_PATH_GENERIC:
      return p.epi == 0 && p.nrep == 0 && generic_supports(p);
    default: return false;
  }
}

static cawq_plan generic_plan() {
  cawq_plan pl = {};
  pl.path = CAWQ_PATH_GENERIC;
  return pl;
}

static cawq_plan heuristic_plan(const GemmProblem& p, const DeviceInfo& dev) {
  const int fp = forced_path();
  if (fp == CAWQ_PATH_DECODE) {
    cawq_plan pl = decode_default_plan(p, dev);
    if (decode_supports(p, pl, dev)) return pl;
  } else if (fp == CAWQ_PATH_PREFILL) {
    cawq_plan pl = prefill_default_plan(p, dev);
    if (prefill_supports(p, pl, dev)) return pl;
  } else if (fp == CAWQ_PATH_GENERIC) {
    return generic_plan();
  }
  if (p.rows <= 16) {
    cawq_plan pl = decode_default_plan(p, dev);
    if (decode_supports(p, pl, dev)) return pl;
  }
  {
    cawq_plan pl = prefill_default_plan(p, dev);
    if (prefill_supports(p, pl, dev)) return pl;
  }
  if (p.rows <= 16) {
    cawq_plan pl = decode_default_plan(p, dev);
    if (decode_supports(p, pl, dev)) return pl;
  }
  return generic_plan();
}

static cawq_plan choose_plan(const GemmProblem& p, const DeviceInfo& dev) {
  if (forced_path() == 0) {
    std::lock_guard<std::mutex> lk(g_plan_mu);
    auto it = g_plan_cache.find(PlanKey(p.rows, p.k, p.n, p.g, p.dtype));
    if (it != g_plan_cache.end() && plan_supports(p, it->second, dev)) return it->second;
  }
  return heuristic_plan(p, dev);
}

static cawq_status run_plan(const GemmProblem& p, const cawq_plan& plan, const DeviceInfo& dev) {
  cudaError_t e;
  switch (plan.path) {
    case CAWQ_PATH_DECODE: e = launch_decode(p, plan, dev); break;
    case CAWQ_PATH_PREFILL: e = launch_prefill(p, plan, dev); break;
    case CAWQ_PATH_GENERIC: e = launch_generic(p); break;
    default: return fail(CAWQ_ERR_INVALID_ARGUMENT, "unknown plan path");
  }
  if (e != cudaSuccess) return cuda_fail(e, "kernel launch");
  return CAWQ_OK;
}

static bool valid_dtype(int dt) { return dt == CAWQ_F32 || dt == CAWQ_F16 || dt == CAWQ_BF16; }

static cawq_status check_gemm_pointers(const void* x, const void* qw, const void* qz,
                                       const void* sc, const void* out) {
  if (!x || !qw || !qz || !sc || !out)
    return fail(CAWQ_ERR_NULL_POINTER, "x, qweight, qzeros, scales and out must be non-null");
  return CAWQ_OK;
}

// The k and v outputs of cawq_gemm_qkv (out / ld_out hold q).
struct QkvOut {
  void* out_k;
  void* out_v;
  size_t ld_k, ld_v, col_k, col_v;
};

static cawq_status gemm_common(const void* x, const uint32_t* qweight, const uint32_t* qzeros,
                               const void* scales, const void* bias, void* out, size_t rows,
                               size_t k, size_t n, size_t g, cawq_dtype dtype,
                               cawq_dtype out_dtype, cawq_order order, size_t ld_out,
                               const cawq_plan* plan, void* stream, bool module_rules,
                               int epi = 0, const QkvOut* qkv = nullptr,
                               void* const* reps = nullptr, int nrep = 0) {
  if (!valid_dtype(dtype) || !valid_dtype(out_dtype))
    return fail(CAWQ_ERR_DTYPE, "dtype must be CAWQ_F32, CAWQ_F16 or CAWQ_BF16");
  if (out_dtype != dtype && out_dtype != CAWQ_F32)
    return fail(CAWQ_ERR_DTYPE, "out_dtype must equal dtype or be CAWQ_F32");
  if (order != CAWQ_ORDER_AWQ && order != CAWQ_ORDER_NATURAL)
    return fail(CAWQ_ERR_INVALID_ARGUMENT, "order must be CAWQ_ORDER_AWQ or CAWQ_ORDER_NATURAL");
  const size_t ocols = qkv ? qkv->col_k : epi ? n / 2 : n;  // columns of `out`
  if (ld_out == 0) ld_out = ocols;
  if (ld_out < ocols)
    return fail(CAWQ_ERR_INVALID_SHAPE, qkv ? "ld_q must be >= n_q"
                                        : epi ? "ld_out must be >= n / 2" : "ld_out must be >= n");
  if (module_rules) {
    if (!(k > 0)) return fail(CAWQ_ERR_INVALID_SHAPE, "input last dim (K) must be > 0");
    if (order == CAWQ_ORDER_AWQ) {
      // AWQGEMMLinear (awq_gemm.rs:77-95 and the kernel rules it launches with)
      if (rows > 0) {
        cawq_status st = validate_module(rows, k, n, g);
        if (st != CAWQ_OK) return st;
      }
    } else {
      // AWQLinear (awq_dequantize.rs:25-28): its forward never runs the GEMM rules
      if (n % 8 != 0) return fail(CAWQ_ERR_INVALID_SHAPE, "assertion failed: self.d_output % 8 == 0");
      if (g == 0 || k % g != 0)
        return fail(CAWQ_ERR_INVALID_SHAPE, "assertion failed: self.d_input % self.group_size == 0");
      if (n % 32 != 0) return fail(CAWQ_ERR_INVALID_SHAPE, "assertion failed: self.d_output % 32 == 0");
    }
  }
  if (rows == 0) return CAWQ_OK;
  cawq_status st = check_gemm_pointers(x, qweight, qzeros, scales, out);
  if (st != CAWQ_OK) return st;
  DeviceInfo dev;
  if ((st = require_sm100(&dev)) != CAWQ_OK) return st;
  GemmProblem p = {x, qweight, qzeros, scales, bias, out, rows, k, n, g, ld_out,
                   dtype, out_dtype, order, static_cast<cudaStream_t>(stream), epi};
  if (qkv) {
    if (!qkv->out_k || !qkv->out_v)
      return fail(CAWQ_ERR_NULL_POINTER, "q_out, k_out and v_out must be non-null");
    p.out_k = qkv->out_k;
    p.out_v = qkv->out_v;
    p.ld_k = qkv->ld_k;
    p.ld_v = qkv->ld_v;
    p.col_k = qkv->col_k;
    p.col_v = qkv->col_v;
  }
  for (int i = 0; i < nrep; ++i) p.rep[i] = reps[i];
  p.nrep = nrep;
  cawq_plan pl = plan ? *plan : choose_plan(p, dev);
  if (plan && !plan_supports(p, pl, dev))
    return fail(CAWQ_ERR_INVALID_ARGUMENT, "the plan cannot run this problem");
  if (!plan && !plan_supports(p, pl, dev)) {
    return fail(CAWQ_ERR_INVALID_SHAPE, "no kernel supports this problem");
  }
  return run_plan(p, pl, dev);
}

}  // namespace cawq

using namespace cawq;

// ========================================================== C ABI
CAWQ_API const char* cawq_last_error(void) { return g_last_error.c_str(); }

CAWQ_API const char* cawq_version(void) { return "cube_awq 0.1 sm_100a"; }

CAWQ_API int cawq_device_supported(int device) {
  int major = 0;
  if (cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, device) != cudaSuccess) {
    cudaGetLastError();
    return 0;
  }
  return major == 10 ? 1 : 0;
}

CAWQ_API cawq_status cawq_device_error(int reset, uint32_t* word) {
  if (!word) return fail(CAWQ_ERR_NULL_POINTER, "word must be non-null");
  cudaError_t e = read_device_error(word, reset);
  if (e != cudaSuccess) return cuda_fail(e, "cawq_device_error");
  return CAWQ_OK;
}

CAWQ_API cawq_status cawq_shape_config_new_with_valid_m(size_t m, size_t n, size_t k,
                                                        size_t tile_m, size_t tile_n,
                                                        size_t inner_k, size_t m_valid,
                                                        cawq_shape_config* out) {
  if (!out) return fail(CAWQ_ERR_NULL_POINTER, "out must be non-null");
  out->m = m;
  out->k = k;
  out->n = n;
  out->tile_m = tile_m;
  out->tile_n = tile_n;
  out->inner_k = inner_k;
  out->line_size = 4;
  out->m_valid = m_valid;
  return CAWQ_OK;
}

CAWQ_API cawq_status cawq_shape_config_new(size_t m, size_t n, size_t k, size_t tile_m,
                                           size_t tile_n, size_t inner_k, cawq_shape_config* out) {
  return cawq_shape_config_new_with_valid_m(m, n, k, tile_m, tile_n, inner_k, m, out);
}

CAWQ_API cawq_status cawq_validate_launch_params(const cawq_shape_config* shape, size_t g) {
  if (!shape) return fail(CAWQ_ERR_NULL_POINTER, "shape must be non-null");
  return validate_prefill(*shape, g);
}

CAWQ_API cawq_status cawq_validate_decode_launch_params(const cawq_shape_config* shape, size_t g) {
  if (!shape) return fail(CAWQ_ERR_NULL_POINTER, "shape must be non-null");
  return validate_decode(*shape, g);
}

CAWQ_API size_t cawq_select_tile_m(size_t m) { return select_tile_m(m); }
CAWQ_API size_t cawq_select_tile_n(size_t n) { return select_tile_n(n); }

static size_t numel(const cawq_tensor_desc& d) {
  size_t v = 1;
  for (int i = 0; i < d.rank; ++i) v *= d.shape[i];
  return v;
}

CAWQ_API cawq_status cawq_awq_gemm_linear(const cawq_gemm_args* a, const cawq_shape_config* shape,
                                          void* stream) {
  if (!a) return fail(CAWQ_ERR_NULL_POINTER, "args must be non-null");
  auto bad = [](const std::string& m) { return fail(CAWQ_ERR_INVALID_SHAPE, m); };
  for (const cawq_tensor_desc* d : {&a->input, &a->qweight, &a->qzeros, &a->scales, &a->output}) {
    if (d->rank < 0 || d->rank > CAWQ_MAX_RANK)
      return fail(CAWQ_ERR_INVALID_ARGUMENT, "tensor rank must be in [0, 8]");
  }
  // awq_kernel_gemm.rs:636-646
  if (a->input.rank < 2) return bad("input must have shape [.., M, K] or [M, K]");
  if (a->qweight.rank < 2) return bad("qweight must have shape [K, N/8]");
  if (a->qzeros.rank < 2) return bad("qzeros must have shape [K/G, N/8]");
  if (a->scales.rank < 2) return bad("scales must have shape [K/G, N]");
  if (a->output.rank < 2) return bad("output must have shape [.., M, N] or [M, N]");
  if (a->qweight.elem_size != 4) return fail(CAWQ_ERR_DTYPE, "qweight must have i32/u32 dtype");
  if (a->qzeros.elem_size != 4) return fail(CAWQ_ERR_DTYPE, "qzeros must have i32/u32 dtype");
  if (!valid_dtype(a->dtype)) return fail(CAWQ_ERR_DTYPE, "dtype must be CAWQ_F32, CAWQ_F16 or CAWQ_BF16");
  const size_t es = dtype_size(a->dtype);
  if (a->input.elem_size != es || a->scales.elem_size != es || a->output.elem_size != es ||
      (a->bias.data && a->bias.elem_size != es))
    return fail(CAWQ_ERR_DTYPE, "input, scales, bias and output must all have the element type F");

  // shape: the caller's ShapeConfig, or the module's choice (awq_gemm.rs:205-207)
  const size_t input_k = a->input.shape[a->input.rank - 1];
  cawq_shape_config sh;
  if (shape) {
    sh = *shape;
  } else {
    const size_t m = input_k ? numel(a->input) / input_k : 0;
    const size_t n = a->qweight.shape[1] * 8;
    sh = {m, input_k, n, select_tile_m(m), select_tile_n(n), module_inner_k(a->group_size), 4, m};
  }
  // awq_kernel_gemm.rs:648-673
  if (!(input_k > 0)) return bad("input K must be > 0");
  if (input_k != sh.k) return bad(fmt("input K must match shape.k (left: %zu, right: %zu)", input_k, sh.k));
  const size_t input_numel = numel(a->input);
  const size_t launch_m = input_numel / input_k;
  if (input_numel % input_k != 0) return bad("input elements must be divisible by K");
  const size_t output_n = a->output.shape[a->output.rank - 1];
  if (!(output_n > 0)) return bad("output N must be > 0");
  if (output_n != sh.n) return bad(fmt("output N must match shape.n (left: %zu, right: %zu)", output_n, sh.n));
  const size_t output_numel = numel(a->output);
  const size_t output_rows = output_numel / output_n;
  if (output_numel % output_n != 0) return bad("output elements must be divisible by N");
  if (output_rows != launch_m)
    return bad(fmt("output rows must match flattened input rows (left: %zu, right: %zu)", output_rows, launch_m));
  // m_valid resolution, awq_kernel_gemm.rs:675-681
  size_t m_valid;
  if (sh.m == launch_m) {
    m_valid = sh.m_valid;
  } else if (sh.m > 0 && launch_m % sh.m == 0 && sh.m_valid == sh.m) {
    m_valid = launch_m;
  } else {
    m_valid = std::min(launch_m, sh.m_valid);
  }
  cawq_shape_config ls = {launch_m, sh.k, sh.n, sh.tile_m, sh.tile_n, sh.inner_k, sh.line_size, m_valid};
  cawq_status st = launch_m <= kDecodeMThreshold ? validate_decode(ls, a->group_size)
                                                 : validate_prefill(ls, a->group_size);
  if (st != CAWQ_OK) return st;
  // awq_kernel_gemm.rs:698-724
  const size_t groups = ls.k / a->group_size;
  if (a->qweight.shape[0] != ls.k) return bad("qweight K must match shape.k");
  if (a->qweight.shape[1] != ls.n / 8) return bad("qweight packed N must be N/8");
  if (a->qzeros.shape[0] != groups) return bad("qzeros rows must be K/group_size");
  if (a->qzeros.shape[1] != ls.n / 8) return bad("qzeros packed N must be N/8");
  if (a->scales.shape[0] != groups) return bad("scales rows must be K/group_size");
  if (a->scales.shape[1] != ls.n) return bad("scales N must match shape.n");
  if (a->bias.data && (a->bias.rank < 1 || numel(a->bias) != ls.n))
    return bad("bias must have shape [N]");
  return gemm_common(a->input.data, static_cast<const uint32_t*>(a->qweight.data),
                     static_cast<const uint32_t*>(a->qzeros.data), a->scales.data, a->bias.data,
                     const_cast<void*>(a->output.data), m_valid, ls.k, ls.n, a->group_size,
                     a->dtype, a->dtype, CAWQ_ORDER_AWQ, ls.n, nullptr, stream, false);
}

CAWQ_API cawq_status cawq_gemm(const void* x, const uint32_t* qweight, const uint32_t* qzeros,
                               const void* scales, const void* bias, void* out, size_t rows,
                               size_t k, size_t n, size_t group_size, cawq_dtype dtype,
                               cawq_dtype out_dtype, cawq_order order, size_t ld_out,
                               void* stream) {
  return gemm_common(x, qweight, qzeros, scales, bias, out, rows, k, n, group_size, dtype,
                     out_dtype, order, ld_out, nullptr, stream, true);
}

CAWQ_API cawq_status cawq_gemm_silu_mul(const void* x, const uint32_t* qweight,
                                        const uint32_t* qzeros, const void* scales,
                                        const void* bias, void* out, size_t rows, size_t k,
                                        size_t n, size_t group_size, cawq_dtype dtype,
                                        size_t ld_out, void* stream) {
  if (dtype != CAWQ_F16 && dtype != CAWQ_BF16)
    return fail(CAWQ_ERR_DTYPE, "the SiLU-gated GEMM takes CAWQ_F16 or CAWQ_BF16");
  if (n % 256 != 0)
    return fail(CAWQ_ERR_INVALID_SHAPE,
                fmt("n = %zu must be a multiple of 256 (128-column gate / up blocks)", n));
  return gemm_common(x, qweight, qzeros, scales, bias, out, rows, k, n, group_size, dtype, dtype,
                     CAWQ_ORDER_AWQ, ld_out, nullptr, stream, true, 1);
}

CAWQ_API cawq_status cawq_gemm_qkv(const void* x, const uint32_t* qweight, const uint32_t* qzeros,
                                   const void* scales, const void* bias, void* q_out, void* k_out,
                                   void* v_out, size_t rows, size_t k, size_t n_q, size_t n_kv,
                                   size_t group_size, cawq_dtype dtype, cawq_dtype out_dtype,
                                   size_t ld_q, size_t ld_k, size_t ld_v, void* stream) {
  if (n_q == 0 || n_kv == 0 || n_q % 32 != 0 || n_kv % 32 != 0)
    return fail(CAWQ_ERR_INVALID_SHAPE,
                fmt("n_q = %zu and n_kv = %zu must be positive multiples of 32", n_q, n_kv));
  if (ld_k == 0) ld_k = n_kv;
  if (ld_v == 0) ld_v = n_kv;
  if (ld_k < n_kv || ld_v < n_kv)
    return fail(CAWQ_ERR_INVALID_SHAPE, "ld_k and ld_v must be >= n_kv");
  if (ld_q >= (1ull << 31) || ld_k >= (1ull << 31) || ld_v >= (1ull << 31))
    return fail(CAWQ_ERR_INVALID_SHAPE, "row strides must be below 2^31 elements");
  const QkvOut qkv = {k_out, v_out, ld_k, ld_v, n_q, n_q + n_kv};
  return gemm_common(x, qweight, qzeros, scales, bias, q_out, rows, k, n_q + 2 * n_kv, group_size,
                     dtype, out_dtype, CAWQ_ORDER_AWQ, ld_q, nullptr, stream, true, 0, &qkv);
}

CAWQ_API cawq_status cawq_interleave_gate_up(const void* src, void* dst, size_t rows,
                                             size_t width_elems, size_t block_elems,
                                             size_t elem_size, void* stream) {
  if (!src || !dst) return fail(CAWQ_ERR_NULL_POINTER, "src and dst must be non-null");
  if (elem_size != 2 && elem_size != 4)
    return fail(CAWQ_ERR_INVALID_ARGUMENT, "elem_size must be 2 or 4");
  if (block_elems == 0 || width_elems % block_elems != 0)
    return fail(CAWQ_ERR_INVALID_SHAPE, "width_elems must be a multiple of block_elems");
  if (rows == 0 || width_elems == 0) return CAWQ_OK;
  DeviceInfo dev;
  cawq_status st = require_sm100(&dev);
  if (st != CAWQ_OK) return st;
  cudaError_t e = launch_interleave_gate_up(src, dst, rows, width_elems, block_elems, elem_size,
                                            static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "interleave launch");
  return CAWQ_OK;
}

CAWQ_API cawq_status cawq_gemm_silu_mul_with_plan(const void* x, const uint32_t* qweight,
                                                  const uint32_t* qzeros, const void* scales,
                                                  const void* bias, void* out, size_t rows,
                                                  size_t k, size_t n, size_t group_size,
                                                  cawq_dtype dtype, size_t ld_out,
                                                  const cawq_plan* plan, void* stream) {
  if (!plan) return fail(CAWQ_ERR_NULL_POINTER, "plan must be non-null");
  if (dtype != CAWQ_F16 && dtype != CAWQ_BF16)
    return fail(CAWQ_ERR_DTYPE, "the SiLU-gated GEMM takes CAWQ_F16 or CAWQ_BF16");
  if (n % 256 != 0)
    return fail(CAWQ_ERR_INVALID_SHAPE,
                fmt("n = %zu must be a multiple of 256 (128-column gate / up blocks)", n));
  return gemm_common(x, qweight, qzeros, scales, bias, out, rows, k, n, group_size, dtype, dtype,
                     CAWQ_ORDER_AWQ, ld_out, plan, stream, true, 1);
}

CAWQ_API cawq_status cawq_gemm_with_plan(const void* x, const uint32_t* qweight,
                                         const uint32_t* qzeros, const void* scales,
                                         const void* bias, void* out, size_t rows, size_t k,
                                         size_t n, size_t group_size, cawq_dtype dtype,
                                         cawq_dtype out_dtype, cawq_order order, size_t ld_out,
                                         const cawq_plan* plan, void* stream) {
  if (!plan) return fail(CAWQ_ERR_NULL_POINTER, "plan must be non-null");
  return gemm_common(x, qweight, qzeros, scales, bias, out, rows, k, n, group_size, dtype,
                     out_dtype, order, ld_out, plan, stream, true);
}

CAWQ_API cawq_status cawq_plan_get(size_t rows, size_t k, size_t n, size_t g, cawq_dtype dtype,
                                   cawq_plan* plan) {
  if (!plan) return fail(CAWQ_ERR_NULL_POINTER, "plan must be non-null");
  DeviceInfo dev;
  cawq_status st = require_sm100(&dev);
  if (st != CAWQ_OK) return st;
  // alignment-agnostic view: assume 256-byte aligned buffers
  const void* al = reinterpret_cast<const void*>(static_cast<uintptr_t>(256));
  GemmProblem p = {al, static_cast<const uint32_t*>(al), static_cast<const uint32_t*>(al), al,
                   nullptr, const_cast<void*>(al), rows, k, n, g, n, dtype, dtype,
                   CAWQ_ORDER_AWQ, nullptr};
  *plan = choose_plan(p, dev);
  return CAWQ_OK;
}

CAWQ_API cawq_status cawq_plan_set(size_t rows, size_t k, size_t n, size_t g, cawq_dtype dtype,
                                   const cawq_plan* plan) {
  if (!plan) return fail(CAWQ_ERR_NULL_POINTER, "plan must be non-null");
  std::lock_guard<std::mutex> lk(g_plan_mu);
  g_plan_cache[PlanKey(rows, k, n, g, dtype)] = *plan;
  return CAWQ_OK;
}

CAWQ_API void cawq_plan_cache_clear(void) {
  std::lock_guard<std::mutex> lk(g_plan_mu);
  g_plan_cache.clear();
}

CAWQ_API cawq_status cawq_autotune(const void* x, const uint32_t* qweight, const uint32_t* qzeros,
                                   const void* scales, void* out, size_t rows, size_t k, size_t n,
                                   size_t g, cawq_dtype dtype, cawq_plan* best, void* stream) {
  if (!best) return fail(CAWQ_ERR_NULL_POINTER, "best must be non-null");
  cawq_status st = check_gemm_pointers(x, qweight, qzeros, scales, out);
  if (st != CAWQ_OK) return st;
  if (rows == 0) return fail(CAWQ_ERR_INVALID_SHAPE, "m must be > 0");
  if ((st = validate_module(rows, k, n, g)) != CAWQ_OK) return st;
  DeviceInfo dev;
  if ((st = require_sm100(&dev)) != CAWQ_OK) return st;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  GemmProblem p = {x, qweight, qzeros, scales, nullptr, out, rows, k, n, g, n,
                   dtype, dtype, CAWQ_ORDER_AWQ, s};
  cawq_plan cands[160];
  int nc = 0, c2 = 0;
  if (rows <= 16) decode_candidates(p, dev, cands, &nc, 128);
  prefill_candidates(p, dev, cands + nc, &c2, 160 - nc - 1);
  nc += c2;
  cands[nc++] = generic_plan();
  cudaEvent_t e0, e1;
  cudaEventCreate(&e0);
  cudaEventCreate(&e1);
  float best_ms = 1e30f;
  cawq_plan best_plan = generic_plan();
  for (int i = 0; i < nc; ++i) {
    if (!plan_supports(p, cands[i], dev)) continue;
    bool okp = true;
    for (int w = 0; w < 3 && okp; ++w) okp = run_plan(p, cands[i], dev) == CAWQ_OK;
    if (!okp) continue;
    const int reps = 20;
    cudaEventRecord(e0, s);
    for (int r = 0; r < reps; ++r) run_plan(p, cands[i], dev);
    cudaEventRecord(e1, s);
    if (cudaEventSynchronize(e1) != cudaSuccess) {
      cudaEventDestroy(e0);
      cudaEventDestroy(e1);
      return cuda_fail(cudaGetLastError(), "autotune");
    }
    float ms = 0.f;
    cudaEventElapsedTime(&ms, e0, e1);
    if (ms < best_ms) {
      best_ms = ms;
      best_plan = cands[i];
    }
  }
  cudaEventDestroy(e0);
  cudaEventDestroy(e1);
  {
    std::lock_guard<std::mutex> lk(g_plan_mu);
    g_plan_cache[PlanKey(rows, k, n, g, dtype)] = best_plan;
  }
  *best = best_plan;
  return CAWQ_OK;
}

// ------------------------------------------------------------ dequant
static cawq_status dequant_common(const uint32_t* qw, const uint32_t* qz, const void* sc,
                                  void* out, size_t k, size_t n, size_t g, cawq_dtype dtype,
                                  cawq_order order, void* stream) {
  if (!valid_dtype(dtype)) return fail(CAWQ_ERR_DTYPE, "dtype must be CAWQ_F32, CAWQ_F16 or CAWQ_BF16");
  if (order != CAWQ_ORDER_AWQ && order != CAWQ_ORDER_NATURAL)
    return fail(CAWQ_ERR_INVALID_ARGUMENT, "order must be CAWQ_ORDER_AWQ or CAWQ_ORDER_NATURAL");
  if (n % 32 != 0) return fail(CAWQ_ERR_INVALID_SHAPE, "assertion failed: out_width % 32 == 0");
  if (!(g > 0)) return fail(CAWQ_ERR_INVALID_SHAPE, "group_size must be > 0");
  if (k % g != 0) return fail(CAWQ_ERR_INVALID_SHAPE, "k must be divisible by group_size");
  if (k == 0 || n == 0) return CAWQ_OK;
  if (!qw || !qz || !sc || !out)
    return fail(CAWQ_ERR_NULL_POINTER, "qweight, qzeros, scales and out must be non-null");
  if (k >= (1ull << 32) || n / 8 >= (1ull << 31))
    return fail(CAWQ_ERR_INVALID_SHAPE, "dequantize supports K < 2^32 and N/8 < 2^31");
  DeviceInfo dev;
  cawq_status st = require_sm100(&dev);
  if (st != CAWQ_OK) return st;
  cudaError_t e = launch_dequant(qw, qz, sc, out, k, n, g, dtype, order,
                                 static_cast<cudaStream_t>(stream), dev.sm_count);
  if (e != cudaSuccess) return cuda_fail(e, "dequantize launch");
  return CAWQ_OK;
}

CAWQ_API cawq_status cawq_dequantize(const uint32_t* qweight, const uint32_t* qzeros,
                                     const void* scales, void* out, size_t k, size_t n,
                                     size_t group_size, cawq_dtype dtype, cawq_order order,
                                     void* stream) {
  return dequant_common(qweight, qzeros, scales, out, k, n, group_size, dtype, order, stream);
}

CAWQ_API cawq_status cawq_dequantize_native(const cawq_tensor_desc* qweight,
                                            const cawq_tensor_desc* qzeros,
                                            const cawq_tensor_desc* scales,
                                            const cawq_tensor_desc* output, size_t group_size,
                                            cawq_dtype dtype, cawq_order order, void* stream) {
  if (!qweight || !qzeros || !scales || !output)
    return fail(CAWQ_ERR_NULL_POINTER, "tensor descriptors must be non-null");
  // awq_kernel.rs:73-84
  if (qweight->elem_size != 4)
    return fail(CAWQ_ERR_DTYPE,
                fmt("AWQ packed q_weight must use 32-bit elements (i32/u32), got elem_size=%zu.",
                    qweight->elem_size));
  if (qzeros->elem_size != 4)
    return fail(CAWQ_ERR_DTYPE,
                fmt("AWQ packed q_zeros must use 32-bit elements (i32/u32), got elem_size=%zu.",
                    qzeros->elem_size));
  if (output->rank < 1 || qweight->rank != 2 || qzeros->rank != 2 || scales->rank != 2)
    return fail(CAWQ_ERR_INVALID_SHAPE,
                "qweight, qzeros and scales must be 2-D and output at least 1-D");
  // awq_kernel.rs:86-87
  const size_t out_width = output->shape[output->rank - 1];
  if (out_width % 32 != 0) return fail(CAWQ_ERR_INVALID_SHAPE, "assertion failed: out_width % 32 == 0");
  if (!valid_dtype(dtype)) return fail(CAWQ_ERR_DTYPE, "dtype must be CAWQ_F32, CAWQ_F16 or CAWQ_BF16");
  if (scales->elem_size != dtype_size(dtype) || output->elem_size != dtype_size(dtype))
    return fail(CAWQ_ERR_DTYPE, "scales and output must have the element type F");
  const size_t k = qweight->shape[0];
  size_t out_rows = 1;
  for (int i = 0; i + 1 < output->rank; ++i) out_rows *= output->shape[i];
  if (qweight->shape[1] * 8 != out_width) return fail(CAWQ_ERR_INVALID_SHAPE, "qweight packed N must be N/8");
  if (out_rows != k) return fail(CAWQ_ERR_INVALID_SHAPE, "output rows must match qweight K");
  if (group_size == 0) return fail(CAWQ_ERR_INVALID_SHAPE, "group_size must be > 0");
  if (qzeros->shape[0] != k / group_size || qzeros->shape[1] != out_width / 8)
    return fail(CAWQ_ERR_INVALID_SHAPE, "qzeros must have shape [K/group_size, N/8]");
  if (scales->shape[0] != k / group_size || scales->shape[1] != out_width)
    return fail(CAWQ_ERR_INVALID_SHAPE, "scales must have shape [K/group_size, N]");
  return dequant_common(static_cast<const uint32_t*>(qweight->data),
                        static_cast<const uint32_t*>(qzeros->data), scales->data,
                        const_cast<void*>(output->data), k, out_width, group_size, dtype, order,
                        stream);
}

// ------------------------------------------------------------ tensor parallel
CAWQ_API cawq_status cawq_tp_column_shard(size_t n, int world, int rank, size_t* n_begin,
                                          size_t* n_len) {
  if (!n_begin || !n_len) return fail(CAWQ_ERR_NULL_POINTER, "outputs must be non-null");
  if (world < 1 || rank < 0 || rank >= world)
    return fail(CAWQ_ERR_INVALID_ARGUMENT, "rank must be in [0, world)");
  if (n % (32ull * world) != 0)
    return fail(CAWQ_ERR_INVALID_SHAPE, fmt("column-parallel shard needs N %% (32 * world) == 0 (N=%zu, world=%d)", n, world));
  *n_len = n / world;
  *n_begin = *n_len * rank;
  return CAWQ_OK;
}

CAWQ_API cawq_status cawq_tp_row_shard(size_t k, size_t g, int world, int rank, size_t* k_begin,
                                       size_t* k_len) {
  if (!k_begin || !k_len) return fail(CAWQ_ERR_NULL_POINTER, "outputs must be non-null");
  if (world < 1 || rank < 0 || rank >= world)
    return fail(CAWQ_ERR_INVALID_ARGUMENT, "rank must be in [0, world)");
  if (g == 0 || k % g != 0) return fail(CAWQ_ERR_INVALID_SHAPE, "k must be divisible by group_size");
  if ((k / g) % world != 0)
    return fail(CAWQ_ERR_INVALID_SHAPE,
                fmt("row-parallel shard needs (K / group_size) %% world == 0 (groups=%zu, world=%d)", k / g, world));
  *k_len = k / world;
  *k_begin = *k_len * rank;
  return CAWQ_OK;
}

CAWQ_API cawq_status cawq_tp_interleave_columns(const void* src, void* dst, size_t rows, size_t n,
                                                int world, cawq_dtype dtype, void* stream) {
  if (!src || !dst) return fail(CAWQ_ERR_NULL_POINTER, "src and dst must be non-null");
  if (world < 1 || n % world != 0) return fail(CAWQ_ERR_INVALID_SHAPE, "n must be divisible by world");
  if (!valid_dtype(dtype)) return fail(CAWQ_ERR_DTYPE, "dtype must be CAWQ_F32, CAWQ_F16 or CAWQ_BF16");
  if (rows == 0 || n == 0) return CAWQ_OK;
  DeviceInfo dev;
  cawq_status st = require_sm100(&dev);
  if (st != CAWQ_OK) return st;
  cudaError_t e = launch_interleave_columns(src, dst, rows, n, world, dtype_size(dtype),
                                            static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "interleave launch");
  return CAWQ_OK;
}

// ------------------------------------------------------ tensor parallel
// NCCL is loaded at run time (libnccl.so.2; in a process that already holds
// torch's copy, that one), so libcube_awq.so links no NCCL.
namespace {

struct NcclApi {
  bool ok = false;
  std::string why;
  ncclResult_t (*get_unique_id)(ncclUniqueId*) = nullptr;
  ncclResult_t (*init_rank_config)(ncclComm_t*, int, ncclUniqueId, int, ncclConfig_t*) = nullptr;
  ncclResult_t (*destroy)(ncclComm_t) = nullptr;
  ncclResult_t (*abort)(ncclComm_t) = nullptr;
  ncclResult_t (*async_error)(ncclComm_t, ncclResult_t*) = nullptr;
  ncclResult_t (*all_gather)(const void*, void*, size_t, ncclDataType_t, ncclComm_t,
                             cudaStream_t) = nullptr;
  ncclResult_t (*all_reduce)(const void*, void*, size_t, ncclDataType_t, ncclRedOp_t, ncclComm_t,
                             cudaStream_t) = nullptr;
  const char* (*error_string)(ncclResult_t) = nullptr;
};

const NcclApi& nccl() {
  static NcclApi api;
  static std::once_flag once;
  std::call_once(once, [] {
    void* h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
    if (!h) h = dlopen("libnccl.so", RTLD_NOW | RTLD_GLOBAL);
    if (!h) {
      api.why = "libnccl.so.2 not found";
      return;
    }
    auto sym = [&](const char* name) { return dlsym(h, name); };
    api.get_unique_id = reinterpret_cast<decltype(api.get_unique_id)>(sym("ncclGetUniqueId"));
    api.init_rank_config =
        reinterpret_cast<decltype(api.init_rank_config)>(sym("ncclCommInitRankConfig"));
    api.destroy = reinterpret_cast<decltype(api.destroy)>(sym("ncclCommDestroy"));
    api.abort = reinterpret_cast<decltype(api.abort)>(sym("ncclCommAbort"));
    api.async_error = reinterpret_cast<decltype(api.async_error)>(sym("ncclCommGetAsyncError"));
    api.all_gather = reinterpret_cast<decltype(api.all_gather)>(sym("ncclAllGather"));
    api.all_reduce = reinterpret_cast<decltype(api.all_reduce)>(sym("ncclAllReduce"));
    api.error_string = reinterpret_cast<decltype(api.error_string)>(sym("ncclGetErrorString"));
    api.ok = api.get_unique_id && api.init_rank_config && api.destroy && api.abort &&
             api.async_error && api.all_gather && api.all_reduce && api.error_string;
    if (!api.ok) api.why = "libnccl.so.2 lacks a required symbol";
  });
  return api;
}

cawq_status nccl_fail(ncclResult_t r, const char* where) {
  const NcclApi& a = nccl();
  return fail(CAWQ_ERR_NCCL, fmt("%s: %s", where, a.ok ? a.error_string(r) : a.why.c_str()));
}

ncclDataType_t nccl_type(int dt) {
  return dt == CAWQ_F32 ? ncclFloat32 : dt == CAWQ_F16 ? ncclFloat16 : ncclBfloat16;
}

}  // namespace

struct cawq_tp_comm {
  ncclComm_t comm = nullptr;
  int world = 0, rank = 0, device = -1;
  int timeout_ms = 60000;
};

// A non-blocking communicator returns ncclInProgress while it sets up; wait
// for the result, at most the communicator's timeout, then abort it.
static cawq_status nccl_settle(cawq_tp_comm* c, ncclResult_t r, const char* where) {
  const NcclApi& a = nccl();
  if (r != ncclSuccess && r != ncclInProgress) return nccl_fail(r, where);
  const auto t0 = std::chrono::steady_clock::now();
  for (;;) {
    ncclResult_t st = ncclSuccess;
    ncclResult_t q = a.async_error(c->comm, &st);
    if (q != ncclSuccess) return nccl_fail(q, where);
    if (st == ncclSuccess) return CAWQ_OK;
    if (st != ncclInProgress) return nccl_fail(st, where);
    const auto ms = std::chrono::duration_cast<std::chrono::milliseconds>(
                        std::chrono::steady_clock::now() - t0)
                        .count();
    if (ms > c->timeout_ms) {
      return fail(CAWQ_ERR_TIMEOUT, fmt("%s: NCCL did not finish within %d ms", where,
                                        c->timeout_ms));
    }
    // an enqueue settles in microseconds; only a communicator set-up waits long
    if (ms < 20) {
      std::this_thread::yield();
    } else {
      std::this_thread::sleep_for(std::chrono::microseconds(200));
    }
  }
}

CAWQ_API cawq_status cawq_tp_unique_id(uint8_t* id) {
  if (!id) return fail(CAWQ_ERR_NULL_POINTER, "id must be non-null");
  static_assert(sizeof(ncclUniqueId) == CAWQ_TP_ID_BYTES, "NCCL unique id size");
  const NcclApi& a = nccl();
  if (!a.ok) return fail(CAWQ_ERR_NCCL, a.why);
  ncclUniqueId u;
  ncclResult_t r = a.get_unique_id(&u);
  if (r != ncclSuccess) return nccl_fail(r, "ncclGetUniqueId");
  std::memcpy(id, &u, sizeof(u));
  return CAWQ_OK;
}

CAWQ_API cawq_status cawq_tp_init(int world, int rank, const uint8_t* id, int timeout_ms,
                                  cawq_tp_comm** comm) {
  if (!id || !comm) return fail(CAWQ_ERR_NULL_POINTER, "id and comm must be non-null");
  *comm = nullptr;
  if (world < 1 || rank < 0 || rank >= world)
    return fail(CAWQ_ERR_INVALID_ARGUMENT, "rank must be in [0, world)");
  DeviceInfo dev;
  cawq_status st = require_sm100(&dev);
  if (st != CAWQ_OK) return st;
  const NcclApi& a = nccl();
  if (!a.ok) return fail(CAWQ_ERR_NCCL, a.why);
  auto* c = new cawq_tp_comm();
  c->world = world;
  c->rank = rank;
  c->device = dev.device;
  c->timeout_ms = timeout_ms > 0 ? timeout_ms : 60000;
  ncclUniqueId u;
  std::memcpy(&u, id, sizeof(u));
  ncclConfig_t cfg = NCCL_CONFIG_INITIALIZER;
  cfg.blocking = 0;
  ncclResult_t r = a.init_rank_config(&c->comm, world, u, rank, &cfg);
  st = nccl_settle(c, r, "ncclCommInitRankConfig");
  if (st != CAWQ_OK) {
    if (c->comm) a.abort(c->comm);
    delete c;
    return st;
  }
  *comm = c;
  return CAWQ_OK;
}

CAWQ_API cawq_status cawq_tp_destroy(cawq_tp_comm* comm) {
  if (!comm) return CAWQ_OK;
  const NcclApi& a = nccl();
  cawq_status st = CAWQ_OK;
  if (comm->comm) {
    ncclResult_t r = a.destroy(comm->comm);
    if (r == ncclInProgress) st = nccl_settle(comm, r, "ncclCommDestroy");
    else if (r != ncclSuccess) st = nccl_fail(r, "ncclCommDestroy");
  }
  delete comm;
  return st;
}

CAWQ_API cawq_status cawq_tp_info(const cawq_tp_comm* comm, int* world, int* rank) {
  if (!comm || !world || !rank) return fail(CAWQ_ERR_NULL_POINTER, "arguments must be non-null");
  *world = comm->world;
  *rank = comm->rank;
  return CAWQ_OK;
}

static cawq_status tp_check(const cawq_tp_comm* comm) {
  if (!comm || !comm->comm) return fail(CAWQ_ERR_NULL_POINTER, "comm must be an initialised communicator");
  int d = -1;
  cudaError_t e = cudaGetDevice(&d);
  if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
  if (d != comm->device)
    return fail(CAWQ_ERR_INVALID_ARGUMENT,
                fmt("current device %d is not the communicator's device %d", d, comm->device));
  return CAWQ_OK;
}

CAWQ_API cawq_status cawq_gemm_colpar(const cawq_tp_comm* comm, const void* x,
                                      const uint32_t* qweight, const uint32_t* qzeros,
                                      const void* scales, const void* bias, void* out,
                                      void* gather, size_t rows, size_t k, size_t n,
                                      size_t group_size, cawq_dtype dtype, void* stream) {
  cawq_status st = tp_check(comm);
  if (st != CAWQ_OK) return st;
  if (!valid_dtype(dtype)) return fail(CAWQ_ERR_DTYPE, "dtype must be CAWQ_F32, CAWQ_F16 or CAWQ_BF16");
  size_t n0 = 0, nl = 0;
  if ((st = cawq_tp_column_shard(n, comm->world, comm->rank, &n0, &nl)) != CAWQ_OK) return st;
  if (rows == 0) return CAWQ_OK;
  if (!out) return fail(CAWQ_ERR_NULL_POINTER, "out must be non-null");
  if (!gather) {
    if (rows != 1) return fail(CAWQ_ERR_NULL_POINTER, "gather workspace is required when rows > 1");
    gather = out;  // [world][1][n/world] is [1][n]
  }
  const size_t es = dtype_size(dtype);
  const size_t count = rows * nl;
  void* mine = static_cast<uint8_t*>(gather) + comm->rank * count * es;
  st = gemm_common(x, qweight, qzeros, scales, bias, mine, rows, k, nl, group_size, dtype, dtype,
                   CAWQ_ORDER_AWQ, nl, nullptr, stream, true);
  if (st != CAWQ_OK) return st;
  const NcclApi& a = nccl();
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  ncclResult_t r = a.all_gather(mine, gather, count, nccl_type(dtype), comm->comm, s);
  if (r == ncclInProgress) {
    st = nccl_settle(const_cast<cawq_tp_comm*>(comm), r, "ncclAllGather");
    if (st != CAWQ_OK) return st;
  } else if (r != ncclSuccess) {
    return nccl_fail(r, "ncclAllGather");
  }
  if (gather == out) return CAWQ_OK;
  cudaError_t e = launch_interleave_columns(gather, out, rows, n, comm->world, es, s);
  if (e != cudaSuccess) return cuda_fail(e, "interleave launch");
  return CAWQ_OK;
}

CAWQ_API cawq_status cawq_gemm_rowpar(const cawq_tp_comm* comm, const void* x,
                                      const uint32_t* qweight, const uint32_t* qzeros,
                                      const void* scales, const void* bias, void* out,
                                      float* partial, size_t rows, size_t k, size_t n,
                                      size_t group_size, cawq_dtype dtype, void* stream) {
  cawq_status st = tp_check(comm);
  if (st != CAWQ_OK) return st;
  if (!valid_dtype(dtype)) return fail(CAWQ_ERR_DTYPE, "dtype must be CAWQ_F32, CAWQ_F16 or CAWQ_BF16");
  size_t k0 = 0, kl = 0;
  if ((st = cawq_tp_row_shard(k, group_size, comm->world, comm->rank, &k0, &kl)) != CAWQ_OK)
    return st;
  if (rows == 0) return CAWQ_OK;
  if (!out || !partial) return fail(CAWQ_ERR_NULL_POINTER, "out and partial must be non-null");
  // (Splitting the rows in two halves, with the first half's all-reduce on a
  // side stream while the second half's GEMM runs, was measured slower on 4
  // GPUs: 499 against 470 us at M = 2048. The GEMM half is sized to fill
  // every SM, and NCCL's kernel takes some of them.)
  st = gemm_common(x, qweight, qzeros, scales, nullptr, partial, rows, kl, n, group_size, dtype,
                   CAWQ_F32, CAWQ_ORDER_AWQ, n, nullptr, stream, true);
  if (st != CAWQ_OK) return st;
  const NcclApi& a = nccl();
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  ncclResult_t r = a.all_reduce(partial, partial, rows * n, ncclFloat32, ncclSum, comm->comm, s);
  if (r == ncclInProgress) {
    st = nccl_settle(const_cast<cawq_tp_comm*>(comm), r, "ncclAllReduce");
    if (st != CAWQ_OK) return st;
  } else if (r != ncclSuccess) {
    return nccl_fail(r, "ncclAllReduce");
  }
  if (out == partial && !bias && dtype == CAWQ_F32) return CAWQ_OK;
  cudaError_t e = launch_rowpar_finish(partial, bias, out, rows, n, dtype, s);
  if (e != cudaSuccess) return cuda_fail(e, "row-parallel epilogue launch");
  return CAWQ_OK;
}

// ------------------------------------------ fused tensor-parallel push
// A cawq_tp_peers made by cawq_tp_p2p_create: the public struct first, then
// what the library needs to release it.
struct P2POwned {
  cawq_tp_peers pub;
  void* own = nullptr;
  bool opened[CAWQ_TP_MAX_PEERS] = {};
};

// An NCCL all-reduce of one float, as a barrier on the communicator's ranks.
static cawq_status tp_barrier(const cawq_tp_comm* comm, float* dev_word, cudaStream_t s) {
  ncclResult_t r = nccl().all_reduce(dev_word, dev_word, 1, ncclFloat32, ncclSum, comm->comm, s);
  if (r == ncclInProgress) {
    cawq_status st = nccl_settle(const_cast<cawq_tp_comm*>(comm), r, "ncclAllReduce");
    if (st != CAWQ_OK) return st;
  } else if (r != ncclSuccess) {
    return nccl_fail(r, "ncclAllReduce");
  }
  cudaError_t e = cudaStreamSynchronize(s);
  return e == cudaSuccess ? CAWQ_OK : cuda_fail(e, "barrier");
}

static void p2p_release(P2POwned* o) {
  for (int j = 0; j < CAWQ_TP_MAX_PEERS; ++j)
    if (o->opened[j]) cudaIpcCloseMemHandle(o->pub.base[j]);
  if (o->own) cudaFree(o->own);
  delete o;
}

CAWQ_API cawq_status cawq_tp_p2p_create(const cawq_tp_comm* comm, size_t bytes, int timeout_ms,
                                        cawq_tp_peers** peers) {
  cawq_status st = tp_check(comm);
  if (st != CAWQ_OK) return st;
  if (!peers) return fail(CAWQ_ERR_NULL_POINTER, "peers must be non-null");
  if (comm->world > CAWQ_TP_MAX_PEERS)
    return fail(CAWQ_ERR_INVALID_ARGUMENT, fmt("world %d above %d", comm->world, CAWQ_TP_MAX_PEERS));
  if (bytes < CAWQ_TP_P2P_HEADER + 512)
    return fail(CAWQ_ERR_INVALID_SHAPE, "bytes must hold the flag header and two slots");
  auto* o = new P2POwned();
  o->pub.world = comm->world;
  o->pub.rank = comm->rank;
  o->pub.bytes = bytes;
  o->pub.timeout_ms = timeout_ms;
  cudaStream_t s = nullptr;
  void* tmp = nullptr;
  auto bail = [&](cawq_status r) {
    if (tmp) cudaFree(tmp);
    if (s) cudaStreamDestroy(s);
    p2p_release(o);
    return r;
  };
  cudaError_t e = cudaMalloc(&o->own, bytes);
  if (e != cudaSuccess) { o->own = nullptr; return bail(cuda_fail(e, "cudaMalloc (peer buffer)")); }
  // zero before any peer can see the buffer: flags start below every epoch
  if ((e = cudaMemset(o->own, 0, bytes)) != cudaSuccess) return bail(cuda_fail(e, "cudaMemset"));
  if ((e = cudaDeviceSynchronize()) != cudaSuccess) return bail(cuda_fail(e, "cudaDeviceSynchronize"));
  o->pub.base[comm->rank] = o->own;
  cudaIpcMemHandle_t h;
  if ((e = cudaIpcGetMemHandle(&h, o->own)) != cudaSuccess)
    return bail(cuda_fail(e, "cudaIpcGetMemHandle"));
  const size_t hb = sizeof(cudaIpcMemHandle_t);
  if ((e = cudaStreamCreateWithFlags(&s, cudaStreamNonBlocking)) != cudaSuccess)
    return bail(cuda_fail(e, "cudaStreamCreate"));
  if ((e = cudaMalloc(&tmp, hb * comm->world + 16)) != cudaSuccess) {
    tmp = nullptr;
    return bail(cuda_fail(e, "cudaMalloc (handle exchange)"));
  }
  uint8_t* dh = static_cast<uint8_t*>(tmp);
  if ((e = cudaMemcpy(dh + comm->rank * hb, &h, hb, cudaMemcpyHostToDevice)) != cudaSuccess)
    return bail(cuda_fail(e, "cudaMemcpy"));
  ncclResult_t r = nccl().all_gather(dh + comm->rank * hb, dh, hb, ncclUint8, comm->comm, s);
  if (r == ncclInProgress) {
    if ((st = nccl_settle(const_cast<cawq_tp_comm*>(comm), r, "ncclAllGather")) != CAWQ_OK)
      return bail(st);
  } else if (r != ncclSuccess) {
    return bail(nccl_fail(r, "ncclAllGather"));
  }
  if ((e = cudaStreamSynchronize(s)) != cudaSuccess) return bail(cuda_fail(e, "handle exchange"));
  std::vector<cudaIpcMemHandle_t> all(comm->world);
  if ((e = cudaMemcpy(all.data(), dh, hb * comm->world, cudaMemcpyDeviceToHost)) != cudaSuccess)
    return bail(cuda_fail(e, "cudaMemcpy"));
  for (int j = 0; j < comm->world; ++j) {
    if (j == comm->rank) continue;
    e = cudaIpcOpenMemHandle(&o->pub.base[j], all[j], cudaIpcMemLazyEnablePeerAccess);
    if (e != cudaSuccess) return bail(cuda_fail(e, "cudaIpcOpenMemHandle"));
    o->opened[j] = true;
  }
  // every rank has mapped every buffer before any push
  float* word = reinterpret_cast<float*>(dh + hb * comm->world);
  if ((e = cudaMemsetAsync(word, 0, sizeof(float), s)) != cudaSuccess)
    return bail(cuda_fail(e, "cudaMemsetAsync"));
  if ((st = tp_barrier(comm, word, s)) != CAWQ_OK) return bail(st);
  cudaFree(tmp);
  cudaStreamDestroy(s);
  *peers = &o->pub;
  return CAWQ_OK;
}

CAWQ_API cawq_status cawq_tp_p2p_destroy(cawq_tp_peers* peers) {
  if (!peers) return CAWQ_OK;
  auto* o = reinterpret_cast<P2POwned*>(peers);
  // A rank's last fused call ended only after every peer's last push into
  // this buffer had completed (its finish step waits for all of them), so
  // once this device is idle nothing writes here any more.
  cudaError_t e = cudaDeviceSynchronize();
  if (e != cudaSuccess) return cuda_fail(e, "cudaDeviceSynchronize");
  p2p_release(o);
  return CAWQ_OK;
}

// Checks a peer table for one fused call and returns this call's slot
// offset (the slot alternates with the epoch's parity).
static cawq_status p2p_table_check(const cawq_tp_peers* peers, uint32_t epoch) {
  if (!peers) return fail(CAWQ_ERR_NULL_POINTER, "peers must be non-null");
  if (peers->world < 1 || peers->world > CAWQ_TP_MAX_PEERS || peers->rank < 0 ||
      peers->rank >= peers->world)
    return fail(CAWQ_ERR_INVALID_ARGUMENT, "peers: world must be 1..8 and rank below it");
  for (int j = 0; j < peers->world; ++j)
    if (!peers->base[j] || reinterpret_cast<uintptr_t>(peers->base[j]) % 256 != 0)
      return fail(CAWQ_ERR_ALIGNMENT, "peers: every base must be non-null and 256-byte aligned");
  if (epoch == 0) return fail(CAWQ_ERR_INVALID_ARGUMENT, "epoch must start at 1");
  return CAWQ_OK;
}

static cawq_status p2p_check(const cawq_tp_peers* peers, uint32_t epoch, size_t need,
                             size_t* slot_off) {
  cawq_status st = p2p_table_check(peers, epoch);
  if (st != CAWQ_OK) return st;
  const size_t slot = peers->bytes > CAWQ_TP_P2P_HEADER
                          ? ((peers->bytes - CAWQ_TP_P2P_HEADER) / 2) & ~static_cast<size_t>(255)
                          : 0;
  if (need > slot)
    return fail(CAWQ_ERR_INVALID_SHAPE,
                fmt("the call needs %zu bytes per slot, the peer buffers have %zu", need, slot));
  *slot_off = CAWQ_TP_P2P_HEADER + (epoch & 1u) * slot;
  return CAWQ_OK;
}

static P2PSync p2p_sync(const cawq_tp_peers* peers, uint32_t epoch) {
  P2PSync s = {};
  for (int j = 0; j < peers->world; ++j) s.flags[j] = static_cast<uint32_t*>(peers->base[j]);
  s.world = peers->world;
  s.rank = peers->rank;
  s.epoch = epoch;
  const int ms = peers->timeout_ms > 0 ? peers->timeout_ms : 2000;
  s.timeout_ns = static_cast<uint64_t>(ms) * 1000000ull;
  return s;
}

CAWQ_API cawq_status cawq_gemm_colpar_p2p(const cawq_tp_peers* peers, uint32_t epoch,
                                          const void* x, const uint32_t* qweight,
                                          const uint32_t* qzeros, const void* scales,
                                          const void* bias, void* out, size_t rows, size_t k,
                                          size_t n, size_t group_size, cawq_dtype dtype,
                                          void* stream) {
  if (dtype != CAWQ_F16 && dtype != CAWQ_BF16)
    return fail(CAWQ_ERR_DTYPE, "the fused tensor-parallel layers take CAWQ_F16 or CAWQ_BF16");
  cawq_status st = p2p_table_check(peers, epoch);
  if (st != CAWQ_OK) return st;
  size_t n0 = 0, nl = 0;
  st = cawq_tp_column_shard(n, peers->world, peers->rank, &n0, &nl);
  if (st != CAWQ_OK) return st;
  const size_t es = dtype_size(dtype);
  size_t off = 0;
  if ((st = p2p_check(peers, epoch, rows * n * es, &off)) != CAWQ_OK) return st;
  if (rows == 0) return CAWQ_OK;
  if (!out) return fail(CAWQ_ERR_NULL_POINTER, "out must be non-null");
  // Above 8 MiB of peer shards per rank the GEMM writes only this rank's
  // buffer and `out`, and a kernel after it pushes the shard into every
  // peer's buffer; below it the epilogue pushes the shard as its tiles
  // finish (the same choice on every rank, from the shapes).
  const bool large = peers->world > 1 && rows * nl * es * (size_t)(peers->world - 1) > (8u << 20) &&
                     reinterpret_cast<uintptr_t>(out) % 16 == 0;
  if (large) {
    void* rep[CAWQ_TP_MAX_PEERS] = {static_cast<uint8_t*>(out) + n0 * es};
    void* own = static_cast<uint8_t*>(peers->base[peers->rank]) + off + n0 * es;
    st = gemm_common(x, qweight, qzeros, scales, bias, own, rows, k, nl, group_size, dtype, dtype,
                     CAWQ_ORDER_AWQ, n, nullptr, stream, true, 0, nullptr, rep, 1);
    if (st != CAWQ_OK) return st;
    cudaError_t e = launch_p2p_colpar_push(p2p_sync(peers, epoch), off, out, rows, n, dtype,
                                           static_cast<cudaStream_t>(stream));
    if (e != cudaSuccess) return cuda_fail(e, "gather launch");
    return CAWQ_OK;
  }
  // this rank's columns of the gathered [rows, n] result, in every buffer
  void* dst[CAWQ_TP_MAX_PEERS];
  int nrep = 0;
  for (int j = 0; j < peers->world; ++j) {
    void* d = static_cast<uint8_t*>(peers->base[j]) + off + n0 * es;
    if (j == peers->rank) dst[CAWQ_TP_MAX_PEERS - 1] = d;
    else dst[nrep++] = d;
  }
  st = gemm_common(x, qweight, qzeros, scales, bias, dst[CAWQ_TP_MAX_PEERS - 1], rows, k, nl,
                   group_size, dtype, dtype, CAWQ_ORDER_AWQ, n, nullptr, stream, true, 0, nullptr,
                   dst, nrep);
  if (st != CAWQ_OK) return st;
  const void* slot = static_cast<uint8_t*>(peers->base[peers->rank]) + off;
  cudaError_t e = launch_p2p_colpar_finish(p2p_sync(peers, epoch), slot, out, rows, n, n, dtype,
                                           static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "gather launch");
  return CAWQ_OK;
}

CAWQ_API cawq_status cawq_gemm_rowpar_p2p(const cawq_tp_peers* peers, uint32_t epoch,
                                          const void* x, const uint32_t* qweight,
                                          const uint32_t* qzeros, const void* scales,
                                          const void* bias, void* out, size_t rows, size_t k,
                                          size_t n, size_t group_size, cawq_dtype dtype,
                                          void* stream) {
  if (dtype != CAWQ_F16 && dtype != CAWQ_BF16)
    return fail(CAWQ_ERR_DTYPE, "the fused tensor-parallel layers take CAWQ_F16 or CAWQ_BF16");
  cawq_status st = p2p_table_check(peers, epoch);
  if (st != CAWQ_OK) return st;
  size_t k0 = 0, kl = 0;
  st = cawq_tp_row_shard(k, group_size, peers->world, peers->rank, &k0, &kl);
  if (st != CAWQ_OK) return st;
  if (n % 32 != 0) return fail(CAWQ_ERR_INVALID_SHAPE, "n must be a multiple of 32");
  size_t off = 0;
  const size_t plane = rows * n * sizeof(float);
  const int world = peers->world;
  // Reduce-scatter + all-gather once the one-shot push would send more than
  // 4 MiB per rank (each rank then sends (world-1)/world of a partial plane
  // and of the result, instead of world-1 whole planes); the same choice on
  // every rank, from the shapes alone.
  const bool rs = world > 1 && n % (32 * (size_t)world) == 0 &&
                  plane * (size_t)(world - 1) > (4u << 20);
  if (rs) {
    const size_t es = dtype == CAWQ_F32 ? 4 : 2;
    const size_t pl = (plane + 255) / 256 * 256;  // partial, receive region, gather region
    if ((st = p2p_check(peers, epoch, 2 * pl + rows * n * es, &off)) != CAWQ_OK) return st;
    if (rows == 0) return CAWQ_OK;
    if (!out) return fail(CAWQ_ERR_NULL_POINTER, "out must be non-null");
    if (reinterpret_cast<uintptr_t>(out) % 16 != 0)
      return fail(CAWQ_ERR_ALIGNMENT, "out must be 16-byte aligned");
    // this rank's fp32 partial [rows, n] into its own buffer
    void* own = static_cast<uint8_t*>(peers->base[peers->rank]) + off;
    st = gemm_common(x, qweight, qzeros, scales, nullptr, own, rows, kl, n, group_size, dtype,
                     CAWQ_F32, CAWQ_ORDER_AWQ, n, nullptr, stream, true);
    if (st != CAWQ_OK) return st;
    P2PSync sa = p2p_sync(peers, epoch), sb = p2p_sync(peers, epoch);
    sb.fofs = 8;  // the gather's own flag words
    cudaError_t e = launch_p2p_rowpar_rs(sa, sb, off, off + pl, off + 2 * pl, bias, out, rows, n,
                                         dtype, static_cast<cudaStream_t>(stream));
    if (e != cudaSuccess) return cuda_fail(e, "reduce-scatter launch");
    return CAWQ_OK;
  }
  if ((st = p2p_check(peers, epoch, plane * peers->world, &off)) != CAWQ_OK) return st;
  if (rows == 0) return CAWQ_OK;
  if (!out) return fail(CAWQ_ERR_NULL_POINTER, "out must be non-null");
  // this rank's fp32 partial into plane [rank] of every buffer's slot
  void* dst[CAWQ_TP_MAX_PEERS];
  int nrep = 0;
  for (int j = 0; j < peers->world; ++j) {
    void* d = static_cast<uint8_t*>(peers->base[j]) + off + peers->rank * plane;
    if (j == peers->rank) dst[CAWQ_TP_MAX_PEERS - 1] = d;
    else dst[nrep++] = d;
  }
  st = gemm_common(x, qweight, qzeros, scales, nullptr, dst[CAWQ_TP_MAX_PEERS - 1], rows, kl, n,
                   group_size, dtype, CAWQ_F32, CAWQ_ORDER_AWQ, n, nullptr, stream, true, 0,
                   nullptr, dst, nrep);
  if (st != CAWQ_OK) return st;
  const float* slot = reinterpret_cast<const float*>(
      static_cast<uint8_t*>(peers->base[peers->rank]) + off);
  cudaError_t e = launch_p2p_rowpar_finish(p2p_sync(peers, epoch), slot, bias, out, rows, n, dtype,
                                           static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "reduce launch");
  return CAWQ_OK;
}

CAWQ_API cawq_status cawq_gemm_rowpar_noalloc(const cawq_tp_comm* comm, const void* x,
                                              const uint32_t* qweight, const uint32_t* qzeros,
                                              const void* scales, const void* bias, void* out,
                                              size_t rows, size_t k, size_t n, size_t group_size,
                                              cawq_dtype dtype, void* stream) {
  // Divide rather than multiply: rows * n can wrap around for absurd sizes.
  if (n != 0 && rows > CAWQ_ROWPAR_SCRATCH_FLOATS / n) {
    return fail(CAWQ_ERR_INVALID_SHAPE,
                fmt("rows * n = %zu exceeds the static scratch of %u floats "
                    "(CAWQ_ROWPAR_SCRATCH_FLOATS); use cawq_gemm_rowpar with a workspace",
                    rows * n, (unsigned)CAWQ_ROWPAR_SCRATCH_FLOATS));
  }
  cawq_status st = tp_check(comm);
  if (st != CAWQ_OK) return st;
  if (!valid_dtype(dtype)) return fail(CAWQ_ERR_DTYPE, "dtype must be CAWQ_F32, CAWQ_F16 or CAWQ_BF16");
  size_t k0 = 0, kl = 0;
  if ((st = cawq_tp_row_shard(k, group_size, comm->world, comm->rank, &k0, &kl)) != CAWQ_OK)
    return st;
  if (rows == 0) return CAWQ_OK;
  if (!out) return fail(CAWQ_ERR_NULL_POINTER, "out must be non-null");
  float* partial = nullptr;
  cudaError_t e = rowpar_static_scratch(&partial);
  if (e != cudaSuccess) return cuda_fail(e, "cudaGetSymbolAddress (row-parallel scratch)");
  st = gemm_common(x, qweight, qzeros, scales, nullptr, partial, rows, kl, n, group_size, dtype,
                   CAWQ_F32, CAWQ_ORDER_AWQ, n, nullptr, stream, true);
  if (st != CAWQ_OK) return st;
  const NcclApi& a = nccl();
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  ncclResult_t r = a.all_reduce(partial, partial, rows * n, ncclFloat32, ncclSum, comm->comm, s);
  if (r == ncclInProgress) {
    st = nccl_settle(const_cast<cawq_tp_comm*>(comm), r, "ncclAllReduce");
    if (st != CAWQ_OK) return st;
  } else if (r != ncclSuccess) {
    return nccl_fail(r, "ncclAllReduce");
  }
  e = launch_rowpar_finish(partial, bias, out, rows, n, dtype, s);
  if (e != cudaSuccess) return cuda_fail(e, "row-parallel epilogue launch");
  return CAWQ_OK;
}

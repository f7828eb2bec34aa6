/*
 * cube_awq.h — C ABI of libcube_awq.so, the B200 (sm_100a) implementation of
 * the AWQ INT4 hot path of joshuawm/cube-awq:
 *
 *   - the fused INT4 dequant-GEMM  Y[M,N] = X[M,K] · ((Q - Z) · S)[K,N]
 *     (reference: src/kernel/awq_kernel_gemm.rs `gemm_awq` / `gemm_awq_decode`),
 *   - the standalone dequantize kernel
 *     (reference: src/kernel/awq_kernel.rs `dequantize_awq_symmetric`).
 *
 * Tensor format (AutoAWQ, exactly as the reference reads it):
 *   qweight u32 [K, N/8], qzeros u32 [K/g, N/8], scales F [K/g, N], bias F [N].
 *   Logical column c of a packed u32 is stored in nibble
 *     CAWQ_ORDER_AWQ:     [0,4,1,5,2,6,3,7][c % 8]   (GEMM, awq_kernel_gemm.rs:10-30)
 *     CAWQ_ORDER_NATURAL: c % 8                      (dequantize, awq_kernel.rs:9-19)
 *   Dequantized value = (float(q) - float(z)) * s, computed in F.
 *
 * Conventions of every entry point:
 *   - All tensors are caller-allocated device memory, row-major and dense.
 *   - `stream` is a cudaStream_t (NULL = legacy default stream). Launches are
 *     asynchronous; the calls never synchronise the device.
 *   - Nothing here aborts the process: failures return a cawq_status and the
 *     calling thread's cawq_last_error() holds a message. Shape-rule messages
 *     are the reference's assert! texts verbatim.
 *   - The GPU entry points need an sm_100 device; on anything else they return
 *     CAWQ_ERR_UNSUPPORTED. There is no CPU fallback.
 */
#ifndef CUBE_AWQ_H_
#define CUBE_AWQ_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define CAWQ_VERSION_MAJOR 0
#define CAWQ_VERSION_MINOR 1
#define CAWQ_MAX_RANK 8

typedef enum cawq_status {
  CAWQ_OK = 0,
  CAWQ_ERR_INVALID_SHAPE = 1, /* a shape rule of the reference failed        */
  CAWQ_ERR_DTYPE = 2,         /* unsupported dtype or packed element size    */
  CAWQ_ERR_ALIGNMENT = 3,     /* pointer alignment the call needs is missing */
  CAWQ_ERR_CUDA = 4,          /* CUDA runtime/driver error                   */
  CAWQ_ERR_NCCL = 5,          /* collective failure (tensor-parallel layer)  */
  CAWQ_ERR_TIMEOUT = 6,       /* a bounded device-side wait gave up          */
  CAWQ_ERR_UNSUPPORTED = 7,   /* valid request, but no sm_100 device         */
  CAWQ_ERR_NULL_POINTER = 8,  /* a required pointer argument was NULL        */
  CAWQ_ERR_INVALID_ARGUMENT = 9
} cawq_status;

/* F of the reference: activations, scales, bias, dequantized weights. */
typedef enum cawq_dtype { CAWQ_F32 = 0, CAWQ_F16 = 1, CAWQ_BF16 = 2 } cawq_dtype;

typedef enum cawq_order { CAWQ_ORDER_AWQ = 0, CAWQ_ORDER_NATURAL = 1 } cawq_order;

/* Kernel families the planner can choose (cawq_plan.path). */
typedef enum cawq_path {
  CAWQ_PATH_AUTO = 0,
  CAWQ_PATH_DECODE = 1,  /* memory-bound small-M kernel (M <= 16)          */
  CAWQ_PATH_PREFILL = 2, /* tcgen05/TMEM tensor-core kernel (large M)      */
  CAWQ_PATH_GENERIC = 3  /* CUDA-core kernel for any shape the rules allow */
} cawq_path;

/*
 * Mirror of the reference's ShapeConfig (awq_kernel_gemm.rs:35-79). The
 * tile fields are the reference's launch tiles; they take part in validation
 * exactly as in the reference. The B200 kernels choose their own tiles
 * (cawq_plan), so the fields do not change the arithmetic.
 */
typedef struct cawq_shape_config {
  size_t m, k, n;
  size_t tile_m;    /* 8 | 16 | 32 in the reference   */
  size_t tile_n;    /* 32 | 64 | 128                  */
  size_t inner_k;   /* 32 | 64                        */
  size_t line_size; /* 4                              */
  size_t m_valid;
} cawq_shape_config;

/* A device buffer with its row-major shape (mirrors TensorHandleRef). */
typedef struct cawq_tensor_desc {
  const void* data;
  int rank;
  size_t shape[CAWQ_MAX_RANK];
  size_t elem_size; /* bytes per element */
} cawq_tensor_desc;

/* Arguments of cawq_awq_gemm_linear. */
typedef struct cawq_gemm_args {
  cawq_tensor_desc input;   /* [.., M, K]  F                           */
  cawq_tensor_desc qweight; /* [K, N/8]    32-bit                      */
  cawq_tensor_desc qzeros;  /* [K/g, N/8]  32-bit                      */
  cawq_tensor_desc scales;  /* [K/g, N]    F                           */
  cawq_tensor_desc bias;    /* [N] F, or data == NULL for no bias      */
  cawq_tensor_desc output;  /* [.., M, N]  F (written)                 */
  cawq_dtype dtype;         /* F                                       */
  size_t group_size;
} cawq_gemm_args;

/* A kernel choice for one (M, K, N, g, dtype) problem. */
typedef struct cawq_plan {
  int path;      /* cawq_path                                            */
  int split;     /* decode: CTAs per cluster splitting K (1..16);
                    prefill: 1, 2, 4, 8                                  */
  int warps;     /* decode: 128-column strips per CTA (even, 2..8);
                    prefill: 1 / 2 = 128 / 256-row X tiles; 4 = the
                    weights as the MMA's A operand in tensor memory,
                    X rows as its N (rows <= 128, f16 / bf16,
                    group_size % 64 == 0; autotune candidate only)      */
  int tile_n;    /* prefill: CTA tile N (warps 4: 256, or 512 for rows
                    <= 64); decode: 0                                    */
  int stages;    /* pipeline stages (prefill warps 4: packed weight
                    stages in flight, 0 = 6)                            */
  int reserved[3]; /* reserved[0] = 1: launch without programmatic
                      dependent launch (no overlap with the previous
                      kernel of the stream).
                      reserved[1] (decode): weight stages past the ring
                      to prefetch into L2 before waiting for the
                      previous kernel (0 = none).
                      reserved[2] (decode): 0 = f16 / bf16 tensor
                      path; 1 = integer tensor path where it applies
                      (rows <= 4, f16 / bf16 X, group_size % 64 == 0:
                      X as exact 16-bit fixed point, int8 MMA)      */
} cawq_plan;

/* ----------------------------------------------------------------------- */
/* Library and device                                                      */
/* ----------------------------------------------------------------------- */

/* Message of the last failed call on this thread ("" if none). */
const char* cawq_last_error(void);

/* Version string, e.g. "cube_awq 0.1 sm_100a". */
const char* cawq_version(void);

/* 1 if `device` is an sm_100 GPU this library has code for, else 0. */
int cawq_device_supported(int device);

/*
 * Reads (and with reset != 0 clears) the device-side error word of the
 * current device: bit 0 = a bounded wait inside a kernel timed out; bit 1 =
 * a fused tensor-parallel call gave up waiting for a peer's flag.
 * Synchronises the device.
 */
cawq_status cawq_device_error(int reset, uint32_t* word);

/* ----------------------------------------------------------------------- */
/* Shape rules (host only; no GPU needed)                                  */
/* ----------------------------------------------------------------------- */

/* Replaces ShapeConfig::new (awq_kernel_gemm.rs:48-57); note the m, n, k order. */
cawq_status cawq_shape_config_new(size_t m, size_t n, size_t k, size_t tile_m,
                                  size_t tile_n, size_t inner_k,
                                  cawq_shape_config* out);

/* Replaces ShapeConfig::new_with_valid_m (awq_kernel_gemm.rs:59-78). */
cawq_status cawq_shape_config_new_with_valid_m(size_t m, size_t n, size_t k,
                                               size_t tile_m, size_t tile_n,
                                               size_t inner_k, size_t m_valid,
                                               cawq_shape_config* out);

/* Replaces validate_launch_params (awq_kernel_gemm.rs:160-162). */
cawq_status cawq_validate_launch_params(const cawq_shape_config* shape,
                                        size_t group_size);

/* Replaces validate_decode_launch_params (awq_kernel_gemm.rs:164-171). */
cawq_status cawq_validate_decode_launch_params(const cawq_shape_config* shape,
                                               size_t group_size);

/* Replaces select_tile_m / select_tile_n (awq_gemm.rs:30-52), including the
 * AWQ_GEMM_FORCE_TILE_M override (awq_gemm.rs:20-28). */
size_t cawq_select_tile_m(size_t m);
size_t cawq_select_tile_n(size_t n);

/* ----------------------------------------------------------------------- */
/* Fused AWQ GEMM                                                          */
/* ----------------------------------------------------------------------- */

/*
 * Replaces awq_gemm_linear<R, F> (awq_kernel_gemm.rs:626-771): the same
 * rank/shape asserts with the same messages, the same m_valid resolution
 * (:675-681) and decode/prefill rule validation (:691-696), then one fused
 * launch. `shape` may be NULL: the module's tile choice (awq_gemm.rs:205-207)
 * is then used for validation. Bias, when present, is added in the epilogue
 * after the full K reduction (awq_gemm.rs:225-228).
 */
cawq_status cawq_awq_gemm_linear(const cawq_gemm_args* args,
                                 const cawq_shape_config* shape, void* stream);

/*
 * Hot-path form of the same GEMM with plain pointers, the call that
 * AWQGEMMLinear::forward (awq_gemm.rs:146-232) makes after flattening:
 *   out[rows, N] = x[rows, K] · deq(qweight, qzeros, scales) (+ bias)
 * x, scales and bias are `dtype`; out is `out_dtype` (dtype, or CAWQ_F32 for
 * the fp32 partial sums of a row-parallel shard). `order` selects the nibble
 * order (CAWQ_ORDER_AWQ as gemm_awq; CAWQ_ORDER_NATURAL gives the fused form
 * of AWQLinear::forward, awq_dequantize.rs:74-108). `ld_out` is the row
 * stride of out in elements (0 = N), so a column shard can write into its
 * slice of a wider output. The rules of the module that owns each order
 * apply: CAWQ_ORDER_AWQ follows AWQGEMMLinear (awq_gemm.rs:77-95 plus the
 * kernel rules of awq_kernel_gemm.rs:89-158 with the module's tiles);
 * CAWQ_ORDER_NATURAL follows AWQLinear (awq_dequantize.rs:25-28).
 */
cawq_status cawq_gemm(const void* x, const uint32_t* qweight,
                      const uint32_t* qzeros, const void* scales,
                      const void* bias, void* out, size_t rows, size_t k,
                      size_t n, size_t group_size, cawq_dtype dtype,
                      cawq_dtype out_dtype, cawq_order order, size_t ld_out,
                      void* stream);

/*
 * Same as cawq_gemm with an explicit plan (path / split / tiles); used by the
 * autotuner and by tests that pin a kernel. Returns CAWQ_ERR_INVALID_ARGUMENT
 * if the plan cannot run this problem.
 */
cawq_status cawq_gemm_with_plan(const void* x, const uint32_t* qweight,
                                const uint32_t* qzeros, const void* scales,
                                const void* bias, void* out, size_t rows,
                                size_t k, size_t n, size_t group_size,
                                cawq_dtype dtype, cawq_dtype out_dtype,
                                cawq_order order, size_t ld_out,
                                const cawq_plan* plan, void* stream);

/*
 * gate_up with its SiLU gate fused into the epilogue (the next step of a
 * SwiGLU MLP): out[rows, n / 2] = silu(x · W_gate + b_gate) * (x · W_up + b_up),
 * computed from the fp32 sums and rounded once to `dtype`. No counterpart
 * kernel in the reference (its decoder runs the GEMM, then the activation).
 * The weights are the gate and up projections with their columns interleaved
 * in 128-column blocks — W columns [256 j, 256 j + 128) are gate columns
 * [128 j, 128 j + 128), the next 128 the matching up columns — so n (= 2 x
 * the MLP width) must be a multiple of 256; qweight / qzeros / scales / bias
 * follow the same column order (cawq_interleave_gate_up builds it from the
 * plain [gate | up] layout). dtype CAWQ_F16 or CAWQ_BF16; ld_out >= n / 2
 * (0 = n / 2). Output column c of row r sits at out[r * ld_out + c].
 */
cawq_status cawq_gemm_silu_mul(const void* x, const uint32_t* qweight,
                               const uint32_t* qzeros, const void* scales,
                               const void* bias, void* out, size_t rows, size_t k,
                               size_t n, size_t group_size, cawq_dtype dtype,
                               size_t ld_out, void* stream);

/* The same with an explicit plan (decode or prefill path). */
cawq_status cawq_gemm_silu_mul_with_plan(const void* x, const uint32_t* qweight,
                                         const uint32_t* qzeros, const void* scales,
                                         const void* bias, void* out, size_t rows,
                                         size_t k, size_t n, size_t group_size,
                                         cawq_dtype dtype, size_t ld_out,
                                         const cawq_plan* plan, void* stream);

/*
 * Reorders the columns of a [gate | up] projection (`width` columns each,
 * width % 128 == 0) into the block-interleaved layout cawq_gemm_silu_mul
 * reads: `rows` rows of `elem_size`-byte elements (4 for packed qweight /
 * qzeros rows with width / 8 words per half, 2 or 4 for scales / bias), row
 * pitch `2 * width_elems * elem_size` bytes in both buffers, where
 * width_elems is the half's element count (width for scales and bias,
 * width / 8 for packed rows). src and dst must not overlap.
 */
cawq_status cawq_interleave_gate_up(const void* src, void* dst, size_t rows, size_t width_elems,
                                    size_t block_elems, size_t elem_size, void* stream);

/*
 * Fused qkv projection with a split epilogue (no counterpart kernel in the
 * reference, which runs q_proj, k_proj and v_proj as three AWQGEMMLinear
 * forwards, src/modules/awq_gemm.rs:146-232). One cawq_gemm over the
 * concatenated [q | k | v] weights (AutoAWQ layout, n = n_q + 2 * n_kv
 * columns; bias likewise concatenated or NULL) whose epilogue writes columns
 * [0, n_q) to q_out (row stride ld_q), [n_q, n_q + n_kv) to k_out (ld_k) and
 * the rest to v_out (ld_v): each output can be a slice of a larger buffer,
 * such as a key / value cache row. n_q and n_kv: positive multiples of 32;
 * a stride of 0 means the output's width. Same rules, plans and dtypes as
 * cawq_gemm with CAWQ_ORDER_AWQ; every output element is the value cawq_gemm
 * writes for that column.
 */
cawq_status cawq_gemm_qkv(const void* x, const uint32_t* qweight, const uint32_t* qzeros,
                          const void* scales, const void* bias, void* q_out, void* k_out,
                          void* v_out, size_t rows, size_t k, size_t n_q, size_t n_kv,
                          size_t group_size, cawq_dtype dtype, cawq_dtype out_dtype,
                          size_t ld_q, size_t ld_k, size_t ld_v, void* stream);

/* ----------------------------------------------------------------------- */
/* Planner / autotuner                                                     */
/* ----------------------------------------------------------------------- */

/* The plan cawq_gemm would use now (cache hit, else the static heuristic). */
cawq_status cawq_plan_get(size_t rows, size_t k, size_t n, size_t group_size,
                          cawq_dtype dtype, cawq_plan* plan);

/* Pins a plan for this problem in the process-wide cache. */
cawq_status cawq_plan_set(size_t rows, size_t k, size_t n, size_t group_size,
                          cawq_dtype dtype, const cawq_plan* plan);

/* Clears the process-wide plan cache. */
void cawq_plan_cache_clear(void);

/*
 * Times every candidate plan for this problem on `stream` with the given
 * device buffers (they are read, and `out` is overwritten), stores the
 * fastest in the cache and returns it. Synchronises the stream.
 */
cawq_status cawq_autotune(const void* x, const uint32_t* qweight,
                          const uint32_t* qzeros, const void* scales,
                          void* out, size_t rows, size_t k, size_t n,
                          size_t group_size, cawq_dtype dtype,
                          cawq_plan* best, void* stream);

/* ----------------------------------------------------------------------- */
/* Standalone dequantize                                                   */
/* ----------------------------------------------------------------------- */

/*
 * Replaces dequantize_native<R, E> (awq_kernel.rs:63-111) and its caller
 * dequantize_awq (kernel/mod.rs:9-51): out[K, N] = (q - z) * s in `dtype`,
 * natural nibble order as the reference kernel reads it (CAWQ_ORDER_AWQ is an
 * extension). The element-size asserts of awq_kernel.rs:73-84 and the
 * out_width % 32 assert of :87 are reproduced with the same messages.
 */
cawq_status cawq_dequantize_native(const cawq_tensor_desc* qweight,
                                   const cawq_tensor_desc* qzeros,
                                   const cawq_tensor_desc* scales,
                                   const cawq_tensor_desc* output,
                                   size_t group_size, cawq_dtype dtype,
                                   cawq_order order, void* stream);

/* Plain-pointer form: out[k, n] from qweight[k, n/8], qzeros[k/g, n/8],
 * scales[k/g, n]. */
cawq_status cawq_dequantize(const uint32_t* qweight, const uint32_t* qzeros,
                            const void* scales, void* out, size_t k, size_t n,
                            size_t group_size, cawq_dtype dtype,
                            cawq_order order, void* stream);

/* ----------------------------------------------------------------------- */
/* Tensor-parallel helpers (no reference counterpart: the reference is     */
/* single-device; these give the shard arithmetic of the sharded layers)   */
/* ----------------------------------------------------------------------- */

/*
 * Column-parallel (N split): rank `rank` of `world` owns output columns
 * [*n_begin, *n_begin + *n_len). Requires N % (32 * world) == 0.
 */
cawq_status cawq_tp_column_shard(size_t n, int world, int rank,
                                 size_t* n_begin, size_t* n_len);

/*
 * Row-parallel (K split on group boundaries): rank owns K rows
 * [*k_begin, *k_begin + *k_len). Requires (K / g) % world == 0.
 */
cawq_status cawq_tp_row_shard(size_t k, size_t group_size, int world, int rank,
                              size_t* k_begin, size_t* k_len);

/*
 * Gathers `world` column shards stored rank-major as src[world][rows][n/world]
 * into dst[rows][n] (the layout an all-gather of [rows, n/world] slices
 * produces, turned back into row-major). Element size from dtype.
 */
cawq_status cawq_tp_interleave_columns(const void* src, void* dst, size_t rows,
                                       size_t n, int world, cawq_dtype dtype,
                                       void* stream);

/* ----------------------------------------------------------------------- */
/* Tensor-parallel layers over NCCL (no reference counterpart)              */
/* ----------------------------------------------------------------------- */

/* Size of the NCCL unique id every rank passes to cawq_tp_init. */
#define CAWQ_TP_ID_BYTES 128

/* A communicator over `world` GPUs, one per rank (opaque). */
typedef struct cawq_tp_comm cawq_tp_comm;

/*
 * Rank 0 creates the id and hands its CAWQ_TP_ID_BYTES bytes to every rank
 * (any out-of-band channel). NCCL (libnccl.so.2) is loaded on first use; the
 * library has no link-time dependency on it.
 */
cawq_status cawq_tp_unique_id(uint8_t* id);

/*
 * Joins the communicator on the current CUDA device. Returns
 * CAWQ_ERR_TIMEOUT (and releases everything) if the other ranks have not
 * joined within `timeout_ms` milliseconds (<= 0: 60 s).
 */
cawq_status cawq_tp_init(int world, int rank, const uint8_t* id, int timeout_ms,
                         cawq_tp_comm** comm);

/* Releases the communicator (after all work on it has finished). */
cawq_status cawq_tp_destroy(cawq_tp_comm* comm);

/* World size / rank of a communicator. */
cawq_status cawq_tp_info(const cawq_tp_comm* comm, int* world, int* rank);

/*
 * Column-parallel layer (gate_up, qkv): this rank holds output columns
 * [rank * N/world, (rank + 1) * N/world) — qweight [K, N/(8 world)],
 * qzeros [K/g, N/(8 world)], scales [K/g, N/world], bias [N/world] or NULL,
 * as cawq_tp_column_shard cuts them. x [rows, K] is replicated. Computes the
 * local [rows, N/world] slice, all-gathers the slices over NCCL and writes
 * the full out [rows, N]. `gather` is caller workspace of rows * N elements
 * of `dtype`; it may be NULL when rows == 1 (the gather then runs in place
 * in `out`). Everything is enqueued on `stream`.
 */
cawq_status cawq_gemm_colpar(const cawq_tp_comm* comm, const void* x, const uint32_t* qweight,
                             const uint32_t* qzeros, const void* scales, const void* bias,
                             void* out, void* gather, size_t rows, size_t k, size_t n,
                             size_t group_size, cawq_dtype dtype, void* stream);

/*
 * Row-parallel layer (down, o): this rank holds K rows
 * [rank * K/world, (rank + 1) * K/world) on group boundaries — qweight
 * [K/world, N/8], qzeros [K/(g world), N/8], scales [K/(g world), N], as
 * cawq_tp_row_shard cuts them — and x [rows, K/world], its columns of the
 * input. Computes the fp32 partial [rows, N] into `partial` (caller
 * workspace, rows * N floats), all-reduces it (sum, fp32) over NCCL, then
 * writes out [rows, N] = partial + bias (bias [N] or NULL, added once).
 * With dtype CAWQ_F32, out may be `partial` itself.
 */
cawq_status cawq_gemm_rowpar(const cawq_tp_comm* comm, const void* x, const uint32_t* qweight,
                             const uint32_t* qzeros, const void* scales, const void* bias,
                             void* out, float* partial, size_t rows, size_t k, size_t n,
                             size_t group_size, cawq_dtype dtype, void* stream);

/*
 * cawq_gemm_rowpar for callers that have no fp32 workspace to pass and may
 * not allocate one. No counterpart in the reference (which is single-device).
 *
 * Who needs it: a host that gives its whole device memory to its own pool at
 * start-up (a serving engine sizing its KV cache, a framework's caching
 * allocator) has nothing left for a cudaMalloc in the middle of a step, and a
 * cudaMalloc / cudaFree there could also stall its other streams; a non-Python
 * host binding this C ABI (the reference's Rust side) holds the layer's
 * tensors and its output but no allocator for a rows * n fp32 buffer.
 *
 * The partial sums go to a scratch array compiled into the library's device
 * image instead, CAWQ_ROWPAR_SCRATCH_FLOATS floats (4 MiB) on each device:
 *   - rows * n above CAWQ_ROWPAR_SCRATCH_FLOATS is refused with
 *     CAWQ_ERR_INVALID_SHAPE (use cawq_gemm_rowpar with a workspace instead);
 *   - the first call on a device looks the array's device address up once
 *     (cudaGetSymbolAddress, on the current device) and keeps it for the
 *     life of the process; make that first call before any stream capture.
 *     Resetting the device (cudaDeviceReset) while the library is loaded is
 *     not supported with this entry point: the kept address would be stale;
 *   - this library allocates nothing in the call, on the device or through
 *     any allocating library routine; NCCL's own connection buffers are
 *     NCCL's, and with its default lazy connection a communicator may set
 *     them up at its first collectives: a caller that must see none at all
 *     makes one call of each size it will use beforehand, or runs with
 *     NCCL_RUNTIME_CONNECT=0 so that cawq_tp_init connects everything;
 *   - nothing in the array has to start at zero: the local GEMM writes all
 *     rows * n partial sums before the all-reduce reads them, so the last
 *     call's contents never leak into the next;
 *   - every call on a device shares the one array: calls that overlap on the
 *     GPU (on other streams, say) race on it and give wrong sums; the caller
 *     orders them.
 * Other arguments and results are those of cawq_gemm_rowpar.
 */
#define CAWQ_ROWPAR_SCRATCH_FLOATS (1u << 20)
cawq_status cawq_gemm_rowpar_noalloc(const cawq_tp_comm* comm, const void* x,
                                     const uint32_t* qweight, const uint32_t* qzeros,
                                     const void* scales, const void* bias, void* out,
                                     size_t rows, size_t k, size_t n, size_t group_size,
                                     cawq_dtype dtype, void* stream);

/* ----------------------------------------------------------------------- */
/* Fused tensor-parallel layers: the collective in the GEMM's epilogue      */
/* (no reference counterpart; the reference is single-device)               */
/* ----------------------------------------------------------------------- */
/*
 * Instead of a GEMM followed by an NCCL collective, the GEMM's epilogue
 * stores its output straight into every rank's peer buffer over NVLink
 * (plain stores through peer mappings, as each output tile is finished),
 * then a small kernel publishes a flag to every peer, waits (bounded) for
 * theirs, and finishes the collective from its own buffer.
 *
 * Peer buffers: one per rank, the same size everywhere, each mapped into
 * every rank's process. A buffer holds CAWQ_TP_P2P_HEADER bytes of flag
 * words (zero before the first call), then two slots of
 * ((bytes - CAWQ_TP_P2P_HEADER) / 2) rounded down to 256 bytes; a call uses
 * slot (epoch & 1), so the slot a peer writes is never the one this rank is
 * still reading. That holds when each rank's fused calls on one table run in
 * order on the GPU (one stream, or streams the caller orders), and only while
 * every wait has succeeded: once a finish kernel's wait has timed out (bit 1
 * of cawq_device_error's word), a peer may already be writing the slot of a
 * later epoch that this rank still reads, so the table is unusable. Every
 * rank then destroys it and the ranks create a new one.
 */
#define CAWQ_TP_MAX_PEERS 8
#define CAWQ_TP_P2P_HEADER 256
typedef struct cawq_tp_peers {
  int world;                     /* ranks, 1..CAWQ_TP_MAX_PEERS              */
  int rank;                      /* this rank                                */
  void* base[CAWQ_TP_MAX_PEERS]; /* every rank's buffer in this process's
                                    address space (base[rank]: its own);
                                    256-byte aligned                        */
  size_t bytes;                  /* size of each buffer                      */
  int timeout_ms;                /* bound of the wait for peers (<= 0: 2 s);
                                    on timeout bit 1 of cawq_device_error's
                                    word is set and the output is not
                                    written                                 */
} cawq_tp_peers;

/*
 * Collective over the communicator's ranks: allocates this rank's buffer of
 * `bytes` on the current device (once, at set-up), zeroes it, exchanges
 * CUDA IPC handles over NCCL and maps every peer's buffer. The table is
 * owned by the library; release it with cawq_tp_p2p_destroy. Callers that
 * map buffers their own way (any symmetric-memory allocator) fill a
 * cawq_tp_peers themselves instead.
 */
cawq_status cawq_tp_p2p_create(const cawq_tp_comm* comm, size_t bytes, int timeout_ms,
                               cawq_tp_peers** peers);
/* Unmaps and frees a table made by cawq_tp_p2p_create, once every rank's
   last fused call has completed (synchronises this device). */
cawq_status cawq_tp_p2p_destroy(cawq_tp_peers* peers);

/*
 * Column-parallel layer with the all-gather over peer memory: the same
 * shards and result as cawq_gemm_colpar (out [rows, n] in full on every
 * rank), f16 / bf16. Two exchanges, chosen from the shapes alone (the same
 * on every rank):
 *   - push (up to 8 MiB of peer shards per rank, or `out` not 16-byte
 *     aligned): the local GEMM's epilogue writes its [rows, n/world] columns
 *     into the slot of every rank's buffer as its tiles finish; after the
 *     flag exchange each rank copies its gathered slot to `out`;
 *   - after the GEMM (larger): the local GEMM writes its columns into its
 *     own slot and into `out`; a kernel then copies them into every other
 *     rank's slot; after the flag exchange each rank copies the other ranks'
 *     columns from its own slot into `out`.
 * Needs rows * n * sizeof(F) bytes per slot. Every rank makes the same fused
 * calls in the same order, each with the next `epoch` of this peer table
 * (1, 2, 3, ...: one counter per table, shared by all layers that use it).
 */
cawq_status cawq_gemm_colpar_p2p(const cawq_tp_peers* peers, uint32_t epoch, const void* x,
                                 const uint32_t* qweight, const uint32_t* qzeros,
                                 const void* scales, const void* bias, void* out, size_t rows,
                                 size_t k, size_t n, size_t group_size, cawq_dtype dtype,
                                 void* stream);
/*
 * Row-parallel layer with the all-reduce over peer memory: the same shards
 * and result as cawq_gemm_rowpar, f16 / bf16. Two exchanges, chosen from the
 * shapes alone (the same on every rank):
 *   - one-shot (when (world - 1) * rows * n * 4 bytes is at most 4 MiB, or
 *     n is not a multiple of 32 * world): the local GEMM's epilogue writes
 *     its fp32 partial [rows, n] into plane [rank] of the slot of every
 *     rank's buffer; each rank then sums the world planes in rank order,
 *     adds the bias once and casts. Needs world * rows * n * 4 bytes per
 *     slot;
 *   - reduce-scatter + all-gather (larger; `out` must be 16-byte aligned):
 *     the local GEMM writes its fp32 partial [rows, n] into its own slot; a
 *     kernel copies column chunk o (n / world columns) of it into rank o's
 *     receive region, for every o != rank; after the flag exchange rank o
 *     sums its chunk over the world partials in rank order, adds the bias,
 *     casts, and writes the chunk to `out` and into every other rank's
 *     gather region; after a second flag exchange (flag words 8..15 of the
 *     header) each rank copies the other chunks from its gather region. Each
 *     rank sends (world - 1) / world of a plane in fp32 and of the result in
 *     F. Needs 2 * (rows * n * 4 rounded up to 256) + rows * n * sizeof(F)
 *     bytes per slot.
 * Epochs as for cawq_gemm_colpar_p2p.
 */
cawq_status cawq_gemm_rowpar_p2p(const cawq_tp_peers* peers, uint32_t epoch, const void* x,
                                 const uint32_t* qweight, const uint32_t* qzeros,
                                 const void* scales, const void* bias, void* out, size_t rows,
                                 size_t k, size_t n, size_t group_size, cawq_dtype dtype,
                                 void* stream);

#ifdef __cplusplus
}
#endif

#endif /* CUBE_AWQ_H_ */

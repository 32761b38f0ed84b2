/*
 * cutile_b200.h — C ABI of libcutile_b200.so, the sm_100a kernel backend that
 * replaces TileTriton's TTIR -> Triton -> cubin pipeline for the cuTile
 * kernels vadd, rowsum, softmax, layernorm-fwd, matmul, batchmatmul, fmha,
 * and the next ones: layernorm backward, transpose, moe.
 *
 * Every entry point:
 *   - takes plain pointers, sizes and strides (no Julia, torch or CUDA types;
 *     `stream` is a cudaStream_t / CUstream passed as void*, NULL = legacy
 *     default stream of the current device);
 *   - works on caller-owned device memory and allocates nothing on the launch
 *     path (the *_host entry points take host pointers plus a device
 *     workspace);
 *   - returns CTB_OK (0) or a negative ctb_status and never aborts; the
 *     message of the last failure on the calling thread is ctb_last_error().
 *
 * Layout convention (the cuTile/TileTriton ABI): an array is a pointer plus
 * per-dimension sizes and strides in *Julia (column-major) dimension order*,
 * in units of elements — exactly what TileTriton's flatten_args passes
 * (reference: src/runtime.jl:163-198, src/shim.jl:42-63).
 */
#ifndef CUTILE_B200_H
#define CUTILE_B200_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define CTB_ABI_VERSION 1
#define CTB_MAX_DIMS 5

typedef enum {
  CTB_OK = 0,
  CTB_ERR_ARG = -1,            /* bad argument count / NULL pointer          */
  CTB_ERR_DTYPE = -2,          /* element type not supported by the kernel   */
  CTB_ERR_SHAPE = -3,          /* sizes inconsistent or out of range         */
  CTB_ERR_LAYOUT = -4,         /* strides / alignment not supported          */
  CTB_ERR_UNKNOWN_KERNEL = -5, /* no prebuilt kernel under that name         */
  CTB_ERR_CUDA = -6,           /* a CUDA runtime/driver call failed          */
  CTB_ERR_TIMEOUT = -7,        /* a bounded device-side wait gave up         */
  CTB_ERR_NO_DEVICE = -8       /* no usable sm_100 device                    */
} ctb_status;

/* Element types (Julia eltypes of the TileArray). */
typedef enum {
  CTB_F16 = 1,
  CTB_BF16 = 2,
  CTB_F32 = 3,
  CTB_F64 = 4,
  CTB_I32 = 5 /* Int32: routing tables (moe) */
} ctb_dtype;

/* One cuTile TileArray after flattening: pointer, sizes, strides (Julia dim
 * order, element units). Replaces the (CuPtr, Int32 x N, Int32 x N) triple
 * that src/runtime.jl:169-187 pushes per :tilearray argument. */
typedef struct {
  void* ptr;
  int32_t ndim;
  int32_t dtype; /* ctb_dtype */
  int32_t sizes[CTB_MAX_DIMS];
  int32_t strides[CTB_MAX_DIMS];
} ctb_array;

/* What a prebuilt kernel expects; the B200 analogue of TritonKernel's
 * recorded metadata (reference: src/runtime.jl:85-95). */
typedef struct {
  char name[32];
  int32_t narrays;  /* number of TileArray arguments, in cuTile order      */
  int32_t nscalars; /* number of non-array runtime arguments (as doubles)  */
  int32_t num_warps;
  int32_t shared_bytes;
} ctb_kernel_info;

/* ---- library / device management ---------------------------------------- */

/* ABI version of the loaded library (CTB_ABI_VERSION). */
int ctb_version(void);

/* Message of the last failed call on this thread ("" if none). */
const char* ctb_last_error(void);

/* Per-device one-time set-up (kernel attributes, device properties) for
 * `device`; idempotent and thread-safe. Replaces the per-kernel CuModule
 * load of src/runtime.jl:39-46 (`_cuda_load`) and the target probe of
 * src/runtime.jl:26-31 (`_default_target`). Fails with CTB_ERR_NO_DEVICE if
 * the device is not compute capability 10.0. */
int ctb_init(int device);

/* Reads and clears the device-side error word of the current device (set
 * when a bounded wait inside a kernel gave up). Synchronises `stream`.
 * Returns CTB_OK or CTB_ERR_TIMEOUT; after CTB_ERR_TIMEOUT the outputs of
 * the launches since the previous check are undefined. */
int ctb_check_device(void* stream);

/* ---- generic registry: the TritonRun.triton_kernel / launch! boundary ----- */

/* Look up the prebuilt kernel for cuTile function `name` specialised on the
 * TileArray element types `dtypes[0..ndtypes)` and ghost Constant values
 * `consts` (tile sizes; they identify the specialisation only — results
 * never depend on them). Replaces triton_kernel / compile_kernel
 * (reference: src/runtime.jl:128-160) and the candidate build of
 * get_kernel (src/shim.jl:20-36). Names: "vadd", "rowsum", "softmax",
 * "layernorm_fwd" (alias "layer_norm_fwd"), "layernorm_bwd", "matmul" (alias
 * "matmul16"), "batchmatmul", "fmha", "transpose". */
int ctb_find_kernel(const char* name, const int32_t* dtypes, int32_t ndtypes,
                    const int64_t* consts, int32_t nconsts, int32_t* handle);

/* Metadata of a handle returned by ctb_find_kernel. */
int ctb_kernel_info_get(int32_t handle, ctb_kernel_info* info);

/* Launch `handle` on `stream` with the flattened cuTile arguments: arrays in
 * argument order, then the remaining primitive arguments as doubles. `grid`
 * is cuTile's grid; it is advisory (outputs never depend on it, the backend
 * picks its own grid). Replaces launch! (src/runtime.jl:206-222) and
 * _launch_one / ShimKernel's call (src/shim.jl:65-114). The seed and the two
 * scratch pointers of the Triton ABI (src/runtime.jl:190-196) have no
 * counterpart: these kernels use no RNG and no global scratch. */
int ctb_launch(int32_t handle, const ctb_array* arrays, int32_t narrays,
               const double* scalars, int32_t nscalars, const int32_t grid[3],
               void* stream);

/* ---- typed entry points (what the registry dispatches to) ---------------- */

/* c[i*sc] = a[i*sa] + b[i*sb], i < n, dtype F16/F32/F64; IEEE round-to-
 * nearest add, no flush-to-zero: bit-exact with the host `a .+ b`.
 * cuTile `vadd(a, b, c, tile)` (reference: test/runtests.jl:31-37). */
int ctb_vadd(int32_t dtype, const void* a, const void* b, void* c, int64_t n,
             int64_t sa, int64_t sb, int64_t sc, void* stream);

/* out[i*so] = sum_j a[i*s_i + j*s_j] for i < m, j < n (f32 in, f32 out).
 * cuTile `rowsum(a, out, tm, tn)` = `sum(tile; dims=2)` over Julia dim 2
 * (reference: test/runtests.jl:50-56). Julia column-major a has s_i = 1,
 * s_j = m. */
int ctb_rowsum_f32(const float* a, float* out, int32_t m, int32_t n,
                   int64_t s_i, int64_t s_j, int64_t so, void* stream);

/* For each of `count` vectors v (vector v starts at x + v*ldx and has `len`
 * contiguous elements): y = exp(x - max(x)) / sum(exp(x - max(x))).
 * cuTile `softmax(output, input, TILE_SIZE)` over Julia dim 1 of a
 * (len x count) array (reference: test/runtests.jl:102-118). */
int ctb_softmax_f32(const float* x, float* y, int32_t len, int32_t count,
                    int64_t ldx, int64_t ldy, void* stream);

/* LayerNorm forward over `rows` vectors of `n` contiguous elements:
 * mean = sum(x)/n, var = sum((x-mean)^2)/n (biased), rstd = 1/sqrt(var+eps),
 * y = (x - mean) * rstd * w + b; stores y, mean[row], rstd[row].
 * cuTile layernorm example forward kernel (example layernorm.jl:27, not
 * vendored in the reference; named in research/sass/examples). */
int ctb_layernorm_fwd_f32(const float* x, const float* w, const float* b,
                          float* y, float* mean, float* rstd, int32_t n,
                          int32_t rows, int64_t ldx, int64_t ldy, float eps,
                          void* stream);

/* LayerNorm backward over `rows` vectors of `n` contiguous elements (the
 * cuTile example's backward kernels, layernorm.jl lines 118 and 186, not
 * vendored in the reference): with xhat = (x - mean) * rstd, g = w * dy,
 *   dx = (g - (xhat * mean(g * xhat) + mean(g))) * rstd,
 *   dw = sum_rows dy * xhat,   db = sum_rows dy.
 * `partial` is caller-provided workspace of 2 * groups * n floats (per-CTA dw
 * and db partial rows, like the example's DW/DB group buffers; no locks are
 * needed). groups >= 1; ctb_layernorm_bwd_groups() gives the value that fills
 * the GPU. n <= 16384, n and the row strides multiples of 4, pointers
 * 16-byte aligned. Deterministic for a given `groups`. If a bounded wait
 * inside the row pass gives up (ctb_check_device then returns
 * CTB_ERR_TIMEOUT), dx, dw and db of that call are undefined. */
int ctb_layernorm_bwd_f32(const float* x, const float* dy, const float* w,
                          const float* mean, const float* rstd, float* dx,
                          float* dw, float* db, int32_t n, int32_t rows,
                          int64_t ldx, int64_t lddy, int64_t lddx,
                          float* partial, int32_t groups, void* stream);

/* Recommended `groups` for ctb_layernorm_bwd_f32 on the current device: one
 * wave of resident CTAs — 4 per SM for n <= 2048, 1 per SM above that — at
 * most rows; -1 if the device cannot be queried. */
int ctb_layernorm_bwd_groups(int32_t n, int32_t rows);

/* Allocation-free variant of ctb_layernorm_bwd_f32 (no counterpart in the
 * reference). For callers that cannot allocate device memory when they need
 * the backward pass — a process that reserved its whole device-memory budget
 * for its own pool, or Julia code running where CUDA.jl's allocator must not
 * be entered. The dW/dB partial workspace comes from an 8 MiB array built
 * into the library (held on every GPU that loads it until exit) instead of
 * from the caller; the caller still passes every input and output.
 * groups <= 0 picks the largest useful value that fits: the value of
 * ctb_layernorm_bwd_groups capped at 2,097,152 / (2 * n) (256 at n = 4096, above
 * the 148 that ctb_layernorm_bwd_groups gives there on B200); where the cap
 * binds, dW/dB can differ from ctb_layernorm_bwd_f32's in the last bits
 * (another summation order); pass the same `groups` to both for identical
 * results. 2 * groups * n must
 * not exceed 2,097,152 floats (CTB_ERR_SHAPE otherwise). The first call on a
 * device (and the first after a cudaDeviceReset) looks up the array's device
 * address; make it before any stream capture. All calls share the array:
 * calls that overlap on a GPU race. */
int ctb_layernorm_bwd_f32_noalloc(const float* x, const float* dy,
                                  const float* w, const float* mean,
                                  const float* rstd, float* dx, float* dw,
                                  float* db, int32_t n, int32_t rows,
                                  int64_t ldx, int64_t lddy, int64_t lddx,
                                  int32_t groups, void* stream);

/* y = x^T: x is Julia M x N (column stride ldx), y is N x M (column stride
 * ldy); dtype F16/F32/F64; a copy, bit-exact. cuTile example transpose.jl
 * (not vendored in the reference; research/bench_final.log:10). */
int ctb_transpose(int32_t dtype, const void* x, void* y, int32_t M, int32_t N,
                  int64_t ldx, int64_t ldy, void* stream);

/* C = A * B, Float16 in, Float32 accumulate, Float16 out (round to nearest),
 * Julia column-major: A is M x K with column stride lda, B is K x N (ldb),
 * C is M x N (ldc). cuTile `matmul16(A, B, C, tm, tn, tk)` (reference:
 * bench/bench_f16.jl:10-22). */
int ctb_gemm_f16(const void* A, const void* B, void* C, int32_t M, int32_t N,
                 int32_t K, int64_t lda, int64_t ldb, int64_t ldc,
                 void* stream);

/* Batched form: for b < batch, C_b = A_b * B_b with A_b = A + b*sA etc.
 * cuTile example batchmatmul.jl:15 (not vendored; report.html:480). */
int ctb_bgemm_f16(const void* A, const void* B, void* C, int32_t M, int32_t N,
                  int32_t K, int32_t batch, int64_t lda, int64_t ldb,
                  int64_t ldc, int64_t sA, int64_t sB, int64_t sC,
                  void* stream);

/* Attention forward, Float16 Q/K/V/O, Float32 softmax accumulation:
 * O[b,h] = softmax(scale * Q K^T [+ causal mask: key j > query i masked]) V.
 * Layout row-major [batch, heads, seq, head_dim] (= Julia (D, S, H, B),
 * head_dim contiguous). head_dim must be 64 or 128; both run on the tcgen05
 * tensor-core kernel when the four pointers are 16-byte aligned (a CUDA-core
 * kernel serves unaligned pointers). cuTile example
 * fmha.jl:20 (not vendored; report.html:2981). */
int ctb_fmha_fwd_f16(const void* Q, const void* K, const void* V, void* O,
                     int32_t batch, int32_t heads, int32_t seq_q,
                     int32_t seq_k, int32_t head_dim, float scale,
                     int32_t causal, void* stream);

/* Host-buffer entry points. The arrays are in host memory (page-locked for
 * the copies to overlap: cudaHostAlloc or cudaHostRegister); rows (elements
 * for vadd) move in chunks through `workspace` (device memory, 256-byte
 * aligned) on three streams of the library so that host-to-device copies, the
 * kernel and device-to-host copies of successive chunks overlap. The caller's
 * `stream` first orders the work after what it already holds and is made to
 * wait for the last copy: the host outputs are complete once `stream` has
 * completed. Contiguous rows only. Calls on one device enqueue one at a time;
 * calls that share a workspace must also be ordered on the device (the same
 * `stream`, or synchronised in between), since each call reuses its slots.
 * ctb_host_workspace_bytes(in bytes per unit, out bytes per unit, units) is a
 * workspace size that keeps three chunks of 1/8 of the work in flight;
 * LayerNorm needs 2 * round_up(4 n, 256) bytes more for w and b. */
int64_t ctb_host_workspace_bytes(int64_t unit_bytes_in, int64_t unit_bytes_out, int64_t units);
int ctb_softmax_f32_host(const float* x, float* y, int32_t len, int32_t count, void* workspace,
                         int64_t workspace_bytes, void* stream);
int ctb_layernorm_fwd_f32_host(const float* x, const float* w, const float* b, float* y,
                               float* mean, float* rstd, int32_t n, int32_t rows, float eps,
                               void* workspace, int64_t workspace_bytes, void* stream);
int ctb_vadd_host(int32_t dtype, const void* a, const void* b, void* c, int64_t n,
                  void* workspace, int64_t workspace_bytes, void* stream);

/* Gather-routed mixture-of-experts GEMM (the cuTile moe example is not
 * vendored in the reference; research/bench_final.log:7 benchmarks it). The
 * contract is the published fused-MoE one: `sorted_token_ids` (EM entries,
 * EM a multiple of 128) lists token*topk slots grouped by expert, each expert
 * padded to a multiple of 128 with ids >= M*topk; `expert_ids[EM/128]` gives
 * each 128-block's expert; `*num_tokens_post_padded` (device int) bounds the
 * blocks in use. For every listed slot s < M*topk of a block of expert e:
 *   C[s, :] = (A[s / topk, :] . B[e]^T) * (mul_routed_weight ? w[s] : 1)
 * A: M x K Float16 row-major (row stride lda); B: E x N x K Float16, K
 * contiguous (row stride ldb, expert stride N*ldb); C: (M*topk) x N Float16
 * row-major (ldc); Float32 accumulation. K, lda, ldb, ldc multiples of 8.
 * `workspace` (16-byte aligned, at least ctb_moe_workspace_bytes(EM, K))
 * receives the routed rows of A in sorted order before the GEMM runs. */
int64_t ctb_moe_workspace_bytes(int32_t EM, int32_t K);

/* Routing for ctb_moe_gemm_f16 on the device, without a host round trip:
 * the `moe_align_block_size` step of the fused-MoE contract (the layout the
 * cuTile moe example consumes; the example is not vendored in the
 * reference). topk_ids: `slots` = M * topk Int32 expert ids in slot order
 * (token-major). Writes sorted_token_ids[capacity] (each expert's slots in
 * slot order, padded with the id `slots` to a multiple of `block`, experts
 * in order, then `slots` up to capacity), expert_ids[capacity / block] (-1
 * past the last used block) and num_tokens_post_padded[1]. capacity must be
 * a multiple of block and at least ctb_moe_align_capacity(slots, E, block),
 * the worst case, so the caller sizes the outputs without knowing the
 * routing; pass EM = capacity to ctb_moe_gemm_f16. E <= 256. Ids outside
 * [0, E) are not listed. One CTA; runs on `stream`. */
int32_t ctb_moe_align_capacity(int32_t slots, int32_t E, int32_t block);
int ctb_moe_align_i32(const int32_t* topk_ids, int32_t slots, int32_t E, int32_t block,
                      int32_t* sorted_token_ids, int32_t* expert_ids,
                      int32_t* num_tokens_post_padded, int32_t capacity, void* stream);
int ctb_moe_gemm_f16(const void* A, const void* B, void* C,
                     const int32_t* sorted_token_ids, const int32_t* expert_ids,
                     const int32_t* num_tokens_post_padded,
                     const float* topk_weights, int32_t mul_routed_weight,
                     int32_t M, int32_t N, int32_t K, int32_t E, int32_t EM,
                     int32_t topk, int32_t block_m, int64_t lda, int64_t ldb, int64_t ldc,
                     void* workspace, int64_t workspace_bytes, void* stream);

/* ---- seeded synthetic inputs (bench / test plumbing, not a cuTile op) ---- */

/* Counter-based SplitMix64 stream: element i uses counter offset + i.
 * Uniform: lo + (hi - lo) * u, u = top 24 bits / 2^24, computed in double
 * and rounded to dtype. Normal: mean + std * Box-Muller(u1, u2) from
 * counters 2(offset+i), 2(offset+i)+1. */
int ctb_fill_uniform(void* ptr, int32_t dtype, int64_t n, uint64_t seed,
                     uint64_t offset, double lo, double hi, void* stream);
int ctb_fill_normal(void* ptr, int32_t dtype, int64_t n, uint64_t seed,
                    uint64_t offset, double mean, double std, void* stream);

/* ---- failure-path self-test (test plumbing, not a cuTile op) ------------- */

/* Launches one CTA whose warp 0 holds 32 TMEM columns and waits on an
 * mbarrier that nothing arrives on, giving up after `limit_ns` (1..1e9);
 * its warp 1 waits on the same barrier with the library's default limit
 * and leaves through the CTA abort flag. The TMEM is released before the
 * CTA returns. `status` (device memory, 3 ints): [0] = 1 when warp 0's wait
 * gave up, [1] = 1 when warp 1's did, [2] = the ns warp 1 waited. The next
 * ctb_check_device returns CTB_ERR_TIMEOUT and clears the error word; the
 * context stays usable. It exercises the exit path that every pipeline wait
 * of this library takes (the reference reports no device-side timeouts:
 * its kernels have no bounded waits). */
int ctb_selftest_wait_timeout(int64_t limit_ns, int* status, void* stream);

#ifdef __cplusplus
}
#endif
#endif /* CUTILE_B200_H */

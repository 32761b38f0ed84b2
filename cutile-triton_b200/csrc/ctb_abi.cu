// Library plumbing of libcutile_b200.so: error strings, per-device set-up,
// the device error word, seeded input fills, and the kernel registry behind
// ctb_find_kernel / ctb_launch — the B200 replacement of TileTriton's
// triton_kernel / launch! (reference: src/runtime.jl:128-222) and of the
// shim's get_kernel / ShimKernel call (src/shim.jl:20-114).
#include "ctb_common.cuh"

#include <cmath>
#include <cstring>
#include <algorithm>
#include <cuda.h>
#include <mutex>

namespace ctb {

// ---- errors -----------------------------------------------------------------
static thread_local std::string t_last_error;

int set_error(int code, const std::string& msg) {
  t_last_error = msg;
  return code;
}
void clear_error() { t_last_error.clear(); }
int cuda_fail(cudaError_t e, const char* what) {
  return set_error(CTB_ERR_CUDA, std::string(what) + ": " + cudaGetErrorName(e) + " (" +
                                     cudaGetErrorString(e) + ")");
}

// ---- per-device properties --------------------------------------------------
constexpr int kMaxDevices = 64;
static DeviceProps g_props[kMaxDevices];
static std::once_flag g_props_once[kMaxDevices];
static int g_props_rc[kMaxDevices];

static int init_device_props(int dev) {
  cudaDeviceProp pr;
  cudaError_t e = cudaGetDeviceProperties(&pr, dev);
  if (e != cudaSuccess) return cuda_fail(e, "cudaGetDeviceProperties");
  if (pr.major != 10)
    return set_error(CTB_ERR_NO_DEVICE, std::string("device ") + pr.name +
                                            " is not compute capability 10.x (sm_100a build)");
  DeviceProps& p = g_props[dev];
  p.sm_count = pr.multiProcessorCount;
  p.max_smem_optin = (int)pr.sharedMemPerBlockOptin;
  p.cc_major = pr.major;
  p.cc_minor = pr.minor;
  return CTB_OK;
}

int current_props(DeviceProps* out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
  if (dev < 0 || dev >= kMaxDevices) return set_error(CTB_ERR_NO_DEVICE, "device ordinal out of range");
  std::string msg;
  std::call_once(g_props_once[dev], [&] {
    g_props_rc[dev] = init_device_props(dev);
    if (g_props_rc[dev]) msg = t_last_error;
  });
  if (g_props_rc[dev]) {
    if (!msg.empty()) t_last_error = msg;
    else t_last_error = "device set-up failed earlier on this device";
    return g_props_rc[dev];
  }
  *out = g_props[dev];
  return CTB_OK;
}

// ---- seeded fills -------------------------------------------------------------
// SplitMix64 finaliser (Steele, Lea, Flood, "Fast splittable pseudorandom
// number generators", OOPSLA 2014) applied to seed + (counter+1) * golden gamma.
__host__ __device__ __forceinline__ uint64_t splitmix64_at(uint64_t seed, uint64_t ctr) {
  uint64_t z = seed + (ctr + 1) * 0x9E3779B97F4A7C15ull;
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  return z ^ (z >> 31);
}
__device__ __forceinline__ double u24(uint64_t z) {
  return (double)(z >> 40) * (1.0 / 16777216.0);
}

template <typename T>
__device__ __forceinline__ T from_double(double v);
template <> __device__ __forceinline__ float from_double<float>(double v) { return __double2float_rn(v); }
template <> __device__ __forceinline__ double from_double<double>(double v) { return v; }
template <> __device__ __forceinline__ __half from_double<__half>(double v) { return __double2half(v); }
template <> __device__ __forceinline__ __nv_bfloat16 from_double<__nv_bfloat16>(double v) {
  return __double2bfloat16(v);
}

template <typename T>
__global__ void fill_uniform_kernel(T* p, int64_t n, uint64_t seed, uint64_t offset, double lo,
                                    double hi) {
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride) {
    const double u = u24(splitmix64_at(seed, offset + (uint64_t)i));
    p[i] = from_double<T>(__dadd_rn(lo, __dmul_rn(__dsub_rn(hi, lo), u)));
  }
}

template <typename T>
__global__ void fill_normal_kernel(T* p, int64_t n, uint64_t seed, uint64_t offset, double mean,
                                   double sd) {
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride) {
    const uint64_t c = 2 * (offset + (uint64_t)i);
    // u1 in (0, 1] so that log(u1) is finite.
    const double u1 = 1.0 - u24(splitmix64_at(seed, c));
    const double u2 = u24(splitmix64_at(seed, c + 1));
    const double z = sqrt(-2.0 * log(u1)) * cospi(2.0 * u2);
    p[i] = from_double<T>(__dadd_rn(mean, __dmul_rn(sd, z)));
  }
}

}  // namespace ctb

using namespace ctb;

// =============================================================================
// C ABI: library management
// =============================================================================
extern "C" int ctb_version(void) { return CTB_ABI_VERSION; }

extern "C" const char* ctb_last_error(void) { return t_last_error.c_str(); }

// Defined in gemm_sm100.cu / fmha_sm100.cu: per-device kernel attributes.
namespace ctb {
int gemm_device_setup();
int fmha_device_setup();
int gemm_take_device_error(unsigned int* out);
int fmha_take_device_error(unsigned int* out);
int moe_take_device_error(unsigned int* out);
int layernorm_bwd_take_device_error(unsigned int* out);
int selftest_take_device_error(unsigned int* out);
}

extern "C" int ctb_init(int device) {
  clear_error();
  int n = 0;
  cudaError_t e = cudaGetDeviceCount(&n);
  if (e != cudaSuccess) return cuda_fail(e, "cudaGetDeviceCount");
  if (device < 0 || device >= n) return set_error(CTB_ERR_NO_DEVICE, "ctb_init: no such device");
  int prev = 0;
  CTB_CUDA_CHECK(cudaGetDevice(&prev));
  CTB_CUDA_CHECK(cudaSetDevice(device));
  DeviceProps p;
  int rc = current_props(&p);
  if (rc == CTB_OK) rc = gemm_device_setup();
  if (rc == CTB_OK) rc = fmha_device_setup();
  cudaSetDevice(prev);
  return rc;
}

namespace ctb {
// ---- per-context set-up --------------------------------------------------------
using PFN_ctxGetCurrent = CUresult (*)(CUcontext*);
using PFN_ctxGetId = CUresult (*)(CUcontext, unsigned long long*);

int current_context_id(unsigned long long* id) {
  // Since CUDA 12 cudaSetDevice makes the device's primary context current
  // (creating it again after a cudaDeviceReset), so the ID is the live one.
  int dev = 0;
  CTB_CUDA_CHECK(cudaGetDevice(&dev));
  CTB_CUDA_CHECK(cudaSetDevice(dev));
  static PFN_ctxGetCurrent get_current = nullptr;
  static PFN_ctxGetId get_id = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &fn, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      get_current = reinterpret_cast<PFN_ctxGetCurrent>(fn);
    if (cudaGetDriverEntryPoint("cuCtxGetId", &fn, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      get_id = reinterpret_cast<PFN_ctxGetId>(fn);
  });
  if (!get_current || !get_id)
    return set_error(CTB_ERR_CUDA, "cuCtxGetCurrent / cuCtxGetId entry points unavailable");
  CUcontext ctx = nullptr;
  if (get_current(&ctx) != CUDA_SUCCESS || ctx == nullptr || get_id(ctx, id) != CUDA_SUCCESS)
    return set_error(CTB_ERR_CUDA, "no current CUDA context");
  return CTB_OK;
}
}  // namespace ctb

extern "C" int ctb_check_device(void* stream) {
  clear_error();
  CTB_CUDA_CHECK(cudaStreamSynchronize(static_cast<cudaStream_t>(stream)));
  unsigned int hg = 0, hf = 0;
  if (int e = gemm_take_device_error(&hg)) return cuda_fail((cudaError_t)e, "reading the GEMM error word");
  if (int e = fmha_take_device_error(&hf)) return cuda_fail((cudaError_t)e, "reading the FMHA error word");
  unsigned int hm = 0;
  if (int e = moe_take_device_error(&hm)) return cuda_fail((cudaError_t)e, "reading the MoE error word");
  unsigned int hl = 0;
  if (int e = layernorm_bwd_take_device_error(&hl))
    return cuda_fail((cudaError_t)e, "reading the layernorm backward error word");
  unsigned int hs = 0;
  if (int e = selftest_take_device_error(&hs))
    return cuda_fail((cudaError_t)e, "reading the self-test error word");
  const unsigned int h = hg | hf | hm | hl | hs;
  if (h) {
    return set_error(CTB_ERR_TIMEOUT, "a bounded device-side wait gave up (error word " +
                                          std::to_string(h) + ")");
  }
  return CTB_OK;
}

// =============================================================================
// C ABI: fills
// =============================================================================
template <typename T>
static int fill_u(void* ptr, int64_t n, uint64_t seed, uint64_t off, double lo, double hi,
                  cudaStream_t st, int sm) {
  const int grid = (int)std::min<int64_t>((n + 255) / 256, (int64_t)sm * 8);
  fill_uniform_kernel<T><<<grid, 256, 0, st>>>((T*)ptr, n, seed, off, lo, hi);
  return launch_status("fill_uniform_kernel");
}
template <typename T>
static int fill_n(void* ptr, int64_t n, uint64_t seed, uint64_t off, double mu, double sd,
                  cudaStream_t st, int sm) {
  const int grid = (int)std::min<int64_t>((n + 255) / 256, (int64_t)sm * 8);
  fill_normal_kernel<T><<<grid, 256, 0, st>>>((T*)ptr, n, seed, off, mu, sd);
  return launch_status("fill_normal_kernel");
}

extern "C" int ctb_fill_uniform(void* ptr, int32_t dtype, int64_t n, uint64_t seed,
                                uint64_t offset, double lo, double hi, void* stream) {
  clear_error();
  if (n < 0) return set_error(CTB_ERR_SHAPE, "fill: negative length");
  if (n == 0) return CTB_OK;
  if (!ptr) return set_error(CTB_ERR_ARG, "fill: NULL pointer");
  DeviceProps p;
  if (int rc = current_props(&p)) return rc;
  auto st = static_cast<cudaStream_t>(stream);
  switch (dtype) {
    case CTB_F32: return fill_u<float>(ptr, n, seed, offset, lo, hi, st, p.sm_count);
    case CTB_F64: return fill_u<double>(ptr, n, seed, offset, lo, hi, st, p.sm_count);
    case CTB_F16: return fill_u<__half>(ptr, n, seed, offset, lo, hi, st, p.sm_count);
    case CTB_BF16: return fill_u<__nv_bfloat16>(ptr, n, seed, offset, lo, hi, st, p.sm_count);
    default: return set_error(CTB_ERR_DTYPE, "fill: unknown dtype");
  }
}

extern "C" int ctb_fill_normal(void* ptr, int32_t dtype, int64_t n, uint64_t seed,
                               uint64_t offset, double mean, double sd, void* stream) {
  clear_error();
  if (n < 0) return set_error(CTB_ERR_SHAPE, "fill: negative length");
  if (n == 0) return CTB_OK;
  if (!ptr) return set_error(CTB_ERR_ARG, "fill: NULL pointer");
  DeviceProps p;
  if (int rc = current_props(&p)) return rc;
  auto st = static_cast<cudaStream_t>(stream);
  switch (dtype) {
    case CTB_F32: return fill_n<float>(ptr, n, seed, offset, mean, sd, st, p.sm_count);
    case CTB_F64: return fill_n<double>(ptr, n, seed, offset, mean, sd, st, p.sm_count);
    case CTB_F16: return fill_n<__half>(ptr, n, seed, offset, mean, sd, st, p.sm_count);
    case CTB_BF16: return fill_n<__nv_bfloat16>(ptr, n, seed, offset, mean, sd, st, p.sm_count);
    default: return set_error(CTB_ERR_DTYPE, "fill: unknown dtype");
  }
}

// =============================================================================
// Registry: cuTile kernel name + element types -> prebuilt launcher
// =============================================================================
extern "C" int ctb_gemm_f32_simt(const float* A, const float* B, float* C, int32_t M, int32_t N,
                                 int32_t K, int32_t batch, int64_t lda, int64_t ldb, int64_t ldc,
                                 int64_t sA, int64_t sB, int64_t sC, void* stream);

namespace {

using Launcher = int (*)(const ctb_array*, const double*, cudaStream_t);

struct Entry {
  const char* name;
  int narrays;
  int nscalars;
  int num_warps;
  int shared_bytes;
  Launcher fn;
};

int need_dims(const ctb_array& a, int nd, const char* k, const char* which) {
  if (a.ndim != nd)
    return set_error(CTB_ERR_SHAPE, std::string(k) + ": " + which + " must have " +
                                        std::to_string(nd) + " dims");
  for (int d = 0; d < nd; ++d)
    if (a.sizes[d] < 0) return set_error(CTB_ERR_SHAPE, std::string(k) + ": negative size");
  return CTB_OK;
}

int L_vadd(const ctb_array* x, const double*, cudaStream_t st) {
  for (int i = 0; i < 3; ++i)
    if (int rc = need_dims(x[i], 1, "vadd", "a/b/c")) return rc;
  if (x[0].dtype != x[1].dtype || x[0].dtype != x[2].dtype)
    return set_error(CTB_ERR_DTYPE, "vadd: a, b, c must share an element type");
  // cuTile's masked tile load/store covers c's extent; a and b must cover it.
  const int64_t n = x[2].sizes[0];
  if (x[0].sizes[0] < n || x[1].sizes[0] < n)
    return set_error(CTB_ERR_SHAPE, "vadd: a and b shorter than c");
  return ctb_vadd(x[0].dtype, x[0].ptr, x[1].ptr, x[2].ptr, n, x[0].strides[0], x[1].strides[0],
                  x[2].strides[0], st);
}

int L_rowsum(const ctb_array* x, const double*, cudaStream_t st) {
  if (int rc = need_dims(x[0], 2, "rowsum", "a")) return rc;
  if (x[0].dtype != CTB_F32 || x[1].dtype != CTB_F32)
    return set_error(CTB_ERR_DTYPE, "rowsum: Float32 only");
  const int m = x[0].sizes[0], n = x[0].sizes[1];
  if (x[1].sizes[0] != m) return set_error(CTB_ERR_SHAPE, "rowsum: out must have size(a,1) rows");
  if (x[1].ndim == 2 && x[1].sizes[1] != 1)
    return set_error(CTB_ERR_SHAPE, "rowsum: out must be m x 1");
  return ctb_rowsum_f32((const float*)x[0].ptr, (float*)x[1].ptr, m, n, x[0].strides[0],
                        x[0].strides[1], x[1].strides[0], st);
}

// softmax(output, input, TILE_SIZE): per column of the Julia (len x count) array.
int L_softmax(const ctb_array* x, const double*, cudaStream_t st) {
  const ctb_array &out = x[0], &in = x[1];
  if (int rc = need_dims(in, 2, "softmax", "input")) return rc;
  if (int rc = need_dims(out, 2, "softmax", "output")) return rc;
  if (in.dtype != CTB_F32 || out.dtype != CTB_F32)
    return set_error(CTB_ERR_DTYPE, "softmax: Float32 only");
  if (in.sizes[0] != out.sizes[0] || in.sizes[1] != out.sizes[1])
    return set_error(CTB_ERR_SHAPE, "softmax: input and output sizes differ");
  if (in.strides[0] != 1 || out.strides[0] != 1)
    return set_error(CTB_ERR_LAYOUT, "softmax: dim 1 must be contiguous (stride 1)");
  return ctb_softmax_f32((const float*)in.ptr, (float*)out.ptr, in.sizes[0], in.sizes[1],
                         in.strides[1], out.strides[1], st);
}

// layer_norm_fwd(X, W, B, Y, Mean, Rstd, eps, TILE_N): X is Julia (N x M),
// each of the M columns normalised over its N contiguous elements.
int L_layernorm(const ctb_array* x, const double* s, cudaStream_t st) {
  const ctb_array &X = x[0], &W = x[1], &B = x[2], &Y = x[3], &Mu = x[4], &Rs = x[5];
  if (int rc = need_dims(X, 2, "layernorm_fwd", "X")) return rc;
  if (int rc = need_dims(Y, 2, "layernorm_fwd", "Y")) return rc;
  for (int i = 0; i < 6; ++i)
    if (x[i].dtype != CTB_F32) return set_error(CTB_ERR_DTYPE, "layernorm_fwd: Float32 only");
  const int n = X.sizes[0], rows = X.sizes[1];
  if (Y.sizes[0] != n || Y.sizes[1] != rows)
    return set_error(CTB_ERR_SHAPE, "layernorm_fwd: X and Y sizes differ");
  if (W.sizes[0] != n || B.sizes[0] != n)
    return set_error(CTB_ERR_SHAPE, "layernorm_fwd: W and B must have size(X,1) elements");
  if (Mu.sizes[0] != rows || Rs.sizes[0] != rows)
    return set_error(CTB_ERR_SHAPE, "layernorm_fwd: Mean and Rstd must have size(X,2) elements");
  if (X.strides[0] != 1 || Y.strides[0] != 1 || W.strides[0] != 1 || B.strides[0] != 1 ||
      Mu.strides[0] != 1 || Rs.strides[0] != 1)
    return set_error(CTB_ERR_LAYOUT, "layernorm_fwd: dim 1 must be contiguous (stride 1)");
  return ctb_layernorm_fwd_f32((const float*)X.ptr, (const float*)W.ptr, (const float*)B.ptr,
                               (float*)Y.ptr, (float*)Mu.ptr, (float*)Rs.ptr, n, rows,
                               X.strides[1], Y.strides[1], (float)s[0], st);
}

// layernorm_bwd(DX, DY, DW, DB, X, W, Mean, Rstd, PARTIAL): X/DY/DX Julia
// (N x M) with contiguous columns; PARTIAL is Julia (N x 2G) workspace.
int L_layernorm_bwd(const ctb_array* a, const double*, cudaStream_t st) {
  const ctb_array &DX = a[0], &DY = a[1], &DW = a[2], &DB = a[3], &X = a[4], &W = a[5],
                  &Mu = a[6], &Rs = a[7], &P = a[8];
  for (int i = 0; i < 9; ++i)
    if (a[i].dtype != CTB_F32) return set_error(CTB_ERR_DTYPE, "layernorm_bwd: Float32 only");
  if (int rc = need_dims(X, 2, "layernorm_bwd", "X")) return rc;
  const int n = X.sizes[0], rows = X.sizes[1];
  if (DX.ndim != 2 || DY.ndim != 2 || DX.sizes[0] != n || DX.sizes[1] != rows ||
      DY.sizes[0] != n || DY.sizes[1] != rows)
    return set_error(CTB_ERR_SHAPE, "layernorm_bwd: X, DY, DX sizes differ");
  if (W.sizes[0] != n || DW.sizes[0] != n || DB.sizes[0] != n || Mu.sizes[0] != rows ||
      Rs.sizes[0] != rows)
    return set_error(CTB_ERR_SHAPE, "layernorm_bwd: W/DW/DB need N, Mean/Rstd need M elements");
  int64_t pe = 1;
  for (int d = 0; d < P.ndim; ++d) pe *= P.sizes[d];
  if (pe < 2 * (int64_t)n || pe % (2 * (int64_t)n) != 0)
    return set_error(CTB_ERR_SHAPE, "layernorm_bwd: PARTIAL must hold 2 x groups x N floats");
  if (X.strides[0] != 1 || DY.strides[0] != 1 || DX.strides[0] != 1)
    return set_error(CTB_ERR_LAYOUT, "layernorm_bwd: dim 1 must be contiguous (stride 1)");
  return ctb_layernorm_bwd_f32((const float*)X.ptr, (const float*)DY.ptr, (const float*)W.ptr,
                               (const float*)Mu.ptr, (const float*)Rs.ptr, (float*)DX.ptr,
                               (float*)DW.ptr, (float*)DB.ptr, n, rows, X.strides[1],
                               DY.strides[1], DX.strides[1], (float*)P.ptr,
                               (int32_t)(pe / (2 * (int64_t)n)), st);
}

// transpose(x, y): y = x', both Julia 2-D with contiguous columns.
int L_transpose(const ctb_array* a, const double*, cudaStream_t st) {
  const ctb_array &X = a[0], &Y = a[1];
  if (int rc = need_dims(X, 2, "transpose", "x")) return rc;
  if (int rc = need_dims(Y, 2, "transpose", "y")) return rc;
  if (X.dtype != Y.dtype) return set_error(CTB_ERR_DTYPE, "transpose: x and y element types differ");
  if (Y.sizes[0] != X.sizes[1] || Y.sizes[1] != X.sizes[0])
    return set_error(CTB_ERR_SHAPE, "transpose: y must be size(x, 2) x size(x, 1)");
  if (X.strides[0] != 1 || Y.strides[0] != 1)
    return set_error(CTB_ERR_LAYOUT, "transpose: dim 1 must be contiguous (stride 1)");
  return ctb_transpose(X.dtype, X.ptr, Y.ptr, X.sizes[0], X.sizes[1], X.strides[1], Y.strides[1], st);
}

// Column-major operand check for matmul: stride (1, ld).
int colmajor_ld(const ctb_array& a, const char* which, int64_t* ld) {
  if (a.strides[0] != 1)
    return set_error(CTB_ERR_LAYOUT, std::string("matmul: ") + which +
                                         " must be column-major (stride 1 along dim 1)");
  *ld = a.strides[1];
  return CTB_OK;
}

int matmul_common(const ctb_array* x, int nd, cudaStream_t st) {
  const char* k = nd == 2 ? "matmul" : "batchmatmul";
  for (int i = 0; i < 3; ++i)
    if (int rc = need_dims(x[i], nd, k, "A/B/C")) return rc;
  const ctb_array &A = x[0], &B = x[1], &C = x[2];
  const int M = A.sizes[0], K = A.sizes[1], N = B.sizes[1];
  if (B.sizes[0] != K || C.sizes[0] != M || C.sizes[1] != N)
    return set_error(CTB_ERR_SHAPE, std::string(k) + ": inner or outer sizes disagree");
  int batch = 1;
  int64_t sA = 0, sB = 0, sC = 0;
  if (nd == 3) {
    batch = C.sizes[2];
    if (A.sizes[2] != batch || B.sizes[2] != batch)
      return set_error(CTB_ERR_SHAPE, "batchmatmul: batch sizes disagree");
    sA = A.strides[2];
    sB = B.strides[2];
    sC = C.strides[2];
  }
  int64_t lda, ldb, ldc;
  if (int rc = colmajor_ld(A, "A", &lda)) return rc;
  if (int rc = colmajor_ld(B, "B", &ldb)) return rc;
  if (int rc = colmajor_ld(C, "C", &ldc)) return rc;
  if (A.dtype == CTB_F16 && B.dtype == CTB_F16 && C.dtype == CTB_F16) {
    if (nd == 2) return ctb_gemm_f16(A.ptr, B.ptr, C.ptr, M, N, K, lda, ldb, ldc, st);
    return ctb_bgemm_f16(A.ptr, B.ptr, C.ptr, M, N, K, batch, lda, ldb, ldc, sA, sB, sC, st);
  }
  if (A.dtype == CTB_F32 && B.dtype == CTB_F32 && C.dtype == CTB_F32)
    return ctb_gemm_f32_simt((const float*)A.ptr, (const float*)B.ptr, (float*)C.ptr, M, N, K,
                             batch, lda, ldb, ldc, sA, sB, sC, st);
  return set_error(CTB_ERR_DTYPE, std::string(k) + ": A, B, C must be all Float16 or all Float32");
}
int L_matmul(const ctb_array* x, const double*, cudaStream_t st) { return matmul_common(x, 2, st); }
int L_bmm(const ctb_array* x, const double*, cudaStream_t st) { return matmul_common(x, 3, st); }

// fmha(Q, K, V, O, scale, causal): Julia (D, S, H, B) arrays, D contiguous,
// densely packed (row-major [B, H, S, D]).
int L_fmha(const ctb_array* x, const double* s, cudaStream_t st) {
  for (int i = 0; i < 4; ++i) {
    if (int rc = need_dims(x[i], 4, "fmha", "Q/K/V/O")) return rc;
    if (x[i].dtype != CTB_F16) return set_error(CTB_ERR_DTYPE, "fmha: Float16 only");
    const int32_t* sz = x[i].sizes;
    const int32_t* sd = x[i].strides;
    if (sd[0] != 1 || sd[1] != sz[0] || sd[2] != (int64_t)sz[0] * sz[1] ||
        sd[3] != (int64_t)sz[0] * sz[1] * sz[2])
      return set_error(CTB_ERR_LAYOUT, "fmha: Q/K/V/O must be densely packed (D, S, H, B)");
  }
  const ctb_array &Q = x[0], &K = x[1], &V = x[2], &O = x[3];
  const int D = Q.sizes[0], Sq = Q.sizes[1], H = Q.sizes[2], Bt = Q.sizes[3];
  const int Sk = K.sizes[1];
  if (K.sizes[0] != D || V.sizes[0] != D || O.sizes[0] != D || V.sizes[1] != Sk ||
      O.sizes[1] != Sq || K.sizes[2] != H || V.sizes[2] != H || O.sizes[2] != H ||
      K.sizes[3] != Bt || V.sizes[3] != Bt || O.sizes[3] != Bt)
    return set_error(CTB_ERR_SHAPE, "fmha: Q/K/V/O sizes disagree");
  return ctb_fmha_fwd_f16(Q.ptr, K.ptr, V.ptr, O.ptr, Bt, H, Sq, Sk, D, (float)s[0],
                          s[1] != 0.0 ? 1 : 0, st);
}

// moe(A, B, C, SORTED, EXPERT_IDS, NTP, WEIGHTS, WORKSPACE, topk, mul_routed_weight):
// Julia arrays A (K, M), B (K, N, E), C (N, M*topk) Float16 with contiguous
// first dims (B's experts N*ldb apart); SORTED (EM), EXPERT_IDS (EM/128), NTP
// (>= 1) Int32 (EM / length(EXPERT_IDS) = 128 or 256 rows per routing block);
// WEIGHTS Float32 (topk, M) contiguous; WORKSPACE Float16
// holding at least K*EM elements.
int L_moe(const ctb_array* x, const double* s, cudaStream_t st) {
  const ctb_array &A = x[0], &B = x[1], &C = x[2], &S = x[3], &EI = x[4], &NT = x[5],
                  &W = x[6], &WS = x[7];
  if (int rc = need_dims(A, 2, "moe", "A")) return rc;
  if (int rc = need_dims(B, 3, "moe", "B")) return rc;
  if (int rc = need_dims(C, 2, "moe", "C")) return rc;
  if (int rc = need_dims(S, 1, "moe", "sorted_token_ids")) return rc;
  if (int rc = need_dims(EI, 1, "moe", "expert_ids")) return rc;
  if (int rc = need_dims(NT, 1, "moe", "num_tokens_post_padded")) return rc;
  if (A.dtype != CTB_F16 || B.dtype != CTB_F16 || C.dtype != CTB_F16 || WS.dtype != CTB_F16)
    return set_error(CTB_ERR_DTYPE, "moe: A, B, C and the workspace must be Float16");
  if (S.dtype != CTB_I32 || EI.dtype != CTB_I32 || NT.dtype != CTB_I32)
    return set_error(CTB_ERR_DTYPE, "moe: routing tables must be Int32");
  const int topk = (int)s[0], mul = s[1] != 0.0 ? 1 : 0;
  if (mul && W.dtype != CTB_F32) return set_error(CTB_ERR_DTYPE, "moe: weights must be Float32");
  const int K = A.sizes[0], M = A.sizes[1], N = B.sizes[1], E = B.sizes[2], EM = S.sizes[0];
  if (B.sizes[0] != K || C.sizes[0] != N || (int64_t)C.sizes[1] != (int64_t)M * topk ||
      NT.sizes[0] < 1 || EI.sizes[0] < 1 ||
      (EM != (int64_t)EI.sizes[0] * 128 && EM != (int64_t)EI.sizes[0] * 256))
    return set_error(CTB_ERR_SHAPE, "moe: A/B/C/routing sizes disagree");
  if (A.strides[0] != 1 || B.strides[0] != 1 || C.strides[0] != 1 || S.strides[0] != 1 ||
      EI.strides[0] != 1 || (int64_t)B.strides[2] != (int64_t)B.strides[1] * N)
    return set_error(CTB_ERR_LAYOUT, "moe: first dims must be contiguous, B's experts packed");
  int64_t ws_elems = 1;
  for (int d = 0; d < WS.ndim; ++d) ws_elems *= WS.sizes[d];
  if (mul) {
    int64_t w_elems = 1;
    for (int d = 0; d < W.ndim; ++d) w_elems *= W.sizes[d];
    if (w_elems < (int64_t)M * topk || W.strides[0] != 1)
      return set_error(CTB_ERR_SHAPE, "moe: weights need topk x M contiguous Float32");
  }
  return ctb_moe_gemm_f16(A.ptr, B.ptr, C.ptr, (const int32_t*)S.ptr, (const int32_t*)EI.ptr,
                          (const int32_t*)NT.ptr, mul ? (const float*)W.ptr : nullptr, mul, M,
                          N, K, E, EM, topk, EM == (int64_t)EI.sizes[0] * 256 ? 256 : 128,
                          A.strides[1], B.strides[1], C.strides[1], WS.ptr,
                          ws_elems * 2, st);
}

const Entry kRegistry[] = {
    {"vadd", 3, 0, 8, 0, L_vadd},
    {"rowsum", 2, 0, 16, 0, L_rowsum},
    {"softmax", 2, 0, 16, 0, L_softmax},
    {"layernorm_fwd", 6, 1, 8, 0, L_layernorm},
    {"layer_norm_fwd", 6, 1, 8, 0, L_layernorm},
    {"layernorm_bwd", 9, 0, 16, 0, L_layernorm_bwd},
    {"matmul", 3, 0, 6, 0, L_matmul},
    {"matmul16", 3, 0, 6, 0, L_matmul},
    {"batchmatmul", 3, 0, 6, 0, L_bmm},
    {"batch_matmul", 3, 0, 6, 0, L_bmm},
    {"fmha", 4, 2, 16, 0, L_fmha},
    {"transpose", 2, 0, 8, 0, L_transpose},
    {"moe", 8, 2, 6, 0, L_moe},
};
constexpr int kRegistrySize = sizeof(kRegistry) / sizeof(kRegistry[0]);

bool dtype_known(int32_t d) { return d >= CTB_F16 && d <= CTB_I32; }

}  // namespace

extern "C" int ctb_find_kernel(const char* name, const int32_t* dtypes, int32_t ndtypes,
                               const int64_t* consts, int32_t nconsts, int32_t* handle) {
  clear_error();
  (void)consts;
  (void)nconsts;  // tile sizes identify the specialisation only
  if (!name || !handle) return set_error(CTB_ERR_ARG, "ctb_find_kernel: NULL argument");
  for (int i = 0; i < kRegistrySize; ++i) {
    if (std::strcmp(kRegistry[i].name, name) != 0) continue;
    if (ndtypes != kRegistry[i].narrays)
      return set_error(CTB_ERR_ARG, std::string(name) + ": expected " +
                                        std::to_string(kRegistry[i].narrays) +
                                        " TileArray element types");
    for (int d = 0; d < ndtypes; ++d)
      if (!dtypes || !dtype_known(dtypes[d]))
        return set_error(CTB_ERR_DTYPE, std::string(name) + ": unknown element type");
    *handle = i;
    return CTB_OK;
  }
  return set_error(CTB_ERR_UNKNOWN_KERNEL,
                   std::string("b200: no prebuilt sm_100a kernel for cuTile function '") + name +
                       "'");
}

extern "C" int ctb_kernel_info_get(int32_t handle, ctb_kernel_info* info) {
  clear_error();
  if (handle < 0 || handle >= kRegistrySize || !info)
    return set_error(CTB_ERR_ARG, "ctb_kernel_info_get: bad handle");
  const Entry& e = kRegistry[handle];
  std::memset(info, 0, sizeof(*info));
  std::strncpy(info->name, e.name, sizeof(info->name) - 1);
  info->narrays = e.narrays;
  info->nscalars = e.nscalars;
  info->num_warps = e.num_warps;
  info->shared_bytes = e.shared_bytes;
  return CTB_OK;
}

extern "C" int ctb_launch(int32_t handle, const ctb_array* arrays, int32_t narrays,
                          const double* scalars, int32_t nscalars, const int32_t grid[3],
                          void* stream) {
  clear_error();
  (void)grid;  // advisory: the backend sizes its own grid
  if (handle < 0 || handle >= kRegistrySize) return set_error(CTB_ERR_ARG, "ctb_launch: bad handle");
  const Entry& e = kRegistry[handle];
  if (narrays != e.narrays || (narrays > 0 && !arrays))
    return set_error(CTB_ERR_ARG, std::string(e.name) + ": expected " +
                                      std::to_string(e.narrays) + " kernel array arguments");
  if (nscalars != e.nscalars || (nscalars > 0 && !scalars))
    return set_error(CTB_ERR_ARG, std::string(e.name) + ": expected " +
                                      std::to_string(e.nscalars) + " scalar arguments");
  for (int i = 0; i < narrays; ++i) {
    if (arrays[i].ndim < 1 || arrays[i].ndim > CTB_MAX_DIMS)
      return set_error(CTB_ERR_SHAPE, std::string(e.name) + ": array rank out of range");
    int64_t elems = 1;
    for (int d = 0; d < arrays[i].ndim; ++d) elems *= arrays[i].sizes[d];
    if (elems > 0 && !arrays[i].ptr)
      return set_error(CTB_ERR_ARG, std::string(e.name) + ": NULL array pointer");
  }
  return e.fn(arrays, scalars, static_cast<cudaStream_t>(stream));
}

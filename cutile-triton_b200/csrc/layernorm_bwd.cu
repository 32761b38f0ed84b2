// LayerNorm backward (cuTile example layernorm.jl kernels at lines 118 and
// 186 — "dx + partial dW/dB" and "reduce dW/dB"; names in the reference's
// research/sass/examples, sources not vendored).
//
// With xhat = (x - mean) * rstd and g = w * dy (per row of n elements):
//   dx = (g - (xhat * mean(g * xhat) + mean(g))) * rstd
//   dW = sum over rows of dy * xhat,  dB = sum over rows of dy
//
// Pass 1 (HBM-bound, one read of x and dy, one write of dx): `groups`
// persistent CTAs each own a contiguous band of rows, keep w and their dW/dB
// partial sums in registers, and write one partial row each into the
// caller's buffer `partial` (2 x groups x n floats: dW partials, then dB).
// Pass 2 folds the `groups` partial rows column by column. No atomics: the
// result is deterministic for a given `groups`.
#include "ctb_common.cuh"

#include <algorithm>
#include <mutex>

namespace ctb {

template <int THREADS, int NV>
__global__ void __launch_bounds__(THREADS) layernorm_bwd_dx_kernel(
    const float* __restrict__ x, const float* __restrict__ dy, const float* __restrict__ w,
    const float* __restrict__ mean, const float* __restrict__ rstd, float* __restrict__ dx,
    float* __restrict__ partial, int n, int rows, int64_t ldx, int64_t lddy, int64_t lddx,
    int groups) {
  __shared__ float2 red[THREADS / 32];
  const int t = threadIdx.x, lane = t & 31, wid = t >> 5;
  const int g = blockIdx.x;
  const int64_t r0 = (int64_t)rows * g / groups, r1 = (int64_t)rows * (g + 1) / groups;
  const float inv_n = 1.0f / (float)n;
  float wv[NV * 4], dwa[NV * 4], dba[NV * 4];
  load_row<THREADS, NV, true>(w, n, 0.f, wv);
#pragma unroll
  for (int i = 0; i < NV * 4; ++i) dwa[i] = dba[i] = 0.f;
  for (int64_t row = r0; row < r1; ++row) {
    float xv[NV * 4], gv[NV * 4];
    load_row<THREADS, NV, true>(x + row * ldx, n, 0.f, xv);
    load_row<THREADS, NV, true>(dy + row * lddy, n, 0.f, gv);
    const float mu = __ldg(mean + row), rs = __ldg(rstd + row);
    float s1 = 0.f, s2 = 0.f;
#pragma unroll
    for (int i = 0; i < NV * 4; ++i) {
      const float xh = (xv[i] - mu) * rs;  // padding slots: dy = 0 there, so they add nothing
      dwa[i] = fmaf(gv[i], xh, dwa[i]);
      dba[i] += gv[i];
      const float gw = gv[i] * wv[i];
      xv[i] = xh;
      gv[i] = gw;
      s1 = fmaf(gw, xh, s1);
      s2 += gw;
    }
    // One CTA reduction of the pair (s1, s2).
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      s1 += __shfl_xor_sync(0xffffffffu, s1, o);
      s2 += __shfl_xor_sync(0xffffffffu, s2, o);
    }
    if (lane == 0) red[wid] = make_float2(s1, s2);
    __syncthreads();
    float2 tot = lane < THREADS / 32 ? red[lane] : make_float2(0.f, 0.f);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      tot.x += __shfl_xor_sync(0xffffffffu, tot.x, o);
      tot.y += __shfl_xor_sync(0xffffffffu, tot.y, o);
    }
    __syncthreads();
    const float c1 = tot.x * inv_n, c2 = tot.y * inv_n;
#pragma unroll
    for (int i = 0; i < NV * 4; ++i) xv[i] = (gv[i] - fmaf(xv[i], c1, c2)) * rs;
    store_row<THREADS, NV, true>(dx + row * lddx, n, xv);
  }
  store_row<THREADS, NV, true>(partial + (int64_t)g * n, n, dwa);
  store_row<THREADS, NV, true>(partial + (int64_t)(groups + g) * n, n, dba);
}

// dW[c] = sum_g partial[g][c], dB[c] = sum_g partial[groups + g][c].
__global__ void __launch_bounds__(256) layernorm_bwd_dwdb_kernel(const float* __restrict__ partial,
                                                                 float* __restrict__ dw,
                                                                 float* __restrict__ db, int n,
                                                                 int groups) {
  const int64_t c = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (c >= 2 * (int64_t)n) return;
  const bool is_db = c >= n;
  const int col = (int)(is_db ? c - n : c);
  const float* p = partial + (is_db ? (int64_t)groups * n : 0) + col;
  float s0 = 0.f, s1 = 0.f, s2 = 0.f, s3 = 0.f;
  int gi = 0;
  for (; gi + 3 < groups; gi += 4) {
    s0 += p[(int64_t)(gi + 0) * n];
    s1 += p[(int64_t)(gi + 1) * n];
    s2 += p[(int64_t)(gi + 2) * n];
    s3 += p[(int64_t)(gi + 3) * n];
  }
  for (; gi < groups; ++gi) s0 += p[(int64_t)gi * n];
  (is_db ? db : dw)[col] = (s0 + s1) + (s2 + s3);
}

int layernorm_bwd_groups(int n, int rows, int sm_count) {
  if (n <= 0 || rows <= 0) return 1;
  // Two resident CTAs per SM; no more groups than rows.
  return std::max(1, std::min(rows, 2 * sm_count));
}

int launch_layernorm_bwd(const float* x, const float* dy, const float* w, const float* mean,
                         const float* rstd, float* dx, float* dw, float* db, int n, int rows,
                         int64_t ldx, int64_t lddy, int64_t lddx, float* partial, int groups,
                         cudaStream_t st) {
  if (n <= 0 || rows < 0 || groups < 1) return set_error(CTB_ERR_SHAPE, "layernorm_bwd: bad sizes");
  if (n > 16384)
    return set_error(CTB_ERR_SHAPE, "layernorm_bwd: rows longer than 16384 elements are not supported");
  if (!x || !dy || !w || !mean || !rstd || !dx || !dw || !db || !partial)
    return set_error(CTB_ERR_ARG, "layernorm_bwd: NULL pointer");
  if (n % 4 || ldx % 4 || lddy % 4 || lddx % 4 || !aligned16(x) || !aligned16(dy) ||
      !aligned16(w) || !aligned16(dx) || !aligned16(partial))
    return set_error(CTB_ERR_LAYOUT,
                     "layernorm_bwd: n and row strides must be multiples of 4, pointers 16-byte aligned");
  if (rows == 0) {
    CTB_CUDA_CHECK(cudaMemsetAsync(dw, 0, sizeof(float) * n, st));
    CTB_CUDA_CHECK(cudaMemsetAsync(db, 0, sizeof(float) * n, st));
    return CTB_OK;
  }
  groups = std::min(groups, rows);
  if (n <= 2048)
    layernorm_bwd_dx_kernel<512, 1><<<groups, 512, 0, st>>>(x, dy, w, mean, rstd, dx, partial, n,
                                                           rows, ldx, lddy, lddx, groups);
  else if (n <= 4096)
    layernorm_bwd_dx_kernel<512, 2><<<groups, 512, 0, st>>>(x, dy, w, mean, rstd, dx, partial, n,
                                                           rows, ldx, lddy, lddx, groups);
  else if (n <= 8192)
    layernorm_bwd_dx_kernel<512, 4><<<groups, 512, 0, st>>>(x, dy, w, mean, rstd, dx, partial, n,
                                                           rows, ldx, lddy, lddx, groups);
  else
    layernorm_bwd_dx_kernel<1024, 4><<<groups, 1024, 0, st>>>(x, dy, w, mean, rstd, dx, partial,
                                                             n, rows, ldx, lddy, lddx, groups);
  if (int rc = launch_status("layernorm_bwd_dx_kernel")) return rc;
  layernorm_bwd_dwdb_kernel<<<(2 * n + 255) / 256, 256, 0, st>>>(partial, dw, db, n, groups);
  return launch_status("layernorm_bwd_dwdb_kernel");
}

}  // namespace ctb

using namespace ctb;

extern "C" int ctb_layernorm_bwd_groups(int32_t n, int32_t rows) {
  clear_error();
  DeviceProps p;
  if (int rc = current_props(&p)) return -1;
  return layernorm_bwd_groups(n, rows, p.sm_count);
}

extern "C" int ctb_layernorm_bwd_f32(const float* x, const float* dy, const float* w,
                                     const float* mean, const float* rstd, float* dx, float* dw,
                                     float* db, int32_t n, int32_t rows, int64_t ldx,
                                     int64_t lddy, int64_t lddx, float* partial, int32_t groups,
                                     void* stream) {
  clear_error();
  DeviceProps p;
  if (int rc = current_props(&p)) return rc;
  return launch_layernorm_bwd(x, dy, w, mean, rstd, dx, dw, db, n, rows, ldx, lddy, lddx, partial,
                              groups, static_cast<cudaStream_t>(stream));
}

// =============================================================================
// Allocation-free LayerNorm backward.
//
// Some callers cannot allocate device memory at the point where they need a
// backward pass: a process that reserved its whole device-memory budget up
// front for its own pool, or Julia code running where CUDA.jl's allocator
// (which may trigger a garbage collection) must not be entered. For them this
// entry point takes the dW/dB partial workspace from a fixed array compiled
// into the library instead of from the caller.
//
// The array below is LNBWD_NOALLOC_FLOATS floats (4 MiB) and lives on every
// GPU that loads the library until the process exits. In host code its name
// is only a host-side stand-in, so its device address is fetched per device
// with cudaGetSymbolAddress on the first call made on that device (with that
// device current); make that first call before any stream capture. All calls
// share the one array: two calls whose kernels overlap on a GPU (different
// streams, or different host threads on one device) race and corrupt each
// other's dW/dB. Each call writes every partial row it later reads, so no
// clearing is needed between calls.
// =============================================================================
namespace ctb {

constexpr int64_t LNBWD_NOALLOC_FLOATS = 1 << 20;  // 4 MiB
static __device__ __align__(256) float g_lnbwd_noalloc_scratch[LNBWD_NOALLOC_FLOATS];

static std::mutex g_noalloc_mu;
static float* g_noalloc_ptr[64];

static int noalloc_scratch(float** out) {
  int dev = 0;
  CTB_CUDA_CHECK(cudaGetDevice(&dev));
  if (dev < 0 || dev >= 64) return set_error(CTB_ERR_NO_DEVICE, "device ordinal out of range");
  std::lock_guard<std::mutex> lk(g_noalloc_mu);
  if (!g_noalloc_ptr[dev]) {
    void* p = nullptr;
    cudaError_t e = cudaGetSymbolAddress(&p, g_lnbwd_noalloc_scratch);
    if (e != cudaSuccess) return cuda_fail(e, "cudaGetSymbolAddress(layernorm_bwd scratch)");
    g_noalloc_ptr[dev] = static_cast<float*>(p);
  }
  *out = g_noalloc_ptr[dev];
  return CTB_OK;
}

}  // namespace ctb

extern "C" int ctb_layernorm_bwd_f32_noalloc(const float* x, const float* dy, const float* w,
                                             const float* mean, const float* rstd, float* dx,
                                             float* dw, float* db, int32_t n, int32_t rows,
                                             int64_t ldx, int64_t lddy, int64_t lddx,
                                             int32_t groups, void* stream) {
  clear_error();
  DeviceProps p;
  if (int rc = current_props(&p)) return rc;
  if (n <= 0 || rows < 0) return set_error(CTB_ERR_SHAPE, "layernorm_bwd_noalloc: bad sizes");
  if (2 * (int64_t)n > LNBWD_NOALLOC_FLOATS)
    return set_error(CTB_ERR_SHAPE, "layernorm_bwd_noalloc: n too large for the built-in scratch");
  const int64_t cap = LNBWD_NOALLOC_FLOATS / (2 * (int64_t)n);  // partial rows that fit
  if (groups <= 0) groups = (int32_t)std::min<int64_t>(layernorm_bwd_groups(n, rows, p.sm_count), cap);
  if ((int64_t)std::min(groups, std::max(rows, 1)) * 2 * n > LNBWD_NOALLOC_FLOATS)
    return set_error(CTB_ERR_SHAPE,
                     "layernorm_bwd_noalloc: 2 x groups x n exceeds the built-in scratch of " +
                         std::to_string(LNBWD_NOALLOC_FLOATS) + " floats");
  float* scratch = nullptr;
  if (int rc = noalloc_scratch(&scratch)) return rc;
  return launch_layernorm_bwd(x, dy, w, mean, rstd, dx, dw, db, n, rows, ldx, lddy, lddx, scratch,
                              groups, static_cast<cudaStream_t>(stream));
}

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
#include "sm100_ptx.cuh"

#include <algorithm>
#include <mutex>

namespace ctb {

// Rows of x and dy stream into a STAGES-deep shared-memory ring through
// 1-D bulk copies (cp.async.bulk, completion counted on an mbarrier per
// stage), so the next rows are in flight while the current one is reduced.
// w is read through the read-only path; dW/dB partials stay in registers.
constexpr unsigned LNBWD_ERR_BIT = 4u;

// Ring depth and CTAs per SM per row-length class. Measured at 16384 x 4096:
// one CTA per SM with a 4-stage ring (128 KB of x/dy in flight per SM, and
// half the dW/dB partial rows of two CTAs per SM) is fastest.
//   n <= 2048  (512 threads, 1 float4):  2 stages x 16 KB, 4 CTAs per SM
//   n <= 4096  (512 threads, 2 float4):  4 stages x 32 KB, 1 CTA per SM
//   n <= 8192  (512 threads, 4 float4):  3 stages x 64 KB, 1 CTA per SM
//   n <= 16384 (1024 threads, 4 float4): 1 stage of 128 KB, 1 CTA per SM
__host__ __device__ constexpr int lnbwd_stages(int threads, int nv) {
  return threads >= 1024 ? 1 : (nv >= 4 ? 3 : (nv >= 2 ? 4 : 2));
}
__host__ __device__ constexpr int lnbwd_ctas_per_sm(int threads, int nv) {
  return threads >= 1024 ? 1 : (nv >= 2 ? 1 : 4);
}
__host__ __device__ constexpr int lnbwd_smem_bytes(int threads, int nv) {
  return lnbwd_stages(threads, nv) * 2 * threads * nv * 16 + 64;
}

__device__ __forceinline__ void bulk_load(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::
          "r"(sm100::smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(src)), "r"(bytes), "r"(sm100::smem_u32(bar))
      : "memory");
}

template <int THREADS, int NV>
__global__ void __launch_bounds__(THREADS, lnbwd_ctas_per_sm(THREADS, NV))
    layernorm_bwd_dx_kernel(const float* __restrict__ x, const float* __restrict__ dy,
                            const float* __restrict__ w, const float* __restrict__ mean,
                            const float* __restrict__ rstd, float* __restrict__ dx,
                            float* __restrict__ partial, int n, int rows, int64_t ldx,
                            int64_t lddy, int64_t lddx, int groups) {
  using namespace sm100;
  constexpr int ROWF = THREADS * NV * 4;  // floats per staged row (n <= ROWF)
  constexpr int LNBWD_STAGES = lnbwd_stages(THREADS, NV);
  extern __shared__ __align__(128) float ring[];  // [STAGES][2][ROWF], then barriers
  uint64_t* full = reinterpret_cast<uint64_t*>(ring + LNBWD_STAGES * 2 * ROWF);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(full + LNBWD_STAGES);
  __shared__ float2 red[THREADS / 32];
  const int t = threadIdx.x, lane = t & 31, wid = t >> 5;
  const int g = blockIdx.x;
  const int64_t r0 = (int64_t)rows * g / groups, r1 = (int64_t)rows * (g + 1) / groups;
  const int nrows = (int)(r1 - r0);
  const uint32_t row_bytes = (uint32_t)n * 4;
  const float inv_n = 1.0f / (float)n;

  if (t == 0) {
    for (int s = 0; s < LNBWD_STAGES; ++s) mbar_init(&full[s], 1);
    *abort_flag = 0;
    fence_mbar_init();
    for (int i = 0; i < LNBWD_STAGES && i < nrows; ++i) {
      mbar_arrive_expect_tx(&full[i], 2 * row_bytes);
      bulk_load(ring + (i * 2) * ROWF, x + (r0 + i) * ldx, row_bytes, &full[i]);
      bulk_load(ring + (i * 2 + 1) * ROWF, dy + (r0 + i) * lddy, row_bytes, &full[i]);
    }
  }
  __syncthreads();

  float dwa[NV * 4], dba[NV * 4];
#pragma unroll
  for (int i = 0; i < NV * 4; ++i) dwa[i] = dba[i] = 0.f;
  for (int i = 0; i < nrows; ++i) {
    const int s = i % LNBWD_STAGES;
    if (!mbar_wait_bounded(&full[s], (i / LNBWD_STAGES) & 1, abort_flag, LNBWD_ERR_BIT)) return;
    const int64_t row = r0 + i;
    const float* xs = ring + (s * 2) * ROWF;
    const float* gs = ring + (s * 2 + 1) * ROWF;
    float xv[NV * 4], gv[NV * 4];
#pragma unroll
    for (int k = 0; k < NV; ++k) {
      const int idx0 = (k * THREADS + t) * 4;
      float4 a = make_float4(0.f, 0.f, 0.f, 0.f), b = a;
      if (idx0 < n) {
        a = *reinterpret_cast<const float4*>(xs + idx0);
        b = *reinterpret_cast<const float4*>(gs + idx0);
      }
      xv[4 * k] = a.x; xv[4 * k + 1] = a.y; xv[4 * k + 2] = a.z; xv[4 * k + 3] = a.w;
      gv[4 * k] = b.x; gv[4 * k + 1] = b.y; gv[4 * k + 2] = b.z; gv[4 * k + 3] = b.w;
    }
    const float mu = __ldg(mean + row), rs = __ldg(rstd + row);
    float s1 = 0.f, s2 = 0.f;
#pragma unroll
    for (int k = 0; k < NV; ++k) {
      const int idx0 = (k * THREADS + t) * 4;
      const float4 wq = idx0 < n ? __ldg(reinterpret_cast<const float4*>(w + idx0))
                                 : make_float4(0.f, 0.f, 0.f, 0.f);
      const float wk[4] = {wq.x, wq.y, wq.z, wq.w};
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int j = 4 * k + e;
        const float xh = (xv[j] - mu) * rs;  // padding slots: dy = 0 there, so they add nothing
        dwa[j] = fmaf(gv[j], xh, dwa[j]);
        dba[j] += gv[j];
        const float gw = gv[j] * wk[e];
        xv[j] = xh;
        gv[j] = gw;
        s1 = fmaf(gw, xh, s1);
        s2 += gw;
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      s1 += __shfl_xor_sync(0xffffffffu, s1, o);
      s2 += __shfl_xor_sync(0xffffffffu, s2, o);
    }
    if (lane == 0) red[wid] = make_float2(s1, s2);
    __syncthreads();  // every thread has also finished reading stage s
    if (t == 0 && i + LNBWD_STAGES < nrows) {
      // Order this CTA's generic-proxy reads of the stage before the refill.
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      mbar_arrive_expect_tx(&full[s], 2 * row_bytes);
      bulk_load(ring + (s * 2) * ROWF, x + (row + LNBWD_STAGES) * ldx, row_bytes, &full[s]);
      bulk_load(ring + (s * 2 + 1) * ROWF, dy + (row + LNBWD_STAGES) * lddy, row_bytes, &full[s]);
    }
    float2 tot = lane < THREADS / 32 ? red[lane] : make_float2(0.f, 0.f);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      tot.x += __shfl_xor_sync(0xffffffffu, tot.x, o);
      tot.y += __shfl_xor_sync(0xffffffffu, tot.y, o);
    }
    __syncthreads();
    const float c1 = tot.x * inv_n, c2 = tot.y * inv_n;
#pragma unroll
    for (int j = 0; j < NV * 4; ++j) xv[j] = (gv[j] - fmaf(xv[j], c1, c2)) * rs;
    store_row<THREADS, NV, true>(dx + row * lddx, n, xv);
  }
  store_row<THREADS, NV, true>(partial + (int64_t)g * n, n, dwa);
  store_row<THREADS, NV, true>(partial + (int64_t)(groups + g) * n, n, dba);
}

// dW[c] = sum_g partial[g][c], dB[c] = sum_g partial[groups + g][c].
// A CTA folds 128 columns (32 threads x float4) with 16 slices of the group
// dimension in parallel, then combines the slices through shared memory.
constexpr int FOLD_SLICES = 16;
__global__ void __launch_bounds__(32 * FOLD_SLICES) layernorm_bwd_dwdb_kernel(
    const float* __restrict__ partial, float* __restrict__ dw, float* __restrict__ db, int n,
    int groups) {
  __shared__ float4 part[FOLD_SLICES][32];
  const int lane = threadIdx.x & 31, slice = threadIdx.x >> 5;
  const int64_t c4 = (int64_t)blockIdx.x * 32 + lane;  // float4 column over [dW | dB]
  const int64_t total4 = (2 * (int64_t)n) / 4;
  float4 a = make_float4(0.f, 0.f, 0.f, 0.f), b = a;
  if (c4 < total4) {
    const bool is_db = c4 >= n / 4;
    const int64_t col4 = is_db ? c4 - n / 4 : c4;
    const float4* p = reinterpret_cast<const float4*>(partial + (is_db ? (int64_t)groups * n : 0)) + col4;
    const int64_t rs = n / 4;
    int gi = slice;
    for (; gi + FOLD_SLICES < groups; gi += 2 * FOLD_SLICES) {
      const float4 u = p[gi * rs], v = p[(gi + FOLD_SLICES) * rs];
      a.x += u.x; a.y += u.y; a.z += u.z; a.w += u.w;
      b.x += v.x; b.y += v.y; b.z += v.z; b.w += v.w;
    }
    if (gi < groups) {
      const float4 u = p[gi * rs];
      a.x += u.x; a.y += u.y; a.z += u.z; a.w += u.w;
    }
  }
  a.x += b.x; a.y += b.y; a.z += b.z; a.w += b.w;
  part[slice][lane] = a;
  __syncthreads();
  if (slice == 0 && c4 < total4) {
#pragma unroll
    for (int k = 1; k < FOLD_SLICES; ++k) {
      const float4 u = part[k][lane];
      a.x += u.x; a.y += u.y; a.z += u.z; a.w += u.w;
    }
    const bool is_db = c4 >= n / 4;
    float* out = is_db ? db + (c4 - n / 4) * 4 : dw + c4 * 4;
    *reinterpret_cast<float4*>(out) = a;
  }
}

int layernorm_bwd_take_device_error(unsigned int* out) { return take_device_error(out); }

int layernorm_bwd_groups(int n, int rows, int sm_count) {
  if (n <= 0 || rows <= 0) return 1;
  const int per_sm = n <= 2048 ? lnbwd_ctas_per_sm(512, 1)
                     : n <= 4096 ? lnbwd_ctas_per_sm(512, 2)
                     : n <= 8192 ? lnbwd_ctas_per_sm(512, 4)
                                 : lnbwd_ctas_per_sm(1024, 4);
  // One wave of resident CTAs; no more groups than rows.
  return std::max(1, std::min(rows, per_sm * sm_count));
}

template <int THREADS, int NV>
static int lnbwd_dx_launch(const float* x, const float* dy, const float* w, const float* mean,
                           const float* rstd, float* dx, float* partial, int n, int rows,
                           int64_t ldx, int64_t lddy, int64_t lddx, int groups, cudaStream_t st) {
  constexpr int smem = lnbwd_smem_bytes(THREADS, NV);
  if (smem > 48 * 1024)
    CTB_CUDA_CHECK(cudaFuncSetAttribute(layernorm_bwd_dx_kernel<THREADS, NV>,
                                        cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
  layernorm_bwd_dx_kernel<THREADS, NV><<<groups, THREADS, smem, st>>>(
      x, dy, w, mean, rstd, dx, partial, n, rows, ldx, lddy, lddx, groups);
  return launch_status("layernorm_bwd_dx_kernel");
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
      !aligned16(w) || !aligned16(dx) || !aligned16(partial) || !aligned16(dw) || !aligned16(db))
    return set_error(CTB_ERR_LAYOUT,
                     "layernorm_bwd: n and row strides must be multiples of 4, pointers 16-byte aligned");
  if (rows == 0) {
    CTB_CUDA_CHECK(cudaMemsetAsync(dw, 0, sizeof(float) * n, st));
    CTB_CUDA_CHECK(cudaMemsetAsync(db, 0, sizeof(float) * n, st));
    return CTB_OK;
  }
  groups = std::min(groups, rows);
  int rc;
  if (n <= 2048)
    rc = lnbwd_dx_launch<512, 1>(x, dy, w, mean, rstd, dx, partial, n, rows, ldx, lddy, lddx, groups, st);
  else if (n <= 4096)
    rc = lnbwd_dx_launch<512, 2>(x, dy, w, mean, rstd, dx, partial, n, rows, ldx, lddy, lddx, groups, st);
  else if (n <= 8192)
    rc = lnbwd_dx_launch<512, 4>(x, dy, w, mean, rstd, dx, partial, n, rows, ldx, lddy, lddx, groups, st);
  else
    rc = lnbwd_dx_launch<1024, 4>(x, dy, w, mean, rstd, dx, partial, n, rows, ldx, lddy, lddx, groups, st);
  if (rc) return rc;
  layernorm_bwd_dwdb_kernel<<<(int)((2 * (int64_t)n / 4 + 31) / 32), 32 * FOLD_SLICES, 0, st>>>(
      partial, dw, db, n, groups);
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
// The array below is LNBWD_NOALLOC_FLOATS floats (8 MiB) and lives on every
// GPU that loads the library until the process exits. In host code its name
// is only a host-side stand-in, so its device address is fetched per device
// with cudaGetSymbolAddress on the first call made on that device (with that
// device current); make that first call before any stream capture. The
// address is remembered together with the CUDA context's unique ID, so after
// a cudaDeviceReset (a new primary context, the module loaded again) the next
// call looks it up again instead of using a stale address. All calls share
// the one array: two calls whose kernels overlap on a GPU (different streams,
// or different host threads on one device) race and corrupt each other's
// dW/dB. Each call writes every partial row it later reads, so no clearing
// is needed between calls.
// =============================================================================
namespace ctb {

constexpr int64_t LNBWD_NOALLOC_FLOATS = 1 << 21;  // 8 MiB
static __device__ __align__(256) float g_lnbwd_noalloc_scratch[LNBWD_NOALLOC_FLOATS];

static std::mutex g_noalloc_mu;
static float* g_noalloc_ptr[64];
static unsigned long long g_noalloc_ctx[64];  // context ID the address belongs to

static int noalloc_scratch(float** out) {
  int dev = 0;
  CTB_CUDA_CHECK(cudaGetDevice(&dev));
  if (dev < 0 || dev >= 64) return set_error(CTB_ERR_NO_DEVICE, "device ordinal out of range");
  unsigned long long ctx = 0;
  if (int rc = current_context_id(&ctx)) return rc;
  std::lock_guard<std::mutex> lk(g_noalloc_mu);
  if (!g_noalloc_ptr[dev] || g_noalloc_ctx[dev] != ctx) {
    void* p = nullptr;
    cudaError_t e = cudaGetSymbolAddress(&p, g_lnbwd_noalloc_scratch);
    if (e != cudaSuccess) return cuda_fail(e, "cudaGetSymbolAddress(layernorm_bwd scratch)");
    g_noalloc_ptr[dev] = static_cast<float*>(p);
    g_noalloc_ctx[dev] = ctx;
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

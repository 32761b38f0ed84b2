// HBM-bound kernels of libcutile_b200.so: vadd, rowsum, softmax, layernorm-fwd.
//
// Design (B200, 148 SMs, HBM3e): every kernel moves its bytes once — 128-bit
// loads with L1 no-allocate, evict-first stores, rows held in registers
// between the reduction and the write-back — and reduces with warp shuffles
// plus one shared-memory hop per CTA. Row kernels size their grid to the
// resident-CTA capacity (SM count x CTAs per SM) and stride over rows.
#include "ctb_common.cuh"

#include <algorithm>
#include <type_traits>

namespace ctb {

// =============================================================================
// vadd: c = a + b (reference: test/runtests.jl:31-47, bench/bench.jl:51-57)
// =============================================================================
// Round-to-nearest adds that the compiler may not contract or flush.
__device__ __forceinline__ float add_rn(float a, float b) { return __fadd_rn(a, b); }
__device__ __forceinline__ double add_rn(double a, double b) { return __dadd_rn(a, b); }
__device__ __forceinline__ __half add_rn(__half a, __half b) { return __hadd(a, b); }

// Contiguous path: 16-byte vectors, UNROLL independent vectors per thread per
// trip so that 2*UNROLL loads are in flight before the first add.
template <typename T, int UNROLL>
__global__ void __launch_bounds__(256) vadd_vec_kernel(const T* __restrict__ a,
                                                       const T* __restrict__ b,
                                                       T* __restrict__ c, int64_t nvec) {
  constexpr int E = 16 / sizeof(T);
  union V {
    uint4 u;
    T e[E];
  };
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  const uint4* a4 = reinterpret_cast<const uint4*>(a);
  const uint4* b4 = reinterpret_cast<const uint4*>(b);
  uint4* c4 = reinterpret_cast<uint4*>(c);
  for (; i + (UNROLL - 1) * stride < nvec; i += UNROLL * stride) {
    V va[UNROLL], vb[UNROLL];
#pragma unroll
    for (int u = 0; u < UNROLL; ++u) {
      va[u].u = __ldcs(a4 + i + u * stride);
      vb[u].u = __ldcs(b4 + i + u * stride);
    }
#pragma unroll
    for (int u = 0; u < UNROLL; ++u) {
#pragma unroll
      for (int e = 0; e < E; ++e) va[u].e[e] = add_rn(va[u].e[e], vb[u].e[e]);
      __stcs(c4 + i + u * stride, va[u].u);
    }
  }
  for (; i < nvec; i += stride) {
    V va, vb;
    va.u = __ldcs(a4 + i);
    vb.u = __ldcs(b4 + i);
#pragma unroll
    for (int e = 0; e < E; ++e) va.e[e] = add_rn(va.e[e], vb.e[e]);
    __stcs(c4 + i, va.u);
  }
}

// Strided / unaligned / tail path.
template <typename T>
__global__ void __launch_bounds__(256) vadd_strided_kernel(const T* __restrict__ a,
                                                           const T* __restrict__ b,
                                                           T* __restrict__ c, int64_t begin,
                                                           int64_t n, int64_t sa, int64_t sb,
                                                           int64_t sc) {
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t i = begin + (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride)
    c[i * sc] = add_rn(a[i * sa], b[i * sb]);
}

template <typename T>
static int launch_vadd(const T* a, const T* b, T* c, int64_t n, int64_t sa, int64_t sb,
                       int64_t sc, cudaStream_t st) {
  DeviceProps p;
  if (int rc = current_props(&p)) return rc;
  if (n == 0) return CTB_OK;
  constexpr int E = 16 / sizeof(T);
  int64_t done = 0;
  if (sa == 1 && sb == 1 && sc == 1 && aligned16(a) && aligned16(b) && aligned16(c)) {
    const int64_t nvec = n / E;
    if (nvec > 0) {
      // 8 resident CTAs of 256 threads per SM fill the SM's 2048 threads.
      const int64_t want = (nvec + 255) / 256;
      const int grid = (int)std::min<int64_t>(want, (int64_t)p.sm_count * 8);
      vadd_vec_kernel<T, 4><<<grid, 256, 0, st>>>(a, b, c, nvec);
      if (int rc = launch_status("vadd_vec_kernel")) return rc;
    }
    done = nvec * E;
  }
  if (done < n) {
    const int64_t rem = n - done;
    const int grid = (int)std::min<int64_t>((rem + 255) / 256, (int64_t)p.sm_count * 8);
    vadd_strided_kernel<T><<<grid, 256, 0, st>>>(a, b, c, done, n, sa, sb, sc);
    if (int rc = launch_status("vadd_strided_kernel")) return rc;
  }
  return CTB_OK;
}

// =============================================================================
// rowsum: out[i] = sum_j a[i, j]   (reference: test/runtests.jl:50-56,
// bench/rocm_compare.jl:68-73; the emitter's reduce keeps dim 2 as size 1,
// src/emitter.jl:1046-1073)
// =============================================================================
// Julia column-major a (s_i == 1): consecutive threads own consecutive rows
// (one float4 = 4 rows each), RS_Y thread rows split the j range, shared
// memory folds the RS_Y partial sums. A CTA of 512 threads covers RS_X x 4
// rows; the launcher takes the widest RS_X (64, 32, 16, 8) that still gives
// two CTAs per SM, so a short matrix (a shard of the job) spreads over every
// SM. Measured (B200, m x 512, GB/s): m = 131072: RS_X 64 6003, 32 5978, 16
// 5781; m = 65536: 4950 / 5301 / 5083; m = 32768: 2963 / 3793 / 4054;
// m = 16384: 1521 / 2314 / 2714.
template <int RS_X>
__global__ void __launch_bounds__(512) rowsum_rows_contig_kernel(
    const float* __restrict__ a, float* __restrict__ out, int m, int n, int64_t sj,
    int64_t so) {
  constexpr int RS_Y = 512 / RS_X;
  __shared__ float4 part[RS_Y][RS_X];
  const int tx = threadIdx.x % RS_X, ty = threadIdx.x / RS_X;
  const int64_t row0 = (int64_t)blockIdx.x * (RS_X * 4) + tx * 4;
  float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
  if (row0 < m) {
    const float* p = a + row0;
    int j = ty;
    // 8 independent loads in flight per thread per trip.
    for (; j + 7 * RS_Y < n; j += 8 * RS_Y) {
      float4 v[8];
#pragma unroll
      for (int u = 0; u < 8; ++u) v[u] = ld_stream_f4(p + (int64_t)(j + u * RS_Y) * sj);
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        acc.x += v[u].x;
        acc.y += v[u].y;
        acc.z += v[u].z;
        acc.w += v[u].w;
      }
    }
    for (; j < n; j += RS_Y) {
      float4 v = ld_stream_f4(p + (int64_t)j * sj);
      acc.x += v.x;
      acc.y += v.y;
      acc.z += v.z;
      acc.w += v.w;
    }
  }
  part[ty][tx] = acc;
  __syncthreads();
  if (ty == 0 && row0 < m) {
#pragma unroll
    for (int y = 1; y < RS_Y; ++y) {
      float4 v = part[y][tx];
      acc.x += v.x;
      acc.y += v.y;
      acc.z += v.z;
      acc.w += v.w;
    }
    out[(row0 + 0) * so] = acc.x;
    out[(row0 + 1) * so] = acc.y;
    out[(row0 + 2) * so] = acc.z;
    out[(row0 + 3) * so] = acc.w;
  }
}

// Row-major a (s_j == 1, rows of n contiguous floats): one warp per row.
template <bool VEC>
__global__ void __launch_bounds__(256) rowsum_cols_contig_kernel(const float* __restrict__ a,
                                                                 float* __restrict__ out, int m,
                                                                 int n, int64_t si, int64_t so) {
  const int lane = threadIdx.x & 31;
  const int64_t warps = (int64_t)gridDim.x * (blockDim.x / 32);
  for (int64_t r = (int64_t)blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32; r < m;
       r += warps) {
    const float* p = a + r * si;
    float s = 0.f;
    if (VEC) {
      const int n4 = n / 4;
      for (int k = lane; k < n4; k += 32) {
        float4 v = ld_stream_f4(p + 4 * k);
        s += (v.x + v.y) + (v.z + v.w);
      }
      for (int k = 4 * n4 + lane; k < n; k += 32) s += p[k];
    } else {
      for (int k = lane; k < n; k += 32) s += p[k];
    }
    s = warp_sum(s);
    if (lane == 0) out[r * so] = s;
  }
}

// Any strides: one thread per row (correct, not fast).
__global__ void __launch_bounds__(256) rowsum_generic_kernel(const float* __restrict__ a,
                                                             float* __restrict__ out, int m,
                                                             int n, int64_t si, int64_t sj,
                                                             int64_t so) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= m) return;
  float s = 0.f;
  for (int j = 0; j < n; ++j) s += a[i * si + (int64_t)j * sj];
  out[i * so] = s;
}

static int launch_rowsum(const float* a, float* out, int m, int n, int64_t si, int64_t sj,
                         int64_t so, cudaStream_t st) {
  DeviceProps p;
  if (int rc = current_props(&p)) return rc;
  if (m == 0) return CTB_OK;
  if (si == 1 && m % 4 == 0 && sj % 4 == 0 && aligned16(a)) {
    auto go = [&](auto rsx) {
      constexpr int X = decltype(rsx)::value;
      rowsum_rows_contig_kernel<X><<<(m + X * 4 - 1) / (X * 4), 512, 0, st>>>(a, out, m, n, sj, so);
    };
    const int64_t want = 2 * (int64_t)p.sm_count;  // CTAs
    if ((m + 255) / 256 >= want) go(std::integral_constant<int, 64>{});
    else if ((m + 127) / 128 >= want) go(std::integral_constant<int, 32>{});
    else if ((m + 63) / 64 >= want) go(std::integral_constant<int, 16>{});
    else go(std::integral_constant<int, 8>{});
    return launch_status("rowsum_rows_contig_kernel");
  }
  if (sj == 1) {
    const bool vec = aligned16(a) && si % 4 == 0;
    const int grid = (int)std::min<int64_t>(((int64_t)m + 7) / 8, (int64_t)p.sm_count * 8);
    if (vec)
      rowsum_cols_contig_kernel<true><<<grid, 256, 0, st>>>(a, out, m, n, si, so);
    else
      rowsum_cols_contig_kernel<false><<<grid, 256, 0, st>>>(a, out, m, n, si, so);
    return launch_status("rowsum_cols_contig_kernel");
  }
  rowsum_generic_kernel<<<(m + 255) / 256, 256, 0, st>>>(a, out, m, n, si, sj, so);
  return launch_status("rowsum_generic_kernel");
}

// =============================================================================
// softmax over contiguous vectors (reference: test/runtests.jl:102-118,
// bench/bench.jl:147-164): NegInf padding, max-subtracted exp, sum, divide.
// =============================================================================
template <int THREADS, int NV, bool VEC>
__global__ void __launch_bounds__(THREADS) softmax_reg_kernel(const float* __restrict__ x,
                                                              float* __restrict__ y, int len,
                                                              int count, int64_t ldx,
                                                              int64_t ldy) {
  __shared__ float red[THREADS / 32];
  for (int64_t row = blockIdx.x; row < count; row += gridDim.x) {
    float v[NV * 4];
    load_row<THREADS, NV, VEC>(x + row * ldx, len, -INFINITY, v);
    float m = -INFINITY;
#pragma unroll
    for (int i = 0; i < NV * 4; ++i) m = fmaxf(m, v[i]);
    m = block_reduce<THREADS / 32, true>(m, red);
    float s = 0.f;
#pragma unroll
    for (int i = 0; i < NV * 4; ++i) {
      v[i] = expf(v[i] - m);  // padding: exp(-inf) = 0
      s += v[i];
    }
    s = block_reduce<THREADS / 32, false>(s, red);
    const float inv = 1.0f / s;
#pragma unroll
    for (int i = 0; i < NV * 4; ++i) v[i] *= inv;
    store_row<THREADS, NV, VEC>(y + row * ldy, len, v);
  }
}

// Vectors longer than the register-resident limit: pass 1 computes the
// running (max, sum) online, pass 2 re-reads, normalises and writes.
constexpr int SMX_LONG_THREADS = 1024;
__global__ void __launch_bounds__(SMX_LONG_THREADS) softmax_long_kernel(
    const float* __restrict__ x, float* __restrict__ y, int len, int count, int64_t ldx,
    int64_t ldy) {
  __shared__ float red[SMX_LONG_THREADS / 32];
  for (int64_t row = blockIdx.x; row < count; row += gridDim.x) {
    const float* xr = x + row * ldx;
    float m = -INFINITY, s = 0.f;
    for (int i = threadIdx.x; i < len; i += SMX_LONG_THREADS) {
      const float xi = xr[i];
      if (xi > m) {
        s = s * expf(m - xi) + 1.f;
        m = xi;
      } else {
        s += expf(xi - m);
      }
    }
    const float gm = block_reduce<SMX_LONG_THREADS / 32, true>(m, red);
    s = (m == -INFINITY) ? 0.f : s * expf(m - gm);
    s = block_reduce<SMX_LONG_THREADS / 32, false>(s, red);
    const float inv = 1.0f / s;
    float* yr = y + row * ldy;
    for (int i = threadIdx.x; i < len; i += SMX_LONG_THREADS) yr[i] = expf(xr[i] - gm) * inv;
  }
}

template <int THREADS, int NV>
static void softmax_reg_launch(const float* x, float* y, int len, int count, int64_t ldx,
                               int64_t ldy, bool vec, cudaStream_t st) {
  if (vec)
    softmax_reg_kernel<THREADS, NV, true><<<count, THREADS, 0, st>>>(x, y, len, count, ldx, ldy);
  else
    softmax_reg_kernel<THREADS, NV, false><<<count, THREADS, 0, st>>>(x, y, len, count, ldx, ldy);
}

static int launch_softmax(const float* x, float* y, int len, int count, int64_t ldx,
                          int64_t ldy, cudaStream_t st) {
  DeviceProps p;
  if (int rc = current_props(&p)) return rc;
  if (count == 0 || len == 0) return CTB_OK;
  const bool vec = len % 4 == 0 && ldx % 4 == 0 && ldy % 4 == 0 && aligned16(x) && aligned16(y);
  if (len <= 512)
    softmax_reg_launch<128, 1>(x, y, len, count, ldx, ldy, vec, st);
  else if (len <= 2048)
    softmax_reg_launch<128, 4>(x, y, len, count, ldx, ldy, vec, st);
  else if (len <= 4096)
    softmax_reg_launch<256, 4>(x, y, len, count, ldx, ldy, vec, st);
  else if (len <= 8192)
    softmax_reg_launch<256, 8>(x, y, len, count, ldx, ldy, vec, st);
  else if (len <= 16384)
    softmax_reg_launch<512, 8>(x, y, len, count, ldx, ldy, vec, st);
  else if (len <= 32768)
    softmax_reg_launch<1024, 8>(x, y, len, count, ldx, ldy, vec, st);
  else {
    const int grid = std::min(count, p.sm_count * 2);
    softmax_long_kernel<<<grid, SMX_LONG_THREADS, 0, st>>>(x, y, len, count, ldx, ldy);
  }
  return launch_status("softmax kernel");
}

// =============================================================================
// layernorm forward (cuTile example layernorm.jl:27; definitions of mean,
// biased variance and rstd as stated in include/cutile_b200.h)
// =============================================================================
// Merge of two partial (mean, M2) pairs over equal counts, each side holding
// half of `total` elements (Chan, Golub and LeVeque 1979, pairwise update):
// mean = (ma + mb) / 2, M2 = M2a + M2b + (mb - ma)^2 * total / 4. The sum is
// written symmetrically so both lanes of an xor-shuffle pair get the same bits.
__device__ __forceinline__ void chan_merge_equal(float& m, float& m2, float mo, float m2o,
                                                 float total) {
  const float d = mo - m;
  m = 0.5f * (m + mo);
  m2 = (m2 + m2o) + d * d * (0.25f * total);
}

// One row per CTA trip. Build-time options (measured in the design notes):
// CTB_LN_WB_REG keeps this thread's gamma/beta columns in registers for the
// whole launch instead of re-reading them through L1 for every row;
// CTB_LN_AHEAD rows are loaded ahead of the row being reduced;
// CTB_LN_FUSED merges (mean, M2) in one block reduction (Chan's update).
#ifndef CTB_LN_WB_REG
#define CTB_LN_WB_REG 0
#endif
#ifndef CTB_LN_AHEAD
#define CTB_LN_AHEAD 1
#endif
#ifndef CTB_LN_FUSED
#define CTB_LN_FUSED 0
#endif
#ifndef CTB_LN_CTA_THREADS
#define CTB_LN_CTA_THREADS 1536  // resident threads per SM the bounds aim at (NV <= 2)
#endif
static_assert(CTB_LN_AHEAD == 1 || CTB_LN_AHEAD == 2, "rows loaded ahead: 1 or 2");
template <int THREADS, int NV, bool VEC>
__global__ void __launch_bounds__(THREADS, (THREADS >= 1024 ? 1 : (NV >= 4 ? 1024 : CTB_LN_CTA_THREADS) / THREADS))
    layernorm_fwd_reg_kernel(
    const float* __restrict__ x, const float* __restrict__ w, const float* __restrict__ b,
    float* __restrict__ y, float* __restrict__ mean, float* __restrict__ rstd, int n, int rows,
    int64_t ldx, int64_t ldy, float eps) {
  constexpr int AHEAD = CTB_LN_AHEAD;
  constexpr bool WB_REG = CTB_LN_WB_REG && VEC;
  __shared__ float red[THREADS / 32];
  __shared__ float2 red2[2][THREADS / 32];  // by row parity: one barrier per row
  const float inv_n = 1.0f / (float)n;
  const int t = threadIdx.x;
  const bool full = CTB_LN_FUSED && VEC && n == THREADS * NV * 4;
  int par = 0;
  float4 wr[WB_REG ? NV : 1], br[WB_REG ? NV : 1];
  if (WB_REG) {
#pragma unroll
    for (int k = 0; k < NV; ++k) {
      const int idx0 = (k * THREADS + t) * 4;
      wr[k] = idx0 < n ? __ldg(reinterpret_cast<const float4*>(w + idx0)) : make_float4(0, 0, 0, 0);
      br[k] = idx0 < n ? __ldg(reinterpret_cast<const float4*>(b + idx0)) : make_float4(0, 0, 0, 0);
    }
  }
  // Software pipeline: the next AHEAD rows' loads are issued before this
  // row's reductions, so AHEAD + 1 rows per CTA are in flight from HBM.
  float nv[AHEAD][NV * 4];
#pragma unroll
  for (int a = 0; a < AHEAD; ++a)
    if (blockIdx.x + (int64_t)a * gridDim.x < rows)
      load_row<THREADS, NV, VEC>(x + (blockIdx.x + (int64_t)a * gridDim.x) * ldx, n, 0.f, nv[a]);
  for (int64_t row = blockIdx.x; row < rows; row += gridDim.x) {
    float v[NV * 4];
#pragma unroll
    for (int i = 0; i < NV * 4; ++i) v[i] = nv[0][i];
#pragma unroll
    for (int a = 0; a + 1 < AHEAD; ++a)
#pragma unroll
      for (int i = 0; i < NV * 4; ++i) nv[a][i] = nv[a + 1][i];
    const int64_t nxt = row + (int64_t)AHEAD * gridDim.x;
    if (nxt < rows) load_row<THREADS, NV, VEC>(x + nxt * ldx, n, 0.f, nv[AHEAD - 1]);
    float mu, var;
    if (full) {
      // Every thread holds NV*4 elements: per-thread (mean, M2), merged
      // pairwise with Chan et al.'s update for equal counts, one barrier.
      float lm = 0.f;
#pragma unroll
      for (int i = 0; i < NV * 4; ++i) lm += v[i];
      lm *= 1.0f / (NV * 4);
      float m2 = 0.f;
#pragma unroll
      for (int i = 0; i < NV * 4; ++i) {
        const float d = v[i] - lm;
        m2 = fmaf(d, d, m2);
      }
      float cnt = NV * 4;  // elements on each side of the next merge
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        chan_merge_equal(lm, m2, __shfl_xor_sync(0xffffffffu, lm, o),
                         __shfl_xor_sync(0xffffffffu, m2, o), cnt * 2.f);
        cnt *= 2.f;
      }
      float2* rb = red2[par];
      if ((t & 31) == 0) rb[t >> 5] = make_float2(lm, m2);
      __syncthreads();
      float2 r = rb[(t & 31) % (THREADS / 32)];
      lm = r.x;
      m2 = r.y;
#pragma unroll
      for (int o = 1; o < THREADS / 32; o <<= 1) {
        chan_merge_equal(lm, m2, __shfl_xor_sync(0xffffffffu, lm, o),
                         __shfl_xor_sync(0xffffffffu, m2, o), cnt * 2.f);
        cnt *= 2.f;
      }
      par ^= 1;
      mu = lm;
      var = m2 * inv_n;
    } else {
      float s = 0.f;
#pragma unroll
      for (int i = 0; i < NV * 4; ++i) s += v[i];
      mu = block_reduce<THREADS / 32, false>(s, red) * inv_n;
      float q = 0.f;
#pragma unroll
      for (int k = 0; k < NV; ++k)
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float d = ((k * THREADS + t) * 4 + e < n) ? v[4 * k + e] - mu : 0.f;
          q = fmaf(d, d, q);
        }
      var = block_reduce<THREADS / 32, false>(q, red) * inv_n;
    }
    const float rs = 1.0f / sqrtf(var + eps);
    float* yr = y + row * ldy;
#pragma unroll
    for (int k = 0; k < NV; ++k) {
      const int idx0 = (k * THREADS + t) * 4;
      if (VEC) {
        if (idx0 < n) {
          const float4 wq = WB_REG ? wr[k] : __ldg(reinterpret_cast<const float4*>(w + idx0));
          const float4 bq = WB_REG ? br[k] : __ldg(reinterpret_cast<const float4*>(b + idx0));
          st_stream_f4(yr + idx0, make_float4(fmaf((v[4 * k] - mu) * rs, wq.x, bq.x),
                                              fmaf((v[4 * k + 1] - mu) * rs, wq.y, bq.y),
                                              fmaf((v[4 * k + 2] - mu) * rs, wq.z, bq.z),
                                              fmaf((v[4 * k + 3] - mu) * rs, wq.w, bq.w)));
        }
      } else {
#pragma unroll
        for (int e = 0; e < 4; ++e)
          if (idx0 + e < n) yr[idx0 + e] = fmaf((v[4 * k + e] - mu) * rs, __ldg(w + idx0 + e), __ldg(b + idx0 + e));
      }
    }
    if (t == 0) {
      mean[row] = mu;
      rstd[row] = rs;
    }
  }
}

// One row per CTA, no persistence (the softmax kernel's shape), for contiguous
// rows of (2048, 4096] floats: 256 threads x 4 float4, 6 CTAs per SM (40
// registers), so six rows per SM have their loads in flight and a finished
// CTA is replaced by the next row's. Measured at 16384 x 4096 against the
// persistent prefetching kernel (5790 GB/s): 6150-6162 GB/s; 512 x 2 at 3-4
// CTAs/SM 5597-5631, 256 x 4 at 8 CTAs/SM (spills) 6047-6055, 1024 x 1 3678.
constexpr int LN_ROW_THREADS = 256, LN_ROW_NV = 4, LN_ROW_CTAS = 6;
template <int THREADS, int NV>
__global__ void __launch_bounds__(THREADS, LN_ROW_CTAS)
    layernorm_fwd_row_kernel(const float* __restrict__ x, const float* __restrict__ w,
                             const float* __restrict__ b, float* __restrict__ y,
                             float* __restrict__ mean, float* __restrict__ rstd, int n,
                             int64_t ldx, int64_t ldy, float eps) {
  __shared__ float red[THREADS / 32];
  const int t = threadIdx.x;
  const int64_t row = blockIdx.x;
  float v[NV * 4];
  load_row<THREADS, NV, true>(x + row * ldx, n, 0.f, v);
  float s = 0.f;
#pragma unroll
  for (int i = 0; i < NV * 4; ++i) s += v[i];
  const float inv_n = 1.0f / (float)n;
  const float mu = block_reduce<THREADS / 32, false>(s, red) * inv_n;
  float q = 0.f;
#pragma unroll
  for (int k = 0; k < NV; ++k)
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const float d = ((k * THREADS + t) * 4 + e < n) ? v[4 * k + e] - mu : 0.f;
      q = fmaf(d, d, q);
    }
  const float var = block_reduce<THREADS / 32, false>(q, red) * inv_n;
  const float rs = 1.0f / sqrtf(var + eps);
  float* yr = y + row * ldy;
#pragma unroll
  for (int k = 0; k < NV; ++k) {
    const int idx0 = (k * THREADS + t) * 4;
    if (idx0 < n) {
      const float4 wq = __ldg(reinterpret_cast<const float4*>(w + idx0));
      const float4 bq = __ldg(reinterpret_cast<const float4*>(b + idx0));
      st_stream_f4(yr + idx0, make_float4(fmaf((v[4 * k] - mu) * rs, wq.x, bq.x),
                                          fmaf((v[4 * k + 1] - mu) * rs, wq.y, bq.y),
                                          fmaf((v[4 * k + 2] - mu) * rs, wq.z, bq.z),
                                          fmaf((v[4 * k + 3] - mu) * rs, wq.w, bq.w)));
    }
  }
  if (t == 0) {
    mean[row] = mu;
    rstd[row] = rs;
  }
}

// Rows longer than the register limit: three passes over x from L2/HBM.
constexpr int LN_LONG_THREADS = 1024;
__global__ void __launch_bounds__(LN_LONG_THREADS) layernorm_fwd_long_kernel(
    const float* __restrict__ x, const float* __restrict__ w, const float* __restrict__ b,
    float* __restrict__ y, float* __restrict__ mean, float* __restrict__ rstd, int n, int rows,
    int64_t ldx, int64_t ldy, float eps) {
  __shared__ float red[LN_LONG_THREADS / 32];
  for (int64_t row = blockIdx.x; row < rows; row += gridDim.x) {
    const float* xr = x + row * ldx;
    float s = 0.f;
    for (int i = threadIdx.x; i < n; i += LN_LONG_THREADS) s += xr[i];
    const float mu = block_reduce<LN_LONG_THREADS / 32, false>(s, red) / (float)n;
    float q = 0.f;
    for (int i = threadIdx.x; i < n; i += LN_LONG_THREADS) {
      const float d = xr[i] - mu;
      q = fmaf(d, d, q);
    }
    const float var = block_reduce<LN_LONG_THREADS / 32, false>(q, red) / (float)n;
    const float rs = 1.0f / sqrtf(var + eps);
    float* yr = y + row * ldy;
    for (int i = threadIdx.x; i < n; i += LN_LONG_THREADS)
      yr[i] = fmaf((xr[i] - mu) * rs, w[i], b[i]);
    if (threadIdx.x == 0) {
      mean[row] = mu;
      rstd[row] = rs;
    }
  }
}

template <int THREADS, int NV>
static int layernorm_reg_launch(const float* x, const float* w, const float* b, float* y,
                                float* mean, float* rstd, int n, int rows, int64_t ldx,
                                int64_t ldy, float eps, bool vec, int sm_count, cudaStream_t st) {
  // Resident CTAs per SM for this configuration decide the persistent grid.
  int occ = 0;
  cudaError_t e;
  if (vec)
    e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(
        &occ, layernorm_fwd_reg_kernel<THREADS, NV, true>, THREADS, 0);
  else
    e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(
        &occ, layernorm_fwd_reg_kernel<THREADS, NV, false>, THREADS, 0);
  if (e != cudaSuccess) return cuda_fail(e, "cudaOccupancyMaxActiveBlocksPerMultiprocessor");
  const int grid = std::min(rows, sm_count * std::max(occ, 1));
  if (vec)
    layernorm_fwd_reg_kernel<THREADS, NV, true>
        <<<grid, THREADS, 0, st>>>(x, w, b, y, mean, rstd, n, rows, ldx, ldy, eps);
  else
    layernorm_fwd_reg_kernel<THREADS, NV, false>
        <<<grid, THREADS, 0, st>>>(x, w, b, y, mean, rstd, n, rows, ldx, ldy, eps);
  return launch_status("layernorm_fwd_reg_kernel");
}

static int launch_layernorm(const float* x, const float* w, const float* b, float* y,
                            float* mean, float* rstd, int n, int rows, int64_t ldx, int64_t ldy,
                            float eps, cudaStream_t st) {
  DeviceProps p;
  if (int rc = current_props(&p)) return rc;
  if (rows == 0) return CTB_OK;
  const bool vec = n % 4 == 0 && ldx % 4 == 0 && ldy % 4 == 0 && aligned16(x) && aligned16(y) &&
                   aligned16(w) && aligned16(b);
  const int sm = p.sm_count;
  if (n <= 512) return layernorm_reg_launch<128, 1>(x, w, b, y, mean, rstd, n, rows, ldx, ldy, eps, vec, sm, st);
  if (n <= 2048) return layernorm_reg_launch<256, 2>(x, w, b, y, mean, rstd, n, rows, ldx, ldy, eps, vec, sm, st);
  if (vec && n > 2048 && n <= LN_ROW_THREADS * LN_ROW_NV * 4) {
    layernorm_fwd_row_kernel<LN_ROW_THREADS, LN_ROW_NV>
        <<<rows, LN_ROW_THREADS, 0, st>>>(x, w, b, y, mean, rstd, n, ldx, ldy, eps);
    return launch_status("layernorm_fwd_row_kernel");
  }
  if (n <= 4096) return layernorm_reg_launch<512, 2>(x, w, b, y, mean, rstd, n, rows, ldx, ldy, eps, vec, sm, st);
  if (n <= 8192) return layernorm_reg_launch<512, 4>(x, w, b, y, mean, rstd, n, rows, ldx, ldy, eps, vec, sm, st);
  if (n <= 16384) return layernorm_reg_launch<1024, 4>(x, w, b, y, mean, rstd, n, rows, ldx, ldy, eps, vec, sm, st);
  const int grid = std::min(rows, sm * 2);
  layernorm_fwd_long_kernel<<<grid, LN_LONG_THREADS, 0, st>>>(x, w, b, y, mean, rstd, n, rows,
                                                              ldx, ldy, eps);
  return launch_status("layernorm_fwd_long_kernel");
}

}  // namespace ctb

// =============================================================================
// C ABI
// =============================================================================
using namespace ctb;

extern "C" int ctb_vadd(int32_t dtype, const void* a, const void* b, void* c, int64_t n,
                        int64_t sa, int64_t sb, int64_t sc, void* stream) {
  clear_error();
  if (n < 0) return set_error(CTB_ERR_SHAPE, "vadd: negative length");
  if (n > 0 && (!a || !b || !c)) return set_error(CTB_ERR_ARG, "vadd: NULL pointer");
  auto st = static_cast<cudaStream_t>(stream);
  switch (dtype) {
    case CTB_F32:
      return launch_vadd((const float*)a, (const float*)b, (float*)c, n, sa, sb, sc, st);
    case CTB_F64:
      return launch_vadd((const double*)a, (const double*)b, (double*)c, n, sa, sb, sc, st);
    case CTB_F16:
      return launch_vadd((const __half*)a, (const __half*)b, (__half*)c, n, sa, sb, sc, st);
    default:
      return set_error(CTB_ERR_DTYPE, "vadd: dtype must be F16, F32 or F64");
  }
}

extern "C" int ctb_rowsum_f32(const float* a, float* out, int32_t m, int32_t n, int64_t s_i,
                              int64_t s_j, int64_t so, void* stream) {
  clear_error();
  if (m < 0 || n < 0) return set_error(CTB_ERR_SHAPE, "rowsum: negative size");
  if (m > 0 && (!a || !out)) return set_error(CTB_ERR_ARG, "rowsum: NULL pointer");
  return launch_rowsum(a, out, m, n, s_i, s_j, so, static_cast<cudaStream_t>(stream));
}

extern "C" int ctb_softmax_f32(const float* x, float* y, int32_t len, int32_t count, int64_t ldx,
                               int64_t ldy, void* stream) {
  clear_error();
  if (len < 0 || count < 0) return set_error(CTB_ERR_SHAPE, "softmax: negative size");
  if (len > 0 && count > 0 && (!x || !y)) return set_error(CTB_ERR_ARG, "softmax: NULL pointer");
  return launch_softmax(x, y, len, count, ldx, ldy, static_cast<cudaStream_t>(stream));
}

extern "C" int ctb_layernorm_fwd_f32(const float* x, const float* w, const float* b, float* y,
                                     float* mean, float* rstd, int32_t n, int32_t rows,
                                     int64_t ldx, int64_t ldy, float eps, void* stream) {
  clear_error();
  if (n <= 0 || rows < 0) return set_error(CTB_ERR_SHAPE, "layernorm_fwd: need n > 0, rows >= 0");
  if (rows > 0 && (!x || !w || !b || !y || !mean || !rstd))
    return set_error(CTB_ERR_ARG, "layernorm_fwd: NULL pointer");
  return launch_layernorm(x, w, b, y, mean, rstd, n, rows, ldx, ldy, eps,
                          static_cast<cudaStream_t>(stream));
}

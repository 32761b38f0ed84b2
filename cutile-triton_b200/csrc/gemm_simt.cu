// General-shape CUDA-core GEMM (any M, N, K, any column strides): the path
// for shapes the tensor-core kernel's TMA descriptors cannot describe (column
// strides that are not a multiple of 16 bytes) and for Float32 matmul, which
// the reference runs as tf32 (reference: test/runtests.jl:70-99). Accumulates
// in Float32 with exact fp32 products, so it is at least as accurate as tf32.
#include "ctb_common.cuh"

namespace ctb {

constexpr int SG_BM = 64, SG_BN = 64, SG_BK = 16;

__device__ __forceinline__ float to_f(float v) { return v; }
__device__ __forceinline__ float to_f(__half v) { return __half2float(v); }
__device__ __forceinline__ void from_f(float* p, float v) { *p = v; }
__device__ __forceinline__ void from_f(__half* p, float v) { *p = __float2half_rn(v); }

// 256 threads; each computes a 4 x 4 block of a 64 x 64 C tile.
template <typename T>
__global__ void __launch_bounds__(256) gemm_simt_kernel(const T* __restrict__ A,
                                                        const T* __restrict__ B,
                                                        T* __restrict__ C, int M, int N, int K,
                                                        int64_t lda, int64_t ldb, int64_t ldc,
                                                        int64_t sA, int64_t sB, int64_t sC) {
  __shared__ float As[SG_BK][SG_BM + 1];
  __shared__ float Bs[SG_BK][SG_BN + 1];
  const int bz = blockIdx.z;
  A += bz * sA;
  B += bz * sB;
  C += bz * sC;
  const int m0 = blockIdx.x * SG_BM, n0 = blockIdx.y * SG_BN;
  const int tx = threadIdx.x % 16, ty = threadIdx.x / 16;
  float acc[4][4] = {};
  for (int k0 = 0; k0 < K; k0 += SG_BK) {
    // A tile: 64 (m) x 16 (k), m fastest (column-major A).
    for (int i = threadIdx.x; i < SG_BM * SG_BK; i += 256) {
      const int mm = i % SG_BM, kk = i / SG_BM;
      const int gm = m0 + mm, gk = k0 + kk;
      As[kk][mm] = (gm < M && gk < K) ? to_f(A[gm + (int64_t)gk * lda]) : 0.f;
    }
    // B tile: 16 (k) x 64 (n), k fastest (column-major B).
    for (int i = threadIdx.x; i < SG_BK * SG_BN; i += 256) {
      const int kk = i % SG_BK, nn = i / SG_BK;
      const int gk = k0 + kk, gn = n0 + nn;
      Bs[kk][nn] = (gk < K && gn < N) ? to_f(B[gk + (int64_t)gn * ldb]) : 0.f;
    }
    __syncthreads();
#pragma unroll
    for (int kk = 0; kk < SG_BK; ++kk) {
      float a[4], b[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) a[i] = As[kk][tx + 16 * i];
#pragma unroll
      for (int j = 0; j < 4; ++j) b[j] = Bs[kk][ty + 16 * j];
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[i][j] = fmaf(a[i], b[j], acc[i][j]);
    }
    __syncthreads();
  }
#pragma unroll
  for (int i = 0; i < 4; ++i)
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int gm = m0 + tx + 16 * i, gn = n0 + ty + 16 * j;
      if (gm < M && gn < N) from_f(&C[gm + (int64_t)gn * ldc], acc[i][j]);
    }
}

template <typename T>
int gemm_simt(const T* A, const T* B, T* C, int M, int N, int K, int batch, int64_t lda,
              int64_t ldb, int64_t ldc, int64_t sA, int64_t sB, int64_t sC, cudaStream_t st) {
  if (M == 0 || N == 0 || batch == 0) return CTB_OK;
  if (batch > 65535) return set_error(CTB_ERR_SHAPE, "gemm: batch > 65535");
  dim3 grid((M + SG_BM - 1) / SG_BM, (N + SG_BN - 1) / SG_BN, batch);
  if (grid.y > 65535) return set_error(CTB_ERR_SHAPE, "gemm: N too large for the general path");
  gemm_simt_kernel<T><<<grid, 256, 0, st>>>(A, B, C, M, N, K, lda, ldb, ldc, sA, sB, sC);
  return launch_status("gemm_simt_kernel");
}

template int gemm_simt<__half>(const __half*, const __half*, __half*, int, int, int, int, int64_t,
                               int64_t, int64_t, int64_t, int64_t, int64_t, cudaStream_t);
template int gemm_simt<float>(const float*, const float*, float*, int, int, int, int, int64_t,
                              int64_t, int64_t, int64_t, int64_t, int64_t, cudaStream_t);

}  // namespace ctb

extern "C" int ctb_gemm_f32_simt(const float* A, const float* B, float* C, int32_t M, int32_t N,
                                 int32_t K, int32_t batch, int64_t lda, int64_t ldb, int64_t ldc,
                                 int64_t sA, int64_t sB, int64_t sC, void* stream) {
  ctb::clear_error();
  if (M < 0 || N < 0 || K < 0 || batch < 0) return ctb::set_error(CTB_ERR_SHAPE, "matmul: negative size");
  return ctb::gemm_simt<float>(A, B, C, M, N, K, batch, lda, ldb, ldc, sA, sB, sC,
                               static_cast<cudaStream_t>(stream));
}

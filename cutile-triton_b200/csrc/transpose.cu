// Transpose: y = x^T (cuTile example transpose.jl, not vendored in the
// reference; benchmarked there at 3212 GB/s on H100, research/bench_final.log:10).
// Julia column-major: x is M x N with column stride ldx, y is N x M with
// column stride ldy; y[j, i] = x[i, j] (a pure copy: bit-exact).
//
// 64 x 64 tiles through shared memory: each thread reads 4 elements along x's
// contiguous dimension and writes 4 along y's, with one padding column so the
// transposed shared-memory reads are conflict-free.
#include "ctb_common.cuh"

#include <algorithm>

namespace ctb {

constexpr int TP_TILE = 64, TP_TX = 16, TP_TY = 16;  // 256 threads, 16 elements each

template <typename T>
__global__ void __launch_bounds__(TP_TX* TP_TY) transpose_kernel(const T* __restrict__ x,
                                                                 T* __restrict__ y, int M, int N,
                                                                 int64_t ldx, int64_t ldy) {
  __shared__ T tile[TP_TILE][TP_TILE + 1];
  const int tx = threadIdx.x % TP_TX, ty = threadIdx.x / TP_TX;
  const int i0 = blockIdx.x * TP_TILE, j0 = blockIdx.y * TP_TILE;  // x rows i, columns j
  // x column j (contiguous in i): tile[j - j0][i - i0]
#pragma unroll
  for (int r = 0; r < TP_TILE / TP_TY; ++r) {
    const int jj = ty + r * TP_TY;
    const int j = j0 + jj;
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const int ii = tx * 4 + e;
      const int i = i0 + ii;
      if (i < M && j < N) tile[jj][ii] = x[i + (int64_t)j * ldx];
    }
  }
  __syncthreads();
  // y column i (contiguous in j): y[j + i * ldy] = tile[j - j0][i - i0]
#pragma unroll
  for (int r = 0; r < TP_TILE / TP_TY; ++r) {
    const int ii = ty + r * TP_TY;
    const int i = i0 + ii;
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const int jj = tx * 4 + e;
      const int j = j0 + jj;
      if (i < M && j < N) y[j + (int64_t)i * ldy] = tile[jj][ii];
    }
  }
}

// Float32 with 16-byte aligned columns: the same tiling with float4 accesses.
__global__ void __launch_bounds__(TP_TX* TP_TY) transpose_f32_vec_kernel(
    const float* __restrict__ x, float* __restrict__ y, int M, int N, int64_t ldx, int64_t ldy) {
  __shared__ float tile[TP_TILE][TP_TILE + 1];
  const int tx = threadIdx.x % TP_TX, ty = threadIdx.x / TP_TX;
  const int i0 = blockIdx.x * TP_TILE, j0 = blockIdx.y * TP_TILE;
  const int ii0 = tx * 4;
#pragma unroll
  for (int r = 0; r < TP_TILE / TP_TY; ++r) {
    const int jj = ty + r * TP_TY;
    const int j = j0 + jj;
    const int i = i0 + ii0;
    if (j < N && i < M) {  // M % 4 == 0 on this path, so i < M covers i + 3
      const float4 v = ld_stream_f4(x + i + (int64_t)j * ldx);
      tile[jj][ii0] = v.x;
      tile[jj][ii0 + 1] = v.y;
      tile[jj][ii0 + 2] = v.z;
      tile[jj][ii0 + 3] = v.w;
    }
  }
  __syncthreads();
#pragma unroll
  for (int r = 0; r < TP_TILE / TP_TY; ++r) {
    const int ii = ty + r * TP_TY;
    const int i = i0 + ii;
    const int j = j0 + ii0;
    if (i < M && j < N)  // N % 4 == 0 on this path
      st_stream_f4(y + j + (int64_t)i * ldy,
                   make_float4(tile[ii0][ii], tile[ii0 + 1][ii], tile[ii0 + 2][ii], tile[ii0 + 3][ii]));
  }
}

template <typename T>
static int launch_transpose(const T* x, T* y, int M, int N, int64_t ldx, int64_t ldy,
                            cudaStream_t st) {
  if (M == 0 || N == 0) return CTB_OK;
  dim3 grid((M + TP_TILE - 1) / TP_TILE, (N + TP_TILE - 1) / TP_TILE);
  if (grid.y > 65535) return set_error(CTB_ERR_SHAPE, "transpose: N too large");
  if (sizeof(T) == 4 && M % 4 == 0 && N % 4 == 0 && ldx % 4 == 0 && ldy % 4 == 0 &&
      aligned16(x) && aligned16(y))
    transpose_f32_vec_kernel<<<grid, TP_TX * TP_TY, 0, st>>>(
        reinterpret_cast<const float*>(x), reinterpret_cast<float*>(y), M, N, ldx, ldy);
  else
    transpose_kernel<T><<<grid, TP_TX * TP_TY, 0, st>>>(x, y, M, N, ldx, ldy);
  return launch_status("transpose_kernel");
}

}  // namespace ctb

extern "C" int ctb_transpose(int32_t dtype, const void* x, void* y, int32_t M, int32_t N,
                             int64_t ldx, int64_t ldy, void* stream) {
  using namespace ctb;
  clear_error();
  if (M < 0 || N < 0) return set_error(CTB_ERR_SHAPE, "transpose: negative size");
  if ((int64_t)M * N > 0 && (!x || !y)) return set_error(CTB_ERR_ARG, "transpose: NULL pointer");
  if ((M > 0 && ldx < M) || (N > 0 && ldy < N))
    return set_error(CTB_ERR_LAYOUT, "transpose: leading dimension smaller than the column length");
  DeviceProps p;
  if (int rc = current_props(&p)) return rc;
  auto st = static_cast<cudaStream_t>(stream);
  switch (dtype) {
    case CTB_F32: return launch_transpose((const float*)x, (float*)y, M, N, ldx, ldy, st);
    case CTB_F16: return launch_transpose((const __half*)x, (__half*)y, M, N, ldx, ldy, st);
    case CTB_F64: return launch_transpose((const double*)x, (double*)y, M, N, ldx, ldy, st);
    case CTB_I32:  // moved bit for bit like Float32
      return launch_transpose((const float*)x, (float*)y, M, N, ldx, ldy, st);
    default: return set_error(CTB_ERR_DTYPE, "transpose: dtype must be F16, F32, F64 or I32");
  }
}

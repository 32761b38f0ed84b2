// CUDA-core attention forward (the cuTile example fmha.jl:20, not vendored in
// the reference; report.html:2981 describes its 4-D head-dim-contiguous tiles):
// one warp per query row, online softmax over key chunks of 32. It serves head
// dims and sequence shapes the tensor-core kernel does not take, and is the
// independent on-device cross-check of that kernel in the tests. Same contract
// as ctb_fmha_fwd_f16.
#include "ctb_common.cuh"

namespace ctb {

constexpr int FS_WARPS = 4;
constexpr int FS_MAXD = 256;

__global__ void __launch_bounds__(FS_WARPS * 32) fmha_simt_kernel(
    const __half* __restrict__ Q, const __half* __restrict__ K, const __half* __restrict__ V,
    __half* __restrict__ O, int Sq, int Sk, int D, float scale, int causal) {
  __shared__ float qs[FS_WARPS][FS_MAXD];
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int64_t bh = blockIdx.y;
  const int i = blockIdx.x * FS_WARPS + warp;  // query row
  if (i >= Sq) return;
  const __half* q = Q + (bh * Sq + i) * D;
  const __half* kb = K + bh * Sk * D;
  const __half* vb = V + bh * Sk * D;
  for (int d = lane; d < D; d += 32) qs[warp][d] = __half2float(q[d]) * scale;
  __syncwarp();
  constexpr int DPL = FS_MAXD / 32;  // output dims per lane (max)
  float acc[DPL];
#pragma unroll
  for (int r = 0; r < DPL; ++r) acc[r] = 0.f;
  float m = -INFINITY, l = 0.f;
  const int kend = causal ? min(Sk, i + 1) : Sk;
  for (int j0 = 0; j0 < kend; j0 += 32) {
    const int j = j0 + lane;
    float s = -INFINITY;
    if (j < kend) {
      const __half* kr = kb + (int64_t)j * D;
      float t = 0.f;
      for (int d = 0; d < D; ++d) t = fmaf(qs[warp][d], __half2float(kr[d]), t);
      s = t;
    }
    const float cm = warp_max(s);
    const float mn = fmaxf(m, cm);
    const float corr = (m == -INFINITY) ? 0.f : expf(m - mn);
    const float pj = (j < kend) ? expf(s - mn) : 0.f;
    l = l * corr + warp_sum(pj);
#pragma unroll
    for (int r = 0; r < DPL; ++r) acc[r] *= corr;
    const int nk = min(32, kend - j0);
    for (int jj = 0; jj < nk; ++jj) {
      const float p = __shfl_sync(0xffffffffu, pj, jj);
      const __half* vr = vb + (int64_t)(j0 + jj) * D;
#pragma unroll
      for (int r = 0; r < DPL; ++r) {
        const int d = lane + 32 * r;
        if (d < D) acc[r] = fmaf(p, __half2float(vr[d]), acc[r]);
      }
    }
    m = mn;
  }
  const float inv = 1.0f / l;
  __half* o = O + (bh * Sq + i) * D;
#pragma unroll
  for (int r = 0; r < DPL; ++r) {
    const int d = lane + 32 * r;
    if (d < D) o[d] = __float2half_rn(acc[r] * inv);
  }
}

int fmha_simt(const __half* Q, const __half* K, const __half* V, __half* O, int B, int H, int Sq,
              int Sk, int D, float scale, int causal, cudaStream_t st) {
  if (D > FS_MAXD) return set_error(CTB_ERR_SHAPE, "fmha: head_dim > 256");
  if ((int64_t)B * H > 65535) return set_error(CTB_ERR_SHAPE, "fmha: batch*heads > 65535 on the general path");
  dim3 grid((Sq + FS_WARPS - 1) / FS_WARPS, B * H);
  fmha_simt_kernel<<<grid, FS_WARPS * 32, 0, st>>>(Q, K, V, O, Sq, Sk, D, scale, causal);
  return launch_status("fmha_simt_kernel");
}

}  // namespace ctb

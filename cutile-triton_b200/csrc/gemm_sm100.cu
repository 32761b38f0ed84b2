// Float16 GEMM / batched GEMM on the 5th-generation tensor cores (tcgen05).
//
// cuTile `matmul16(A, B, C, tm, tn, tk)` (reference: bench/bench_f16.jl:10-22)
// and the batchmatmul example: C = A*B with f16 inputs, f32 accumulation in
// tensor memory, f16 output rounded to nearest. Julia column-major operands:
// A (M x K, M contiguous) is an MN-major UMMA A operand, B (K x N, K
// contiguous) a K-major B operand, C (M x N) is M contiguous, so a TMEM
// accumulator lane (= row m) maps to consecutive C addresses across a warp.
//
// Kernel shape: persistent, one CTA per SM, 128 x 256 x 64 tiles, 4-stage
// TMA -> shared memory ring, 6 warps:
//   warp 0      TMA producer (one elected thread)
//   warp 1      TMEM owner + MMA issuer (one elected thread)
//   warps 2..5  epilogue: tcgen05.ld -> f16 -> global
// Two 256-column accumulators in TMEM (512 columns) let the epilogue of tile
// i overlap the main loop of tile i+1. No cluster multicast anywhere.
#include "sm100_ptx.cuh"

#include <cudaTypedefs.h>

#include <algorithm>
#include <mutex>

namespace ctb {

template <typename T>
int gemm_simt(const T* A, const T* B, T* C, int M, int N, int K, int batch, int64_t lda,
              int64_t ldb, int64_t ldc, int64_t sA, int64_t sB, int64_t sC, cudaStream_t st);

namespace gemm {

constexpr int BM = 128, BN = 256, BK = 64, STAGES = 4;
constexpr int THREADS = 192;
constexpr int A_HALF_BYTES = 64 * BK * 2;          // one 64(m) x 64(k) TMA box = 8 KB
constexpr int A_STAGE_BYTES = BM * BK * 2;         // 16 KB
constexpr int B_STAGE_BYTES = BN * BK * 2;         // 32 KB
constexpr int STAGE_BYTES = A_STAGE_BYTES + B_STAGE_BYTES;
constexpr int TMEM_COLS = 2 * BN;                  // two accumulators
constexpr int GROUP_M = 8;                         // L2-friendly tile order
constexpr int SMEM_BYTES = STAGES * STAGE_BYTES + 1024 /*align slack*/ + 256 /*barriers*/;
constexpr unsigned ERR_BIT = 1u;

struct Params {
  __half* C;
  int M, N, K, batch;
  int64_t ldc, sC;
  int tiles_m, tiles_n, num_kb;
  int64_t num_tiles;
};

__device__ __forceinline__ void tile_coords(const Params& p, int64_t t, int& b, int& mt,
                                            int& nt) {
  const int64_t per_batch = (int64_t)p.tiles_m * p.tiles_n;
  b = (int)(t / per_batch);
  const int r = (int)(t - (int64_t)b * per_batch);
  const int group_span = GROUP_M * p.tiles_n;
  const int g = r / group_span;
  const int first_m = g * GROUP_M;
  const int gsize = min(p.tiles_m - first_m, GROUP_M);
  const int rr = r - g * group_span;
  mt = first_m + rr % gsize;
  nt = rr / gsize;
}

__global__ void __launch_bounds__(THREADS, 1)
    gemm_f16_tcgen05_kernel(const __grid_constant__ CUtensorMap tmA,
                            const __grid_constant__ CUtensorMap tmB, const Params p) {
  using namespace sm100;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  // 128-byte swizzle atoms need 1024-byte aligned tiles.
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + STAGES * STAGE_BYTES);
  uint64_t* empty = full + STAGES;
  uint64_t* tmem_full = empty + STAGES;   // [2]
  uint64_t* tmem_empty = tmem_full + 2;   // [2]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tmem_empty + 2);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&tmem_full[i], 1);
      mbar_init(&tmem_empty[i], 128);
    }
    *abort_flag = 0;
    fence_mbar_init();
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
  }
  if (warp == 1) tmem_alloc(tmem_slot, TMEM_COLS);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    // ---------------- TMA producer ----------------
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      for (int64_t t = blockIdx.x; t < p.num_tiles && !*abort_flag; t += gridDim.x) {
        int b, mt, nt;
        tile_coords(p, t, b, mt, nt);
        const int m0 = mt * BM, n0 = nt * BN;
        for (int kb = 0; kb < p.num_kb; ++kb) {
          if (!mbar_wait_bounded(&empty[stage], phase ^ 1, abort_flag, ERR_BIT)) break;
          uint8_t* sa = smem + stage * STAGE_BYTES;
          uint8_t* sb = sa + A_STAGE_BYTES;
          mbar_arrive_expect_tx(&full[stage], STAGE_BYTES);
          tma_load_3d(sa, &tmA, &full[stage], m0, kb * BK, b);
          tma_load_3d(sa + A_HALF_BYTES, &tmA, &full[stage], m0 + 64, kb * BK, b);
          tma_load_3d(sb, &tmB, &full[stage], kb * BK, n0, b);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
      }
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer ----------------
    // The whole warp runs the loop converged (descriptors stay warp-uniform)
    // and elect.sync picks the issuing lane; wait results are made uniform.
    {
      constexpr uint32_t idesc = idesc_f16_f32(BM, BN, /*a MN-major*/ true, /*b K-major*/ false);
      int stage = 0;
      uint32_t phase = 0;
      int it = 0;
      bool ok = true;
      for (int64_t t = blockIdx.x; ok && t < p.num_tiles; t += gridDim.x, ++it) {
        const int buf = it & 1;
        const uint32_t acc_phase = (it >> 1) & 1;
        if (!(ok = __all_sync(0xffffffffu, mbar_wait_bounded(&tmem_empty[buf], acc_phase ^ 1, abort_flag, ERR_BIT)))) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + buf * BN;
        for (int kb = 0; kb < p.num_kb; ++kb) {
          if (!(ok = __all_sync(0xffffffffu, mbar_wait_bounded(&full[stage], phase, abort_flag, ERR_BIT)))) break;
          tc_fence_after();
          const uint32_t sa = smem_u32(smem + stage * STAGE_BYTES);
          // A, MN-major SW128: LBO = 8 KB between the two 64-row halves,
          // SBO = 1 KB between 8-k-row groups; K step of 16 = 2 KB.
          const uint64_t ad = smem_desc_sw128(sa, A_HALF_BYTES, 1024);
          // B, K-major SW128: SBO = 1 KB between 8-row groups; K step of 16
          // halves = 32 bytes inside the swizzled 128-byte row. Steps are
          // added to the (address >> 4) field.
          const uint64_t bd = smem_desc_sw128(sa + A_STAGE_BYTES, 16, 1024);
#pragma unroll
          for (int k = 0; k < BK / 16; ++k)
            mma_f16_ss_elect(d_tmem, ad + (uint64_t)(k * 2048 >> 4), bd + (uint64_t)(k * 32 >> 4),
                             idesc, (kb | k) != 0);
          mma_commit_elect(&empty[stage]);  // frees the stage when these MMAs finish
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
        if (!ok) break;
        mma_commit_elect(&tmem_full[buf]);  // accumulator ready for the epilogue
      }
    }
  } else {
    // ---------------- epilogue (warps 2..5) ----------------
    const int q = warp & 3;  // TMEM lane quarter this warp may access
    const uint32_t lane_base = (uint32_t)(q * 32) << 16;
    int it = 0;
    for (int64_t t = blockIdx.x; t < p.num_tiles && !*abort_flag; t += gridDim.x, ++it) {
      const int buf = it & 1;
      const uint32_t acc_phase = (it >> 1) & 1;
      if (!mbar_wait_bounded(&tmem_full[buf], acc_phase, abort_flag, ERR_BIT)) break;
      tc_fence_after();
      int b, mt, nt;
      tile_coords(p, t, b, mt, nt);
      const int m = mt * BM + q * 32 + lane;
      const int n0 = nt * BN;
      __half* cb = p.C + (int64_t)b * p.sC;
#pragma unroll 1
      for (int c = 0; c < BN; c += 32) {
        uint32_t r[32];
        tmem_ld_32x32b_x32(tmem_base + buf * BN + c + lane_base, r);
        tmem_ld_wait();
        if (m < p.M) {
#pragma unroll
          for (int j = 0; j < 32; ++j) {
            const int n = n0 + c + j;
            if (n < p.N) cb[(int64_t)m + (int64_t)n * p.ldc] = __float2half_rn(__uint_as_float(r[j]));
          }
        }
      }
      tc_fence_before();
      mbar_arrive(&tmem_empty[buf]);
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, TMEM_COLS);
  }
}

// Writes zeros into an M x N column-major block (K == 0 case).
__global__ void zero_cols_kernel(__half* C, int M, int N, int batch, int64_t ldc, int64_t sC) {
  const int64_t total = (int64_t)M * N * batch;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t m = i % M, rest = i / M, n = rest % N, b = rest / N;
    C[b * sC + m + n * ldc] = __float2half_rn(0.f);
  }
}

}  // namespace gemm

// ---- host --------------------------------------------------------------------
static PFN_cuTensorMapEncodeTiled_v12000 g_encode = nullptr;
static std::once_flag g_encode_once;

int encode_tmap(CUtensorMap* map, CUtensorMapDataType dtype, int rank, const void* base,
                const uint64_t* dims, const uint64_t* strides_bytes, const uint32_t* box,
                CUtensorMapSwizzle swizzle) {
  std::call_once(g_encode_once, [] {
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      g_encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
  });
  if (!g_encode) return set_error(CTB_ERR_CUDA, "cuTensorMapEncodeTiled entry point unavailable");
  cuuint32_t estr[5] = {1, 1, 1, 1, 1};
  CUresult r = g_encode(map, dtype, (cuuint32_t)rank, const_cast<void*>(base),
                        reinterpret_cast<const cuuint64_t*>(dims),
                        reinterpret_cast<const cuuint64_t*>(strides_bytes),
                        reinterpret_cast<const cuuint32_t*>(box), estr,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle,
                        CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    return set_error(CTB_ERR_LAYOUT, "cuTensorMapEncodeTiled rejected the operand (CUresult " +
                                         std::to_string((int)r) + ")");
  return CTB_OK;
}

int gemm_take_device_error(unsigned int* out) { return take_device_error(out); }

static bool g_gemm_attr_done[64];
static std::mutex g_gemm_mu;

int gemm_device_setup() {
  int dev = 0;
  CTB_CUDA_CHECK(cudaGetDevice(&dev));
  std::lock_guard<std::mutex> lk(g_gemm_mu);
  if (dev < 64 && g_gemm_attr_done[dev]) return CTB_OK;
  CTB_CUDA_CHECK(cudaFuncSetAttribute(gemm::gemm_f16_tcgen05_kernel,
                                      cudaFuncAttributeMaxDynamicSharedMemorySize,
                                      gemm::SMEM_BYTES));
  if (dev < 64) g_gemm_attr_done[dev] = true;
  return CTB_OK;
}

// Tensor-core path eligibility: TMA needs 16-byte aligned bases and strides.
static bool tma_ok(const void* p, int64_t ld, int64_t bs, int batch) {
  if (!aligned16(p)) return false;
  if ((ld * 2) % 16 != 0 || ld <= 0) return false;
  if (batch > 1 && ((bs * 2) % 16 != 0 || bs <= 0)) return false;
  return true;
}

static int gemm_f16_dispatch(const __half* A, const __half* B, __half* C, int M, int N, int K,
                             int batch, int64_t lda, int64_t ldb, int64_t ldc, int64_t sA,
                             int64_t sB, int64_t sC, cudaStream_t st) {
  if (M < 0 || N < 0 || K < 0 || batch < 0) return set_error(CTB_ERR_SHAPE, "matmul: negative size");
  if (M == 0 || N == 0 || batch == 0) return CTB_OK;
  if (!C || (K > 0 && (!A || !B))) return set_error(CTB_ERR_ARG, "matmul: NULL pointer");
  if (lda < M || ldb < K || ldc < M)
    return set_error(CTB_ERR_LAYOUT, "matmul: leading dimension smaller than the column length");
  DeviceProps pr;
  if (int rc = current_props(&pr)) return rc;
  if (K == 0) {
    gemm::zero_cols_kernel<<<pr.sm_count * 4, 256, 0, st>>>(C, M, N, batch, ldc, sC);
    return launch_status("zero_cols_kernel");
  }
  if (!tma_ok(A, lda, sA, batch) || !tma_ok(B, ldb, sB, batch))
    return gemm_simt<__half>(A, B, C, M, N, K, batch, lda, ldb, ldc, sA, sB, sC, st);
  if (int rc = gemm_device_setup()) return rc;

  CUtensorMap tmA, tmB;
  {
    const uint64_t dims[3] = {(uint64_t)M, (uint64_t)K, (uint64_t)batch};
    const uint64_t strides[2] = {(uint64_t)lda * 2,
                                 (uint64_t)(batch > 1 ? sA : lda * K) * 2};
    const uint32_t box[3] = {64, gemm::BK, 1};
    if (int rc = encode_tmap(&tmA, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3, A, dims, strides, box,
                             CU_TENSOR_MAP_SWIZZLE_128B))
      return rc;
  }
  {
    const uint64_t dims[3] = {(uint64_t)K, (uint64_t)N, (uint64_t)batch};
    const uint64_t strides[2] = {(uint64_t)ldb * 2,
                                 (uint64_t)(batch > 1 ? sB : ldb * N) * 2};
    const uint32_t box[3] = {gemm::BK, gemm::BN, 1};
    if (int rc = encode_tmap(&tmB, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3, B, dims, strides, box,
                             CU_TENSOR_MAP_SWIZZLE_128B))
      return rc;
  }
  gemm::Params p;
  p.C = C;
  p.M = M;
  p.N = N;
  p.K = K;
  p.batch = batch;
  p.ldc = ldc;
  p.sC = sC;
  p.tiles_m = (M + gemm::BM - 1) / gemm::BM;
  p.tiles_n = (N + gemm::BN - 1) / gemm::BN;
  p.num_kb = (K + gemm::BK - 1) / gemm::BK;
  p.num_tiles = (int64_t)p.tiles_m * p.tiles_n * batch;
  const int grid = (int)std::min<int64_t>(p.num_tiles, pr.sm_count);
  gemm::gemm_f16_tcgen05_kernel<<<grid, gemm::THREADS, gemm::SMEM_BYTES, st>>>(tmA, tmB, p);
  return launch_status("gemm_f16_tcgen05_kernel");
}

}  // namespace ctb

using namespace ctb;

extern "C" int ctb_gemm_f16(const void* A, const void* B, void* C, int32_t M, int32_t N,
                            int32_t K, int64_t lda, int64_t ldb, int64_t ldc, void* stream) {
  clear_error();
  return gemm_f16_dispatch((const __half*)A, (const __half*)B, (__half*)C, M, N, K, 1, lda, ldb,
                           ldc, 0, 0, 0, static_cast<cudaStream_t>(stream));
}

extern "C" int ctb_bgemm_f16(const void* A, const void* B, void* C, int32_t M, int32_t N,
                             int32_t K, int32_t batch, int64_t lda, int64_t ldb, int64_t ldc,
                             int64_t sA, int64_t sB, int64_t sC, void* stream) {
  clear_error();
  return gemm_f16_dispatch((const __half*)A, (const __half*)B, (__half*)C, M, N, K, batch, lda,
                           ldb, ldc, sA, sB, sC, static_cast<cudaStream_t>(stream));
}

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
// i overlap the main loop of tile i+1. Every TMA load fills one CTA's own shared memory.
#include "sm100_ptx.cuh"

#include <cstdlib>
#include <cstring>

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
#ifndef CTB_GEMM_GROUP_M
#define CTB_GEMM_GROUP_M 8
#endif
constexpr int GROUP_M = CTB_GEMM_GROUP_M;          // L2-friendly tile order (m-tiles per group)
// Epilogue staging for TMA stores: per epilogue warp two 32(m) x 32(n) Float16
// boxes of 2 KB.
constexpr int EPI_BOX_BYTES = 32 * 32 * 2;
constexpr int EPI_BYTES = 4 * 2 * EPI_BOX_BYTES;
constexpr int SMEM_BYTES =
    STAGES * STAGE_BYTES + EPI_BYTES + 1024 /*align slack*/ + 256 /*barriers*/;
constexpr unsigned ERR_BIT = 1u;

struct Params {
  __half* C;
  int M, N, K, batch;
  int64_t ldc, sC;
  int tiles_m, tiles_n, num_kb;
  int64_t num_tiles;
  int tma_store;  // C written by TMA tensor stores (else 2-byte stores per element)
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

#ifdef CTB_GEMM_TRACE
// Debug-only timeline (%globaltimer ns) of CTA 0's first tile: 0 start,
// 1 set-up done, 2 first B/A loads issued, 3 last loads issued, 4 MMA got
// stage 0, 5 MMA issued the last stage, 6 epilogue got the accumulator,
// 7 epilogue stored, 8 all roles done, 9 TMEM released.
__device__ unsigned long long g_gemm_trace[10];
#define GEMM_TRACE(ev)                                    \
  do {                                                    \
    if (blockIdx.x == 0) g_gemm_trace[ev] = global_ns(); \
  } while (0)
#else
#define GEMM_TRACE(ev) \
  do {                 \
  } while (0)
#endif

__global__ void __launch_bounds__(THREADS, 1)
    gemm_f16_tcgen05_kernel(const __grid_constant__ CUtensorMap tmA,
                            const __grid_constant__ CUtensorMap tmB,
                            const __grid_constant__ CUtensorMap tmC, const Params p) {
  using namespace sm100;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  // 128-byte swizzle atoms need 1024-byte aligned tiles.
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  uint8_t* epi_stage = smem + STAGES * STAGE_BYTES;  // [4 warps][2 boxes]
  uint64_t* full = reinterpret_cast<uint64_t*>(epi_stage + EPI_BYTES);
  uint64_t* empty = full + STAGES;
  uint64_t* tmem_full = empty + STAGES;   // [2]
  uint64_t* tmem_empty = tmem_full + 2;   // [2]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tmem_empty + 2);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  if (threadIdx.x == 0) GEMM_TRACE(0);

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
  if (threadIdx.x == 0) GEMM_TRACE(1);

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
          if (t == blockIdx.x && kb == 0) GEMM_TRACE(2);
          if (t == blockIdx.x && kb == p.num_kb - 1) GEMM_TRACE(3);
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
          if (it == 0 && kb == 0 && lane == 0) GEMM_TRACE(4);
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
        if (it == 0 && lane == 0) GEMM_TRACE(5);
      }
    }
  } else {
    // ---------------- epilogue (warps 2..5) ----------------
    // TMEM lane m holds row m of the tile. With TMA stores each warp stages
    // its 32 rows x 32 columns per chunk in shared memory (column-major, as C)
    // and one lane stores the box; two staging boxes per warp alternate, and
    // the next chunk's TMEM load is in flight while a chunk is staged.
    const int q = warp & 3;  // TMEM lane quarter this warp may access
    const uint32_t lane_base = (uint32_t)(q * 32) << 16;
    __half* stage_w = reinterpret_cast<__half*>(epi_stage + q * 2 * EPI_BOX_BYTES);
    int sbuf = 0;
    int it = 0;
    for (int64_t t = blockIdx.x; t < p.num_tiles && !*abort_flag; t += gridDim.x, ++it) {
      const int buf = it & 1;
      const uint32_t acc_phase = (it >> 1) & 1;
      if (!mbar_wait_bounded(&tmem_full[buf], acc_phase, abort_flag, ERR_BIT)) break;
      tc_fence_after();
      if (it == 0 && warp == 2 && lane == 0) GEMM_TRACE(6);
      int b, mt, nt;
      tile_coords(p, t, b, mt, nt);
      const int m0 = mt * BM + q * 32;
      const int m = m0 + lane;
      const int n0 = nt * BN;
      const uint32_t tcol = tmem_base + buf * BN + lane_base;
      if (p.tma_store) {
        auto stage_chunk = [&](uint32_t (&r)[32], int c) {
          if (m0 >= p.M || n0 + c >= p.N) return;  // warp-uniform: box wholly outside C
          __half* sb = stage_w + sbuf * (EPI_BOX_BYTES / 2);
          if (lane == 0) bulk_wait_read<1>();  // this box's previous store has read it
          __syncwarp();
#pragma unroll
          for (int j = 0; j < 32; ++j) sb[j * 32 + lane] = __float2half_rn(__uint_as_float(r[j]));
          fence_async_shared();
          __syncwarp();
          if (lane == 0) {
            tma_store_3d(&tmC, sb, m0, n0 + c, b);
            bulk_commit();
          }
          sbuf ^= 1;
        };
        uint32_t ra[32], rb[32];
        tmem_ld_32x32b_x32(tcol, ra);
#pragma unroll 1
        for (int c = 0; c < BN; c += 64) {
          tmem_ld_wait_regs(ra);
          tmem_ld_32x32b_x32(tcol + c + 32, rb);
          stage_chunk(ra, c);
          tmem_ld_wait_regs(rb);
          if (c + 64 < BN) tmem_ld_32x32b_x32(tcol + c + 64, ra);
          stage_chunk(rb, c + 32);
        }
      } else {
        __half* cb = p.C + (int64_t)b * p.sC;
#pragma unroll 1
        for (int c = 0; c < BN; c += 32) {
          uint32_t r[32];
          tmem_ld_32x32b_x32(tcol + c, r);
          tmem_ld_wait_regs(r);
          if (m < p.M) {
#pragma unroll
            for (int j = 0; j < 32; ++j) {
              const int n = n0 + c + j;
              if (n < p.N)
                cb[(int64_t)m + (int64_t)n * p.ldc] = __float2half_rn(__uint_as_float(r[j]));
            }
          }
        }
      }
      tc_fence_before();
      mbar_arrive(&tmem_empty[buf]);
      if (it == 0 && warp == 2 && lane == 0) GEMM_TRACE(7);
    }
    if (lane == 0) bulk_wait<0>();  // staged boxes must outlive their stores
  }

  tc_fence_before();
  __syncthreads();
  if (threadIdx.x == 0) GEMM_TRACE(8);
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, TMEM_COLS);
    if (lane == 0) GEMM_TRACE(9);
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


// -----------------------------------------------------------------------------
// CTA-pair variant: one 256 x 256 tile per pair of SMs (tcgen05 cta_group::2).
// Each CTA loads its own 128 rows of A and 128 columns of B per 64-deep
// k-block (32 KB, against 48 KB per SM for a 128 x 256 tile on one SM: TMA
// delivers about 78 bytes per clock per SM from L2, and one SM's 128 x 256 x
// 64 step needs 96 per clock at the full MMA rate). The even CTA issues
// 256 x 256 x 16 MMAs that read both CTAs' operands; each CTA keeps its 128
// accumulator rows in its own tensor memory and writes them out itself.
// Barriers: full[s] lives in the even CTA and counts both CTAs' bytes;
// empty[s] and tmem_full[b] exist in both CTAs and are arrived by commits to
// both CTAs; tmem_empty[b] lives in the even CTA and counts all 256 epilogue
// threads of the pair.
// -----------------------------------------------------------------------------
constexpr int P_STAGES = 6;
constexpr int P_A_BYTES = 128 * BK * 2;  // this CTA's 128 rows of A (two 64-row boxes)
constexpr int P_B_BYTES = 128 * BK * 2;  // this CTA's 128 columns of B
constexpr int P_STAGE_BYTES = P_A_BYTES + P_B_BYTES;
constexpr int P_SMEM_BYTES = P_STAGES * P_STAGE_BYTES + EPI_BYTES + 1024 + 256;

__global__ void __launch_bounds__(THREADS, 1)
    gemm_f16_pair_kernel(const __grid_constant__ CUtensorMap tmA,
                         const __grid_constant__ CUtensorMap tmB,
                         const __grid_constant__ CUtensorMap tmC, const Params p) {
  using namespace sm100;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  uint8_t* epi_stage = smem + P_STAGES * P_STAGE_BYTES;
  uint64_t* full = reinterpret_cast<uint64_t*>(epi_stage + EPI_BYTES);
  uint64_t* empty = full + P_STAGES;
  uint64_t* tmem_full = empty + P_STAGES;  // [2]
  uint64_t* tmem_empty = tmem_full + 2;    // [2]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tmem_empty + 2);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const uint32_t rank = cluster_ctarank();
  const bool leader = rank == 0;
  const int64_t pair = blockIdx.x / 2, num_pairs = gridDim.x / 2;

  if (threadIdx.x == 0) {
    for (int s = 0; s < P_STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&tmem_full[i], 1);
      mbar_init(&tmem_empty[i], 256);
    }
    *abort_flag = 0;
    fence_mbar_init();
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
    tma_prefetch_desc(&tmC);
  }
  if (warp == 1) tmem_alloc_pair(tmem_slot, TMEM_COLS);
  tc_fence_before();
  cluster_sync_all();  // barriers initialised in both CTAs before any cross-CTA use
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  const uint32_t full_leader = mapa_shared(smem_u32(&full[0]), 0);

  if (warp == 0) {
    // ---------------- TMA producer (both CTAs) ----------------
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      for (int64_t t = pair; t < p.num_tiles && !*abort_flag; t += num_pairs) {
        int b, mt, nt;
        tile_coords(p, t, b, mt, nt);
        const int m0 = mt * 256 + (int)rank * 128, n0 = nt * 256 + (int)rank * 128;
        for (int kb = 0; kb < p.num_kb; ++kb) {
          if (!mbar_wait_bounded(&empty[stage], phase ^ 1, abort_flag, ERR_BIT)) break;
          uint8_t* sa = smem + stage * P_STAGE_BYTES;
          if (leader) mbar_arrive_expect_tx(&full[stage], 2 * P_STAGE_BYTES);
          const uint32_t bar = full_leader + stage * 8;
          tma_load_3d_pair(sa, &tmA, bar, m0, kb * BK, b);
          tma_load_3d_pair(sa + A_HALF_BYTES, &tmA, bar, m0 + 64, kb * BK, b);
          tma_load_3d_pair(sa + P_A_BYTES, &tmB, bar, kb * BK, n0, b);
          if (++stage == P_STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
      }
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer (even CTA only) ----------------
    if (leader) {
      constexpr uint32_t idesc = idesc_f16_f32(256, 256, /*a MN-major*/ true, /*b K-major*/ false);
      int stage = 0;
      uint32_t phase = 0;
      int it = 0;
      bool ok = true;
      for (int64_t t = pair; ok && t < p.num_tiles; t += num_pairs, ++it) {
        const int buf = it & 1;
        const uint32_t acc_phase = (it >> 1) & 1;
        if (!(ok = __all_sync(0xffffffffu, mbar_wait_bounded(&tmem_empty[buf], acc_phase ^ 1,
                                                             abort_flag, ERR_BIT))))
          break;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + buf * BN;
        for (int kb = 0; kb < p.num_kb; ++kb) {
          if (!(ok = __all_sync(0xffffffffu,
                                mbar_wait_bounded(&full[stage], phase, abort_flag, ERR_BIT))))
            break;
          tc_fence_after();
          const uint32_t sa = smem_u32(smem + stage * P_STAGE_BYTES);
          const uint64_t ad = smem_desc_sw128(sa, A_HALF_BYTES, 1024);
          const uint64_t bd = smem_desc_sw128(sa + P_A_BYTES, 16, 1024);
#pragma unroll
          for (int k = 0; k < BK / 16; ++k)
            mma_f16_ss_pair_elect(d_tmem, ad + (uint64_t)(k * 2048 >> 4),
                                  bd + (uint64_t)(k * 32 >> 4), idesc, (kb | k) != 0);
          mma_commit_pair_both_elect(&empty[stage]);  // frees the stage in both CTAs
          if (++stage == P_STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
        if (!ok) break;
        mma_commit_pair_both_elect(&tmem_full[buf]);
      }
    }
  } else {
    // ---------------- epilogue (warps 2..5 of both CTAs) ----------------
    const int q = warp & 3;
    const uint32_t lane_base = (uint32_t)(q * 32) << 16;
    __half* stage_w = reinterpret_cast<__half*>(epi_stage + q * 2 * EPI_BOX_BYTES);
    const uint32_t tmem_empty_leader = mapa_shared(smem_u32(&tmem_empty[0]), 0);
    int sbuf = 0;
    int it = 0;
    for (int64_t t = pair; t < p.num_tiles && !*abort_flag; t += num_pairs, ++it) {
      const int buf = it & 1;
      const uint32_t acc_phase = (it >> 1) & 1;
      if (!mbar_wait_bounded(&tmem_full[buf], acc_phase, abort_flag, ERR_BIT)) break;
      tc_fence_after();
      int b, mt, nt;
      tile_coords(p, t, b, mt, nt);
      const int m0 = mt * 256 + (int)rank * 128 + q * 32;
      const int m = m0 + lane;
      const int n0 = nt * BN;
      const uint32_t tcol = tmem_base + buf * BN + lane_base;
      if (p.tma_store) {
        auto stage_chunk = [&](uint32_t (&r)[32], int c) {
          if (m0 >= p.M || n0 + c >= p.N) return;
          __half* sb = stage_w + sbuf * (EPI_BOX_BYTES / 2);
          if (lane == 0) bulk_wait_read<1>();
          __syncwarp();
#pragma unroll
          for (int j = 0; j < 32; ++j) sb[j * 32 + lane] = __float2half_rn(__uint_as_float(r[j]));
          fence_async_shared();
          __syncwarp();
          if (lane == 0) {
            tma_store_3d(&tmC, sb, m0, n0 + c, b);
            bulk_commit();
          }
          sbuf ^= 1;
        };
        uint32_t ra[32], rb[32];
        tmem_ld_32x32b_x32(tcol, ra);
#pragma unroll 1
        for (int c = 0; c < BN; c += 64) {
          tmem_ld_wait_regs(ra);
          tmem_ld_32x32b_x32(tcol + c + 32, rb);
          stage_chunk(ra, c);
          tmem_ld_wait_regs(rb);
          if (c + 64 < BN) tmem_ld_32x32b_x32(tcol + c + 64, ra);
          stage_chunk(rb, c + 32);
        }
      } else {
        __half* cb = p.C + (int64_t)b * p.sC;
#pragma unroll 1
        for (int c = 0; c < BN; c += 32) {
          uint32_t r[32];
          tmem_ld_32x32b_x32(tcol + c, r);
          tmem_ld_wait_regs(r);
          if (m < p.M) {
#pragma unroll
            for (int j = 0; j < 32; ++j) {
              const int n = n0 + c + j;
              if (n < p.N)
                cb[(int64_t)m + (int64_t)n * p.ldc] = __float2half_rn(__uint_as_float(r[j]));
            }
          }
        }
      }
      tc_fence_before();
      if (leader) mbar_arrive(&tmem_empty[buf]);
      else mbar_arrive_cluster(tmem_empty_leader + buf * 8);
    }
    if (lane == 0) bulk_wait<0>();
  }

  tc_fence_before();
  cluster_sync_all();  // no CTA leaves while its peer may still touch its shared memory
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc_pair(tmem_base, TMEM_COLS);
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
#ifndef CTB_NO_TMAP_CACHE
  // A tensor map is a pure function of these arguments (base address and
  // geometry, nothing about the memory's contents or lifetime), so a map
  // encoded once can be reused for any later call with the same arguments.
  // Small per-thread cache, round-robin replacement, no locking.
  struct Key {
    const void* base;
    uint64_t dims[5], strides[4];
    uint32_t box[5];
    int32_t dtype, rank, swizzle, pad;
  };
  struct Slot {
    Key key;
    CUtensorMap map;
    bool used;
  };
  static thread_local Slot cache[32];
  static thread_local unsigned next_slot = 0;
  Key k;
  std::memset(&k, 0, sizeof(k));
  k.base = base;
  k.dtype = (int32_t)dtype;
  k.rank = rank;
  k.swizzle = (int32_t)swizzle;
  for (int i = 0; i < rank && i < 5; ++i) {
    k.dims[i] = dims[i];
    k.box[i] = box[i];
    if (i < rank - 1 && i < 4) k.strides[i] = strides_bytes[i];
  }
  for (Slot& sl : cache)
    if (sl.used && std::memcmp(&sl.key, &k, sizeof(k)) == 0) {
      *map = sl.map;
      return CTB_OK;
    }
#endif
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
#ifndef CTB_NO_TMAP_CACHE
  Slot& sl = cache[next_slot++ % 32];
  sl.key = k;
  sl.map = *map;
  sl.used = true;
#endif
  return CTB_OK;
}

int gemm_take_device_error(unsigned int* out) { return take_device_error(out); }

#ifdef CTB_GEMM_TRACE
extern "C" int ctb_gemm_trace_read(unsigned long long* out) {
  return cudaMemcpyFromSymbol(out, gemm::g_gemm_trace, sizeof(gemm::g_gemm_trace)) == cudaSuccess
             ? 0
             : -6;
}
#endif

static unsigned long long g_gemm_attr_done[64];  // context ID the set-up was done in
static int g_gemm_pairs[64];
static std::mutex g_gemm_mu;

int gemm_device_setup() {
  int dev = 0;
  CTB_CUDA_CHECK(cudaGetDevice(&dev));
  std::lock_guard<std::mutex> lk(g_gemm_mu);
  unsigned long long ctx = 0;
  if (int rc = current_context_id(&ctx)) return rc;
  if (dev < 64 && g_gemm_attr_done[dev] == ctx) return CTB_OK;
  CTB_CUDA_CHECK(cudaFuncSetAttribute(gemm::gemm_f16_tcgen05_kernel,
                                      cudaFuncAttributeMaxDynamicSharedMemorySize,
                                      gemm::SMEM_BYTES));
  CTB_CUDA_CHECK(cudaFuncSetAttribute(gemm::gemm_f16_pair_kernel,
                                      cudaFuncAttributeMaxDynamicSharedMemorySize,
                                      gemm::P_SMEM_BYTES));
  // Resident CTA pairs (clusters of 2 at one CTA per SM) for the persistent grid.
  cudaLaunchConfig_t cfg = {};
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.gridDim = dim3(2, 1, 1);
  cfg.blockDim = dim3(gemm::THREADS, 1, 1);
  cfg.dynamicSmemBytes = gemm::P_SMEM_BYTES;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  int clusters = 0;
  CTB_CUDA_CHECK(cudaOccupancyMaxActiveClusters(&clusters, gemm::gemm_f16_pair_kernel, &cfg));
  if (dev < 64) {
    g_gemm_pairs[dev] = clusters;
    g_gemm_attr_done[dev] = ctx;
  }
  return CTB_OK;
}

// Pair kernel choice: CTB_GEMM_PAIR=0 never, =1 whenever possible, unset: when
// the 256 x 256 tiles fill at least one wave of resident pairs.
static int gemm_pair_mode() {
  static const int mode = [] {
    const char* e = getenv("CTB_GEMM_PAIR");
    return e ? (e[0] == '1' ? 1 : 0) : -1;
  }();
  return mode;
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
  CUtensorMap tmC;
  const bool c_tma = tma_ok(C, ldc, sC, batch);
  if (c_tma) {
    const uint64_t dims[3] = {(uint64_t)M, (uint64_t)N, (uint64_t)batch};
    const uint64_t strides[2] = {(uint64_t)ldc * 2,
                                 (uint64_t)(batch > 1 ? sC : ldc * N) * 2};
    const uint32_t box[3] = {32, 32, 1};
    if (int rc = encode_tmap(&tmC, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3, C, dims, strides, box,
                             CU_TENSOR_MAP_SWIZZLE_NONE))
      return rc;
  } else {
    std::memset(&tmC, 0, sizeof(tmC));
  }
  int dev = 0;
  CTB_CUDA_CHECK(cudaGetDevice(&dev));
  const int pairs = (dev >= 0 && dev < 64) ? g_gemm_pairs[dev] : 0;
  const int64_t pair_tiles = (int64_t)((M + 255) / 256) * ((N + 255) / 256) * batch;
  const int mode = gemm_pair_mode();
  if (pairs > 0 && mode != 0 && (mode == 1 || pair_tiles >= pairs)) {
    CUtensorMap tmB2;
    const uint64_t dims[3] = {(uint64_t)K, (uint64_t)N, (uint64_t)batch};
    const uint64_t strides[2] = {(uint64_t)ldb * 2, (uint64_t)(batch > 1 ? sB : ldb * N) * 2};
    const uint32_t box[3] = {gemm::BK, 128, 1};
    if (int rc = encode_tmap(&tmB2, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3, B, dims, strides, box,
                             CU_TENSOR_MAP_SWIZZLE_128B))
      return rc;
    gemm::Params pp;
    pp.tma_store = c_tma ? 1 : 0;
    pp.C = C;
    pp.M = M;
    pp.N = N;
    pp.K = K;
    pp.batch = batch;
    pp.ldc = ldc;
    pp.sC = sC;
    pp.tiles_m = (M + 255) / 256;
    pp.tiles_n = (N + 255) / 256;
    pp.num_kb = (K + gemm::BK - 1) / gemm::BK;
    pp.num_tiles = pair_tiles;
    cudaLaunchConfig_t cfg = {};
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 2;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.gridDim = dim3((unsigned)(2 * std::min<int64_t>(pair_tiles, pairs)), 1, 1);
    cfg.blockDim = dim3(gemm::THREADS, 1, 1);
    cfg.dynamicSmemBytes = gemm::P_SMEM_BYTES;
    cfg.stream = st;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    CTB_CUDA_CHECK(cudaLaunchKernelEx(&cfg, gemm::gemm_f16_pair_kernel, tmA, tmB2, tmC, pp));
    return launch_status("gemm_f16_pair_kernel");
  }
  gemm::Params p;
  p.tma_store = c_tma ? 1 : 0;
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
  gemm::gemm_f16_tcgen05_kernel<<<grid, gemm::THREADS, gemm::SMEM_BYTES, st>>>(tmA, tmB, tmC, p);
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

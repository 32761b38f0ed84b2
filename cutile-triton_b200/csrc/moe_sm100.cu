// Gather-routed mixture-of-experts GEMM on the tcgen05 tensor cores.
//
// The cuTile moe example (benchmarked in the reference at 52 TFLOP/s with
// Triton and 95 with tileiras, research/bench_final.log:7, bench_native.log:10)
// is not vendored, so this follows the published fused-MoE contract (the
// Triton/vLLM `fused_moe` kernel): tokens are sorted by expert and padded to
// blocks of BM = 128 (`sorted_token_ids`, entries >= M*topk are padding);
// `expert_ids[b]` is the expert of block b; `num_tokens_post_padded` (device
// scalar) bounds the blocks in use. For each sorted id s < M*topk in a block
// of expert e:
//   C[s, :] = (A[s / topk, :] . B[e]^T) * (mul_routed_weight ? w[s] : 1)
// with A (M x K) and C (M*topk x N) row-major Float16 and B (E x N x K)
// Float16 with K contiguous; Float32 accumulation in TMEM, Float16 out.
//
// Two launches. (1) moe_gather_rows_kernel copies A[s / topk] into row i
// of a workspace A_perm[EM x K] for every listed slot s = sorted[i] (rows of
// padding slots are skipped: row i of the product depends only on row i of
// A_perm, and those results are never stored). An m-block's rows are read by
// all N / 256 tiles of that block, so gathering them once costs one extra
// pass over M * topk * K halves instead of one gather per tile and stage.
// (2) The GEMM's persistent 128 x 256 x 64 tcgen05 pipeline on A_perm: one
// producer thread loads A_perm's 128 x 64 box and the expert's 256 x 64 B
// slab by TMA per stage; the epilogue thread of TMEM lane r scatters row r of
// the tile to C[s] with 16-byte stores. Every TMA load fills one CTA's own shared memory; every wait is
// bounded.
#include "sm100_ptx.cuh"

#include <algorithm>
#include <cstdlib>
#include <mutex>

namespace ctb {

namespace moe {

constexpr int BM = 128, BN = 256, BK = 64, STAGES = 4;
constexpr int THREADS = 6 * 32;  // 0 TMA producer, 1 MMA, 2-5 epilogue
constexpr int A_STAGE_BYTES = BM * BK * 2;  // 16 KB
constexpr int B_STAGE_BYTES = BN * BK * 2;  // 32 KB
constexpr int STAGE_BYTES = A_STAGE_BYTES + B_STAGE_BYTES;
constexpr int TMEM_COLS = 2 * BN;
constexpr int SMEM_BYTES = STAGES * STAGE_BYTES + 1024 + 256;
constexpr unsigned ERR_BIT = 8u;
#ifndef CTB_MOE_GROUP_ROWS
#define CTB_MOE_GROUP_ROWS 4096
#endif

struct Params {
  const __half* A;
  __half* C;
  const int32_t* sorted;
  const int32_t* expert_ids;
  const int32_t* ntp;  // num_tokens_post_padded (device)
  const float* w;
  int mul;
  int M, N, K, E, EM, topk;
  int64_t lda, ldc;
  int tiles_n, num_kb, num_mblk;  // num_mblk: tiles of tile_rows rows in sorted order
  int group_m;  // m-blocks per raster group
  int bm;         // rows per routing block (128 or 256): one expert per block
  int tile_rows;  // rows per output tile: 128 (one SM) or 256 (a CTA pair, bm == 256)
};

// Blocks in use: those below num_tokens_post_padded.
__device__ __forceinline__ int blocks_in_use(const Params& p) {
  const int ntp = __ldg(p.ntp);
  return max(min(p.num_mblk, (ntp + p.tile_rows - 1) / p.tile_rows), 0);
}

// Raster order: groups of group_m consecutive m-blocks (about one expert's
// tokens), n-tiles outer and m-blocks inner inside a group, so one wave of
// CTAs shares a few B slabs and a few MB of gathered A rows in L2 instead of
// streaming an expert's whole weight matrix per 128-row block.
__device__ __forceinline__ void tile_coords(const Params& p, int mblk, int64_t t, int& mb,
                                            int& n0) {
  const int64_t span = (int64_t)p.group_m * p.tiles_n;
  const int g = (int)(t / span);
  const int first = g * p.group_m;
  const int gsize = min(mblk - first, p.group_m);
  const int rr = (int)(t - g * span);
  mb = first + rr % gsize;
  n0 = (rr / gsize) * BN;
}

__global__ void __launch_bounds__(THREADS, 1)
    moe_gemm_tcgen05_kernel(const __grid_constant__ CUtensorMap tmA,
                            const __grid_constant__ CUtensorMap tmB, const Params p) {
  using namespace sm100;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + STAGES * STAGE_BYTES);
  uint64_t* empty = full + STAGES;
  uint64_t* tmem_full = empty + STAGES;  // [2]
  uint64_t* tmem_empty = tmem_full + 2;  // [2]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tmem_empty + 2);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);  // the producer's expect_tx arrival
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
  const int mblk = blocks_in_use(p);
  const int64_t num_tiles = (int64_t)mblk * p.tiles_n;

  if (warp == 0) {
    // ---------------- producer: A_perm and B by TMA ----------------
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      for (int64_t t = blockIdx.x; t < num_tiles && !*abort_flag; t += gridDim.x) {
        int mb, n0;
        tile_coords(p, mblk, t, mb, n0);
        int e = __ldg(p.expert_ids + (int64_t)mb * p.tile_rows / p.bm);
        if (e < 0 || e >= p.E) e = p.E;  // out of range: the TMA fills zeros
        for (int kb = 0; kb < p.num_kb; ++kb) {
          if (!mbar_wait_bounded(&empty[stage], phase ^ 1, abort_flag, ERR_BIT)) break;
          uint8_t* sa = smem + stage * STAGE_BYTES;
          mbar_arrive_expect_tx(&full[stage], STAGE_BYTES);
          tma_load_2d(sa, &tmA, &full[stage], kb * BK, mb * BM);
          tma_load_3d(sa + A_STAGE_BYTES, &tmB, &full[stage], kb * BK, n0, e);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
      }
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer (warp-converged, elect.sync issues) ----------------
    constexpr uint32_t idesc = idesc_f16_f32(BM, BN, false, false);  // A, B both K-major
    int stage = 0;
    uint32_t phase = 0;
    int it = 0;
    bool ok = true;
    for (int64_t t = blockIdx.x; ok && t < num_tiles; t += gridDim.x, ++it) {
      const int buf = it & 1;
      if (!(ok = __all_sync(0xffffffffu, mbar_wait_bounded(&tmem_empty[buf], ((it >> 1) & 1) ^ 1,
                                                           abort_flag, ERR_BIT))))
        break;
      tc_fence_after();
      const uint32_t d_tmem = tmem_base + buf * BN;
      for (int kb = 0; kb < p.num_kb; ++kb) {
        if (!(ok = __all_sync(0xffffffffu,
                              mbar_wait_bounded(&full[stage], phase, abort_flag, ERR_BIT))))
          break;
        tc_fence_after();
        const uint32_t sa = smem_u32(smem + stage * STAGE_BYTES);
        const uint64_t ad = smem_desc_sw128(sa, 16, 1024);
        const uint64_t bd = smem_desc_sw128(sa + A_STAGE_BYTES, 16, 1024);
#pragma unroll
        for (int k = 0; k < BK / 16; ++k)  // 16 halves = 32 bytes inside the swizzled row
          mma_f16_ss_elect(d_tmem, ad + (uint64_t)(k * 32 >> 4), bd + (uint64_t)(k * 32 >> 4),
                           idesc, (kb | k) != 0);
        mma_commit_elect(&empty[stage]);
        if (++stage == STAGES) {
          stage = 0;
          phase ^= 1;
        }
      }
      if (!ok) break;
      mma_commit_elect(&tmem_full[buf]);
    }
  } else {
    // ---------------- epilogue (warps 2..5): scatter rows to C ----------------
    const int q = warp & 3;
    const uint32_t lane_base = (uint32_t)(q * 32) << 16;
    const int r = q * 32 + lane;
    int it = 0;
    for (int64_t t = blockIdx.x; t < num_tiles; t += gridDim.x, ++it) {
      const int buf = it & 1;
      if (!mbar_wait_bounded(&tmem_full[buf], (it >> 1) & 1, abort_flag, ERR_BIT)) break;
      tc_fence_after();
      int mb, n0;
      tile_coords(p, mblk, t, mb, n0);
      const int sid = __ldg(p.sorted + (int64_t)mb * BM + r);
      const int e = __ldg(p.expert_ids + (int64_t)mb * p.tile_rows / p.bm);
      const bool valid = sid >= 0 && sid < p.M * p.topk && e >= 0 && e < p.E;
      const float wt = (valid && p.mul) ? __ldg(p.w + sid) : 1.f;
      __half* crow = p.C + (int64_t)(valid ? sid : 0) * p.ldc;
#pragma unroll 1
      for (int c = 0; c < BN; c += 32) {
        uint32_t v[32];
        tmem_ld_32x32b_x32(tmem_base + buf * BN + c + lane_base, v);
        tmem_ld_wait();
        const int n = n0 + c;
        if (!valid || n >= p.N) continue;
        if (n + 32 <= p.N) {
          uint4* dst = reinterpret_cast<uint4*>(crow + n);
#pragma unroll
          for (int u = 0; u < 4; ++u) {
            uint4 o;
            uint32_t* ow = &o.x;
#pragma unroll
            for (int h = 0; h < 4; ++h) {
              __half2 hv = __floats2half2_rn(__uint_as_float(v[8 * u + 2 * h]) * wt,
                                             __uint_as_float(v[8 * u + 2 * h + 1]) * wt);
              ow[h] = *reinterpret_cast<uint32_t*>(&hv);
            }
            dst[u] = o;
          }
        } else {
#pragma unroll
          for (int i = 0; i < 32; ++i)
            if (n + i < p.N) crow[n + i] = __float2half_rn(__uint_as_float(v[i]) * wt);
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

// CTA-pair variant for 256-row routing blocks (every block of one expert):
// the even CTA of a cluster of two issues 256 x 256 x 16 tcgen05 MMAs
// (cta_group::2) over both CTAs' operands; each CTA loads its own 128 rows of
// A_perm and 128 columns of the expert's B by TMA (32 KB per k-block, counted
// on the even CTA's full barrier), keeps its 128 accumulator rows in its own
// tensor memory and scatters them itself. Same barrier protocol as the pair
// GEMM: commits to both CTAs free stages and publish accumulators,
// both CTAs' epilogue threads arrive on the even CTA's accumulator-empty
// barrier, cluster barriers at start and end.
constexpr int P_STAGES = 6;
constexpr int P_A_BYTES = 128 * BK * 2;
constexpr int P_B_BYTES = 128 * BK * 2;
constexpr int P_STAGE_BYTES = P_A_BYTES + P_B_BYTES;
constexpr int P_SMEM_BYTES = P_STAGES * P_STAGE_BYTES + 1024 + 256;

__global__ void __launch_bounds__(THREADS, 1)
    moe_gemm_pair_kernel(const __grid_constant__ CUtensorMap tmA,
                         const __grid_constant__ CUtensorMap tmB, const Params p) {
  using namespace sm100;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + P_STAGES * P_STAGE_BYTES);
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
  }
  if (warp == 1) tmem_alloc_pair(tmem_slot, TMEM_COLS);
  tc_fence_before();
  cluster_sync_all();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  const int mblk = blocks_in_use(p);
  const int64_t num_tiles = (int64_t)mblk * p.tiles_n;
  const uint32_t full_leader = mapa_shared(smem_u32(&full[0]), 0);

  if (warp == 0) {
    // ---------------- producer (both CTAs): own halves of A_perm and B ----------------
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      for (int64_t t = pair; t < num_tiles && !*abort_flag; t += num_pairs) {
        int mb, n0;
        tile_coords(p, mblk, t, mb, n0);
        int e = __ldg(p.expert_ids + (int64_t)mb * p.tile_rows / p.bm);
        if (e < 0 || e >= p.E) e = p.E;  // out of range: the TMA fills zeros
        const int row0 = mb * 256 + (int)rank * 128, col0 = n0 + (int)rank * 128;
        for (int kb = 0; kb < p.num_kb; ++kb) {
          if (!mbar_wait_bounded(&empty[stage], phase ^ 1, abort_flag, ERR_BIT)) break;
          uint8_t* sa = smem + stage * P_STAGE_BYTES;
          if (leader) mbar_arrive_expect_tx(&full[stage], 2 * P_STAGE_BYTES);
          const uint32_t bar = full_leader + stage * 8;
          tma_load_2d_pair(sa, &tmA, bar, kb * BK, row0);
          tma_load_3d_pair(sa + P_A_BYTES, &tmB, bar, kb * BK, col0, e);
          if (++stage == P_STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
      }
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer (even CTA) ----------------
    if (leader) {
      constexpr uint32_t idesc = idesc_f16_f32(256, BN, false, false);  // A, B both K-major
      int stage = 0;
      uint32_t phase = 0;
      int it = 0;
      bool ok = true;
      for (int64_t t = pair; ok && t < num_tiles; t += num_pairs, ++it) {
        const int buf = it & 1;
        if (!(ok = __all_sync(0xffffffffu, mbar_wait_bounded(&tmem_empty[buf],
                                                             ((it >> 1) & 1) ^ 1, abort_flag,
                                                             ERR_BIT))))
          break;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + buf * BN;
        for (int kb = 0; kb < p.num_kb; ++kb) {
          if (!(ok = __all_sync(0xffffffffu,
                                mbar_wait_bounded(&full[stage], phase, abort_flag, ERR_BIT))))
            break;
          tc_fence_after();
          const uint32_t sa = smem_u32(smem + stage * P_STAGE_BYTES);
          const uint64_t ad = smem_desc_sw128(sa, 16, 1024);
          const uint64_t bd = smem_desc_sw128(sa + P_A_BYTES, 16, 1024);
#pragma unroll
          for (int k = 0; k < BK / 16; ++k)
            mma_f16_ss_pair_elect(d_tmem, ad + (uint64_t)(k * 32 >> 4),
                                  bd + (uint64_t)(k * 32 >> 4), idesc, (kb | k) != 0);
          mma_commit_pair_both_elect(&empty[stage]);
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
    // ---------------- epilogue (warps 2..5 of both CTAs): scatter rows ----------------
    const int q = warp & 3;
    const uint32_t lane_base = (uint32_t)(q * 32) << 16;
    const int r = (int)rank * 128 + q * 32 + lane;  // row within the 256-row block
    const uint32_t tmem_empty_leader = mapa_shared(smem_u32(&tmem_empty[0]), 0);
    int it = 0;
    for (int64_t t = pair; t < num_tiles; t += num_pairs, ++it) {
      const int buf = it & 1;
      if (!mbar_wait_bounded(&tmem_full[buf], (it >> 1) & 1, abort_flag, ERR_BIT)) break;
      tc_fence_after();
      int mb, n0;
      tile_coords(p, mblk, t, mb, n0);
      const int sid = __ldg(p.sorted + (int64_t)mb * 256 + r);
      const int e = __ldg(p.expert_ids + (int64_t)mb * p.tile_rows / p.bm);
      const bool valid = sid >= 0 && sid < p.M * p.topk && e >= 0 && e < p.E;
      const float wt = (valid && p.mul) ? __ldg(p.w + sid) : 1.f;
      __half* crow = p.C + (int64_t)(valid ? sid : 0) * p.ldc;
#pragma unroll 1
      for (int c = 0; c < BN; c += 32) {
        uint32_t v[32];
        tmem_ld_32x32b_x32(tmem_base + buf * BN + c + lane_base, v);
        tmem_ld_wait_regs(v);
        const int n = n0 + c;
        if (!valid || n >= p.N) continue;
        if (n + 32 <= p.N) {
          uint4* dst = reinterpret_cast<uint4*>(crow + n);
#pragma unroll
          for (int u = 0; u < 4; ++u) {
            uint4 o;
            uint32_t* ow = &o.x;
#pragma unroll
            for (int h = 0; h < 4; ++h) {
              __half2 hv = __floats2half2_rn(__uint_as_float(v[8 * u + 2 * h]) * wt,
                                             __uint_as_float(v[8 * u + 2 * h + 1]) * wt);
              ow[h] = *reinterpret_cast<uint32_t*>(&hv);
            }
            dst[u] = o;
          }
        } else {
#pragma unroll
          for (int i = 0; i < 32; ++i)
            if (n + i < p.N) crow[n + i] = __float2half_rn(__uint_as_float(v[i]) * wt);
        }
      }
      tc_fence_before();
      if (leader) mbar_arrive(&tmem_empty[buf]);
      else mbar_arrive_cluster(tmem_empty_leader + buf * 8);
    }
  }

  tc_fence_before();
  cluster_sync_all();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc_pair(tmem_base, TMEM_COLS);
  }
}

// Row i of A_perm = A[sorted[i] / topk] for listed slots of blocks in use.
// One CTA per EM row; 16-byte vectors (K is a multiple of 8).
__global__ void __launch_bounds__(128) moe_gather_rows_kernel(const Params p, __half* Ap,
                                                               int64_t ldp) {
  const int i = blockIdx.x;
  if (i >= blocks_in_use(p) * p.tile_rows) return;
  const int sid = __ldg(p.sorted + i);
  if (sid < 0 || sid >= p.M * p.topk) return;
  const uint4* src = reinterpret_cast<const uint4*>(p.A + (int64_t)(sid / p.topk) * p.lda);
  uint4* dst = reinterpret_cast<uint4*>(Ap + (int64_t)i * ldp);
  for (int v = threadIdx.x; v < p.K / 8; v += blockDim.x) dst[v] = __ldg(src + v);
}

}  // namespace moe

int moe_take_device_error(unsigned int* out) { return take_device_error(out); }

static unsigned long long g_moe_attr_done[64];  // context ID the set-up was done in
static int g_moe_pairs[64];
static std::mutex g_moe_mu;

static int moe_device_setup() {
  int dev = 0;
  CTB_CUDA_CHECK(cudaGetDevice(&dev));
  std::lock_guard<std::mutex> lk(g_moe_mu);
  unsigned long long ctx = 0;
  if (int rc = current_context_id(&ctx)) return rc;
  if (dev < 64 && g_moe_attr_done[dev] == ctx) return CTB_OK;
  CTB_CUDA_CHECK(cudaFuncSetAttribute(moe::moe_gemm_tcgen05_kernel,
                                      cudaFuncAttributeMaxDynamicSharedMemorySize,
                                      moe::SMEM_BYTES));
  CTB_CUDA_CHECK(cudaFuncSetAttribute(moe::moe_gemm_pair_kernel,
                                      cudaFuncAttributeMaxDynamicSharedMemorySize,
                                      moe::P_SMEM_BYTES));
  cudaLaunchConfig_t cfg = {};
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.gridDim = dim3(2, 1, 1);
  cfg.blockDim = dim3(moe::THREADS, 1, 1);
  cfg.dynamicSmemBytes = moe::P_SMEM_BYTES;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  int clusters = 0;
  CTB_CUDA_CHECK(cudaOccupancyMaxActiveClusters(&clusters, moe::moe_gemm_pair_kernel, &cfg));
  if (dev < 64) {
    g_moe_pairs[dev] = clusters;
    g_moe_attr_done[dev] = ctx;
  }
  return CTB_OK;
}

}  // namespace ctb

using namespace ctb;

extern "C" int64_t ctb_moe_workspace_bytes(int32_t EM, int32_t K) {
  return EM > 0 && K > 0 ? (int64_t)EM * K * 2 : 0;
}

extern "C" int ctb_moe_gemm_f16(const void* A, const void* B, void* C,
                                const int32_t* sorted_token_ids, const int32_t* expert_ids,
                                const int32_t* num_tokens_post_padded, const float* topk_weights,
                                int32_t mul_routed_weight, int32_t M, int32_t N, int32_t K,
                                int32_t E, int32_t EM, int32_t topk, int32_t block_m,
                                int64_t lda, int64_t ldb, int64_t ldc, void* workspace,
                                int64_t workspace_bytes, void* stream) {
  clear_error();
  if (M < 0 || N < 0 || K < 0 || E < 1 || EM < 0 || topk < 1)
    return set_error(CTB_ERR_SHAPE, "moe: bad sizes");
  if (block_m != 128 && block_m != 256)
    return set_error(CTB_ERR_SHAPE, "moe: block_m must be 128 or 256");
  if (EM % block_m != 0)
    return set_error(CTB_ERR_SHAPE, "moe: sorted_token_ids length must be a multiple of block_m");
  if ((int64_t)M * topk == 0 || N == 0 || EM == 0) return CTB_OK;
  if (K == 0) return set_error(CTB_ERR_SHAPE, "moe: K must be positive");
  if (!A || !B || !C || !sorted_token_ids || !expert_ids || !num_tokens_post_padded ||
      (mul_routed_weight && !topk_weights) || !workspace)
    return set_error(CTB_ERR_ARG, "moe: NULL pointer");
  if (workspace_bytes < ctb_moe_workspace_bytes(EM, K) || !aligned16(workspace))
    return set_error(CTB_ERR_ARG,
                     "moe: workspace must be 16-byte aligned and hold EM x K Float16");
  if (K % 8 || lda % 8 || ldc % 8 || ldb % 8 || lda < K || ldb < K || ldc < N ||
      !aligned16(A) || !aligned16(B) || !aligned16(C))
    return set_error(CTB_ERR_LAYOUT,
                     "moe: K and the row strides must be multiples of 8, pointers 16-byte aligned");
  DeviceProps pr;
  if (int rc = current_props(&pr)) return rc;
  if (int rc = moe_device_setup()) return rc;
  CUtensorMap tmA, tmB;
  const uint64_t dimsA[2] = {(uint64_t)K, (uint64_t)EM};
  const uint64_t stridesA[1] = {(uint64_t)K * 2};
  const uint32_t boxA[2] = {moe::BK, moe::BM};
  if (int rc = encode_tmap(&tmA, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, workspace, dimsA, stridesA,
                           boxA, CU_TENSOR_MAP_SWIZZLE_128B))
    return rc;
  const uint64_t dims[3] = {(uint64_t)K, (uint64_t)N, (uint64_t)E};
  const uint64_t strides[2] = {(uint64_t)ldb * 2, (uint64_t)ldb * N * 2};
  const uint32_t box[3] = {moe::BK, moe::BN, 1};
  if (int rc = encode_tmap(&tmB, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3, B, dims, strides, box,
                           CU_TENSOR_MAP_SWIZZLE_128B))
    return rc;
  moe::Params p;
  p.A = (const __half*)A;
  p.C = (__half*)C;
  p.sorted = sorted_token_ids;
  p.expert_ids = expert_ids;
  p.ntp = num_tokens_post_padded;
  p.w = topk_weights;
  p.mul = mul_routed_weight ? 1 : 0;
  p.M = M;
  p.N = N;
  p.K = K;
  p.E = E;
  p.EM = EM;
  p.topk = topk;
  p.lda = lda;
  p.ldc = ldc;
  p.tiles_n = (N + moe::BN - 1) / moe::BN;
  p.num_kb = (K + moe::BK - 1) / moe::BK;
  // 256-row blocks run on CTA pairs unless CTB_MOE_PAIR=0 or no pair can be
  // resident; the single-SM kernel serves any block size (per 128-row tile).
  int pairs = 0;
  {
    int dev = 0;
    CTB_CUDA_CHECK(cudaGetDevice(&dev));
    pairs = (dev >= 0 && dev < 64) ? g_moe_pairs[dev] : 0;
  }
  static const bool pair_off = [] {
    const char* e = getenv("CTB_MOE_PAIR");
    return e && e[0] == '0';
  }();
  const bool use_pair = block_m == 256 && pairs > 0 && !pair_off;
  p.bm = block_m;
  p.tile_rows = use_pair ? 256 : 128;
  p.num_mblk = EM / p.tile_rows;
  // Raster groups of about 4096 routed rows (32 blocks of 128 measured best of
  // 1..300 blocks on the 8-expert top-2 workload; the same rows for 256-row blocks).
  p.group_m = std::max(1, CTB_MOE_GROUP_ROWS / p.tile_rows);
  const int64_t max_tiles = (int64_t)p.num_mblk * p.tiles_n;
  const int grid = (int)std::min<int64_t>(max_tiles, pr.sm_count);
  moe::moe_gather_rows_kernel<<<EM, 128, 0, static_cast<cudaStream_t>(stream)>>>(
      p, (__half*)workspace, K);
  if (int rc = launch_status("moe_gather_rows_kernel")) return rc;
  if (use_pair) {
    CUtensorMap tmB2;
    const uint32_t box2[3] = {moe::BK, 128, 1};
    if (int rc = encode_tmap(&tmB2, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3, B, dims, strides, box2,
                             CU_TENSOR_MAP_SWIZZLE_128B))
      return rc;
    cudaLaunchConfig_t cfg = {};
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 2;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.gridDim = dim3((unsigned)(2 * std::min<int64_t>(max_tiles, pairs)), 1, 1);
    cfg.blockDim = dim3(moe::THREADS, 1, 1);
    cfg.dynamicSmemBytes = moe::P_SMEM_BYTES;
    cfg.stream = static_cast<cudaStream_t>(stream);
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    CTB_CUDA_CHECK(cudaLaunchKernelEx(&cfg, moe::moe_gemm_pair_kernel, tmA, tmB2, p));
    return launch_status("moe_gemm_pair_kernel");
  }
  moe::moe_gemm_tcgen05_kernel<<<grid, moe::THREADS, moe::SMEM_BYTES,
                                 static_cast<cudaStream_t>(stream)>>>(tmA, tmB, p);
  return launch_status("moe_gemm_tcgen05_kernel");
}

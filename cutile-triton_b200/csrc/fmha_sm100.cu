// Attention forward on the 5th-generation tensor cores (tcgen05), head_dim 64 or 128
// (the one-SM kernel is a template on head_dim; the CTA-pair variant is 128 only).
//
// cuTile example fmha.jl:20 (not vendored in the reference; report.html:2981
// describes its 4-D tiles with head_dim contiguous): O = softmax(scale*QK^T
// [+ causal mask]) V per (batch, head), Float16 Q/K/V/O, Float32 scores,
// running max/sum and output accumulator.
//
// One CTA = one (batch*head, 256-query block), split into two 128-row query
// tiles Q0/Q1 that ping-pong: while softmax warpgroup 0 turns S0 into P0,
// the tensor core computes S1 (or P1*V), and vice versa.
//   warps 0-3   softmax + epilogue for Q0, one thread per query row holding
//               its 128 scores in registers (warp w reads TMEM lanes 32*(w%4))
//   warps 4-7   softmax + epilogue for Q1
//   warp  8     TMEM owner + MMA issuer (one thread)
//   warp  9     TMA producer (one thread): Q once, then a 2-stage K / V ring
//   warps 10-15 idle; with warps 8-9 they lend registers (setmaxnreg) so the
//               softmax warps can run at 192 registers
// TMEM (512 columns): S0 [0,128) S1 [128,256) O0 [256,256+HD) O1 [256+HD,256+2HD).
// P_t (Float16, two per 32-bit column) overwrites S_t columns 0-63 once the
// row's scores are in registers, and feeds P_t*V as the TMEM A operand.
// Scores are kept in log2 units (exp2 with scale*log2(e) folded in). The
// running max is only moved when it grows by more than 8 (a factor 256), so
// the O rescale in TMEM is rare; numerator and denominator always share the
// same max, so the result is unchanged.
// Every TMA load fills one CTA's own shared memory; every wait is bounded.
#include "sm100_ptx.cuh"

#include <algorithm>
#include <mutex>
#include <type_traits>

namespace ctb {

int fmha_simt(const __half* Q, const __half* K, const __half* V, __half* O, int B, int H, int Sq,
              int Sk, int D, float scale, int causal, cudaStream_t st);

namespace fmha {

constexpr int D = 128;            // head dim handled by this kernel
constexpr int BQ = 128;           // rows per query tile (UMMA M)
constexpr int BKV = 128;          // keys per block (UMMA N of S, K of P*V)
constexpr int SM_THREADS_PER_TILE = 128;      // 4 softmax warps per query tile
constexpr int MMA_WARP = 8, TMA_WARP = 9;     // warps 10-15 only lend registers
constexpr int THREADS = 16 * 32;
// Register split (setmaxnreg): launched at 128 per thread (512 x 128 = 65536);
// the two softmax warpgroups rise to 192, the other two drop to 64:
// 256 x 192 + 256 x 64 = 65536.
constexpr int REG_SOFTMAX = 192, REG_OTHER = 64;
constexpr int TILE_BYTES = BQ * D * 2;       // 32 KB: one 128 x 128 f16 tile
constexpr int HALF_BYTES = TILE_BYTES / 2;   // one 64-wide (128-byte) TMA box
constexpr int BOX_BYTES = BQ * 64 * 2;       // one 128-row x 64-column TMA box (16 KB)
// The one-SM kernel is built for head_dim HD = 64 or 128 (HD / 64 boxes per tile).
template <int HD> __host__ __device__ constexpr int tile_bytes() { return BQ * HD * 2; }
template <int HD> __host__ __device__ constexpr int smem_bytes() { return 6 * tile_bytes<HD>() + 1024 + 256; }
constexpr float RESCALE_THRESHOLD = 8.0f;    // log2 units
#ifndef CTB_FMHA_P_PARTS
#define CTB_FMHA_P_PARTS 2
#endif
constexpr int P_PARTS = CTB_FMHA_P_PARTS;     // P published in this many key ranges per block
static_assert(P_PARTS == 1 || P_PARTS == 2 || P_PARTS == 4, "P is published in 1, 2 or 4 parts");
static_assert(BKV / 16 % P_PARTS == 0, "each part must hold whole 16-key MMA steps");
// Timing probes (wrong results; never the default): 1 = no exponentials,
// 3 = no exponentials and no TMEM traffic from the softmax warps. 0 = the kernel.
#ifndef CTB_FMHA_EXP_MODE
#define CTB_FMHA_EXP_MODE 0
#endif
// Timing probe (wrong results; never the default): 1 = skip the P*V MMAs, 2 = skip the S MMAs.
#ifndef CTB_FMHA_SKIP
#define CTB_FMHA_SKIP 0
#endif
#ifndef CTB_FMHA_HEAD_MAJOR
#define CTB_FMHA_HEAD_MAJOR 1
#endif
constexpr unsigned ERR_BIT = 2u;

struct Params {
  __half* O;
  int Sq, Sk, BH, n_qblk;
  float scale_log2;
  int causal;
};

__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

__device__ __forceinline__ uint32_t pack_half2(float lo, float hi) {
  __half2 h = __floats2half2_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&h);
}

// ---- paired fp32 arithmetic (sm_100 f32x2 instructions) -----------------------
__device__ __forceinline__ uint64_t f2_pack(float a, float b) {
  uint64_t r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(a), "f"(b));
  return r;
}
__device__ __forceinline__ void f2_unpack(uint64_t v, float& a, float& b) {
  asm("mov.b64 {%0, %1}, %2;" : "=f"(a), "=f"(b) : "l"(v));
}
__device__ __forceinline__ uint64_t f2_fma(uint64_t a, uint64_t b, uint64_t c) {
  uint64_t r;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(r) : "l"(a), "l"(b), "l"(c));
  return r;
}
__device__ __forceinline__ uint64_t f2_add(uint64_t a, uint64_t b) {
  uint64_t r;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
  return r;
}
__device__ __forceinline__ uint64_t f2_sub(uint64_t a, uint64_t b) {
  uint64_t r;
  asm("sub.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
  return r;
}
__device__ __forceinline__ float max3(float a, float b, float c) {
  float r;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(r) : "f"(a), "f"(b), "f"(c));
  return r;
}

// 2^x for a pair on the FMA pipe, x in [-126, 126]: Cody-Waite split
// x = j + f with j = round(x) (1.5*2^23 rounding shifter) and f in
// [-0.5, 0.5]; 2^f from a degree-3 polynomial fitted here for minimum
// relative error on [-0.5, 0.5] (max 7.5e-5, below Float16's half ulp);
// 2^j added to the exponent field. Offloads the MUFU ex2 unit.
__device__ __forceinline__ uint64_t exp2_poly2(uint64_t x) {
  const uint64_t shifter = f2_pack(12582912.0f, 12582912.0f);
  const uint64_t t = f2_add(x, shifter);
  const uint64_t f = f2_sub(x, f2_sub(t, shifter));
  uint64_t p = f2_fma(f2_pack(0.05517146f, 0.05517146f), f, f2_pack(0.24261075f, 0.24261075f));
  p = f2_fma(p, f, f2_pack(0.69326097f, 0.69326097f));
  p = f2_fma(p, f, f2_pack(0.9999281f, 0.9999281f));
  float pa, pb, ta, tb;
  f2_unpack(p, pa, pb);
  f2_unpack(t, ta, tb);
  const float ra = __int_as_float(__float_as_int(pa) + (__float_as_int(ta) << 23));
  const float rb = __int_as_float(__float_as_int(pb) + (__float_as_int(tb) << 23));
  return f2_pack(ra, rb);
}

#ifdef CTB_FMHA_TRACE
// Debug-only timeline of CTA 0 (clock64 cycles): [event][block] where events
// are 0/1 softmax tile t got S (t = 0, 1), 2/3 softmax tile t arrived P,
// 4/5 MMA issued P_t*V, 6/7 MMA issued S_t(j+1), 8 MMA got V.
__device__ long long g_fmha_trace[15][128];  // 9-12: completion of PV0, S0', PV1, S1'
__device__ long long g_fmha_mma[4][9];  // block 30 of CTA 0: stamps around each MMA issue
__device__ long long g_fmha_clk[4];     // CTA 0, thread 0: clock64 / globaltimer at start and end
__device__ long long g_fmha_sm[2][10];  // CTA 0 block 30, first thread of each softmax tile
#define FMHA_SM_STAMP(t, i, j)                                                               \
  do {                                                                                     \
    if (blockIdx.x == 0 && (j) == 30 && threadIdx.x % 128 == 0) g_fmha_sm[(t)][(i)] = clock64(); \
  } while (0)
#define FMHA_MMA_STAMP(g, i, on)                                          \
  do {                                                                    \
    if ((on) && blockIdx.x == 0) g_fmha_mma[(g)][(i)] = clock64();        \
  } while (0)
#define FMHA_TRACE(ev, j)                                                      \
  do {                                                                       \
    if (blockIdx.x == 0 && (j) < 128) g_fmha_trace[(ev)][(j)] = clock64();   \
  } while (0)
#else
#define FMHA_TRACE(ev, j) \
  do {                    \
  } while (0)
#define FMHA_MMA_STAMP(g, i, on) \
  do {                           \
  } while (0)
#define FMHA_SM_STAMP(t, i, j) \
  do {                         \
  } while (0)
#endif

__device__ __forceinline__ void named_barrier_sync(int id, int nthreads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(nthreads) : "memory");
}

// Pairs of P evaluated with exp2_poly2 instead of MUFU ex2: one in EMU_EVERY.
#ifndef CTB_FMHA_EMU_EVERY
#define CTB_FMHA_EMU_EVERY 1000  // measured fastest on B200: no offload
#endif
constexpr int EMU_EVERY = CTB_FMHA_EMU_EVERY;

// S_t = Q_t K^T for one key block: HD/16 MMAs of K = 16 over head_dim, Q and
// K both K-major 128-byte-swizzled (HD/64 boxes 64 wide, 16 KB each).
template <int HD>
__device__ __forceinline__ void issue_s(uint32_t tmem, uint32_t sQa, uint32_t sKa, int t,
                                        int stage, uint64_t* s_full_t, bool tr = false) {
  using namespace sm100;
  constexpr uint32_t idesc_s = idesc_f16_f32(BQ, BKV, false, false);
  const uint32_t qa = sQa + t * tile_bytes<HD>(), ka = sKa + stage * tile_bytes<HD>();
  FMHA_MMA_STAMP(2 * t, 0, tr);
#if CTB_FMHA_SKIP == 2
  mma_commit_elect(s_full_t);
  return;  // timing probe: no S MMAs
#endif
#pragma unroll
  for (int kk = 0; kk < HD / 16; ++kk) {
    const uint32_t off = (kk >> 2) * BOX_BYTES + (kk & 3) * 32;
    mma_f16_ss_elect(tmem + t * BKV, smem_desc_sw128(qa + off, 16, 1024),
               smem_desc_sw128(ka + off, 16, 1024), idesc_s, kk != 0);
    FMHA_MMA_STAMP(2 * t, kk + 1, tr);
  }
  mma_commit_elect(s_full_t);
}

// O_t (+)= P_t V for one half (64 keys) of a key block: P_t from TMEM (128 keys packed in S_t
// columns 0-63; 16 keys = 8 columns per step), V as an MN-major B operand: 64-wide head_dim blocks at LBO = 16 KB,
// 8-key groups at SBO = 1 KB, 16 keys per step = 2 KB.
template <int HD>
__device__ __forceinline__ void issue_pv(uint32_t tmem, uint32_t sVa, int t, int stage, int j,
                                         int part, bool tr = false) {
  using namespace sm100;
  constexpr uint32_t idesc_o = idesc_f16_f32(BQ, HD, false, true);
  constexpr int STEPS = BKV / 16 / P_PARTS;  // 16-key MMA steps per published part
  const uint32_t va = sVa + stage * tile_bytes<HD>();
#if CTB_FMHA_SKIP == 1
  return;  // timing probe: no P*V MMAs
#endif
#pragma unroll
  for (int k4 = 0; k4 < STEPS; ++k4) {
    const int kk = part * STEPS + k4;
    if (kk == 0) FMHA_MMA_STAMP(2 * t + 1, 0, tr);
    mma_f16_ts_elect(tmem + 256 + t * HD, tmem + t * BKV + kk * 8,
                     smem_desc_sw128(va + kk * 2048, BOX_BYTES, 1024), idesc_o,
                     (j > 0 || kk > 0) ? 1u : 0u);
    FMHA_MMA_STAMP(2 * t + 1, kk + 1, tr);
  }
}

// Softmax and epilogue of one query tile, one thread per query row (TMEM
// lane): for each of the tile's nb key blocks, read S from TMEM, mask, update
// the running max (rescaling O in TMEM when it moves), write P over S and
// signal it per published part through `arrive_p(part)`; then normalise O
// and store the row. `tile_row0` is the first query row of this CTA's part
// of the tile (rows below it never need the causal mask for a block ending
// at or before it).
template <int HD, class ArriveP>
__device__ __forceinline__ void softmax_rows(const Params& p, int t, uint32_t s_col,
                                             uint32_t o_col, int qrow, int tile_row0, int bh,
                                             int nb, uint64_t* s_full_t, uint64_t* o_full_t,
                                             volatile int* abort_flag, ArriveP&& arrive_p) {
  using namespace sm100;
  [[maybe_unused]] const int lane = threadIdx.x % 32;  // timing probe only
  const float sl2 = p.scale_log2;
  float m_use = -INFINITY, l = 0.f;
  for (int j = 0; j < nb; ++j) {
    // Warp-uniform, so a warp never splits around the per-warp P arrivals.
    if (!__all_sync(0xffffffffu, mbar_wait_bounded(s_full_t, j & 1, abort_flag, ERR_BIT))) break;
    if (threadIdx.x % 128 == 0) FMHA_TRACE(t, j);
    FMHA_SM_STAMP(t, 0, j);
    tc_fence_after();
    uint32_t r[4][32];
#pragma unroll
    for (int c = 0; c < 4; ++c) {
#if CTB_FMHA_EXP_MODE == 3
#pragma unroll
      for (int i = 0; i < 32; ++i) r[c][i] = __float_as_uint((float)(i - lane));  // probe: no S read
#else
      tmem_ld_32x32b_x32(s_col + c * 32, r[c]);
#endif
    }
    const int k0 = j * BKV;
    const bool need_mask = (k0 + BKV > p.Sk) || (p.causal && k0 + BKV - 1 > tile_row0);
    tmem_ld_wait();
    FMHA_SM_STAMP(t, 1, j);
    if (need_mask) {
#pragma unroll
      for (int c = 0; c < 4; ++c)
#pragma unroll
        for (int i = 0; i < 32; ++i) {
          const int key = k0 + c * 32 + i;
          if (key >= p.Sk || (p.causal && key > qrow)) r[c][i] = __float_as_uint(-INFINITY);
        }
    }
    float mx[4];
#pragma unroll
    for (int c = 0; c < 4; ++c) {
      mx[c] = __uint_as_float(r[c][0]);
#pragma unroll
      for (int i = 1; i < 31; i += 2)
        mx[c] = max3(mx[c], __uint_as_float(r[c][i]), __uint_as_float(r[c][i + 1]));
      mx[c] = fmaxf(mx[c], __uint_as_float(r[c][31]));
    }
    const float m_blk = fmaxf(fmaxf(mx[0], mx[1]), fmaxf(mx[2], mx[3])) * sl2;
    FMHA_SM_STAMP(t, 2, j);
    float factor = 1.f;
    bool rescale = false;
    if (j == 0) {
      m_use = m_blk;
    } else if (m_blk > m_use + RESCALE_THRESHOLD) {
      factor = ex2(m_use - m_blk);
      l *= factor;
      m_use = m_blk;
      rescale = true;
    }
    if (__any_sync(0xffffffffu, rescale)) {
      // O_t is stable here: P_t*V of block j-1 completed before S_t of block j,
      // and P_t*V of block j waits for this thread's p_full arrivals below.
#pragma unroll 1
      for (int c = 0; c < HD / 16; ++c) {
        uint32_t o[16];
        tmem_ld_32x32b_x16(o_col + c * 16, o);
        tmem_ld_wait();
#pragma unroll
        for (int i = 0; i < 16; ++i) o[i] = __float_as_uint(__uint_as_float(o[i]) * factor);
        tmem_st_32x32b_x16(o_col + c * 16, o);
      }
    }
    FMHA_SM_STAMP(t, 3, j);
    // Rows whose keys are all masked so far keep m_use = -inf; exp2 of
    // (-inf) - (-inf) would be NaN, so shift by 0 for them.
    const float mref = (m_use == -INFINITY) ? 0.f : m_use;
    const uint64_t sl2x2 = f2_pack(sl2, sl2), nm2 = f2_pack(-mref, -mref);
    uint64_t acc0 = 0, acc1 = 0;  // paired partial row sums (+0.0f bit patterns)
    // P chunk c (16 packed columns) lands in columns [16c, 16c + 16), all read
    // above. Each half (keys 0-63, 64-127) is published as soon as it is stored.
#pragma unroll
    for (int c = 0; c < 4; ++c) {
      uint32_t pk[16];
      auto chunk = [&](auto emu_tag) {
      constexpr bool emu = decltype(emu_tag)::value;
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        const uint64_t x = f2_fma(f2_pack(__uint_as_float(r[c][2 * i]),
                                          __uint_as_float(r[c][2 * i + 1])),
                                  sl2x2, nm2);
        float xa, xb;
        f2_unpack(x, xa, xb);
        uint64_t e;
#if CTB_FMHA_EXP_MODE == 1 || CTB_FMHA_EXP_MODE == 3
        e = x;  // timing probe only: no exponentials (wrong results)
#else
        // `emu` is uniform over the chunk (masked blocks take the MUFU path
        // for every pair), so the pair loop has no branches to schedule around.
        if (emu && (i % EMU_EVERY) == EMU_EVERY - 1)
          e = exp2_poly2(f2_pack(fmaxf(xa, -126.f), fmaxf(xb, -126.f)));
        else
          e = f2_pack(ex2(xa), ex2(xb));
#endif
        if (i & 1) acc1 = f2_add(acc1, e);
        else acc0 = f2_add(acc0, e);
        float ea, eb;
        f2_unpack(e, ea, eb);
        pk[i] = pack_half2(ea, eb);
      }
      };
      if (EMU_EVERY <= 16 && !need_mask)
        chunk(std::integral_constant<bool, (EMU_EVERY <= 16)>{});
      else
        chunk(std::integral_constant<bool, false>{});
#if CTB_FMHA_EXP_MODE < 3
      tmem_st_32x32b_x16(s_col + c * 16, pk);
#else
      if (pk[0] == 0x12345678u && pk[15] == 0x9abcdef0u) tmem_st_32x32b_x16(s_col + c * 16, pk);  // probe: no P write
#endif
      FMHA_SM_STAMP(t, 4 + c, j);
      if ((c + 1) % (4 / P_PARTS) == 0) {
        tmem_st_wait();
        tc_fence_before();
        arrive_p(c / (4 / P_PARTS));
      }
    }
    float s0, s1, s2, s3;
    f2_unpack(acc0, s0, s1);
    f2_unpack(acc1, s2, s3);
    l += (s0 + s1) + (s2 + s3);
    FMHA_SM_STAMP(t, 8, j);
    if (threadIdx.x % 128 == 0) FMHA_TRACE(2 + t, j);
  }
  // ------------------------------------------------------------ epilogue
  if (mbar_wait_bounded(o_full_t, 0, abort_flag, ERR_BIT)) {
    tc_fence_after();
    const float inv = 1.f / l;
    __half* orow = p.O + ((int64_t)bh * p.Sq + qrow) * HD;
#pragma unroll 1
    for (int c = 0; c < HD / 32; ++c) {
      uint32_t o[32];
      tmem_ld_32x32b_x32(o_col + c * 32, o);
      tmem_ld_wait();
      if (qrow < p.Sq) {
        uint4* dst = reinterpret_cast<uint4*>(orow + c * 32);
#pragma unroll
        for (int v = 0; v < 4; ++v) {
          uint4 w;
          w.x = pack_half2(__uint_as_float(o[8 * v + 0]) * inv, __uint_as_float(o[8 * v + 1]) * inv);
          w.y = pack_half2(__uint_as_float(o[8 * v + 2]) * inv, __uint_as_float(o[8 * v + 3]) * inv);
          w.z = pack_half2(__uint_as_float(o[8 * v + 4]) * inv, __uint_as_float(o[8 * v + 5]) * inv);
          w.w = pack_half2(__uint_as_float(o[8 * v + 6]) * inv, __uint_as_float(o[8 * v + 7]) * inv);
          dst[v] = w;
        }
      }
    }
  }
}

template <int HD>
__global__ void __launch_bounds__(THREADS, 1)
    fmha_fwd_tcgen05_kernel(const __grid_constant__ CUtensorMap tmQ,
                            const __grid_constant__ CUtensorMap tmK,
                            const __grid_constant__ CUtensorMap tmV, const Params p) {
  using namespace sm100;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  uint8_t* sQ = smem;                        // Q0, Q1
  uint8_t* sK = smem + 2 * tile_bytes<HD>();       // 2 stages
  uint8_t* sV = smem + 4 * tile_bytes<HD>();       // 2 stages
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + 6 * tile_bytes<HD>());
  uint64_t* q_full = bars + 0;
  uint64_t* k_full = bars + 1;   // [2]
  uint64_t* k_empty = bars + 3;  // [2]
  uint64_t* v_full = bars + 5;   // [2]
  uint64_t* v_empty = bars + 7;  // [2]
  uint64_t* s_full = bars + 9;   // [2]
  uint64_t* p_full = bars + 20;  // [2 tiles][P_PARTS key ranges]
  uint64_t* o_full = bars + 13;  // [2]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 15);
#ifdef CTB_FMHA_TRACE
  uint64_t* grp_done = bars + 16;  // [4]: trace-only completion of each MMA group
#endif
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
#ifdef CTB_FMHA_TRACE
  if (blockIdx.x == 0 && threadIdx.x == 0) {
    g_fmha_clk[0] = clock64();
    g_fmha_clk[1] = (long long)global_ns();
  }
#endif
  // CTAs of one (batch, head) are adjacent, so the CTAs resident at a time
  // share a few heads' K and V through L2 instead of streaming one head
  // each from HBM; within a head the heaviest (latest, for causal) query
  // blocks go first.
  const int lin = blockIdx.x;
#if CTB_FMHA_HEAD_MAJOR
  const int bh = lin / p.n_qblk;
  const int qblk = p.n_qblk - 1 - lin % p.n_qblk;
#else
  const int qblk = p.n_qblk - 1 - lin / p.BH;
  const int bh = lin % p.BH;
#endif
  const int q0 = qblk * 2 * BQ;
  int nb = (p.Sk + BKV - 1) / BKV;
  // Causal: tile 1 needs the key blocks up to its last row, tile 0 one fewer
  // (the block past its last row is fully masked for it and is skipped).
  int nb0 = nb;
  if (p.causal) {
    nb = min(nb, (q0 + 2 * BQ + BKV - 1) / BKV);
    nb0 = min(nb, (q0 + BQ + BKV - 1) / BKV);
  }

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&k_full[i], 1);
      mbar_init(&k_empty[i], 1);
      mbar_init(&v_full[i], 1);
      mbar_init(&v_empty[i], 1);
      mbar_init(&s_full[i], 1);
      for (int q = 0; q < P_PARTS; ++q) mbar_init(&p_full[P_PARTS * i + q], SM_THREADS_PER_TILE);
      mbar_init(&o_full[i], 1);
#ifdef CTB_FMHA_TRACE
      mbar_init(&grp_done[2 * i], 1);
      mbar_init(&grp_done[2 * i + 1], 1);
#endif
    }
    *abort_flag = 0;
    fence_mbar_init();
    tma_prefetch_desc(&tmQ);
    tma_prefetch_desc(&tmK);
    tma_prefetch_desc(&tmV);
  }
  if (warp == MMA_WARP) tmem_alloc(tmem_slot, 512);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp >= 8) {
    // Control warpgroups (MMA issuer, TMA producer, idle warps): give
    // registers to the softmax warps.
    asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(REG_OTHER));
  }
  if (warp == TMA_WARP) {
    // ------------------------------------------------------------ TMA producer
    if (lane == 0) {
      mbar_arrive_expect_tx(q_full, 2 * tile_bytes<HD>());
      for (int t = 0; t < 2; ++t)
        for (int h = 0; h < HD / 64; ++h)
          tma_load_3d(sQ + t * tile_bytes<HD>() + h * BOX_BYTES, &tmQ, q_full, h * 64, q0 + t * BQ, bh);
      for (int j = 0; j < nb && !*abort_flag; ++j) {
        const int s = j & 1;
        const uint32_t ph = (j >> 1) & 1;
        if (!mbar_wait_bounded(&k_empty[s], ph ^ 1, abort_flag, ERR_BIT)) break;
        mbar_arrive_expect_tx(&k_full[s], tile_bytes<HD>());
        for (int h = 0; h < HD / 64; ++h)
          tma_load_3d(sK + s * tile_bytes<HD>() + h * BOX_BYTES, &tmK, &k_full[s], h * 64, j * BKV, bh);
        FMHA_TRACE(13, j);
        if (!mbar_wait_bounded(&v_empty[s], ph ^ 1, abort_flag, ERR_BIT)) break;
        mbar_arrive_expect_tx(&v_full[s], tile_bytes<HD>());
        for (int h = 0; h < HD / 64; ++h)
          tma_load_3d(sV + s * tile_bytes<HD>() + h * BOX_BYTES, &tmV, &v_full[s], h * 64, j * BKV, bh);
        FMHA_TRACE(14, j);
      }
    }
  } else if (warp == MMA_WARP) {
    // ------------------------------------------------------------ MMA issuer
    {  // the whole warp runs the issue loop converged; elect.sync issues
      const uint32_t sQa = smem_u32(sQ), sKa = smem_u32(sK), sVa = smem_u32(sV);
      // Wait results are made warp-uniform so the warp never diverges around elect.sync.
      bool ok = __all_sync(0xffffffffu, mbar_wait_bounded(q_full, 0, abort_flag, ERR_BIT));
      if (ok) ok = __all_sync(0xffffffffu, mbar_wait_bounded(&k_full[0], 0, abort_flag, ERR_BIT));
      if (ok) {
        tc_fence_after();
        issue_s<HD>(tmem, sQa, sKa, 0, 0, &s_full[0]);
        issue_s<HD>(tmem, sQa, sKa, 1, 0, &s_full[1]);
        mma_commit_elect(&k_empty[0]);
      }
      // Tensor-pipe order per key block j: PV0(j) S0(j+1) PV1(j) S1(j+1). The
      // pipe executes one thread's MMAs in issue order, so S_t(j+1) never
      // overwrites P_t(j) before P_t(j)*V has read it.
      for (int j = 0; ok && j < nb; ++j) {
        const int s = j & 1, sn = (j + 1) & 1;
        const uint32_t ph = (j >> 1) & 1, phn = ((j + 1) >> 1) & 1;
        const bool more = j + 1 < nb;
        if (!(ok = __all_sync(0xffffffffu, mbar_wait_bounded(&v_full[s], ph, abort_flag, ERR_BIT)))) break;
        if (lane == 0) FMHA_TRACE(8, j);
        // P*V on the first 64 keys starts while the softmax finishes the rest.
        if (j < nb0) {
          for (int q = 0; q < P_PARTS && ok; ++q) {
            if (!(ok = __all_sync(0xffffffffu, mbar_wait_bounded(&p_full[q], j & 1, abort_flag, ERR_BIT)))) break;
            tc_fence_after();
            issue_pv<HD>(tmem, sVa, 0, s, j, q, lane == 0 && j == 30);
          }
          if (!ok) break;
          if (j + 1 == nb0 && nb0 < nb) mma_commit_elect(&o_full[0]);  // tile 0 done early
        }
#ifdef CTB_FMHA_TRACE
        mma_commit_elect(&grp_done[0]);
#endif
        if (lane == 0) FMHA_TRACE(4, j);
        if (more) {
          if (!(ok = __all_sync(0xffffffffu, mbar_wait_bounded(&k_full[sn], phn, abort_flag, ERR_BIT)))) break;
          tc_fence_after();
          if (j + 1 < nb0) issue_s<HD>(tmem, sQa, sKa, 0, sn, &s_full[0], lane == 0 && j == 30);
#ifdef CTB_FMHA_TRACE
        mma_commit_elect(&grp_done[1]);
#endif
          if (lane == 0) FMHA_TRACE(6, j);
        }
        for (int q = 0; q < P_PARTS && ok; ++q) {
          if (!(ok = __all_sync(0xffffffffu, mbar_wait_bounded(&p_full[P_PARTS + q], j & 1, abort_flag, ERR_BIT)))) break;
          tc_fence_after();
          issue_pv<HD>(tmem, sVa, 1, s, j, q, lane == 0 && j == 30);
        }
        if (!ok) break;
#ifdef CTB_FMHA_TRACE
        mma_commit_elect(&grp_done[2]);
#endif
        if (lane == 0) FMHA_TRACE(5, j);
        mma_commit_elect(&v_empty[s]);
        if (more) {
          issue_s<HD>(tmem, sQa, sKa, 1, sn, &s_full[1], lane == 0 && j == 30);
#ifdef CTB_FMHA_TRACE
        mma_commit_elect(&grp_done[3]);
#endif
          if (lane == 0) FMHA_TRACE(7, j);
          mma_commit_elect(&k_empty[sn]);
        }
      }
      if (nb0 == nb) mma_commit_elect(&o_full[0]);
      mma_commit_elect(&o_full[1]);
    }
#ifdef CTB_FMHA_TRACE
  } else if (warp == 10) {
    if (lane == 0 && blockIdx.x == 0) {
      for (int j = 0; j < nb && j < 128; ++j)
        for (int g = 0; g < 4; ++g) {
          if ((g == 1 || g == 3) && j + 1 >= nb) continue;
          if (!mbar_wait_bounded(&grp_done[g], j & 1, abort_flag, ERR_BIT)) break;
          g_fmha_trace[9 + g][j] = clock64();
        }
    }
#endif
  } else if (warp < 8) {
    // ------------------------------------------------------------ softmax warpgroups
    // One thread per query row, all 128 scores of a block in registers.
    asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(REG_SOFTMAX));
    const int t = warp >> 2;        // query tile
    const int quarter = warp & 3;   // TMEM lanes 32*quarter .. +31
    const uint32_t lane_off = (uint32_t)(quarter * 32) << 16;
    const uint32_t s_col = tmem + lane_off + t * BKV;
    const uint32_t o_col = tmem + lane_off + 256 + t * HD;
    const int qrow = q0 + t * BQ + quarter * 32 + lane;
    softmax_rows<HD>(p, t, s_col, o_col, qrow, q0 + t * BQ, bh, t == 0 ? nb0 : nb, &s_full[t], &o_full[t], abort_flag,
                 [&](int part) { mbar_arrive(&p_full[t * P_PARTS + part]); });
  }

  tc_fence_before();
  __syncthreads();
  if (warp == MMA_WARP) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
#ifdef CTB_FMHA_TRACE
  if (blockIdx.x == 0 && threadIdx.x == 0) {
    g_fmha_clk[2] = clock64();
    g_fmha_clk[3] = (long long)global_ns();
  }
#endif
}


// =============================================================================
// CTA-pair variant (cta_group::2). A cluster of two CTAs on two SMs takes one
// (batch*head, 512-query block) as two 256-row query tiles; tile t's rows
// q0 + 256 t + 128 r + [0, 128) live in CTA r (its Q in shared memory, its S,
// P and O in its own tensor memory, lanes = rows). Each CTA loads only half
// of every key block's operands: keys [64 r, 64 r + 64) of K (the N half of
// S = Q K^T) and head_dim columns [64 r, 64 r + 64) of V (the N half of
// O += P V). The even CTA issues 256-row MMAs that read both CTAs' halves.
// Per 128-key block an SM's shared memory then feeds 2 x 8 S steps of 6 KB
// (against 8 KB on one SM) and 2 x 8 P*V steps of 2 KB, and receives 32 KB
// of K/V (against 64 KB), so shared-memory bandwidth no longer paces the
// tensor pipe. Roles per CTA are those of the one-SM kernel; the MMA warp
// only issues in the even CTA, and the softmax warps of both CTAs arrive on
// the even CTA's P barriers (one arrival per warp).
// Barriers: q_full, k_full[s], v_full[s] and p_full live in the even CTA
// and count both CTAs; k_empty, v_empty, s_full and o_full exist in both
// CTAs and receive a commit each.
// Causal: tile t only runs the key blocks that reach its last row.
// =============================================================================
#ifndef CTB_FMHA_PAIR_STAGES
#define CTB_FMHA_PAIR_STAGES 4
#endif
constexpr int PR_STAGES = CTB_FMHA_PAIR_STAGES;    // K/V ring depth
constexpr int PR_QROWS = 4 * BQ;                     // query rows per pair
constexpr int PR_K_BYTES = 64 * D * 2;               // 64 keys x 128 head_dim: two 8 KB boxes
constexpr int PR_K_BOX_BYTES = PR_K_BYTES / 2;
constexpr int PR_V_BYTES = BKV * 64 * 2;             // 128 keys x 64 head_dim columns
constexpr int PR_SMEM_BYTES = 2 * TILE_BYTES + PR_STAGES * (PR_K_BYTES + PR_V_BYTES) + 1024 + 512;
static_assert(PR_SMEM_BYTES <= 232448, "pair FMHA shared memory exceeds the per-CTA limit");

// S_t = Q_t K^T over the pair: M = 256 (128 rows per CTA), N = 128 keys (64 per CTA).
__device__ __forceinline__ void issue_s_pair(uint32_t tmem, uint32_t sQa, uint32_t sKa, int t,
                                             int stage, uint64_t* s_full_t) {
  using namespace sm100;
  constexpr uint32_t idesc_s = idesc_f16_f32(2 * BQ, BKV, false, false);
  const uint32_t qa = sQa + t * TILE_BYTES, ka = sKa + stage * PR_K_BYTES;
#pragma unroll
  for (int kk = 0; kk < D / 16; ++kk) {
    const uint32_t qoff = (kk >> 2) * HALF_BYTES + (kk & 3) * 32;
    const uint32_t koff = (kk >> 2) * PR_K_BOX_BYTES + (kk & 3) * 32;
    mma_f16_ss_pair_elect(tmem + t * BKV, smem_desc_sw128(qa + qoff, 16, 1024),
                          smem_desc_sw128(ka + koff, 16, 1024), idesc_s, kk != 0);
  }
  mma_commit_pair_both_elect(s_full_t);
}

// O_t (+)= P_t V for one published part of a key block: M = 256, N = 128
// head_dim (64 per CTA, one 128-byte swizzle atom wide), 16 keys per step.
__device__ __forceinline__ void issue_pv_pair(uint32_t tmem, uint32_t sVa, int t, int stage, int j,
                                              int part) {
  using namespace sm100;
  constexpr uint32_t idesc_o = idesc_f16_f32(2 * BQ, D, false, true);
  constexpr int STEPS = BKV / 16 / P_PARTS;
  const uint32_t va = sVa + stage * PR_V_BYTES;
#pragma unroll
  for (int k4 = 0; k4 < STEPS; ++k4) {
    const int kk = part * STEPS + k4;
    mma_f16_ts_pair_elect(tmem + 256 + t * D, tmem + t * BKV + kk * 8,
                          smem_desc_sw128(va + kk * 2048, PR_V_BYTES, 1024), idesc_o,
                          (j > 0 || kk > 0) ? 1u : 0u);
  }
}

__global__ void __launch_bounds__(THREADS, 1)
    fmha_fwd_pair_kernel(const __grid_constant__ CUtensorMap tmQ,
                         const __grid_constant__ CUtensorMap tmK,
                         const __grid_constant__ CUtensorMap tmV, const Params p) {
  using namespace sm100;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  uint8_t* sQ = smem;                                   // Q tiles 0, 1 (this CTA's rows)
  uint8_t* sK = smem + 2 * TILE_BYTES;                  // PR_STAGES x 16 KB
  uint8_t* sV = sK + PR_STAGES * PR_K_BYTES;            // PR_STAGES x 16 KB
  uint64_t* bars = reinterpret_cast<uint64_t*>(sV + PR_STAGES * PR_V_BYTES);
  uint64_t* q_full = bars;
  uint64_t* k_full = q_full + 1;               // [PR_STAGES]
  uint64_t* k_empty = k_full + PR_STAGES;      // [PR_STAGES]
  uint64_t* v_full = k_empty + PR_STAGES;      // [PR_STAGES]
  uint64_t* v_empty = v_full + PR_STAGES;      // [PR_STAGES]
  uint64_t* s_full = v_empty + PR_STAGES;      // [2]
  uint64_t* o_full = s_full + 2;               // [2]
  uint64_t* p_full = o_full + 2;               // [2 tiles][P_PARTS]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(p_full + 2 * P_PARTS);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int rank = (int)cluster_ctarank();
  const bool leader = rank == 0;
  const int pair = blockIdx.x / 2;
  // Query blocks of one (batch, head) are adjacent pairs; heaviest first.
  const int bh = pair / p.n_qblk;
  const int qblk = p.n_qblk - 1 - pair % p.n_qblk;
  const int q0 = qblk * PR_QROWS;
  const int nb = (p.Sk + BKV - 1) / BKV;
  int nbt[2];
#pragma unroll
  for (int t = 0; t < 2; ++t)
    nbt[t] = p.causal ? min(nb, (q0 + (t + 1) * 2 * BQ + BKV - 1) / BKV) : nb;

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int i = 0; i < PR_STAGES; ++i) {
      mbar_init(&k_full[i], 1);
      mbar_init(&k_empty[i], 1);
      mbar_init(&v_full[i], 1);
      mbar_init(&v_empty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&s_full[i], 1);
      mbar_init(&o_full[i], 1);
      for (int q = 0; q < P_PARTS; ++q) mbar_init(&p_full[P_PARTS * i + q], 2 * 4);  // 4 warps x 2 CTAs
    }
    *abort_flag = 0;
    fence_mbar_init();
    tma_prefetch_desc(&tmQ);
    tma_prefetch_desc(&tmK);
    tma_prefetch_desc(&tmV);
  }
  if (warp == MMA_WARP) tmem_alloc_pair(tmem_slot, 512);
  tc_fence_before();
  cluster_sync_all();  // barriers of both CTAs initialised before any cross-CTA use
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp >= 8) asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(REG_OTHER));
  if (warp == TMA_WARP) {
    // ------------------------------------------------------------ TMA producer (both CTAs)
    if (lane == 0) {
      const uint32_t q_bar = mapa_shared(smem_u32(q_full), 0);
      const uint32_t kf_bar = mapa_shared(smem_u32(k_full), 0);
      const uint32_t vf_bar = mapa_shared(smem_u32(v_full), 0);
      if (leader) mbar_arrive_expect_tx(q_full, 2 * 2 * TILE_BYTES);
      for (int t = 0; t < 2; ++t)
        for (int h = 0; h < 2; ++h)
          tma_load_3d_pair(sQ + t * TILE_BYTES + h * HALF_BYTES, &tmQ, q_bar, h * 64,
                           q0 + t * 2 * BQ + rank * BQ, bh);
      for (int j = 0; j < nbt[1] && !*abort_flag; ++j) {
        const int s = j % PR_STAGES;
        const uint32_t ph = (j / PR_STAGES) & 1;
        if (!mbar_wait_bounded(&k_empty[s], ph ^ 1, abort_flag, ERR_BIT)) break;
        if (leader) mbar_arrive_expect_tx(&k_full[s], 2 * PR_K_BYTES);
        for (int h = 0; h < 2; ++h)
          tma_load_3d_pair(sK + s * PR_K_BYTES + h * PR_K_BOX_BYTES, &tmK, kf_bar + 8 * s, h * 64,
                           j * BKV + rank * 64, bh);
        if (!mbar_wait_bounded(&v_empty[s], ph ^ 1, abort_flag, ERR_BIT)) break;
        if (leader) mbar_arrive_expect_tx(&v_full[s], 2 * PR_V_BYTES);
        tma_load_3d_pair(sV + s * PR_V_BYTES, &tmV, vf_bar + 8 * s, rank * 64, j * BKV, bh);
      }
    }
  } else if (warp == MMA_WARP) {
    // ------------------------------------------------------------ MMA issuer (even CTA)
    if (leader) {
      const uint32_t sQa = smem_u32(sQ), sKa = smem_u32(sK), sVa = smem_u32(sV);
      bool ok = __all_sync(0xffffffffu, mbar_wait_bounded(q_full, 0, abort_flag, ERR_BIT));
      if (ok) ok = __all_sync(0xffffffffu, mbar_wait_bounded(&k_full[0], 0, abort_flag, ERR_BIT));
      if (ok) {
        tc_fence_after();
        issue_s_pair(tmem, sQa, sKa, 0, 0, &s_full[0]);
        issue_s_pair(tmem, sQa, sKa, 1, 0, &s_full[1]);
        mma_commit_pair_both_elect(&k_empty[0]);
      }
      // Per key block j: PV0(j) S0(j+1) PV1(j) S1(j+1), as on one SM; the pipe
      // runs one thread's MMAs in order, so S_t(j+1) follows P_t(j)*V.
      for (int j = 0; ok && j < nbt[1]; ++j) {
        const int s = j % PR_STAGES, sn = (j + 1) % PR_STAGES;
        const uint32_t ph = (j / PR_STAGES) & 1, phn = ((j + 1) / PR_STAGES) & 1;
        if (!(ok = __all_sync(0xffffffffu, mbar_wait_bounded(&v_full[s], ph, abort_flag, ERR_BIT)))) break;
        if (j < nbt[0]) {
          for (int q = 0; q < P_PARTS && ok; ++q) {
            if (!(ok = __all_sync(0xffffffffu, mbar_wait_bounded(&p_full[q], j & 1, abort_flag, ERR_BIT)))) break;
            tc_fence_after();
            issue_pv_pair(tmem, sVa, 0, s, j, q);
          }
          if (!ok) break;
          if (j + 1 == nbt[0]) mma_commit_pair_both_elect(&o_full[0]);
        }
        bool k_ready = false;
        if (j + 1 < nbt[0]) {
          if (!(ok = __all_sync(0xffffffffu, mbar_wait_bounded(&k_full[sn], phn, abort_flag, ERR_BIT)))) break;
          k_ready = true;
          tc_fence_after();
          issue_s_pair(tmem, sQa, sKa, 0, sn, &s_full[0]);
        }
        for (int q = 0; q < P_PARTS && ok; ++q) {
          if (!(ok = __all_sync(0xffffffffu, mbar_wait_bounded(&p_full[P_PARTS + q], j & 1, abort_flag, ERR_BIT)))) break;
          tc_fence_after();
          issue_pv_pair(tmem, sVa, 1, s, j, q);
        }
        if (!ok) break;
        mma_commit_pair_both_elect(&v_empty[s]);
        if (j + 1 < nbt[1]) {
          if (!k_ready) {
            if (!(ok = __all_sync(0xffffffffu, mbar_wait_bounded(&k_full[sn], phn, abort_flag, ERR_BIT)))) break;
            tc_fence_after();
          }
          issue_s_pair(tmem, sQa, sKa, 1, sn, &s_full[1]);
          mma_commit_pair_both_elect(&k_empty[sn]);
        }
      }
      mma_commit_pair_both_elect(&o_full[1]);
    }
  } else if (warp < 8) {
    // ------------------------------------------------------------ softmax warpgroups (both CTAs)
    asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(REG_SOFTMAX));
    const int t = warp >> 2;
    const int quarter = warp & 3;
    const uint32_t lane_off = (uint32_t)(quarter * 32) << 16;
    const uint32_t s_col = tmem + lane_off + t * BKV;
    const uint32_t o_col = tmem + lane_off + 256 + t * D;
    const int row0 = q0 + t * 2 * BQ + rank * BQ;
    const int qrow = row0 + quarter * 32 + lane;
    const uint32_t p_bar = mapa_shared(smem_u32(&p_full[t * P_PARTS]), 0);
    softmax_rows<D>(p, t, s_col, o_col, qrow, row0, bh, nbt[t], &s_full[t], &o_full[t], abort_flag,
                 [&](int part) {
                   __syncwarp();
                   if (lane == 0) mbar_arrive_cluster(p_bar + 8 * part);
                 });
  }

  tc_fence_before();
  cluster_sync_all();  // no CTA leaves while its peer may still touch its shared or tensor memory
  if (warp == MMA_WARP) {
    tc_fence_after();
    tmem_dealloc_pair(tmem, 512);
  }
}

}  // namespace fmha

int fmha_take_device_error(unsigned int* out) { return take_device_error(out); }

#ifdef CTB_FMHA_TRACE
extern "C" int ctb_fmha_trace_read(long long* out) {
  return cudaMemcpyFromSymbol(out, fmha::g_fmha_trace, sizeof(fmha::g_fmha_trace)) == cudaSuccess ? 0 : -6;
}
extern "C" int ctb_fmha_trace_sm_read(long long* out) {
  return cudaMemcpyFromSymbol(out, fmha::g_fmha_sm, sizeof(fmha::g_fmha_sm)) == cudaSuccess ? 0 : -6;
}
extern "C" int ctb_fmha_trace_clk_read(long long* out) {
  return cudaMemcpyFromSymbol(out, fmha::g_fmha_clk, sizeof(fmha::g_fmha_clk)) == cudaSuccess ? 0 : -6;
}
extern "C" int ctb_fmha_trace_mma_read(long long* out) {
  return cudaMemcpyFromSymbol(out, fmha::g_fmha_mma, sizeof(fmha::g_fmha_mma)) == cudaSuccess ? 0 : -6;
}
#endif

static unsigned long long g_fmha_attr_done[64];  // context ID the set-up was done in
static int g_fmha_pairs[64];                     // resident CTA pairs of the pair kernel
static std::mutex g_fmha_mu;

static cudaLaunchConfig_t fmha_pair_config(cudaLaunchAttribute* attr, unsigned grid,
                                           cudaStream_t st) {
  cudaLaunchConfig_t cfg = {};
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.gridDim = dim3(grid, 1, 1);
  cfg.blockDim = dim3(fmha::THREADS, 1, 1);
  cfg.dynamicSmemBytes = fmha::PR_SMEM_BYTES;
  cfg.stream = st;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cfg;
}

int fmha_device_setup() {
  int dev = 0;
  CTB_CUDA_CHECK(cudaGetDevice(&dev));
  std::lock_guard<std::mutex> lk(g_fmha_mu);
  unsigned long long ctx = 0;
  if (int rc = current_context_id(&ctx)) return rc;
  if (dev < 64 && g_fmha_attr_done[dev] == ctx) return CTB_OK;
  CTB_CUDA_CHECK(cudaFuncSetAttribute(fmha::fmha_fwd_tcgen05_kernel<128>,
                                      cudaFuncAttributeMaxDynamicSharedMemorySize,
                                      fmha::smem_bytes<128>()));
  CTB_CUDA_CHECK(cudaFuncSetAttribute(fmha::fmha_fwd_tcgen05_kernel<64>,
                                      cudaFuncAttributeMaxDynamicSharedMemorySize,
                                      fmha::smem_bytes<64>()));
  CTB_CUDA_CHECK(cudaFuncSetAttribute(fmha::fmha_fwd_pair_kernel,
                                      cudaFuncAttributeMaxDynamicSharedMemorySize,
                                      fmha::PR_SMEM_BYTES));
  cudaLaunchAttribute attr[1];
  cudaLaunchConfig_t cfg = fmha_pair_config(attr, 2, 0);
  int clusters = 0;
  CTB_CUDA_CHECK(cudaOccupancyMaxActiveClusters(&clusters, fmha::fmha_fwd_pair_kernel, &cfg));
  if (dev < 64) {
    g_fmha_pairs[dev] = clusters;
    g_fmha_attr_done[dev] = ctx;
  }
  return CTB_OK;
}

// CTB_FMHA_PAIR=1 runs attention on the CTA-pair kernel (when a pair can be
// resident). It is not the default: on B200 at B8 H32 S8192 D128 it measured
// 980 / 830 TFLOP/s (non-causal / causal) against 1238 / 969 for the one-SM
// kernel in the same process; both are paced by the per-tile chain S ->
// softmax -> P*V -> next S, not by shared-memory bandwidth, and the pair adds
// a cross-SM hand-off to every link of that chain.
static bool fmha_use_pair() {
  static const bool on = [] {
    const char* e = getenv("CTB_FMHA_PAIR");
    return e && e[0] == '1';
  }();
  if (!on) return false;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return false;
  return g_fmha_pairs[dev] > 0;
}

static int fmha_tc(const __half* Q, const __half* K, const __half* V, __half* O, int B, int H,
                   int Sq, int Sk, int hd, float scale, int causal, cudaStream_t st) {
  if (int rc = fmha_device_setup()) return rc;
  const int BH = B * H;
  const bool pair = hd == fmha::D && fmha_use_pair();
  CUtensorMap tq, tk, tv;
  const uint32_t box[3] = {64, 128, 1};
  const uint32_t kbox[3] = {64, pair ? 64u : 128u, 1};  // a CTA of a pair loads 64 keys
  {
    const uint64_t dims[3] = {(uint64_t)hd, (uint64_t)Sq, (uint64_t)BH};
    const uint64_t strides[2] = {(uint64_t)hd * 2, (uint64_t)Sq * hd * 2};
    if (int rc = encode_tmap(&tq, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3, Q, dims, strides, box,
                             CU_TENSOR_MAP_SWIZZLE_128B))
      return rc;
  }
  {
    const uint64_t dims[3] = {(uint64_t)hd, (uint64_t)Sk, (uint64_t)BH};
    const uint64_t strides[2] = {(uint64_t)hd * 2, (uint64_t)Sk * hd * 2};
    if (int rc = encode_tmap(&tk, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3, K, dims, strides, kbox,
                             CU_TENSOR_MAP_SWIZZLE_128B))
      return rc;
    if (int rc = encode_tmap(&tv, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3, V, dims, strides, box,
                             CU_TENSOR_MAP_SWIZZLE_128B))
      return rc;
  }
  fmha::Params p;
  p.O = O;
  p.Sq = Sq;
  p.Sk = Sk;
  p.BH = BH;
  p.n_qblk = (Sq + 2 * fmha::BQ - 1) / (2 * fmha::BQ);
  p.scale_log2 = scale * 1.4426950408889634f;
  p.causal = causal;
  if (pair) {
    p.n_qblk = (Sq + fmha::PR_QROWS - 1) / fmha::PR_QROWS;
    const int64_t grid = 2 * (int64_t)p.n_qblk * BH;
    if (grid > 0x7fffffff) return set_error(CTB_ERR_SHAPE, "fmha: too many query blocks");
    cudaLaunchAttribute attr[1];
    cudaLaunchConfig_t cfg = fmha_pair_config(attr, (unsigned)grid, st);
    CTB_CUDA_CHECK(cudaLaunchKernelEx(&cfg, fmha::fmha_fwd_pair_kernel, tq, tk, tv, p));
    return launch_status("fmha_fwd_pair_kernel");
  }
  const int64_t grid = (int64_t)p.n_qblk * BH;
  if (grid > 0x7fffffff) return set_error(CTB_ERR_SHAPE, "fmha: too many query blocks");
  if (hd == 64)
    fmha::fmha_fwd_tcgen05_kernel<64>
        <<<(unsigned)grid, fmha::THREADS, fmha::smem_bytes<64>(), st>>>(tq, tk, tv, p);
  else
    fmha::fmha_fwd_tcgen05_kernel<128>
        <<<(unsigned)grid, fmha::THREADS, fmha::smem_bytes<128>(), st>>>(tq, tk, tv, p);
  return launch_status("fmha_fwd_tcgen05_kernel");
}

}  // namespace ctb

using namespace ctb;

extern "C" int ctb_fmha_fwd_f16(const void* Q, const void* K, const void* V, void* O,
                                int32_t batch, int32_t heads, int32_t seq_q, int32_t seq_k,
                                int32_t head_dim, float scale, int32_t causal, void* stream) {
  clear_error();
  if (batch < 0 || heads < 0 || seq_q < 0 || seq_k < 1 || head_dim < 1)
    return set_error(CTB_ERR_SHAPE, "fmha: need batch, heads, seq_q >= 0 and seq_k, head_dim >= 1");
  if ((int64_t)batch * heads * seq_q == 0) return CTB_OK;
  if (!Q || !K || !V || !O) return set_error(CTB_ERR_ARG, "fmha: NULL pointer");
  if (!(scale > 0.f)) return set_error(CTB_ERR_ARG, "fmha: scale must be positive");
  DeviceProps p;
  if (int rc = current_props(&p)) return rc;
  auto st = static_cast<cudaStream_t>(stream);
  const bool tc_ok = (head_dim == 128 || head_dim == 64) && aligned16(Q) && aligned16(K) && aligned16(V) &&
                     aligned16(O) && (int64_t)batch * heads <= 0x7fffffff;
  if (tc_ok)
    return fmha_tc((const __half*)Q, (const __half*)K, (const __half*)V, (__half*)O, batch, heads,
                   seq_q, seq_k, head_dim, scale, causal ? 1 : 0, st);
  return fmha_simt((const __half*)Q, (const __half*)K, (const __half*)V, (__half*)O, batch, heads,
                   seq_q, seq_k, head_dim, scale, causal ? 1 : 0, st);
}

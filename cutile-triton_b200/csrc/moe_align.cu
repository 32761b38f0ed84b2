// Fused-MoE routing on the device: the `moe_align_block_size` step of the
// published fused-MoE contract (the layout the moe GEMM of this library
// reads; the cuTile moe example that the reference benchmarks is not
// vendored). Every (token, choice) slot s = token * topk + j with expert
// e = topk_ids[s] is listed in sorted_token_ids, experts in order, slots of
// one expert in slot order, each expert's list padded with the id `slots`
// to a multiple of `block`; expert_ids[b] is the expert of block b (-1 for
// blocks past the last expert); num_tokens_post_padded is the padded total.
//
// One CTA of 1024 threads, so nothing leaves the device and no host sync is
// needed: the caller sizes the outputs for the worst case
// (ctb_moe_align_capacity) and the GEMM reads the true total from device
// memory. Stable counting sort: (1) per-expert counts with shared-memory
// atomics, (2) padded starts by a scan over experts, (3) slots placed in
// chunks of 1024: a slot's rank inside its warp comes from __match_any_sync,
// the warps' counts per expert are scanned in shared memory, and a running
// count per expert carries across chunks.
#include "ctb_common.cuh"

#include <algorithm>

namespace ctb {
namespace {

constexpr int ALIGN_THREADS = 1024;
constexpr int ALIGN_WARPS = ALIGN_THREADS / 32;
constexpr int ALIGN_MAX_EXPERTS = 256;

__global__ void __launch_bounds__(ALIGN_THREADS) moe_align_kernel(
    const int32_t* __restrict__ ids, int slots, int E, int block, int32_t* __restrict__ sorted,
    int32_t* __restrict__ expert_ids, int32_t* __restrict__ ntp, int capacity) {
  __shared__ int count[ALIGN_MAX_EXPERTS];
  __shared__ int start[ALIGN_MAX_EXPERTS + 1];
  __shared__ int run[ALIGN_MAX_EXPERTS];
  __shared__ int hist[ALIGN_WARPS][ALIGN_MAX_EXPERTS];
  const int t = threadIdx.x, lane = t & 31, warp = t >> 5;
  for (int e = t; e < E; e += ALIGN_THREADS) {
    count[e] = 0;
    run[e] = 0;
  }
  for (int i = t; i < capacity; i += ALIGN_THREADS) sorted[i] = slots;  // padding id
  __syncthreads();
  for (int s = t; s < slots; s += ALIGN_THREADS) {
    const int e = ids[s];
    if (e >= 0 && e < E) atomicAdd(&count[e], 1);
  }
  __syncthreads();
  if (t == 0) {
    int acc = 0;
    for (int e = 0; e < E; ++e) {
      start[e] = acc;
      acc += (count[e] + block - 1) / block * block;
    }
    start[E] = acc;
    *ntp = acc;
  }
  __syncthreads();
  const int used_blocks = start[E] / block;
  for (int b = t; b < capacity / block; b += ALIGN_THREADS) {
    int e = -1;
    if (b < used_blocks) {  // the expert whose padded range holds block b
      int lo = 0, hi = E - 1;
      while (lo < hi) {
        const int mid = (lo + hi + 1) >> 1;
        if (start[mid] <= b * block) lo = mid;
        else hi = mid - 1;
      }
      e = lo;
    }
    expert_ids[b] = e;
  }
  for (int base = 0; base < slots; base += ALIGN_THREADS) {
    const int s = base + t;
    const int e = s < slots ? ids[s] : -1;
    const bool valid = e >= 0 && e < E;
    const unsigned same = __match_any_sync(0xffffffffu, valid ? e : -1);
    const int rank = __popc(same & ((1u << lane) - 1u));
    for (int k = t; k < ALIGN_WARPS * E; k += ALIGN_THREADS) hist[k / E][k % E] = 0;
    __syncthreads();
    if (valid && rank == 0) hist[warp][e] = __popc(same);
    __syncthreads();
    // Exclusive scan over the warps, per expert; then advance the running counts.
    for (int ee = t; ee < E; ee += ALIGN_THREADS) {
      int acc = 0;
      for (int w = 0; w < ALIGN_WARPS; ++w) {
        const int c = hist[w][ee];
        hist[w][ee] = acc;
        acc += c;
      }
      count[ee] = acc;  // this chunk's total (count[] is no longer needed as a total)
    }
    __syncthreads();
    if (valid) sorted[start[e] + run[e] + hist[warp][e] + rank] = s;
    __syncthreads();
    for (int ee = t; ee < E; ee += ALIGN_THREADS) run[ee] += count[ee];
    __syncthreads();
  }
}

}  // namespace
}  // namespace ctb

using namespace ctb;

extern "C" int32_t ctb_moe_align_capacity(int32_t slots, int32_t E, int32_t block) {
  if (slots < 0 || E < 1 || block < 1) return -1;
  const int64_t worst = (int64_t)slots + (int64_t)E * (block - 1);
  const int64_t cap = std::max<int64_t>((worst + block - 1) / block * block, block);
  return cap > 0x7fffffff ? -1 : (int32_t)cap;
}

extern "C" int ctb_moe_align_i32(const int32_t* topk_ids, int32_t slots, int32_t E,
                                 int32_t block, int32_t* sorted_token_ids, int32_t* expert_ids,
                                 int32_t* num_tokens_post_padded, int32_t capacity,
                                 void* stream) {
  clear_error();
  if (slots < 0 || E < 1 || block < 1) return set_error(CTB_ERR_SHAPE, "moe_align: bad sizes");
  if (E > ALIGN_MAX_EXPERTS)
    return set_error(CTB_ERR_SHAPE, "moe_align: at most 256 experts on the device path");
  const int32_t need = ctb_moe_align_capacity(slots, E, block);
  if (need < 0 || capacity < need || capacity % block != 0)
    return set_error(CTB_ERR_SHAPE,
                     "moe_align: capacity must be a multiple of block and at least "
                     "ctb_moe_align_capacity(slots, E, block) = " + std::to_string(need));
  if ((slots > 0 && !topk_ids) || !sorted_token_ids || !expert_ids || !num_tokens_post_padded)
    return set_error(CTB_ERR_ARG, "moe_align: NULL pointer");
  DeviceProps p;
  if (int rc = current_props(&p)) return rc;
  moe_align_kernel<<<1, ALIGN_THREADS, 0, static_cast<cudaStream_t>(stream)>>>(
      topk_ids, slots, E, block, sorted_token_ids, expert_ids, num_tokens_post_padded, capacity);
  return launch_status("moe_align_kernel");
}

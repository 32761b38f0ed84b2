// Test-only entry point: proves that a bounded device-side wait gives up,
// reports CTB_ERR_TIMEOUT through ctb_check_device and leaves the context
// usable. The kernel takes the same exit path as the pipeline kernels when a
// wait runs out: the waiting thread flags the error word and the CTA abort
// flag, the other warp sees the flag and drains, and the TMEM the CTA holds is
// released before it returns. Nothing traps, faults or spins without limit:
// every wait is bounded by wall time (%globaltimer).
#include "ctb_common.cuh"
#include "sm100_ptx.cuh"

namespace ctb {
namespace {
using namespace sm100;

constexpr unsigned kSelftestErrBit = 1u << 5;

// One CTA of two warps. Warp 0 holds 32 TMEM columns and waits on an mbarrier
// that nothing arrives on, with `limit_ns`; warp 1 waits on the same barrier
// with the library's default limit and must leave through the abort flag long
// before that. status[0] = 1 if warp 0's wait returned false, status[1] = 1 if
// warp 1's did, status[2] = the ns warp 1 waited.
__global__ void __launch_bounds__(64) selftest_wait_timeout_kernel(uint64_t limit_ns,
                                                                   int* status) {
  __shared__ __align__(8) uint64_t never;
  __shared__ uint32_t tmem_slot;
  __shared__ volatile int abort_flag;
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  if (threadIdx.x == 0) {
    mbar_init(&never, 1);
    abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 0) tmem_alloc(&tmem_slot, 32);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (lane == 0) {
    if (warp == 0) {
      const bool ok = mbar_wait_bounded(&never, 0, &abort_flag, kSelftestErrBit, limit_ns);
      status[0] = ok ? 0 : 1;
    } else {
      const uint64_t t0 = global_ns();
      const bool ok = mbar_wait_bounded(&never, 0, &abort_flag, kSelftestErrBit);
      status[1] = ok ? 0 : 1;
      const uint64_t waited = global_ns() - t0;
      status[2] = waited > 0x7fffffffull ? 0x7fffffff : (int)waited;
    }
  }
  __syncwarp();
  tc_fence_before();
  __syncthreads();
  if (warp == 0) tmem_dealloc(tmem_slot, 32);
}

}  // namespace

int selftest_take_device_error(unsigned int* out) { return take_device_error(out); }

}  // namespace ctb

extern "C" int ctb_selftest_wait_timeout(int64_t limit_ns, int* status, void* stream) {
  using namespace ctb;
  clear_error();
  if (limit_ns <= 0 || limit_ns > 1000000000ll)
    return set_error(CTB_ERR_ARG, "ctb_selftest_wait_timeout: limit_ns must be in (0, 1e9]");
  if (status == nullptr) return set_error(CTB_ERR_ARG, "ctb_selftest_wait_timeout: status is NULL");
  DeviceProps p;
  if (int rc = current_props(&p)) return rc;
  selftest_wait_timeout_kernel<<<1, 64, 0, static_cast<cudaStream_t>(stream)>>>(
      (uint64_t)limit_ns, status);
  return launch_status("selftest_wait_timeout_kernel");
}

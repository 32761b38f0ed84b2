// Shared helpers for the sm_100a kernels of libcutile_b200.so: status
// plumbing, the device error word, vector loads/stores and CTA reductions.
#pragma once

#include <cuda_runtime.h>
#include <cuda_fp16.h>
#include <cuda_bf16.h>
#include <stdint.h>
#include <string>

#include "../../include/cutile_b200.h"

namespace ctb {

// ---- host-side status -------------------------------------------------------
// Records `msg` as this thread's last error and returns `code`.
int set_error(int code, const std::string& msg);
void clear_error();
// Maps a CUDA error to CTB_ERR_CUDA with `what` as context.
int cuda_fail(cudaError_t e, const char* what);

#define CTB_CUDA_CHECK(call)                                   \
  do {                                                         \
    cudaError_t _e = (call);                                   \
    if (_e != cudaSuccess) return ::ctb::cuda_fail(_e, #call); \
  } while (0)

// After a kernel launch: report a launch-configuration error.
inline int launch_status(const char* what) {
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, what);
  return CTB_OK;
}

struct DeviceProps {
  int sm_count = 0;
  int max_smem_optin = 0;
  int cc_major = 0, cc_minor = 0;
};
// Properties of the current device (cached per device; ctb_init fills them).
int current_props(DeviceProps* out);

// Unique ID (never reused within a process) of the current device's primary
// context. Per-device set-up (kernel attributes, symbol addresses) is
// remembered with this ID, so after a cudaDeviceReset it is done again.
int current_context_id(unsigned long long* id);

// ---- device error word ------------------------------------------------------
// Set by a kernel whose bounded wait gave up; read by ctb_check_device.
// Bits: 1 = GEMM, 2 = FMHA, 4 = LayerNorm backward, 8 = MoE pipeline wait,
// 32 = the wait self-test (ctb_selftest_wait_timeout).
// The library is built without relocatable device code, so every translation
// unit owns its copy; a unit whose kernels flag errors exposes a reader
// (take_device_error) that ctb_check_device polls.
static __device__ unsigned int g_device_error = 0;

// Reads and clears this translation unit's error word on the current device.
static inline int take_device_error(unsigned int* out) {
  unsigned int zero = 0;
  cudaError_t e = cudaMemcpyFromSymbol(out, g_device_error, sizeof(*out));
  if (e == cudaSuccess && *out) e = cudaMemcpyToSymbol(g_device_error, &zero, sizeof(zero));
  return e == cudaSuccess ? 0 : (int)e;
}

__device__ __forceinline__ void flag_device_error(unsigned int bit) {
  atomicOr(&g_device_error, bit);
}

// ---- vector memory helpers --------------------------------------------------
// Streaming loads: data is read once, do not allocate in L1.
__device__ __forceinline__ float4 ld_stream_f4(const float* p) {
  float4 v;
  asm volatile("ld.global.nc.L1::no_allocate.v4.f32 {%0,%1,%2,%3}, [%4];"
               : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
               : "l"(p));
  return v;
}
// Evict-first stores for outputs that are not re-read by this kernel.
__device__ __forceinline__ void st_stream_f4(float* p, float4 v) {
  asm volatile("st.global.cs.v4.f32 [%0], {%1,%2,%3,%4};" ::"l"(p), "f"(v.x),
               "f"(v.y), "f"(v.z), "f"(v.w)
               : "memory");
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// CTA-wide reduction for NWARPS warps; `red` is NWARPS floats of shared memory.
// Every thread returns the total. Contains two __syncthreads.
template <int NWARPS, bool IS_MAX>
__device__ __forceinline__ float block_reduce(float v, float* red) {
  v = IS_MAX ? warp_max(v) : warp_sum(v);
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  if (NWARPS == 1) return v;
  if (lane == 0) red[warp] = v;
  __syncthreads();
  float t = lane < NWARPS ? red[lane] : (IS_MAX ? -INFINITY : 0.f);
  t = IS_MAX ? warp_max(t) : warp_sum(t);
  __syncthreads();  // `red` may be reused by the caller's next reduction
  return t;
}

// -----------------------------------------------------------------------------
// Register-resident row staging shared by softmax and layernorm: a CTA of
// THREADS threads holds one row of up to THREADS*NV*4 floats, NV float4 per
// thread, element index (k*THREADS + t)*4 + e. Padding slots get `pad`.
// -----------------------------------------------------------------------------
template <int THREADS, int NV, bool VEC>
__device__ __forceinline__ void load_row(const float* __restrict__ p, int len, float pad,
                                         float (&v)[NV * 4]) {
  const int t = threadIdx.x;
  if (VEC) {
#pragma unroll
    for (int k = 0; k < NV; ++k) {
      const int idx = (k * THREADS + t) * 4;
      if (idx < len) {  // len % 4 == 0 on this path
        float4 q = ld_stream_f4(p + idx);
        v[4 * k + 0] = q.x;
        v[4 * k + 1] = q.y;
        v[4 * k + 2] = q.z;
        v[4 * k + 3] = q.w;
      } else {
        v[4 * k + 0] = v[4 * k + 1] = v[4 * k + 2] = v[4 * k + 3] = pad;
      }
    }
  } else {
#pragma unroll
    for (int k = 0; k < NV; ++k)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int idx = (k * THREADS + t) * 4 + e;
        v[4 * k + e] = idx < len ? p[idx] : pad;
      }
  }
}

template <int THREADS, int NV, bool VEC>
__device__ __forceinline__ void store_row(float* __restrict__ p, int len,
                                          const float (&v)[NV * 4]) {
  const int t = threadIdx.x;
#pragma unroll
  for (int k = 0; k < NV; ++k) {
    const int idx0 = (k * THREADS + t) * 4;
    if (VEC) {
      if (idx0 < len)
        st_stream_f4(p + idx0, make_float4(v[4 * k], v[4 * k + 1], v[4 * k + 2], v[4 * k + 3]));
    } else {
#pragma unroll
      for (int e = 0; e < 4; ++e)
        if (idx0 + e < len) p[idx0 + e] = v[4 * k + e];
    }
  }
}

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

}  // namespace ctb

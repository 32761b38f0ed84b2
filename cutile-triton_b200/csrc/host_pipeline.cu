// Host-buffer entry points: the caller's data lives in (page-locked) host
// memory and the results go back there. Rows (or elements) move in chunks
// through a device workspace on three streams of the library — host-to-device
// copies, kernels, device-to-host copies — so that, in steady state, chunk
// i+1 is copied in while chunk i is computed and chunk i-1 is copied out.
// PCIe moves data both ways at once, so a row-wise kernel fed from host memory
// runs at the one-way copy rate instead of half of it. They replace the round
// trip a Julia caller writes around a launch — device arrays filled from host
// data, `launch!`, `Array(c)` back (the pattern of test/runtests.jl:42-46) —
// with one call.
//
// Ordering with the caller: the copy stream first waits for everything
// already enqueued on the caller's stream, and the caller's stream is made to
// wait for the last device-to-host copy; the host buffers are complete once
// the caller's stream has completed. One cudaMemcpyAsync per chunk and array.
#include "ctb_common.cuh"

#include <algorithm>
#include <functional>
#include <mutex>

#include "../../include/cutile_b200.h"

namespace ctb {
namespace {

#ifndef CTB_HOST_SLOTS
#define CTB_HOST_SLOTS 3
#endif
#ifndef CTB_HOST_CHUNKS
#define CTB_HOST_CHUNKS 8
#endif
constexpr int NSLOT = CTB_HOST_SLOTS;        // chunks in flight through the workspace
constexpr int MIN_CHUNKS = CTB_HOST_CHUNKS;  // split work at least this finely when it is large
constexpr int64_t MIN_CHUNK_BYTES = 4 << 20;
constexpr int MAX_ARRAYS = 3;

struct DeviceStreams {
  bool ready = false;
  cudaStream_t h2d = nullptr, comp = nullptr, d2h = nullptr;
  cudaEvent_t in_done[NSLOT], comp_done[NSLOT], out_done[NSLOT], entry, exit;
  std::mutex mu;  // one pipeline enqueues at a time per device (events are reused)
};
DeviceStreams g_streams[64];

int device_streams(DeviceStreams** out) {
  int dev = 0;
  CTB_CUDA_CHECK(cudaGetDevice(&dev));
  if (dev < 0 || dev >= 64) return set_error(CTB_ERR_NO_DEVICE, "device ordinal out of range");
  DeviceStreams& d = g_streams[dev];
  *out = &d;
  std::lock_guard<std::mutex> lk(d.mu);
  if (d.ready) return CTB_OK;
  CTB_CUDA_CHECK(cudaStreamCreateWithFlags(&d.h2d, cudaStreamNonBlocking));
  CTB_CUDA_CHECK(cudaStreamCreateWithFlags(&d.comp, cudaStreamNonBlocking));
  CTB_CUDA_CHECK(cudaStreamCreateWithFlags(&d.d2h, cudaStreamNonBlocking));
  for (int i = 0; i < NSLOT; ++i) {
    CTB_CUDA_CHECK(cudaEventCreateWithFlags(&d.in_done[i], cudaEventDisableTiming));
    CTB_CUDA_CHECK(cudaEventCreateWithFlags(&d.comp_done[i], cudaEventDisableTiming));
    CTB_CUDA_CHECK(cudaEventCreateWithFlags(&d.out_done[i], cudaEventDisableTiming));
  }
  CTB_CUDA_CHECK(cudaEventCreateWithFlags(&d.entry, cudaEventDisableTiming));
  CTB_CUDA_CHECK(cudaEventCreateWithFlags(&d.exit, cudaEventDisableTiming));
  d.ready = true;
  return CTB_OK;
}

int64_t round_up(int64_t v, int64_t a) { return (v + a - 1) / a * a; }

// A unit is a row (or an element for vadd); array k holds unit_bytes[k] per unit.
struct Pipe {
  int64_t units = 0;
  int64_t unit_align = 1;  // chunk sizes in units are multiples of this
  int nin = 0, nout = 0;
  const char* hin[MAX_ARRAYS] = {};
  int64_t in_bytes[MAX_ARRAYS] = {};
  char* hout[MAX_ARRAYS] = {};
  int64_t out_bytes[MAX_ARRAYS] = {};
  // Launch the kernel for units [u0, u0 + nu) on `st`: din/dout point at the chunk.
  std::function<int(char* const* din, char* const* dout, int64_t nu, cudaStream_t st)> compute;
};

int64_t slot_bytes_for(const Pipe& p, int64_t nu) {
  int64_t b = 0;
  for (int k = 0; k < p.nin; ++k) b += round_up(nu * p.in_bytes[k], 256);
  for (int k = 0; k < p.nout; ++k) b += round_up(nu * p.out_bytes[k], 256);
  return b;
}

int run(Pipe& p, char* ws, int64_t ws_bytes, cudaStream_t user) {
  if (p.units == 0) return CTB_OK;
  DeviceStreams* d = nullptr;
  if (int rc = device_streams(&d)) return rc;
  // Largest chunk the workspace holds NSLOT times, then no larger than 1/MIN_CHUNKS
  // of the work (but not below MIN_CHUNK_BYTES of traffic) so the stages overlap.
  int64_t per_unit = slot_bytes_for(p, 1);
  int64_t nu = std::max<int64_t>(1, (ws_bytes / NSLOT) / std::max<int64_t>(per_unit, 1));
  while (nu > 1 && slot_bytes_for(p, nu) * NSLOT > ws_bytes) --nu;
  int64_t traffic_unit = 0;
  for (int k = 0; k < p.nin; ++k) traffic_unit += p.in_bytes[k];
  for (int k = 0; k < p.nout; ++k) traffic_unit += p.out_bytes[k];
  const int64_t fine = std::max<int64_t>((p.units + MIN_CHUNKS - 1) / MIN_CHUNKS,
                                         MIN_CHUNK_BYTES / std::max<int64_t>(traffic_unit, 1));
  nu = std::min(nu, std::max<int64_t>(fine, 1));
  nu = std::min(nu, p.units);
  if (p.unit_align > 1 && nu < p.units) nu = std::max(p.unit_align, nu / p.unit_align * p.unit_align);
  const int64_t slot_bytes = slot_bytes_for(p, nu);
  if (slot_bytes * NSLOT > ws_bytes)
    return set_error(CTB_ERR_ARG, "host pipeline: workspace too small for one chunk per slot");
  if (reinterpret_cast<uintptr_t>(ws) % 256)
    return set_error(CTB_ERR_LAYOUT, "host pipeline: workspace must be 256-byte aligned");

  std::lock_guard<std::mutex> lk(d->mu);
  CTB_CUDA_CHECK(cudaEventRecord(d->entry, user));
  CTB_CUDA_CHECK(cudaStreamWaitEvent(d->h2d, d->entry, 0));
  CTB_CUDA_CHECK(cudaStreamWaitEvent(d->comp, d->entry, 0));
  CTB_CUDA_CHECK(cudaStreamWaitEvent(d->d2h, d->entry, 0));
  int rc = CTB_OK;
  int64_t chunk = 0;
  for (int64_t u0 = 0; u0 < p.units; u0 += nu, ++chunk) {
    const int64_t n = std::min(nu, p.units - u0);
    const int slot = (int)(chunk % NSLOT);
    char* base = ws + slot * slot_bytes;
    char* din[MAX_ARRAYS];
    char* dout[MAX_ARRAYS];
    for (int k = 0; k < p.nin; ++k) {
      din[k] = base;
      base += round_up(nu * p.in_bytes[k], 256);
    }
    for (int k = 0; k < p.nout; ++k) {
      dout[k] = base;
      base += round_up(nu * p.out_bytes[k], 256);
    }
    // In: the slot's inputs were last read by the kernel of chunk - NSLOT.
    if (chunk >= NSLOT) CTB_CUDA_CHECK(cudaStreamWaitEvent(d->h2d, d->comp_done[slot], 0));
    for (int k = 0; k < p.nin; ++k)
      CTB_CUDA_CHECK(cudaMemcpyAsync(din[k], p.hin[k] + u0 * p.in_bytes[k], n * p.in_bytes[k],
                                     cudaMemcpyHostToDevice, d->h2d));
    CTB_CUDA_CHECK(cudaEventRecord(d->in_done[slot], d->h2d));
    // Compute: after this chunk's inputs, and after the slot's previous outputs left.
    CTB_CUDA_CHECK(cudaStreamWaitEvent(d->comp, d->in_done[slot], 0));
    if (chunk >= NSLOT) CTB_CUDA_CHECK(cudaStreamWaitEvent(d->comp, d->out_done[slot], 0));
    rc = p.compute(din, dout, n, d->comp);
    if (rc) break;
    CTB_CUDA_CHECK(cudaEventRecord(d->comp_done[slot], d->comp));
    // Out.
    CTB_CUDA_CHECK(cudaStreamWaitEvent(d->d2h, d->comp_done[slot], 0));
    for (int k = 0; k < p.nout; ++k)
      CTB_CUDA_CHECK(cudaMemcpyAsync(p.hout[k] + u0 * p.out_bytes[k], dout[k], n * p.out_bytes[k],
                                     cudaMemcpyDeviceToHost, d->d2h));
    CTB_CUDA_CHECK(cudaEventRecord(d->out_done[slot], d->d2h));
    // Chunk u0 + n onward: advance the unit offset seen by compute through din/dout only.
  }
  // The caller's stream waits for every stage (also on the error path).
  CTB_CUDA_CHECK(cudaEventRecord(d->exit, d->h2d));
  CTB_CUDA_CHECK(cudaStreamWaitEvent(user, d->exit, 0));
  CTB_CUDA_CHECK(cudaEventRecord(d->exit, d->comp));
  CTB_CUDA_CHECK(cudaStreamWaitEvent(user, d->exit, 0));
  CTB_CUDA_CHECK(cudaEventRecord(d->exit, d->d2h));
  CTB_CUDA_CHECK(cudaStreamWaitEvent(user, d->exit, 0));
  return rc;
}

}  // namespace
}  // namespace ctb

using namespace ctb;

extern "C" int64_t ctb_host_workspace_bytes(int64_t unit_bytes_in, int64_t unit_bytes_out,
                                            int64_t units) {
  // Three slots of one eighth of the work each (at least 4 MB of traffic per
  // chunk, at most the whole work), plus 256-byte padding per array.
  if (unit_bytes_in < 0 || unit_bytes_out < 0 || units <= 0) return 0;
  const int64_t per = std::max<int64_t>(unit_bytes_in + unit_bytes_out, 1);
  int64_t nu = std::max<int64_t>((units + MIN_CHUNKS - 1) / MIN_CHUNKS, MIN_CHUNK_BYTES / per);
  nu = std::min(nu, units);
  return NSLOT * (nu * per + 6 * 256);
}

extern "C" int ctb_softmax_f32_host(const float* x, float* y, int32_t len, int32_t count,
                                    void* workspace, int64_t workspace_bytes, void* stream) {
  clear_error();
  if (len < 0 || count < 0) return set_error(CTB_ERR_SHAPE, "softmax_host: negative size");
  if ((int64_t)len * count == 0) return CTB_OK;
  if (!x || !y || !workspace) return set_error(CTB_ERR_ARG, "softmax_host: NULL pointer");
  Pipe p;
  p.units = count;
  p.nin = 1;
  p.hin[0] = reinterpret_cast<const char*>(x);
  p.in_bytes[0] = 4 * (int64_t)len;
  p.nout = 1;
  p.hout[0] = reinterpret_cast<char*>(y);
  p.out_bytes[0] = 4 * (int64_t)len;
  p.compute = [len](char* const* din, char* const* dout, int64_t nu, cudaStream_t st) {
    return ctb_softmax_f32(reinterpret_cast<const float*>(din[0]), reinterpret_cast<float*>(dout[0]),
                           len, (int32_t)nu, len, len, st);
  };
  return run(p, static_cast<char*>(workspace), workspace_bytes, static_cast<cudaStream_t>(stream));
}

extern "C" int ctb_layernorm_fwd_f32_host(const float* x, const float* w, const float* b, float* y,
                                          float* mean, float* rstd, int32_t n, int32_t rows,
                                          float eps, void* workspace, int64_t workspace_bytes,
                                          void* stream) {
  clear_error();
  if (n <= 0 || rows < 0) return set_error(CTB_ERR_SHAPE, "layernorm_fwd_host: need n > 0, rows >= 0");
  if (rows == 0) return CTB_OK;
  if (!x || !w || !b || !y || !mean || !rstd || !workspace)
    return set_error(CTB_ERR_ARG, "layernorm_fwd_host: NULL pointer");
  // w and b (host) go to the head of the workspace once; the rest is the ring.
  const int64_t wb_bytes = round_up(4 * (int64_t)n, 256);
  if (workspace_bytes < 2 * wb_bytes)
    return set_error(CTB_ERR_ARG, "layernorm_fwd_host: workspace too small");
  char* ws = static_cast<char*>(workspace);
  float* dw = reinterpret_cast<float*>(ws);
  float* db = reinterpret_cast<float*>(ws + wb_bytes);
  cudaStream_t user = static_cast<cudaStream_t>(stream);
  CTB_CUDA_CHECK(cudaMemcpyAsync(dw, w, 4 * (size_t)n, cudaMemcpyHostToDevice, user));
  CTB_CUDA_CHECK(cudaMemcpyAsync(db, b, 4 * (size_t)n, cudaMemcpyHostToDevice, user));
  Pipe p;
  p.units = rows;
  p.nin = 1;
  p.hin[0] = reinterpret_cast<const char*>(x);
  p.in_bytes[0] = 4 * (int64_t)n;
  p.nout = 3;
  p.hout[0] = reinterpret_cast<char*>(y);
  p.out_bytes[0] = 4 * (int64_t)n;
  p.hout[1] = reinterpret_cast<char*>(mean);
  p.out_bytes[1] = 4;
  p.hout[2] = reinterpret_cast<char*>(rstd);
  p.out_bytes[2] = 4;
  p.compute = [=](char* const* din, char* const* dout, int64_t nu, cudaStream_t st) {
    return ctb_layernorm_fwd_f32(reinterpret_cast<const float*>(din[0]), dw, db,
                                 reinterpret_cast<float*>(dout[0]),
                                 reinterpret_cast<float*>(dout[1]),
                                 reinterpret_cast<float*>(dout[2]), n, (int32_t)nu, n, n, eps, st);
  };
  return run(p, ws + 2 * wb_bytes, workspace_bytes - 2 * wb_bytes, user);
}

extern "C" int ctb_vadd_host(int32_t dtype, const void* a, const void* b, void* c, int64_t n,
                             void* workspace, int64_t workspace_bytes, void* stream) {
  clear_error();
  const int64_t es = dtype == CTB_F16 ? 2 : dtype == CTB_F32 ? 4 : dtype == CTB_F64 ? 8 : 0;
  if (!es) return set_error(CTB_ERR_DTYPE, "vadd_host: dtype must be F16, F32 or F64");
  if (n < 0) return set_error(CTB_ERR_SHAPE, "vadd_host: negative length");
  if (n == 0) return CTB_OK;
  if (!a || !b || !c || !workspace) return set_error(CTB_ERR_ARG, "vadd_host: NULL pointer");
  Pipe p;
  p.units = n;
  p.unit_align = 256;  // chunk starts stay 16-byte aligned in the workspace and the host arrays
  p.nin = 2;
  p.hin[0] = static_cast<const char*>(a);
  p.hin[1] = static_cast<const char*>(b);
  p.in_bytes[0] = p.in_bytes[1] = es;
  p.nout = 1;
  p.hout[0] = static_cast<char*>(c);
  p.out_bytes[0] = es;
  p.compute = [dtype](char* const* din, char* const* dout, int64_t nu, cudaStream_t st) {
    return ctb_vadd(dtype, din[0], din[1], dout[0], nu, 1, 1, 1, st);
  };
  return run(p, static_cast<char*>(workspace), workspace_bytes, static_cast<cudaStream_t>(stream));
}

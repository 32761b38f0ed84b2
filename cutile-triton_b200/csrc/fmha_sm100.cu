// Attention forward entry point. The tensor-core (tcgen05) kernel lives here;
// shapes it does not take go to the CUDA-core kernel in fmha_simt.cu.
#include "ctb_common.cuh"

namespace ctb {

int fmha_simt(const __half* Q, const __half* K, const __half* V, __half* O, int B, int H, int Sq,
              int Sk, int D, float scale, int causal, cudaStream_t st);

int fmha_device_setup() { return CTB_OK; }
int fmha_take_device_error(unsigned int* out) { return take_device_error(out); }

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
  DeviceProps p;
  if (int rc = current_props(&p)) return rc;
  return fmha_simt((const __half*)Q, (const __half*)K, (const __half*)V, (__half*)O, batch, heads,
                   seq_q, seq_k, head_dim, scale, causal, static_cast<cudaStream_t>(stream));
}

// noalloc.cu -- cra_bwd_noalloc: the backward for callers that cannot
// allocate device memory.  Its scratch is a fixed array in this library's
// device image instead of a caller-provided workspace; see include/cra.h for
// the contract (size limit, first-call set-up, no overlapping calls).
#include <cuda_runtime.h>

#include <cstdio>
#include <mutex>

#include "../../include/cra.h"
#include "params.h"

namespace {

// The backward's scratch on every device that loads the library.
static __device__ __align__(256) unsigned char g_bwd_scratch[CRA_BWD_NOALLOC_SCRATCH_BYTES];

constexpr int kMaxDevices = 64;
std::mutex g_mu;
void* g_scratch_ptr[kMaxDevices] = {};

// Device address of g_bwd_scratch on the current device.  In host code the
// array's name is only a host-side stand-in, so its address must be looked up
// (once per device, with that device current) before it is passed to kernels.
int scratch_address(void** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cra::set_last_error(CRA_ERR_CUDA, "cra_bwd_noalloc: cudaGetDevice failed");
  if (dev < 0 || dev >= kMaxDevices)
    return cra::set_last_error(CRA_ERR_UNSUPPORTED, "cra_bwd_noalloc: device index beyond 63");
  std::lock_guard<std::mutex> lock(g_mu);
  if (!g_scratch_ptr[dev]) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_bwd_scratch);
    if (e != cudaSuccess || !p)
      return cra::set_last_error(CRA_ERR_CUDA, "cra_bwd_noalloc: cudaGetSymbolAddress of the scratch array failed");
    g_scratch_ptr[dev] = p;
  }
  *out = g_scratch_ptr[dev];
  return CRA_OK;
}

}  // namespace

extern "C" int cra_bwd_noalloc(const void* q, const void* k, const void* v, const void* o, const void* d_o,
                               const float* lse, const void* g_k, const void* g_v, const int32_t* g_src,
                               const int64_t* q_strides, const int64_t* k_strides, const int64_t* v_strides,
                               const int64_t* o_strides, const int64_t* do_strides, int batch, int heads,
                               int kv_heads, int seq_len, int head_dim, int dtype, int use_relay, int top_k,
                               float softmax_scale, const float* relay_log_scale, void* dq, void* dk, void* dv,
                               const int64_t* dq_strides, const int64_t* dk_strides, const int64_t* dv_strides,
                               float* d_relay_log_scale, int* dev_error, void* stream) {
  const size_t need = cra_bwd_workspace_bytes(batch, heads, kv_heads, seq_len, head_dim, use_relay, top_k);
  if (need > CRA_BWD_NOALLOC_SCRATCH_BYTES) {  // too large for the fixed scratch
    char text[160];
    snprintf(text, sizeof(text), "cra_bwd_noalloc: these sizes need %zu bytes of scratch > %u (the fixed maximum)",
             need, static_cast<unsigned>(CRA_BWD_NOALLOC_SCRATCH_BYTES));
    return cra::set_last_error(CRA_ERR_WORKSPACE, text);
  }
  void* scratch = nullptr;
  const int s = scratch_address(&scratch);
  if (s != CRA_OK) return s;
  return cra_bwd(q, k, v, o, d_o, lse, g_k, g_v, g_src, q_strides, k_strides, v_strides, o_strides, do_strides,
                 batch, heads, kv_heads, seq_len, head_dim, dtype, use_relay, top_k, softmax_scale, relay_log_scale,
                 dq, dk, dv, dq_strides, dk_strides, dv_strides, d_relay_log_scale, scratch,
                 CRA_BWD_NOALLOC_SCRATCH_BYTES, dev_error, stream);
}

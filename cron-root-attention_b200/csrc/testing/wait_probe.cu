// wait_probe.cu -- test-only library (libcra_waitprobe.so, never loaded by the
// package): exercises the bounded-wait path every libcra kernel relies on.
//
// Built with a short CRA_WAIT_LIMIT_NS.  Each CTA initialises an mbarrier that
// nothing ever arrives at, waits on it with the same warp_wait / mbar_wait the
// attention kernels use, and must come back with "gave up": the wait records
// CRA_DEV_WAIT_TIMEOUT in the caller's error word, sets the CTA's abort flag
// (so the other warps' waits return at once) and the kernel exits normally.
// Nothing is in flight (no TMA copy, no MMA), nothing traps, and the CUDA
// context stays usable, which the test checks by running the real library
// afterwards.
#include "../sm100.cuh"

namespace {

__global__ void __launch_bounds__(128) wait_probe_kernel(int* err, int* out) {
  __shared__ alignas(8) uint64_t bar;
  __shared__ int abort_flag;
  if (threadIdx.x == 0) {
    cra::mbar_init(cra::smem_u32(&bar), 1);
    abort_flag = 0;
    cra::fence_barrier_init();
  }
  __syncthreads();
  const cra::Abort ab{&abort_flag, err};
  const bool ok = cra::warp_wait(cra::smem_u32(&bar), 0, ab);  // phase 0 never completes
  __syncthreads();
  if (threadIdx.x == 0) out[blockIdx.x] = ok ? 1 : 2 + abort_flag;  // 3 = gave up, abort flag set
}

}  // namespace

// Launches `blocks` probe CTAs on `stream`; out[i] receives 3 when CTA i gave
// up on its wait with the abort flag set (1 would mean the wait completed).
extern "C" __attribute__((visibility("default"))) int cra_test_wait_timeout(int* err, int* out, int blocks,
                                                                             void* stream) {
  if (!err || !out || blocks < 1) return 1;
  wait_probe_kernel<<<blocks, 128, 0, static_cast<cudaStream_t>(stream)>>>(err, out);
  return cudaGetLastError() == cudaSuccess ? 0 : 5;
}

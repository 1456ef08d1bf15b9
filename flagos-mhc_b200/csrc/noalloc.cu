// noalloc.cu -- mhc_pre_fwd_noalloc: the pre forward with its scratch memory in a
// fixed static device array instead of a caller-provided workspace.
//
// Who needs this: callers that cannot call cudaMalloc at the point where they run
// the operator -- code under a memory manager that owns the whole device budget
// and forbids raw device allocation (an arena or pooled allocator of a serving
// runtime), or a host-language binding (cgo, JNI, a C plugin) that links only
// this library and has no device allocator of its own.  They still pass device
// pointers for every input and output; only the scratch is taken care of here.
//
// Limits and sharing:
//   - The array holds MHC_PRE_FWD_NOALLOC_SCRATCH_BYTES (16 MiB).  Every GPU that
//     loads the library reserves it until the process exits.  A problem whose
//     scratch need (mhc_pre_fwd_workspace_bytes) exceeds it is rejected with
//     MHC_ERR_SCRATCH_LIMIT before anything is launched.
//   - All calls on a device share the one array and it keeps the previous call's
//     contents.  The pre forward overwrites every scratch word it reads, so
//     nothing has to start at zero.  Two calls whose kernels overlap on the GPU
//     (different streams without ordering between them) race on the array.
//   - The device address of the array is looked up (cudaGetSymbolAddress, with
//     the caller's device current) on every call that is not being captured into
//     a CUDA graph; a captured call reuses the address of the last uncaptured call
//     on that device.  So make one call on each device before any stream capture
//     begins, and again after a cudaDeviceReset, before capturing.
//   - Shapes that fit (the need grows with T: per-token partial sums, plus for
//     bf16/fp16 x the hi/lo split of phi, 2*N*(N+2) rounded up to 16 rows of N*D
//     bf16): N=4 at D <= 7168 up to T = 167,770 tokens; N=8 at D = 4096 up to
//     T = 51,780; N=8 at D = 7168 never fits (the split phi alone is 18.4 MB).
#include <mutex>

#include "common.cuh"
#include "pre_common.cuh"

namespace mhc {

static __device__ __align__(256) unsigned char g_pre_fwd_scratch[MHC_PRE_FWD_NOALLOC_SCRATCH_BYTES];

static std::mutex g_scratch_mu;
static void* g_scratch_addr[64];  // per device: the last address looked up

// The host-side name g_pre_fwd_scratch is only a stand-in for the array; kernels
// must be given the address that cudaGetSymbolAddress returns for the current
// device and context.  The lookup runs on every call made outside stream capture,
// so a context that was torn down and re-created (cudaDeviceReset, or a caller that
// switches driver contexts) gets the array of the context that is current now.
// Inside a capture the address of the last uncaptured call on this device is used.
static int scratch_address(cudaStream_t stream, void** out) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return MHC_ERR_CUDA;
  if (dev < 0 || dev >= 64) return MHC_ERR_DEVICE;
  cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
  if (cudaStreamIsCapturing(stream, &cs) != cudaSuccess) return MHC_ERR_CUDA;
  std::lock_guard<std::mutex> lock(g_scratch_mu);
  if (cs == cudaStreamCaptureStatusNone) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_pre_fwd_scratch) != cudaSuccess || p == nullptr)
      return MHC_ERR_CUDA;
    g_scratch_addr[dev] = p;
  } else if (g_scratch_addr[dev] == nullptr) {
    return MHC_ERR_CUDA;  // first call on this device made inside a capture
  }
  *out = g_scratch_addr[dev];
  return MHC_OK;
}

}  // namespace mhc

extern "C" int mhc_pre_fwd_noalloc(const void* x, const float* phi, const float* alpha,
                                   const float* base, int64_t T, int32_t N, int64_t D,
                                   int32_t dtype, float norm_eps, float hc_eps,
                                   float clamp_min, float clamp_max, int32_t iter_times,
                                   void* y, float* post_out, float* comb_frag, float* inv_rms,
                                   float* x_scaled, float* mixes, float* h_res_logits,
                                   float* pre, void* stream) {
  const size_t need = mhc_pre_fwd_workspace_bytes(T, N, D, dtype);
  if (need > (size_t)MHC_PRE_FWD_NOALLOC_SCRATCH_BYTES) return MHC_ERR_SCRATCH_LIMIT;
  void* scratch = nullptr;
  if (T > 0) {
    // argument errors are reported by mhc_pre_fwd below; only look the array up
    // once the call would actually launch
    const int st = mhc::scratch_address((cudaStream_t)stream, &scratch);
    if (st != MHC_OK) return st;
  }
  return mhc_pre_fwd(x, phi, alpha, base, T, N, D, dtype, norm_eps, hc_eps, clamp_min,
                     clamp_max, iter_times, y, post_out, comb_frag, inv_rms, x_scaled, mixes,
                     h_res_logits, pre, scratch, (size_t)MHC_PRE_FWD_NOALLOC_SCRATCH_BYTES,
                     stream);
}

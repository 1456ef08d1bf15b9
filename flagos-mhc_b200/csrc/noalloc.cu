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
//   - The device address of the array is looked up on the first call on each
//     device (cudaGetSymbolAddress with that device current).  Make that first
//     call before any stream capture begins.
#include <mutex>

#include "common.cuh"
#include "pre_common.cuh"

namespace mhc {

static __device__ __align__(256) unsigned char g_pre_fwd_scratch[MHC_PRE_FWD_NOALLOC_SCRATCH_BYTES];

static std::mutex g_scratch_mu;
static void* g_scratch_addr[64];  // per device; the symbol's device address

// The host-side name g_pre_fwd_scratch is only a stand-in for the array; kernels
// must be given the address returned by cudaGetSymbolAddress for the current device.
static int scratch_address(void** out) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return MHC_ERR_CUDA;
  if (dev < 0 || dev >= 64) return MHC_ERR_DEVICE;
  std::lock_guard<std::mutex> lock(g_scratch_mu);
  if (g_scratch_addr[dev] == nullptr) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_pre_fwd_scratch) != cudaSuccess || p == nullptr)
      return MHC_ERR_CUDA;
    g_scratch_addr[dev] = p;
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
    const int st = mhc::scratch_address(&scratch);
    if (st != MHC_OK) return st;
  }
  return mhc_pre_fwd(x, phi, alpha, base, T, N, D, dtype, norm_eps, hc_eps, clamp_min,
                     clamp_max, iter_times, y, post_out, comb_frag, inv_rms, x_scaled, mixes,
                     h_res_logits, pre, scratch, (size_t)MHC_PRE_FWD_NOALLOC_SCRATCH_BYTES,
                     stream);
}

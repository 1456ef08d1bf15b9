// capi.cu -- the extern "C" boundary: argument checks, then dispatch.
#include <math.h>
#include <stdlib.h>

#include <atomic>

#include "common.cuh"
#include "pre_common.cuh"

namespace mhc {

int post_fwd_dispatch(int32_t N, int32_t dtype, const void* x, const float* h_res,
                      const void* h_out, const float* h_post, void* out, int64_t T, int64_t D,
                      TokStride st, cudaStream_t s);
int post_bwd_dispatch(int32_t N, int32_t dtype, const void* gy, const void* x,
                      const float* h_res, const void* h_out, const float* h_post, void* gx,
                      float* ghres, void* ghout, float* ghpost, int64_t T, int64_t D,
                      TokStride st, cudaStream_t s);

int pre_fwd_tc_device_error();
int pre_bwd_tc_device_error();
int pre_bwd_tc8_device_error();
int pre_bwd_tc32_device_error();
int peer_device_error();
int post_mix_device_error();
bool post_mix_eligible(int64_t T, int32_t N, int64_t D, int32_t dtype, const void* x,
                       const void* h_out, const void* out);
int post_mix_layers(int64_t T, int64_t D);
size_t post_mix_ws_bytes(int64_t D);
int post_mix_run(const void* x, const float* h_res, const void* h_out, const float* h_post,
                 void* out, int64_t T, int64_t D, int32_t dtype, const float* phi_next,
                 float* premix, int32_t layers, void* ws, cudaStream_t s);
int tc_host_device_error();

static std::atomic<unsigned long long> g_launches{0};
void note_launch() { g_launches.fetch_add(1, std::memory_order_relaxed); }

// MHC_PDL: 0 = no launch carries the attribute; 1 = every launch does; 2 (default) =
// every launch but the first of each entry point call.
static int pdl_mode() {
  static const int m = [] {
    const char* v = getenv("MHC_PDL");
    return (v && (v[0] == '0' || v[0] == '1')) ? v[0] - '0' : 2;
  }();
  return m;
}
bool pdl_enabled() { return pdl_mode() != 0; }

static thread_local bool g_first_launch = false;
void pdl_new_call() { g_first_launch = true; }
bool pdl_first_launch() {
  const bool f = g_first_launch;
  g_first_launch = false;
  return f && pdl_mode() == 2;
}

// Per-device cache of the SM count and of the sm_100 check (set once per device).
static int g_sms[64];
static int g_arch_ok[64];  // 0 unknown, 1 ok, 2 not sm_100

int sm_count() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 148;
  if (g_sms[dev] == 0) {
    int v = 0;
    if (cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || v <= 0)
      v = 148;
    g_sms[dev] = v;
  }
  return g_sms[dev];
}

static int check_device() {
  pdl_new_call();
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return MHC_ERR_CUDA;
  if (dev < 0 || dev >= 64) return MHC_ERR_DEVICE;
  if (g_arch_ok[dev] == 0) {
    int major = 0, minor = 0;
    if (cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev) != cudaSuccess ||
        cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, dev) != cudaSuccess)
      return MHC_ERR_CUDA;
    g_arch_ok[dev] = (major == 10 && minor == 0) ? 1 : 2;
  }
  return g_arch_ok[dev] == 1 ? MHC_OK : MHC_ERR_DEVICE;
}

static bool dtype_ok(int32_t d) { return d == MHC_F32 || d == MHC_F16 || d == MHC_BF16; }

static int check_common(int64_t T, int32_t N, int64_t D, int32_t dtype) {
  if (T < 0 || D <= 0) return MHC_ERR_INVALID_ARGUMENT;
  if (N < 1 || N > kMaxN) return MHC_ERR_UNSUPPORTED_N;
  if (!dtype_ok(dtype)) return MHC_ERR_UNSUPPORTED_DTYPE;
  return MHC_OK;
}

static int small_params(float hc_eps, float cmin, float cmax, int32_t iters, SmallParams* sp) {
  if (!(iters >= 0) || !isfinite(hc_eps)) return MHC_ERR_INVALID_ARGUMENT;
  sp->a0 = sp->a1 = sp->a2 = 0.f;  // read from the alpha tensor on the device
  sp->hc_eps = hc_eps;
  sp->clamp_min = cmin;
  sp->clamp_max = cmax;
  sp->clamp_on = (cmin != 0.0f || cmax != 0.0f) ? 1 : 0;  // src/mhc_pre_clamp_sinkhorn.py:923
  sp->iters = iters;
  return MHC_OK;
}

}  // namespace mhc

using namespace mhc;

#define RETURN_IF(x)            \
  do {                          \
    int _st = (x);              \
    if (_st != MHC_OK) return _st; \
  } while (0)

extern "C" {

const char* mhc_status_string(int status) {
  switch (status) {
    case MHC_OK: return "ok";
    case MHC_ERR_INVALID_ARGUMENT: return "invalid argument";
    case MHC_ERR_UNSUPPORTED_N: return "unsupported hcMult (N must be 1..8)";
    case MHC_ERR_UNSUPPORTED_DTYPE: return "unsupported dtype";
    case MHC_ERR_WORKSPACE: return "workspace missing, too small or not 256-byte aligned";
    case MHC_ERR_CUDA: return "CUDA error";
    case MHC_ERR_DEVICE: return "current device is not an sm_100 (B200) GPU";
    case MHC_ERR_TIMEOUT: return "a bounded device-side wait timed out";
    case MHC_ERR_SCRATCH_LIMIT:
      return "problem needs more scratch than the static array of the no-alloc entry point holds";
    default: return "unknown status";
  }
}

int mhc_version(void) { return 100; }

uint64_t mhc_kernel_launches(void) { return g_launches.load(std::memory_order_relaxed); }

int mhc_device_status(void) {
  if (cudaDeviceSynchronize() != cudaSuccess) return MHC_ERR_CUDA;
  const int a = pre_fwd_tc_device_error();
  const int b = pre_bwd_tc_device_error();
  const int c = pre_bwd_tc8_device_error();
  const int d = peer_device_error();
  const int e = tc_host_device_error();
  const int f = post_mix_device_error();
  const int g = pre_bwd_tc32_device_error();
  const int all[7] = {a, b, c, d, e, f, g};
  for (int v : all)
    if (v != MHC_OK) return v;
  return MHC_OK;
}

int mhc_post_fwd_strided(const void* x, int64_t x_token_stride, const float* h_res,
                         const void* h_out, int64_t h_out_token_stride, const float* h_post,
                         void* out, int64_t T, int32_t N, int64_t D, int32_t dtype,
                         void* stream) {
  RETURN_IF(check_common(T, N, D, dtype));
  if (x_token_stride < (int64_t)N * D || h_out_token_stride < D) return MHC_ERR_INVALID_ARGUMENT;
  if (T == 0) return MHC_OK;
  if (!x || !h_res || !h_out || !h_post || !out) return MHC_ERR_INVALID_ARGUMENT;
  RETURN_IF(check_device());
  const TokStride st{x_token_stride, 0, h_out_token_stride};
  return post_fwd_dispatch(N, dtype, x, h_res, h_out, h_post, out, T, D, st,
                           (cudaStream_t)stream);
}

int mhc_post_fwd(const void* x, const float* h_res, const void* h_out, const float* h_post,
                 void* out, int64_t T, int32_t N, int64_t D, int32_t dtype, void* stream) {
  return mhc_post_fwd_strided(x, (int64_t)N * D, h_res, h_out, D, h_post, out, T, N, D, dtype,
                              stream);
}

int mhc_post_bwd_strided(const void* grad_y, int64_t grad_y_token_stride, const void* x,
                         int64_t x_token_stride, const float* h_res, const void* h_out,
                         int64_t h_out_token_stride, const float* h_post, void* grad_x,
                         float* grad_h_res, void* grad_h_out, float* grad_h_post, int64_t T,
                         int32_t N, int64_t D, int32_t dtype, void* stream) {
  RETURN_IF(check_common(T, N, D, dtype));
  if (grad_y_token_stride < (int64_t)N * D || x_token_stride < (int64_t)N * D ||
      h_out_token_stride < D)
    return MHC_ERR_INVALID_ARGUMENT;
  if (T == 0) return MHC_OK;
  if (!grad_y || !x || !h_res || !h_out || !h_post || !grad_x || !grad_h_res || !grad_h_out ||
      !grad_h_post)
    return MHC_ERR_INVALID_ARGUMENT;
  RETURN_IF(check_device());
  const TokStride st{x_token_stride, grad_y_token_stride, h_out_token_stride};
  return post_bwd_dispatch(N, dtype, grad_y, x, h_res, h_out, h_post, grad_x, grad_h_res,
                           grad_h_out, grad_h_post, T, D, st, (cudaStream_t)stream);
}

int mhc_post_bwd(const void* grad_y, const void* x, const float* h_res, const void* h_out,
                 const float* h_post, void* grad_x, float* grad_h_res, void* grad_h_out,
                 float* grad_h_post, int64_t T, int32_t N, int64_t D, int32_t dtype,
                 void* stream) {
  return mhc_post_bwd_strided(grad_y, (int64_t)N * D, x, (int64_t)N * D, h_res, h_out, D,
                              h_post, grad_x, grad_h_res, grad_h_out, grad_h_post, T, N, D,
                              dtype, stream);
}

size_t mhc_pre_fwd_workspace_bytes(int64_t T, int32_t N, int64_t D, int32_t dtype) {
  if (check_common(T, N, D, dtype) != MHC_OK) return 0;
  return pre_fwd_ws_bytes(T, N, D, dtype);
}

int mhc_pre_fwd_strided(const void* x, int64_t x_token_stride, const float* phi,
                        const float* alpha, const float* base, int64_t T, int32_t N, int64_t D,
                        int32_t dtype, float norm_eps, float hc_eps, float clamp_min,
                        float clamp_max, int32_t iter_times, void* y, float* post_out,
                        float* comb_frag, float* inv_rms, float* x_scaled, float* mixes,
                        float* h_res_logits, float* pre, void* workspace,
                        size_t workspace_bytes, void* stream) {
  RETURN_IF(check_common(T, N, D, dtype));
  if (x_token_stride < (int64_t)N * D) return MHC_ERR_INVALID_ARGUMENT;
  PreFwdArgs a{};
  RETURN_IF(small_params(hc_eps, clamp_min, clamp_max, iter_times, &a.sp));
  if (T == 0) return MHC_OK;
  if (!x || !phi || !alpha || !base || !y || !post_out || !comb_frag || !inv_rms || !mixes ||
      !pre)
    return MHC_ERR_INVALID_ARGUMENT;
  const size_t need = pre_fwd_ws_bytes(T, N, D, dtype);
  if (need > 0 && (!workspace || workspace_bytes < need || !aligned16(workspace) ||
                   (reinterpret_cast<uintptr_t>(workspace) & 255) != 0))
    return MHC_ERR_WORKSPACE;
  RETURN_IF(check_device());
  a.x = x; a.phi = phi; a.alpha = alpha; a.base = base;
  a.T = T; a.D = D; a.N = N; a.dtype = dtype; a.norm_eps = norm_eps;
  a.x_ts = x_token_stride;
  a.y = y; a.post_out = post_out; a.comb_frag = comb_frag; a.inv_rms = inv_rms;
  a.x_scaled = x_scaled; a.mixes = mixes; a.h_res_logits = h_res_logits; a.pre = pre;
  a.workspace = workspace; a.workspace_bytes = workspace_bytes;
  return pre_fwd_dispatch(a, (cudaStream_t)stream);
}

int mhc_pre_fwd(const void* x, const float* phi, const float* alpha, const float* base,
                int64_t T, int32_t N, int64_t D, int32_t dtype, float norm_eps, float hc_eps,
                float clamp_min, float clamp_max, int32_t iter_times, void* y, float* post_out,
                float* comb_frag, float* inv_rms, float* x_scaled, float* mixes,
                float* h_res_logits, float* pre, void* workspace, size_t workspace_bytes,
                void* stream) {
  return mhc_pre_fwd_strided(x, (int64_t)N * D, phi, alpha, base, T, N, D, dtype, norm_eps,
                             hc_eps, clamp_min, clamp_max, iter_times, y, post_out, comb_frag,
                             inv_rms, x_scaled, mixes, h_res_logits, pre, workspace,
                             workspace_bytes, stream);
}

size_t mhc_pre_bwd_workspace_bytes(int64_t T, int32_t N, int64_t D, int32_t dtype,
                                   int32_t iter_times) {
  if (check_common(T, N, D, dtype) != MHC_OK || iter_times < 0) return 0;
  return pre_bwd_ws_bytes(T, N, D, dtype, iter_times);
}

}  // extern "C"

static int pre_bwd_entry(const void* x, int64_t x_ts, const float* phi, const float* alpha,
                         const float* base,
                         const float* inv_rms, const float* mixes, const float* pre,
                         const void* grad_y, const float* grad_post_out,
                         const float* grad_comb_frag, int64_t gy_ts, int64_t T, int32_t N,
                         int64_t D, int32_t dtype, float hc_eps, float clamp_min, float clamp_max,
                         int32_t iter_times, const void* grad_x_acc, void* grad_x,
                         float* grad_phi, float* grad_alpha, float* grad_base, void* workspace,
                         size_t workspace_bytes, void* stream) {
  RETURN_IF(check_common(T, N, D, dtype));
  if (x_ts < (int64_t)N * D || gy_ts < D) return MHC_ERR_INVALID_ARGUMENT;
  PreBwdArgs a{};
  RETURN_IF(small_params(hc_eps, clamp_min, clamp_max, iter_times, &a.sp));
  if (!phi || !alpha || !base || !grad_phi || !grad_alpha || !grad_base)
    return MHC_ERR_INVALID_ARGUMENT;
  if (T > 0 && (!x || !inv_rms || !mixes || !pre || !grad_y || !grad_post_out ||
                !grad_comb_frag || !grad_x))
    return MHC_ERR_INVALID_ARGUMENT;
  const size_t need = pre_bwd_ws_bytes(T, N, D, dtype, iter_times);
  if (T > 0 && need > 0 &&
      (!workspace || workspace_bytes < need || (reinterpret_cast<uintptr_t>(workspace) & 255) != 0))
    return MHC_ERR_WORKSPACE;
  RETURN_IF(check_device());
  a.x = x; a.phi = phi; a.alpha = alpha; a.base = base; a.inv_rms = inv_rms; a.mixes = mixes;
  a.pre = pre; a.grad_y = grad_y; a.grad_post = grad_post_out; a.grad_comb = grad_comb_frag;
  a.T = T; a.D = D; a.N = N; a.dtype = dtype;
  a.x_ts = x_ts; a.gy_ts = gy_ts;
  a.grad_x = grad_x; a.grad_phi = grad_phi; a.grad_alpha = grad_alpha; a.grad_base = grad_base;
  a.grad_x_acc = grad_x_acc;
  a.workspace = workspace; a.workspace_bytes = workspace_bytes;
  return pre_bwd_dispatch(a, (cudaStream_t)stream);
}

extern "C" {

int mhc_pre_bwd(const void* x, const float* phi, const float* alpha, const float* base,
                const float* inv_rms, const float* mixes, const float* pre, const void* grad_y,
                const float* grad_post_out, const float* grad_comb_frag, int64_t T, int32_t N,
                int64_t D, int32_t dtype, float norm_eps, float hc_eps, float clamp_min,
                float clamp_max, int32_t iter_times, void* grad_x, float* grad_phi,
                float* grad_alpha, float* grad_base, void* workspace, size_t workspace_bytes,
                void* stream) {
  (void)norm_eps;  // inv_rms arrives precomputed
  return pre_bwd_entry(x, (int64_t)N * D, phi, alpha, base, inv_rms, mixes, pre, grad_y,
                       grad_post_out, grad_comb_frag, D, T, N, D, dtype, hc_eps, clamp_min,
                       clamp_max, iter_times, nullptr, grad_x, grad_phi, grad_alpha, grad_base,
                       workspace, workspace_bytes, stream);
}

int mhc_pre_bwd_accumulate(const void* x, const float* phi, const float* alpha,
                           const float* base, const float* inv_rms, const float* mixes,
                           const float* pre, const void* grad_y, const float* grad_post_out,
                           const float* grad_comb_frag, int64_t T, int32_t N, int64_t D,
                           int32_t dtype, float norm_eps, float hc_eps, float clamp_min,
                           float clamp_max, int32_t iter_times, const void* grad_x_accumulate,
                           void* grad_x, float* grad_phi, float* grad_alpha, float* grad_base,
                           void* workspace, size_t workspace_bytes, void* stream) {
  (void)norm_eps;
  if (T > 0 && !grad_x_accumulate) return MHC_ERR_INVALID_ARGUMENT;
  return pre_bwd_entry(x, (int64_t)N * D, phi, alpha, base, inv_rms, mixes, pre, grad_y,
                       grad_post_out, grad_comb_frag, D, T, N, D, dtype, hc_eps, clamp_min,
                       clamp_max, iter_times, grad_x_accumulate, grad_x, grad_phi, grad_alpha,
                       grad_base, workspace, workspace_bytes, stream);
}

int mhc_pre_bwd_strided(const void* x, int64_t x_token_stride, const float* phi,
                        const float* alpha, const float* base, const float* inv_rms,
                        const float* mixes, const float* pre, const void* grad_y,
                        int64_t grad_y_token_stride, const float* grad_post_out,
                        const float* grad_comb_frag, int64_t T, int32_t N, int64_t D,
                        int32_t dtype, float norm_eps, float hc_eps, float clamp_min,
                        float clamp_max, int32_t iter_times, const void* grad_x_accumulate,
                        void* grad_x, float* grad_phi, float* grad_alpha, float* grad_base,
                        void* workspace, size_t workspace_bytes, void* stream) {
  (void)norm_eps;
  return pre_bwd_entry(x, x_token_stride, phi, alpha, base, inv_rms, mixes, pre, grad_y,
                       grad_post_out, grad_comb_frag, grad_y_token_stride, T, N, D, dtype,
                       hc_eps, clamp_min, clamp_max, iter_times, grad_x_accumulate, grad_x,
                       grad_phi, grad_alpha, grad_base, workspace, workspace_bytes, stream);
}

}  // extern "C"

extern "C" {

int mhc_post_fwd_mix_supported(int64_t T, int32_t N, int64_t D, int32_t dtype) {
  // pointers are only checked for alignment: any 256-byte aligned stand-in will do
  const void* p = reinterpret_cast<const void*>(uintptr_t(256));
  return post_mix_eligible(T, N, D, dtype, p, p, p) ? 1 : 0;
}

int32_t mhc_post_fwd_mix_layers(int64_t T, int32_t N, int64_t D, int32_t dtype) {
  if (!mhc_post_fwd_mix_supported(T, N, D, dtype)) return 0;
  return post_mix_layers(T, D);
}

size_t mhc_post_fwd_mix_workspace_bytes(int64_t T, int32_t N, int64_t D, int32_t dtype) {
  if (!mhc_post_fwd_mix_supported(T, N, D, dtype)) return 0;
  return post_mix_ws_bytes(D);
}

int mhc_post_fwd_mix(const void* x, const float* h_res, const void* h_out, const float* h_post,
                     void* out, int64_t T, int32_t N, int64_t D, int32_t dtype,
                     const float* phi_next, float* premix, void* workspace,
                     size_t workspace_bytes, void* stream) {
  RETURN_IF(check_common(T, N, D, dtype));
  if (T == 0) return MHC_OK;
  if (!x || !h_res || !h_out || !h_post || !out || !phi_next || !premix)
    return MHC_ERR_INVALID_ARGUMENT;
  if (!post_mix_eligible(T, N, D, dtype, x, h_out, out) || !aligned16(phi_next))
    return MHC_ERR_INVALID_ARGUMENT;
  const size_t need = post_mix_ws_bytes(D);
  if (!workspace || workspace_bytes < need || (reinterpret_cast<uintptr_t>(workspace) & 255))
    return MHC_ERR_WORKSPACE;
  RETURN_IF(check_device());
  return post_mix_run(x, h_res, h_out, h_post, out, T, D, dtype, phi_next, premix,
                      post_mix_layers(T, D), workspace, (cudaStream_t)stream);
}

int mhc_pre_fwd_premixed(const void* x, const float* premix, int32_t premix_layers,
                         const float* alpha, const float* base, int64_t T, int32_t N,
                         int64_t D, int32_t dtype, float norm_eps, float hc_eps,
                         float clamp_min, float clamp_max, int32_t iter_times, void* y,
                         float* post_out, float* comb_frag, float* inv_rms, float* x_scaled,
                         float* mixes, float* h_res_logits, float* pre, void* stream) {
  RETURN_IF(check_common(T, N, D, dtype));
  PreFwdArgs a{};
  RETURN_IF(small_params(hc_eps, clamp_min, clamp_max, iter_times, &a.sp));
  if (N != 4) return MHC_ERR_UNSUPPORTED_N;
  if (T == 0) return MHC_OK;
  if (!x || !premix || premix_layers < 1 || !alpha || !base || !y || !post_out || !comb_frag ||
      !inv_rms || !mixes || !pre)
    return MHC_ERR_INVALID_ARGUMENT;
  RETURN_IF(check_device());
  a.x = x; a.alpha = alpha; a.base = base;
  a.T = T; a.D = D; a.N = N; a.dtype = dtype; a.norm_eps = norm_eps;
  a.x_ts = (int64_t)N * D;
  a.y = y; a.post_out = post_out; a.comb_frag = comb_frag; a.inv_rms = inv_rms;
  a.x_scaled = x_scaled; a.mixes = mixes; a.h_res_logits = h_res_logits; a.pre = pre;
  a.premix = premix; a.premix_layers = premix_layers;
  return pre_fwd_dispatch(a, (cudaStream_t)stream);
}

}  // extern "C"

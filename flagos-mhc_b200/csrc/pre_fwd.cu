// pre_fwd.cu -- mhc_pre_clamp_sinkhorn forward, generic path (any dtype, N 1..8).
//
// Three stream-ordered kernels:
//   1. pre_mix_kernel     raw[t,k] = <x[t,:], phi[k,:]>, sumsq[t] = <x[t,:], x[t,:]>
//                         (token tile x K-chunk tiling in shared memory, fp32 FMA)
//   2. pre_small_kernel   per token: inv_rms, mixes = inv*raw, heads, clamp,
//                         softmax, Sinkhorn (one thread per token)
//   3. pre_apply_kernel   per token: x_scaled = x*inv (optional), y = sum_n pre[n] x[n]
// Reference replaced: src/mhc_pre_clamp_sinkhorn.py:857-971 (rms_scale, torch.mm,
// sinkhorn kernels, y_scale); semantics :974-1022.
#include "common.cuh"
#include "pre_common.cuh"

#include <type_traits>

namespace mhc {

constexpr int kMixTT = 32;   // tokens per CTA
constexpr int kMixKC = 128;  // columns per K chunk

template <typename E, int N>
__global__ void __launch_bounds__(256)
pre_mix_kernel(const E* __restrict__ x, const float* __restrict__ phi,
               float* __restrict__ raw, float* __restrict__ sumsq, int64_t T, int64_t HC,
               int64_t x_ts) {
  pdl_enter();
  constexpr int HM = hc_mix(N);
  extern __shared__ float smem[];
  float* xs = smem;                              // [kMixTT][kMixKC + 1]
  float* ps = smem + kMixTT * (kMixKC + 1);      // [HM][kMixKC]
  const int tid = threadIdx.x;
  const int tt = tid >> 3, kl = tid & 7;
  const int64_t t0 = (int64_t)blockIdx.x * kMixTT;
  float acc[HM];
#pragma unroll
  for (int k = 0; k < HM; ++k) acc[k] = 0.f;
  float sq = 0.f;
  for (int64_t kc = 0; kc < HC; kc += kMixKC) {
    for (int idx = tid; idx < kMixTT * kMixKC; idx += 256) {
      const int r = idx / kMixKC, c = idx % kMixKC;
      const int64_t t = t0 + r;
      xs[r * (kMixKC + 1) + c] = (t < T && kc + c < HC) ? ld1<E>(x + t * x_ts + kc + c) : 0.f;
    }
    for (int idx = tid; idx < HM * kMixKC; idx += 256) {
      const int k = idx / kMixKC, c = idx % kMixKC;
      ps[idx] = (kc + c < HC) ? __ldg(phi + (int64_t)k * HC + kc + c) : 0.f;
    }
    __syncthreads();
#pragma unroll 4
    for (int i = 0; i < kMixKC / 8; ++i) {
      const int c = kl + 8 * i;
      const float xv = xs[tt * (kMixKC + 1) + c];
      sq = fmaf(xv, xv, sq);
#pragma unroll
      for (int k = 0; k < HM; ++k) acc[k] = fmaf(xv, ps[k * kMixKC + c], acc[k]);
    }
    __syncthreads();
  }
#pragma unroll
  for (int o = 1; o < 8; o <<= 1) {
    sq += __shfl_xor_sync(0xffffffffu, sq, o);
#pragma unroll
    for (int k = 0; k < HM; ++k) acc[k] += __shfl_xor_sync(0xffffffffu, acc[k], o);
  }
  const int64_t t = t0 + tt;
  if (kl == 0 && t < T) {
#pragma unroll
    for (int k = 0; k < HM; ++k) raw[t * HM + k] = acc[k];
    sumsq[t] = sq;
  }
}

template <int N>
__global__ void __launch_bounds__(128)
pre_small_kernel(const float* __restrict__ raw, const float* __restrict__ sumsq,
                 const float* __restrict__ alpha, const float* __restrict__ base, int64_t T,
                 int64_t HC, float norm_eps, SmallParams sp, float* __restrict__ inv_rms,
                 float* __restrict__ mixes, float* __restrict__ pre, float* __restrict__ post,
                 float* __restrict__ comb, float* __restrict__ logits_out) {
  pdl_enter();
  constexpr int HM = hc_mix(N);
  __shared__ float sbase[HM];
  for (int i = threadIdx.x; i < HM; i += blockDim.x) sbase[i] = base[i];
  __syncthreads();
  sp.a0 = alpha[0]; sp.a1 = alpha[1]; sp.a2 = alpha[2];
  const int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (t >= T) return;
  const float inv = inv_rms_from_sumsq(sumsq[t], HC, norm_eps);
  float mix[HM];
#pragma unroll
  for (int k = 0; k < HM; ++k) mix[k] = raw[t * HM + k] * inv;
  small_outputs<N>(mix, sbase, sp, t, inv, inv_rms, mixes, pre, post, comb, logits_out);
}

template <typename E, int N, bool VEC>
__global__ void __launch_bounds__(256)
pre_apply_kernel(const E* __restrict__ x, const float* __restrict__ inv_rms,
                 const float* __restrict__ pre, E* __restrict__ y, float* __restrict__ x_scaled,
                 int64_t T, int64_t D, int64_t xs) {
  pdl_enter();
  constexpr int P = VEC ? Pack<E>::n : 1;
  const int lane = threadIdx.x & 31;
  const int64_t nwarps = (int64_t)gridDim.x * (blockDim.x >> 5);
  const int64_t nchunk = D / P;
  for (int64_t t = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); t < T;
       t += nwarps) {
    const float inv = inv_rms[t];
    float pr[N];
#pragma unroll
    for (int n = 0; n < N; ++n) pr[n] = pre[t * N + n];
    const E* xt = x + t * xs;
    float* xst = x_scaled ? x_scaled + t * N * D : nullptr;
    for (int64_t c = lane; c < nchunk; c += 32) {
      float xv[N][P];
#pragma unroll
      for (int n = 0; n < N; ++n) load_pack<E, VEC>(xt + n * D + c * P, xv[n]);
      float o[P];
#pragma unroll
      for (int e = 0; e < P; ++e) {
        float s = 0.f;
#pragma unroll
        for (int n = 0; n < N; ++n) s = fmaf(xv[n][e], pr[n], s);
        o[e] = s;
      }
      store_pack<E, VEC>(y + t * D + c * P, o);
      if (xst) {
#pragma unroll
        for (int n = 0; n < N; ++n) {
          float* dst = xst + n * D + c * P;
#pragma unroll
          for (int e = 0; e < P; e += 4) {
            if constexpr (P >= 4) {
              __stcs(reinterpret_cast<float4*>(dst + e),
                     make_float4(xv[n][e] * inv, xv[n][e + 1] * inv, xv[n][e + 2] * inv,
                                 xv[n][e + 3] * inv));
            } else {
              dst[e] = xv[n][e] * inv;
            }
          }
        }
      }
    }
  }
}

// 16-bit x (bf16 or fp16), D % 16 == 0: a lane handles 16 consecutive d per row with
// 32-byte accesses (one load per row of x, one store of y, two stores of x_scaled per row).
template <typename E, int N>
__global__ void __launch_bounds__(256)
pre_apply_x16_kernel(const E* __restrict__ x, const float* __restrict__ inv_rms,
                     const float* __restrict__ pre, E* __restrict__ y,
                     float* __restrict__ x_scaled, int64_t T, int64_t D, int64_t xs) {
  pdl_enter();
  const int lane = threadIdx.x & 31;
  const int64_t nwarps = (int64_t)gridDim.x * (blockDim.x >> 5);
  const int64_t nchunk = D / 16;
  for (int64_t t = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); t < T;
       t += nwarps) {
    const float inv = inv_rms[t];
    float pr[N];
#pragma unroll
    for (int n = 0; n < N; ++n) pr[n] = pre[t * N + n];
    const E* xt = x + t * xs;
    float* xst = x_scaled ? x_scaled + t * N * D : nullptr;
    for (int64_t c = lane; c < nchunk; c += 32) {
      U8 xv[N];
#pragma unroll
      for (int n = 0; n < N; ++n) xv[n] = ld_global_32B(xt + n * D + c * 16);
      float o[16];
#pragma unroll
      for (int e = 0; e < 16; ++e) o[e] = 0.f;
#pragma unroll
      for (int n = 0; n < N; ++n) {
        float f[16];
        widen<E>(xv[n].a, f);
        widen<E>(xv[n].b, f + 8);
#pragma unroll
        for (int e = 0; e < 16; ++e) o[e] = fmaf(f[e], pr[n], o[e]);
        if (xst) {
          float* dst = xst + n * D + c * 16;
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            uint4 a = make_uint4(__float_as_uint(f[8 * h] * inv), __float_as_uint(f[8 * h + 1] * inv),
                                 __float_as_uint(f[8 * h + 2] * inv), __float_as_uint(f[8 * h + 3] * inv));
            uint4 b = make_uint4(__float_as_uint(f[8 * h + 4] * inv), __float_as_uint(f[8 * h + 5] * inv),
                                 __float_as_uint(f[8 * h + 6] * inv), __float_as_uint(f[8 * h + 7] * inv));
            st_global_32B(dst + 8 * h, a, b);
          }
        }
      }
      st_global_32B(y + t * D + c * 16, narrow<E>(o), narrow<E>(o + 8));
    }
  }
}

// ---------------------------------------------------------------------------
// Host side
// ---------------------------------------------------------------------------
bool pre_fwd_tc_eligible(const PreFwdArgs& a);
size_t pre_fwd_tc_ws_bytes(int64_t T, int32_t N, int64_t D, int32_t dtype);
int pre_fwd_tc_mix(const PreFwdArgs& a, cudaStream_t s);
int pre_fwd_finish_premix(const PreFwdArgs& a, cudaStream_t s);

// the generic path and the tensor-core path use the workspace differently; size for both
size_t pre_fwd_ws_bytes(int64_t T, int32_t N, int64_t D, int32_t dtype) {
  const int HM = hc_mix(N);
  const size_t generic = align_up((size_t)T * HM * 4) + align_up((size_t)T * 4);
  const size_t tc = (N == 4 || N == 8) ? pre_fwd_tc_ws_bytes(T, N, D, dtype) : 0;
  return generic > tc ? generic : tc;
}

template <typename E, int N>
static int pre_fwd_impl(const PreFwdArgs& a, cudaStream_t s) {
  constexpr int HM = hc_mix(N);
  const int64_t T = a.T, D = a.D, HC = (int64_t)N * D;
  char* ws = (char*)a.workspace;
  float* raw = (float*)ws;
  float* sumsq = (float*)(ws + align_up((size_t)T * HM * 4));
  if (T > 0 && a.premix != nullptr) {
    const int st = pre_fwd_finish_premix(a, s);
    if (st != MHC_OK) return st;
  } else if (T > 0 && pre_fwd_tc_eligible(a)) {
    const int st = pre_fwd_tc_mix(a, s);
    if (st != MHC_OK) return st;
  } else if (T > 0) {
    const size_t smem = (size_t)(kMixTT * (kMixKC + 1) + HM * kMixKC) * sizeof(float);
    MHC_CUDA_CHECK(cudaFuncSetAttribute(pre_mix_kernel<E, N>,
                                        cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    launch(pre_mix_kernel<E, N>, (unsigned)cdiv(T, kMixTT), 256, smem, s, 
        (const E*)a.x, a.phi, raw, sumsq, T, HC, a.x_ts);
    MHC_LAUNCH_CHECK();
    launch(pre_small_kernel<N>, (unsigned)cdiv(T, 128), 128, 0, s, 
        raw, sumsq, a.alpha, a.base, T, HC, a.norm_eps, a.sp, a.inv_rms, a.mixes, a.pre,
        a.post_out, a.comb_frag, a.h_res_logits);
    MHC_LAUNCH_CHECK();
  }
  if (T > 0) {
    const bool vec = (D % Pack<E>::n == 0) && rows_aligned(a.x, a.x_ts, sizeof(E), 16) &&
                     aligned16(a.y) &&
                     (a.x_scaled == nullptr || aligned16(a.x_scaled));
    const int64_t want = cdiv(T, 8), cap = (int64_t)sm_count() * 8;
    dim3 grid((unsigned)(want < cap ? want : cap));
    const bool v16 = sizeof(E) == 2 && D % 16 == 0 &&
                     rows_aligned(a.x, a.x_ts, sizeof(E), 32) &&
                     (reinterpret_cast<uintptr_t>(a.y) & 31) == 0 &&
                     (a.x_scaled == nullptr || (reinterpret_cast<uintptr_t>(a.x_scaled) & 31) == 0);
    if constexpr (sizeof(E) == 2) {
      if (v16) {
        launch(pre_apply_x16_kernel<E, N>, grid, 256, 0, s, (const E*)a.x, a.inv_rms, a.pre, (E*)a.y,
                                                        a.x_scaled, T, D, a.x_ts);
        MHC_LAUNCH_CHECK();
        return MHC_OK;
      }
    }
    if (vec)
      launch(pre_apply_kernel<E, N, true>, grid, 256, 0, s, (const E*)a.x, a.inv_rms, a.pre,
                                                        (E*)a.y, a.x_scaled, T, D, a.x_ts);
    else
      launch(pre_apply_kernel<E, N, false>, grid, 256, 0, s, (const E*)a.x, a.inv_rms, a.pre,
                                                         (E*)a.y, a.x_scaled, T, D, a.x_ts);
    MHC_LAUNCH_CHECK();
  }
  return MHC_OK;
}

template <int N>
static int pre_fwd_n(const PreFwdArgs& a, cudaStream_t s) {
  switch (a.dtype) {
    case MHC_F32: return pre_fwd_impl<float, N>(a, s);
    case MHC_F16: return pre_fwd_impl<__half, N>(a, s);
    case MHC_BF16: return pre_fwd_impl<__nv_bfloat16, N>(a, s);
    default: return MHC_ERR_UNSUPPORTED_DTYPE;
  }
}

int pre_fwd_dispatch(const PreFwdArgs& a, cudaStream_t s) { MHC_DISPATCH_N(a.N, pre_fwd_n, a, s); }

}  // namespace mhc

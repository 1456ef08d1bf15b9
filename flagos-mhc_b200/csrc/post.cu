// post.cu -- mhc_post forward and backward: one warp streams one token.
//
// Both kernels are pure HBM streams.  A warp owns a token, loads its N x N
// h_res and N h_post once into registers, then walks D in 16-byte packs
// (8 bf16/fp16 or 4 fp32 per lane per row), so every byte of x / h_out /
// grad_y is read exactly once and every output byte written exactly once.
// Reference kernels replaced: src/mhc_post.py:207-271 (forward, blockT),
// src/mhc_post_backward.py:293-421 (fused backward).
#include "common.cuh"

#include <type_traits>

namespace mhc {

// out[t,i,:] = sum_j h_res[t,j,i] x[t,j,:] + h_post[t,i] h_out[t,:]
template <typename E, int N, bool VEC>
__global__ void __launch_bounds__(256)
post_fwd_kernel(const E* __restrict__ x, const float* __restrict__ h_res,
                const E* __restrict__ h_out, const float* __restrict__ h_post,
                E* __restrict__ out, int64_t T, int64_t D) {
  constexpr int P = VEC ? Pack<E>::n : 1;
  const int lane = threadIdx.x & 31;
  const int64_t nwarps = (int64_t)gridDim.x * (blockDim.x >> 5);
  const int64_t nchunk = D / P;
  for (int64_t t = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); t < T;
       t += nwarps) {
    float hr[N * N], hp[N];
#pragma unroll
    for (int e = 0; e < N * N; ++e) hr[e] = __ldg(h_res + t * N * N + e);
#pragma unroll
    for (int i = 0; i < N; ++i) hp[i] = __ldg(h_post + t * N + i);
    const E* xt = x + t * N * D;
    const E* ht = h_out + t * D;
    E* ot = out + t * N * D;
#pragma unroll 2
    for (int64_t c = lane; c < nchunk; c += 32) {
      float xv[N][P], hv[P];
#pragma unroll
      for (int j = 0; j < N; ++j) load_pack<E, VEC>(xt + j * D + c * P, xv[j]);
      load_pack<E, VEC>(ht + c * P, hv);
#pragma unroll
      for (int i = 0; i < N; ++i) {
        float o[P];
#pragma unroll
        for (int e = 0; e < P; ++e) {
          float s = 0.f;
#pragma unroll
          for (int j = 0; j < N; ++j) s = fmaf(hr[j * N + i], xv[j][e], s);
          o[e] = fmaf(hp[i], hv[e], s);
        }
        store_pack<E, VEC>(ot + i * D + c * P, o);
      }
    }
  }
}

// grad_x[j]   = sum_i h_res[j,i] gy[i]      grad_h_out  = sum_i h_post[i] gy[i]
// grad_hres[j,i] = <x[j], gy[i]>            grad_h_post[i] = <h_out, gy[i]>
template <typename E, int N, bool VEC>
__global__ void __launch_bounds__(256, 2)
post_bwd_kernel(const E* __restrict__ gy, const E* __restrict__ x,
                const float* __restrict__ h_res, const E* __restrict__ h_out,
                const float* __restrict__ h_post, E* __restrict__ gx,
                float* __restrict__ ghres, E* __restrict__ ghout,
                float* __restrict__ ghpost, int64_t T, int64_t D) {
  constexpr int P = VEC ? Pack<E>::n : 1;
  const int lane = threadIdx.x & 31;
  const int64_t nwarps = (int64_t)gridDim.x * (blockDim.x >> 5);
  const int64_t nchunk = D / P;
  for (int64_t t = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); t < T;
       t += nwarps) {
    float hr[N * N], hp[N];
#pragma unroll
    for (int e = 0; e < N * N; ++e) hr[e] = __ldg(h_res + t * N * N + e);
#pragma unroll
    for (int i = 0; i < N; ++i) hp[i] = __ldg(h_post + t * N + i);
    float acc_r[N * N], acc_p[N];
#pragma unroll
    for (int e = 0; e < N * N; ++e) acc_r[e] = 0.f;
#pragma unroll
    for (int i = 0; i < N; ++i) acc_p[i] = 0.f;
    const E* gyt = gy + t * N * D;
    const E* xt = x + t * N * D;
    const E* ht = h_out + t * D;
    E* gxt = gx + t * N * D;
    E* ghot = ghout + t * D;
#pragma unroll 2
    for (int64_t c = lane; c < nchunk; c += 32) {
      float g[N][P], xv[N][P], hv[P];
#pragma unroll
      for (int i = 0; i < N; ++i) load_pack<E, VEC>(gyt + i * D + c * P, g[i]);
#pragma unroll
      for (int j = 0; j < N; ++j) load_pack<E, VEC>(xt + j * D + c * P, xv[j]);
      load_pack<E, VEC>(ht + c * P, hv);
#pragma unroll
      for (int j = 0; j < N; ++j) {
        float o[P];
#pragma unroll
        for (int e = 0; e < P; ++e) {
          float s = 0.f;
#pragma unroll
          for (int i = 0; i < N; ++i) s = fmaf(hr[j * N + i], g[i][e], s);
          o[e] = s;
        }
        store_pack<E, VEC>(gxt + j * D + c * P, o);
      }
      {
        float o[P];
#pragma unroll
        for (int e = 0; e < P; ++e) {
          float s = 0.f;
#pragma unroll
          for (int i = 0; i < N; ++i) s = fmaf(hp[i], g[i][e], s);
          o[e] = s;
        }
        store_pack<E, VEC>(ghot + c * P, o);
      }
#pragma unroll
      for (int e = 0; e < P; ++e) {
#pragma unroll
        for (int i = 0; i < N; ++i) {
          acc_p[i] = fmaf(hv[e], g[i][e], acc_p[i]);
#pragma unroll
          for (int j = 0; j < N; ++j) acc_r[j * N + i] = fmaf(xv[j][e], g[i][e], acc_r[j * N + i]);
        }
      }
    }
#pragma unroll
    for (int e = 0; e < N * N; ++e) acc_r[e] = warp_sum(acc_r[e]);
#pragma unroll
    for (int i = 0; i < N; ++i) acc_p[i] = warp_sum(acc_p[i]);
    // every lane now holds all sums; lane k writes element k
#pragma unroll
    for (int e = 0; e < N * N; ++e)
      if (lane == (e & 31)) ghres[t * N * N + e] = acc_r[e];
#pragma unroll
    for (int i = 0; i < N; ++i)
      if (lane == ((N * N + i) & 31)) ghpost[t * N + i] = acc_p[i];
  }
}

// post forward for 16-bit storage, D % 16 == 0, 32-byte aligned rows: a lane handles 16
// consecutive d of every row with 32-byte loads/stores (half the memory requests of the
// 16-byte path).  (The backward keeps 16-byte packs: with 32-byte packs its operands need
// ~220 registers and the lower occupancy costs more than the wider accesses gain.)
// Operands stay packed in registers and are widened where used.
__device__ __forceinline__ float unpack16(const U8& v, int e) {
  const uint32_t w = (e < 8) ? (&v.a.x)[e >> 1] : (&v.b.x)[(e - 8) >> 1];
  return (e & 1) ? bf16_hi(w) : bf16_lo(w);
}
__device__ __forceinline__ float unpack16h(const U8& v, int e) {
  const uint32_t w = (e < 8) ? (&v.a.x)[e >> 1] : (&v.b.x)[(e - 8) >> 1];
  const __half2 h = *reinterpret_cast<const __half2*>(&w);
  return (e & 1) ? __high2float(h) : __low2float(h);
}
template <typename E>
__device__ __forceinline__ float up16(const U8& v, int e) {
  if constexpr (std::is_same<E, __half>::value) return unpack16h(v, e);
  else return unpack16(v, e);
}
template <typename E>
__device__ __forceinline__ void store16(E* p, const float* o) {
  st_global_32B(p, narrow<E>(o), narrow<E>(o + 8));
}

template <typename E, int N>
__global__ void __launch_bounds__(256, 2)
post_fwd_x16_kernel(const E* __restrict__ x, const float* __restrict__ h_res,
                    const E* __restrict__ h_out, const float* __restrict__ h_post,
                    E* __restrict__ out, int64_t T, int64_t D) {
  const int lane = threadIdx.x & 31;
  const int64_t nwarps = (int64_t)gridDim.x * (blockDim.x >> 5);
  const int64_t nchunk = D / 16;
  for (int64_t t = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); t < T;
       t += nwarps) {
    float hr[N * N], hp[N];
#pragma unroll
    for (int e = 0; e < N * N; ++e) hr[e] = __ldg(h_res + t * N * N + e);
#pragma unroll
    for (int i = 0; i < N; ++i) hp[i] = __ldg(h_post + t * N + i);
    const E* xt = x + t * N * D;
    const E* ht = h_out + t * D;
    E* ot = out + t * N * D;
    for (int64_t c = lane; c < nchunk; c += 32) {
      U8 xv[N];
#pragma unroll
      for (int j = 0; j < N; ++j) xv[j] = ld_global_32B(xt + j * D + c * 16);
      const U8 hv = ld_global_32B(ht + c * 16);
#pragma unroll
      for (int i = 0; i < N; ++i) {
        float o[16];
#pragma unroll
        for (int e = 0; e < 16; ++e) {
          float acc = 0.f;
#pragma unroll
          for (int j = 0; j < N; ++j) acc = fmaf(hr[j * N + i], up16<E>(xv[j], e), acc);
          o[e] = fmaf(hp[i], up16<E>(hv, e), acc);
        }
        store16<E>(ot + i * D + c * 16, o);
      }
    }
  }
}

static inline bool aligned32(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 31) == 0; }

// ---------------------------------------------------------------------------
// Host launchers
// ---------------------------------------------------------------------------
static int post_grid(int64_t T) {
  const int64_t want = cdiv(T, 8);
  const int64_t cap = (int64_t)sm_count() * 8;
  return (int)(want < cap ? want : cap);
}

template <typename E, int N>
static int post_fwd_launch(const void* x, const float* h_res, const void* h_out,
                           const float* h_post, void* out, int64_t T, int64_t D,
                           cudaStream_t s) {
  const bool vec = (D % Pack<E>::n == 0) && aligned16(x) && aligned16(h_out) && aligned16(out);
  dim3 grid(post_grid(T)), block(256);
  if constexpr (sizeof(E) == 2 && N <= 4) {
    if (D % 16 == 0 && aligned32(x) && aligned32(h_out) && aligned32(out)) {
      post_fwd_x16_kernel<E, N><<<grid, block, 0, s>>>((const E*)x, h_res, (const E*)h_out,
                                                      h_post, (E*)out, T, D);
      MHC_LAUNCH_CHECK();
      return MHC_OK;
    }
  }
  if (vec)
    post_fwd_kernel<E, N, true><<<grid, block, 0, s>>>(
        (const E*)x, h_res, (const E*)h_out, h_post, (E*)out, T, D);
  else
    post_fwd_kernel<E, N, false><<<grid, block, 0, s>>>(
        (const E*)x, h_res, (const E*)h_out, h_post, (E*)out, T, D);
  MHC_LAUNCH_CHECK();
  return MHC_OK;
}

template <typename E, int N>
static int post_bwd_launch(const void* gy, const void* x, const float* h_res,
                           const void* h_out, const float* h_post, void* gx, float* ghres,
                           void* ghout, float* ghpost, int64_t T, int64_t D, cudaStream_t s) {
  const bool vec = (D % Pack<E>::n == 0) && aligned16(gy) && aligned16(x) &&
                   aligned16(h_out) && aligned16(gx) && aligned16(ghout);
  dim3 grid(post_grid(T)), block(256);
  if (vec)
    post_bwd_kernel<E, N, true><<<grid, block, 0, s>>>(
        (const E*)gy, (const E*)x, h_res, (const E*)h_out, h_post, (E*)gx, ghres,
        (E*)ghout, ghpost, T, D);
  else
    post_bwd_kernel<E, N, false><<<grid, block, 0, s>>>(
        (const E*)gy, (const E*)x, h_res, (const E*)h_out, h_post, (E*)gx, ghres,
        (E*)ghout, ghpost, T, D);
  MHC_LAUNCH_CHECK();
  return MHC_OK;
}

template <int N>
static int post_fwd_n(int32_t dtype, const void* x, const float* h_res, const void* h_out,
                      const float* h_post, void* out, int64_t T, int64_t D, cudaStream_t s) {
  switch (dtype) {
    case MHC_F32: return post_fwd_launch<float, N>(x, h_res, h_out, h_post, out, T, D, s);
    case MHC_F16: return post_fwd_launch<__half, N>(x, h_res, h_out, h_post, out, T, D, s);
    case MHC_BF16:
      return post_fwd_launch<__nv_bfloat16, N>(x, h_res, h_out, h_post, out, T, D, s);
    default: return MHC_ERR_UNSUPPORTED_DTYPE;
  }
}

template <int N>
static int post_bwd_n(int32_t dtype, const void* gy, const void* x, const float* h_res,
                      const void* h_out, const float* h_post, void* gx, float* ghres,
                      void* ghout, float* ghpost, int64_t T, int64_t D, cudaStream_t s) {
  switch (dtype) {
    case MHC_F32:
      return post_bwd_launch<float, N>(gy, x, h_res, h_out, h_post, gx, ghres, ghout, ghpost,
                                       T, D, s);
    case MHC_F16:
      return post_bwd_launch<__half, N>(gy, x, h_res, h_out, h_post, gx, ghres, ghout, ghpost,
                                        T, D, s);
    case MHC_BF16:
      return post_bwd_launch<__nv_bfloat16, N>(gy, x, h_res, h_out, h_post, gx, ghres, ghout,
                                               ghpost, T, D, s);
    default: return MHC_ERR_UNSUPPORTED_DTYPE;
  }
}

int post_fwd_dispatch(int32_t N, int32_t dtype, const void* x, const float* h_res,
                      const void* h_out, const float* h_post, void* out, int64_t T, int64_t D,
                      cudaStream_t s) {
  MHC_DISPATCH_N(N, post_fwd_n, dtype, x, h_res, h_out, h_post, out, T, D, s);
}

int post_bwd_dispatch(int32_t N, int32_t dtype, const void* gy, const void* x,
                      const float* h_res, const void* h_out, const float* h_post, void* gx,
                      float* ghres, void* ghout, float* ghpost, int64_t T, int64_t D,
                      cudaStream_t s) {
  MHC_DISPATCH_N(N, post_bwd_n, dtype, gy, x, h_res, h_out, h_post, gx, ghres, ghout, ghpost,
                 T, D, s);
}

}  // namespace mhc

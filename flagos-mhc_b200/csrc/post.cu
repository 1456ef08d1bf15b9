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
                E* __restrict__ out, int64_t T, int64_t D, TokStride st) {
  pdl_enter();
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
    const E* xt = x + t * st.x;
    const E* ht = h_out + t * st.ho;
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
                float* __restrict__ ghpost, int64_t T, int64_t D, TokStride st) {
  pdl_enter();
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
    const E* gyt = gy + t * st.gy;
    const E* xt = x + t * st.x;
    const E* ht = h_out + t * st.ho;
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

// SPLIT (small T): a block takes one token, warp w a contiguous range of its D steps.
template <typename E, int N, bool SPLIT>
__global__ void __launch_bounds__(256, 2)
post_fwd_x16_kernel(const E* __restrict__ x, const float* __restrict__ h_res,
                    const E* __restrict__ h_out, const float* __restrict__ h_post,
                    E* __restrict__ out, int64_t T, int64_t D, TokStride st) {
  pdl_enter();
  const int lane = threadIdx.x & 31;
  const int nw = blockDim.x >> 5, w = threadIdx.x >> 5;
  const int64_t nchunk = D / 16;
  const int64_t nst = (nchunk + 31) / 32;
  const int64_t clo = SPLIT ? nst * w / nw * 32 : 0;
  const int64_t chi_ = SPLIT ? nst * (w + 1) / nw * 32 : nchunk;
  const int64_t chi = chi_ < nchunk ? chi_ : nchunk;
  const int64_t tstride = SPLIT ? gridDim.x : (int64_t)gridDim.x * nw;
  for (int64_t t = SPLIT ? blockIdx.x : (int64_t)blockIdx.x * nw + w; t < T; t += tstride) {
    float hr[N * N], hp[N];
#pragma unroll
    for (int e = 0; e < N * N; ++e) hr[e] = __ldg(h_res + t * N * N + e);
#pragma unroll
    for (int i = 0; i < N; ++i) hp[i] = __ldg(h_post + t * N + i);
    const E* xt = x + t * st.x;
    const E* ht = h_out + t * st.ho;
    E* ot = out + t * N * D;
    for (int64_t c = clo + lane; c < chi; c += 32) {
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
// N = 8, 16-bit storage, D % 32 == 0: one warp per token, lane (g, c) = (lane/4, lane%4)
// owns row g at the 8 consecutive d of chunk c of every 32-wide step, so every load and
// store is a 16-byte pack.  The per-token 8x8 products run on mma.sync m16n8k16 (fp32
// accumulate); the fp32 h_res / h_post enter as bf16 (or fp16) hi + lo halves, which
// reproduces the fp32 products to ~2^-17.  A generic N=8 lane would need 64 h_res and 64
// accumulators in registers.
//   grad_h_res[j,i] = <x[j], gy[i]>, grad_h_post[i] = <h_out, gy[i]>:  A = [x rows; h_out]
//     (16 x 16 d), B = gy rows (16 d x 8), both straight from the lane's registers (the
//     k slots of a lane map to its own d, identically for A and B).
//   grad_x[j,d] = sum_i h_res[j,i] gy[i,d], grad_h_out[d] = sum_i h_post[i] gy[i,d]:
//     A = [h_res_hi | h_res_lo ; h_post_hi | h_post_lo] (rows j, then row 8), B = gy
//     transposed by movmatrix (one per register r), which makes the result land back in
//     the lane's own row / d layout.
//   out[i,d] = sum_j h_res[j,i] x[j,d] + h_post[i] h_out[d]: the same with A = h_res^T
//     and B = x transposed, plus the h_post term in fp32.
template <typename E>
__device__ __forceinline__ uint32_t pack_e2(float a, float b) {
  if constexpr (std::is_same<E, __half>::value) {
    const __half2 h = __floats2half2_rn(a, b);
    return *reinterpret_cast<const uint32_t*>(&h);
  } else {
    const __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
    return *reinterpret_cast<const uint32_t*>(&h);
  }
}
template <typename E>
__device__ __forceinline__ float round_e(float v) {
  if constexpr (std::is_same<E, __half>::value) return __half2float(__float2half_rn(v));
  else return __bfloat162float(__float2bfloat16_rn(v));
}
// hi / lo halves of two fp32 values, packed as (lo index in the low 16 bits)
template <typename E>
__device__ __forceinline__ void split_e2(float a, float b, uint32_t& hi, uint32_t& lo) {
  const float ah = round_e<E>(a), bh = round_e<E>(b);
  hi = pack_e2<E>(ah, bh);
  lo = pack_e2<E>(a - ah, b - bh);
}
template <typename E>
__device__ __forceinline__ void mma16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0,
                                         uint32_t b1, float c0, float c1, float c2, float c3) {
  if constexpr (std::is_same<E, __half>::value)
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
        "{%8,%9}, {%10,%11,%12,%13};"
        : "=f"(d[0]), "=f"(d[1]), "=f"(d[2]), "=f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1), "f"(c0), "f"(c1),
          "f"(c2), "f"(c3));
  else
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
        "{%8,%9}, {%10,%11,%12,%13};"
        : "=f"(d[0]), "=f"(d[1]), "=f"(d[2]), "=f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1), "f"(c0), "f"(c1),
          "f"(c2), "f"(c3));
}
// transpose of the warp's 8x8 16-bit matrix held one 32-bit register per lane
__device__ __forceinline__ uint32_t movtrans(uint32_t a) {
  uint32_t d;
  asm volatile("movmatrix.sync.aligned.m8n8.trans.b16 %0, %1;" : "=r"(d) : "r"(a));
  return d;
}
template <typename E>
__device__ __forceinline__ void widen2(uint32_t w, float* f) {
  if constexpr (std::is_same<E, __half>::value) {
    const __half2 h = *reinterpret_cast<const __half2*>(&w);
    f[0] = __low2float(h);
    f[1] = __high2float(h);
  } else {
    f[0] = bf16_lo(w);
    f[1] = bf16_hi(w);
  }
}

// V 16-byte packs per lane and row per step (V = 2: 32-byte accesses, 64-wide steps)
template <int V>
__device__ __forceinline__ void ld_row_packs(const void* p, uint32_t (&r)[4 * V]) {
  if constexpr (V >= 2) {
#pragma unroll
    for (int h = 0; h < V / 2; ++h) {
      const U8 v = ld_global_32B((const char*)p + 32 * h);
      r[8 * h + 0] = v.a.x; r[8 * h + 1] = v.a.y; r[8 * h + 2] = v.a.z; r[8 * h + 3] = v.a.w;
      r[8 * h + 4] = v.b.x; r[8 * h + 5] = v.b.y; r[8 * h + 6] = v.b.z; r[8 * h + 7] = v.b.w;
    }
  } else {
    const uint4 v = ld_stream(p);
    r[0] = v.x; r[1] = v.y; r[2] = v.z; r[3] = v.w;
  }
}
template <typename E, int V>
__device__ __forceinline__ void st_row_packs(void* p, const float* o) {
  if constexpr (V >= 2) {
#pragma unroll
    for (int h = 0; h < V / 2; ++h)
      st_global_32B((char*)p + 32 * h, narrow<E>(o + 16 * h), narrow<E>(o + 16 * h + 8));
  } else {
    st_stream(p, narrow<E>(o));
  }
}

template <typename E, int V>
__global__ void __launch_bounds__(256)
post_fwd_n8_kernel(const E* __restrict__ x, const float* __restrict__ h_res,
                   const E* __restrict__ h_out, const float* __restrict__ h_post,
                   E* __restrict__ out, int64_t T, int64_t D, TokStride st) {
  pdl_enter();
  constexpr int N = 8, R = 4 * V;
  const int lane = threadIdx.x & 31, g = lane >> 2, c = lane & 3;
  const int64_t nwarps = (int64_t)gridDim.x * (blockDim.x >> 5);
  for (int64_t t = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); t < T;
       t += nwarps) {
    // A = [h_res^T hi | h_res^T lo] rows i = g: (h_res[2c][g], h_res[2c+1][g])
    const float* hr = h_res + t * N * N;
    uint32_t a[4];
    split_e2<E>(__ldg(hr + (2 * c) * N + g), __ldg(hr + (2 * c + 1) * N + g), a[0], a[2]);
    a[1] = a[3] = 0u;
    const float hp = __ldg(h_post + t * N + g);
    const E* xr = x + t * st.x + g * D;
    const E* ht = h_out + t * st.ho;
    E* orow = out + (t * N + g) * D;
#pragma unroll 2
    for (int64_t d0 = 8 * V * c; d0 < D; d0 += 32 * V) {
      uint32_t xv[R], hv[R];
      ld_row_packs<V>(xr + d0, xv);
      ld_row_packs<V>(ht + d0, hv);
      float o[2 * R];
#pragma unroll
      for (int r = 0; r < R; ++r) {
        const uint32_t b = movtrans(xv[r]);
        float cc[4];
        mma16816<E>(cc, a, b, b, 0.f, 0.f, 0.f, 0.f);
        float h2[2];
        widen2<E>(hv[r], h2);
        o[2 * r] = fmaf(hp, h2[0], cc[0]);
        o[2 * r + 1] = fmaf(hp, h2[1], cc[1]);
      }
      st_row_packs<E, V>(orow + d0, o);
    }
  }
}

template <typename E, int V>
__global__ void __launch_bounds__(256)
post_bwd_n8_kernel(const E* __restrict__ gy, const E* __restrict__ x,
                   const float* __restrict__ h_res, const E* __restrict__ h_out,
                   const float* __restrict__ h_post, E* __restrict__ gx,
                   float* __restrict__ ghres, E* __restrict__ ghout,
                   float* __restrict__ ghpost, int64_t T, int64_t D, TokStride st) {
  pdl_enter();
  constexpr int N = 8, R = 4 * V;
  const int lane = threadIdx.x & 31, g = lane >> 2, c = lane & 3;
  const int64_t nwarps = (int64_t)gridDim.x * (blockDim.x >> 5);
  for (int64_t t = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); t < T;
       t += nwarps) {
    // A of grad_x: rows j = g: (h_res[g][2c], h_res[g][2c+1]) hi | lo; row 8: h_post
    const float* hr = h_res + t * N * N;
    uint32_t a[4];
    split_e2<E>(__ldg(hr + g * N + 2 * c), __ldg(hr + g * N + 2 * c + 1), a[0], a[2]);
    if (g == 0) {
      split_e2<E>(__ldg(h_post + t * N + 2 * c), __ldg(h_post + t * N + 2 * c + 1), a[1], a[3]);
    } else {
      a[1] = a[3] = 0u;
    }
    float acc[4] = {0.f, 0.f, 0.f, 0.f};
    const E* xr = x + t * st.x + g * D;
    const E* gyr = gy + t * st.gy + g * D;
    const E* ht = h_out + t * st.ho;
    E* gxr = gx + (t * N + g) * D;
    E* ght = ghout + t * D;
#pragma unroll 2
    for (int64_t d0 = 8 * V * c; d0 < D; d0 += 32 * V) {
      uint32_t xv[R], gv[R], hv[R];
      ld_row_packs<V>(xr + d0, xv);
      ld_row_packs<V>(gyr + d0, gv);
#pragma unroll
      for (int r = 0; r < R; ++r) hv[r] = 0u;
      if (g == 0) ld_row_packs<V>(ht + d0, hv);
      // <x[j], gy[i]> and <h_out, gy[i]>: k-16 slices of this step (4 d per lane each)
      float dd[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
      for (int sl = 0; sl < R / 2; ++sl) {
        const uint32_t as[4] = {xv[2 * sl], hv[2 * sl], xv[2 * sl + 1], hv[2 * sl + 1]};
        mma16816<E>(dd, as, gv[2 * sl], gv[2 * sl + 1], dd[0], dd[1], dd[2], dd[3]);
      }
#pragma unroll
      for (int u = 0; u < 4; ++u) acc[u] += dd[u];
      float o[2 * R], oh[2 * R];
#pragma unroll
      for (int r = 0; r < R; ++r) {
        const uint32_t b = movtrans(gv[r]);
        float cc[4];
        mma16816<E>(cc, a, b, b, 0.f, 0.f, 0.f, 0.f);
        o[2 * r] = cc[0];
        o[2 * r + 1] = cc[1];
        oh[2 * r] = cc[2];
        oh[2 * r + 1] = cc[3];
      }
      st_row_packs<E, V>(gxr + d0, o);
      if (g == 0) st_row_packs<E, V>(ght + d0, oh);
    }
    ghres[t * N * N + g * N + 2 * c] = acc[0];
    ghres[t * N * N + g * N + 2 * c + 1] = acc[1];
    if (g == 0) {
      ghpost[t * N + 2 * c] = acc[2];
      ghpost[t * N + 2 * c + 1] = acc[3];
    }
  }
}

// N = 4, 16-bit storage: the N=8 scheme with two tokens per warp.  Lane (g, c) owns row
// g & 3 of token 2p + g/4; the mma rows 0-3 / 4-7 are the two tokens' rows, rows 8 and 12
// their h_out (grad_h_post) or h_post (grad_h_out).  grad_x takes a block-diagonal A
// (each token's h_res hi | lo against its own grad_y rows); the dot products of rows of
// different tokens come out of the same MMAs and are dropped.
// SPLIT (small T): a block of warps takes one token pair, warp w a contiguous range of
// the D steps; the dot-product partials are added across the warps in a fixed order.
template <typename E, int V, bool SPLIT>
__global__ void __launch_bounds__(256)
post_bwd_n4x2_kernel(const E* __restrict__ gy, const E* __restrict__ x,
                     const float* __restrict__ h_res, const E* __restrict__ h_out,
                     const float* __restrict__ h_post, E* __restrict__ gx,
                     float* __restrict__ ghres, E* __restrict__ ghout,
                     float* __restrict__ ghpost, int64_t T, int64_t D, TokStride st) {
  pdl_enter();
  constexpr int N = 4, R = 4 * V;
  const int lane = threadIdx.x & 31, g = lane >> 2, c = lane & 3;
  const int tb = g >> 2, j = g & 3;            // token of the pair, row of the token
  const bool mine = (c >> 1) == tb;            // mma columns 2c, 2c+1 belong to this token
  const bool hrow = j == 0;                    // lanes holding row 8 / 12 (h_out, h_post)
  const int i0 = (2 * c) & 3;                  // those columns' index within the token
  const int64_t npairs = (T + 1) / 2;
  const int nw = blockDim.x >> 5, w = threadIdx.x >> 5;
  const int64_t nsteps = D / (32 * V);
  const int64_t dlo = SPLIT ? nsteps * w / nw * (32 * V) : 0;
  const int64_t dhi = SPLIT ? nsteps * (w + 1) / nw * (32 * V) : D;
  __shared__ float red[SPLIT ? 8 : 1][32][4];
  const int64_t pstride = SPLIT ? gridDim.x : (int64_t)gridDim.x * nw;
  for (int64_t p = SPLIT ? blockIdx.x : (int64_t)blockIdx.x * nw + w; p < npairs;
       p += pstride) {
    const int64_t t = 2 * p + tb;
    const bool live = t < T;
    uint32_t a[4] = {0u, 0u, 0u, 0u};
    if (live && mine) {
      const float* hr = h_res + t * N * N + j * N + i0;
      split_e2<E>(__ldg(hr), __ldg(hr + 1), a[0], a[2]);
      if (hrow) split_e2<E>(__ldg(h_post + t * N + i0), __ldg(h_post + t * N + i0 + 1), a[1], a[3]);
    }
    float acc[4] = {0.f, 0.f, 0.f, 0.f};
    const int64_t row = live ? (t * N + j) * D : 0;
    const E* xr = x + (live ? t * st.x + j * D : 0);
    const E* gyr = gy + (live ? t * st.gy + j * D : 0);
    const E* ht = h_out + (live ? t * st.ho : 0);
    E* gxr = gx + row;
    E* ght = ghout + (live ? t * D : 0);
#pragma unroll 2
    for (int64_t d0 = dlo + 8 * V * c; d0 < dhi; d0 += 32 * V) {
      uint32_t xv[R], gv[R], hv[R];
#pragma unroll
      for (int r = 0; r < R; ++r) xv[r] = gv[r] = hv[r] = 0u;
      if (live) {
        ld_row_packs<V>(xr + d0, xv);
        ld_row_packs<V>(gyr + d0, gv);
        if (hrow) ld_row_packs<V>(ht + d0, hv);
      }
      float dd[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
      for (int sl = 0; sl < R / 2; ++sl) {
        const uint32_t as[4] = {xv[2 * sl], hv[2 * sl], xv[2 * sl + 1], hv[2 * sl + 1]};
        mma16816<E>(dd, as, gv[2 * sl], gv[2 * sl + 1], dd[0], dd[1], dd[2], dd[3]);
      }
#pragma unroll
      for (int u = 0; u < 4; ++u) acc[u] += dd[u];
      float o[2 * R], oh[2 * R];
#pragma unroll
      for (int r = 0; r < R; ++r) {
        const uint32_t b = movtrans(gv[r]);
        float cc[4];
        mma16816<E>(cc, a, b, b, 0.f, 0.f, 0.f, 0.f);
        o[2 * r] = cc[0];
        o[2 * r + 1] = cc[1];
        oh[2 * r] = cc[2];
        oh[2 * r + 1] = cc[3];
      }
      if (live) {
        st_row_packs<E, V>(gxr + d0, o);
        if (hrow) st_row_packs<E, V>(ght + d0, oh);
      }
    }
    if constexpr (SPLIT) {
#pragma unroll
      for (int u = 0; u < 4; ++u) red[w][lane][u] = acc[u];
      __syncthreads();
      if (w == 0) {
        for (int ww = 1; ww < nw; ++ww)
#pragma unroll
          for (int u = 0; u < 4; ++u) acc[u] += red[ww][lane][u];
      }
      __syncthreads();
      if (w != 0) continue;
    }
    if (live && mine) {
      ghres[t * N * N + j * N + i0] = acc[0];
      ghres[t * N * N + j * N + i0 + 1] = acc[1];
      if (hrow) {
        ghpost[t * N + i0] = acc[2];
        ghpost[t * N + i0 + 1] = acc[3];
      }
    }
  }
}

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
                           TokStride st, cudaStream_t s) {
  // a strided input counts as aligned to A bytes when every token's row start is
  const auto al = [](const void* p, int64_t ts, uintptr_t A) {
    return (reinterpret_cast<uintptr_t>(p) % A) == 0 && ((uint64_t)ts * sizeof(E)) % A == 0;
  };
  const bool vec = (D % Pack<E>::n == 0) && al(x, st.x, 16) && al(h_out, st.ho, 16) && aligned16(out);
  dim3 grid(post_grid(T)), block(256);
  if constexpr (sizeof(E) == 2 && N == 8) {
    if (D % 128 == 0 && al(x, st.x, 32) && al(h_out, st.ho, 32) && aligned32(out)) {
      launch(post_fwd_n8_kernel<E, 4>, grid, block, 0, s, (const E*)x, h_res, (const E*)h_out,
                                                      h_post, (E*)out, T, D, st);
      MHC_LAUNCH_CHECK();
      return MHC_OK;
    }
    if (D % 64 == 0 && al(x, st.x, 32) && al(h_out, st.ho, 32) && aligned32(out)) {
      launch(post_fwd_n8_kernel<E, 2>, grid, block, 0, s, (const E*)x, h_res, (const E*)h_out,
                                                      h_post, (E*)out, T, D, st);
      MHC_LAUNCH_CHECK();
      return MHC_OK;
    }
    if (D % 32 == 0 && vec) {
      launch(post_fwd_n8_kernel<E, 1>, grid, block, 0, s, (const E*)x, h_res, (const E*)h_out,
                                                      h_post, (E*)out, T, D, st);
      MHC_LAUNCH_CHECK();
      return MHC_OK;
    }
  }
  if constexpr (sizeof(E) == 2 && N <= 4) {
    if (D % 16 == 0 && al(x, st.x, 32) && al(h_out, st.ho, 32) && aligned32(out)) {
      if (T < (int64_t)sm_count() * 8)  // small T (fewer than 8 tokens per SM): a block per token
        launch(post_fwd_x16_kernel<E, N, true>, (unsigned)T, block, 0, s, 
            (const E*)x, h_res, (const E*)h_out, h_post, (E*)out, T, D, st);
      else
        launch(post_fwd_x16_kernel<E, N, false>, grid, block, 0, s, 
            (const E*)x, h_res, (const E*)h_out, h_post, (E*)out, T, D, st);
      MHC_LAUNCH_CHECK();
      return MHC_OK;
    }
  }
  if (vec)
    launch(post_fwd_kernel<E, N, true>, grid, block, 0, s, 
        (const E*)x, h_res, (const E*)h_out, h_post, (E*)out, T, D, st);
  else
    launch(post_fwd_kernel<E, N, false>, grid, block, 0, s, 
        (const E*)x, h_res, (const E*)h_out, h_post, (E*)out, T, D, st);
  MHC_LAUNCH_CHECK();
  return MHC_OK;
}

template <typename E, int N>
static int post_bwd_launch(const void* gy, const void* x, const float* h_res,
                           const void* h_out, const float* h_post, void* gx, float* ghres,
                           void* ghout, float* ghpost, int64_t T, int64_t D, TokStride st,
                           cudaStream_t s) {
  const auto al = [](const void* p, int64_t ts, uintptr_t A) {
    return (reinterpret_cast<uintptr_t>(p) % A) == 0 && ((uint64_t)ts * sizeof(E)) % A == 0;
  };
  const bool vec = (D % Pack<E>::n == 0) && al(gy, st.gy, 16) && al(x, st.x, 16) &&
                   al(h_out, st.ho, 16) && aligned16(gx) && aligned16(ghout);
  dim3 grid(post_grid(T)), block(256);
  if constexpr (sizeof(E) == 2 && N == 4) {
    const bool a32 = al(gy, st.gy, 32) && al(x, st.x, 32) && al(h_out, st.ho, 32) && aligned32(gx) &&
                     aligned32(ghout);
    const int64_t npairs = (T + 1) / 2;
    dim3 pgrid(post_grid(npairs));
    // small T (fewer pairs than 8 per SM): a block per pair, its warps split D
    const bool split = npairs < (int64_t)sm_count() * 8;
    dim3 sgrid((unsigned)npairs);
#define MHC_N4X2(VV)                                                                        \
  do {                                                                                      \
    if (split)                                                                              \
      launch(post_bwd_n4x2_kernel<E, VV, true>, sgrid, block, 0, s,                             \
          (const E*)gy, (const E*)x, h_res, (const E*)h_out, h_post, (E*)gx, ghres,         \
          (E*)ghout, ghpost, T, D, st);                                                         \
    else                                                                                    \
      launch(post_bwd_n4x2_kernel<E, VV, false>, pgrid, block, 0, s,                            \
          (const E*)gy, (const E*)x, h_res, (const E*)h_out, h_post, (E*)gx, ghres,         \
          (E*)ghout, ghpost, T, D, st);                                                         \
    MHC_LAUNCH_CHECK();                                                                     \
    return MHC_OK;                                                                          \
  } while (0)
    if (D % 128 == 0 && a32) MHC_N4X2(4);
    if (D % 64 == 0 && a32) MHC_N4X2(2);
#undef MHC_N4X2
  }
  if constexpr (sizeof(E) == 2 && N == 8) {
    if (D % 128 == 0 && al(gy, st.gy, 32) && al(x, st.x, 32) && al(h_out, st.ho, 32) && aligned32(gx) &&
        aligned32(ghout)) {
      launch(post_bwd_n8_kernel<E, 4>, grid, block, 0, s, (const E*)gy, (const E*)x, h_res,
                                                      (const E*)h_out, h_post, (E*)gx, ghres,
                                                      (E*)ghout, ghpost, T, D, st);
      MHC_LAUNCH_CHECK();
      return MHC_OK;
    }
    if (D % 64 == 0 && al(gy, st.gy, 32) && al(x, st.x, 32) && al(h_out, st.ho, 32) && aligned32(gx) &&
        aligned32(ghout)) {
      launch(post_bwd_n8_kernel<E, 2>, grid, block, 0, s, (const E*)gy, (const E*)x, h_res,
                                                      (const E*)h_out, h_post, (E*)gx, ghres,
                                                      (E*)ghout, ghpost, T, D, st);
      MHC_LAUNCH_CHECK();
      return MHC_OK;
    }
    if (D % 32 == 0 && vec) {
      launch(post_bwd_n8_kernel<E, 1>, grid, block, 0, s, (const E*)gy, (const E*)x, h_res,
                                                      (const E*)h_out, h_post, (E*)gx, ghres,
                                                      (E*)ghout, ghpost, T, D, st);
      MHC_LAUNCH_CHECK();
      return MHC_OK;
    }
  }
  if (vec)
    launch(post_bwd_kernel<E, N, true>, grid, block, 0, s, 
        (const E*)gy, (const E*)x, h_res, (const E*)h_out, h_post, (E*)gx, ghres,
        (E*)ghout, ghpost, T, D, st);
  else
    launch(post_bwd_kernel<E, N, false>, grid, block, 0, s, 
        (const E*)gy, (const E*)x, h_res, (const E*)h_out, h_post, (E*)gx, ghres,
        (E*)ghout, ghpost, T, D, st);
  MHC_LAUNCH_CHECK();
  return MHC_OK;
}

template <int N>
static int post_fwd_n(int32_t dtype, const void* x, const float* h_res, const void* h_out,
                      const float* h_post, void* out, int64_t T, int64_t D, TokStride st,
                      cudaStream_t s) {
  switch (dtype) {
    case MHC_F32: return post_fwd_launch<float, N>(x, h_res, h_out, h_post, out, T, D, st, s);
    case MHC_F16: return post_fwd_launch<__half, N>(x, h_res, h_out, h_post, out, T, D, st, s);
    case MHC_BF16:
      return post_fwd_launch<__nv_bfloat16, N>(x, h_res, h_out, h_post, out, T, D, st, s);
    default: return MHC_ERR_UNSUPPORTED_DTYPE;
  }
}

template <int N>
static int post_bwd_n(int32_t dtype, const void* gy, const void* x, const float* h_res,
                      const void* h_out, const float* h_post, void* gx, float* ghres,
                      void* ghout, float* ghpost, int64_t T, int64_t D, TokStride st,
                      cudaStream_t s) {
  switch (dtype) {
    case MHC_F32:
      return post_bwd_launch<float, N>(gy, x, h_res, h_out, h_post, gx, ghres, ghout, ghpost,
                                       T, D, st, s);
    case MHC_F16:
      return post_bwd_launch<__half, N>(gy, x, h_res, h_out, h_post, gx, ghres, ghout, ghpost,
                                        T, D, st, s);
    case MHC_BF16:
      return post_bwd_launch<__nv_bfloat16, N>(gy, x, h_res, h_out, h_post, gx, ghres, ghout,
                                               ghpost, T, D, st, s);
    default: return MHC_ERR_UNSUPPORTED_DTYPE;
  }
}

int post_fwd_dispatch(int32_t N, int32_t dtype, const void* x, const float* h_res,
                      const void* h_out, const float* h_post, void* out, int64_t T, int64_t D,
                      TokStride st, cudaStream_t s) {
  MHC_DISPATCH_N(N, post_fwd_n, dtype, x, h_res, h_out, h_post, out, T, D, st, s);
}

int post_bwd_dispatch(int32_t N, int32_t dtype, const void* gy, const void* x,
                      const float* h_res, const void* h_out, const float* h_post, void* gx,
                      float* ghres, void* ghout, float* ghpost, int64_t T, int64_t D,
                      TokStride st, cudaStream_t s) {
  MHC_DISPATCH_N(N, post_bwd_n, dtype, gy, x, h_res, h_out, h_post, gx, ghres, ghout, ghpost,
                 T, D, st, s);
}

}  // namespace mhc

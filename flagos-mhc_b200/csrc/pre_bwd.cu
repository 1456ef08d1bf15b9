// pre_bwd.cu -- mhc_pre_clamp_sinkhorn backward, generic path (any dtype, N 1..8).
//
// Stream-ordered kernels:
//   1. pre_bwd_dots_kernel    grad_pre[t,n] = <grad_y[t,:], x[t,n,:]>      (warp / token)
//   2. pre_small_bwd_kernel   small-stage VJP -> grad_mixes[t,:], the RMS coefficient
//                             coef[t] = inv^2/HC * <grad_mixes, mixes>, and per-block
//                             partial sums of grad_alpha / grad_base       (thread / token)
//   3. pre_reduce_ab_kernel   fixed-order sum of those partials
//   4. pre_bwd_gx_kernel      grad_x = gy*pre[n] + inv*(grad_mixes.phi) - coef*x
//   5. pre_bwd_gphi_kernel    split-T partials of grad_phi = (inv*grad_mixes)^T x
//   6. pre_reduce_gphi_kernel fixed-order sum of the split-T partials
// Reference replaced: src/mhc_pre_clamp_sinkhorn_backward.py:1292-1391 (y_bwd, small
// stage, two torch.mm, fused rms-bwd); VJP order of :1144-1209.
//
// Two identities remove the reference's x_scaled traffic:
//   <x, gxs>  = sum_k grad_mixes[k] * mixes[k] / inv       (mixes = inv * x.phi^T)
//   grad_phi  = (inv * grad_mixes)^T x                      (x_scaled = inv * x)
#include "common.cuh"
#include "pre_common.cuh"

#include <type_traits>

namespace mhc {

// Arguments of the comb-VJP blocks that ride along with pre_bwd_dots_kernel (N = 4): 16
// tokens per 256-thread block write d = dL/dlogit to dlog [T][16].
struct VjpArgs {
  const float* mixes;
  const float* alpha;
  const float* base;
  const float* gcomb;
  float* hist;
  float* dlog;
  unsigned* ticket;  // zeroed here for the element-parallel kernel's last-block sum
  SmallParams sp;
  int nblk;  // blocks of this role (0: none)
};

__device__ __forceinline__ float comb_vjp_elem(float ml, float base_l, const SmallParams& sp,
                                               float gcomb_e, float* __restrict__ hist,
                                               int64_t T, int64_t t, int64_t tc, bool valid,
                                               int e, int gl0);

// SPLIT (small T): a block takes one token, warp w a contiguous range of its chunks; the
// warps' sums are added in a fixed order.
template <typename E, int N, bool VEC, bool SPLIT>
__global__ void __launch_bounds__(256)
pre_bwd_dots_kernel(const E* __restrict__ x, const E* __restrict__ gy,
                    float* __restrict__ gpre, int64_t T, int64_t D, int64_t xs, int64_t gys,
                    int ndots, const float* __restrict__ phi, E* __restrict__ p0,
                    E* __restrict__ p1, int nphi, VjpArgs va) {
  pdl_enter();
  if (va.nblk > 0 && blockIdx.x == 0 && threadIdx.x == 0) *va.ticket = 0u;
  // blocks after the grad_pre and phi-operand blocks: the comb part of the small-stage
  // VJP, which needs no grad_pre and so overlaps this streaming pass
  if ((int)blockIdx.x >= ndots + nphi) {
    if constexpr (N == 4) {
      const int lane = threadIdx.x & 31, e = lane & 15, gl0 = lane & 16;
      const int64_t t = (int64_t)(blockIdx.x - ndots - nphi) * (blockDim.x / 16) +
                        threadIdx.x / 16;
      const bool valid = t < T;
      const int64_t tc = valid ? t : T - 1;
      SmallParams sp = va.sp;
      sp.a0 = va.alpha[0]; sp.a1 = va.alpha[1]; sp.a2 = va.alpha[2];
      const float ml = va.mixes[tc * 24 + 8 + e];
      const float d = comb_vjp_elem(ml, __ldg(va.base + 8 + e), sp, va.gcomb[tc * 16 + e],
                                    va.hist, T, t, tc, valid, e, gl0);
      if (valid) va.dlog[t * 16 + e] = d;
    }
    return;
  }
  // blocks beyond the first ndots write the tensor-core pass's phi operand rows (they
  // depend only on phi, and ride along with this streaming kernel instead of a launch
  // of their own)
  if ((int)blockIdx.x >= ndots) {
    if constexpr (sizeof(E) == 2)
      bwd_phi_prep_item<E>(phi, p0, p1, (int64_t)N * D, 1.f,
                           (int64_t)(blockIdx.x - ndots) * blockDim.x + threadIdx.x);
    return;
  }
  constexpr int P = VEC ? Pack<E>::n : 1;
  const int lane = threadIdx.x & 31;
  const int nw = blockDim.x >> 5, w = threadIdx.x >> 5;
  const int64_t nchunk = D / P;
  const int64_t nst = (nchunk + 31) / 32;
  const int64_t clo = SPLIT ? nst * w / nw * 32 : 0;
  const int64_t chi_ = SPLIT ? nst * (w + 1) / nw * 32 : nchunk;
  const int64_t chi = chi_ < nchunk ? chi_ : nchunk;
  __shared__ double red[SPLIT ? 8 : 1][N];
  const int64_t tstride = SPLIT ? ndots : (int64_t)ndots * nw;
  for (int64_t t = SPLIT ? blockIdx.x : (int64_t)blockIdx.x * nw + w; t < T; t += tstride) {
    // <gy, x[n]> cancels heavily (its terms have random signs), so each pack's fp32 sum
    // is added into an fp64 accumulator: the rounding of the long chain no longer
    // dominates the result's relative error (one fp64 add per pack)
    double acc[N];
#pragma unroll
    for (int n = 0; n < N; ++n) acc[n] = 0.0;
    const E* xt = x + t * xs;
    const E* gt = gy + t * gys;
    for (int64_t c = clo + lane; c < chi; c += 32) {
      float g[P], xv[N][P];
      load_pack<E, VEC>(gt + c * P, g);
#pragma unroll
      for (int n = 0; n < N; ++n) load_pack<E, VEC>(xt + n * D + c * P, xv[n]);
#pragma unroll
      for (int n = 0; n < N; ++n) {
        float part = 0.f;
#pragma unroll
        for (int e = 0; e < P; ++e) part = fmaf(g[e], xv[n][e], part);
        acc[n] += (double)part;
      }
    }
#pragma unroll
    for (int n = 0; n < N; ++n)
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) acc[n] += __shfl_xor_sync(0xffffffffu, acc[n], o);
    if constexpr (SPLIT) {
      if (lane == 0)
#pragma unroll
        for (int n = 0; n < N; ++n) red[w][n] = acc[n];
      __syncthreads();
      if (w == 0)
#pragma unroll
        for (int n = 0; n < N; ++n) {
          acc[n] = 0.0;
          for (int ww = 0; ww < nw; ++ww) acc[n] += red[ww][n];
        }
      __syncthreads();
      if (w != 0) continue;
    }
#pragma unroll
    for (int n = 0; n < N; ++n)
      if (lane == n) gpre[t * N + n] = (float)acc[n];
  }
}

// bf16 hi/lo operand rows of one token for the tensor-core main pass (N = 4):
//   G' = [g_hi | g_lo | g_hi | 0] (K = 80: g0 holds 0..63, g1 holds 64..79)
//   Gp = [(inv g)_hi | (inv g)_lo | 0] (64)
__device__ __forceinline__ void write_tc_operand_rows(const float* g, float inv, int64_t t,
                                                      __nv_bfloat16* g0, __nv_bfloat16* g1,
                                                      __nv_bfloat16* gp) {
  constexpr int HM = 24;
  __nv_bfloat16 row[80], prow[64];
#pragma unroll
  for (int k = 0; k < HM; ++k) {
    const __nv_bfloat16 hi = __float2bfloat16_rn(g[k]);
    const __nv_bfloat16 lo = __float2bfloat16_rn(g[k] - __bfloat162float(hi));
    row[k] = hi;
    row[HM + k] = lo;
    row[2 * HM + k] = hi;
    const float p = g[k] * inv;
    const __nv_bfloat16 phi_ = __float2bfloat16_rn(p);
    prow[k] = phi_;
    prow[HM + k] = __float2bfloat16_rn(p - __bfloat162float(phi_));
  }
#pragma unroll
  for (int k = 3 * HM; k < 80; ++k) row[k] = __float2bfloat16_rn(0.f);
#pragma unroll
  for (int k = 2 * HM; k < 64; ++k) prow[k] = __float2bfloat16_rn(0.f);
  const uint4* rv = reinterpret_cast<const uint4*>(row);
  const uint4* pv = reinterpret_cast<const uint4*>(prow);
  uint4* d0 = reinterpret_cast<uint4*>(g0 + t * 64);
  uint4* d1 = reinterpret_cast<uint4*>(g1 + t * 16);
  uint4* dp = reinterpret_cast<uint4*>(gp + t * 64);
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    d0[j] = rv[j];
    dp[j] = pv[j];
  }
  d1[0] = rv[8];
  d1[1] = rv[9];
}

// Small-stage VJP of one token; thread per token.  The Sinkhorn iterates are kept in
// `hist` ((iters-1) matrices, layout [iter][elem][T] so the stores coalesce).
template <int N>
__global__ void __launch_bounds__(128)
pre_small_bwd_kernel(const float* __restrict__ mixes, const float* __restrict__ alpha,
                     const float* __restrict__ base, const float* __restrict__ gpre,
                     const float* __restrict__ gpost, const float* __restrict__ gcomb,
                     const float* __restrict__ inv_rms, int64_t T, int64_t HC, SmallParams sp,
                     float* __restrict__ hist, float* __restrict__ gm_out,
                     float* __restrict__ coef_out, float* __restrict__ partials,
                     __nv_bfloat16* __restrict__ g0, __nv_bfloat16* __restrict__ g1,
                     __nv_bfloat16* __restrict__ gp) {
  pdl_enter();
  constexpr int HM = hc_mix(N);
  constexpr int NN = N * N;
  constexpr int NP = 3 + HM;
  __shared__ float sbase[HM];
  __shared__ float red[128][NP + 1];
  for (int i = threadIdx.x; i < HM; i += blockDim.x) sbase[i] = base[i];
  __syncthreads();
  sp.a0 = alpha[0]; sp.a1 = alpha[1]; sp.a2 = alpha[2];
  const int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  float contrib[NP];
#pragma unroll
  for (int i = 0; i < NP; ++i) contrib[i] = 0.f;
  if (t < T) {
    float mix[HM];
#pragma unroll
    for (int k = 0; k < HM; ++k) mix[k] = mixes[t * HM + k];
    float logits[NN], P[NN], M[NN];
    logits_softmax<N>(mix, sbase, sp, logits, P);
#pragma unroll
    for (int e = 0; e < NN; ++e) M[e] = P[e] + sp.hc_eps;
    col_norm<N>(M, sp.hc_eps);
    for (int it = 1; it < sp.iters; ++it) {
#pragma unroll
      for (int e = 0; e < NN; ++e) hist[((int64_t)(it - 1) * NN + e) * T + t] = M[e];
      row_norm<N>(M, sp.hc_eps);
      col_norm<N>(M, sp.hc_eps);
    }
    // ---- backward through the Sinkhorn iterations ----
    float g[NN];
#pragma unroll
    for (int e = 0; e < NN; ++e) g[e] = gcomb[t * NN + e];
    // the iterate of the next (older) iteration is loaded while this one is processed
    // (N <= 4: one iteration's loads would otherwise wait a full round trip each)
    float Qn[NN];
    if (sp.iters > 1) {
#pragma unroll
      for (int e = 0; e < NN; ++e) Qn[e] = hist[((int64_t)(sp.iters - 2) * NN + e) * T + t];
    }
    for (int it = sp.iters - 1; it >= 1; --it) {
      float Q[NN], rs[N], cs[N];  // reciprocals of the row / column divisors
      if constexpr (N <= 4) {
#pragma unroll
        for (int e = 0; e < NN; ++e) Q[e] = Qn[e];
        if (it > 1) {
#pragma unroll
          for (int e = 0; e < NN; ++e) Qn[e] = hist[((int64_t)(it - 2) * NN + e) * T + t];
        }
      } else {
#pragma unroll
        for (int e = 0; e < NN; ++e) Q[e] = hist[((int64_t)(it - 1) * NN + e) * T + t];
      }
      row_norm<N>(Q, sp.hc_eps, rs);       // Q = M_in / (rowsum + eps)
      float U[NN];
#pragma unroll
      for (int e = 0; e < NN; ++e) U[e] = Q[e];
      col_norm<N>(U, sp.hc_eps, cs);       // U = Q / (colsum + eps)
      // col-norm VJP: dQ = (g - sum_i g*U) / cs
#pragma unroll
      for (int j = 0; j < N; ++j) {
        float s = 0.f;
#pragma unroll
        for (int i = 0; i < N; ++i) s += g[i * N + j] * U[i * N + j];
#pragma unroll
        for (int i = 0; i < N; ++i) g[i * N + j] = (g[i * N + j] - s) * cs[j];
      }
      // row-norm VJP: dM = (dQ - sum_j dQ*Q) / rs
#pragma unroll
      for (int i = 0; i < N; ++i) {
        float s = 0.f;
#pragma unroll
        for (int j = 0; j < N; ++j) s += g[i * N + j] * Q[i * N + j];
#pragma unroll
        for (int j = 0; j < N; ++j) g[i * N + j] = (g[i * N + j] - s) * rs[i];
      }
    }
    // iteration 0: U0 = M0 / cs0, M0 = P + eps
    {
      float U[NN], cs[N];
#pragma unroll
      for (int e = 0; e < NN; ++e) U[e] = P[e] + sp.hc_eps;
      col_norm<N>(U, sp.hc_eps, cs);
#pragma unroll
      for (int j = 0; j < N; ++j) {
        float s = 0.f;
#pragma unroll
        for (int i = 0; i < N; ++i) s += g[i * N + j] * U[i * N + j];
#pragma unroll
        for (int i = 0; i < N; ++i) g[i * N + j] = (g[i * N + j] - s) * cs[j];
      }
    }
    // softmax VJP: dl = P * (dP - sum_j dP*P); clamp passes where min <= l <= max
    float gmx[HM];
#pragma unroll
    for (int i = 0; i < N; ++i) {
      float s = 0.f;
#pragma unroll
      for (int j = 0; j < N; ++j) s += g[i * N + j] * P[i * N + j];
#pragma unroll
      for (int j = 0; j < N; ++j) {
        const int e = i * N + j;
        float d = P[e] * (g[e] - s);
        if (sp.clamp_on && !(logits[e] >= sp.clamp_min && logits[e] <= sp.clamp_max)) d = 0.f;
        gmx[2 * N + e] = d * sp.a2;
        contrib[2] = fmaf(d, mix[2 * N + e], contrib[2]);
        contrib[3 + 2 * N + e] = d;
      }
    }
#pragma unroll
    for (int n = 0; n < N; ++n) {
      const float s0 = sigmoidf_(mix[n] * sp.a0 + sbase[n]);
      const float s1 = sigmoidf_(mix[N + n] * sp.a1 + sbase[N + n]);
      const float dz0 = gpre[t * N + n] * s0 * (1.0f - s0);
      const float dz1 = gpost[t * N + n] * 2.0f * s1 * (1.0f - s1);
      gmx[n] = dz0 * sp.a0;
      gmx[N + n] = dz1 * sp.a1;
      contrib[0] = fmaf(dz0, mix[n], contrib[0]);
      contrib[1] = fmaf(dz1, mix[N + n], contrib[1]);
      contrib[3 + n] = dz0;
      contrib[3 + N + n] = dz1;
    }
    float dot = 0.f;
#pragma unroll
    for (int k = 0; k < HM; ++k) {
      if (gm_out) gm_out[t * HM + k] = gmx[k];
      dot = fmaf(gmx[k], mix[k], dot);
    }
    const float inv = inv_rms[t];
    coef_out[t] = inv * inv / (float)HC * dot;
    if constexpr (N == 4) {
      if (g0) write_tc_operand_rows(gmx, inv, t, g0, g1, gp);
    }
  }
#pragma unroll
  for (int i = 0; i < NP; ++i) red[threadIdx.x][i] = contrib[i];
  __syncthreads();
  for (int i = threadIdx.x; i < NP; i += blockDim.x) {
    float s = 0.f;
    for (int r = 0; r < 128; ++r) s += red[r][i];
    partials[(int64_t)blockIdx.x * NP + i] = s;
  }
}

// Row-parallel small-stage VJP (N = 4, 8): N lanes per token, lane n owning row n of the
// Sinkhorn matrices.  Column sums (normalisation and the column-norm VJP) are gathered by
// shuffles and added in row order; row sums stay in the lane.  The chain of one token is
// N times shorter than in pre_small_bwd_kernel and a warp serves 32/N tokens.  hist
// layout [iter][T][N*N] (a token's iterate contiguous: its N lanes store one segment).
// Contributions to grad_alpha / grad_base are summed by fixed shuffle trees per warp and in
// warp order per block (deterministic), then by pre_reduce_ab_kernel; the token's
// grad_mixes are gathered in shared memory for its lane 0, which forms the RMS
// coefficient (same order as the one-thread kernel) and the tensor-core operand rows.
template <int N>
__global__ void __launch_bounds__(128)
pre_small_bwd_rows_kernel(const float* __restrict__ mixes, const float* __restrict__ alpha,
                          const float* __restrict__ base, const float* __restrict__ gpre,
                          const float* __restrict__ gpost, const float* __restrict__ gcomb,
                          const float* __restrict__ inv_rms, int64_t T, int64_t HC,
                          SmallParams sp, float* __restrict__ hist, float* __restrict__ gm_out,
                          float* __restrict__ coef_out, float* __restrict__ partials,
                          __nv_bfloat16* __restrict__ g0, __nv_bfloat16* __restrict__ g1,
                          __nv_bfloat16* __restrict__ gp) {
  pdl_enter();
  constexpr int HM = hc_mix(N);
  constexpr int NN = N * N;
  constexpr int NP = 3 + HM;
  constexpr int TPB = 128 / N;  // tokens per block
  static_assert(N == 4 || N == 8, "row groups of 4 or 8 lanes");
  __shared__ float sbase[HM];
  __shared__ float wred[4][NP];  // per-warp sums of the contributions
  __shared__ float sg[TPB][HM];
  for (int i = threadIdx.x; i < HM; i += blockDim.x) sbase[i] = base[i];
  __syncthreads();
  sp.a0 = alpha[0]; sp.a1 = alpha[1]; sp.a2 = alpha[2];
  const int lane = threadIdx.x & 31, n = lane % N, gl0 = (lane / N) * N;
  const int tl = threadIdx.x / N;
  const int64_t t = (int64_t)blockIdx.x * TPB + tl;
  const bool valid = t < T;
  const int64_t tc = valid ? t : T - 1;  // invalid lanes still take part in the shuffles
  auto colsum = [&](float v) {  // sum over the group's rows of one column, row order
    float c = 0.f;
#pragma unroll
    for (int i = 0; i < N; ++i) c += __shfl_sync(0xffffffffu, v, gl0 + i);
    return c;
  };
  const float* mx = mixes + tc * HM;
  const float m_pre = mx[n], m_post = mx[N + n];
  float ml[N], logit[N], P[N], M[N];
#pragma unroll
  for (int j = 0; j < N; ++j) ml[j] = mx[2 * N + n * N + j];
  // forward recompute: logits row, clamp, softmax row, +eps, Sinkhorn
#pragma unroll
  for (int j = 0; j < N; ++j) {
    logit[j] = ml[j] * sp.a2 + sbase[2 * N + n * N + j];
    P[j] = sp.clamp_on ? fminf(fmaxf(logit[j], sp.clamp_min), sp.clamp_max) : logit[j];
  }
  {
    float m = P[0];
#pragma unroll
    for (int j = 1; j < N; ++j) m = fmaxf(m, P[j]);
    float s = 0.f;
#pragma unroll
    for (int j = 0; j < N; ++j) {
      P[j] = expf(P[j] - m);
      s += P[j];
    }
    const float rs = 1.0f / s;
#pragma unroll
    for (int j = 0; j < N; ++j) P[j] *= rs;
  }
#pragma unroll
  for (int j = 0; j < N; ++j) M[j] = P[j] + sp.hc_eps;
  auto col_norm_row = [&](float* R, float* cs) {
#pragma unroll
    for (int j = 0; j < N; ++j) {
      const float c = 1.0f / (colsum(R[j]) + sp.hc_eps);
      if (cs) cs[j] = c;
      R[j] *= c;
    }
  };
  auto row_norm_row = [&](float* R) {
    float r = 0.f;
#pragma unroll
    for (int j = 0; j < N; ++j) r += R[j];
    const float rr = 1.0f / (r + sp.hc_eps);
#pragma unroll
    for (int j = 0; j < N; ++j) R[j] *= rr;
    return rr;
  };
  col_norm_row(M, nullptr);
  for (int it = 1; it < sp.iters; ++it) {
    if (valid) {
      float4* h4 = reinterpret_cast<float4*>(hist + ((int64_t)(it - 1) * T + t) * NN + n * N);
#pragma unroll
      for (int q = 0; q < N / 4; ++q)
        h4[q] = make_float4(M[4 * q], M[4 * q + 1], M[4 * q + 2], M[4 * q + 3]);
    }
    row_norm_row(M);
    col_norm_row(M, nullptr);
  }
  // backward through the Sinkhorn iterations (the next older iterate is loaded ahead)
  float g[N], Qn[N];
#pragma unroll
  for (int j = 0; j < N; ++j) g[j] = gcomb[tc * NN + n * N + j];
  auto load_row = [&](int it, float* R) {
    const float4* h4 =
        reinterpret_cast<const float4*>(hist + ((int64_t)(it - 1) * T + tc) * NN + n * N);
#pragma unroll
    for (int q = 0; q < N / 4; ++q) {
      const float4 v = valid ? h4[q] : make_float4(0.f, 0.f, 0.f, 0.f);
      R[4 * q] = v.x; R[4 * q + 1] = v.y; R[4 * q + 2] = v.z; R[4 * q + 3] = v.w;
    }
  };
  if (sp.iters > 1) load_row(sp.iters - 1, Qn);
  auto col_vjp = [&](const float* U, const float* cs) {  // dQ = (g - sum_i g*U) / colsum
#pragma unroll
    for (int j = 0; j < N; ++j) {
      float s = 0.f;  // fma chain in row order, as the one-thread kernel's loop compiles
#pragma unroll
      for (int i = 0; i < N; ++i)
        s = fmaf(__shfl_sync(0xffffffffu, g[j], gl0 + i), __shfl_sync(0xffffffffu, U[j], gl0 + i),
                 s);
      g[j] = (g[j] - s) * cs[j];
    }
  };
  for (int it = sp.iters - 1; it >= 1; --it) {
    float Q[N], U[N], cs[N];
#pragma unroll
    for (int j = 0; j < N; ++j) Q[j] = Qn[j];
    if (it > 1) load_row(it - 1, Qn);
    const float rs = row_norm_row(Q);      // Q = M_in / (rowsum + eps)
#pragma unroll
    for (int j = 0; j < N; ++j) U[j] = Q[j];
    col_norm_row(U, cs);                   // U = Q / (colsum + eps)
    col_vjp(U, cs);
    float s = 0.f;                         // row-norm VJP: dM = (dQ - sum_j dQ*Q) / rowsum
#pragma unroll
    for (int j = 0; j < N; ++j) s += g[j] * Q[j];
#pragma unroll
    for (int j = 0; j < N; ++j) g[j] = (g[j] - s) * rs;
  }
  {  // iteration 0: U0 = M0 / cs0, M0 = P + eps
    float U[N], cs[N];
#pragma unroll
    for (int j = 0; j < N; ++j) U[j] = P[j] + sp.hc_eps;
    col_norm_row(U, cs);
    col_vjp(U, cs);
  }
  // softmax VJP of row n: dl = P * (dP - sum_j dP*P); clamp passes where min <= l <= max
  float c2 = 0.f, gl[N], dl[N];
  {
    float s = 0.f;
#pragma unroll
    for (int j = 0; j < N; ++j) s += g[j] * P[j];
#pragma unroll
    for (int j = 0; j < N; ++j) {
      float d = P[j] * (g[j] - s);
      if (sp.clamp_on && !(logit[j] >= sp.clamp_min && logit[j] <= sp.clamp_max)) d = 0.f;
      gl[j] = d * sp.a2;
      c2 = fmaf(d, ml[j], c2);
      dl[j] = valid ? d : 0.f;
    }
  }
  const float s0 = sigmoidf_(m_pre * sp.a0 + sbase[n]);
  const float s1 = sigmoidf_(m_post * sp.a1 + sbase[N + n]);
  const float dz0 = gpre[tc * N + n] * s0 * (1.0f - s0);
  const float dz1 = gpost[tc * N + n] * 2.0f * s1 * (1.0f - s1);
  // contributions to grad_alpha (3) and grad_base (HM): sums over the warp's tokens by
  // fixed xor trees (common entries over all lanes, row entries over lanes of equal n),
  // then over the block's 4 warps in order
  {
    float cm[3] = {valid ? dz0 * m_pre : 0.f, valid ? dz1 * m_post : 0.f, valid ? c2 : 0.f};
    float rw[2 + N];
    rw[0] = valid ? dz0 : 0.f;
    rw[1] = valid ? dz1 : 0.f;
#pragma unroll
    for (int j = 0; j < N; ++j) rw[2 + j] = dl[j];
#pragma unroll
    for (int c = 0; c < 3; ++c) cm[c] = warp_sum(cm[c]);
#pragma unroll
    for (int o = N; o < 32; o <<= 1)
#pragma unroll
      for (int c = 0; c < 2 + N; ++c) rw[c] += __shfl_xor_sync(0xffffffffu, rw[c], o);
    const int w = threadIdx.x >> 5;
    if (lane < 3) wred[w][lane] = lane == 0 ? cm[0] : (lane == 1 ? cm[1] : cm[2]);
    if (lane < N) {
      wred[w][3 + n] = rw[0];
      wred[w][3 + N + n] = rw[1];
#pragma unroll
      for (int j = 0; j < N; ++j) wred[w][3 + 2 * N + n * N + j] = rw[2 + j];
    }
  }
  sg[tl][n] = dz0 * sp.a0;
  sg[tl][N + n] = dz1 * sp.a1;
#pragma unroll
  for (int j = 0; j < N; ++j) sg[tl][2 * N + n * N + j] = gl[j];
  if (valid && gm_out) {
    gm_out[t * HM + n] = dz0 * sp.a0;
    gm_out[t * HM + N + n] = dz1 * sp.a1;
#pragma unroll
    for (int j = 0; j < N; ++j) gm_out[t * HM + 2 * N + n * N + j] = gl[j];
  }
  __syncwarp();
  if (n == 0 && valid) {
    float gmx[HM], dot = 0.f;
#pragma unroll
    for (int k = 0; k < HM; ++k) {
      gmx[k] = sg[tl][k];
      dot = fmaf(gmx[k], mx[k], dot);
    }
    const float inv = inv_rms[t];
    coef_out[t] = inv * inv / (float)HC * dot;
    if constexpr (N == 4) {
      if (g0) write_tc_operand_rows(gmx, inv, t, g0, g1, gp);
    }
  }
  __syncthreads();
  for (int i = threadIdx.x; i < NP; i += blockDim.x)
    partials[(int64_t)blockIdx.x * NP + i] = ((wred[0][i] + wred[1][i]) + wred[2][i]) + wred[3][i];
}

// The comb part of the N = 4 small-stage VJP for one token on a group of 16 lanes (lane e
// owns element [e / 4][e % 4]): forward recompute of the clamp, row softmax, +eps and the
// Sinkhorn iterations (iterates stored in hist [iter][T][16]), the VJP back through them
// and through the softmax, and the clamp mask.  Returns d = dL/dlogit of the lane's
// element.  It depends on mixes and grad_comb only -- not on grad_pre -- so it can run
// while grad_pre is still being summed.  Every row / column sum gathers its 4 values by
// shuffles and adds them in index order (the order of the row-parallel kernel).
__device__ __forceinline__ float comb_vjp_elem(float ml, float base_l, const SmallParams& sp,
                                               float gcomb_e, float* __restrict__ hist,
                                               int64_t T, int64_t t, int64_t tc, bool valid,
                                               int e, int gl0) {
  constexpr int N = 4, NN = 16;
  const int n = e / N, j = e % N;
  auto at = [&](float v, int src) { return __shfl_sync(0xffffffffu, v, gl0 + src); };
  auto rowsum = [&](float v) {  // sum of row n, column order
    float r = 0.f;
#pragma unroll
    for (int jj = 0; jj < N; ++jj) r += at(v, n * N + jj);
    return r;
  };
  auto colsum = [&](float v) {  // sum of column j, row order
    float c = 0.f;
#pragma unroll
    for (int i = 0; i < N; ++i) c += at(v, i * N + j);
    return c;
  };
  // forward recompute: logit, clamp, softmax row, +eps, Sinkhorn
  const float logit = ml * sp.a2 + base_l;
  float P = sp.clamp_on ? fminf(fmaxf(logit, sp.clamp_min), sp.clamp_max) : logit;
  {
    float m = at(P, n * N);
#pragma unroll
    for (int jj = 1; jj < N; ++jj) m = fmaxf(m, at(P, n * N + jj));
    const float ex = expf(P - m);
    const float rs = 1.0f / rowsum(ex);
    P = ex * rs;
  }
  float M = P + sp.hc_eps;
  M *= 1.0f / (colsum(M) + sp.hc_eps);
  for (int it = 1; it < sp.iters; ++it) {
    if (valid) hist[((int64_t)(it - 1) * T + t) * NN + e] = M;
    M *= 1.0f / (rowsum(M) + sp.hc_eps);
    M *= 1.0f / (colsum(M) + sp.hc_eps);
  }
  // backward through the Sinkhorn iterations (the next older iterate is loaded ahead)
  float g = gcomb_e;
  auto load_el = [&](int it) {
    return valid ? hist[((int64_t)(it - 1) * T + tc) * NN + e] : 0.f;
  };
  float Qn = sp.iters > 1 ? load_el(sp.iters - 1) : 0.f;
  auto col_vjp = [&](float U, float cs) {  // dQ = (g - sum_i g*U) / colsum
    float s = 0.f;
#pragma unroll
    for (int i = 0; i < N; ++i) s = fmaf(at(g, i * N + j), at(U, i * N + j), s);
    g = (g - s) * cs;
  };
  for (int it = sp.iters - 1; it >= 1; --it) {
    float Q = Qn;
    if (it > 1) Qn = load_el(it - 1);
    const float rs = 1.0f / (rowsum(Q) + sp.hc_eps);
    Q *= rs;                                   // Q = M_in / (rowsum + eps)
    const float cs = 1.0f / (colsum(Q) + sp.hc_eps);
    const float U = Q * cs;                    // U = Q / (colsum + eps)
    col_vjp(U, cs);
    float s = 0.f;                             // row-norm VJP
#pragma unroll
    for (int jj = 0; jj < N; ++jj) s = fmaf(at(g, n * N + jj), at(Q, n * N + jj), s);
    g = (g - s) * rs;
  }
  {  // iteration 0: U0 = M0 / cs0, M0 = P + eps
    const float U0 = P + sp.hc_eps;
    const float cs = 1.0f / (colsum(U0) + sp.hc_eps);
    col_vjp(U0 * cs, cs);
  }
  // softmax VJP of row n: dl = P * (dP - sum_j dP*P); clamp passes where min <= l <= max
  float d;
  {
    float s = 0.f;
#pragma unroll
    for (int jj = 0; jj < N; ++jj) s = fmaf(at(g, n * N + jj), at(P, n * N + jj), s);
    d = P * (g - s);
    if (sp.clamp_on && !(logit >= sp.clamp_min && logit <= sp.clamp_max)) d = 0.f;
  }
  return d;
}

// Element-parallel small-stage VJP (N = 4): N*N = 16 lanes per token (two tokens per
// warp), lane (n, j) owning element [n][j] of the Sinkhorn matrices.  Every row or column
// sum gathers its N values by shuffles and adds them in index order -- the operations and
// the order of pre_small_bwd_rows_kernel -- but each lane carries one element instead of
// a row, so a token's dependent chain is about N times shorter and four times as many
// warps share the latency.  Used while the GPU would otherwise be short of warps (small
// T).  The grad_alpha / grad_base contributions of a block's tokens are added in token
// order through shared memory (deterministic), then by pre_reduce_ab_kernel.
template <int N, bool PRE_D>
__global__ void __launch_bounds__(128)
pre_small_bwd_elems_kernel(const float* __restrict__ dlog, const float* __restrict__ mixes,
                           const float* __restrict__ alpha,
                           const float* __restrict__ base, const float* __restrict__ gpre,
                           const float* __restrict__ gpost, const float* __restrict__ gcomb,
                           const float* __restrict__ inv_rms, int64_t T, int64_t HC,
                           SmallParams sp, float* __restrict__ hist, float* __restrict__ gm_out,
                           float* __restrict__ coef_out, float* __restrict__ partials,
                           __nv_bfloat16* __restrict__ g0, __nv_bfloat16* __restrict__ g1,
                           __nv_bfloat16* __restrict__ gp, unsigned* __restrict__ ticket,
                           float* __restrict__ grad_alpha, float* __restrict__ grad_base) {
  pdl_enter();
  constexpr int HM = hc_mix(N);
  constexpr int NN = N * N;
  constexpr int NP = 3 + HM;
  constexpr int TPB = 128 / NN;  // tokens per block
  static_assert(N == 4, "16 lanes per token");
  __shared__ float sbase[HM];
  __shared__ float sg[TPB][HM];
  __shared__ float sc[TPB][NP];  // per-token contributions to grad_alpha | grad_base
  for (int i = threadIdx.x; i < HM; i += blockDim.x) sbase[i] = base[i];
  __syncthreads();
  sp.a0 = alpha[0]; sp.a1 = alpha[1]; sp.a2 = alpha[2];
  const int lane = threadIdx.x & 31;
  const int e = lane % NN, n = e / N, j = e % N;
  const int gl0 = (lane / NN) * NN;  // first lane of this token's group
  const int tl = threadIdx.x / NN;
  const int64_t t = (int64_t)blockIdx.x * TPB + tl;
  const bool valid = t < T;
  const int64_t tc = valid ? t : T - 1;  // invalid lanes still take part in the shuffles
  auto at = [&](float v, int src) { return __shfl_sync(0xffffffffu, v, gl0 + src); };
  auto rowsum = [&](float v) {  // sum of row n, column order
    float r = 0.f;
#pragma unroll
    for (int jj = 0; jj < N; ++jj) r += at(v, n * N + jj);
    return r;
  };
  auto colsum = [&](float v) {  // sum of column j, row order
    float c = 0.f;
#pragma unroll
    for (int i = 0; i < N; ++i) c += at(v, i * N + j);
    return c;
  };
  const float* mx = mixes + tc * HM;
  const float ml = mx[2 * N + n * N + j];
  float d;
  if constexpr (PRE_D) {
    d = valid ? dlog[tc * NN + e] : 0.f;
  } else {
    d = comb_vjp_elem(ml, sbase[2 * N + e], sp, gcomb[tc * NN + e], hist, T, t, tc, valid, e,
                      gl0);
  }
  const float gl = d * sp.a2;
  float c2 = 0.f;  // this row's fma chain over j, as the row-parallel kernel forms it
#pragma unroll
  for (int jj = 0; jj < N; ++jj) c2 = fmaf(at(d, n * N + jj), at(ml, n * N + jj), c2);
  const float m_pre = mx[n], m_post = mx[N + n];
  const float s0 = sigmoidf_(m_pre * sp.a0 + sbase[n]);
  const float s1 = sigmoidf_(m_post * sp.a1 + sbase[N + n]);
  const float dz0 = gpre[tc * N + n] * s0 * (1.0f - s0);
  const float dz1 = gpost[tc * N + n] * 2.0f * s1 * (1.0f - s1);
  // per-token contributions (rows add in row order)
  sc[tl][3 + 2 * N + e] = valid ? d : 0.f;
  if (j == 0) {
    sc[tl][3 + n] = valid ? dz0 : 0.f;
    sc[tl][3 + N + n] = valid ? dz1 : 0.f;
  }
  float a0c = valid ? dz0 * m_pre : 0.f, a1c = valid ? dz1 * m_post : 0.f,
        a2c = valid ? c2 : 0.f;
  float r0 = 0.f, r1 = 0.f, r2 = 0.f;
#pragma unroll
  for (int i = 0; i < N; ++i) {
    r0 += at(a0c, i * N);
    r1 += at(a1c, i * N);
    r2 += at(a2c, i * N);
  }
  if (e == 0) {
    sc[tl][0] = r0;
    sc[tl][1] = r1;
    sc[tl][2] = r2;
  }
  if (j == 0) {
    sg[tl][n] = dz0 * sp.a0;
    sg[tl][N + n] = dz1 * sp.a1;
  }
  sg[tl][2 * N + e] = gl;
  if (valid && gm_out) {
    if (j == 0) {
      gm_out[t * HM + n] = dz0 * sp.a0;
      gm_out[t * HM + N + n] = dz1 * sp.a1;
    }
    gm_out[t * HM + 2 * N + e] = gl;
  }
  __syncwarp();
  if (e == 0 && valid) {
    float gmx[HM], dot = 0.f;
#pragma unroll
    for (int k = 0; k < HM; ++k) {
      gmx[k] = sg[tl][k];
      dot = fmaf(gmx[k], mx[k], dot);
    }
    const float inv = inv_rms[t];
    coef_out[t] = inv * inv / (float)HC * dot;
    if (g0) write_tc_operand_rows(gmx, inv, t, g0, g1, gp);
  }
  __syncthreads();
  for (int i = threadIdx.x; i < NP; i += blockDim.x) {
    float acc = 0.f;
#pragma unroll
    for (int k = 0; k < TPB; ++k) acc += sc[k][i];
    partials[(int64_t)blockIdx.x * NP + i] = acc;
  }
  if (ticket == nullptr) return;
  // the last block to finish adds every block's partials into grad_alpha / grad_base, in
  // the order pre_reduce_ab_kernel uses (lane-strided blocks, then a fixed warp tree), so
  // which block happens to be last does not change the result
  __shared__ bool last;
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    last = atomicAdd(ticket, 1u) == gridDim.x - 1;
  }
  __syncthreads();
  if (!last) return;
  __threadfence();
  const int w = threadIdx.x >> 5, nw = blockDim.x >> 5;
  for (int o = w; o < NP; o += nw) {
    Kahan k;
    // eight loads in flight per lane, added in block order
    for (int b0 = lane; b0 < (int)gridDim.x; b0 += 32 * 8) {
      float v[8];
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        const int b = b0 + 32 * u;
        v[u] = b < (int)gridDim.x ? __ldcg(partials + (int64_t)b * NP + o) : 0.f;
      }
#pragma unroll
      for (int u = 0; u < 8; ++u)
        if (b0 + 32 * u < (int)gridDim.x) k.add(v[u]);
    }
    const float acc = warp_sum(k.s);
    if (lane == 0) {
      if (o < 3) grad_alpha[o] = acc;
      else grad_base[o - 3] = acc;
    }
  }
  if (threadIdx.x == 0) *ticket = 0u;  // ready for the next call
}

// One warp per output value: lanes take strided partials, then a fixed-shape tree
// (warp_sum) -- deterministic for a given number of blocks.
__global__ void pre_reduce_ab_kernel(const float* __restrict__ partials, int nblk, int HM,
                                     float* __restrict__ grad_alpha,
                                     float* __restrict__ grad_base) {
  pdl_enter();
  const int NP = 3 + HM;
  const int w = (int)((blockIdx.x * blockDim.x + threadIdx.x) >> 5), lane = threadIdx.x & 31;
  if (w >= NP) return;
  Kahan k;
  for (int b = lane; b < nblk; b += 32) k.add(partials[(int64_t)b * NP + w]);
  const float acc = warp_sum(k.s);
  if (lane == 0) {
    if (w < 3) grad_alpha[w] = acc;
    else grad_base[w - 3] = acc;
  }
}

constexpr int kGxTT = 16;   // tokens per CTA
constexpr int kGxCC = 256;  // columns per CTA (one per thread)

template <typename E, int N>
__global__ void __launch_bounds__(kGxCC)
pre_bwd_gx_kernel(const E* __restrict__ x, const E* __restrict__ gy,
                  const float* __restrict__ phi, const float* __restrict__ gm,
                  const float* __restrict__ inv_rms, const float* __restrict__ coef,
                  const float* __restrict__ pre, const E* acc, E* gx,  // may alias
                  int64_t T, int64_t D, int64_t xs, int64_t gys) {
  pdl_enter();
  constexpr int HM = hc_mix(N);
  const int64_t HC = (int64_t)N * D;
  __shared__ float sgm[kGxTT][HM];
  __shared__ float sinv[kGxTT], scoef[kGxTT], spre[kGxTT][N];
  const int64_t t0 = (int64_t)blockIdx.x * kGxTT;
  for (int i = threadIdx.x; i < kGxTT * HM; i += blockDim.x) {
    const int64_t t = t0 + i / HM;
    sgm[i / HM][i % HM] = t < T ? gm[t * HM + i % HM] : 0.f;
  }
  for (int i = threadIdx.x; i < kGxTT; i += blockDim.x) {
    const int64_t t = t0 + i;
    sinv[i] = t < T ? inv_rms[t] : 0.f;
    scoef[i] = t < T ? coef[t] : 0.f;
  }
  for (int i = threadIdx.x; i < kGxTT * N; i += blockDim.x) {
    const int64_t t = t0 + i / N;
    spre[i / N][i % N] = t < T ? pre[t * N + i % N] : 0.f;
  }
  __syncthreads();
  const int64_t c = (int64_t)blockIdx.y * kGxCC + threadIdx.x;
  if (c >= HC) return;
  const int n = (int)(c / D);
  const int64_t d = c - (int64_t)n * D;
  float ph[HM];
#pragma unroll
  for (int k = 0; k < HM; ++k) ph[k] = __ldg(phi + (int64_t)k * HC + c);
  for (int tt = 0; tt < kGxTT; ++tt) {
    const int64_t t = t0 + tt;
    if (t >= T) break;
    float gxs = 0.f;
#pragma unroll
    for (int k = 0; k < HM; ++k) gxs = fmaf(sgm[tt][k], ph[k], gxs);
    const float xv = ld1<E>(x + t * xs + c);
    const float g = ld1<E>(gy + t * gys + d);
    const float r = fmaf(sinv[tt], gxs, -scoef[tt] * xv);
    float v = fmaf(g, spre[tt][n], r);
    if (acc) v += ld1<E>(acc + t * HC + c);
    st1<E>(gx + t * HC + c, v);
  }
}

constexpr int kGpCC = 256;  // columns per CTA
constexpr int kGpTS = 32;   // tokens staged per step

template <typename E, int N>
__global__ void __launch_bounds__(kGpCC)
pre_bwd_gphi_kernel(const E* __restrict__ x, const float* __restrict__ gm,
                    const float* __restrict__ inv_rms, float* __restrict__ part, int64_t T,
                    int64_t HC, int64_t tokens_per_split, int64_t xs) {
  pdl_enter();
  constexpr int HM = hc_mix(N);
  __shared__ float sg[kGpTS][HM];
  const int64_t c = (int64_t)blockIdx.x * kGpCC + threadIdx.x;
  const int64_t tb = (int64_t)blockIdx.y * tokens_per_split;
  const int64_t te = min(T, tb + tokens_per_split);
  float acc[HM];
#pragma unroll
  for (int k = 0; k < HM; ++k) acc[k] = 0.f;
  for (int64_t ts = tb; ts < te; ts += kGpTS) {
    __syncthreads();
    for (int i = threadIdx.x; i < kGpTS * HM; i += blockDim.x) {
      const int64_t t = ts + i / HM;
      sg[i / HM][i % HM] = t < te ? gm[t * HM + i % HM] * inv_rms[t] : 0.f;
    }
    __syncthreads();
    if (c < HC) {
      const int nt = (int)min((int64_t)kGpTS, te - ts);
      for (int tt = 0; tt < nt; ++tt) {
        const float xv = ld1<E>(x + (ts + tt) * xs + c);
#pragma unroll
        for (int k = 0; k < HM; ++k) acc[k] = fmaf(sg[tt][k], xv, acc[k]);
      }
    }
  }
  if (c < HC) {
#pragma unroll
    for (int k = 0; k < HM; ++k) part[((int64_t)blockIdx.y * HM + k) * HC + c] = acc[k];
  }
}

__global__ void pre_reduce_gphi_kernel(const float* __restrict__ part, int nsplit, int64_t n,
                                       float* __restrict__ out) {
  pdl_enter();
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  Kahan s;
  for (int p = 0; p < nsplit; ++p) s.add(part[(int64_t)p * n + i]);
  out[i] = s.s;
}

// ---------------------------------------------------------------------------
// Host side
// ---------------------------------------------------------------------------
static int gphi_splits(int64_t T) {
  int64_t s = cdiv(T, 2048);
  return (int)(s < 1 ? 1 : (s > 16 ? 16 : s));
}

bool pre_bwd_tc_eligible(const PreBwdArgs& a);
size_t pre_bwd_tc_ws_bytes(int64_t T, int64_t D);
void pre_bwd_tc_operand_ptrs(void* ws, int64_t T, int64_t D, __nv_bfloat16** g0,
                             __nv_bfloat16** g1, __nv_bfloat16** gp, __nv_bfloat16** p0,
                             __nv_bfloat16** p1);
int pre_bwd_tc_main(const PreBwdArgs& a, void* ws, const float* gm, const float* coef,
                    cudaStream_t s);
bool pre_bwd_tc8_eligible(const PreBwdArgs& a);
bool pre_bwd_tc32_eligible(const PreBwdArgs& a);
size_t pre_bwd_tc32_ws_bytes(int64_t T, int32_t N, int64_t D);
int pre_bwd_tc32_main(const PreBwdArgs& a, void* ws, const float* gm, const float* coef,
                      cudaStream_t s);
size_t pre_bwd_tc8_ws_bytes(int64_t T, int64_t D);
int pre_bwd_tc8_main(const PreBwdArgs& a, void* ws, const float* gm, const float* coef,
                     cudaStream_t s);

struct BwdWs {
  float *gpre, *gm, *coef, *partials, *hist, *gphi_part, *dlog;
  unsigned* ticket;
  size_t total;
};

static BwdWs bwd_layout(char* base, int64_t T, int32_t N, int64_t D, int32_t iters) {
  const int HM = hc_mix(N);
  const int64_t HC = (int64_t)N * D;
  const int64_t nblk = cdiv(T, 8);  // blocks of the small-stage VJP (>= 8 tokens each)
  const int64_t hist_n = (int64_t)(iters > 1 ? iters - 1 : 0) * N * N * T;
  BwdWs w;
  size_t off = 0;
  auto take = [&](size_t bytes) { float* p = (float*)(base + off); off += align_up(bytes); return p; };
  w.gpre = take((size_t)T * N * 4);
  w.gm = take((size_t)T * HM * 4);
  w.coef = take((size_t)T * 4);
  w.partials = take((size_t)nblk * (3 + HM) * 4);
  w.hist = take((size_t)hist_n * 4);
  w.gphi_part = take((size_t)gphi_splits(T) * HM * HC * 4);
  w.dlog = take((size_t)T * N * N * 4);
  w.ticket = (unsigned*)take(4);
  w.total = off;
  return w;
}

static bool tc_shape(int64_t T, int32_t N, int64_t D, int32_t dtype) {
  return (dtype == MHC_BF16 || dtype == MHC_F16) && N == 4 && D % 128 == 0 && T > 0;
}

static bool tc8_shape(int64_t T, int32_t N, int64_t D, int32_t dtype) {
  return (dtype == MHC_BF16 || dtype == MHC_F16) && N == 8 && D % 64 == 0 && T > 0;
}

// generic region, then (bf16 / fp16, N=4, D%128==0 or N=8, D%64==0; fp32, N=4 or 8,
// D%32==0) the tensor-core region
size_t pre_bwd_ws_bytes(int64_t T, int32_t N, int64_t D, int32_t dtype, int32_t iters) {
  size_t n = bwd_layout(nullptr, T, N, D, iters).total;
  if (tc_shape(T, N, D, dtype)) n += align_up(pre_bwd_tc_ws_bytes(T, D));
  if (tc8_shape(T, N, D, dtype)) n += align_up(pre_bwd_tc8_ws_bytes(T, D));
  if (dtype == MHC_F32 && (N == 4 || N == 8) && D % 32 == 0 && T > 0)
    n += align_up(pre_bwd_tc32_ws_bytes(T, N, D));
  return n;
}

template <typename E, int N>
static int pre_bwd_impl(const PreBwdArgs& a, cudaStream_t s) {
  constexpr int HM = hc_mix(N);
  const int64_t T = a.T, D = a.D, HC = (int64_t)N * D;
  BwdWs w = bwd_layout((char*)a.workspace, T, N, D, a.sp.iters);
  const bool acc_ok = a.grad_x_acc == nullptr || aligned16(a.grad_x_acc);
  constexpr bool is_bf16 = std::is_same<E, __nv_bfloat16>::value;
  const bool use_tc = sizeof(E) == 2 && acc_ok &&
                      pre_bwd_tc_eligible(a);
  const bool use_tc8 = sizeof(E) == 2 && acc_ok &&
                       pre_bwd_tc8_eligible(a);
  const bool use_tc32 = sizeof(E) == 4 && pre_bwd_tc32_eligible(a);
  char* tc_ws = (char*)a.workspace + w.total;
  __nv_bfloat16 *g0 = nullptr, *g1 = nullptr, *gp = nullptr, *p0 = nullptr, *p1 = nullptr;
  // bf16: pass 1 writes the operand rows (and the dots kernel the phi operand rows); fp16:
  // they need the maxima first (written from grad_mixes by pre_bwd_tc_main)
  if (use_tc && is_bf16) pre_bwd_tc_operand_ptrs(tc_ws, T, D, &g0, &g1, &gp, &p0, &p1);
  PreBwdArgs args = a;
  args.phi_prepped = p0 != nullptr;
  const int nphi = p0 ? (int)cdiv(3 * HC, 256) : 0;
  if (T == 0) {
    MHC_CUDA_CHECK(cudaMemsetAsync(a.grad_alpha, 0, 3 * sizeof(float), s));
    MHC_CUDA_CHECK(cudaMemsetAsync(a.grad_base, 0, HM * sizeof(float), s));
    MHC_CUDA_CHECK(cudaMemsetAsync(a.grad_phi, 0, (size_t)HM * HC * sizeof(float), s));
    return MHC_OK;
  }
  const bool vec = (D % Pack<E>::n == 0) && rows_aligned(a.x, a.x_ts, sizeof(E), 16) &&
                   rows_aligned(a.grad_y, a.gy_ts, sizeof(E), 16);
  const int64_t want = cdiv(T, 8), cap = (int64_t)sm_count() * 8;
  dim3 sgrid((unsigned)(want < cap ? want : cap));
  // small T (fewer than 8 tokens per SM): a block per token, its warps split the row
  const bool dsplit = T < cap;
  const int ndots = dsplit ? (int)T : (int)sgrid.x;
  // small-stage VJP.  Row-parallel (N lanes per token, N = 4, 8) while a thread per token
  // would not give every SM a block: its chain is N times shorter but it issues ~3N^2
  // shuffles per lane and iteration, so once the GPU is full the one-thread kernel wins
  // (T=32768, N=4: 1.169 vs 1.191 ms pre backward; T=1: 56 vs 49.5 us).  For N=4 it runs
  // element-parallel (16 lanes per token) and in two parts: the comb part, which needs no
  // grad_pre, as extra blocks of the grad_pre kernel (hidden under its HBM stream), then a
  // short kernel for the heads, the coefficients and the operand rows.
  constexpr bool rows_ok = N == 4 || N == 8;
  const bool rows = rows_ok && cdiv(T, 128) < sm_count();
  const bool elems = rows && N == 4;
  VjpArgs va{a.mixes, a.alpha, a.base, a.grad_comb, w.hist, w.dlog, w.ticket, a.sp,
             elems ? (int)cdiv(T, 16) : 0};
  auto dots = vec ? (dsplit ? pre_bwd_dots_kernel<E, N, true, true>
                            : pre_bwd_dots_kernel<E, N, true, false>)
                  : pre_bwd_dots_kernel<E, N, false, false>;
  launch(dots, (unsigned)(ndots + nphi + va.nblk), 256, 0, s, (const E*)a.x,
         (const E*)a.grad_y, w.gpre, T, D, a.x_ts, a.gy_ts, ndots, a.phi, (E*)p0, (E*)p1, nphi,
         va);
  MHC_LAUNCH_CHECK();
  const int nblk = (int)cdiv(T, elems ? 128 / (N * N) : rows ? 128 / N : 128);
  if (elems)
    launch(pre_small_bwd_elems_kernel<4, true>, nblk, 128, 0, s, (const float*)w.dlog,
        a.mixes, a.alpha, a.base, w.gpre, a.grad_post, a.grad_comb, a.inv_rms, T, HC, a.sp,
        w.hist, (use_tc && is_bf16) ? nullptr : w.gm, w.coef, w.partials, g0, g1, gp, w.ticket,
        a.grad_alpha, a.grad_base);
  else if (rows)
    launch(pre_small_bwd_rows_kernel<rows_ok ? N : 4>, nblk, 128, 0, s,
        a.mixes, a.alpha, a.base, w.gpre, a.grad_post, a.grad_comb, a.inv_rms, T, HC, a.sp,
        w.hist, (use_tc && is_bf16) ? nullptr : w.gm, w.coef, w.partials, g0, g1, gp);
  else
    launch(pre_small_bwd_kernel<N>, nblk, 128, 0, s,
        a.mixes, a.alpha, a.base, w.gpre, a.grad_post, a.grad_comb, a.inv_rms, T, HC, a.sp,
        w.hist, (use_tc && is_bf16) ? nullptr : w.gm, w.coef, w.partials, g0, g1, gp);
  MHC_LAUNCH_CHECK();
  if (!elems) {  // the element-parallel kernel's last block adds the partials itself
    launch(pre_reduce_ab_kernel, (unsigned)cdiv((3 + HM) * 32, 256), 256, 0, s, w.partials,
           nblk, HM, a.grad_alpha, a.grad_base);
    MHC_LAUNCH_CHECK();
  }
  if (use_tc) return pre_bwd_tc_main(args, tc_ws, w.gm, w.coef, s);
  if (use_tc8) return pre_bwd_tc8_main(a, tc_ws, w.gm, w.coef, s);
  if (use_tc32) return pre_bwd_tc32_main(a, tc_ws, w.gm, w.coef, s);
  dim3 ggrid((unsigned)cdiv(T, kGxTT), (unsigned)cdiv(HC, kGxCC));
  launch(pre_bwd_gx_kernel<E, N>, ggrid, kGxCC, 0, s, (const E*)a.x, (const E*)a.grad_y, a.phi,
                                                  w.gm, a.inv_rms, w.coef, a.pre,
                                                  (const E*)a.grad_x_acc, (E*)a.grad_x, T, D, a.x_ts,
                                                  a.gy_ts);
  MHC_LAUNCH_CHECK();
  const int ns = gphi_splits(T);
  const int64_t tps = cdiv(T, ns);
  dim3 pgrid((unsigned)cdiv(HC, kGpCC), (unsigned)ns);
  launch(pre_bwd_gphi_kernel<E, N>, pgrid, kGpCC, 0, s, (const E*)a.x, w.gm, a.inv_rms,
                                                    w.gphi_part, T, HC, tps, a.x_ts);
  MHC_LAUNCH_CHECK();
  const int64_t n = (int64_t)HM * HC;
  launch(pre_reduce_gphi_kernel, (unsigned)cdiv(n, 256), 256, 0, s, w.gphi_part, ns, n, a.grad_phi);
  MHC_LAUNCH_CHECK();
  return MHC_OK;
}

template <int N>
static int pre_bwd_n(const PreBwdArgs& a, cudaStream_t s) {
  switch (a.dtype) {
    case MHC_F32: return pre_bwd_impl<float, N>(a, s);
    case MHC_F16: return pre_bwd_impl<__half, N>(a, s);
    case MHC_BF16: return pre_bwd_impl<__nv_bfloat16, N>(a, s);
    default: return MHC_ERR_UNSUPPORTED_DTYPE;
  }
}

int pre_bwd_dispatch(const PreBwdArgs& a, cudaStream_t s) { MHC_DISPATCH_N(a.N, pre_bwd_n, a, s); }

}  // namespace mhc

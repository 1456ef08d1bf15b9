// pre_common.cuh -- argument blocks and per-token helpers of the pre operator.
#pragma once
#include "common.cuh"

namespace mhc {

struct PreFwdArgs {
  const void* x;
  const float* phi;
  const float* alpha;
  const float* base;
  int64_t T, D;
  int64_t x_ts;          // elements between consecutive tokens of x (>= N*D)
  int32_t N, dtype;
  float norm_eps;
  SmallParams sp;
  void* y;
  float* post_out;
  float* comb_frag;
  float* inv_rms;
  float* x_scaled;      // may be null
  float* mixes;
  float* h_res_logits;  // may be null
  float* pre;
  void* workspace;
  size_t workspace_bytes;
  const float* premix;    // optional: mix partials from the layer-fused post forward
  int32_t premix_layers;  // K ranges in premix
};

struct PreBwdArgs {
  const void* x;
  const float* phi;
  const float* alpha;
  const float* base;
  const float* inv_rms;
  const float* mixes;
  const float* pre;
  const void* grad_y;
  const float* grad_post;
  const float* grad_comb;
  int64_t T, D;
  int64_t x_ts, gy_ts;    // token strides of x (>= N*D) and grad_y (>= D), in elements
  int32_t N, dtype;
  SmallParams sp;
  void* grad_x;
  const void* grad_x_acc;  // optional: grad_x = this op's contribution + grad_x_acc
  float* grad_phi;
  float* grad_alpha;
  float* grad_base;
  void* workspace;
  size_t workspace_bytes;
  bool phi_prepped;  // set internally: the phi operand rows are already written
};

// Backward phi operand rows for the N = 4 tensor-core pass, item idx = 3 * column + group:
// P0 [HC][64] = [phi_hi 0..23 | phi_hi 0..23 | phi_lo 0..15], P1 [HC][16] = [phi_lo 16..23 |
// 0 x 8]; item (c, g) writes column c's entries of mixes 8g..8g+7.  sc scales phi first
// (fp16 operands; 1 for bf16).
template <typename E>
__device__ __forceinline__ void bwd_phi_prep_item(const float* __restrict__ phi,
                                                  E* __restrict__ p0, E* __restrict__ p1,
                                                  int64_t HC, float sc, int64_t idx) {
  const int64_t c = idx / 3;
  const int g = (int)(idx - c * 3);
  if (c >= HC) return;
  float hi[8], lo[8];
#pragma unroll
  for (int k = 0; k < 8; ++k) {
    const float p = phi[(int64_t)(8 * g + k) * HC + c] * sc;
    hi[k] = from_e(to_e<E>(p));
    lo[k] = p - hi[k];
  }
  uint4* d0 = reinterpret_cast<uint4*>(p0 + c * 64);
  const uint4 vh = narrow<E>(hi), vl = narrow<E>(lo);
  d0[g] = vh;
  d0[3 + g] = vh;
  if (g < 2) {
    d0[6 + g] = vl;
  } else {
    uint4* d1 = reinterpret_cast<uint4*>(p1 + c * 16);
    d1[0] = vl;
    d1[1] = make_uint4(0u, 0u, 0u, 0u);
  }
}

// a token-strided input whose every row start is aligned to A bytes
inline bool rows_aligned(const void* p, int64_t ts, size_t esize, uintptr_t A) {
  return (reinterpret_cast<uintptr_t>(p) % A) == 0 && ((uint64_t)ts * esize) % A == 0;
}

// inv_rms = rsqrt(mean(x^2) + eps) over the N*D row (src/mhc_pre_clamp_sinkhorn.py:987-988)
__device__ __forceinline__ float inv_rms_from_sumsq(float sumsq, int64_t HC, float eps) {
  const float ms = sumsq / (float)HC;
  return 1.0f / sqrtf(ms + eps);
}

// Forward small stage of one token plus the stores of its per-token outputs.
template <int N>
__device__ __forceinline__ void small_outputs(const float* mix, const float* base,
                                              const SmallParams& sp, int64_t t, float inv,
                                              float* inv_rms, float* mixes, float* pre,
                                              float* post, float* comb, float* logits_out) {
  constexpr int HM = hc_mix(N);
  float pr[N], po[N], lg[N * N], M[N * N];
  small_forward<N>(mix, base, sp, pr, po, lg, M);
  inv_rms[t] = inv;
#pragma unroll
  for (int k = 0; k < HM; ++k) mixes[t * HM + k] = mix[k];
#pragma unroll
  for (int n = 0; n < N; ++n) {
    pre[t * N + n] = pr[n];
    post[t * N + n] = po[n];
  }
#pragma unroll
  for (int e = 0; e < N * N; ++e) comb[t * N * N + e] = M[e];
  if (logits_out) {
#pragma unroll
    for (int e = 0; e < N * N; ++e) logits_out[t * N * N + e] = lg[e];
  }
}

size_t pre_fwd_ws_bytes(int64_t T, int32_t N, int64_t D, int32_t dtype);
size_t pre_bwd_ws_bytes(int64_t T, int32_t N, int64_t D, int32_t dtype, int32_t iters);
int pre_fwd_dispatch(const PreFwdArgs& a, cudaStream_t s);
int pre_bwd_dispatch(const PreBwdArgs& a, cudaStream_t s);

}  // namespace mhc

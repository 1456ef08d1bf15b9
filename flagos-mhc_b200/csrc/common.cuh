// common.cuh -- element packs, reductions and the per-token small stage
// (heads, clamp, row softmax, Sinkhorn) shared by the mHC kernels.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <utility>

#include "../../include/mhc_b200.h"

namespace mhc {

constexpr int kMaxN = 8;                       // hcMult supported: 1..8

// Elements between consecutive tokens of the token-major inputs (x: N*D when packed;
// grad_y of the post backward: N*D; h_out and grad_y of the pre backward: D).  Within a
// token the (N, D) block is contiguous.  Outputs are always packed.
struct TokStride {
  int64_t x, gy, ho;
};
__host__ __device__ constexpr int hc_mix(int n) { return n * (n + 2); }

// ---------------------------------------------------------------------------
// 16-byte packs of the storage type, widened to fp32 in registers.
// ---------------------------------------------------------------------------
template <typename E> struct Pack;
template <> struct Pack<float> { static constexpr int n = 4; };
template <> struct Pack<__half> { static constexpr int n = 8; };
template <> struct Pack<__nv_bfloat16> { static constexpr int n = 8; };

__device__ __forceinline__ float bf16_lo(uint32_t u) { return __uint_as_float(u << 16); }
__device__ __forceinline__ float bf16_hi(uint32_t u) { return __uint_as_float(u & 0xffff0000u); }

// Widen one 16-byte word.
template <typename E> __device__ __forceinline__ void widen(const uint4& v, float* f);
template <> __device__ __forceinline__ void widen<float>(const uint4& v, float* f) {
  f[0] = __uint_as_float(v.x); f[1] = __uint_as_float(v.y);
  f[2] = __uint_as_float(v.z); f[3] = __uint_as_float(v.w);
}
template <> __device__ __forceinline__ void widen<__nv_bfloat16>(const uint4& v, float* f) {
  f[0] = bf16_lo(v.x); f[1] = bf16_hi(v.x); f[2] = bf16_lo(v.y); f[3] = bf16_hi(v.y);
  f[4] = bf16_lo(v.z); f[5] = bf16_hi(v.z); f[6] = bf16_lo(v.w); f[7] = bf16_hi(v.w);
}
template <> __device__ __forceinline__ void widen<__half>(const uint4& v, float* f) {
  const __half2* h = reinterpret_cast<const __half2*>(&v);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    float2 t = __half22float2(h[i]);
    f[2 * i] = t.x; f[2 * i + 1] = t.y;
  }
}

// Narrow 16 bytes' worth of fp32 values (round to nearest even).
template <typename E> __device__ __forceinline__ uint4 narrow(const float* f);
template <> __device__ __forceinline__ uint4 narrow<float>(const float* f) {
  return make_uint4(__float_as_uint(f[0]), __float_as_uint(f[1]), __float_as_uint(f[2]),
                    __float_as_uint(f[3]));
}
template <> __device__ __forceinline__ uint4 narrow<__nv_bfloat16>(const float* f) {
  uint4 r;
  __nv_bfloat162 t;
  t = __floats2bfloat162_rn(f[0], f[1]); r.x = *reinterpret_cast<uint32_t*>(&t);
  t = __floats2bfloat162_rn(f[2], f[3]); r.y = *reinterpret_cast<uint32_t*>(&t);
  t = __floats2bfloat162_rn(f[4], f[5]); r.z = *reinterpret_cast<uint32_t*>(&t);
  t = __floats2bfloat162_rn(f[6], f[7]); r.w = *reinterpret_cast<uint32_t*>(&t);
  return r;
}
template <> __device__ __forceinline__ uint4 narrow<__half>(const float* f) {
  uint4 r;
  __half2 t;
  t = __floats2half2_rn(f[0], f[1]); r.x = *reinterpret_cast<uint32_t*>(&t);
  t = __floats2half2_rn(f[2], f[3]); r.y = *reinterpret_cast<uint32_t*>(&t);
  t = __floats2half2_rn(f[4], f[5]); r.z = *reinterpret_cast<uint32_t*>(&t);
  t = __floats2half2_rn(f[6], f[7]); r.w = *reinterpret_cast<uint32_t*>(&t);
  return r;
}

// Scalar element access (ragged D / unaligned fallback).
template <typename E> __device__ __forceinline__ float ld1(const E* p);
template <> __device__ __forceinline__ float ld1<float>(const float* p) { return __ldg(p); }
template <> __device__ __forceinline__ float ld1<__half>(const __half* p) { return __half2float(__ldg(p)); }
template <> __device__ __forceinline__ float ld1<__nv_bfloat16>(const __nv_bfloat16* p) {
  return __bfloat162float(__ldg(p));
}
template <typename E> __device__ __forceinline__ void st1(E* p, float v);
template <> __device__ __forceinline__ void st1<float>(float* p, float v) { *p = v; }
template <> __device__ __forceinline__ void st1<__half>(__half* p, float v) { *p = __float2half_rn(v); }
template <> __device__ __forceinline__ void st1<__nv_bfloat16>(__nv_bfloat16* p, float v) {
  *p = __float2bfloat16_rn(v);
}

// Read-once 16-byte load (bypasses L1, evict-first in L2).
__device__ __forceinline__ uint4 ld_stream(const void* p) {
  return __ldcs(reinterpret_cast<const uint4*>(p));
}
__device__ __forceinline__ uint4 ld_keep(const void* p) {
  return __ldg(reinterpret_cast<const uint4*>(p));
}
__device__ __forceinline__ void st_stream(void* p, const uint4& v) {
  __stcs(reinterpret_cast<uint4*>(p), v);
}

// Load P elements (P = Pack<E>::n when VEC, else 1 per call site loop).
template <typename E, bool VEC>
__device__ __forceinline__ void load_pack(const E* p, float* f) {
  if constexpr (VEC) {
    widen<E>(ld_stream(p), f);
  } else {
    f[0] = ld1<E>(p);
  }
}
template <typename E, bool VEC>
__device__ __forceinline__ void store_pack(E* p, const float* f) {
  if constexpr (VEC) {
    st_stream(p, narrow<E>(f));
  } else {
    st1<E>(p, f[0]);
  }
}

// 32-byte global accesses (sm_100): a thread that owns one row writes whole 32-byte
// sectors, halving the memory requests of row-per-thread epilogues.
struct alignas(32) U8 {
  uint4 a, b;
};
__device__ __forceinline__ void st_global_32B(void* p, const uint4& a, const uint4& b) {
  asm volatile("st.global.cs.v8.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8};" ::"l"(p), "r"(a.x),
               "r"(a.y), "r"(a.z), "r"(a.w), "r"(b.x), "r"(b.y), "r"(b.z), "r"(b.w)
               : "memory");
}
__device__ __forceinline__ void prefetch_l2(const void* p) {
  asm volatile("prefetch.global.L2 [%0];" ::"l"(p));
}
__device__ __forceinline__ U8 ld_global_32B(const void* p) {
  U8 v;
  asm volatile("ld.global.cs.v8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
               : "=r"(v.a.x), "=r"(v.a.y), "=r"(v.a.z), "=r"(v.a.w), "=r"(v.b.x), "=r"(v.b.y),
                 "=r"(v.b.z), "=r"(v.b.w)
               : "l"(p));
  return v;
}

// Compensated (Kahan) summation: s + c carries the running sum with the low-order bits
// that s alone would drop.  Every fixed-order partial reduction of the parameter
// gradients (grad_phi, grad_alpha, grad_base) goes through it.
struct Kahan {
  float s = 0.f, c = 0.f;
  __device__ __forceinline__ void add(float v) {
    const float y = v - c;
    const float t = s + y;
    c = (t - s) - y;
    s = t;
  }
};
__device__ __forceinline__ float4 kahan_add4(Kahan* k, float4 v) {
  k[0].add(v.x); k[1].add(v.y); k[2].add(v.z); k[3].add(v.w);
  return make_float4(k[0].s, k[1].s, k[2].s, k[3].s);
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// 16-bit element conversions (round to nearest even)
template <typename E> __device__ __forceinline__ E to_e(float v);
template <> __device__ __forceinline__ __nv_bfloat16 to_e<__nv_bfloat16>(float v) {
  return __float2bfloat16_rn(v);
}
template <> __device__ __forceinline__ __half to_e<__half>(float v) { return __float2half_rn(v); }
__device__ __forceinline__ float from_e(__nv_bfloat16 v) { return __bfloat162float(v); }
__device__ __forceinline__ float from_e(__half v) { return __half2float(v); }

// fp16 tensor-core operands: values are multiplied by 2^s before their hi/lo split, with
// 2^s chosen from their maximum magnitude (bits of a non-negative float) so that the
// maximum stays below 2^14: the hi halves stay finite and the lo halves normal.
__device__ __forceinline__ float f16_operand_scale(unsigned max_bits) {
  const float m = __uint_as_float(max_bits);
  if (!(m > 0.f) || !isfinite(m)) return 1.f;
  int e;
  frexpf(m, &e);  // m < 2^e
  return ldexpf(1.f, 14 - e);
}

// v with the low 13 mantissa bits cleared: the part of an fp32 operand kind::tf32 uses.
__device__ __forceinline__ float tf32_hi(float v) {
  return __uint_as_float(__float_as_uint(v) & 0xffffe000u);
}

__device__ __forceinline__ float sigmoidf_(float z) { return 1.0f / (1.0f + expf(-z)); }

// ---------------------------------------------------------------------------
// Per-token small stage, forward (one thread owns one token).
// Follows src/mhc_pre_clamp_sinkhorn.py:995-1010:
//   pre  = sigmoid(mix[:N]*a0 + b[:N]) + eps
//   post = 2*sigmoid(mix[N:2N]*a1 + b[N:2N])
//   l    = mix[2N:]*a2 + b[2N:]     (row-major N x N)
//   P = softmax_row(clamp(l)); M = P + eps; M /= colsum + eps;
//   (iters-1) x { M /= rowsum + eps; M /= colsum + eps }
// ---------------------------------------------------------------------------
struct SmallParams {
  float a0, a1, a2;
  float hc_eps;
  float clamp_min, clamp_max;
  int clamp_on;
  int iters;
};

template <int N>
__device__ __forceinline__ void softmax_rows(const float* l, float* P) {
#pragma unroll
  for (int i = 0; i < N; ++i) {
    float m = l[i * N];
#pragma unroll
    for (int j = 1; j < N; ++j) m = fmaxf(m, l[i * N + j]);
    float s = 0.f;
#pragma unroll
    for (int j = 0; j < N; ++j) {
      P[i * N + j] = expf(l[i * N + j] - m);
      s += P[i * N + j];
    }
    const float rs = 1.0f / s;
#pragma unroll
    for (int j = 0; j < N; ++j) P[i * N + j] *= rs;
  }
}

// Normalisations divide by (sum + eps) through one reciprocal per row / column, as the
// reference's own kernels do (`inv_s = 1/(s+eps)` then multiply); rc_out receives the
// reciprocals when the caller needs them for the backward.
template <int N>
__device__ __forceinline__ void col_norm(float* M, float eps, float* rc_out = nullptr) {
#pragma unroll
  for (int j = 0; j < N; ++j) {
    float c = 0.f;
#pragma unroll
    for (int i = 0; i < N; ++i) c += M[i * N + j];
    const float rc = 1.0f / (c + eps);
    if (rc_out) rc_out[j] = rc;
#pragma unroll
    for (int i = 0; i < N; ++i) M[i * N + j] *= rc;
  }
}

template <int N>
__device__ __forceinline__ void row_norm(float* M, float eps, float* rr_out = nullptr) {
#pragma unroll
  for (int i = 0; i < N; ++i) {
    float r = 0.f;
#pragma unroll
    for (int j = 0; j < N; ++j) r += M[i * N + j];
    const float rr = 1.0f / (r + eps);
    if (rr_out) rr_out[i] = rr;
#pragma unroll
    for (int j = 0; j < N; ++j) M[i * N + j] *= rr;
  }
}

// logits (pre-clamp) and P = softmax(clamp(logits)) from the mixes of one token.
template <int N>
__device__ __forceinline__ void logits_softmax(const float* mix, const float* base,
                                               const SmallParams& sp, float* logits,
                                               float* P) {
  float lc[N * N];
#pragma unroll
  for (int e = 0; e < N * N; ++e) {
    float l = mix[2 * N + e] * sp.a2 + base[2 * N + e];
    logits[e] = l;
    lc[e] = sp.clamp_on ? fminf(fmaxf(l, sp.clamp_min), sp.clamp_max) : l;
  }
  softmax_rows<N>(lc, P);
}

// Full forward of the small stage for one token.
template <int N>
__device__ __forceinline__ void small_forward(const float* mix, const float* base,
                                              const SmallParams& sp, float* pre, float* post,
                                              float* logits, float* M) {
#pragma unroll
  for (int n = 0; n < N; ++n) {
    pre[n] = sigmoidf_(mix[n] * sp.a0 + base[n]) + sp.hc_eps;
    post[n] = 2.0f * sigmoidf_(mix[N + n] * sp.a1 + base[N + n]);
  }
  logits_softmax<N>(mix, base, sp, logits, M);
#pragma unroll
  for (int e = 0; e < N * N; ++e) M[e] += sp.hc_eps;
  col_norm<N>(M, sp.hc_eps);
  for (int it = 1; it < sp.iters; ++it) {
    row_norm<N>(M, sp.hc_eps);
    col_norm<N>(M, sp.hc_eps);
  }
}

// ---------------------------------------------------------------------------
// Status plumbing shared by the host launchers.
// ---------------------------------------------------------------------------
#define MHC_CUDA_CHECK(expr)                                        \
  do {                                                              \
    cudaError_t _e = (expr);                                        \
    if (_e != cudaSuccess) return MHC_ERR_CUDA;                     \
  } while (0)

// Every kernel launch is followed by this check; it also counts the launch
// (mhc_kernel_launches() in the C ABI reports the running total).
#define MHC_LAUNCH_CHECK()                                          \
  do {                                                              \
    cudaError_t _e = cudaGetLastError();                            \
    if (_e != cudaSuccess) return MHC_ERR_CUDA;                     \
    ::mhc::note_launch();                                           \
  } while (0)

void note_launch();

// ---------------------------------------------------------------------------
// Programmatic dependent launch.  Every kernel of this library is launched with
// cudaLaunchAttributeProgrammaticStreamSerialization, so its CTAs may become
// resident while the previous kernel on the stream is still finishing (its last
// wave); each kernel runs only set-up that reads no global memory (shared-memory
// carve-up, mbarrier init, TMEM allocation, tensor-map prefetch) before
// pdl_wait(), which returns once the previous grid has completed and its writes
// are visible.  pdl_trigger() (issued by every CTA right after its pdl_wait())
// lets the next kernel launch as soon as all CTAs of this one are running.
// Without the attribute (or with no kernel in flight before it) both are no-ops.
// ---------------------------------------------------------------------------
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}
__device__ __forceinline__ void pdl_enter() {
  pdl_wait();
  pdl_trigger();
}

// MHC_PDL=0 in the environment launches without the attribute (A/B measurements).
bool pdl_enabled();
// Each entry point calls pdl_new_call() before its first launch; that launch then goes
// without the attribute, so PDL links the kernels of one call only.
void pdl_new_call();
bool pdl_first_launch();

template <typename... KArgs, typename... Args>
inline cudaError_t launch(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem,
                          cudaStream_t stream, Args&&... args) {
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cfg.attrs = attr;
  cfg.numAttrs = (!pdl_first_launch() && pdl_enabled()) ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

#define MHC_DISPATCH_N(N_, FN, ...)                          \
  switch (N_) {                                              \
    case 1: return FN<1>(__VA_ARGS__);                       \
    case 2: return FN<2>(__VA_ARGS__);                       \
    case 3: return FN<3>(__VA_ARGS__);                       \
    case 4: return FN<4>(__VA_ARGS__);                       \
    case 5: return FN<5>(__VA_ARGS__);                       \
    case 6: return FN<6>(__VA_ARGS__);                       \
    case 7: return FN<7>(__VA_ARGS__);                       \
    case 8: return FN<8>(__VA_ARGS__);                       \
    default: return MHC_ERR_UNSUPPORTED_N;                   \
  }

int sm_count();  // multiprocessors of the current device (cached per device)

inline int64_t cdiv(int64_t a, int64_t b) { return (a + b - 1) / b; }
inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }
inline size_t align_up(size_t n, size_t a = 256) { return (n + a - 1) / a * a; }

}  // namespace mhc

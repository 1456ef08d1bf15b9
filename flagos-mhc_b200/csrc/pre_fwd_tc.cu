// pre_fwd_tc.cu -- mhc_pre_clamp_sinkhorn forward, tensor-core path (bf16 x).
//
// pre_phi_split_kernel   phi (fp32) -> phi_hl (bf16) [NP x HC]: rows [0,HM) = hi,
//                        rows [HM,2HM) = lo = phi - hi, rows beyond = 0.  x is exact in
//                        bf16, so x.phi^T = x.hi^T + x.lo^T in fp32 accumulation
//                        reproduces the fp32 contraction to ~2^-17 per product.
// pre_mix_tc_kernel      persistent, one 128-token tile at a time:
//                          warp 0     TMA producer: x tile [128 x 64*NB] + phi_hl
//                                     [NP x 64*NB] per stage into an S-stage ring (NB
//                                     adjacent 128B-swizzled boxes per stage)
//                          warp 1     TMEM owner + MMA issuer: tcgen05.mma M=128 N=NP
//                                     K=16 x4 per stage; accumulation in K segments of
//                                     KSEG stages, double-buffered in TMEM
//                          warps 2-5  sum of squares of their token row from the staged
//                                     x tile (same pass over x), the fp32 sum of the
//                                     segment partials (hi+lo) from TMEM, then inv_rms,
//                                     mixes, heads, clamp, softmax, Sinkhorn and the
//                                     stores of the per-token outputs
// x is read from HBM once here; pre_apply_kernel (pre_fwd.cu) reads it once more for
// y and x_scaled, which need inv_rms / pre of the whole row first.
#include "pre_common.cuh"
#include "tc.cuh"

namespace mhc {

template <int N, int NB>
struct MixCfg {
  static constexpr int HM = hc_mix(N);
  static constexpr int NP = (2 * HM + 15) / 16 * 16;            // MMA N (hi + lo rows)
  static constexpr int BUFCOL = (NP + 16 + 31) / 32 * 32;       // TMEM columns per buffer
  static constexpr int TMEM_COLS = (2 * BUFCOL <= 32) ? 32 : (2 * BUFCOL <= 64) ? 64
                                   : (2 * BUFCOL <= 128) ? 128 : (2 * BUFCOL <= 256) ? 256 : 512;
  static constexpr int BOX = 64;                                 // columns per TMA box (128 B)
  static constexpr int KC = BOX * NB;                            // K per stage: NB adjacent boxes
  // Stages per TMEM segment.  The tensor core's fp32 accumulation loses precision
  // roughly in proportion to the number of chained MMAs; folding every 64 MMAs into
  // fp32 registers keeps x.phi^T within a few 1e-6 of the fp32 contraction at any K.
  static constexpr int KSEG = 16 / NB;                           // stages per segment (64 MMAs)
  static constexpr int A_BOX = 128 * BOX * 2;                   // 16 KB
  static constexpr int A_BYTES = A_BOX * NB;
  static constexpr int B_BOX = NP * BOX * 2;
  static constexpr int B_BOX_STRIDE = (B_BOX + 1023) / 1024 * 1024;
  static constexpr int B_BYTES = B_BOX * NB;                     // TMA bytes per stage
  static constexpr int B_STRIDE = B_BOX_STRIDE * NB;
  static constexpr int STAGES = (200 * 1024) / (A_BYTES + B_STRIDE) > 8
                                    ? 8 : (200 * 1024) / (A_BYTES + B_STRIDE);
  static constexpr int SMEM = 1024 /*align slack*/ + STAGES * (A_BYTES + B_STRIDE) + 256;
  static constexpr int THREADS = 192;
};

// fp32 x (kind::tf32): the tensor core reads the top 19 bits of an fp32 operand (sign,
// exponent, 10 mantissa bits).  x is used as stored, so the MMA sees x_hi = x with the low
// 13 mantissa bits cleared; the sum-of-squares warps write x_lo = x - x_hi (exact in fp32)
// into a second buffer of the stage.  phi is split the same way into rows [phi_hi;
// phi_lo] (pre_phi_split_tf32_kernel), and D = x_hi.[phi_hi;phi_lo]^T + x_lo.[phi_hi;
// phi_lo]^T, so columns [0,HM) + [HM,2HM) hold x.phi^T up to the tf32 rounding of the
// lo parts (~2^-21 relative per product).
template <int N, int NB, typename E>
struct MixCfgE : MixCfg<N, NB> {
  static constexpr bool F32 = false;
  static constexpr int XL_BYTES = 0;
};
template <int N, int NB>
struct MixCfgE<N, NB, float> {
  static constexpr bool F32 = true;
  static constexpr int HM = hc_mix(N);
  static constexpr int NP = (2 * HM + 15) / 16 * 16;
  static constexpr int BUFCOL = (NP + 16 + 31) / 32 * 32;
  static constexpr int TMEM_COLS = (2 * BUFCOL <= 32) ? 32 : (2 * BUFCOL <= 64) ? 64
                                   : (2 * BUFCOL <= 128) ? 128 : (2 * BUFCOL <= 256) ? 256 : 512;
  static constexpr int BOX = 32;                                 // fp32 columns per box (128 B)
  static constexpr int KC = BOX * NB;
  static constexpr int KSEG = 8 / NB;                            // 64 MMAs per segment
  static constexpr int A_BOX = 128 * BOX * 4;                    // 16 KB
  static constexpr int A_BYTES = A_BOX * NB;
  static constexpr int XL_BYTES = A_BYTES;
  static constexpr int B_BOX = NP * BOX * 4;
  static constexpr int B_BOX_STRIDE = (B_BOX + 1023) / 1024 * 1024;
  static constexpr int B_BYTES = B_BOX * NB;
  static constexpr int B_STRIDE = B_BOX_STRIDE * NB;
  static constexpr int STAGES = (200 * 1024) / (2 * A_BYTES + B_STRIDE) > 8
                                    ? 8 : (200 * 1024) / (2 * A_BYTES + B_STRIDE);
  static constexpr int SMEM = 1024 + STAGES * (2 * A_BYTES + B_STRIDE) + 256;
  static constexpr int THREADS = 192;
};

// phi (fp32 [HM][HC]) -> [NP][HC] fp32 rows for kind::tf32: [0,HM) = phi with the low 13
// mantissa bits cleared, [HM,2HM) = the remainder, the rest 0.  Vectorised: HC % 4 == 0.
__global__ void pre_phi_split_tf32_kernel(const float* __restrict__ phi, float* __restrict__ hl,
                                          int HM, int NP, int64_t HC) {
  pdl_enter();
  const int r = blockIdx.y;
  const int64_t n4 = HC / 4;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  float4* dhi = reinterpret_cast<float4*>(hl + (int64_t)r * HC);
  if (r < HM) {
    const float4* src = reinterpret_cast<const float4*>(phi + (int64_t)r * HC);
    float4* dlo = reinterpret_cast<float4*>(hl + (int64_t)(HM + r) * HC);
    for (int64_t j = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; j < n4; j += stride) {
      const float4 a = __ldg(src + j);
      const float4 h = make_float4(tf32_hi(a.x), tf32_hi(a.y), tf32_hi(a.z), tf32_hi(a.w));
      dhi[j] = h;
      dlo[j] = make_float4(a.x - h.x, a.y - h.y, a.z - h.z, a.w - h.w);
    }
  } else if (r >= 2 * HM) {
    for (int64_t j = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; j < n4; j += stride)
      dhi[j] = make_float4(0.f, 0.f, 0.f, 0.f);
  }
}

// fp16 operands (x fp16): phi is split after scaling by 2^s so that max|phi| * 2^s < 2^14,
// keeping the lo halves out of fp16's subnormal range and the hi halves finite; the mix
// is multiplied by 2^-s afterwards (exact).  This kernel finds max|phi| (the bit patterns
// of non-negative floats order like the floats).
__global__ void pre_phi_maxabs_kernel(const float* __restrict__ phi, int64_t n,
                                      unsigned* __restrict__ slot) {
  pdl_enter();
  float m = 0.f;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x)
    m = fmaxf(m, fabsf(phi[i]));
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
  if ((threadIdx.x & 31) == 0) atomicMax(slot, __float_as_uint(m));
}

// phi (fp32) -> phi_hl [NP x HC] in E: rows [0,HM) = hi, [HM,2HM) = lo = phi - hi, rest 0.
// maxslot == nullptr: no scaling (bf16's exponent range is fp32's).
template <typename E>
__global__ void pre_phi_split_kernel(const float* __restrict__ phi, E* __restrict__ hl, int HM,
                                     int NP, int64_t HC, const unsigned* __restrict__ maxslot,
                                     float* __restrict__ descale) {
  pdl_enter();
  float scale = 1.f;
  if (maxslot != nullptr) {
    scale = f16_operand_scale(*maxslot);
    if (blockIdx.x == 0 && threadIdx.x == 0) *descale = 1.f / scale;
  }
  const int64_t n = (int64_t)NP * HC;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = i / HC, c = i - r * HC;
    float v = 0.f;
    if (r < HM) {
      v = phi[r * HC + c] * scale;
    } else if (r < 2 * HM) {
      const float p = phi[(r - HM) * HC + c] * scale;
      v = p - from_e(to_e<E>(p));
    }
    hl[i] = to_e<E>(v);
  }
}

// Vectorised split for HC % 8 == 0: blockIdx.y = source row r < HM (writes hi row r and
// lo row HM + r, 8 columns per thread and step) or one of the zero rows [2HM, NP).
template <typename E>
__global__ void pre_phi_split8_kernel(const float* __restrict__ phi, E* __restrict__ hl, int HM,
                                      int NP, int64_t HC, const unsigned* __restrict__ maxslot,
                                      float* __restrict__ descale) {
  pdl_enter();
  float scale = 1.f;
  if (maxslot != nullptr) {
    scale = f16_operand_scale(*maxslot);
    if (blockIdx.x == 0 && blockIdx.y == 0 && threadIdx.x == 0) *descale = 1.f / scale;
  }
  const int r = blockIdx.y;
  const int64_t n8 = HC / 8;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  if (r < HM) {
    const float4* src = reinterpret_cast<const float4*>(phi + (int64_t)r * HC);
    uint4* dhi = reinterpret_cast<uint4*>(hl + (int64_t)r * HC);
    uint4* dlo = reinterpret_cast<uint4*>(hl + (int64_t)(HM + r) * HC);
    for (int64_t j = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; j < n8; j += stride) {
      const float4 a = __ldg(src + 2 * j), b = __ldg(src + 2 * j + 1);
      float p[8] = {a.x * scale, a.y * scale, a.z * scale, a.w * scale,
                    b.x * scale, b.y * scale, b.z * scale, b.w * scale};
      float lo[8];
#pragma unroll
      for (int k = 0; k < 8; ++k) lo[k] = p[k] - from_e(to_e<E>(p[k]));
      dhi[j] = narrow<E>(p);
      dlo[j] = narrow<E>(lo);
    }
  } else {
    uint4* dz = reinterpret_cast<uint4*>(hl + (int64_t)(HM + r) * HC);  // rows 2HM .. NP-1
    for (int64_t j = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; j < n8; j += stride)
      dz[j] = make_uint4(0u, 0u, 0u, 0u);
  }
}

template <int N, int NB, typename E>
__global__ void __launch_bounds__(MixCfg<N, NB>::THREADS, 1)
pre_mix_tc_kernel(const __grid_constant__ CUtensorMap tm_x,
                  const __grid_constant__ CUtensorMap tm_phi, const float* __restrict__ alpha,
                  const float* __restrict__ base, int64_t T, int64_t HC, float norm_eps,
                  SmallParams sp, float* __restrict__ inv_rms, float* __restrict__ mixes,
                  float* __restrict__ pre, float* __restrict__ post, float* __restrict__ comb,
                  float* __restrict__ logits_out, int ksplit, float* __restrict__ part,
                  const float* __restrict__ descale) {
  pdl_enter();
  using C = MixCfgE<N, NB, E>;
  constexpr int HM = C::HM, S = C::STAGES;
  constexpr bool F32 = C::F32;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = (uint8_t*)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
  uint8_t* sA = smem;
  uint8_t* sB = smem + S * C::A_BYTES;
  uint8_t* sXL = sB + S * C::B_STRIDE;  // fp32: x_lo of each stage
  uint64_t* full = (uint64_t*)(sXL + S * C::XL_BYTES);
  uint64_t* empty = full + S;
  uint64_t* xready = empty + S;         // fp32: the stage's x_lo is written
  uint64_t* tfull = xready + S;
  uint64_t* tempty = tfull + 2;
  uint64_t* tdone = tempty + 2;
  uint32_t* tmem_slot = (uint32_t*)(tdone + 1);
  volatile int* abort_flag = (volatile int*)(tmem_slot + 1);
  __shared__ float sbase[HM];

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t ntiles = (T + 127) / 128;
  const int nk = (int)((HC + C::KC - 1) / C::KC);

  for (int i = threadIdx.x; i < HM; i += blockDim.x) sbase[i] = base[i];
  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      tc::mbar_init(&full[s], 1);
      tc::mbar_init(&empty[s], 1 + 4);
      tc::mbar_init(&xready[s], 4);
    }
    for (int b = 0; b < 2; ++b) {
      tc::mbar_init(&tfull[b], 1);
      tc::mbar_init(&tempty[b], 4);
    }
    tc::mbar_init(tdone, 1);
    *abort_flag = 0;
    tc::fence_barrier_init();
  }
  if (warp == 0 && lane == 0) {
    tc::prefetch_tmap(&tm_x);
    tc::prefetch_tmap(&tm_phi);
  }
  if (warp == 1) {
    tc::tmem_alloc(tmem_slot, C::TMEM_COLS);
    tc::tmem_relinquish();
  }
  tc::tc_fence_before();
  __syncthreads();
  tc::tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    // ------------------------------------------------------------ TMA producer
    if (lane == 0) {
      uint32_t it = 0;
      bool ok = true;
      const uint64_t pol_stream = tc::l2_evict_first(), pol_keep = tc::l2_evict_last();
      for (int64_t u = blockIdx.x; u < ntiles * ksplit && ok; u += gridDim.x) {
        const int64_t tile = u / ksplit;
        const int spl = (int)(u - tile * ksplit);
        const int kcb = (int)((int64_t)nk * spl / ksplit), kce = (int)((int64_t)nk * (spl + 1) / ksplit);
        for (int kc = kcb; kc < kce; ++kc, ++it) {
          const int s = it % S;
          const uint32_t ph = (it / S) & 1;
          if (!tc::mbar_wait(&empty[s], ph ^ 1, abort_flag)) { ok = false; break; }
          tc::mbar_arrive_expect_tx(&full[s], C::A_BYTES + C::B_BYTES);
#pragma unroll
          for (int b = 0; b < NB; ++b) {
            const int col = kc * C::KC + b * C::BOX;
            tc::tma_load_2d_hint(sA + s * C::A_BYTES + b * C::A_BOX, &tm_x, &full[s], col,
                                 (int)(tile * 128), pol_stream);
            tc::tma_load_2d_hint(sB + s * C::B_STRIDE + b * C::B_BOX_STRIDE, &tm_phi, &full[s],
                                 col, 0, pol_keep);
          }
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t idesc = F32 ? tc::idesc_tf32(128, C::NP, false, false)
                                     : tc::idesc_16<E>(128, C::NP, false, false);
      uint32_t it = 0, j = 0;
      bool ok = true;
      for (int64_t u = blockIdx.x; u < ntiles * ksplit && ok; u += gridDim.x) {
        const int64_t tile = u / ksplit;
        const int spl = (int)(u - tile * ksplit);
        const int kcb = (int)((int64_t)nk * spl / ksplit), kce = (int)((int64_t)nk * (spl + 1) / ksplit);
        (void)tile;
        for (int kc0 = kcb; kc0 < kce && ok; kc0 += C::KSEG, ++j) {
          const int buf = j & 1;
          if (!tc::mbar_wait(&tempty[buf], ((j >> 1) & 1) ^ 1, abort_flag)) { ok = false; break; }
          tc::tc_fence_after();
          const uint32_t d = tmem + buf * C::BUFCOL;
          const int kc1 = kc0 + C::KSEG < kce ? kc0 + C::KSEG : kce;
          for (int kc = kc0; kc < kc1; ++kc, ++it) {
            const int s = it % S;
            if (!tc::mbar_wait(&full[s], (it / S) & 1, abort_flag)) { ok = false; break; }
            if (F32 && !tc::mbar_wait(&xready[s], (it / S) & 1, abort_flag)) { ok = false; break; }
            tc::tc_fence_after();
#pragma unroll
            for (int b = 0; b < NB; ++b) {
              const uint64_t a0 = tc::smem_desc(
                  tc::smem_u32(sA + s * C::A_BYTES + b * C::A_BOX), 16, 1024, tc::kSwizzle128);
              const uint64_t b0 = tc::smem_desc(
                  tc::smem_u32(sB + s * C::B_STRIDE + b * C::B_BOX_STRIDE), 16, 1024,
                  tc::kSwizzle128);
              if constexpr (F32) {
                const uint64_t l0 = tc::smem_desc(
                    tc::smem_u32(sXL + s * C::XL_BYTES + b * C::A_BOX), 16, 1024,
                    tc::kSwizzle128);
#pragma unroll
                for (int k = 0; k < C::BOX / 8; ++k) {  // K = 8 tf32 (32 B) per MMA
                  tc::mma_tf32(d, a0 + 2 * k, b0 + 2 * k, idesc,
                               (kc != kc0 || b != 0 || k != 0) ? 1u : 0u);
                  tc::mma_tf32(d, l0 + 2 * k, b0 + 2 * k, idesc, 1u);
                }
              } else {
#pragma unroll
                for (int k = 0; k < C::BOX / 16; ++k)
                  tc::mma_bf16(d, a0 + 2 * k, b0 + 2 * k, idesc,
                               (kc != kc0 || b != 0 || k != 0) ? 1u : 0u);
              }
            }
            tc::mma_commit(&empty[s]);
          }
          if (!ok) break;
          tc::mma_commit(&tfull[buf]);
        }
      }
      // all MMAs of this CTA have completed before TMEM is released
      tc::mma_commit(tdone);
      volatile int never = 0;
      tc::mbar_wait(tdone, 0, &never);
    }
  } else {
    // ------------------------------------------------------------ sumsq + epilogue
    const int q = warp & 3;             // TMEM lane quarter this warp may access
    const int r = q * 32 + lane;        // token row within the tile
    sp.a0 = alpha[0]; sp.a1 = alpha[1]; sp.a2 = alpha[2];
    const uint32_t tq = tmem + ((uint32_t)(q * 32) << 16);
    uint32_t it = 0, j = 0;
    for (int64_t u = blockIdx.x; u < ntiles * ksplit; u += gridDim.x) {
      const int64_t tile = u / ksplit;
      const int spl = (int)(u - tile * ksplit);
      const int kcb = (int)((int64_t)nk * spl / ksplit), kce = (int)((int64_t)nk * (spl + 1) / ksplit);
      float sq = 0.f;
      float mix[HM];
#pragma unroll
      for (int k = 0; k < HM; ++k) mix[k] = 0.f;
      bool ok = true;
      for (int kc = kcb; kc < kce; ++kc, ++it) {
        const int s = it % S;
        if (!__all_sync(0xffffffffu, tc::mbar_wait(&full[s], (it / S) & 1, abort_flag))) {
          ok = false;
          break;
        }
        float csq = 0.f;
        constexpr int EPC = 16 / (int)sizeof(E);  // elements per 16-byte chunk
#pragma unroll
        for (int bc = 0; bc < 8 * NB; ++bc) {
          const uint4* row =
              reinterpret_cast<const uint4*>(sA + s * C::A_BYTES + (bc >> 3) * C::A_BOX + r * 128);
          const int c = bc & 7;
          // visit the row's 16-byte chunks in swizzled order: the 8 rows of an atom then
          // hit 8 different bank groups (a plain c order is a 32-way bank conflict)
          const uint4 v = row[c ^ (r & 7)];
          float f[EPC];
          widen<E>(v, f);
#pragma unroll
          for (int e = 0; e < EPC; ++e) csq = fmaf(f[e], f[e], csq);
          if constexpr (F32) {
            uint4* lrow = reinterpret_cast<uint4*>(sXL + s * C::XL_BYTES + (bc >> 3) * C::A_BOX +
                                                   r * 128);
            lrow[c ^ (r & 7)] = make_uint4(__float_as_uint(f[0] - tf32_hi(f[0])),
                                           __float_as_uint(f[1] - tf32_hi(f[1])),
                                           __float_as_uint(f[2] - tf32_hi(f[2])),
                                           __float_as_uint(f[3] - tf32_hi(f[3])));
          }
        }
        sq += csq;
        // the stage is refilled by TMA (async proxy): order these generic-proxy reads
        // (and, fp32, the x_lo writes the MMAs read) before that, then release the stage
        tc::fence_proxy_async();
        __syncwarp();
        if (lane == 0) {
          if constexpr (F32) tc::mbar_arrive(&xready[s]);
          tc::mbar_arrive(&empty[s]);
        }
        if ((kc - kcb + 1) % C::KSEG == 0 || kc + 1 == kce) {
          // end of a K segment: fold its TMEM partial (hi + lo rows) into registers
          const int buf = j & 1;
          if (!__all_sync(0xffffffffu, tc::mbar_wait(&tfull[buf], (j >> 1) & 1, abort_flag))) {
            ok = false;
            break;
          }
          tc::tc_fence_after();
          const uint32_t taddr = tq + buf * C::BUFCOL;
#pragma unroll
          for (int k0 = 0; k0 < HM; k0 += 16) {
            float hi[16], lo[16];
            tc::tmem_ld16(taddr + k0, hi);
            tc::tmem_ld16(taddr + HM + k0, lo);
            tc::tmem_ld_wait();
#pragma unroll
            for (int e = 0; e < 16; ++e)
              if (k0 + e < HM) mix[k0 + e] += hi[e] + lo[e];
          }
          tc::tc_fence_before();
          __syncwarp();
          if (lane == 0) tc::mbar_arrive(&tempty[buf]);
          ++j;
        }
      }
      if (!ok) break;
      const int64_t t = tile * 128 + r;
      if (part != nullptr) {
        // split K (few tiles): this K range's partial sums; pre_mix_finish_kernel adds
        // the ranges in order and runs the small stage
        if (t < T) {
          float* dst = part + ((int64_t)spl * T + t) * (HM + 1);
#pragma unroll
          for (int k = 0; k < HM; ++k) dst[k] = mix[k];
          dst[HM] = sq;
        }
      } else if (t < T) {
        const float inv = inv_rms_from_sumsq(sq, HC, norm_eps);
        const float sc = descale ? inv * *descale : inv;  // descale: an exact power of two
#pragma unroll
        for (int k = 0; k < HM; ++k) mix[k] *= sc;
        small_outputs<N>(mix, sbase, sp, t, inv, inv_rms, mixes, pre, post, comb, logits_out);
      }
    }
  }
  if (*abort_flag && threadIdx.x == 0) flag_timeout();
  tc::tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc::tc_fence_after();
    tc::tmem_dealloc(tmem, C::TMEM_COLS);
  }
}

// One token's forward small stage on a group of N lanes of a warp (N a power of two):
// lane n of the group owns row n of the N x N matrices; mrow = (mix[n], mix[N+n],
// mix[2N+nN .. 2N+nN+N-1]), already scaled by inv_rms.  Column sums are gathered by
// shuffles and added in row order, so the operations are those of small_forward in the
// same order, with a chain N times shorter.  All 32 lanes call it (valid == false:
// nothing is stored).
template <int N>
__device__ __forceinline__ void small_rows_outputs(const float* mrow, float inv,
                                                   const float* base, const SmallParams& sp,
                                                   int n, int64_t t, bool valid, int g0,
                                                   float* inv_rms, float* mixes, float* pre,
                                                   float* post, float* comb, float* logits_out) {
  constexpr int HM = hc_mix(N);
  const float pr = sigmoidf_(mrow[0] * sp.a0 + base[n]) + sp.hc_eps;
  const float po = 2.0f * sigmoidf_(mrow[1] * sp.a1 + base[N + n]);
  float l[N], M[N];
#pragma unroll
  for (int j = 0; j < N; ++j) {
    l[j] = mrow[2 + j] * sp.a2 + base[2 * N + n * N + j];
    M[j] = sp.clamp_on ? fminf(fmaxf(l[j], sp.clamp_min), sp.clamp_max) : l[j];
  }
  float m = M[0];
#pragma unroll
  for (int j = 1; j < N; ++j) m = fmaxf(m, M[j]);
  float s = 0.f;
#pragma unroll
  for (int j = 0; j < N; ++j) {
    M[j] = expf(M[j] - m);
    s += M[j];
  }
  const float rs = 1.0f / s;
#pragma unroll
  for (int j = 0; j < N; ++j) M[j] *= rs;
#pragma unroll
  for (int j = 0; j < N; ++j) M[j] += sp.hc_eps;
  auto col_norm_rows = [&]() {
#pragma unroll
    for (int j = 0; j < N; ++j) {
      float v[N];
#pragma unroll
      for (int i = 0; i < N; ++i) v[i] = __shfl_sync(0xffffffffu, M[j], g0 + i);
      float c = 0.f;
#pragma unroll
      for (int i = 0; i < N; ++i) c += v[i];
      const float rc = 1.0f / (c + sp.hc_eps);
      M[j] *= rc;
    }
  };
  col_norm_rows();
  for (int it = 1; it < sp.iters; ++it) {
    float r = 0.f;
#pragma unroll
    for (int j = 0; j < N; ++j) r += M[j];
    const float rr = 1.0f / (r + sp.hc_eps);
#pragma unroll
    for (int j = 0; j < N; ++j) M[j] *= rr;
    col_norm_rows();
  }
  if (!valid) return;
  if (n == 0) inv_rms[t] = inv;
  mixes[t * HM + n] = mrow[0];
  mixes[t * HM + N + n] = mrow[1];
  pre[t * N + n] = pr;
  post[t * N + n] = po;
#pragma unroll
  for (int j = 0; j < N; ++j) {
    mixes[t * HM + 2 * N + n * N + j] = mrow[2 + j];
    comb[t * N * N + n * N + j] = M[j];
    if (logits_out) logits_out[t * N * N + n * N + j] = l[j];
  }
}

// Split-K finish (the tensor-core mix runs for N = 4, 8): adds the K-range partials of
// each token in range order and runs the small stage row-parallel (small_rows_outputs).
// WARP (many ranges, few tokens): a warp per token; lane l adds ranges l, l+32, ... and a
// fixed-shape warp tree combines the lanes (deterministic); lanes n, n+N, ... then take
// row n.  Otherwise N lanes per token, lane n adding only the components its row needs.
// (A thread per token running the whole chain took 46 us at T=8192; one lane per warp
// running it is issue-bound.)
template <int N, bool WARP>
__global__ void __launch_bounds__(128)
pre_mix_finish_kernel(const float* __restrict__ part, int ksplit, const float* __restrict__ alpha,
                      const float* __restrict__ base, int64_t T, int64_t HC, float norm_eps,
                      SmallParams sp, float* __restrict__ inv_rms, float* __restrict__ mixes,
                      float* __restrict__ pre, float* __restrict__ post, float* __restrict__ comb,
                      float* __restrict__ logits_out, const float* __restrict__ descale) {
  pdl_enter();
  constexpr int HM = hc_mix(N);
  static_assert((N & (N - 1)) == 0 && N > 1 && N <= 8, "row groups of N lanes");
  __shared__ float sbase[HM];
  for (int i = threadIdx.x; i < HM; i += blockDim.x) sbase[i] = base[i];
  __syncthreads();
  sp.a0 = alpha[0]; sp.a1 = alpha[1]; sp.a2 = alpha[2];
  const int lane = threadIdx.x & 31, n = lane % N;
  float mrow[N + 3];  // mix[n], mix[N+n], mix[2N+nN .. 2N+nN+N-1], sum of squares
#pragma unroll
  for (int c = 0; c < N + 3; ++c) mrow[c] = 0.f;
  int64_t t;
  bool valid;
  if constexpr (WARP) {
    t = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    if (t >= T) return;  // whole warps
    valid = lane < N;
    float mix[HM], sq = 0.f;
#pragma unroll
    for (int k = 0; k < HM; ++k) mix[k] = 0.f;
    for (int p = lane; p < ksplit; p += 32) {
      const float* src = part + ((int64_t)p * T + t) * (HM + 1);
#pragma unroll
      for (int k = 0; k < HM; ++k) mix[k] += src[k];
      sq += src[HM];
    }
#pragma unroll
    for (int k = 0; k < HM; ++k) mix[k] = warp_sum(mix[k]);
    sq = warp_sum(sq);
#pragma unroll
    for (int nn = 0; nn < N; ++nn) {  // row n's entries without dynamic register indexing
      if (nn != n) continue;
      mrow[0] = mix[nn];
      mrow[1] = mix[N + nn];
#pragma unroll
      for (int j = 0; j < N; ++j) mrow[2 + j] = mix[2 * N + nn * N + j];
    }
    mrow[N + 2] = sq;
  } else {
    t = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) / N;
    valid = t < T;
    const int64_t tc = valid ? t : T - 1;  // invalid lanes still take part in the shuffles
    for (int p = 0; p < ksplit; ++p) {
      const float* src = part + ((int64_t)p * T + tc) * (HM + 1);
      mrow[0] += src[n];
      mrow[1] += src[N + n];
#pragma unroll
      for (int j = 0; j < N; ++j) mrow[2 + j] += src[2 * N + n * N + j];
      mrow[N + 2] += src[HM];
    }
  }
  const float inv = inv_rms_from_sumsq(mrow[N + 2], HC, norm_eps);
  const float sc = descale ? inv * *descale : inv;
#pragma unroll
  for (int c = 0; c < N + 2; ++c) mrow[c] *= sc;
  small_rows_outputs<N>(mrow, inv, sbase, sp, n, t, valid, (lane / N) * N, inv_rms, mixes, pre,
                        post, comb, logits_out);
}

// Split-K finish for N = 4 with N*N = 16 lanes per token, lane (n, j) owning element
// [n][j]: the lane adds the K-range partials of the components it needs in range order,
// then runs the small stage with one matrix element per lane.  Row and column sums gather
// their N values by shuffles and add them in index order, as small_rows_outputs does, so
// every output is bitwise that kernel's; the chain of a token is about N times shorter.
__global__ void __launch_bounds__(128)
pre_mix_finish_elems_kernel(const float* __restrict__ part, int ksplit,
                            const float* __restrict__ alpha, const float* __restrict__ base,
                            int64_t T, int64_t HC, float norm_eps, SmallParams sp,
                            float* __restrict__ inv_rms, float* __restrict__ mixes,
                            float* __restrict__ pre, float* __restrict__ post,
                            float* __restrict__ comb, float* __restrict__ logits_out,
                            const float* __restrict__ descale) {
  pdl_enter();
  constexpr int N = 4, NN = 16, HM = hc_mix(N);
  __shared__ float sbase[HM];
  for (int i = threadIdx.x; i < HM; i += blockDim.x) sbase[i] = base[i];
  __syncthreads();
  sp.a0 = alpha[0]; sp.a1 = alpha[1]; sp.a2 = alpha[2];
  const int lane = threadIdx.x & 31, e = lane % NN, n = e / N, j = e % N;
  const int gl0 = (lane / NN) * NN;
  const int64_t t = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) / NN;
  const bool valid = t < T;
  const int64_t tc = valid ? t : T - 1;  // invalid lanes still take part in the shuffles
  auto at = [&](float v, int src) { return __shfl_sync(0xffffffffu, v, gl0 + src); };
  // components of this lane: the logit mix of element e; row heads (j == 0); sum of squares
  float mlog = 0.f, mpre = 0.f, mpost = 0.f, sq = 0.f;
#pragma unroll 4
  for (int p = 0; p < ksplit; ++p) {
    const float* src = part + ((int64_t)p * T + tc) * (HM + 1);
    mlog += src[2 * N + e];
    if (j == 0) {
      mpre += src[n];
      mpost += src[N + n];
    }
    if (e == 0) sq += src[HM];
  }
  const float inv = at(e == 0 ? inv_rms_from_sumsq(sq, HC, norm_eps) : 0.f, 0);
  const float sc = descale ? inv * *descale : inv;
  mlog *= sc;
  mpre *= sc;
  mpost *= sc;
  const float pr = sigmoidf_(mpre * sp.a0 + sbase[n]) + sp.hc_eps;
  const float po = 2.0f * sigmoidf_(mpost * sp.a1 + sbase[N + n]);
  const float l = mlog * sp.a2 + sbase[2 * N + e];
  float M = sp.clamp_on ? fminf(fmaxf(l, sp.clamp_min), sp.clamp_max) : l;
  float m = at(M, n * N);
#pragma unroll
  for (int jj = 1; jj < N; ++jj) m = fmaxf(m, at(M, n * N + jj));
  M = expf(M - m);
  float s = 0.f;
#pragma unroll
  for (int jj = 0; jj < N; ++jj) s += at(M, n * N + jj);
  M *= 1.0f / s;
  M += sp.hc_eps;
  auto col_norm = [&]() {
    float c = 0.f;
#pragma unroll
    for (int i = 0; i < N; ++i) c += at(M, i * N + j);
    M *= 1.0f / (c + sp.hc_eps);
  };
  col_norm();
  for (int it = 1; it < sp.iters; ++it) {
    float r = 0.f;
#pragma unroll
    for (int jj = 0; jj < N; ++jj) r += at(M, n * N + jj);
    M *= 1.0f / (r + sp.hc_eps);
    col_norm();
  }
  if (!valid) return;
  if (e == 0) inv_rms[t] = inv;
  if (j == 0) {
    mixes[t * HM + n] = mpre;
    mixes[t * HM + N + n] = mpost;
    pre[t * N + n] = pr;
    post[t * N + n] = po;
  }
  mixes[t * HM + 2 * N + e] = mlog;
  comb[t * NN + e] = M;
  if (logits_out) logits_out[t * NN + e] = l;
}

// ---------------------------------------------------------------------------
// Host side
// ---------------------------------------------------------------------------
bool pre_fwd_tc_eligible(const PreFwdArgs& a) {
  const int64_t HC = (int64_t)a.N * a.D;
  const bool f32 = a.dtype == MHC_F32;
  return (a.dtype == MHC_BF16 || a.dtype == MHC_F16 || f32) && (a.N == 4 || a.N == 8) &&
         HC % 8 == 0 && rows_aligned(a.x, a.x_ts, f32 ? 4 : 2, 16) &&
         (!f32 || aligned16(a.phi)) && a.T > 0 && a.T <= (int64_t)INT32_MAX - 256;
}

// K elements per pipeline stage: two 64-column boxes (16-bit, N=4), one (16-bit, N=8), one
// 32-column box (fp32).
static int64_t mix_stage_k(int32_t N, int32_t dtype) {
  return dtype == MHC_F32 ? 32 : (N <= 4 ? 2 : 1) * 64;
}

// Split K across CTAs when the tiles cannot fill the GPU (small T): K ranges per tile.
static int mix_ksplit(int64_t T, int32_t N, int64_t D, int32_t dtype) {
  const int64_t ntiles = cdiv(T, 128), sms = sm_count();
  if (ntiles <= 0 || 2 * ntiles > sms) return 1;
  const int64_t nk = cdiv((int64_t)N * D, mix_stage_k(N, dtype));
  int64_t k = sms / ntiles;
  if (k > nk / 4) k = nk / 4;  // at least 4 K chunks per range
  return (int)(k < 1 ? 1 : k);
}

// workspace: phi as hi/lo rows (16-bit, or fp32 for kind::tf32), (split K only) the
// partials [ksplit][T][HM+1], then the fp16 scale slots (max|phi| bits, 2^-s)
size_t pre_fwd_tc_ws_bytes(int64_t T, int32_t N, int64_t D, int32_t dtype) {
  const int HM = hc_mix(N);
  const int NP = (2 * HM + 15) / 16 * 16;
  const int ks = mix_ksplit(T, N, D, dtype);
  return align_up((size_t)NP * N * D * (dtype == MHC_F32 ? 4 : 2)) +
         (ks > 1 ? align_up((size_t)ks * T * (HM + 1) * 4) : 0) + 256;
}

template <int N, int NB, typename E>
static int pre_fwd_tc_nb(const PreFwdArgs& a, cudaStream_t s) {
  using C = MixCfgE<N, NB, E>;
  constexpr bool f16 = std::is_same<E, __half>::value;
  constexpr bool f32 = std::is_same<E, float>::value;
  const int64_t T = a.T, HC = (int64_t)N * a.D;
  const int ks = mix_ksplit(T, N, a.D, a.dtype);
  E* phi_hl = (E*)a.workspace;
  const size_t phi_bytes = align_up((size_t)C::NP * HC * sizeof(E));
  float* part = ks > 1 ? (float*)((char*)a.workspace + phi_bytes) : nullptr;
  char* slots = (char*)a.workspace + phi_bytes +
                (ks > 1 ? align_up((size_t)ks * T * (C::HM + 1) * 4) : 0);
  unsigned* maxslot = f16 ? (unsigned*)slots : nullptr;
  float* descale = f16 ? (float*)(slots + 16) : nullptr;
  if constexpr (f32) {
    const int64_t bx = std::min<int64_t>(cdiv(HC / 4, 256), 64);
    launch(pre_phi_split_tf32_kernel, dim3((unsigned)bx, (unsigned)C::NP), 256, 0, s, a.phi,
           (float*)phi_hl, C::HM, C::NP, HC);
    MHC_LAUNCH_CHECK();
  } else {
    const int64_t n = (int64_t)C::NP * HC;
    const int grid = (int)std::min<int64_t>(cdiv(n, 256), (int64_t)sm_count() * 8);
    if (f16) {
      MHC_CUDA_CHECK(cudaMemsetAsync(maxslot, 0, sizeof(unsigned), s));
      const int64_t m = (int64_t)C::HM * HC;
      launch(pre_phi_maxabs_kernel, (int)std::min<int64_t>(cdiv(m, 256), (int64_t)sm_count() * 4), 256, 0, s, a.phi, m, maxslot);
      MHC_LAUNCH_CHECK();
    }
    if (HC % 8 == 0 && aligned16(a.phi)) {
      const int64_t bx = std::min<int64_t>(cdiv(HC / 8, 256), 64);
      launch(pre_phi_split8_kernel<E>, dim3((unsigned)bx, (unsigned)(C::NP - C::HM)), 256, 0, s,
             a.phi, phi_hl, C::HM, C::NP, HC, maxslot, descale);
    } else {
      launch(pre_phi_split_kernel<E>, grid, 256, 0, s, a.phi, phi_hl, C::HM, C::NP, HC, maxslot,
             descale);
    }
    MHC_LAUNCH_CHECK();
  }
  const CUtensorMapDataType dt =
      f32 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32
          : f16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
  constexpr int eb = (int)sizeof(E);
  CUtensorMap tx, tp;
  int st = make_tmap_2d(&tx, a.x, dt, eb, HC, T, a.x_ts * eb, C::BOX, 128,
                        CU_TENSOR_MAP_SWIZZLE_128B);
  if (st != MHC_OK) return st;
  st = make_tmap_2d(&tp, phi_hl, dt, eb, HC, C::NP, HC * eb, C::BOX, C::NP,
                    CU_TENSOR_MAP_SWIZZLE_128B);
  if (st != MHC_OK) return st;
  static bool attr_set[64];
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 0 && dev < 64 && !attr_set[dev]) {
    MHC_CUDA_CHECK(cudaFuncSetAttribute(pre_mix_tc_kernel<N, NB, E>,
                                        cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM));
    attr_set[dev] = true;
  }
  const int64_t ntiles = cdiv(T, 128);
  const int grid = (int)std::min<int64_t>(ntiles * ks, sm_count());
  launch(pre_mix_tc_kernel<N, NB, E>, grid, C::THREADS, C::SMEM, s, 
      tx, tp, a.alpha, a.base, T, HC, a.norm_eps, a.sp, a.inv_rms, a.mixes, a.pre, a.post_out,
      a.comb_frag, a.h_res_logits, ks, part, descale);
  MHC_LAUNCH_CHECK();
  if (part) {
    // a warp per token only for many K ranges (few tokens): lanes then share the loads
    const bool warp_tok = ks > 16;
    if (!warp_tok && N == 4) {
      launch(pre_mix_finish_elems_kernel, (unsigned)cdiv(T, 128 / 16), 128, 0, s, part, ks,
             a.alpha, a.base, T, HC, a.norm_eps, a.sp, a.inv_rms, a.mixes, a.pre, a.post_out,
             a.comb_frag, a.h_res_logits, descale);
    } else {
      auto fin = warp_tok ? pre_mix_finish_kernel<N, true> : pre_mix_finish_kernel<N, false>;
      launch(fin, (unsigned)cdiv(T, warp_tok ? 4 : 128 / N), 128, 0, s, part, ks, a.alpha,
             a.base, T, HC, a.norm_eps, a.sp, a.inv_rms, a.mixes, a.pre, a.post_out,
             a.comb_frag, a.h_res_logits, descale);
    }
    MHC_LAUNCH_CHECK();
  }
  return MHC_OK;
}

// Two adjacent 64-column boxes per stage: each DRAM row visit then fetches 256 B of a
// token row instead of 128 B (measured: the mix pass 0.36 -> 0.31 ms at T=32768, D=7168;
// four boxes gain nothing more).  N=8's larger phi operand keeps one box per stage so the
// ring still holds several stages.
template <int N>
static int pre_fwd_tc_n(const PreFwdArgs& a, cudaStream_t s) {
  if (a.dtype == MHC_F32) return pre_fwd_tc_nb<N, 1, float>(a, s);
  if (a.dtype == MHC_F16) return pre_fwd_tc_nb<N, (N <= 4 ? 2 : 1), __half>(a, s);
  return pre_fwd_tc_nb<N, (N <= 4 ? 2 : 1), __nv_bfloat16>(a, s);
}

// Runs the tensor-core mix (+ fused small stage); the caller then runs pre_apply.
// phi (fp32, N*(N+2) rows) -> phi_hl [NP][HC] (16-bit hi / lo rows, zero rows) for the
// layer-fused post forward; fp16: max|phi| and the descale factor go to slots / slots+16.
int pre_phi_split_launch(const float* phi, void* phi_hl, int32_t N, int64_t HC, bool f16,
                         void* slots, cudaStream_t s) {
  if (N != 4 || HC % 8 != 0 || !aligned16(phi)) return MHC_ERR_INVALID_ARGUMENT;
  using C = MixCfg<4, 2>;
  unsigned* maxslot = f16 ? (unsigned*)slots : nullptr;
  float* descale = f16 ? (float*)((char*)slots + 16) : nullptr;
  if (f16) {
    MHC_CUDA_CHECK(cudaMemsetAsync(maxslot, 0, sizeof(unsigned), s));
    const int64_t m = (int64_t)C::HM * HC;
    launch(pre_phi_maxabs_kernel, (int)std::min<int64_t>(cdiv(m, 256), (int64_t)sm_count() * 4),
           256, 0, s, phi, m, maxslot);
    MHC_LAUNCH_CHECK();
  }
  const int64_t bx = std::min<int64_t>(cdiv(HC / 8, 256), 64);
  if (f16)
    launch(pre_phi_split8_kernel<__half>, dim3((unsigned)bx, (unsigned)(C::NP - C::HM)), 256, 0,
           s, phi, (__half*)phi_hl, C::HM, C::NP, HC, maxslot, descale);
  else
    launch(pre_phi_split8_kernel<__nv_bfloat16>, dim3((unsigned)bx, (unsigned)(C::NP - C::HM)),
           256, 0, s, phi, (__nv_bfloat16*)phi_hl, C::HM, C::NP, HC, maxslot, descale);
  MHC_LAUNCH_CHECK();
  return MHC_OK;
}

// The pre operator's small stage from precomputed mix partials ([layers][T][HM+1]: raw
// mix of each K range, already descaled, and its sum of squares) -- the input written by
// the layer-fused post forward.
int pre_fwd_finish_premix(const PreFwdArgs& a, cudaStream_t s) {
  const int64_t T = a.T, HC = (int64_t)a.N * a.D;
  const int ks = a.premix_layers;
  if (a.N == 4 && ks <= 16) {
    launch(pre_mix_finish_elems_kernel, (unsigned)cdiv(T, 128 / 16), 128, 0, s, a.premix, ks,
           a.alpha, a.base, T, HC, a.norm_eps, a.sp, a.inv_rms, a.mixes, a.pre, a.post_out,
           a.comb_frag, a.h_res_logits, (const float*)nullptr);
  } else if (a.N == 4) {
    launch(pre_mix_finish_kernel<4, true>, (unsigned)cdiv(T, 4), 128, 0, s, a.premix, ks,
           a.alpha, a.base, T, HC, a.norm_eps, a.sp, a.inv_rms, a.mixes, a.pre, a.post_out,
           a.comb_frag, a.h_res_logits, (const float*)nullptr);
  } else {
    return MHC_ERR_UNSUPPORTED_N;
  }
  MHC_LAUNCH_CHECK();
  return MHC_OK;
}

int pre_fwd_tc_mix(const PreFwdArgs& a, cudaStream_t s) {
  switch (a.N) {
    case 4: return pre_fwd_tc_n<4>(a, s);
    case 8: return pre_fwd_tc_n<8>(a, s);
    default: return MHC_ERR_UNSUPPORTED_N;
  }
}

int pre_fwd_tc_device_error() { return read_and_clear_tu_error(); }

}  // namespace mhc

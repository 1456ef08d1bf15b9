// pre_bwd_tc32.cu -- mhc_pre_clamp_sinkhorn backward, tensor-core main pass for fp32 x
// (N = 4 or 8, D % 32 == 0).
//
// After pass 1 (pre_bwd.cu: grad_pre dots + small-stage VJP, which write grad_mixes and
// coef in fp32), two streaming tcgen05 kernels produce grad_x and grad_phi:
//
//   bwd32_gx_kernel    a 128-token tile at a time, over all columns in 32-column steps:
//                        gxs = G'(128 x KG) P'(KG x 32)       (kind::f16, bf16 operands)
//                        grad_x = pre[n] gy + inv gxs - coef x  (epilogue, fp32 x / gy)
//                      G' and P' hold products of bf16 pieces of grad_mixes and phi
//                      (more of them than the 16-bit paths use, for fp32 accuracy); x
//                      never enters this product.
//   bwd32_gphi_kernel  a 128-column tile at a time, over 32-token steps:
//                        D[c, k] += x^T(c, t) Gp(t, k) + x_lo^T(c, t) Gp(t, k)
//                      (kind::tf32, M = 128 columns, N = [(inv g)_hi | (inv g)_lo] in
//                      tf32 parts, K = 8 tokens per MMA).  kind::tf32 takes K-major
//                      operands here (the MN-major form of the 16-bit kernels left D at
//                      zero on B200), so both come token-contiguous: Gp is written
//                      transposed ([k][T]) by its prep kernel, and four warps transpose
//                      each [32 tok][128 col] x tile into x^T and x_lo^T = (x - x_hi)^T
//                      in shared memory.  The tensor core reads the top 19 bits of x
//                      (x_hi), so the two products carry x to ~2^-21.  Segments of at
//                      most SUBT steps are accumulated in one of two TMEM buffers and
//                      folded into fp32 registers; each CTA writes one partial per column
//                      tile it touches and bwd32_gphi_reduce_kernel sums them in CTA order
//                      (deterministic).
#include "pre_common.cuh"
#include "tc.cuh"

namespace mhc {

namespace bwd32 {
template <int N>
struct Cfg {
  static constexpr int HM = hc_mix(N);
  // gxs K: NPROD blocks of HM (products of bf16 pieces of grad_mixes and phi), padded to
  // 64.  N=4: all six products of total order <= 2 of three-piece splits (g0p0, g1p0,
  // g0p1, g2p0, g1p1, g0p2): grad_mixes.phi to ~2^-24 (three products of two-piece splits,
  // as the 16-bit paths use, leave ~1e-5).
  static constexpr int NPROD = 6;
  static constexpr int KG = (NPROD * HM + 63) / 64 * 64;
  static constexpr int NPH = (2 * HM + 15) / 16 * 16;  // grad_phi MMA N (hi | lo)
  // columns per gx step: one fp32 box of 128 B (N=4) or 64 B rows (N=8, whose 128 KB G'
  // tile leaves room only for narrower stages)
  static constexpr int CB = N == 4 ? 32 : 16;
  static constexpr int RB = CB * 4;               // bytes per x / grad_y box row
  // ---- gx kernel
  static constexpr int G_ATOM = 128 * 64 * 2;     // [128 tok][64 k] bf16 SW128
  static constexpr int G_BYTES = (KG / 64) * G_ATOM;
  static constexpr int P_ATOM = CB * 64 * 2;      // [CB col][64 k] bf16 SW128
  static constexpr int P_BYTES = (KG / 64) * P_ATOM;
  static constexpr int X_BYTES = 128 * RB;        // [128 tok][CB col] fp32, SW128 / SW64
  static constexpr int GY_BYTES = X_BYTES;
  static constexpr int OUT_BYTES = 32 * 16 * 4;   // per epilogue warp: [32 tok][16 col], SW64
  static constexpr int EPI_WARPS = CB / 4;        // 4 lane quarters x CB/16 column halves
  static constexpr int GX_THREADS = 32 * (2 + EPI_WARPS);
  // P' (from L2) and x (from DRAM) rings deep enough to run several steps ahead
  static constexpr int PS = 4, XS = N == 4 ? 4 : 2;
  static constexpr int OFF_G = 0;
  static constexpr int OFF_P = OFF_G + G_BYTES;
  static constexpr int OFF_X = OFF_P + PS * P_BYTES;
  static constexpr int OFF_GY = OFF_X + XS * X_BYTES;
  static constexpr int OFF_OUT = OFF_GY + GY_BYTES;
  static constexpr int OFF_BAR = OFF_OUT + EPI_WARPS * OUT_BYTES;
  static constexpr int GX_SMEM = 1024 + OFF_BAR + 512;
  static constexpr int DS = 32;                   // TMEM columns between the D1 buffers
  static constexpr int GX_TMEM = 2 * DS;          // D1[2] (CB of DS columns used)
  // ---- grad_phi kernel
  static constexpr int CT = 128;                  // columns per tile (MMA M)
  static constexpr int TT = 32;                   // tokens per step (one 128 B row of fp32)
  static constexpr int XBOX = TT * 32 * 4;        // [32 tok][32 col] fp32 SW128 (4 KB)
  static constexpr int XT_BYTES = (CT / 32) * XBOX;  // 16 KB: x tile, and x^T / x_lo^T
  static constexpr int GP_BYTES = NPH * TT * 4;   // Gp^T [NPH][32 tok] SW128
  static constexpr int GP_STRIDE = (GP_BYTES + 1023) / 1024 * 1024;
  // TMA stages [x tile | Gp^T] (deep: they cover the DRAM latency) and two buffers of
  // [x^T | x_lo^T] (the MMA operands the transpose warps write)
  static constexpr int XSTAGE = XT_BYTES + GP_STRIDE;
  static constexpr int TB_BYTES = 2 * XT_BYTES;
  static constexpr int S = (220 * 1024 - 2 * TB_BYTES) / XSTAGE > 8
                               ? 8 : (220 * 1024 - 2 * TB_BYTES) / XSTAGE;
  static constexpr int OFF_TB = S * XSTAGE;
  static constexpr int SUBT = 8;                  // steps per TMEM segment (64 MMAs)
  static constexpr int GP_THREADS = 32 * 10;      // TMA, MMA, 4 x_lo warps, 4 fold warps
  static constexpr int GP_OFF_BAR = OFF_TB + 2 * TB_BYTES;
  static constexpr int GP_SMEM = 1024 + GP_OFF_BAR + 256;
  static constexpr int DCOL = (NPH + 31) / 32 * 32;  // TMEM columns per D buffer
  static constexpr int GP_TMEM = 2 * DCOL <= 128 ? 128 : 2 * DCOL <= 256 ? 256 : 512;
  static_assert(GX_SMEM <= 232448 && GP_SMEM <= 232448, "shared memory");
  static_assert(OFF_P % 1024 == 0 && OFF_X % 1024 == 0 && OFF_GY % 1024 == 0 &&
                OFF_OUT % 1024 == 0 && XBOX % 1024 == 0 && XSTAGE % 1024 == 0, "alignment");
};
}  // namespace bwd32

// fp16 operand maxima kernel lives in pre_bwd_tc.cu; nothing here is scaled (bf16 / tf32
// share fp32's exponent range).

// bf16 pieces of f: f ~ p0 + p1 + p2 (each the rounding of what the previous ones leave).
__device__ __forceinline__ float bf16_piece(float f, int i) {
  const float p0 = __bfloat162float(__float2bfloat16_rn(f));
  if (i == 0) return p0;
  const float r = f - p0;
  const float p1 = __bfloat162float(__float2bfloat16_rn(r));
  if (i == 1) return p1;
  return __bfloat162float(__float2bfloat16_rn(r - p1));
}
// block b of the gxs K: (piece of grad_mixes, piece of phi)
__host__ __device__ constexpr int gxs_g_piece(int b) { return b == 1 || b == 4 ? 1 : b == 3 ? 2 : 0; }
__host__ __device__ constexpr int gxs_p_piece(int b) { return b == 2 || b == 4 ? 1 : b == 5 ? 2 : 0; }

// phi (fp32 [HM][HC]) -> P' [HC][KG] bf16: block b = piece gxs_p_piece(b) of phi, then 0.
// Thread per (column, 8-element chunk).
template <int N>
__global__ void bwd32_phi_prep_kernel(const float* __restrict__ phi,
                                      __nv_bfloat16* __restrict__ p, int64_t HC) {
  pdl_enter();
  using C = bwd32::Cfg<N>;
  constexpr int HM = C::HM, KG = C::KG;
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= HC * (KG / 8)) return;
  const int64_t c = i / (KG / 8);
  const int j = (int)(i - c * (KG / 8));
  float v[8];
#pragma unroll
  for (int e = 0; e < 8; ++e) {
    const int k = 8 * j + e;
    float r = 0.f;
    if (k < C::NPROD * HM)
      r = bf16_piece(phi[(int64_t)(k % HM) * HC + c], gxs_p_piece(k / HM));
    v[e] = r;
  }
  reinterpret_cast<uint4*>(p + c * KG)[j] = narrow<__nv_bfloat16>(v);
}

// grad_mixes (fp32 [T][HM]) -> G' [T][KG] bf16: block b = piece gxs_g_piece(b), then 0.
// Thread per (token, 8-element chunk).
template <int N>
__global__ void bwd32_g_prep_kernel(const float* __restrict__ gm,
                                    __nv_bfloat16* __restrict__ g, int64_t T) {
  pdl_enter();
  using C = bwd32::Cfg<N>;
  constexpr int HM = C::HM, KG = C::KG;
  constexpr int CH = KG / 8;
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= T * CH) return;
  const int64_t t = i / CH;
  const int j = (int)(i - t * CH);
  const float* gr = gm + t * HM;
  {
    float v[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      const int k = 8 * j + e;
      float r = 0.f;
      if (k < C::NPROD * HM) r = bf16_piece(gr[k % HM], gxs_g_piece(k / HM));
      v[e] = r;
    }
    reinterpret_cast<uint4*>(g + t * KG)[j] = narrow<__nv_bfloat16>(v);
  }
}

// Gp^T [NPH][tp] fp32 (token-contiguous rows, tp = T rounded up to 4): row k < HM =
// (inv g)_hi (the tf32 part), row HM + k = (inv g)_lo, tokens beyond T = 0.  Thread per
// (row, token), token fastest (coalesced stores).
template <int N>
__global__ void bwd32_gpt_prep_kernel(const float* __restrict__ gm,
                                      const float* __restrict__ inv_rms,
                                      float* __restrict__ gpt, int64_t T, int64_t tp) {
  pdl_enter();
  using C = bwd32::Cfg<N>;
  constexpr int HM = C::HM;
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= (int64_t)C::NPH * tp) return;
  const int k = (int)(i / tp);
  const int64_t t = i - (int64_t)k * tp;
  float r = 0.f;
  if (t < T && k < 2 * HM) {
    const float f = gm[t * HM + (k % HM)] * inv_rms[t];
    const float hi = tf32_hi(f);
    r = k < HM ? hi : f - hi;
  }
  gpt[i] = r;
}

struct Bwd32GxMaps {
  CUtensorMap x, gy, g, p, gx, gxa;
};

// Step cursor of the gx kernel: step = (token tile, column block b, sub-chunk n) with n
// fastest, so one grad_y block serves N consecutive steps.
template <int N>
struct Gx32Cursor {
  int64_t tile, j, S;
  int blk, n;
  bool tile_start, blk_start;
  __device__ void init(int64_t gs, int64_t steps_per_tile) {
    S = steps_per_tile;
    tile = gs / S;
    j = gs - tile * S;
    blk = (int)(j / N);
    n = (int)(j - (int64_t)blk * N);
    tile_start = blk_start = true;
  }
  __device__ void next() {
    tile_start = blk_start = false;
    ++j;
    if (++n == N) { n = 0; ++blk; blk_start = true; }
    if (j == S) { j = 0; blk = 0; n = 0; ++tile; tile_start = blk_start = true; }
  }
};

template <int N, bool ACC>
__global__ void __launch_bounds__(bwd32::Cfg<N>::GX_THREADS, 1)
bwd32_gx_kernel(const __grid_constant__ Bwd32GxMaps maps, const float* __restrict__ inv_rms,
                const float* __restrict__ coef, const float* __restrict__ pre, int64_t T,
                int64_t D, int64_t total_steps) {
  pdl_enter();
  using C = bwd32::Cfg<N>;
  constexpr int CB = C::CB, XS = C::XS, PS = C::PS, EPI_WARPS = C::EPI_WARPS;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* sm = (uint8_t*)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
  uint64_t* bar = (uint64_t*)(sm + C::OFF_BAR);
  uint64_t* xfull = bar;              // [XS]
  uint64_t* xempty = xfull + XS;      // [XS] epilogue warps read the x tile
  uint64_t* pfull = xempty + XS;      // [PS]
  uint64_t* pempty = pfull + PS;      // [PS] the step's MMAs are done with P'
  uint64_t* d1full = pempty + PS;     // [2]
  uint64_t* d1empty = d1full + 2;     // [2]
  uint64_t* gfull = d1empty + 2;
  uint64_t* gempty = gfull + 1;       // the tile's MMAs are done with G'
  uint64_t* yfull = gfull + 2;
  uint64_t* yempty = gfull + 3;       // epilogue warps read the grad_y block
  uint64_t* tdone = gfull + 4;
  uint64_t* accbar = gfull + 5;       // [EPI_WARPS] the warp's grad_x_acc box landed
  uint32_t* tmem_slot = (uint32_t*)(gfull + 5 + EPI_WARPS);
  volatile int* abort_flag = (volatile int*)(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t HC = N * D, S = HC / CB;
  const int64_t s0 = total_steps * blockIdx.x / gridDim.x;
  const int64_t s1 = total_steps * (blockIdx.x + 1) / gridDim.x;

  if (threadIdx.x == 0) {
    for (int b = 0; b < XS; ++b) {
      tc::mbar_init(&xfull[b], 1);
      tc::mbar_init(&xempty[b], EPI_WARPS);
    }
    for (int b = 0; b < PS; ++b) {
      tc::mbar_init(&pfull[b], 1);
      tc::mbar_init(&pempty[b], 1);
    }
    for (int b = 0; b < 2; ++b) {
      tc::mbar_init(&d1full[b], 1);
      tc::mbar_init(&d1empty[b], EPI_WARPS);
    }
    tc::mbar_init(gfull, 1);
    tc::mbar_init(gempty, 1);
    tc::mbar_init(yfull, 1);
    tc::mbar_init(yempty, EPI_WARPS);
    tc::mbar_init(tdone, 1);
    for (int w = 0; w < EPI_WARPS; ++w) tc::mbar_init(&accbar[w], 1);
    *abort_flag = 0;
    tc::fence_barrier_init();
  }
  if (warp == 0 && lane == 0) {
    tc::prefetch_tmap(&maps.x);
    tc::prefetch_tmap(&maps.gy);
    tc::prefetch_tmap(&maps.g);
    tc::prefetch_tmap(&maps.p);
    tc::prefetch_tmap(&maps.gx);
  }
  if (warp == 1) {
    tc::tmem_alloc(tmem_slot, C::GX_TMEM);
    tc::tmem_relinquish();
  }
  tc::tc_fence_before();
  __syncthreads();
  tc::tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    // ------------------------------------------------------------ TMA producer
    if (lane == 0) {
      Gx32Cursor<N> c;
      c.init(s0, S);
      uint32_t gi = 0, yi = 0;
      const uint64_t pol_stream = tc::l2_evict_first(), pol_keep = tc::l2_evict_last();
      for (int64_t gs = s0; gs < s1; ++gs, c.next()) {
        const uint32_t k = (uint32_t)(gs - s0);
        const int row = (int)(c.tile * 128);
        const int col = (int)(c.n * D + c.blk * CB);
        if (c.tile_start) {
          if (!tc::mbar_wait(gempty, (gi & 1) ^ 1, abort_flag)) break;
          tc::mbar_arrive_expect_tx(gfull, C::G_BYTES);
          for (int a = 0; a < C::KG / 64; ++a)
            tc::tma_load_2d_hint(sm + C::OFF_G + a * C::G_ATOM, &maps.g, gfull, 64 * a, row,
                                 pol_keep);
          ++gi;
        }
        if (c.blk_start) {
          if (!tc::mbar_wait(yempty, (yi & 1) ^ 1, abort_flag)) break;
          tc::mbar_arrive_expect_tx(yfull, C::GY_BYTES);
          tc::tma_load_2d_hint(sm + C::OFF_GY, &maps.gy, yfull, c.blk * CB, row, pol_stream);
          ++yi;
        }
        const int pb = k % PS;
        if (!tc::mbar_wait(&pempty[pb], ((k / PS) & 1) ^ 1, abort_flag)) break;
        tc::mbar_arrive_expect_tx(&pfull[pb], C::P_BYTES);
        for (int a = 0; a < C::KG / 64; ++a)
          tc::tma_load_2d_hint(sm + C::OFF_P + pb * C::P_BYTES + a * C::P_ATOM, &maps.p,
                               &pfull[pb], 64 * a, col, pol_keep);
        const int s = k % XS;
        if (!tc::mbar_wait(&xempty[s], ((k / XS) & 1) ^ 1, abort_flag)) break;
        tc::mbar_arrive_expect_tx(&xfull[s], C::X_BYTES);
        tc::tma_load_2d_hint(sm + C::OFF_X + s * C::X_BYTES, &maps.x, &xfull[s], col, row,
                             pol_stream);
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t idesc = tc::idesc_bf16(128, CB, false, false);
      const uint32_t sg = tc::smem_u32(sm + C::OFF_G), sp = tc::smem_u32(sm + C::OFF_P);
      Gx32Cursor<N> c;
      c.init(s0, S);
      uint32_t gi = 0;
      for (int64_t gs = s0; gs < s1; ++gs, c.next()) {
        const uint32_t k = (uint32_t)(gs - s0);
        if (c.tile_start) {
          if (!tc::mbar_wait(gfull, gi & 1, abort_flag)) break;
          ++gi;
        }
        const int pb = k % PS;
        if (!tc::mbar_wait(&pfull[pb], (k / PS) & 1, abort_flag)) break;
        const int e = k & 1;
        if (!tc::mbar_wait(&d1empty[e], ((k >> 1) & 1) ^ 1, abort_flag)) break;
        tc::tc_fence_after();
        const uint32_t d1 = tmem + e * C::DS;
#pragma unroll
        for (int a = 0; a < C::KG / 64; ++a) {
          const uint64_t da = tc::smem_desc(sg + a * C::G_ATOM, 16, 1024, tc::kSwizzle128);
          const uint64_t db = tc::smem_desc(sp + pb * C::P_BYTES + a * C::P_ATOM, 16, 1024,
                                            tc::kSwizzle128);
#pragma unroll
          for (int kk = 0; kk < 4; ++kk)
            tc::mma_bf16(d1, da + 2 * kk, db + 2 * kk, idesc, (a | kk) != 0);
        }
        tc::mma_commit(&d1full[e]);
        tc::mma_commit(&pempty[pb]);
        if (c.j == S - 1 || gs == s1 - 1) tc::mma_commit(gempty);
      }
      tc::mma_commit(tdone);
      volatile int never = 0;
      tc::mbar_wait(tdone, 0, &never);
    }
  } else {
    // ------------------------------------------------------------ epilogue warps
    // lane quarter q (TMEM lanes 32q..), column half hh (16 of the step's CB columns)
    const int q = warp & 3, hh = (warp - 2) >> 2;
    // 16-byte chunk position in a swizzled box row: 128 B rows swizzle by r & 7, 64 B
    // rows by (r >> 1) & 3
    auto xsw = [&](int chunk, int r) {
      return C::RB == 128 ? (chunk ^ (r & 7)) : (chunk ^ ((r >> 1) & 3));
    };
    const int r = q * 32 + lane;
    uint8_t* ob = sm + C::OFF_OUT + (warp - 2) * C::OUT_BYTES;
    uint8_t* orow = ob + lane * 64;
    const int osw = (lane >> 1) & 3;
    uint64_t* mybar = &accbar[warp - 2];
    uint32_t ai = 0;
    Gx32Cursor<N> c;
    c.init(s0, S);
    uint32_t yi = 0;
    float inv = 0.f, cf = 0.f;
    uint4 gyv[4];
    for (int64_t gs = s0; gs < s1; ++gs, c.next()) {
      const uint32_t k = (uint32_t)(gs - s0);
      const int64_t t = c.tile * 128 + r;
      const bool live = t < T;
      if (c.tile_start) {
        inv = live ? inv_rms[t] : 0.f;
        cf = live ? coef[t] : 0.f;
      }
      const float prn = live ? pre[t * N + c.n] : 0.f;
      const int e = k & 1, s = k % XS;
      const int64_t row0 = c.tile * 128 + q * 32;
      const bool ld_acc = ACC && row0 < T;
      if (ld_acc && lane == 0) {
        tc::bulk_wait_read<0>();
        tc::mbar_arrive_expect_tx(mybar, C::OUT_BYTES);
        tc::tma_load_2d(ob, &maps.gxa, mybar, (int)(c.n * D + c.blk * CB + hh * 16), (int)row0);
      }
      if (!__all_sync(0xffffffffu, tc::mbar_wait(&d1full[e], (k >> 1) & 1, abort_flag))) break;
      tc::tc_fence_after();
      // row r, columns [16hh, 16hh+16) of a [128][CB] fp32 swizzled tile
      if (c.blk_start) {
        if (!__all_sync(0xffffffffu, tc::mbar_wait(yfull, yi & 1, abort_flag))) break;
        const uint8_t* yrow = sm + C::OFF_GY + r * C::RB;
#pragma unroll
        for (int jv = 0; jv < 4; ++jv)
          gyv[jv] = *reinterpret_cast<const uint4*>(yrow + (xsw(4 * hh + jv, r) << 4));
      }
      if (!__all_sync(0xffffffffu, tc::mbar_wait(&xfull[s], (k / XS) & 1, abort_flag))) break;
      const uint8_t* xrow = sm + C::OFF_X + s * C::X_BYTES + r * C::RB;
      uint4 xv[4];
#pragma unroll
      for (int jv = 0; jv < 4; ++jv)
        xv[jv] = *reinterpret_cast<const uint4*>(xrow + (xsw(4 * hh + jv, r) << 4));
      tc::fence_proxy_async();  // generic smem reads before the TMA refills
      __syncwarp();
      if (lane == 0) {
        tc::mbar_arrive(&xempty[s]);
        if (c.blk_start) tc::mbar_arrive(yempty);
        tc::bulk_wait_read<0>();  // this warp's previous grad_x box has left the buffer
      }
      if (c.blk_start) ++yi;
      __syncwarp();
      if (ld_acc) {
        if (!__all_sync(0xffffffffu, tc::mbar_wait(mybar, ai & 1, abort_flag))) break;
        ++ai;
      }
      const uint32_t ta = tmem + ((uint32_t)(q * 32) << 16) + e * C::DS + hh * 16;
      float acc[16];
      tc::tmem_ld16(ta, acc);
      tc::tmem_ld_wait();
      tc::tc_fence_before();
      __syncwarp();
      if (lane == 0) tc::mbar_arrive(&d1empty[e]);
#pragma unroll
      for (int jv = 0; jv < 4; ++jv) {
        float xf[4], gf[4], o[4];
        widen<float>(xv[jv], xf);
        widen<float>(gyv[jv], gf);
#pragma unroll
        for (int u = 0; u < 4; ++u)
          o[u] = fmaf(gf[u], prn, fmaf(inv, acc[4 * jv + u], -cf * xf[u]));
        if (ld_acc) {
          float a4[4];
          widen<float>(*reinterpret_cast<const uint4*>(orow + ((jv ^ osw) << 4)), a4);
#pragma unroll
          for (int u = 0; u < 4; ++u) o[u] += a4[u];
        }
        *reinterpret_cast<uint4*>(orow + ((jv ^ osw) << 4)) = narrow<float>(o);
      }
      tc::fence_proxy_async();  // generic smem writes -> TMA store reads
      __syncwarp();
      if (lane == 0 && row0 < T) {
        tc::tma_store_2d(&maps.gx, ob, (int)(c.n * D + c.blk * CB + hh * 16), (int)row0);
        tc::bulk_commit_group();
      }
    }
    if (lane == 0) tc::bulk_wait_all<0>();
  }
  if (*abort_flag && threadIdx.x == 0) flag_timeout();
  tc::tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc::tc_fence_after();
    tc::tmem_dealloc(tmem, C::GX_TMEM);
  }
}

struct Bwd32GpMaps {
  CUtensorMap x, gpt;
};

// grad_phi work: step = (128-column tile ct, 64-token tile) with token tiles fastest; CTA
// b owns steps [total*b/G, total*(b+1)/G).  Partial slot of CTA b for tile ct = b - (first
// CTA that touches ct).
__host__ __device__ inline int64_t bwd32_cta_of_step(int64_t s, int64_t total, int64_t G) {
  return ((s + 1) * G - 1) / total;
}

template <int N>
__global__ void __launch_bounds__(bwd32::Cfg<N>::GP_THREADS, 1)
bwd32_gphi_kernel(const __grid_constant__ Bwd32GpMaps maps, float* __restrict__ part,
                  int64_t ntiles, int64_t total_steps, int maxslot) {
  pdl_enter();
  using C = bwd32::Cfg<N>;
  constexpr int HM = C::HM, S = C::S, NPH = C::NPH, SUBT = C::SUBT;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* sm = (uint8_t*)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
  uint64_t* bar = (uint64_t*)(sm + C::GP_OFF_BAR);
  uint64_t* full = bar;            // [S] x tile and Gp^T landed
  uint64_t* empty = full + S;      // [S] the step's MMAs are done with the stage
  uint64_t* lready = empty + S;    // [2] x^T and x_lo^T written into buffer b (4 warps)
  uint64_t* tfree = lready + 2;    // [2] the MMAs are done with buffer b
  uint64_t* dfull = tfree + 2;     // [2] segment accumulated in TMEM buffer b
  uint64_t* dempty = dfull + 2;    // [2] the fold warps read buffer b
  uint64_t* tdone = dempty + 2;
  uint32_t* tmem_slot = (uint32_t*)(tdone + 1);
  volatile int* abort_flag = (volatile int*)(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t G = gridDim.x;
  const int64_t s0 = total_steps * blockIdx.x / G;
  const int64_t s1 = total_steps * (blockIdx.x + 1) / G;

  if (threadIdx.x == 0) {
    for (int b = 0; b < S; ++b) {
      tc::mbar_init(&full[b], 1);
      tc::mbar_init(&empty[b], 1);
    }
    for (int b = 0; b < 2; ++b) {
      tc::mbar_init(&lready[b], 4);
      tc::mbar_init(&tfree[b], 1);
      tc::mbar_init(&dfull[b], 1);
      tc::mbar_init(&dempty[b], 4);
    }
    tc::mbar_init(tdone, 1);
    *abort_flag = 0;
    tc::fence_barrier_init();
  }
  if (warp == 0 && lane == 0) {
    tc::prefetch_tmap(&maps.x);
    tc::prefetch_tmap(&maps.gpt);
  }
  if (warp == 1) {
    tc::tmem_alloc(tmem_slot, C::GP_TMEM);
    tc::tmem_relinquish();
  }
  tc::tc_fence_before();
  __syncthreads();
  tc::tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  // segment = at most SUBT consecutive token tiles of one column tile
  auto seg_end = [&](int64_t gs, int64_t tile) {
    return gs == s1 - 1 || tile == ntiles - 1 || (tile % SUBT) == SUBT - 1;
  };

  if (warp == 0) {
    // ------------------------------------------------------------ TMA producer
    if (lane == 0) {
      int64_t ct = s0 / ntiles, tile = s0 - ct * ntiles;
      const uint64_t pol_stream = tc::l2_evict_first(), pol_keep = tc::l2_evict_last();
      for (int64_t gs = s0; gs < s1; ++gs) {
        const uint32_t k = (uint32_t)(gs - s0);
        const int s = k % S;
        if (!tc::mbar_wait(&empty[s], ((k / S) & 1) ^ 1, abort_flag)) break;
        tc::mbar_arrive_expect_tx(&full[s], C::XT_BYTES + C::GP_BYTES);
        uint8_t* st = sm + s * C::XSTAGE;
        for (int b = 0; b < C::CT / 32; ++b)
          tc::tma_load_2d_hint(st + b * C::XBOX, &maps.x, &full[s], (int)(ct * C::CT + 32 * b),
                               (int)(tile * C::TT), pol_stream);
        tc::tma_load_2d_hint(st + C::XT_BYTES, &maps.gpt, &full[s], (int)(tile * C::TT), 0,
                             pol_keep);
        if (++tile == ntiles) { tile = 0; ++ct; }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t idesc = tc::idesc_tf32(128, NPH, false, false);
      const uint32_t sbase = tc::smem_u32(sm);
      int64_t tile = s0 % ntiles;
      uint32_t seg = 0;
      bool seg_first = true;
      for (int64_t gs = s0; gs < s1; ++gs) {
        const uint32_t k = (uint32_t)(gs - s0);
        const int s = k % S;
        const int db = seg & 1;
        if (seg_first && !tc::mbar_wait(&dempty[db], ((seg >> 1) & 1) ^ 1, abort_flag)) break;
        const int tb = k & 1;
        if (!tc::mbar_wait(&full[s], (k / S) & 1, abort_flag)) break;
        if (!tc::mbar_wait(&lready[tb], (k >> 1) & 1, abort_flag)) break;
        tc::tc_fence_after();
        const uint32_t sxt = sbase + C::OFF_TB + tb * C::TB_BYTES, slt = sxt + C::XT_BYTES,
                       sgp = sbase + s * C::XSTAGE + C::XT_BYTES;
        const uint32_t d = tmem + db * C::DCOL;
        // K-major, 128B swizzle: rows of 32 tokens, 8-row atoms of 1 KB; K = 8 tokens
        // (32 B) per MMA
        const uint64_t bg = tc::smem_desc(sgp, 16, 1024, tc::kSwizzle128);
        const uint64_t ax = tc::smem_desc(sxt, 16, 1024, tc::kSwizzle128);
        const uint64_t al = tc::smem_desc(slt, 16, 1024, tc::kSwizzle128);
#pragma unroll
        for (int kk = 0; kk < C::TT / 8; ++kk) {
          tc::mma_tf32(d, ax + 2 * kk, bg + 2 * kk, idesc, (seg_first && kk == 0) ? 0u : 1u);
          tc::mma_tf32(d, al + 2 * kk, bg + 2 * kk, idesc, 1u);
        }
        tc::mma_commit(&empty[s]);
        tc::mma_commit(&tfree[tb]);
        seg_first = false;
        if (seg_end(gs, tile)) {
          tc::mma_commit(&dfull[db]);
          ++seg;
          seg_first = true;
        }
        if (++tile == ntiles) tile = 0;
      }
      tc::mma_commit(tdone);
      volatile int never = 0;
      tc::mbar_wait(tdone, 0, &never);
    }
  } else if (warp < 6) {
    // ------------------------------------------------------------ transpose warps
    // thread = column c of the tile: gathers x[0..31][c] from the row-major TMA tile
    // (a warp reads 32 consecutive floats of one token row), writes row c of x^T and of
    // x_lo^T (eight 16-byte chunks each, in the 128B-swizzled K-major layout)
    const int c = threadIdx.x - 64;
    const int b = c >> 5, cc = c & 31;
    const int csw = c & 7;
    for (int64_t gs = s0; gs < s1; ++gs) {
      const uint32_t k = (uint32_t)(gs - s0);
      const int s = k % S, tb = k & 1;
      if (!__all_sync(0xffffffffu, tc::mbar_wait(&full[s], (k / S) & 1, abort_flag))) break;
      if (!__all_sync(0xffffffffu, tc::mbar_wait(&tfree[tb], ((k >> 1) & 1) ^ 1, abort_flag)))
        break;
      const float* xb = reinterpret_cast<const float*>(sm + s * C::XSTAGE + b * C::XBOX);
      uint8_t* tbuf = sm + C::OFF_TB + tb * C::TB_BYTES;
      uint4* xt = reinterpret_cast<uint4*>(tbuf + c * 128);
      uint4* lt = reinterpret_cast<uint4*>(tbuf + C::XT_BYTES + c * 128);
#pragma unroll
      for (int j = 0; j < C::TT / 4; ++j) {
        float v[4];
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          const int t = 4 * j + u;  // token row t of the box: chunk (cc/4) ^ (t&7)
          v[u] = xb[t * 32 + ((((cc >> 2) ^ (t & 7)) << 2) | (cc & 3))];
        }
        xt[j ^ csw] = make_uint4(__float_as_uint(v[0]), __float_as_uint(v[1]),
                                 __float_as_uint(v[2]), __float_as_uint(v[3]));
        lt[j ^ csw] = make_uint4(__float_as_uint(v[0] - tf32_hi(v[0])),
                                 __float_as_uint(v[1] - tf32_hi(v[1])),
                                 __float_as_uint(v[2] - tf32_hi(v[2])),
                                 __float_as_uint(v[3] - tf32_hi(v[3])));
      }
      tc::fence_proxy_async();  // generic writes -> the MMAs (async proxy) read them
      __syncwarp();
      if (lane == 0) tc::mbar_arrive(&lready[tb]);
    }
  } else {
    // ------------------------------------------------------------ fold warps
    // lane quarter q: thread = column 32q + lane of the tile.  Folds each segment (hi +
    // lo columns) into fp32 registers; writes the CTA's partial for a column tile when
    // its last step in that tile is done.
    const int q = warp & 3;
    const int cl = q * 32 + lane;
    float acc[HM];
#pragma unroll
    for (int kx = 0; kx < HM; ++kx) acc[kx] = 0.f;
    int64_t ct = s0 / ntiles, tile = s0 - ct * ntiles;
    uint32_t seg = 0;
    for (int64_t gs = s0; gs < s1; ++gs) {
      const bool last_in_ct = gs == s1 - 1 || tile == ntiles - 1;
      if (seg_end(gs, tile)) {
        const int db = seg & 1;
        if (!__all_sync(0xffffffffu, tc::mbar_wait(&dfull[db], (seg >> 1) & 1, abort_flag)))
          break;
        tc::tc_fence_after();
        const uint32_t ta = tmem + ((uint32_t)(q * 32) << 16) + db * C::DCOL;
#pragma unroll
        for (int c16 = 0; c16 < (HM + 15) / 16; ++c16) {
          float hi[16], lo[16];
          tc::tmem_ld16(ta + 16 * c16, hi);
          tc::tmem_ld16(ta + HM + 16 * c16, lo);
          tc::tmem_ld_wait();
#pragma unroll
          for (int u = 0; u < 16; ++u)
            if (16 * c16 + u < HM) acc[16 * c16 + u] += hi[u] + lo[u];
        }
        tc::tc_fence_before();
        __syncwarp();
        if (lane == 0) tc::mbar_arrive(&dempty[db]);
        ++seg;
        if (last_in_ct) {
          const int64_t slot =
              (int64_t)blockIdx.x - bwd32_cta_of_step(ct * ntiles, total_steps, G);
          float* dst = part + ((ct * maxslot + slot) * HM) * C::CT + cl;
#pragma unroll
          for (int kx = 0; kx < HM; ++kx) {
            dst[(int64_t)kx * C::CT] = acc[kx];
            acc[kx] = 0.f;
          }
        }
      }
      if (++tile == ntiles) { tile = 0; ++ct; }
    }
  }
  if (*abort_flag && threadIdx.x == 0) flag_timeout();
  tc::tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc::tc_fence_after();
    tc::tmem_dealloc(tmem, C::GP_TMEM);
  }
}

// grad_phi[k][ct*CT + cc] = sum over the CTAs that touched column tile ct, in CTA order.
template <int N>
__global__ void bwd32_gphi_reduce_kernel(const float* __restrict__ part,
                                         float* __restrict__ gphi, int64_t HC, int64_t ntiles,
                                         int64_t total_steps, int64_t G, int maxslot) {
  pdl_enter();
  using C = bwd32::Cfg<N>;
  constexpr int HM = C::HM, CT = C::CT;
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= (int64_t)HM * HC) return;
  const int64_t kx = i / HC, c = i - kx * HC;
  const int64_t ct = c / CT, cc = c - ct * CT;
  const int64_t b0 = bwd32_cta_of_step(ct * ntiles, total_steps, G);
  const int64_t b1 = bwd32_cta_of_step(ct * ntiles + ntiles - 1, total_steps, G);
  Kahan k;
  for (int64_t sl = 0; sl <= b1 - b0; ++sl) k.add(part[((ct * maxslot + sl) * HM + kx) * CT + cc]);
  gphi[i] = k.s;
}

// ---------------------------------------------------------------------------
// Host side
// ---------------------------------------------------------------------------
bool pre_bwd_tc32_eligible(const PreBwdArgs& a) {
  const int64_t T = a.T, D = a.D;
  return a.dtype == MHC_F32 && (a.N == 4 || a.N == 8) && D % 32 == 0 &&
         ((int64_t)a.N * D) % bwd32::Cfg<4>::CT == 0 && T > 0 &&
         T <= (int64_t)INT32_MAX - 256 && (int64_t)a.N * D <= INT32_MAX &&
         rows_aligned(a.x, a.x_ts, 4, 16) && rows_aligned(a.grad_y, a.gy_ts, 4, 16) &&
         aligned16(a.grad_x) && (a.grad_x_acc == nullptr || aligned16(a.grad_x_acc));
}

struct Bwd32Geom {
  int64_t ntiles, ncol, total_gp;
  int grid_gp, maxslot;
};

template <int N>
static Bwd32Geom bwd32_geometry(int64_t T, int64_t D) {
  using C = bwd32::Cfg<N>;
  Bwd32Geom g;
  g.ntiles = cdiv(T, C::TT);
  g.ncol = (N * D) / C::CT;
  g.total_gp = g.ncol * g.ntiles;
  int n = sm_count();
  if (g.total_gp < n) n = (int)g.total_gp;
  g.grid_gp = n < 1 ? 1 : n;
  g.maxslot = 1;
  for (int64_t ct = 0; ct < g.ncol; ++ct) {
    const int64_t b0 = bwd32_cta_of_step(ct * g.ntiles, g.total_gp, g.grid_gp);
    const int64_t b1 = bwd32_cta_of_step(ct * g.ntiles + g.ntiles - 1, g.total_gp, g.grid_gp);
    if (b1 - b0 + 1 > g.maxslot) g.maxslot = (int)(b1 - b0 + 1);
  }
  return g;
}

struct Bwd32Ws {
  __nv_bfloat16 *g, *p;
  float *gpt, *part;
  int64_t tp;  // token stride of Gp^T
  size_t total;
};

template <int N>
static Bwd32Ws bwd32_layout(char* base, int64_t T, int64_t D) {
  using C = bwd32::Cfg<N>;
  const Bwd32Geom geo = bwd32_geometry<N>(T, D);
  const int64_t HC = N * D;
  Bwd32Ws w;
  size_t off = 0;
  auto take = [&](size_t bytes) { char* p = base + off; off += align_up(bytes); return p; };
  w.g = (__nv_bfloat16*)take((size_t)T * C::KG * 2);
  w.tp = (T + 3) / 4 * 4;
  w.gpt = (float*)take((size_t)C::NPH * w.tp * 4);
  w.p = (__nv_bfloat16*)take((size_t)HC * C::KG * 2);
  w.part = (float*)take((size_t)geo.ncol * geo.maxslot * C::HM * C::CT * 4);
  w.total = off;
  return w;
}

size_t pre_bwd_tc32_ws_bytes(int64_t T, int32_t N, int64_t D) {
  if (N == 4) return bwd32_layout<4>(nullptr, T, D).total;
  if (N == 8) return bwd32_layout<8>(nullptr, T, D).total;
  return 0;
}

template <int N>
static int pre_bwd_tc32_run(const PreBwdArgs& a, void* ws, const float* gm, const float* coef,
                            cudaStream_t s) {
  using C = bwd32::Cfg<N>;
  const int64_t T = a.T, D = a.D, HC = N * D;
  const Bwd32Geom geo = bwd32_geometry<N>(T, D);
  Bwd32Ws w = bwd32_layout<N>((char*)ws, T, D);
  launch(bwd32_phi_prep_kernel<N>, (unsigned)cdiv(HC * (C::KG / 8), 256), 256, 0, s, a.phi,
         w.p, HC);
  MHC_LAUNCH_CHECK();
  launch(bwd32_g_prep_kernel<N>, (unsigned)cdiv(T * (C::KG / 8), 256), 256, 0, s, gm, w.g, T);
  MHC_LAUNCH_CHECK();
  launch(bwd32_gpt_prep_kernel<N>, (unsigned)cdiv(C::NPH * w.tp, 256), 256, 0, s, gm,
         a.inv_rms, w.gpt, T, w.tp);
  MHC_LAUNCH_CHECK();

  const CUtensorMapDataType bf = CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
  const CUtensorMapDataType f4 = CU_TENSOR_MAP_DATA_TYPE_FLOAT32;
  int st;
  Bwd32GxMaps mx;
  const CUtensorMapSwizzle xswz =
      C::RB == 128 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_64B;
  if ((st = make_tmap_2d(&mx.x, a.x, f4, 4, HC, T, a.x_ts * 4, C::CB, 128, xswz)))
    return st;
  if ((st = make_tmap_2d(&mx.gy, a.grad_y, f4, 4, D, T, a.gy_ts * 4, C::CB, 128, xswz)))
    return st;
  if ((st = make_tmap_2d(&mx.g, w.g, bf, 2, C::KG, T, C::KG * 2, 64, 128,
                         CU_TENSOR_MAP_SWIZZLE_128B)))
    return st;
  if ((st = make_tmap_2d(&mx.p, w.p, bf, 2, C::KG, HC, C::KG * 2, 64, C::CB,
                         CU_TENSOR_MAP_SWIZZLE_128B)))
    return st;
  if ((st = make_tmap_2d(&mx.gx, a.grad_x, f4, 4, HC, T, HC * 4, 16, 32,
                         CU_TENSOR_MAP_SWIZZLE_64B)))
    return st;
  mx.gxa = mx.gx;
  if (a.grad_x_acc &&
      (st = make_tmap_2d(&mx.gxa, a.grad_x_acc, f4, 4, HC, T, HC * 4, 16, 32,
                         CU_TENSOR_MAP_SWIZZLE_64B)))
    return st;
  Bwd32GpMaps mp;
  if ((st = make_tmap_2d(&mp.x, a.x, f4, 4, HC, T, a.x_ts * 4, 32, C::TT,
                         CU_TENSOR_MAP_SWIZZLE_128B)))
    return st;
  if ((st = make_tmap_2d(&mp.gpt, w.gpt, f4, 4, w.tp, C::NPH, w.tp * 4, C::TT, C::NPH,
                         CU_TENSOR_MAP_SWIZZLE_128B)))
    return st;

  static bool attr_set[64];
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 0 && dev < 64 && !attr_set[dev]) {
    MHC_CUDA_CHECK(cudaFuncSetAttribute(bwd32_gx_kernel<N, false>,
                                        cudaFuncAttributeMaxDynamicSharedMemorySize, C::GX_SMEM));
    MHC_CUDA_CHECK(cudaFuncSetAttribute(bwd32_gx_kernel<N, true>,
                                        cudaFuncAttributeMaxDynamicSharedMemorySize, C::GX_SMEM));
    MHC_CUDA_CHECK(cudaFuncSetAttribute(bwd32_gphi_kernel<N>,
                                        cudaFuncAttributeMaxDynamicSharedMemorySize, C::GP_SMEM));
    attr_set[dev] = true;
  }
  const int64_t total_gx = cdiv(T, 128) * (HC / C::CB);
  int ngx = sm_count();
  if (total_gx < ngx) ngx = (int)total_gx;
  auto kgx = a.grad_x_acc ? bwd32_gx_kernel<N, true> : bwd32_gx_kernel<N, false>;
  launch(kgx, ngx, C::GX_THREADS, C::GX_SMEM, s, mx, a.inv_rms, coef, a.pre, T, D, total_gx);
  MHC_LAUNCH_CHECK();
  launch(bwd32_gphi_kernel<N>, geo.grid_gp, C::GP_THREADS, C::GP_SMEM, s, mp, w.part,
         geo.ntiles, geo.total_gp, geo.maxslot);
  MHC_LAUNCH_CHECK();
  launch(bwd32_gphi_reduce_kernel<N>, (unsigned)cdiv((int64_t)C::HM * HC, 256), 256, 0, s,
         w.part, a.grad_phi, HC, geo.ntiles, geo.total_gp, (int64_t)geo.grid_gp, geo.maxslot);
  MHC_LAUNCH_CHECK();
  return MHC_OK;
}

int pre_bwd_tc32_main(const PreBwdArgs& a, void* ws, const float* gm, const float* coef,
                      cudaStream_t s) {
  if (a.N == 8) return pre_bwd_tc32_run<8>(a, ws, gm, coef, s);
  return pre_bwd_tc32_run<4>(a, ws, gm, coef, s);
}

int pre_bwd_tc32_device_error() { return read_and_clear_tu_error(); }

}  // namespace mhc

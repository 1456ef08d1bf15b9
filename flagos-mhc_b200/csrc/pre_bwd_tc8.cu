// pre_bwd_tc8.cu -- mhc_pre_clamp_sinkhorn backward, tensor-core main pass for N = 8
// (hcMix = 80, bf16 or fp16 x, D % 64 == 0).
//
// After pass 1 (pre_bwd.cu: grad_pre dots + small-stage VJP, which writes grad_mixes
// and coef in fp32), two streaming tcgen05 kernels produce grad_x and grad_phi:
//
//   bwd8_gx_kernel    a 128-token tile at a time, over all columns in 64-column steps:
//                       gxs = G'(128 x 256) P'(256 x 64)      (M=128 tokens, N=64, K=256)
//                       grad_x = pre[n] gy + inv gxs - coef x  (epilogue)
//                     G' = [g_hi | g_lo | g_hi | 0] stays in shared memory for the tile,
//                     P' = [phi_hi ; phi_hi ; phi_lo ; 0] of each step (16.8 MB at D=4096,
//                     L2-resident) streams through a double buffer, so the three bf16
//                     products reproduce the fp32 contraction to ~2^-17 per term.
//   bwd8_gphi_kernel  a 256-column tile at a time, over token tiles:
//                       D[c, k] += x^T(c, t) Gp(t, k)          (M=128 columns x2, N=160
//                       = (inv g)_hi | (inv g)_lo, K = 128 tokens per step; both operands
//                       MN-major straight from the TMA tiles)
//                     accumulated in TMEM for at most 32 token tiles (256 chained MMAs),
//                     then folded into fp32 registers; each CTA writes one partial per
//                     column tile it touches, and bwd8_gphi_reduce_kernel sums them in a
//                     fixed order (deterministic).
//
// Why not the N=4 single pass: grad_phi of one column range over all eight sub-chunks
// needs 8 x 160 fp32 TMEM columns, more than TMEM holds next to the gxs accumulators.
// Splitting the contractions costs one more read of x; both kernels stream it at HBM
// rate, and the tensor pipes stay under half busy.
#include "pre_common.cuh"
#include "tc.cuh"

namespace mhc {

// fp16 operand maxima (pre_bwd_tc.cu)
__global__ void pre_bwd_f16_max_kernel(const float* __restrict__ phi, int64_t nphi,
                                       const float* __restrict__ gm,
                                       const float* __restrict__ inv_rms, int64_t T, int hm,
                                       unsigned* __restrict__ scl);

namespace bwd8 {
constexpr int N = 8;
constexpr int HM = 80;
constexpr int KG = 256;   // gxs K (240 used)
constexpr int GPW = 192;  // Gp row width (160 used)
constexpr int NPH = 160;  // grad_phi MMA N
constexpr int CB = 64;    // columns per gx step
constexpr int SUBT = 32;  // token tiles per grad_phi TMEM segment

// ---- gx kernel
namespace gx {
constexpr int G_ATOM = 128 * 64 * 2;       // [128 tok][64 k] SW128
constexpr int G_BYTES = 4 * G_ATOM;        // 64 KB
constexpr int P_ATOM = 64 * 64 * 2;        // [64 col][64 k] SW128
constexpr int P_BYTES = 4 * P_ATOM;        // 32 KB
constexpr int X_BYTES = 128 * 64 * 2;      // [128 tok][64 col] SW128
constexpr int GY_BYTES = 128 * 64 * 2;
constexpr int OUT_BYTES = 32 * 32 * 2;     // per epilogue warp, 64B swizzle
constexpr int EPI_WARPS = 8;
constexpr int THREADS = 32 * (2 + EPI_WARPS);
constexpr int PS = 2, XS = 4;
constexpr int OFF_G = 0;
constexpr int OFF_P = OFF_G + G_BYTES;
constexpr int OFF_X = OFF_P + PS * P_BYTES;
constexpr int OFF_GY = OFF_X + XS * X_BYTES;
constexpr int OFF_OUT = OFF_GY + GY_BYTES;
constexpr int OFF_BAR = OFF_OUT + EPI_WARPS * OUT_BYTES;
constexpr int SMEM = 1024 + OFF_BAR + 512;
constexpr int TMEM_COLS = 128;             // D1[2] x 64 columns
static_assert(SMEM <= 232448, "shared memory");
}  // namespace gx

// ---- grad_phi kernel
namespace gp {
constexpr int CT = 256;                    // columns per tile
constexpr int XBOX = 128 * 64 * 2;         // [128 tok][64 col]
constexpr int X_BYTES = 4 * XBOX;          // 64 KB
constexpr int GBOX = 128 * 64 * 2;         // [128 tok][64 k]
constexpr int G_BYTES = 3 * GBOX;          // 48 KB
constexpr int STAGE = X_BYTES + G_BYTES;
constexpr int S = 2;
constexpr int EPI_WARPS = 8;
constexpr int THREADS = 32 * (2 + EPI_WARPS);
constexpr int OFF_BAR = S * STAGE;
constexpr int SMEM = 1024 + OFF_BAR + 256;
constexpr int TMEM_COLS = 512;             // D[2] x 160 columns
static_assert(SMEM <= 232448, "shared memory");
}  // namespace gp
}  // namespace bwd8

// phi (fp32 [80][HC]) -> P' [HC][256] (E = bf16 or fp16): [phi_hi | phi_hi | phi_lo | 0]
// per column.  Thread per (column, 8-element chunk): the 16-byte stores of a warp are
// contiguous.  fp16: phi is scaled by 2^s from max|phi| (scl[0]) first, so that the lo
// halves stay clear of fp16's subnormal range; the epilogue divides it out (exact).
template <typename E>
__global__ void bwd8_phi_prep_kernel(const float* __restrict__ phi, E* __restrict__ p,
                                     int64_t HC, const unsigned* __restrict__ scl) {
  pdl_enter();
  using namespace bwd8;
  const float sc = scl ? f16_operand_scale(scl[0]) : 1.f;
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= HC * (KG / 8)) return;
  const int64_t c = i / (KG / 8);
  const int j = (int)(i - c * (KG / 8));
  float v[8];
#pragma unroll
  for (int e = 0; e < 8; ++e) {
    const int k = 8 * j + e;
    float r = 0.f;
    if (k < 2 * HM) {
      r = from_e(to_e<E>(phi[(int64_t)(k % HM) * HC + c] * sc));
    } else if (k < 3 * HM) {
      const float f = phi[(int64_t)(k - 2 * HM) * HC + c] * sc;
      r = f - from_e(to_e<E>(f));
    }
    v[e] = r;
  }
  reinterpret_cast<uint4*>(p + c * KG)[j] = narrow<E>(v);
}

// grad_mixes (fp32 [T][80]) and inv_rms -> G' [T][256] = [g_hi | g_lo | g_hi | 0] and
// Gp [T][192] = [(inv g)_hi | (inv g)_lo | 0] (E).  Thread per (token, 8-chunk).  fp16:
// g and inv g are scaled by 2^s from their maxima (scl[1], scl[2]).
template <typename E>
__global__ void bwd8_g_prep_kernel(const float* __restrict__ gm, const float* __restrict__ inv_rms,
                                   E* __restrict__ g, E* __restrict__ gpo,
                                   int64_t T, const unsigned* __restrict__ scl) {
  pdl_enter();
  using namespace bwd8;
  const float sg = scl ? f16_operand_scale(scl[1]) : 1.f;
  const float sgp = scl ? f16_operand_scale(scl[2]) : 1.f;
  constexpr int CH = KG / 8 + GPW / 8;  // 56 chunks per token
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= T * CH) return;
  const int64_t t = i / CH;
  const int j = (int)(i - t * CH);
  const float* gr = gm + t * HM;
  float v[8];
  if (j < KG / 8) {
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      const int k = 8 * j + e;
      float r = 0.f;
      if (k < 3 * HM) {
        const float f = gr[k % HM] * sg;
        const float hi = from_e(to_e<E>(f));
        r = (k >= HM && k < 2 * HM) ? f - hi : hi;
      }
      v[e] = r;
    }
    reinterpret_cast<uint4*>(g + t * KG)[j] = narrow<E>(v);
  } else {
    const int jj = j - KG / 8;
    const float inv = inv_rms[t];
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      const int k = 8 * jj + e;
      float r = 0.f;
      if (k < 2 * HM) {
        const float f = gr[k % HM] * inv * sgp;
        const float hi = from_e(to_e<E>(f));
        r = k < HM ? hi : f - hi;
      }
      v[e] = r;
    }
    reinterpret_cast<uint4*>(gpo + t * GPW)[jj] = narrow<E>(v);
  }
}

struct Bwd8GxMaps {
  CUtensorMap x, gy, g, p, gx, gxa;
};

// Step cursor of the gx kernel: step = (token tile, column block b, sub-chunk n) with n
// fastest, so one grad_y block serves N consecutive steps.
struct Gx8Cursor {
  int64_t tile, j, S;
  int blk, n;
  bool tile_start, blk_start;
  __device__ void init(int64_t gs, int64_t steps_per_tile) {
    S = steps_per_tile;
    tile = gs / S;
    j = gs - tile * S;
    blk = (int)(j / bwd8::N);
    n = (int)(j - (int64_t)blk * bwd8::N);
    tile_start = blk_start = true;
  }
  __device__ void next() {
    tile_start = blk_start = false;
    ++j;
    if (++n == bwd8::N) { n = 0; ++blk; blk_start = true; }
    if (j == S) { j = 0; blk = 0; n = 0; ++tile; tile_start = blk_start = true; }
  }
};

// E: bf16 or fp16 (x, grad_y, grad_x and the operand rows).  scl: fp16 only, the
// operand maxima; gxs then carries the factor 2^(s_g + s_phi), divided out with inv.
template <bool ACC, typename E>
__global__ void __launch_bounds__(bwd8::gx::THREADS, 1)
bwd8_gx_kernel(const __grid_constant__ Bwd8GxMaps maps, const float* __restrict__ inv_rms,
               const float* __restrict__ coef, const float* __restrict__ pre, int64_t T,
               int64_t D, int64_t total_steps, const unsigned* __restrict__ scl) {
  pdl_enter();
  using namespace bwd8;
  using namespace bwd8::gx;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* sm = (uint8_t*)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
  uint64_t* bar = (uint64_t*)(sm + OFF_BAR);
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
    tc::tmem_alloc(tmem_slot, TMEM_COLS);
    tc::tmem_relinquish();
  }
  tc::tc_fence_before();
  __syncthreads();
  tc::tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    // ------------------------------------------------------------ TMA producer
    if (lane == 0) {
      Gx8Cursor c;
      c.init(s0, S);
      uint32_t gi = 0, yi = 0;
      const uint64_t pol_stream = tc::l2_evict_first(), pol_keep = tc::l2_evict_last();
      for (int64_t gs = s0; gs < s1; ++gs, c.next()) {
        const uint32_t k = (uint32_t)(gs - s0);
        const int row = (int)(c.tile * 128);
        const int col = (int)(c.n * D + c.blk * CB);
        if (c.tile_start) {
          if (!tc::mbar_wait(gempty, (gi & 1) ^ 1, abort_flag)) break;
          tc::mbar_arrive_expect_tx(gfull, G_BYTES);
          for (int a = 0; a < 4; ++a)
            tc::tma_load_2d_hint(sm + OFF_G + a * G_ATOM, &maps.g, gfull, 64 * a, row, pol_keep);
          ++gi;
        }
        if (c.blk_start) {
          if (!tc::mbar_wait(yempty, (yi & 1) ^ 1, abort_flag)) break;
          tc::mbar_arrive_expect_tx(yfull, GY_BYTES);
          tc::tma_load_2d_hint(sm + OFF_GY, &maps.gy, yfull, c.blk * CB, row, pol_stream);
          ++yi;
        }
        const int pb = k % PS;
        if (!tc::mbar_wait(&pempty[pb], ((k / PS) & 1) ^ 1, abort_flag)) break;
        tc::mbar_arrive_expect_tx(&pfull[pb], P_BYTES);
        for (int a = 0; a < 4; ++a)
          tc::tma_load_2d_hint(sm + OFF_P + pb * P_BYTES + a * P_ATOM, &maps.p, &pfull[pb], 64 * a,
                               col, pol_keep);
        const int s = k % XS;
        if (!tc::mbar_wait(&xempty[s], ((k / XS) & 1) ^ 1, abort_flag)) break;
        tc::mbar_arrive_expect_tx(&xfull[s], X_BYTES);
        tc::tma_load_2d_hint(sm + OFF_X + s * X_BYTES, &maps.x, &xfull[s], col, row, pol_stream);
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t idesc = tc::idesc_16<E>(128, CB, false, false);
      const uint32_t sg = tc::smem_u32(sm + OFF_G), sp = tc::smem_u32(sm + OFF_P);
      Gx8Cursor c;
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
        const uint32_t d1 = tmem + e * CB;
#pragma unroll
        for (int a = 0; a < 4; ++a) {
          const uint64_t da = tc::smem_desc(sg + a * G_ATOM, 16, 1024, tc::kSwizzle128);
          const uint64_t db = tc::smem_desc(sp + pb * P_BYTES + a * P_ATOM, 16, 1024,
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
    // lane quarter q (TMEM lanes 32q..), column half hh (32 of the step's 64 columns)
    const int q = warp & 3, hh = (warp - 2) >> 2;
    const int r = q * 32 + lane;
    uint8_t* ob = sm + OFF_OUT + (warp - 2) * OUT_BYTES;
    uint8_t* orow = ob + lane * 64;
    const int osw = (lane >> 1) & 3;
    uint64_t* mybar = &accbar[warp - 2];
    uint32_t ai = 0;  // grad_x_acc boxes this warp loaded
    Gx8Cursor c;
    c.init(s0, S);
    uint32_t yi = 0;
    float inv = 0.f, cf = 0.f;
    const float unscale =
        scl ? 1.f / (f16_operand_scale(scl[1]) * f16_operand_scale(scl[0])) : 1.f;
    uint4 gyv[4];
    for (int64_t gs = s0; gs < s1; ++gs, c.next()) {
      const uint32_t k = (uint32_t)(gs - s0);
      const int64_t t = c.tile * 128 + r;
      const bool live = t < T;
      if (c.tile_start) {
        inv = live ? inv_rms[t] * unscale : 0.f;
        cf = live ? coef[t] : 0.f;
      }
      const float prn = live ? pre[t * N + c.n] : 0.f;
      const int e = k & 1, s = k % XS;
      // accumulate mode: this warp's grad_x_acc box goes into its output buffer (once the
      // previous grad_x store has read it), overlapping the waits below
      const int64_t row0 = c.tile * 128 + q * 32;
      const bool ld_acc = ACC && row0 < T;
      if (ld_acc && lane == 0) {
        tc::bulk_wait_read<0>();
        tc::mbar_arrive_expect_tx(mybar, OUT_BYTES);
        tc::tma_load_2d(ob, &maps.gxa, mybar, (int)(c.n * D + c.blk * CB + hh * 32), (int)row0);
      }
      if (!__all_sync(0xffffffffu, tc::mbar_wait(&d1full[e], (k >> 1) & 1, abort_flag))) break;
      tc::tc_fence_after();
      // row r, columns [32hh, 32hh+32) of a [128][64] 128B-swizzled tile
      const int rsw = r & 7;
      if (c.blk_start) {
        if (!__all_sync(0xffffffffu, tc::mbar_wait(yfull, yi & 1, abort_flag))) break;
        const uint8_t* yrow = sm + OFF_GY + r * 128;
#pragma unroll
        for (int jv = 0; jv < 4; ++jv)
          gyv[jv] = *reinterpret_cast<const uint4*>(yrow + (((4 * hh + jv) ^ rsw) << 4));
      }
      if (!__all_sync(0xffffffffu, tc::mbar_wait(&xfull[s], (k / XS) & 1, abort_flag))) break;
      const uint8_t* xrow = sm + OFF_X + s * X_BYTES + r * 128;
      uint4 xv[4];
#pragma unroll
      for (int jv = 0; jv < 4; ++jv)
        xv[jv] = *reinterpret_cast<const uint4*>(xrow + (((4 * hh + jv) ^ rsw) << 4));
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
      const uint32_t ta = tmem + ((uint32_t)(q * 32) << 16) + e * CB + hh * 32;
      const float2 pr2 = make_float2(prn, prn), inv2 = make_float2(inv, inv),
                   ncf2 = make_float2(-cf, -cf);
#pragma unroll
      for (int jp = 0; jp < 2; ++jp) {
        float acc[16];
        tc::tmem_ld16(ta + 16 * jp, acc);
        tc::tmem_ld_wait();
        if (jp == 1) {
          tc::tc_fence_before();
          __syncwarp();
          if (lane == 0) tc::mbar_arrive(&d1empty[e]);
        }
#pragma unroll
        for (int jj = 0; jj < 2; ++jj) {
          const int jv = 2 * jp + jj;
          float xf[8], gf[8], o[8];
          widen<E>(xv[jv], xf);
          widen<E>(gyv[jv], gf);
#pragma unroll
          for (int u = 0; u < 8; u += 2) {
            const float2 cx = __fmul2_rn(ncf2, make_float2(xf[u], xf[u + 1]));
            const float2 rr =
                __ffma2_rn(inv2, make_float2(acc[8 * jj + u], acc[8 * jj + u + 1]), cx);
            const float2 oo = __ffma2_rn(make_float2(gf[u], gf[u + 1]), pr2, rr);
            o[u] = oo.x;
            o[u + 1] = oo.y;
          }
          if (ld_acc) {
            float a8[8];
            widen<E>(*reinterpret_cast<const uint4*>(orow + ((jv ^ osw) << 4)), a8);
#pragma unroll
            for (int u = 0; u < 8; ++u) o[u] += a8[u];
          }
          *reinterpret_cast<uint4*>(orow + ((jv ^ osw) << 4)) = narrow<E>(o);
        }
      }
      tc::fence_proxy_async();  // generic smem writes -> TMA store reads
      __syncwarp();
      if (lane == 0 && row0 < T) {
        tc::tma_store_2d(&maps.gx, ob, (int)(c.n * D + c.blk * CB + hh * 32), (int)row0);
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
    tc::tmem_dealloc(tmem, TMEM_COLS);
  }
}

struct Bwd8GpMaps {
  CUtensorMap x, gp;
};

// grad_phi work: step = (256-column tile ct, token tile) with token tiles fastest; CTA b
// owns steps [total*b/G, total*(b+1)/G).  Partial slot of CTA b for tile ct =
// b - (first CTA that touches ct).
__host__ __device__ inline int64_t bwd8_cta_of_step(int64_t s, int64_t total, int64_t G) {
  return ((s + 1) * G - 1) / total;
}

template <typename E>
__global__ void __launch_bounds__(bwd8::gp::THREADS, 1)
bwd8_gphi_kernel(const __grid_constant__ Bwd8GpMaps maps, float* __restrict__ part,
                 int64_t ntiles, int64_t total_steps, int maxslot) {
  pdl_enter();
  using namespace bwd8;
  using namespace bwd8::gp;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* sm = (uint8_t*)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
  uint64_t* bar = (uint64_t*)(sm + OFF_BAR);
  uint64_t* full = bar;            // [S]
  uint64_t* empty = full + S;      // [S] the step's MMAs are done with the stage
  uint64_t* dfull = empty + S;     // segment accumulated in TMEM
  uint64_t* dempty = dfull + 1;    // epilogue folded it into registers
  uint64_t* tdone = dfull + 2;
  uint32_t* tmem_slot = (uint32_t*)(dfull + 3);
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
    tc::mbar_init(dfull, 1);
    tc::mbar_init(dempty, EPI_WARPS);
    tc::mbar_init(tdone, 1);
    *abort_flag = 0;
    tc::fence_barrier_init();
  }
  if (warp == 0 && lane == 0) {
    tc::prefetch_tmap(&maps.x);
    tc::prefetch_tmap(&maps.gp);
  }
  if (warp == 1) {
    tc::tmem_alloc(tmem_slot, TMEM_COLS);
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
    if (lane == 0) {
      int64_t ct = s0 / ntiles, tile = s0 - ct * ntiles;
      const uint64_t pol_stream = tc::l2_evict_first(), pol_keep = tc::l2_evict_last();
      for (int64_t gs = s0; gs < s1; ++gs) {
        const uint32_t k = (uint32_t)(gs - s0);
        const int s = k % S;
        if (!tc::mbar_wait(&empty[s], ((k / S) & 1) ^ 1, abort_flag)) break;
        tc::mbar_arrive_expect_tx(&full[s], STAGE);
        uint8_t* st = sm + s * STAGE;
        for (int b = 0; b < 4; ++b)
          tc::tma_load_2d_hint(st + b * XBOX, &maps.x, &full[s], (int)(ct * CT + 64 * b),
                               (int)(tile * 128), pol_stream);
        for (int b = 0; b < 3; ++b)
          tc::tma_load_2d_hint(st + X_BYTES + b * GBOX, &maps.gp, &full[s], 64 * b,
                               (int)(tile * 128), pol_keep);
        if (++tile == ntiles) { tile = 0; ++ct; }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t idesc = tc::idesc_16<E>(128, NPH, true, true);
      const uint32_t sbase = tc::smem_u32(sm);
      int64_t ct = s0 / ntiles, tile = s0 - ct * ntiles;
      uint32_t seg = 0;
      bool seg_first = true;
      for (int64_t gs = s0; gs < s1; ++gs) {
        const uint32_t k = (uint32_t)(gs - s0);
        const int s = k % S;
        if (seg_first && !tc::mbar_wait(dempty, (seg & 1) ^ 1, abort_flag)) break;
        if (!tc::mbar_wait(&full[s], (k / S) & 1, abort_flag)) break;
        tc::tc_fence_after();
        const uint32_t sx = sbase + s * STAGE, sgp = sx + X_BYTES;
#pragma unroll
        for (int m = 0; m < 2; ++m) {
#pragma unroll
          for (int kk = 0; kk < 8; ++kk) {
            const uint64_t ax = tc::smem_desc(sx + m * 2 * XBOX + kk * 2048, XBOX, 1024,
                                              tc::kSwizzle128);
            const uint64_t bg = tc::smem_desc(sgp + kk * 2048, GBOX, 1024, tc::kSwizzle128);
            tc::mma_bf16(tmem + m * NPH, ax, bg, idesc, (seg_first && kk == 0) ? 0u : 1u);
          }
        }
        tc::mma_commit(&empty[s]);
        seg_first = false;
        if (seg_end(gs, tile)) {
          tc::mma_commit(dfull);
          ++seg;
          seg_first = true;
        }
        if (++tile == ntiles) { tile = 0; ++ct; }
      }
      tc::mma_commit(tdone);
      volatile int never = 0;
      tc::mbar_wait(tdone, 0, &never);
    }
  } else {
    // epilogue: lane quarter q, column half m; thread = column m*128 + 32q + lane of the
    // tile.  Folds each segment (hi + lo) into fp32 registers; writes the CTA's partial
    // for a column tile when its last step in that tile is done.
    const int q = warp & 3, m = (warp - 2) >> 2;
    const int cl = m * 128 + q * 32 + lane;
    float acc[HM];
#pragma unroll
    for (int kx = 0; kx < HM; ++kx) acc[kx] = 0.f;
    int64_t ct = s0 / ntiles, tile = s0 - ct * ntiles;
    uint32_t seg = 0;
    for (int64_t gs = s0; gs < s1; ++gs) {
      const bool last_in_ct = gs == s1 - 1 || tile == ntiles - 1;
      if (seg_end(gs, tile)) {
        if (!__all_sync(0xffffffffu, tc::mbar_wait(dfull, seg & 1, abort_flag))) break;
        tc::tc_fence_after();
        const uint32_t ta = tmem + ((uint32_t)(q * 32) << 16) + m * NPH;
#pragma unroll
        for (int c16 = 0; c16 < HM / 16; ++c16) {
          float hi[16], lo[16];
          tc::tmem_ld16(ta + 16 * c16, hi);
          tc::tmem_ld16(ta + HM + 16 * c16, lo);
          tc::tmem_ld_wait();
#pragma unroll
          for (int u = 0; u < 16; ++u) acc[16 * c16 + u] += hi[u] + lo[u];
        }
        tc::tc_fence_before();
        __syncwarp();
        if (lane == 0) tc::mbar_arrive(dempty);
        ++seg;
        if (last_in_ct) {
          const int64_t slot =
              (int64_t)blockIdx.x - bwd8_cta_of_step(ct * ntiles, total_steps, G);
          float* dst = part + ((ct * maxslot + slot) * HM) * CT + cl;
#pragma unroll
          for (int kx = 0; kx < HM; ++kx) {
            dst[(int64_t)kx * CT] = acc[kx];
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
    tc::tmem_dealloc(tmem, TMEM_COLS);
  }
}

// grad_phi[k][ct*256 + cc] = sum over the CTAs that touched column tile ct, in CTA order.
__global__ void bwd8_gphi_reduce_kernel(const float* __restrict__ part, float* __restrict__ gphi,
                                        int64_t HC, int64_t ntiles, int64_t total_steps,
                                        int64_t G, int maxslot,
                                        const unsigned* __restrict__ scl) {
  pdl_enter();
  using namespace bwd8;
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= (int64_t)HM * HC) return;
  const int64_t kx = i / HC, c = i - kx * HC;
  const int64_t ct = c / gp::CT, cc = c - ct * gp::CT;
  const int64_t b0 = bwd8_cta_of_step(ct * ntiles, total_steps, G);
  const int64_t b1 = bwd8_cta_of_step(ct * ntiles + ntiles - 1, total_steps, G);
  Kahan k;
  for (int64_t sl = 0; sl <= b1 - b0; ++sl) k.add(part[((ct * maxslot + sl) * HM + kx) * gp::CT + cc]);
  float s = k.s;
  if (scl) s *= 1.f / f16_operand_scale(scl[2]);  // exact: a power of two
  gphi[i] = s;
}

// ---------------------------------------------------------------------------
// Host side
// ---------------------------------------------------------------------------
bool pre_bwd_tc8_eligible(const PreBwdArgs& a) {
  const int64_t T = a.T, D = a.D;
  return (a.dtype == MHC_BF16 || a.dtype == MHC_F16) && a.N == 8 && D % bwd8::CB == 0 && T > 0 &&
         T <= (int64_t)INT32_MAX - 256 && (int64_t)a.N * D <= INT32_MAX &&
         rows_aligned(a.x, a.x_ts, 2, 16) && rows_aligned(a.grad_y, a.gy_ts, 2, 16) &&
         aligned16(a.grad_x);
}

struct Bwd8Geom {
  int64_t ntiles, ncol, total_gp;
  int grid_gp, maxslot;
};

static Bwd8Geom bwd8_geometry(int64_t T, int64_t D) {
  Bwd8Geom g;
  g.ntiles = cdiv(T, 128);
  g.ncol = (bwd8::N * D) / bwd8::gp::CT;
  g.total_gp = g.ncol * g.ntiles;
  int n = sm_count();
  if (g.total_gp < n) n = (int)g.total_gp;
  g.grid_gp = n < 1 ? 1 : n;
  // most CTAs that touch one column tile (partial slots per tile)
  g.maxslot = 1;
  for (int64_t ct = 0; ct < g.ncol; ++ct) {
    const int64_t b0 = bwd8_cta_of_step(ct * g.ntiles, g.total_gp, g.grid_gp);
    const int64_t b1 = bwd8_cta_of_step(ct * g.ntiles + g.ntiles - 1, g.total_gp, g.grid_gp);
    if (b1 - b0 + 1 > g.maxslot) g.maxslot = (int)(b1 - b0 + 1);
  }
  return g;
}

struct Bwd8Ws {
  __nv_bfloat16 *g, *gp, *p;  // fp16 x: the same buffers hold fp16 rows
  float* part;
  unsigned* scl;  // fp16: max |phi|, |grad_mixes|, |inv * grad_mixes| (float bits)
  size_t total;
};

static Bwd8Ws bwd8_layout(char* base, int64_t T, int64_t D) {
  using namespace bwd8;
  const Bwd8Geom geo = bwd8_geometry(T, D);
  const int64_t HC = N * D;
  Bwd8Ws w;
  size_t off = 0;
  auto take = [&](size_t bytes) { char* p = base + off; off += align_up(bytes); return p; };
  w.g = (__nv_bfloat16*)take((size_t)T * KG * 2);
  w.gp = (__nv_bfloat16*)take((size_t)T * GPW * 2);
  w.p = (__nv_bfloat16*)take((size_t)HC * KG * 2);
  w.part = (float*)take((size_t)geo.ncol * geo.maxslot * HM * gp::CT * 4);
  w.scl = (unsigned*)take(256);
  w.total = off;
  return w;
}

size_t pre_bwd_tc8_ws_bytes(int64_t T, int64_t D) { return bwd8_layout(nullptr, T, D).total; }

template <typename E>
static int pre_bwd_tc8_run(const PreBwdArgs& a, void* ws, const float* gm, const float* coef,
                           cudaStream_t s) {
  using namespace bwd8;
  constexpr bool f16 = std::is_same<E, __half>::value;
  const int64_t T = a.T, D = a.D, HC = N * D;
  const Bwd8Geom geo = bwd8_geometry(T, D);
  Bwd8Ws w = bwd8_layout((char*)ws, T, D);
  const unsigned* scl = f16 ? w.scl : nullptr;
  if (f16) {
    MHC_CUDA_CHECK(cudaMemsetAsync(w.scl, 0, 3 * sizeof(unsigned), s));
    const int64_t n = std::max<int64_t>((int64_t)HM * HC, T * HM);
    launch(pre_bwd_f16_max_kernel,
           (unsigned)std::min<int64_t>(cdiv(n, 256), (int64_t)sm_count() * 4), 256, 0, s,
           a.phi, (int64_t)HM * HC, gm, a.inv_rms, T, HM, w.scl);
    MHC_LAUNCH_CHECK();
  }
  launch(bwd8_phi_prep_kernel<E>, (unsigned)cdiv(HC * (KG / 8), 256), 256, 0, s, a.phi,
         (E*)w.p, HC, scl);
  MHC_LAUNCH_CHECK();
  launch(bwd8_g_prep_kernel<E>, (unsigned)cdiv(T * (KG / 8 + GPW / 8), 256), 256, 0, s,
         gm, a.inv_rms, (E*)w.g, (E*)w.gp, T, scl);
  MHC_LAUNCH_CHECK();

  const CUtensorMapDataType bf =
      f16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
  int st;
  Bwd8GxMaps mx;
  if ((st = make_tmap_2d(&mx.x, a.x, bf, 2, HC, T, a.x_ts * 2, 64, 128,
                         CU_TENSOR_MAP_SWIZZLE_128B)))
    return st;
  if ((st = make_tmap_2d(&mx.gy, a.grad_y, bf, 2, D, T, a.gy_ts * 2, 64, 128,
                         CU_TENSOR_MAP_SWIZZLE_128B)))
    return st;
  if ((st = make_tmap_2d(&mx.g, w.g, bf, 2, KG, T, KG * 2, 64, 128, CU_TENSOR_MAP_SWIZZLE_128B)))
    return st;
  if ((st = make_tmap_2d(&mx.p, w.p, bf, 2, KG, HC, KG * 2, 64, 64, CU_TENSOR_MAP_SWIZZLE_128B)))
    return st;
  if ((st = make_tmap_2d(&mx.gx, a.grad_x, bf, 2, HC, T, HC * 2, 32, 32,
                         CU_TENSOR_MAP_SWIZZLE_64B)))
    return st;
  mx.gxa = mx.gx;
  if (a.grad_x_acc &&
      (st = make_tmap_2d(&mx.gxa, a.grad_x_acc, bf, 2, HC, T, HC * 2, 32, 32,
                         CU_TENSOR_MAP_SWIZZLE_64B)))
    return st;
  Bwd8GpMaps mp;
  if ((st = make_tmap_2d(&mp.x, a.x, bf, 2, HC, T, a.x_ts * 2, 64, 128,
                         CU_TENSOR_MAP_SWIZZLE_128B)))
    return st;
  if ((st = make_tmap_2d(&mp.gp, w.gp, bf, 2, GPW, T, GPW * 2, 64, 128,
                         CU_TENSOR_MAP_SWIZZLE_128B)))
    return st;

  static bool attr_set[64];
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 0 && dev < 64 && !attr_set[dev]) {
    MHC_CUDA_CHECK(cudaFuncSetAttribute(bwd8_gx_kernel<false, E>,
                                        cudaFuncAttributeMaxDynamicSharedMemorySize, gx::SMEM));
    MHC_CUDA_CHECK(cudaFuncSetAttribute(bwd8_gx_kernel<true, E>,
                                        cudaFuncAttributeMaxDynamicSharedMemorySize, gx::SMEM));
    MHC_CUDA_CHECK(cudaFuncSetAttribute(bwd8_gphi_kernel<E>,
                                        cudaFuncAttributeMaxDynamicSharedMemorySize, gp::SMEM));
    attr_set[dev] = true;
  }
  const int64_t total_gx = geo.ntiles * (HC / CB);
  int ngx = sm_count();
  if (total_gx < ngx) ngx = (int)total_gx;
  auto kgx = a.grad_x_acc ? bwd8_gx_kernel<true, E> : bwd8_gx_kernel<false, E>;
  launch(kgx, ngx, gx::THREADS, gx::SMEM, s, mx, a.inv_rms, coef, a.pre, T, D, total_gx, scl);
  MHC_LAUNCH_CHECK();
  launch(bwd8_gphi_kernel<E>, geo.grid_gp, gp::THREADS, gp::SMEM, s, mp, w.part, geo.ntiles,
                                                              geo.total_gp, geo.maxslot);
  MHC_LAUNCH_CHECK();
  launch(bwd8_gphi_reduce_kernel, (unsigned)cdiv((int64_t)HM * HC, 256), 256, 0, s, 
      w.part, a.grad_phi, HC, geo.ntiles, geo.total_gp, geo.grid_gp, geo.maxslot, scl);
  MHC_LAUNCH_CHECK();
  return MHC_OK;
}

int pre_bwd_tc8_main(const PreBwdArgs& a, void* ws, const float* gm, const float* coef,
                     cudaStream_t s) {
  if (a.dtype == MHC_F16) return pre_bwd_tc8_run<__half>(a, ws, gm, coef, s);
  return pre_bwd_tc8_run<__nv_bfloat16>(a, ws, gm, coef, s);
}

int pre_bwd_tc8_device_error() { return read_and_clear_tu_error(); }

}  // namespace mhc

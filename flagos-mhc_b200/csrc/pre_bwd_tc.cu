// pre_bwd_tc.cu -- mhc_pre_clamp_sinkhorn backward, tensor-core main pass (bf16, N=4,
// D % 128 == 0).
//
// After pass 1 (pre_bwd.cu: grad_pre dots + small-stage VJP, which also writes the
// bf16 hi/lo operand rows below), one persistent kernel streams x once more and
// produces grad_x and grad_phi together:
//
//   gxs[t,c]    = sum_k grad_mixes[t,k] phi[k,c]        (tcgen05, M=128 tokens, N=128
//                 columns, K=80: A' = [g_hi|g_lo|g_hi], B' = [phi_hi;phi_hi;phi_lo])
//   grad_x[t,c] = gy[t,d] pre[t,n] + inv[t] gxs[t,c] - coef[t] x[t,c]       (epilogue)
//   grad_phi[k,c] += sum_t gp[t,k] x[t,c],  gp = inv*grad_mixes              (tcgen05,
//                 M=128 columns, N=64 (hi 24 | lo 24 | 0), K=128 tokens; x is the
//                 MN-major A operand straight from the staged x tile)
//
// Work: column group g = a 128-wide range of d, all N=4 sub-chunks n (512 columns of
// HC); items (g, token tile i) in g-major order, split into equal contiguous runs, one
// per CTA.  Each group's tiles are cut into cells of SUBT tiles; grad_phi stays in
// TMEM (4 x 64 columns) for the part of a cell a CTA owns and is then flushed into a
// partial buffer, so no accumulation chain exceeds SUBT*8 MMAs (the tensor core's
// fp32 accumulation error grows with the chain length).  pre_bwd_gphi_reduce_kernel
// sums the partials of each column in a fixed order (deterministic).  The phi operand
// of each step (20 KB of the 4.6 MB operand rows, which stay in L2) is streamed into a
// double buffer; grad_x leaves through per-warp shared-memory boxes and TMA stores, so
// an x stage is released as soon as the epilogue and the grad_phi MMAs have read it.
//
// Roles (576 threads): warp 0 TMA producer; warp 1 TMEM owner + MMA issuer; warps 2-17
// epilogue (warp w reads TMEM lane quarter w%4, column quarter (w-2)/4).
#include "pre_common.cuh"
#include "tc.cuh"



namespace mhc {

namespace bwdtc {
constexpr int N = 4;
constexpr int HM = 24;
constexpr int GC = 128;                     // columns of d per group
constexpr int KG = 80;                      // gxs K (72 used)
constexpr int SUBT = 32;                    // max token tiles per grad_phi cell
// shared memory (bytes, offsets from a 1024-aligned base)
constexpr int P0_BYTES = 128 * 64 * 2;      // [128 cols][64 k] SW128
constexpr int P1_BYTES = 128 * 16 * 2;      // [128 cols][16 k] SW32
constexpr int G0_BYTES = 128 * 64 * 2;      // [128 tok][64 k]
constexpr int G1_BYTES = 128 * 16 * 2;      // [128 tok][16 k]
constexpr int GP_BYTES = 128 * 64 * 2;      // [128 tok][64 n]
constexpr int X_BYTES = 2 * 128 * 64 * 2;   // two [128 tok][64 col] boxes
constexpr int P_BYTES = P0_BYTES + P1_BYTES;  // phi operand of one sub-chunk (20 KB)
constexpr int OUT_BYTES = 32 * 32 * 2;      // per epilogue warp: [32 tok][32 col], 64B swizzle
constexpr int THREADS = 576;
constexpr int EPI_WARPS = 16;
constexpr int PS = 2;                       // phi operand buffers (streamed from L2 per step)
constexpr int XS = 3;                       // x stages (G is single-buffered)
constexpr int OFF_P = 0;                    // [PS] x {P0, P1}
constexpr int OFF_G0 = OFF_P + PS * P_BYTES;
constexpr int OFF_G1 = OFF_G0 + G0_BYTES;
constexpr int OFF_GP = OFF_G1 + G1_BYTES;
constexpr int OFF_X = OFF_GP + GP_BYTES;
constexpr int OFF_OUT = OFF_X + XS * X_BYTES;
constexpr int OFF_BAR = OFF_OUT + EPI_WARPS * OUT_BYTES;
constexpr int SMEM = 1024 + OFF_BAR + 512;
static_assert(SMEM <= 232448, "shared memory");
static_assert(P_BYTES % 1024 == 0 && OFF_X % 1024 == 0 && OFF_OUT % 1024 == 0, "alignment");
// TMEM columns: D2[n] (grad_phi, 64 each) at n*64, D1[b] (gxs, 128 each) at 256 + b*128
constexpr int TMEM_COLS = 512;
}  // namespace bwdtc

struct BwdTcMaps {
  CUtensorMap x, g0, g1, gp, p0, p1, gx, gxa;
};

// A cell is `subt` consecutive token tiles of one column group; subt never exceeds the
// shortest CTA run, so every cell is split across at most two CTAs: slot 0 belongs to
// the CTA holding the cell's first tile, slot 1 to a CTA whose run starts inside it.
struct BwdGeom {
  int64_t ntiles;  // 128-token tiles
  int64_t subt;    // tiles per cell
  int64_t cpg;     // cells per group
  int64_t items;   // groups * ntiles
  int ncta;
};

// Walks a CTA's items in order with counters only (no 64-bit division on the issue
// paths): column group g, token tile i in the group, position of i in its grad_phi
// cell, and whether the item starts / ends the CTA's segment of that cell.
struct ItemCursor {
  int64_t item, it0, it1, g;
  int i, isub, ntiles, subt;
  bool seg_start, seg_end;
  __device__ void flags() {
    seg_start = item == it0 || isub == 0;
    seg_end = item == it1 - 1 || isub == subt - 1 || i == ntiles - 1;
  }
  __device__ void init(int64_t a, int64_t b, int64_t nt, int64_t st) {
    item = a; it0 = a; it1 = b; ntiles = (int)nt; subt = (int)st;
    g = a / nt;
    i = (int)(a - g * nt);
    isub = i % subt;
    flags();
  }
  __device__ void next() {
    ++item;
    if (++i == ntiles) { i = 0; isub = 0; ++g; }
    else if (++isub == subt) isub = 0;
    flags();
  }
};

// E: bf16 or fp16 (x, grad_y, grad_x and the operand rows).  scl: fp16 only, the maxima
// (phi, grad_mixes, inv*grad_mixes) the operand rows were scaled by.
template <bool ACC, typename E>
__global__ void __launch_bounds__(bwdtc::THREADS, 1)
pre_bwd_tc_kernel(const __grid_constant__ BwdTcMaps maps, const E* __restrict__ gy,
                  const float* __restrict__ inv_rms, const float* __restrict__ coef,
                  const float* __restrict__ pre, E* __restrict__ gx,
                  float* __restrict__ gphi_part, int64_t T, int64_t D, BwdGeom geo,
                  const unsigned* __restrict__ scl, int64_t gys) {
  pdl_enter();
  using namespace bwdtc;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* sm = (uint8_t*)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
  uint64_t* bar = (uint64_t*)(sm + OFF_BAR);
  uint64_t* xfull = bar;             // [XS] x tile landed
  uint64_t* xempty = bar + XS;       // [XS] epilogue warps and grad_phi MMAs read the tile
  uint64_t* gfull = bar + 2 * XS;    // G0/G1 (gxs operand) of an item landed
  uint64_t* gempty = gfull + 1;      // the item's gxs MMAs are done with G0/G1
  uint64_t* pfull = gfull + 2;       // [PS] phi operand of a step landed
  uint64_t* pempty = gfull + 4;      // [PS] the step's gxs MMAs are done with it
  uint64_t* d1full = gfull + 6;      // [2]
  uint64_t* d1empty = gfull + 8;     // [2]
  uint64_t* d2full = gfull + 10;
  uint64_t* d2empty = gfull + 11;
  uint64_t* tdone = gfull + 12;
  uint64_t* gpfull = gfull + 13;     // GP (grad_phi operand) of an item landed
  uint64_t* gpempty = gfull + 14;    // the item's grad_phi MMAs are done with GP
  uint64_t* accbar = gfull + 15;     // [EPI_WARPS] the warp's grad_x_acc box landed
  uint32_t* tmem_slot = (uint32_t*)(gfull + 15 + EPI_WARPS);
  volatile int* abort_flag = (volatile int*)(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t ntiles = geo.ntiles;
  const int64_t it0 = geo.items * blockIdx.x / gridDim.x;
  const int64_t it1 = geo.items * (blockIdx.x + 1) / gridDim.x;

  if (threadIdx.x == 0) {
    for (int b = 0; b < XS; ++b) {
      tc::mbar_init(&xfull[b], 1);
      tc::mbar_init(&xempty[b], EPI_WARPS + 1);  // 16 epilogue warps + 1 MMA commit
    }
    for (int b = 0; b < 2; ++b) {
      tc::mbar_init(&d1full[b], 1);
      tc::mbar_init(&d1empty[b], EPI_WARPS);
    }
    tc::mbar_init(gfull, 1);
    tc::mbar_init(gempty, 1);
    tc::mbar_init(gpfull, 1);
    tc::mbar_init(gpempty, 1);
    for (int b = 0; b < PS; ++b) {
      tc::mbar_init(&pfull[b], 1);
      tc::mbar_init(&pempty[b], 1);
    }
    tc::mbar_init(d2full, 1);
    tc::mbar_init(d2empty, EPI_WARPS);
    tc::mbar_init(tdone, 1);
    for (int w = 0; w < EPI_WARPS; ++w) tc::mbar_init(&accbar[w], 1);
    *abort_flag = 0;
    tc::fence_barrier_init();
  }
  if (warp == 0 && lane == 0) {
    tc::prefetch_tmap(&maps.x);
    tc::prefetch_tmap(&maps.g0);
    tc::prefetch_tmap(&maps.gp);
    tc::prefetch_tmap(&maps.p0);
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

  // segment = the part of one cell this CTA owns
  const int64_t subt = geo.subt;

  if (warp == 0) {
    // ------------------------------------------------------------ TMA producer
    if (lane == 0) {
      uint32_t xi = 0, gi = 0;
      bool ok = true;
      ItemCursor cur;
      cur.init(it0, it1, ntiles, subt);
      for (; cur.item < it1 && ok; cur.next()) {
        const int i = cur.i;
        const int d0 = (int)(cur.g * GC);
        for (int n = 0; n < N; ++n, ++xi) {
          // the step's phi operand (4.6 MB in all, L2-resident): ahead of its x tile,
          // since the gxs MMAs need it one step before the x tile is used
          const int pb = xi & 1;
          if (!tc::mbar_wait(&pempty[pb], ((xi >> 1) & 1) ^ 1, abort_flag)) { ok = false; break; }
          tc::mbar_arrive_expect_tx(&pfull[pb], P_BYTES);
          uint8_t* pdst = sm + OFF_P + pb * P_BYTES;
          tc::tma_load_2d(pdst, &maps.p0, &pfull[pb], 0, (int)(n * D + d0));
          tc::tma_load_2d(pdst + P0_BYTES, &maps.p1, &pfull[pb], 0, (int)(n * D + d0));
          const int s = xi % XS;
          if (!tc::mbar_wait(&xempty[s], ((xi / XS) & 1) ^ 1, abort_flag)) { ok = false; break; }
          tc::mbar_arrive_expect_tx(&xfull[s], X_BYTES);
          uint8_t* dst = sm + OFF_X + s * X_BYTES;
          const int col = (int)(n * D + d0);
          tc::tma_load_2d(dst, &maps.x, &xfull[s], col, (int)(i * 128));
          tc::tma_load_2d(dst + X_BYTES / 2, &maps.x, &xfull[s], col + 64, (int)(i * 128));
          if (n == 0) {
            // the item's G operands (single buffers): G0/G1 once the previous item's
            // gxs MMAs are done, GP once its grad_phi MMAs are done (one step later)
            if (!tc::mbar_wait(gempty, (gi & 1) ^ 1, abort_flag)) { ok = false; break; }
            tc::mbar_arrive_expect_tx(gfull, G0_BYTES + G1_BYTES);
            tc::tma_load_2d(sm + OFF_G0, &maps.g0, gfull, 0, (int)(i * 128));
            tc::tma_load_2d(sm + OFF_G1, &maps.g1, gfull, 0, (int)(i * 128));
            if (!tc::mbar_wait(gpempty, (gi & 1) ^ 1, abort_flag)) { ok = false; break; }
            tc::mbar_arrive_expect_tx(gpfull, GP_BYTES);
            tc::tma_load_2d(sm + OFF_GP, &maps.gp, gpfull, 0, (int)(i * 128));
            ++gi;
          }
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    // Software-pipelined by one step: iteration st issues the gxs MMAs of step st (they
    // need only the per-item G and the stationary P, never x) and the grad_phi MMAs of
    // step st-1 (which need the x tile), so D1 does not wait on the x load of its step.
    if (lane == 0) {
      constexpr uint32_t id_gxs = tc::idesc_16<E>(128, 128, false, false);
      constexpr uint32_t id_gphi = tc::idesc_16<E>(128, 64, true, true);
      // step = (item, n); A runs one step ahead of B (the grad_phi step)
      struct StepPos {
        ItemCursor c;
        int n, s;          // sub-chunk, x stage
        uint32_t gi, xph;  // item index in the run, x stage phase
        __device__ void next() {
          if (++s == XS) { s = 0; xph ^= 1; }
          if (++n == N) { n = 0; ++gi; c.next(); }
        }
      };
      StepPos A, B;
      A.c.init(it0, it1, ntiles, subt);
      A.n = 0; A.s = 0; A.gi = 0; A.xph = 0;
      B = A;
      const int64_t nsteps = (it1 - it0) * N;
      uint32_t seg_b = 0;
      const uint32_t sg0 = tc::smem_u32(sm + OFF_G0), sg1 = tc::smem_u32(sm + OFF_G1);
      const uint32_t sp = tc::smem_u32(sm + OFF_P);
      const uint32_t sx0 = tc::smem_u32(sm + OFF_X), sgp = tc::smem_u32(sm + OFF_GP);
      bool ok = true;
      auto issue_gxs = [&](int64_t st) -> bool {
        // ---- gxs of step st (position A)
        const int n = A.n;
        const int e = (int)(st & 1);
        if (n == 0 && !tc::mbar_wait(gfull, A.gi & 1, abort_flag)) return false;
        if (!tc::mbar_wait(&pfull[e], (uint32_t)(st >> 1) & 1, abort_flag)) return false;
        if (!tc::mbar_wait(&d1empty[e], ((uint32_t)(st >> 1) & 1) ^ 1, abort_flag)) return false;
        tc::tc_fence_after();
        const uint32_t d1 = tmem + 256 + e * 128;
        const uint64_t a0 = tc::smem_desc(sg0, 16, 1024, tc::kSwizzle128);
        const uint32_t spb = sp + e * P_BYTES;
        const uint64_t b0 = tc::smem_desc(spb, 16, 1024, tc::kSwizzle128);
#pragma unroll
        for (int k = 0; k < 4; ++k) tc::mma_bf16(d1, a0 + 2 * k, b0 + 2 * k, id_gxs, k != 0);
        tc::mma_bf16(d1, tc::smem_desc(sg1, 16, 256, tc::kSwizzle32),
                     tc::smem_desc(spb + P0_BYTES, 16, 256, tc::kSwizzle32), id_gxs, 1);
        tc::mma_commit(&d1full[e]);
        tc::mma_commit(&pempty[e]);
        if (n == N - 1) tc::mma_commit(gempty);  // last gxs use of this item's G0/G1
        A.next();
        return true;
      };
      auto issue_gphi = [&]() -> bool {
        // ---- grad_phi of the step at position B: D2[n] (+)= x_tile^T * Gp
        const int n = B.n, s = B.s;
        const bool seg_start = B.c.seg_start;
        if (n == 0 && seg_start && !tc::mbar_wait(d2empty, (seg_b & 1) ^ 1, abort_flag)) return false;
        if (n == 0 && !tc::mbar_wait(gpfull, B.gi & 1, abort_flag)) return false;
        if (!tc::mbar_wait(&xfull[s], B.xph, abort_flag)) return false;
        tc::tc_fence_after();
        const uint32_t d2 = tmem + n * 64;
        const uint32_t sx = sx0 + s * X_BYTES;
#pragma unroll
        for (int kk = 0; kk < 8; ++kk) {
          const uint64_t ax = tc::smem_desc(sx + kk * 2048, X_BYTES / 2, 1024, tc::kSwizzle128);
          const uint64_t bg = tc::smem_desc(sgp + kk * 2048, GP_BYTES, 1024, tc::kSwizzle128);
          tc::mma_bf16(d2, ax, bg, id_gphi, (seg_start && kk == 0) ? 0u : 1u);
        }
        tc::mma_commit(&xempty[s]);
        if (n == N - 1) {
          tc::mma_commit(gpempty);
          if (B.c.seg_end) {
            tc::mma_commit(d2full);
            ++seg_b;
          }
        }
        B.next();
        return true;
      };
      for (int64_t st = 0; st <= nsteps && ok; ++st) {
        // At an item boundary the previous item's last grad_phi MMAs go first: they
        // release GP, which the producer waits for before the item's next x tiles.
        if (A.n == 0) {
          if (st >= 1 && !issue_gphi()) { ok = false; break; }
          if (st < nsteps && !issue_gxs(st)) { ok = false; break; }
        } else {
          if (st < nsteps && !issue_gxs(st)) { ok = false; break; }
          if (st >= 1 && !issue_gphi()) { ok = false; break; }
        }
      }
      tc::mma_commit(tdone);
      volatile int never = 0;
      tc::mbar_wait(tdone, 0, &never);
    }
  } else {
    // ------------------------------------------------------------ epilogue warps
    // 16 warps: lane quarter q = warp % 4 (the TMEM lanes this warp may read), column
    // quarter h = (warp - 2) / 4 (32 of the group's 128 columns).
    // fp16: gxs comes out scaled by 2^(sg + sphi); folding 2^-(sg + sphi) into inv is exact
    const float gdsc = std::is_same<E, __half>::value
                           ? 1.f / (f16_operand_scale(scl[1]) * f16_operand_scale(scl[0]))
                           : 1.f;
    const int q = warp & 3;
    const int h = (warp - 2) >> 2;
    const int r = q * 32 + lane;            // token row (D1) / column row (D2)
    uint8_t* ob = sm + OFF_OUT + (warp - 2) * OUT_BYTES;
    uint64_t* mybar = &accbar[warp - 2];
    uint32_t ai = 0;  // grad_x_acc boxes this warp loaded
    uint32_t di = 0, seg = 0;
    bool first_seg = true;
    ItemCursor cur;
    cur.init(it0, it1, ntiles, subt);
    const bool starts_inside = cur.isub != 0;  // this CTA's run began inside a cell
    // per-item operands of this lane's row: loaded one item ahead (issued right after the
    // last step of the previous item used them), so their latency hides behind the flush
    // and the barrier waits instead of stalling the first step
    float inv = 0.f, cf = 0.f, pr[N];
    uint4 gyv[4];
    auto load_item = [&](int64_t g_, int64_t i_) {
      const int64_t tt = i_ * 128 + r;
      if (tt < T) {
        inv = inv_rms[tt];
        cf = coef[tt];
#pragma unroll
        for (int n = 0; n < N; ++n) pr[n] = pre[tt * N + n];
        const E* gyr = gy + tt * gys + g_ * GC + h * 32;
        const U8 g01 = ld_global_32B(gyr), g23 = ld_global_32B(gyr + 16);
        gyv[0] = g01.a; gyv[1] = g01.b; gyv[2] = g23.a; gyv[3] = g23.b;
      } else {
        inv = 0.f;
        cf = 0.f;
#pragma unroll
        for (int n = 0; n < N; ++n) pr[n] = 0.f;
#pragma unroll
        for (int j = 0; j < 4; ++j) gyv[j] = make_uint4(0, 0, 0, 0);
      }
    };
    if (cur.item < it1) load_item(cur.g, cur.i);
    for (; cur.item < it1; cur.next()) {
      const int64_t item = cur.item, i = cur.i;
      const int64_t d0 = cur.g * GC;
      const int64_t row0 = i * 128 + q * 32;  // first token row of this warp's store box
      bool ok = true;
      for (int n = 0; n < N; ++n, ++di) {
        const int e = di & 1, s = di % XS;
        const uint32_t xph = (di / XS) & 1;
        // accumulate mode: this warp's grad_x_acc box goes into its output buffer (once
        // the previous grad_x store has read it), overlapping the waits below
        const bool ld_acc = ACC && row0 < T;
        if (ld_acc && lane == 0) {
          tc::bulk_wait_read<0>();
          tc::mbar_arrive_expect_tx(mybar, OUT_BYTES);
          tc::tma_load_2d(ob, &maps.gxa, mybar, (int)(n * D + d0 + h * 32), (int)row0);
        }
        if (!__all_sync(0xffffffffu, tc::mbar_wait(&d1full[e], (di >> 1) & 1, abort_flag))) {
          ok = false;
          break;
        }
        tc::tc_fence_after();
        if (!__all_sync(0xffffffffu, tc::mbar_wait(&xfull[s], xph, abort_flag))) {
          ok = false;
          break;
        }
        // x row r, columns [32h, 32h+32): box h/2, 16-byte chunks 4(h%2)..+3 (swizzled)
        const uint8_t* xrow = sm + OFF_X + s * X_BYTES + (h >> 1) * (X_BYTES / 2) + r * 128;
        uint4 xv[4];
#pragma unroll
        for (int j = 0; j < 4; ++j)
          xv[j] = *reinterpret_cast<const uint4*>(xrow + ((((h & 1) * 4 + j) ^ (r & 7)) << 4));
        // the stage is free once every epilogue warp has read its x and the grad_phi
        // MMAs are done (their commit is the barrier's last arrival)
        tc::fence_proxy_async();        // generic smem reads before the TMA refill
        __syncwarp();
        if (lane == 0) tc::mbar_arrive(&xempty[s]);
        // gxs in two halves of 16 columns (keeps the live registers under the 96 that
        // 18 warps per CTA allow).  grad_x goes through this warp's own 2 KB buffer
        // ([32 tok][32 col], 64-byte swizzle: chunk c of row r at (c ^ (r/2 % 4))) and
        // one TMA store per warp and step; the buffer is reused once that store has
        // read it.
        const uint32_t ta = tmem + ((uint32_t)(q * 32) << 16) + 256 + e * 128 + h * 32;
        uint8_t* orow = ob + lane * 64;
        const int osw = (lane >> 1) & 3;
        if (lane == 0) tc::bulk_wait_read<0>();
        __syncwarp();
        if (ld_acc) {
          if (!__all_sync(0xffffffffu, tc::mbar_wait(mybar, ai & 1, abort_flag))) {
            ok = false;
            break;
          }
          ++ai;
        }
        const float prn = pr[n];
        const float2 pr2 = make_float2(prn, prn), inv2 = make_float2(inv * gdsc, inv * gdsc),
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
          uint4 ov[2];
#pragma unroll
          for (int jj = 0; jj < 2; ++jj) {
            const int j = 2 * jp + jj;
            float xf[8], gf[8], o[8];
            widen<E>(xv[j], xf);
            widen<E>(gyv[j], gf);
            // packed fp32 pairs (each lane rounds exactly like fmaf / a plain multiply)
#pragma unroll
            for (int u = 0; u < 8; u += 2) {
              const float2 cx = __fmul2_rn(ncf2, make_float2(xf[u], xf[u + 1]));
              const float2 rr = __ffma2_rn(inv2, make_float2(acc[8 * jj + u], acc[8 * jj + u + 1]), cx);
              const float2 oo = __ffma2_rn(make_float2(gf[u], gf[u + 1]), pr2, rr);
              o[u] = oo.x;
              o[u + 1] = oo.y;
            }
            if (ld_acc) {
              float a8[8];
              widen<E>(
                  *reinterpret_cast<const uint4*>(orow + (((2 * jp + jj) ^ osw) << 4)), a8);
#pragma unroll
              for (int u = 0; u < 8; ++u) o[u] += a8[u];
            }
            ov[jj] = narrow<E>(o);
          }
#pragma unroll
          for (int jj = 0; jj < 2; ++jj)
            *reinterpret_cast<uint4*>(orow + (((2 * jp + jj) ^ osw) << 4)) = ov[jj];
        }
        tc::fence_proxy_async();          // generic smem writes -> TMA store reads
        __syncwarp();
        if (lane == 0 && row0 < T) {
          tc::tma_store_2d(&maps.gx, ob, (int)(n * D + d0 + h * 32), (int)row0);
          tc::bulk_commit_group();
        }
        if (item + 1 < it1 && (n == 0 || n == N - 1)) {
          const bool wrap = cur.i + 1 == ntiles;
          const int64_t gn = wrap ? cur.g + 1 : cur.g, in = wrap ? 0 : i + 1;
          if (n == 0) {
            // pull the next item's grad_y row segment into L2 while this item runs
            const int64_t tn = in * 128 + r;
            if (tn < T) prefetch_l2(gy + tn * gys + gn * GC + h * 32);
          } else {
            load_item(gn, in);  // this item's operands are dead after its last step
          }
        }
      }
      if (!ok) break;
      if (cur.seg_end) {
        // flush: D2[h] row r = column d0 + r; cols k: hi k, lo 24 + k
        if (!__all_sync(0xffffffffu, tc::mbar_wait(d2full, seg & 1, abort_flag))) break;
        tc::tc_fence_after();
        // slot 1 iff this CTA's run began inside the cell
        const int64_t slot = (cur.g * geo.cpg + cur.i / cur.subt) * 2 +
                             ((first_seg && starts_inside) ? 1 : 0);
        first_seg = false;
        float v[48];
        const uint32_t ta = tmem + ((uint32_t)(q * 32) << 16) + h * 64;
#pragma unroll
        for (int m = 0; m < 3; ++m) tc::tmem_ld16(ta + m * 16, v + m * 16);
        tc::tmem_ld_wait();
        float* dst = gphi_part + (slot * N + h) * HM * GC;
#pragma unroll
        for (int k = 0; k < HM; ++k) dst[k * GC + r] = v[k] + v[HM + k];
        tc::tc_fence_before();
        __syncwarp();
        if (lane == 0) tc::mbar_arrive(d2empty);
        ++seg;
      }
    }
  }
  if (warp >= 2 && lane == 0) tc::bulk_wait_all<0>();  // grad_x stores have landed
  if (*abort_flag && threadIdx.x == 0) flag_timeout();
  tc::tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc::tc_fence_after();
    tc::tmem_dealloc(tmem, bwdtc::TMEM_COLS);
  }
}

// phi (fp32 [HM][HC]) -> per-column bf16 operand rows P' = [phi_hi | phi_hi | phi_lo | 0]
// split into P0 [HC][64] and P1 [HC][16].
// P0 / P1: the phi operand rows (bwd_phi_prep_item), three threads per column.
template <typename E>
__global__ void pre_bwd_phi_prep_kernel(const float* __restrict__ phi, E* __restrict__ p0,
                                        E* __restrict__ p1, int64_t HC,
                                        const unsigned* __restrict__ scl) {
  pdl_enter();
  const float sc = scl ? f16_operand_scale(scl[0]) : 1.f;
  bwd_phi_prep_item<E>(phi, p0, p1, HC, sc, (int64_t)blockIdx.x * blockDim.x + threadIdx.x);
}

// grad_phi[k][n*D + g*128 + c] = sum over the cells of group g (in order) of slot 0,
// plus slot 1 where a CTA run boundary falls strictly inside the cell.  A block of 256
// outputs lies inside one group (N*HM*GC is a multiple of 256); the group's split flags
// are computed once per block.
constexpr int kMaxCellsPerGroup = 4096;
__global__ void __launch_bounds__(256)
pre_bwd_gphi_reduce_kernel(const float* __restrict__ part, float* __restrict__ grad_phi,
                           int64_t D, BwdGeom geo, const unsigned* __restrict__ scl) {
  pdl_enter();
  using namespace bwdtc;
  constexpr int64_t SLOT = (int64_t)N * HM * GC;
  static_assert(SLOT % 1024 == 0, "a block (256 threads x 4 columns) stays in one group");
  __shared__ unsigned char split[kMaxCellsPerGroup];
  const int64_t idx0 = (int64_t)blockIdx.x * blockDim.x * 4;
  const int64_t g = idx0 / SLOT;
  auto cell_split = [&](int64_t ci) -> bool {
    const int64_t lo = g * geo.ntiles + ci * geo.subt;
    int64_t hi = lo + geo.subt;
    if (hi > (g + 1) * geo.ntiles) hi = (g + 1) * geo.ntiles;
    // first run boundary items*b/ncta above lo
    int64_t b = lo * geo.ncta / geo.items;
    while (geo.items * b / geo.ncta <= lo) ++b;
    return b < geo.ncta && geo.items * b / geo.ncta < hi;
  };
  const bool table = geo.cpg <= kMaxCellsPerGroup;
  if (table)
    for (int64_t ci = threadIdx.x; ci < geo.cpg; ci += blockDim.x) split[ci] = cell_split(ci);
  __syncthreads();
  // four consecutive columns c of one (n, k) row per thread (GC is a multiple of 4)
  const int64_t inner = idx0 - g * SLOT + 4 * (int64_t)threadIdx.x;  // (n, k, c) in a slot
  const int n = (int)(inner / (HM * GC));
  const int k = (int)((inner / GC) % HM);
  const int c = (int)(inner % GC);
  Kahan k4[4];
  float4 s = make_float4(0.f, 0.f, 0.f, 0.f);
  for (int64_t ci = 0; ci < geo.cpg; ++ci) {
    const int64_t cell = g * geo.cpg + ci;
    const float4 a = __ldcg(reinterpret_cast<const float4*>(part + (cell * 2) * SLOT + inner));
    s = kahan_add4(k4, a);
    if (table ? split[ci] != 0 : cell_split(ci)) {
      const float4 b =
          __ldcg(reinterpret_cast<const float4*>(part + (cell * 2 + 1) * SLOT + inner));
      s = kahan_add4(k4, b);
    }
  }
  if (scl) {  // exact: a power of two
    const float f = 1.f / f16_operand_scale(scl[2]);
    s.x *= f; s.y *= f; s.z *= f; s.w *= f;
  }
  *reinterpret_cast<float4*>(grad_phi + (int64_t)k * (N * D) + n * D + g * GC + c) = s;
}

// fp16 operands: maxima of |phi|, |grad_mixes| and |inv * grad_mixes| (atomicMax on the
// bits of non-negative floats, which order like the floats).
__global__ void pre_bwd_f16_max_kernel(const float* __restrict__ phi, int64_t nphi,
                                       const float* __restrict__ gm,
                                       const float* __restrict__ inv_rms, int64_t T, int hm,
                                       unsigned* __restrict__ scl) {
  pdl_enter();
  float mp = 0.f, mg = 0.f, mgp = 0.f;
  const int64_t ng = T * hm, n = nphi > ng ? nphi : ng;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x) {
    if (i < nphi) mp = fmaxf(mp, fabsf(phi[i]));
    if (i < ng) {
      const float g = fabsf(gm[i]);
      mg = fmaxf(mg, g);
      mgp = fmaxf(mgp, g * inv_rms[i / hm]);
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    mp = fmaxf(mp, __shfl_xor_sync(0xffffffffu, mp, o));
    mg = fmaxf(mg, __shfl_xor_sync(0xffffffffu, mg, o));
    mgp = fmaxf(mgp, __shfl_xor_sync(0xffffffffu, mgp, o));
  }
  if ((threadIdx.x & 31) == 0) {
    atomicMax(&scl[0], __float_as_uint(mp));
    atomicMax(&scl[1], __float_as_uint(mg));
    atomicMax(&scl[2], __float_as_uint(mgp));
  }
}

// fp16 operand rows of one token from grad_mixes (the bf16 path writes them in pass 1):
//   G' = [g_hi | g_lo | g_hi | 0] * 2^sg (K=80: g0 holds 0..63, g1 64..79)
//   Gp = [(inv g)_hi | (inv g)_lo | 0] * 2^sgp (64)
__global__ void pre_bwd_g_prep_f16_kernel(const float* __restrict__ gm,
                                          const float* __restrict__ inv_rms, __half* __restrict__ g0,
                                          __half* __restrict__ g1, __half* __restrict__ gp,
                                          int64_t T, const unsigned* __restrict__ scl) {
  pdl_enter();
  using namespace bwdtc;
  const int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (t >= T) return;
  const float sg = f16_operand_scale(scl[1]), sgp = f16_operand_scale(scl[2]);
  const float inv = inv_rms[t];
  __half row[80], prow[64];
#pragma unroll
  for (int k = 0; k < HM; ++k) {
    const float g = gm[t * HM + k] * sg;
    const __half hi = __float2half_rn(g);
    row[k] = hi;
    row[HM + k] = __float2half_rn(g - __half2float(hi));
    row[2 * HM + k] = hi;
    const float p = gm[t * HM + k] * inv * sgp;
    const __half ph = __float2half_rn(p);
    prow[k] = ph;
    prow[HM + k] = __float2half_rn(p - __half2float(ph));
  }
#pragma unroll
  for (int k = 3 * HM; k < 80; ++k) row[k] = __float2half_rn(0.f);
#pragma unroll
  for (int k = 2 * HM; k < 64; ++k) prow[k] = __float2half_rn(0.f);
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

// ---------------------------------------------------------------------------
// Host side
// ---------------------------------------------------------------------------
bool pre_bwd_tc_eligible(const PreBwdArgs& a) {
  const int64_t T = a.T, D = a.D;
  const int32_t N = a.N;
  return (a.dtype == MHC_BF16 || a.dtype == MHC_F16) && N == 4 && D % bwdtc::GC == 0 && T > 0 &&

         T <= (int64_t)INT32_MAX - 256 && (int64_t)N * D <= INT32_MAX &&
         rows_aligned(a.x, a.x_ts, 2, 16) && rows_aligned(a.grad_y, a.gy_ts, 2, 16) &&
         aligned16(a.grad_x);
}

static BwdGeom bwd_tc_geometry(int64_t T, int64_t D) {
  BwdGeom g;
  g.ntiles = cdiv(T, 128);
  g.items = (D / bwdtc::GC) * g.ntiles;
  int n = sm_count();
  if (g.items < n) n = (int)g.items;
  g.ncta = n < 1 ? 1 : n;
  const int64_t shortest_run = g.items / g.ncta;  // >= 1
  g.subt = shortest_run < bwdtc::SUBT ? shortest_run : bwdtc::SUBT;
  if (g.subt < 1) g.subt = 1;
  g.cpg = cdiv(g.ntiles, g.subt);
  return g;
}

struct BwdTcWs {
  __nv_bfloat16 *g0, *g1, *gp, *p0, *p1;
  float* part;
  unsigned* scl;  // fp16: max |phi|, |grad_mixes|, |inv * grad_mixes| (float bits)
  size_t total;
};

static BwdTcWs bwd_tc_layout(char* base, int64_t T, int64_t D) {
  using namespace bwdtc;
  const BwdGeom geo = bwd_tc_geometry(T, D);
  const int64_t Tp = geo.ntiles * 128, HC = N * D;
  BwdTcWs w;
  size_t off = 0;
  auto take = [&](size_t bytes) { char* p = base + off; off += align_up(bytes); return p; };
  w.g0 = (__nv_bfloat16*)take((size_t)Tp * 64 * 2);
  w.g1 = (__nv_bfloat16*)take((size_t)Tp * 16 * 2);
  w.gp = (__nv_bfloat16*)take((size_t)Tp * 64 * 2);
  w.p0 = (__nv_bfloat16*)take((size_t)HC * 64 * 2);
  w.p1 = (__nv_bfloat16*)take((size_t)HC * 16 * 2);
  w.part = (float*)take((size_t)(D / GC) * geo.cpg * 2 * N * HM * GC * 4);
  w.scl = (unsigned*)take(256);
  w.total = off;
  return w;
}

size_t pre_bwd_tc_ws_bytes(int64_t T, int64_t D) { return bwd_tc_layout(nullptr, T, D).total; }

// Pointers to the bf16 operand rows pass 1 writes (inside the tc workspace region).
void pre_bwd_tc_operand_ptrs(void* ws, int64_t T, int64_t D, __nv_bfloat16** g0,
                             __nv_bfloat16** g1, __nv_bfloat16** gp, __nv_bfloat16** p0,
                             __nv_bfloat16** p1) {
  BwdTcWs w = bwd_tc_layout((char*)ws, T, D);
  *g0 = w.g0;
  *g1 = w.g1;
  *gp = w.gp;
  *p0 = w.p0;
  *p1 = w.p1;
}

template <typename E>
static int pre_bwd_tc_run(const PreBwdArgs& a, void* ws, const float* gm, const float* coef,
                          cudaStream_t s) {
  using namespace bwdtc;
  constexpr bool f16 = std::is_same<E, __half>::value;
  const int64_t T = a.T, D = a.D, HC = N * D;
  const BwdGeom geo = bwd_tc_geometry(T, D);
  BwdTcWs w = bwd_tc_layout((char*)ws, T, D);
  const unsigned* scl = f16 ? w.scl : nullptr;
  if (f16) {
    MHC_CUDA_CHECK(cudaMemsetAsync(w.scl, 0, 3 * sizeof(unsigned), s));
    const int64_t n = std::max<int64_t>((int64_t)HM * HC, T * HM);
    launch(pre_bwd_f16_max_kernel, (unsigned)std::min<int64_t>(cdiv(n, 256), (int64_t)sm_count() * 4), 256, 0, s, a.phi, (int64_t)HM * HC, gm, a.inv_rms, T, HM, w.scl);
    MHC_LAUNCH_CHECK();
    launch(pre_bwd_g_prep_f16_kernel, (unsigned)cdiv(T, 128), 128, 0, s, 
        gm, a.inv_rms, (__half*)w.g0, (__half*)w.g1, (__half*)w.gp, T, w.scl);
    MHC_LAUNCH_CHECK();
  }
  if (!a.phi_prepped) {  // bf16: pre_bwd_dots_kernel's extra blocks wrote P0 / P1
    launch(pre_bwd_phi_prep_kernel<E>, (unsigned)cdiv(3 * HC, 256), 256, 0, s, a.phi,
           (E*)w.p0, (E*)w.p1, HC, scl);
    MHC_LAUNCH_CHECK();
  }
  BwdTcMaps m;
  const CUtensorMapDataType bf =
      f16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
  int st;
  // operand rows: row extent T, so rows of the last tile beyond T read as zeros
  if ((st = make_tmap_2d(&m.x, a.x, bf, 2, HC, T, a.x_ts * 2, 64, 128,
                         CU_TENSOR_MAP_SWIZZLE_128B)))
    return st;
  if ((st = make_tmap_2d(&m.g0, w.g0, bf, 2, 64, T, 128, 64, 128, CU_TENSOR_MAP_SWIZZLE_128B)))
    return st;
  if ((st = make_tmap_2d(&m.g1, w.g1, bf, 2, 16, T, 32, 16, 128, CU_TENSOR_MAP_SWIZZLE_32B)))
    return st;
  if ((st = make_tmap_2d(&m.gp, w.gp, bf, 2, 64, T, 128, 64, 128, CU_TENSOR_MAP_SWIZZLE_128B)))
    return st;
  if ((st = make_tmap_2d(&m.p0, w.p0, bf, 2, 64, HC, 128, 64, 128, CU_TENSOR_MAP_SWIZZLE_128B)))
    return st;
  if ((st = make_tmap_2d(&m.p1, w.p1, bf, 2, 16, HC, 32, 16, 128, CU_TENSOR_MAP_SWIZZLE_32B)))
    return st;
  // grad_x store boxes: 32 columns (64 B) x 32 token rows, one per epilogue warp and step
  if ((st = make_tmap_2d(&m.gx, a.grad_x, bf, 2, HC, T, HC * 2, 32, 32,
                         CU_TENSOR_MAP_SWIZZLE_64B)))
    return st;
  m.gxa = m.gx;
  if (a.grad_x_acc &&
      (st = make_tmap_2d(&m.gxa, a.grad_x_acc, bf, 2, HC, T, HC * 2, 32, 32,
                         CU_TENSOR_MAP_SWIZZLE_64B)))
    return st;
  static bool attr_set[64];
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 0 && dev < 64 && !attr_set[dev]) {
    MHC_CUDA_CHECK(cudaFuncSetAttribute(pre_bwd_tc_kernel<false, E>,
                                        cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM));
    MHC_CUDA_CHECK(cudaFuncSetAttribute(pre_bwd_tc_kernel<true, E>,
                                        cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM));
    attr_set[dev] = true;
  }
  auto kern = a.grad_x_acc ? pre_bwd_tc_kernel<true, E> : pre_bwd_tc_kernel<false, E>;
  launch(kern, geo.ncta, THREADS, SMEM, s, m, (const E*)a.grad_y,
                                                    a.inv_rms, coef, a.pre,
                                                    (E*)a.grad_x, w.part, T, D, geo, scl, a.gy_ts);
  MHC_LAUNCH_CHECK();
  const int64_t n = (D / GC) * N * HM * GC;
  launch(pre_bwd_gphi_reduce_kernel, (unsigned)cdiv(n, 1024), 256, 0, s, w.part, a.grad_phi, D, geo,
                                                                   scl);
  MHC_LAUNCH_CHECK();
  return MHC_OK;
}

int pre_bwd_tc_main(const PreBwdArgs& a, void* ws, const float* gm, const float* coef,
                    cudaStream_t s) {
  if (a.dtype == MHC_F16) return pre_bwd_tc_run<__half>(a, ws, gm, coef, s);
  return pre_bwd_tc_run<__nv_bfloat16>(a, ws, gm, coef, s);
}

int pre_bwd_tc_device_error() { return read_and_clear_tu_error(); }

}  // namespace mhc

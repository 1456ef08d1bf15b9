// post_mix_tc.cu -- layer-level fusion of the forward pass (N = 4, bf16 / fp16 storage).
//
// In a stack of mHC layers the post operator of layer l writes x_{l+1} (src/autograd.py:
// 14-32) and the pre operator of layer l+1 starts by reading all of x_{l+1} again for
// mixes = x_{l+1} . phi_{l+1}^T and sum(x_{l+1}^2) (src/mhc_pre_clamp_sinkhorn.py:897-903).
// post_mix_tc_kernel does both in one pass: it computes each 64-column chunk of
// out = x_{l+1} in shared memory, TMA-stores it, and feeds the same shared-memory tile to
// tcgen05.mma as the A operand against phi_{l+1} (bf16 hi/lo rows), so x_{l+1} is never
// read back for the mix.  Its output ("premix") is the raw mix and sum of squares per
// token, as partials [layers][T][HM+1] fp32 that add up to them, which mhc_pre_fwd_premixed turns into the
// pre operator's outputs (small stage, then y / x_scaled).
//
// Per CTA (persistent over (128-token tile, K range) units), 320 threads:
//   warp 0     TMA producer: x rows j=0..3 and h_out of the chunk ([128 tok x 64] boxes,
//              128-byte swizzle) and the four phi boxes [48 x 64] of columns i*D + d0
//   warp 1     TMEM owner + MMA issuer: per chunk and row i, 4 x tcgen05.mma M=128 N=48
//              K=16 (A = out row i, written in place of x row i; B = phi box i);
//              segments of 64 MMAs alternate between two TMEM buffers
//   warps 2-9  two warps per token-row quarter (TMEM lane quarter warp % 4), each taking
//              four of the chunk's eight 16-byte columns: out[i] = sum_j h_res[j,i] x[j] +
//              h_post[i] h_out in fp32 (the expression of post_fwd_x16_kernel, so out is
//              bitwise mhc_post's), rounded, written over x row i of the stage; sum of
//              squares of the rounded values; the first warp of each pair TMA-stores the
//              pair's 32 rows; each warp folds half of every finished TMEM segment.
// premix gets two layers per K range (one per warp half: its mix components, zeros
// elsewhere, and its share of the sum of squares); the consumer adds the layers.
// A stage is released when its MMAs have completed and the four store warps' bulk
// stores have read it.  Measured alternatives, all slower: 32-column chunks with a 64-byte
// swizzle and four stages (64-byte row pieces are a poor DRAM read pattern); out stored
// from registers in 32-byte pieces (1.03 ms at T=32768, scattered sectors); TMA stores
// without an L2 policy (0.98 ms); this kernel: 0.87 ms, against 0.58 ms with no out
// stores at all, so the store path is what still costs.
// Every wait is bounded (MHC_ERR_TIMEOUT).  No TMA multicast.
#include "pre_common.cuh"
#include "tc.cuh"

namespace mhc {

namespace pmix {
constexpr int N = 4, HM = 24, NP = 48;
constexpr int BOX = 64;                     // columns of d per chunk (128 B rows)
constexpr int XBOX = 128 * BOX * 2;         // 16 KB: 128 token rows of one x row / h_out
constexpr int PBOX = NP * BOX * 2;          // 6 KB: the 48 hi/lo rows of phi
constexpr int STAGE = 5 * XBOX + 4 * PBOX;  // x rows 0..3 (out in place), h_out, phi 0..3
constexpr int STAGES = 2;
constexpr int KSEG = 4;                     // chunks per TMEM segment (4 x 16 = 64 MMAs)
constexpr int BUFCOL = 64;                  // TMEM columns per accumulator buffer
constexpr int TMEM_COLS = 128;
constexpr int THREADS = 320;
constexpr int SMEM = 1024 + STAGES * STAGE + 512;
static_assert(SMEM <= 227 * 1024, "shared memory");
static_assert(STAGE % 1024 == 0 && PBOX % 1024 == 0, "box alignment");
}  // namespace pmix

__device__ __forceinline__ uint4 lds128(uint32_t addr) {
  uint4 v;
  asm volatile("ld.shared.v4.u32 {%0, %1, %2, %3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "r"(addr));
  return v;
}
__device__ __forceinline__ void sts128(uint32_t addr, uint4 v) {
  asm volatile("st.shared.v4.u32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(v.x), "r"(v.y),
               "r"(v.z), "r"(v.w)
               : "memory");
}

struct PostMixMaps {
  CUtensorMap x, ho, phi, out;
};

template <typename E>
__global__ void __launch_bounds__(pmix::THREADS, 1)
post_mix_tc_kernel(const __grid_constant__ PostMixMaps maps, const float* __restrict__ h_res,
                   const float* __restrict__ h_post, int64_t T, int64_t D, int ksplit,
                   float* __restrict__ premix, const float* __restrict__ descale) {
  pdl_enter();
  using namespace pmix;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = (uint8_t*)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
  uint64_t* full = (uint64_t*)(smem + STAGES * STAGE);
  uint64_t* outfull = full + STAGES;
  uint64_t* empty = outfull + STAGES;
  uint64_t* pair = empty + STAGES;        // [STAGES][4]: second warp of a pair has written
  uint64_t* tfull = pair + 4 * STAGES;
  uint64_t* tempty = tfull + 2;
  uint64_t* tdone = tempty + 2;
  uint32_t* tmem_slot = (uint32_t*)(tdone + 1);
  volatile int* abort_flag = (volatile int*)(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t ntiles = (T + 127) / 128;
  const int nk = (int)(D / BOX);
  const int64_t units = ntiles * ksplit;
  auto stage_x = [&](int s, int row) { return smem + s * STAGE + row * XBOX; };
  auto stage_p = [&](int s, int i) { return smem + s * STAGE + 5 * XBOX + i * PBOX; };

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      tc::mbar_init(&full[s], 1);
      tc::mbar_init(&outfull[s], 8);
      tc::mbar_init(&empty[s], 1 + 4);
      for (int q = 0; q < 4; ++q) tc::mbar_init(&pair[s * 4 + q], 1);
    }
    for (int b = 0; b < 2; ++b) {
      tc::mbar_init(&tfull[b], 1);
      tc::mbar_init(&tempty[b], 8);
    }
    tc::mbar_init(tdone, 1);
    *abort_flag = 0;
    tc::fence_barrier_init();
  }
  if (warp == 0 && lane == 0) {
    tc::prefetch_tmap(&maps.x);
    tc::prefetch_tmap(&maps.ho);
    tc::prefetch_tmap(&maps.phi);
    tc::prefetch_tmap(&maps.out);
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
      uint32_t it = 0;
      bool ok = true;
      const uint64_t pol_stream = tc::l2_evict_first(), pol_keep = tc::l2_evict_last();
      for (int64_t u = blockIdx.x; u < units && ok; u += gridDim.x) {
        const int64_t tile = u / ksplit;
        const int spl = (int)(u - tile * ksplit);
        const int kcb = nk * spl / ksplit, kce = nk * (spl + 1) / ksplit;
        for (int kc = kcb; kc < kce; ++kc, ++it) {
          const int s = it % STAGES;
          if (!tc::mbar_wait(&empty[s], ((it / STAGES) & 1) ^ 1, abort_flag)) {
            ok = false;
            break;
          }
          tc::mbar_arrive_expect_tx(&full[s], STAGE);
          const int d0 = kc * BOX, row0 = (int)(tile * 128);
#pragma unroll
          for (int j = 0; j < N; ++j)
            tc::tma_load_2d_hint(stage_x(s, j), &maps.x, &full[s], (int)(j * D) + d0, row0,
                                 pol_stream);
          tc::tma_load_2d_hint(stage_x(s, 4), &maps.ho, &full[s], d0, row0, pol_stream);
#pragma unroll
          for (int i = 0; i < N; ++i)
            tc::tma_load_2d_hint(stage_p(s, i), &maps.phi, &full[s], (int)(i * D) + d0, 0,
                                 pol_keep);
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t idesc = tc::idesc_16<E>(128, NP, false, false);
      uint32_t it = 0, j = 0;
      bool ok = true;
      for (int64_t u = blockIdx.x; u < units && ok; u += gridDim.x) {
        const int64_t tile = u / ksplit;
        const int spl = (int)(u - tile * ksplit);
        const int kcb = nk * spl / ksplit, kce = nk * (spl + 1) / ksplit;
        for (int kc0 = kcb; kc0 < kce && ok; kc0 += KSEG, ++j) {
          const int buf = j & 1;
          if (!tc::mbar_wait(&tempty[buf], ((j >> 1) & 1) ^ 1, abort_flag)) {
            ok = false;
            break;
          }
          tc::tc_fence_after();
          const uint32_t d = tmem + buf * BUFCOL;
          const int kc1 = kc0 + KSEG < kce ? kc0 + KSEG : kce;
          for (int kc = kc0; kc < kc1; ++kc, ++it) {
            const int s = it % STAGES;
            if (!tc::mbar_wait(&outfull[s], (it / STAGES) & 1, abort_flag)) {
              ok = false;
              break;
            }
            tc::tc_fence_after();
#pragma unroll
            for (int i = 0; i < N; ++i) {
              const uint64_t a0 =
                  tc::smem_desc(tc::smem_u32(stage_x(s, i)), 16, 1024, tc::kSwizzle128);
              const uint64_t b0 =
                  tc::smem_desc(tc::smem_u32(stage_p(s, i)), 16, 1024, tc::kSwizzle128);
#pragma unroll
              for (int k = 0; k < BOX / 16; ++k)
                tc::mma_bf16(d, a0 + 2 * k, b0 + 2 * k, idesc,
                             (kc != kc0 || i != 0 || k != 0) ? 1u : 0u);
            }
            tc::mma_commit(&empty[s]);
          }
          if (!ok) break;
          tc::mma_commit(&tfull[buf]);
        }
      }
      tc::mma_commit(tdone);  // every MMA of this CTA has completed before TMEM is freed
      volatile int never = 0;
      tc::mbar_wait(tdone, 0, &never);
    }
  } else {
    // ------------------------------------------------------------ post math + mix fold
    const int q = warp & 3;          // TMEM lane quarter this warp may access
    const int h = (warp - 2) >> 2;   // which four of the chunk's eight 16-byte columns
    const int r = q * 32 + lane;     // token row within the tile
    const uint32_t tq = tmem + ((uint32_t)(q * 32) << 16);
    const float dsc = descale ? *descale : 1.f;
    // out leaves L2 first: with the default policy its TMA stores made the L2 read ~40% of
    // their bytes back from DRAM (0.98 ms against 0.87 ms at T=32768)
    const uint64_t pol_out = tc::l2_evict_first();
    const int kb = h ? 16 : 0, kn = h ? HM - 16 : 16;  // mix components this warp folds
    uint32_t it = 0, j = 0;
    bool ok = true;
    for (int64_t u = blockIdx.x; u < units && ok; u += gridDim.x) {
      const int64_t tile = u / ksplit;
      const int spl = (int)(u - tile * ksplit);
      const int kcb = nk * spl / ksplit, kce = nk * (spl + 1) / ksplit;
      const int64_t t = tile * 128 + r;
      const bool live = t < T;
      float hr[N * N], hp[N];
#pragma unroll
      for (int e = 0; e < N * N; ++e) hr[e] = live ? __ldg(h_res + t * N * N + e) : 0.f;
#pragma unroll
      for (int i = 0; i < N; ++i) hp[i] = live ? __ldg(h_post + t * N + i) : 0.f;
      float sq = 0.f, mix[16];
#pragma unroll
      for (int k = 0; k < 16; ++k) mix[k] = 0.f;
      for (int kc = kcb; kc < kce; ++kc, ++it) {
        const int s = it % STAGES;
        const uint32_t ph = (it / STAGES) & 1;
        if (!__all_sync(0xffffffffu, tc::mbar_wait(&full[s], ph, abort_flag))) {
          ok = false;
          break;
        }
        float csq = 0.f;
        const uint32_t sbase = tc::smem_u32(stage_x(s, 0));
#pragma unroll 2
        for (int cc = 0; cc < 4; ++cc) {
          // physical 16-byte column of logical column 4h+cc (128-byte swizzle): the same in
          // all five boxes; the 8 rows of a swizzle atom use 8 different bank groups.
          // Shared-window addresses: ld/st.shared, not generic loads.
          const uint32_t off = sbase + r * 128 + (((4 * h + cc) ^ (r & 7)) << 4);
          float xf[N][8], hf[8];
#pragma unroll
          for (int jj = 0; jj < N; ++jj) widen<E>(lds128(off + jj * XBOX), xf[jj]);
          widen<E>(lds128(off + 4 * XBOX), hf);
#pragma unroll
          for (int i = 0; i < N; ++i) {
            float o[8];
#pragma unroll
            for (int e = 0; e < 8; ++e) {
              float acc = 0.f;
#pragma unroll
              for (int jj = 0; jj < N; ++jj) acc = fmaf(hr[jj * N + i], xf[jj][e], acc);
              o[e] = fmaf(hp[i], hf[e], acc);
            }
            const uint4 ov = narrow<E>(o);
            float of[8];
            widen<E>(ov, of);
#pragma unroll
            for (int e = 0; e < 8; ++e) csq = fmaf(of[e], of[e], csq);
            sts128(off + i * XBOX, ov);  // out row i over x row i
          }
        }
        sq += csq;
        // generic-proxy writes before the async-proxy reads (MMA operand, TMA store)
        tc::fence_proxy_async();
        __syncwarp();
        if (lane == 0) {
          tc::mbar_arrive(&outfull[s]);
          if (h == 1) tc::mbar_arrive(&pair[s * 4 + q]);
        }
        if (h == 0) {
          // store the pair's 32 rows once the partner warp has written its columns
          const bool pok = tc::mbar_wait(&pair[s * 4 + q], ph, abort_flag);
          if (!__all_sync(0xffffffffu, pok)) {
            ok = false;
            break;
          }
          if (lane == 0) {
            if (tile * 128 + q * 32 < T) {
#pragma unroll
              for (int i = 0; i < N; ++i)
                tc::tma_store_2d_hint(&maps.out, stage_x(s, i) + q * 32 * 128,
                                      (int)(i * D) + kc * BOX, (int)(tile * 128 + q * 32),
                                      pol_out);
            }
            tc::bulk_commit_group();
            tc::bulk_wait_read<0>();  // the stores have read the stage
            tc::mbar_arrive(&empty[s]);
          }
        }
        __syncwarp();
        if ((kc - kcb + 1) % KSEG == 0 || kc + 1 == kce) {
          const int buf = j & 1;
          if (!__all_sync(0xffffffffu, tc::mbar_wait(&tfull[buf], (j >> 1) & 1, abort_flag))) {
            ok = false;
            break;
          }
          tc::tc_fence_after();
          const uint32_t taddr = tq + buf * BUFCOL;
          float hi[16], lo[16];
          tc::tmem_ld16(taddr + kb, hi);
          tc::tmem_ld16(taddr + HM + kb, lo);
          tc::tmem_ld_wait();
#pragma unroll
          for (int e = 0; e < 16; ++e)
            if (e < kn) mix[e] += hi[e] + lo[e];
          tc::tc_fence_before();
          __syncwarp();
          if (lane == 0) tc::mbar_arrive(&tempty[buf]);
          ++j;
        }
      }
      if (!ok) break;
      if (live) {  // dsc: an exact power of two
        float* dst = premix + (((int64_t)(2 * spl + h)) * T + t) * (HM + 1);
        if (h == 0) {
#pragma unroll
          for (int k = 0; k < 16; ++k) dst[k] = mix[k] * dsc;
#pragma unroll
          for (int k = 16; k < HM; ++k) dst[k] = 0.f;
        } else {
#pragma unroll
          for (int k = 0; k < 16; ++k) dst[k] = 0.f;
#pragma unroll
          for (int k = 16; k < HM; ++k) dst[k] = mix[k - 16] * dsc;
        }
        dst[HM] = sq;
      }
    }
    if (h == 0 && lane == 0) tc::bulk_wait_all<0>();  // out stores have landed
  }
  if (*abort_flag && threadIdx.x == 0) flag_timeout();
  tc::tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc::tc_fence_after();
    tc::tmem_dealloc(tmem, pmix::TMEM_COLS);
  }
}

// phi split for the mix (in pre_fwd_tc.cu)
int pre_phi_split_launch(const float* phi, void* phi_hl, int32_t N, int64_t HC, bool f16,
                         void* slots, cudaStream_t s);

bool post_mix_eligible(int64_t T, int32_t N, int64_t D, int32_t dtype, const void* x,
                       const void* h_out, const void* out) {
  return (dtype == MHC_BF16 || dtype == MHC_F16) && N == 4 && D % pmix::BOX == 0 && T > 0 &&
         T <= (int64_t)INT32_MAX - 256 && (int64_t)N * D <= INT32_MAX && aligned16(x) &&
         aligned16(h_out) && aligned16(out);
}

// premix layers: two per K range; D is split into K ranges when the tiles cannot fill the
// GPU (as the standalone mix does)
static int post_mix_ranges(int64_t T, int64_t D) {
  const int64_t ntiles = cdiv(T, 128), sms = sm_count();
  if (ntiles <= 0 || 2 * ntiles > sms) return 1;
  const int64_t nk = D / pmix::BOX;
  int64_t k = sms / ntiles;
  if (k > nk / 2) k = nk / 2;  // at least 2 chunks per range
  return (int)(k < 1 ? 1 : k);
}

int post_mix_layers(int64_t T, int64_t D) { return 2 * post_mix_ranges(T, D); }

size_t post_mix_ws_bytes(int64_t D) {
  return align_up((size_t)pmix::NP * pmix::N * D * 2) + 256;
}

int post_mix_run(const void* x, const float* h_res, const void* h_out, const float* h_post,
                 void* out, int64_t T, int64_t D, int32_t dtype, const float* phi_next,
                 float* premix, int32_t layers, void* ws, cudaStream_t s) {
  using namespace pmix;
  const bool f16 = dtype == MHC_F16;
  const int64_t HC = (int64_t)N * D;
  void* phi_hl = ws;
  char* slots = (char*)ws + align_up((size_t)NP * HC * 2);
  const int st0 = pre_phi_split_launch(phi_next, phi_hl, N, HC, f16, slots, s);
  if (st0 != MHC_OK) return st0;
  const float* descale = f16 ? (const float*)(slots + 16) : nullptr;
  const CUtensorMapDataType dt =
      f16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
  PostMixMaps m;
  int st;
  if ((st = make_tmap_2d(&m.x, x, dt, 2, HC, T, HC * 2, BOX, 128, CU_TENSOR_MAP_SWIZZLE_128B)))
    return st;
  if ((st = make_tmap_2d(&m.ho, h_out, dt, 2, D, T, D * 2, BOX, 128, CU_TENSOR_MAP_SWIZZLE_128B)))
    return st;
  if ((st = make_tmap_2d(&m.phi, phi_hl, dt, 2, HC, NP, HC * 2, BOX, NP,
                         CU_TENSOR_MAP_SWIZZLE_128B)))
    return st;
  if ((st = make_tmap_2d(&m.out, out, dt, 2, HC, T, HC * 2, BOX, 32, CU_TENSOR_MAP_SWIZZLE_128B)))
    return st;
  static bool attr_set[64][2];
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 0 && dev < 64 && !attr_set[dev][f16]) {
    MHC_CUDA_CHECK(cudaFuncSetAttribute(
        f16 ? (const void*)post_mix_tc_kernel<__half> : (const void*)post_mix_tc_kernel<__nv_bfloat16>,
        cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM));
    attr_set[dev][f16] = true;
  }
  const int ranges = layers / 2;  // premix holds two layers per K range
  const int64_t units = cdiv(T, 128) * ranges;
  const int grid = (int)std::min<int64_t>(units, sm_count());
  if (f16)
    launch(post_mix_tc_kernel<__half>, grid, THREADS, SMEM, s, m, h_res, h_post, T, D, ranges,
           premix, descale);
  else
    launch(post_mix_tc_kernel<__nv_bfloat16>, grid, THREADS, SMEM, s, m, h_res, h_post, T, D,
           ranges, premix, descale);
  MHC_LAUNCH_CHECK();
  return MHC_OK;
}

int post_mix_device_error() { return read_and_clear_tu_error(); }

}  // namespace mhc

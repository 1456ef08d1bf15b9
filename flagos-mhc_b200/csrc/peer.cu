// peer.cu -- the cross-GPU sum of the pre operator's parameter gradients
// (grad_phi | grad_alpha | grad_base, one packed fp32 vector) over NVLink peer
// memory, in one kernel per rank.
//
// Token-sharded data parallelism splits T over the ranks; grad_phi =
// sum_t (inv*grad_mixes)[t]^T x[t] (the reference's torch.mm(grad_mixes.t(),
// x_scaled), src/mhc_pre_clamp_sinkhorn_backward.py:1372-1373) is then a sum of
// one partial per rank.  Every rank owns a "peer region" (cudaMalloc'd here and
// mapped into the other ranks' address spaces with CUDA IPC):
//
//   [ stage: n floats ][ result: n floats ][ flags: 2 x kMaxRanks x kMaxCtas u32 ]
//   [ control: epoch u32, ticket u32 ]
//
// The call's epoch comes from the host (nonzero) or, when the host passes 0, from this
// rank's control word: every CTA reads it at the start and uses it + 1; the last CTA to
// finish stores the new value.  The device-kept epoch makes the call capturable in a CUDA
// graph (a replay cannot change a kernel argument).
// (stage: this rank's input; result: the sum over the ranks of the slice it owns)
//
// The packed vector is cut into `world` slices (rank r owns slice r) and every
// slice into `G` parts (CTA c of every rank handles part c of every slice), so a
// CTA only ever waits for the CTAs with its own index on the other GPUs:
//   1. CTA c copies part c of every slice of its rank's input into its stage and
//      stores `epoch` into flag A[rank][c] of every rank;
//   2. it waits until flag A[p][c] == epoch for every rank p, reads part c of its
//      own slice from every rank's stage (NVLink loads), sums them in rank order
//      0..world-1 (so every rank ends with bitwise the same vector), writes the sum
//      into part c of its own result area and stores flag B[rank][c] on every rank;
//   3. it waits until flag B[p][c] == epoch for every p and copies part c of every
//      slice s from rank s's result area (NVLink loads for s != rank) to `dst`.
// Every data write goes to the writer's own memory; only flags cross NVLink as stores.
// A writer orders its data before its flags with a GPU-scope fence: a GPU's L2 is the
// point of coherence for its memory, remote NVLink reads included, so data that is in
// the writer's L2 when a reader sees the flag is what the reader loads.  (A system-scope
// fence, which also drains towards the host, cost ~20 us per signal on B200.)
// Reuse: a rank's stage is reread only after every peer signalled B for the previous
// call, and its result area is rewritten only after every peer signalled A for the next
// call (a peer signals A after its own previous call, phase-3 reads included, has ended).
// All waits poll with a deadline taken from the global timer; a CTA that runs out
// records MHC_ERR_TIMEOUT (read back by mhc_device_status) and returns without
// touching peer memory again.  No TMA and no multicast: plain 16-byte loads through
// peer pointers and 4-byte flag stores.
#include <string.h>

#include "common.cuh"

namespace mhc {

void note_launch();
constexpr int kMaxRanks = 8;
constexpr int kMaxCtas = 256;
constexpr int kPeerThreads = 256;

struct PeerArgs {
  float* region[kMaxRanks];  // every rank's peer region, mapped into this process
  const float* src;          // this rank's packed gradient
  float* dst;                // where the sum goes (may equal src)
  int64_t n;                 // floats in the packed vector
  int64_t cap;               // floats the stage / result areas hold
  int rank, world, ctas;
  uint32_t epoch;
  uint64_t timeout_ns;
};

static __device__ int g_peer_error;

__device__ __forceinline__ uint64_t gtimer() {
  uint64_t t;
  asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
  return t;
}
__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void st_relaxed_sys(uint32_t* p, uint32_t v) {
  asm volatile("st.relaxed.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

__host__ __device__ inline int64_t peer_flag_offset(int64_t cap) {
  return 2 * cap;  // in floats; cap is a multiple of 64, so the flags are 256-byte aligned
}
__device__ __forceinline__ uint32_t* flag_ptr(float* region, int64_t cap, int which, int rank,
                                              int cta) {
  return reinterpret_cast<uint32_t*>(region + peer_flag_offset(cap)) +
         (which * kMaxRanks + rank) * kMaxCtas + cta;
}

// Threads 0..world-1 each poll one rank's flag; the CTA agrees on the outcome.
__device__ bool cta_wait_flags(const PeerArgs& a, int which, uint32_t epoch, uint64_t deadline) {
  __shared__ int ok;
  if (threadIdx.x == 0) ok = 1;
  __syncthreads();
  if (threadIdx.x < a.world) {
    const uint32_t* f = flag_ptr(a.region[a.rank], a.cap, which, threadIdx.x, blockIdx.x);
    while ((int32_t)(ld_acquire_sys(f) - epoch) < 0) {
      if (gtimer() > deadline) {
        ok = 0;
        atomicExch(&g_peer_error, MHC_ERR_TIMEOUT);
        break;
      }
      __nanosleep(32);
    }
  }
  __syncthreads();
  return ok != 0;
}

// Publishes this CTA's (local) writes to every rank: the barrier makes them happen before
// thread 0's GPU-scope fence, which orders them before the flag stores.
template <int W>
__device__ __forceinline__ void cta_signal(const PeerArgs& a, int which, int c, uint32_t epoch) {
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
#pragma unroll
    for (int p = 0; p < W; ++p) st_relaxed_sys(flag_ptr(a.region[p], a.cap, which, a.rank, c), epoch);
  }
}

// Units of 4 floats: [u0, u1) of the whole vector is part `c` of slice `s`.
__device__ __forceinline__ void part_range(const PeerArgs& a, int s, int c, int64_t* u0,
                                           int64_t* u1) {
  const int64_t units = (a.n + 3) / 4;
  const int64_t per_slice = (units + a.world - 1) / a.world;
  const int64_t s0 = s * per_slice, s1 = min(units, s0 + per_slice);
  const int64_t per_part = (per_slice + a.ctas - 1) / a.ctas;
  *u0 = min(s1, s0 + c * per_part);
  *u1 = min(s1, *u0 + per_part);
}

__device__ __forceinline__ float4 ld4(const float* p, int64_t u, int64_t n) {
  if (4 * u + 3 < n) return __ldcg(reinterpret_cast<const float4*>(p) + u);
  float v[4];
#pragma unroll
  for (int k = 0; k < 4; ++k) v[k] = (4 * u + k < n) ? __ldcg(p + 4 * u + k) : 0.f;
  return make_float4(v[0], v[1], v[2], v[3]);
}
__device__ __forceinline__ void st4(float* p, int64_t u, int64_t n, float4 v) {
  if (4 * u + 3 < n) {
    __stcg(reinterpret_cast<float4*>(p) + u, v);
    return;
  }
  const float w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
  for (int k = 0; k < 4; ++k)
    if (4 * u + k < n) __stcg(p + 4 * u + k, w[k]);
}

__host__ __device__ inline int64_t peer_ctrl_offset(int64_t cap) {  // in floats
  return 2 * cap + 2 * kMaxRanks * kMaxCtas;
}

template <int W>
__device__ void peer_grad_sum_body(const PeerArgs& a, uint32_t epoch) {
  const int c = blockIdx.x;
  const uint64_t deadline = gtimer() + a.timeout_ns;
  float* mine = a.region[a.rank];
  // 1. stage part c of every slice, then announce it to every rank
#pragma unroll
  for (int s = 0; s < W; ++s) {
    int64_t u0, u1;
    part_range(a, s, c, &u0, &u1);
    for (int64_t u = u0 + threadIdx.x; u < u1; u += blockDim.x) st4(mine, u, a.n, ld4(a.src, u, a.n));
  }
  cta_signal<W>(a, 0, c, epoch);
  // 2. sum part c of this rank's slice over the ranks, in rank order; scatter it.
  // U units per thread and pass, all W*U loads issued before the first add, so many
  // NVLink requests are in flight per thread.
  if (!cta_wait_flags(a, 0, epoch, deadline)) return;
  {
    constexpr int U = W <= 4 ? 4 : 2;
    int64_t u0, u1;
    part_range(a, a.rank, c, &u0, &u1);
    for (int64_t ub = u0 + threadIdx.x; ub < u1; ub += U * blockDim.x) {
      float4 v[U][W];
#pragma unroll
      for (int q = 0; q < U; ++q) {
        const int64_t u = ub + (int64_t)q * blockDim.x;
#pragma unroll
        for (int p = 0; p < W; ++p)
          v[q][p] = u < u1 ? ld4(a.region[p], u, a.n) : make_float4(0.f, 0.f, 0.f, 0.f);
      }
#pragma unroll
      for (int q = 0; q < U; ++q) {
        const int64_t u = ub + (int64_t)q * blockDim.x;
        if (u >= u1) break;
        float4 acc = v[q][0];
#pragma unroll
        for (int p = 1; p < W; ++p) {
          acc.x += v[q][p].x; acc.y += v[q][p].y; acc.z += v[q][p].z; acc.w += v[q][p].w;
        }
        st4(mine + a.cap, u, a.n, acc);
      }
    }
  }
  cta_signal<W>(a, 1, c, epoch);
  // 3. every rank's slice part c is final in its owner's result area: gather them
  if (!cta_wait_flags(a, 1, epoch, deadline)) return;
  // all W slices' loads of a pass are issued before the first store
  int64_t b0[W], b1[W], len = 0;
#pragma unroll
  for (int s = 0; s < W; ++s) {
    part_range(a, s, c, &b0[s], &b1[s]);
    len = max(len, b1[s] - b0[s]);
  }
  for (int64_t i = threadIdx.x; i < len; i += blockDim.x) {
    float4 v[W];
#pragma unroll
    for (int s = 0; s < W; ++s)
      v[s] = b0[s] + i < b1[s] ? ld4(a.region[s] + a.cap, b0[s] + i, a.n)
                               : make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
    for (int s = 0; s < W; ++s)
      if (b0[s] + i < b1[s]) st4(a.dst, b0[s] + i, a.n, v[s]);
  }
}

template <int W>
__global__ void __launch_bounds__(kPeerThreads) peer_grad_sum_kernel(const PeerArgs a) {
  pdl_enter();
  uint32_t* ctrl = reinterpret_cast<uint32_t*>(a.region[a.rank] + peer_ctrl_offset(a.cap));
  const uint32_t epoch = a.epoch != 0 ? a.epoch : *(volatile uint32_t*)ctrl + 1u;
  peer_grad_sum_body<W>(a, epoch);
  if (a.epoch != 0) return;
  // device-kept epoch: the last CTA to finish (every CTA has read the old value by then)
  // stores the new one for the next call
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    if (atomicAdd(ctrl + 1, 1u) == (unsigned)gridDim.x - 1) {
      ctrl[0] = epoch;
      ctrl[1] = 0u;
      __threadfence();
    }
  }
}

static int64_t peer_cap(int64_t n) { return (n + 63) / 64 * 64; }

int peer_device_error() {
  int v = 0, z = 0;
  if (cudaMemcpyFromSymbol(&v, g_peer_error, sizeof(int)) != cudaSuccess) return MHC_ERR_CUDA;
  if (v != 0 && cudaMemcpyToSymbol(g_peer_error, &z, sizeof(int)) != cudaSuccess)
    return MHC_ERR_CUDA;
  return v;
}

}  // namespace mhc

using namespace mhc;

extern "C" {

size_t mhc_peer_region_bytes(int64_t n) {
  if (n <= 0) return 0;
  return (size_t)(peer_ctrl_offset(peer_cap(n)) * 4 + 256);
}

int mhc_peer_region_alloc(int64_t n, void** region) {
  if (!region || n <= 0) return MHC_ERR_INVALID_ARGUMENT;
  *region = nullptr;
  const size_t bytes = mhc_peer_region_bytes(n);
  void* p = nullptr;
  if (cudaMalloc(&p, bytes) != cudaSuccess) return MHC_ERR_CUDA;
  // flags start at 0; epochs start at 1
  if (cudaMemset(p, 0, bytes) != cudaSuccess || cudaDeviceSynchronize() != cudaSuccess) {
    cudaFree(p);
    return MHC_ERR_CUDA;
  }
  *region = p;
  return MHC_OK;
}

int mhc_peer_region_free(void* region) {
  if (!region) return MHC_OK;
  return cudaFree(region) == cudaSuccess ? MHC_OK : MHC_ERR_CUDA;
}

int mhc_peer_handle(void* region, void* handle_out) {
  if (!region || !handle_out) return MHC_ERR_INVALID_ARGUMENT;
  cudaIpcMemHandle_t h;
  if (cudaIpcGetMemHandle(&h, region) != cudaSuccess) return MHC_ERR_CUDA;
  memcpy(handle_out, &h, sizeof(h));
  return MHC_OK;
}

int mhc_peer_handle_bytes(void) { return (int)sizeof(cudaIpcMemHandle_t); }

int mhc_peer_open(const void* handle, void** peer_region) {
  if (!handle || !peer_region) return MHC_ERR_INVALID_ARGUMENT;
  cudaIpcMemHandle_t h;
  memcpy(&h, handle, sizeof(h));
  void* p = nullptr;
  if (cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess) != cudaSuccess)
    return MHC_ERR_CUDA;
  *peer_region = p;
  return MHC_OK;
}

int mhc_peer_close(void* peer_region) {
  if (!peer_region) return MHC_OK;
  return cudaIpcCloseMemHandle(peer_region) == cudaSuccess ? MHC_OK : MHC_ERR_CUDA;
}

int mhc_grad_sum_peers(const float* src, float* dst, int64_t n, void* const* regions,
                       int32_t rank, int32_t world, uint32_t epoch, uint64_t timeout_ns,
                       void* stream) {
  if (n < 0 || world < 1 || world > kMaxRanks || rank < 0 || rank >= world || !regions ||
      timeout_ns == 0)
    return MHC_ERR_INVALID_ARGUMENT;
  if (n == 0) return MHC_OK;
  if (!src || !dst || ((uintptr_t)src & 15) || ((uintptr_t)dst & 15))
    return MHC_ERR_INVALID_ARGUMENT;
  PeerArgs a{};
  for (int p = 0; p < world; ++p) {
    if (!regions[p] || ((uintptr_t)regions[p] & 255)) return MHC_ERR_INVALID_ARGUMENT;
    a.region[p] = static_cast<float*>(regions[p]);
  }
  a.src = src; a.dst = dst; a.n = n; a.cap = peer_cap(n);
  a.rank = rank; a.world = world; a.epoch = epoch; a.timeout_ns = timeout_ns;
  const int64_t units = (n + 3) / 4, per_slice = (units + world - 1) / world;
  // about one float4 per thread and slice (latency-bound: many requests in flight);
  // at most kMaxCtas (flag slots)
  int64_t g = (per_slice + kPeerThreads - 1) / kPeerThreads;
  a.ctas = (int)(g < 1 ? 1 : (g > kMaxCtas ? kMaxCtas : g));
  using K = void (*)(const PeerArgs);
  static const K kernels[kMaxRanks] = {peer_grad_sum_kernel<1>, peer_grad_sum_kernel<2>,
                                       peer_grad_sum_kernel<3>, peer_grad_sum_kernel<4>,
                                       peer_grad_sum_kernel<5>, peer_grad_sum_kernel<6>,
                                       peer_grad_sum_kernel<7>, peer_grad_sum_kernel<8>};
  pdl_new_call();
  launch(kernels[world - 1], a.ctas, kPeerThreads, 0, (cudaStream_t)stream, a);
  note_launch();
  return cudaGetLastError() == cudaSuccess ? MHC_OK : MHC_ERR_CUDA;
}

}  // extern "C"

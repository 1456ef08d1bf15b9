// tc_host.cu -- host helpers of the tensor-core kernels: tensor-map encoding
// through the driver entry point (no link-time dependency on libcuda).
#include <mutex>

#include "tc.cuh"

namespace mhc {

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                  const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                  const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                  CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn encoder() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  });
  return fn;
}

int make_tmap_2d(CUtensorMap* map, const void* base, CUtensorMapDataType dt, int elem,
                 uint64_t cols, uint64_t rows, uint64_t row_stride_bytes, uint32_t box_cols,
                 uint32_t box_rows, CUtensorMapSwizzle swz) {
  EncodeTiledFn enc = encoder();
  if (!enc) return MHC_ERR_CUDA;
  if ((reinterpret_cast<uintptr_t>(base) & 15) || (row_stride_bytes & 15) ||
      ((uint64_t)box_cols * elem) % 16)
    return MHC_ERR_INVALID_ARGUMENT;
  cuuint64_t dims[2] = {cols, rows};
  cuuint64_t strides[1] = {row_stride_bytes};
  cuuint32_t box[2] = {box_cols, box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = enc(map, dt, 2, const_cast<void*>(base), dims, strides, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, swz, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? MHC_OK : MHC_ERR_CUDA;
}

// Exercises the bounded mbarrier wait every tensor-core kernel uses, on a phase
// that nothing ever completes: the wait gives up after `limit` polls, the CTA
// records MHC_ERR_TIMEOUT in this unit's error word and returns.
__global__ void wait_selftest_kernel(uint32_t limit) {
  pdl_enter();
  __shared__ __align__(8) uint64_t bar;
  __shared__ int abort_flag;
  if (threadIdx.x == 0) {
    tc::mbar_init(&bar, 1);
    abort_flag = 0;
    tc::fence_barrier_init();
  }
  __syncthreads();
  if (threadIdx.x == 0 && !tc::mbar_wait(&bar, 0, &abort_flag, limit)) flag_timeout();
}

int tc_host_device_error() { return read_and_clear_tu_error(); }

}  // namespace mhc

extern "C" int mhc_selftest_wait_timeout(uint32_t spin_limit, void* stream) {
  if (spin_limit == 0) return MHC_ERR_INVALID_ARGUMENT;
  mhc::pdl_new_call();
  mhc::launch(mhc::wait_selftest_kernel, 1, 32, 0, (cudaStream_t)stream, spin_limit);
  MHC_LAUNCH_CHECK();
  return MHC_OK;
}

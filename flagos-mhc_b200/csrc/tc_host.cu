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

}  // namespace mhc

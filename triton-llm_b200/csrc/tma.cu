// Tensor-map (TMA descriptor) helpers shared by the kernels of libtllm.so.
// cuTensorMapEncodeTiled is a driver entry point; it is looked up once through
// the runtime so the library does not link libcuda directly.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <mutex>

#include "common.cuh"

namespace tllm {

PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void *ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr,
                                cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(ptr);
  });
  return fn;
}

// 2-D row-major tensor (outer rows of `inner` elements, rows stride_bytes
// apart) with a (box_inner x box_outer) box.
int make_map_2d(CUtensorMap *m, const void *base, int dtype, long inner,
                long outer, long stride_bytes, int box_inner, int box_outer,
                bool swizzle128) {
  auto fn = tensor_map_encoder();
  if (!fn) {
    set_error("cuTensorMapEncodeTiled is not available from the driver");
    return TLLM_ERR_CUDA;
  }
  cuuint64_t dims[2] = {(cuuint64_t)inner, (cuuint64_t)outer};
  cuuint64_t strides[1] = {(cuuint64_t)stride_bytes};
  cuuint32_t box[2] = {(cuuint32_t)box_inner, (cuuint32_t)box_outer};
  cuuint32_t estr[2] = {1, 1};
  CUtensorMapDataType t = dtype == TLLM_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16
                                             : CU_TENSOR_MAP_DATA_TYPE_FLOAT32;
  CUresult r = fn(m, t, 2, const_cast<void *>(base), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE,
                  swizzle128 ? CU_TENSOR_MAP_SWIZZLE_128B
                             : CU_TENSOR_MAP_SWIZZLE_NONE,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    set_error("cuTensorMapEncodeTiled(2d) failed (%d): inner=%ld outer=%ld "
              "stride=%ld box=%dx%d", (int)r, inner, outer, stride_bytes,
              box_inner, box_outer);
    return TLLM_ERR_CUDA;
  }
  return TLLM_OK;
}

// N-d tiled map (rank 2..5): dims[0] innermost, strides_bytes[i] = stride of
// dim i+1.
int make_map(CUtensorMap *m, const void *base, int dtype, int rank,
             const long *dims, const long *strides_bytes, const int *box,
             bool swizzle128) {
  auto fn = tensor_map_encoder();
  if (!fn) {
    set_error("cuTensorMapEncodeTiled is not available from the driver");
    return TLLM_ERR_CUDA;
  }
  cuuint64_t d[5], st[4];
  cuuint32_t b[5], e[5];
  for (int i = 0; i < rank; ++i) {
    d[i] = (cuuint64_t)dims[i];
    b[i] = (cuuint32_t)box[i];
    e[i] = 1;
    if (i + 1 < rank) st[i] = (cuuint64_t)strides_bytes[i];
  }
  CUtensorMapDataType t = dtype == TLLM_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16
                                             : CU_TENSOR_MAP_DATA_TYPE_FLOAT32;
  CUresult r = fn(m, t, rank, const_cast<void *>(base), d, st, b, e,
                  CU_TENSOR_MAP_INTERLEAVE_NONE,
                  swizzle128 ? CU_TENSOR_MAP_SWIZZLE_128B
                             : CU_TENSOR_MAP_SWIZZLE_NONE,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    set_error("cuTensorMapEncodeTiled(%dd) failed (%d): dims %ld x %ld box %d x %d",
              rank, (int)r, dims[0], dims[1], box[0], box[1]);
    return TLLM_ERR_CUDA;
  }
  return TLLM_OK;
}

}  // namespace tllm

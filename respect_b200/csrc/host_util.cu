#include <cudaTypedefs.h>

#include <mutex>

#include "common.cuh"
#include "host_util.h"

namespace rb {

namespace {
PFN_cuTensorMapEncodeTiled_v12000 g_encode = nullptr;
std::once_flag g_encode_once;

void load_encode() {
  void* fn = nullptr;
  cudaDriverEntryPointQueryResult q;
  if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) == cudaSuccess &&
      q == cudaDriverEntryPointSuccess)
    g_encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
}
}  // namespace

int encode_tiled(CUtensorMap* m, CUtensorMapDataType dt, int rank, const void* base,
                 const uint64_t* dims, const uint64_t* strides_bytes, const uint32_t* box,
                 CUtensorMapSwizzle swizzle) {
  std::call_once(g_encode_once, load_encode);
  if (!g_encode) return RB_ERR_CUDA;
  if (!aligned16(base)) return RB_ERR_UNSUPPORTED;
  for (int i = 0; i + 1 < rank; ++i)
    if (strides_bytes[i] % 16 != 0) return RB_ERR_UNSUPPORTED;
  cuuint64_t d[5], s[4];
  cuuint32_t b[5], e[5];
  for (int i = 0; i < rank; ++i) {
    d[i] = dims[i];
    b[i] = box[i];
    e[i] = 1;
    if (i + 1 < rank) s[i] = strides_bytes[i];
  }
  CUresult r = g_encode(m, dt, static_cast<cuuint32_t>(rank), const_cast<void*>(base), d, s, b, e,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? RB_OK : RB_ERR_UNSUPPORTED;
}

int encode_2d_bf16(CUtensorMap* m, const void* base, uint64_t inner, uint64_t outer, int64_t ld,
                   uint32_t box_inner, uint32_t box_outer) {
  if (ld <= 0 || inner == 0 || outer == 0) return RB_ERR_INVALID_ARG;
  const uint64_t dims[2] = {inner, outer};
  const uint64_t strides[1] = {static_cast<uint64_t>(ld) * 2};
  const uint32_t box[2] = {box_inner, box_outer};
  return encode_tiled(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, base, dims, strides, box,
                      CU_TENSOR_MAP_SWIZZLE_128B);
}

int device_sm_count() {
  static int cache[64] = {0};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 148;
  if (cache[dev] == 0) {
    int n = 0;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) n = 148;
    cache[dev] = n;
  }
  return cache[dev];
}

}  // namespace rb

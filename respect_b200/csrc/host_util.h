// Host-side helpers: tensor-map encoding through the driver entry point (no
// link-time dependency on libcuda), device attribute caching, status mapping.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace rb {

// 2-D bf16 tensor map with the 128-byte swizzle: `inner` elements per row
// (contiguous), `outer` rows `ld` elements apart, box [box_inner, box_outer].
// Out-of-range elements of a box read as zero.
int encode_2d_bf16(CUtensorMap* m, const void* base, uint64_t inner, uint64_t outer, int64_t ld,
                   uint32_t box_inner, uint32_t box_outer);

// General tiled encoder (rank <= 5), strides in bytes for dims 1..rank-1.
int encode_tiled(CUtensorMap* m, CUtensorMapDataType dt, int rank, const void* base,
                 const uint64_t* dims, const uint64_t* strides_bytes, const uint32_t* box,
                 CUtensorMapSwizzle swizzle);

// Streaming multiprocessor count of the current device (cached per device).
int device_sm_count();

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// Launch with (pdl = true) or without programmatic stream serialization.
template <typename... KArgs, typename... Args>
int launch_k(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st, bool pdl,
             Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, kern, static_cast<KArgs>(args)...) == cudaSuccess ? 0 : 4;
}

}  // namespace rb

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

}  // namespace rb

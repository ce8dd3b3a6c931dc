// Host-side construction of TMA tensor maps (driver entry point looked up
// once through the runtime, so the library links only against cudart).
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace gdn {

// 3-D bf16 tensor map over [dim2][dim1][dim0] (dim0 contiguous) with byte
// strides stride1 (between dim1 rows) and stride2 (between dim2 planes), box
// [box2 = 1][box1][box0], zero fill out of range; no swizzle, or with swizzle128
// the 128-byte swizzle (box0 * 2 must then be at most 128 bytes, and the shared
// destination 1024-byte aligned).  False when the driver entry point is missing
// or the encoder rejects the arguments.
bool encode_tmap_3d_bf16(CUtensorMap* map, const void* base, uint64_t dim0, uint64_t dim1, uint64_t dim2,
                         uint64_t stride1_bytes, uint64_t stride2_bytes, uint32_t box0, uint32_t box1,
                         bool swizzle128 = false);

}  // namespace gdn

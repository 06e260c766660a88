// Host-side construction of TMA tensor maps.  The driver entry point is
// resolved through the runtime (cudaGetDriverEntryPoint), so the library does
// not link libcuda directly.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <cudaTypedefs.h>
#include <cstdint>

namespace qa {

// 2-D K-major tile map over a row-major [rows, inner] 16-bit matrix whose rows
// are `ld` elements apart.  Box = [box_rows, box_inner] with 128-byte
// swizzling (box_inner * 2 must be 128).  Out-of-range elements read as zero.
int make_tmap_2d(CUtensorMap* map, const void* base, bool bf16, long long inner, long long rows,
                 long long ld, int box_inner, int box_rows);

// General tiled map over a 16-bit tensor of `rank` dimensions (innermost
// first): dims[i] elements, stride_bytes[i] between consecutive indices of
// dimension i+1 (rank-1 entries), box[i] elements traversed per copy with a
// traversal stride estr[i] (ceil(box[i] / estr[i]) elements land in shared
// memory), swizzle 64 or 128 (bytes).  Out-of-range elements read as zero.
int make_tmap_nd(CUtensorMap* map, const void* base, bool bf16, int rank, const long long* dims,
                 const long long* stride_bytes, const int* box, const int* estr, int swizzle);

}  // namespace qa

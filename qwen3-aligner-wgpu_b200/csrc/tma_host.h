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

}  // namespace qa

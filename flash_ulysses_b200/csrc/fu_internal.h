// Internal helpers shared by the C-ABI translation units.
#pragma once

#include <cuda.h>

namespace fu {
// Records a printf-style message for fu_last_error() and returns `code`.
int set_error(int code, const char* fmt, ...);

// The driver's cuTensorMapEncodeTiled (signature as in cuda.h), fetched once at
// run time so the library needs no link-time dependency on libcuda; NULL if the
// driver does not provide it.
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                  const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                  const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                  CUtensorMapL2promotion, CUtensorMapFloatOOBfill);
EncodeTiledFn encode_tiled_fn();
}  // namespace fu

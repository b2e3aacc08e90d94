// Host-side helpers shared by the C-ABI entry points: thread-local error
// message, status helpers, the TMA descriptor encoder (driver entry point
// resolved through the runtime, so the library needs no -lcuda link) and the
// device-side error flag.
#pragma once

#include <cstdarg>
#include <cstdint>
#include <cstdio>
#include <cuda.h>
#include <cuda_runtime.h>

#include "../../include/taomate_b200.h"

namespace tmb {

int set_error(int status, const char* fmt, ...);
int check_cuda(cudaError_t e, const char* what);

// Device error flag (one int per device image of the library); its address
// is cached per device after the first call on that device.
int* device_error_flag();

// cuTensorMapEncodeTiled, resolved once.
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                  const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                  const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                  CUtensorMapL2promotion, CUtensorMapFloatOOBfill);
EncodeTiledFn encode_tiled();

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

}  // namespace tmb

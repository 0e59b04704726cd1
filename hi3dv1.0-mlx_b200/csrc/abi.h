// Host-side helpers shared by the entry points (not part of the public ABI).
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "hi3d_b200.h"

namespace hi3d {

// Record a formatted error message for hi3d_last_error_string(); returns `code`.
int set_error(int code, const char* fmt, ...);

// HI3D_OK, or HI3D_ERR_CUDA with the launch error recorded.
int check_launch(const char* what);

// Streaming multiprocessors of the current device (cached per device).
int sm_count();

// Encode a tiled TMA descriptor (dims/strides innermost first; strides are
// given for dims 1..rank-1 in bytes).
int encode_tmap(CUtensorMap* map, CUtensorMapDataType type, int rank, const void* base, const uint64_t* dims,
                const uint64_t* strides_bytes, const uint32_t* box, CUtensorMapSwizzle swizzle);

inline cudaStream_t as_stream(void* s) { return reinterpret_cast<cudaStream_t>(s); }

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

}  // namespace hi3d

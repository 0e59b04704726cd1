// Device status words of the translation units (host side).
#pragma once

#include <cuda_runtime.h>

namespace hi3d {

struct DeviceStatus {
  int code;    // first error code seen (HI3D_ERR_*), 0 if none
  int where;   // kernel-specific site id
  int block;   // blockIdx.x of the reporting CTA
  int detail;  // extra info (phase, index)
};

typedef cudaError_t (*StatusReader)(DeviceStatus* out, bool reset);

// Called by every translation unit's static initialiser (see common.cuh).
void register_status_reader(StatusReader fn);

}  // namespace hi3d

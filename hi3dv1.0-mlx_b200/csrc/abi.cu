// Library-level parts of the C ABI: status strings, the device status word,
// and the driver entry point used to encode TMA tensor maps.
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <mutex>

#include "abi.h"
#include "common.cuh"

namespace hi3d {

static StatusReader g_readers[16];
static int g_num_readers = 0;

void register_status_reader(StatusReader fn) {
  if (g_num_readers < 16) g_readers[g_num_readers++] = fn;
}

static thread_local char t_last_error[512] = "";

int set_error(int code, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(t_last_error, sizeof(t_last_error), fmt, ap);
  va_end(ap);
  return code;
}

int check_launch(const char* what) {
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return set_error(HI3D_ERR_CUDA, "%s: launch failed: %s", what, cudaGetErrorString(e));
  return HI3D_OK;
}

int sm_count() {
  static int counts[64] = {};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 148;
  if (counts[dev] == 0) {
    int n = 0;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) n = 148;
    counts[dev] = n;
  }
  return counts[dev];
}

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  });
  return fn;
}

int encode_tmap(CUtensorMap* map, CUtensorMapDataType type, int rank, const void* base, const uint64_t* dims,
                const uint64_t* strides_bytes, const uint32_t* box, CUtensorMapSwizzle swizzle) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return set_error(HI3D_ERR_CUDA, "cuTensorMapEncodeTiled is not available from the driver");
  cuuint32_t elem_strides[5] = {1, 1, 1, 1, 1};
  CUresult r = fn(map, type, (cuuint32_t)rank, const_cast<void*>(base), (const cuuint64_t*)dims,
                  (const cuuint64_t*)strides_bytes, (const cuuint32_t*)box, elem_strides,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    return set_error(HI3D_ERR_INVALID_ARGUMENT, "cuTensorMapEncodeTiled failed (%d): rank %d dims %llu,%llu", (int)r,
                     rank, (unsigned long long)dims[0], (unsigned long long)(rank > 1 ? dims[1] : 0));
  return HI3D_OK;
}

// One thread waits on an mbarrier that nothing arrives at; the bounded wait
// gives up after `limit_ns`, records HI3D_ERR_DEVICE_TIMEOUT at site
// kSiteWaitSelftest and the kernel returns normally.
constexpr int kSiteWaitSelftest = 900;

__global__ void wait_timeout_selftest_kernel(uint64_t limit_ns) {
  __shared__ __align__(8) uint64_t bar;
  __shared__ int abort;
  if (threadIdx.x == 0) {
    mbar_init(&bar, 1);
    abort = 0;
    fence_barrier_init();
  }
  __syncthreads();
  if (threadIdx.x == 0) mbar_wait_slow(&bar, 0, &abort, kSiteWaitSelftest, limit_ns);
  __syncthreads();
}

}  // namespace hi3d

using namespace hi3d;

extern "C" int hi3d_wait_timeout_selftest(int64_t limit_ns, void* stream) {
  if (limit_ns < 1000 || limit_ns > 1000000000)
    return set_error(HI3D_ERR_INVALID_ARGUMENT, "wait_timeout_selftest: limit %lld ns outside [1e3, 1e9]",
                     (long long)limit_ns);
  wait_timeout_selftest_kernel<<<1, 32, 0, as_stream(stream)>>>((uint64_t)limit_ns);
  return check_launch("wait_timeout_selftest");
}

extern "C" int hi3d_version(void) { return 100; }

extern "C" const char* hi3d_last_error_string(void) { return t_last_error; }

extern "C" int hi3d_device_status(int* code, int* where, int* block, int* detail, int reset) {
  cudaError_t e = cudaDeviceSynchronize();
  if (e != cudaSuccess) return set_error(HI3D_ERR_CUDA, "cudaDeviceSynchronize: %s", cudaGetErrorString(e));
  DeviceStatus first = {0, 0, 0, 0};
  for (int i = 0; i < g_num_readers; ++i) {
    DeviceStatus s;
    e = g_readers[i](&s, reset != 0);
    if (e != cudaSuccess) return set_error(HI3D_ERR_CUDA, "reading device status: %s", cudaGetErrorString(e));
    if (first.code == 0 && s.code != 0) first = s;
  }
  if (code) *code = first.code;
  if (where) *where = first.where;
  if (block) *block = first.block;
  if (detail) *detail = first.detail;
  return HI3D_OK;
}

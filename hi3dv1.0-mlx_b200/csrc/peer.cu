// Cross-GPU barrier for the K/V gather of the query-sharded block.
//
// The QKV projection of every rank stores its K/V rows into all peers' gather
// buffers (symmetric memory: each peer's buffer mapped into this process, plain
// stores over NVLink; hi3d_gemm_qkv_rope_peers).  Before a rank's attention may
// read its buffer, every peer's projection must have finished: each rank writes
// an epoch number into its word of every peer's flag array with a release store
// at system scope, then polls its own flag array with acquire loads until every
// peer's word has reached the epoch.  The projection ran earlier on the same
// stream, so its stores are performed before this kernel's release store.
//
// The gather buffers alternate between two sets from block to block, so a
// rank's stores for block i + 1 cannot overwrite rows a peer still reads in
// block i - 1: the peer's attention of block i - 1 precedes its arrival at the
// barrier of block i, which this rank waited for before block i + 1.
//
// Every wait is bounded (wall clock, plus a poll-count backstop): a peer that
// never arrives leaves HI3D_ERR_DEVICE_TIMEOUT in the device status word and the
// kernel returns, so the host sees an error instead of a hung GPU.
#include "abi.h"
#include "common.cuh"

namespace hi3d {
namespace {

constexpr int kSitePeerBarrier = 950;

__device__ __forceinline__ void st_release_sys(uint32_t* p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// One thread per peer: signal the peer, then wait for the peer's signal.
__global__ void peer_barrier_kernel(uint32_t* const* flags, int rank, int world, uint32_t epoch, uint64_t limit_ns) {
  const int peer = threadIdx.x;
  if (peer >= world || peer == rank) return;
  st_release_sys(flags[peer] + rank, epoch);
  const uint32_t* mine = flags[rank] + peer;
  const uint64_t t0 = global_ns();
  for (uint32_t polls = 0;; ++polls) {
    if ((int32_t)(ld_acquire_sys(mine) - epoch) >= 0) return;
    if (global_ns() - t0 > limit_ns || polls > kSpinLimit) {
      report_error(HI3D_ERR_DEVICE_TIMEOUT, kSitePeerBarrier, peer);
      return;
    }
    __nanosleep(64);
  }
}

}  // namespace
}  // namespace hi3d

using namespace hi3d;

extern "C" int hi3d_peer_barrier(void* const* flags_dev, int rank, int world, uint32_t epoch, int64_t limit_ns,
                                 void* stream) {
  if (!flags_dev || world < 1 || world > 8 || rank < 0 || rank >= world)
    return set_error(HI3D_ERR_INVALID_ARGUMENT, "peer_barrier: bad arguments (world in [1, 8])");
  if (limit_ns < 1000 || limit_ns > 60000000000ll)
    return set_error(HI3D_ERR_INVALID_ARGUMENT, "peer_barrier: limit %lld ns outside [1e3, 6e10]",
                     (long long)limit_ns);
  if (world == 1) return HI3D_OK;
  peer_barrier_kernel<<<1, 32, 0, as_stream(stream)>>>(reinterpret_cast<uint32_t* const*>(flags_dev), rank, world,
                                                       epoch, (uint64_t)limit_ns);
  return check_launch("peer_barrier");
}

// Query-sharded self-attention over the GPUs of one node, one process per GPU.
//
// Each rank holds a contiguous slice of S rows of one sequence: its queries, keys
// and values ([S, H, D], token-major).  The K/V slices of all ranks are
// all-gathered over NCCL on a high-priority side stream; the caller's stream waits
// for the gather and attends all keys in one launch (key-split by the cost model
// below when the grid is short of waves).  Attending the own keys while the gather
// runs and merging partials was measured slower: the partial kernel and the merge
// cost more than the exposed gather.
//
// NCCL is loaded at run time (dlopen of libnccl.so.2), so the library has no link
// dependency on it; inside a process that already loaded NCCL (e.g. through
// PyTorch) the same copy is used.
#include <dlfcn.h>
#include <nccl.h>

#include <chrono>
#include <cmath>
#include <cstring>
#include <mutex>
#include <thread>

#include "abi.h"

namespace hi3d {
namespace {

struct NcclApi {
  ncclResult_t (*get_unique_id)(ncclUniqueId*) = nullptr;
  ncclResult_t (*comm_init_rank)(ncclComm_t*, int, ncclUniqueId, int) = nullptr;
  ncclResult_t (*comm_destroy)(ncclComm_t) = nullptr;
  ncclResult_t (*all_gather)(const void*, void*, size_t, ncclDataType_t, ncclComm_t, cudaStream_t) = nullptr;
  ncclResult_t (*group_start)() = nullptr;
  ncclResult_t (*group_end)() = nullptr;
  ncclResult_t (*comm_get_async_error)(ncclComm_t, ncclResult_t*) = nullptr;
  ncclResult_t (*comm_abort)(ncclComm_t) = nullptr;
  const char* (*error_string)(ncclResult_t) = nullptr;
  bool ok = false;
};

const NcclApi& nccl() {
  static NcclApi api;
  static std::once_flag once;
  std::call_once(once, [] {
    void* h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
    if (!h) h = dlopen("libnccl.so", RTLD_NOW | RTLD_GLOBAL);
    if (!h) return;
    api.get_unique_id = reinterpret_cast<decltype(api.get_unique_id)>(dlsym(h, "ncclGetUniqueId"));
    api.comm_init_rank = reinterpret_cast<decltype(api.comm_init_rank)>(dlsym(h, "ncclCommInitRank"));
    api.comm_destroy = reinterpret_cast<decltype(api.comm_destroy)>(dlsym(h, "ncclCommDestroy"));
    api.all_gather = reinterpret_cast<decltype(api.all_gather)>(dlsym(h, "ncclAllGather"));
    api.group_start = reinterpret_cast<decltype(api.group_start)>(dlsym(h, "ncclGroupStart"));
    api.group_end = reinterpret_cast<decltype(api.group_end)>(dlsym(h, "ncclGroupEnd"));
    api.error_string = reinterpret_cast<decltype(api.error_string)>(dlsym(h, "ncclGetErrorString"));
    api.comm_get_async_error =
        reinterpret_cast<decltype(api.comm_get_async_error)>(dlsym(h, "ncclCommGetAsyncError"));
    api.comm_abort = reinterpret_cast<decltype(api.comm_abort)>(dlsym(h, "ncclCommAbort"));
    api.ok = api.get_unique_id && api.comm_init_rank && api.comm_destroy && api.all_gather && api.group_start &&
             api.group_end && api.error_string && api.comm_get_async_error && api.comm_abort;
  });
  return api;
}

int nccl_error(const char* what, ncclResult_t r) {
  return set_error(HI3D_ERR_NCCL, "%s: %s", what, nccl().error_string ? nccl().error_string(r) : "NCCL error");
}

// A communicator with the side stream and events of the K/V gather.  `aborted`
// is set once ncclCommAbort has run (by hi3d_nccl_comm_abort, or by
// hi3d_nccl_comm_wait on an asynchronous error or at its limit); the
// communicator then refuses new work and is only destroyed.
struct Comm {
  ncclComm_t comm = nullptr;
  int rank = 0, world = 1, device = 0;
  cudaStream_t side = nullptr;
  cudaEvent_t inputs_ready = nullptr, gathered = nullptr;
  bool aborted = false;
};

int abort_comm(Comm* c) {
  if (c->aborted) return HI3D_OK;
  c->aborted = true;
  ncclResult_t r = nccl().comm_abort(c->comm);
  c->comm = nullptr;
  return r == ncclSuccess ? HI3D_OK : nccl_error("ncclCommAbort", r);
}

// Key splits per query block (as the Python side, attention.auto_splits): the s minimising
// the modelled launch time ceil(ctas * s / sms) * (overhead + key_blocks / s), with the fixed
// cost of a CTA (set-up, first scores, epilogue) ≈ 2.25 key blocks and a split launch (the
// partial kernel, whose fp32 partials and merge follow) charged 1.2x the single pass, taken only
// when it beats no split by more than 3 % and leaves at least two key blocks per split.
int auto_splits(int64_t ctas, int64_t key_blocks, int sms) {
  constexpr double kOverhead = 2.25, kPartial = 1.2;
  auto cost = [&](int s) {
    return std::ceil((double)ctas * s / sms) * (kOverhead + (double)key_blocks / s) * (s > 1 ? kPartial : 1.0);
  };
  int best = 1;
  double best_t = cost(1);
  for (int s = 2; s <= 8; ++s) {
    if (key_blocks < 2 * s) break;
    const double t = cost(s);
    if (t < best_t * 0.97) {
      best = s;
      best_t = t;
    }
  }
  return best;
}

// The one attention launch of the sharded block: this rank's s_rows queries over all
// world * s_rows keys, as one dense sequence ([rows, heads, head_dim] token-major operands).
hi3d_attn_args gathered_args(const void* q, const void* k_all, const void* v_all, void* out, int64_t s_rows,
                             int64_t total, int heads, int head_dim, int dtype, float scale) {
  const int64_t row = (int64_t)heads * head_dim;
  hi3d_attn_args a{};
  a.q = q;
  a.k = k_all;
  a.v = v_all;
  a.out = out;
  a.q_row = a.k_row = a.v_row = a.o_row = row;
  a.q_head = a.k_head = a.v_head = a.o_head = head_dim;
  a.q_batch = a.o_batch = s_rows * row;
  a.k_batch = a.v_batch = 0;
  a.nq = s_rows;
  a.nk = total;
  a.max_seqlen_q = s_rows;
  a.num_seqs = 1;
  a.heads = heads;
  a.head_dim = head_dim;
  a.dtype = dtype;
  a.scale = scale;
  return a;
}

int plan_splits(int world, int64_t s_rows, int heads, int head_dim) {
  const int bk = head_dim == 64 ? 128 : 64;
  const int64_t keys = s_rows * world;
  return keys > 0 ? auto_splits((s_rows + 255) / 256 * heads, (keys + bk - 1) / bk, sm_count()) : 1;
}

}  // namespace
}  // namespace hi3d

using namespace hi3d;

extern "C" int hi3d_nccl_unique_id(void* id) {
  if (!id) return set_error(HI3D_ERR_INVALID_ARGUMENT, "nccl_unique_id: null pointer");
  if (!nccl().ok) return set_error(HI3D_ERR_NCCL, "nccl_unique_id: libnccl.so.2 could not be loaded");
  ncclUniqueId u;
  ncclResult_t r = nccl().get_unique_id(&u);
  if (r != ncclSuccess) return nccl_error("ncclGetUniqueId", r);
  memcpy(id, &u, sizeof(u));
  return HI3D_OK;
}

extern "C" int hi3d_nccl_comm_init(const void* id, int world, int rank, void** comm) {
  if (!id || !comm || world < 1 || rank < 0 || rank >= world)
    return set_error(HI3D_ERR_INVALID_ARGUMENT, "nccl_comm_init: bad arguments");
  if (!nccl().ok) return set_error(HI3D_ERR_NCCL, "nccl_comm_init: libnccl.so.2 could not be loaded");
  Comm* c = new Comm;
  c->rank = rank;
  c->world = world;
  cudaGetDevice(&c->device);
  ncclUniqueId u;
  memcpy(&u, id, sizeof(u));
  ncclResult_t r = nccl().comm_init_rank(&c->comm, world, u, rank);
  if (r != ncclSuccess) {
    delete c;
    return nccl_error("ncclCommInitRank", r);
  }
  // the gather's side stream at the highest priority: its NCCL kernel takes the next SMs that
  // free up while the attention grid occupies the GPU
  int lo_prio = 0, hi_prio = 0;
  cudaError_t e = cudaDeviceGetStreamPriorityRange(&lo_prio, &hi_prio);
  if (e == cudaSuccess) e = cudaStreamCreateWithPriority(&c->side, cudaStreamNonBlocking, hi_prio);
  if (e == cudaSuccess) e = cudaEventCreateWithFlags(&c->inputs_ready, cudaEventDisableTiming);
  if (e == cudaSuccess) e = cudaEventCreateWithFlags(&c->gathered, cudaEventDisableTiming);
  if (e != cudaSuccess) {
    nccl().comm_destroy(c->comm);
    delete c;
    return set_error(HI3D_ERR_CUDA, "nccl_comm_init: stream/event: %s", cudaGetErrorString(e));
  }
  *comm = c;
  return HI3D_OK;
}

extern "C" int hi3d_nccl_comm_check(void* comm) {
  if (!comm) return set_error(HI3D_ERR_INVALID_ARGUMENT, "nccl_comm_check: null communicator");
  Comm* c = static_cast<Comm*>(comm);
  if (c->aborted) return set_error(HI3D_ERR_NCCL, "nccl_comm_check: communicator aborted");
  ncclResult_t async = ncclSuccess;
  ncclResult_t r = nccl().comm_get_async_error(c->comm, &async);
  if (r != ncclSuccess) return nccl_error("ncclCommGetAsyncError", r);
  if (async != ncclSuccess && async != ncclInProgress) return nccl_error("asynchronous NCCL error", async);
  return HI3D_OK;
}

extern "C" int hi3d_nccl_comm_abort(void* comm) {
  if (!comm) return set_error(HI3D_ERR_INVALID_ARGUMENT, "nccl_comm_abort: null communicator");
  return abort_comm(static_cast<Comm*>(comm));
}

extern "C" int hi3d_nccl_comm_wait(void* comm, void* stream, int64_t timeout_ms) {
  if (!comm || timeout_ms < 0) return set_error(HI3D_ERR_INVALID_ARGUMENT, "nccl_comm_wait: bad arguments");
  Comm* c = static_cast<Comm*>(comm);
  if (c->aborted) return set_error(HI3D_ERR_NCCL, "nccl_comm_wait: communicator aborted");
  cudaStream_t st = as_stream(stream);
  const auto t0 = std::chrono::steady_clock::now();
  for (;;) {
    // the caller's stream waits on the gather, so its completion covers the side stream's
    // work of every hi3d_sharded_attn enqueued on it; the side stream is checked as well
    cudaError_t e1 = cudaStreamQuery(st), e2 = cudaStreamQuery(c->side);
    if (e1 != cudaSuccess && e1 != cudaErrorNotReady)
      return set_error(HI3D_ERR_CUDA, "nccl_comm_wait: %s", cudaGetErrorString(e1));
    if (e2 != cudaSuccess && e2 != cudaErrorNotReady)
      return set_error(HI3D_ERR_CUDA, "nccl_comm_wait: %s", cudaGetErrorString(e2));
    if (e1 == cudaSuccess && e2 == cudaSuccess) return HI3D_OK;
    ncclResult_t async = ncclSuccess;
    ncclResult_t r = nccl().comm_get_async_error(c->comm, &async);
    if (r != ncclSuccess || (async != ncclSuccess && async != ncclInProgress)) {
      const ncclResult_t why = r != ncclSuccess ? r : async;
      abort_comm(c);
      return nccl_error("nccl_comm_wait: asynchronous NCCL error, communicator aborted", why);
    }
    const auto ms =
        std::chrono::duration_cast<std::chrono::milliseconds>(std::chrono::steady_clock::now() - t0).count();
    if (ms >= timeout_ms) {
      abort_comm(c);
      return set_error(HI3D_ERR_NCCL, "nccl_comm_wait: work not finished after %lld ms, communicator aborted",
                       (long long)timeout_ms);
    }
    std::this_thread::sleep_for(std::chrono::microseconds(100));
  }
}

extern "C" int hi3d_nccl_comm_destroy(void* comm) {
  if (!comm) return HI3D_OK;
  Comm* c = static_cast<Comm*>(comm);
  if (!c->aborted) cudaStreamSynchronize(c->side);
  if (c->inputs_ready) cudaEventDestroy(c->inputs_ready);
  if (c->gathered) cudaEventDestroy(c->gathered);
  if (c->side) cudaStreamDestroy(c->side);
  ncclResult_t r = c->comm ? nccl().comm_destroy(c->comm) : ncclSuccess;
  delete c;
  return r == ncclSuccess ? HI3D_OK : nccl_error("ncclCommDestroy", r);
}

extern "C" int hi3d_sharded_attn_workspace_size(void* comm, int64_t s_rows, int heads, int head_dim,
                                                int64_t* bytes) {
  if (!comm || !bytes || s_rows < 0 || heads <= 0)
    return set_error(HI3D_ERR_INVALID_ARGUMENT, "sharded_attn_workspace_size: bad arguments");
  if (head_dim != 64 && head_dim != 96 && head_dim != 128)
    return set_error(HI3D_ERR_UNSUPPORTED, "sharded_attn_workspace_size: head_dim %d (supported: 64, 96, 128)",
                     head_dim);
  const Comm* c = static_cast<const Comm*>(comm);
  const int splits = plan_splits(c->world, s_rows, heads, head_dim);
  if (splits == 1) {
    *bytes = 256;  // the single pass needs none; a non-empty buffer keeps the contract simple
    return HI3D_OK;
  }
  // the layout of hi3d_flash_attn_split_workspace_size: fp32 O partials, then the log-sum-exps
  const int64_t po = (int64_t)splits * s_rows * heads * head_dim * 4;
  *bytes = ((po + 255) & ~int64_t(255)) + po / head_dim + 256;
  return HI3D_OK;
}

extern "C" int hi3d_sharded_attn(void* comm, const void* q, const void* k, const void* v, void* k_all, void* v_all,
                                 void* out, int64_t s_rows, int heads, int head_dim, float scale, int dtype,
                                 void* workspace, int64_t workspace_bytes, void* stream) {
  if (!comm || !q || !k || !v || !k_all || !v_all || !out || s_rows < 0 || heads <= 0)
    return set_error(HI3D_ERR_INVALID_ARGUMENT, "sharded_attn: bad arguments");
  if (head_dim != 64 && head_dim != 96 && head_dim != 128)
    return set_error(HI3D_ERR_UNSUPPORTED, "sharded_attn: head_dim %d (supported: 64, 96, 128)", head_dim);
  if (static_cast<Comm*>(comm)->aborted) return set_error(HI3D_ERR_NCCL, "sharded_attn: communicator aborted");
  if (dtype != HI3D_F16 && dtype != HI3D_BF16)
    return set_error(HI3D_ERR_INVALID_ARGUMENT, "sharded_attn: dtype must be f16 or bf16");
  Comm* c = static_cast<Comm*>(comm);
  int64_t need = 0;
  int rc = hi3d_sharded_attn_workspace_size(comm, s_rows, heads, head_dim, &need);
  if (rc) return rc;
  if (s_rows == 0) return HI3D_OK;
  if (!workspace || workspace_bytes < need || !aligned16(workspace))
    return set_error(HI3D_ERR_CAPACITY, "sharded_attn: workspace %lld bytes, need %lld (16-byte aligned)",
                     (long long)workspace_bytes, (long long)need);
  cudaStream_t st = as_stream(stream);
  const int64_t row = (int64_t)heads * head_dim;  // elements per token row

  // K/V gather on the high-priority side stream, after the caller's stream has produced k and v;
  // the caller's stream then waits for it.  A single pass over all keys is faster than attending
  // the own slice while the gather runs: the partial kernel and the merge cost more than the
  // exposed gather.
  cudaError_t e = cudaEventRecord(c->inputs_ready, st);
  if (e == cudaSuccess) e = cudaStreamWaitEvent(c->side, c->inputs_ready, 0);
  if (e != cudaSuccess) return set_error(HI3D_ERR_CUDA, "sharded_attn: %s", cudaGetErrorString(e));
  const ncclDataType_t nt = dtype == HI3D_BF16 ? ncclBfloat16 : ncclFloat16;
  ncclResult_t r = nccl().group_start();
  if (r == ncclSuccess) r = nccl().all_gather(k, k_all, (size_t)(s_rows * row), nt, c->comm, c->side);
  if (r == ncclSuccess) r = nccl().all_gather(v, v_all, (size_t)(s_rows * row), nt, c->comm, c->side);
  ncclResult_t r2 = nccl().group_end();
  if (r != ncclSuccess) return nccl_error("ncclAllGather", r);
  if (r2 != ncclSuccess) return nccl_error("ncclGroupEnd", r2);
  e = cudaEventRecord(c->gathered, c->side);
  if (e == cudaSuccess) e = cudaStreamWaitEvent(st, c->gathered, 0);
  if (e != cudaSuccess) return set_error(HI3D_ERR_CUDA, "sharded_attn: %s", cudaGetErrorString(e));

  const hi3d_attn_args a = gathered_args(q, k_all, v_all, out, s_rows, s_rows * c->world, heads, head_dim, dtype,
                                         scale);
  return hi3d_flash_attn_fwd_split(&a, plan_splits(c->world, s_rows, heads, head_dim), workspace, workspace_bytes,
                                   st);
}

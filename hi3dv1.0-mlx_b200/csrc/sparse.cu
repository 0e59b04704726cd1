// Sparse voxel structure and convolution on the GPU.
//
// * Neighbour map (sparse.py:29-43 of the reference): the reference fills a
//   padded dense index grid and reads 27 shifted views.  Here the voxels are
//   inserted into an open-addressing hash table (64-bit packed coordinate key,
//   linear probing, capacity a power of two >= 2N) and every (row, offset)
//   pair is one probe.  table[o, k] = row of coordinate q[o] * stride + d_k,
//   N where absent, offsets in OFFSETS order k = (dx+1)*9 + (dy+1)*3 + (dz+1).
//   With stride 2 and q = the downsampled coordinates the same table drives
//   the stride-2 convolution (tap k reads 2 o + r_k - 1).
// * Downsample structure (sparse.py:217-233): unique coords // 2 in
//   lexicographic order, inverse and counts, via a radix sort of packed keys.
// * Submanifold 3x3x3 convolution (sparse.py:191-214): out[o] = b +
//   sum_k in[table[o, k]] W_k as a gather-GEMM on tcgen05: 128-row output
//   tiles, A rows gathered straight from HBM into the swizzled shared-memory
//   operand layout with cp.async (absent neighbours zero-filled by a 0-byte
//   source), per-tap weights by TMA, fp32 accumulators in TMEM.  Taps with no
//   neighbour in the whole tile are skipped (a 27-bit mask per tile).
#include <cub/cub.cuh>
#include <mutex>

#include "abi.h"
#include "common.cuh"

namespace hi3d {
namespace sparse {

constexpr uint64_t kEmpty = ~0ull;
// device status sites of the hash build (`where` of hi3d_device_status; `detail` = row)
constexpr int kSiteCoordRange = 210;  // a coordinate outside [0, 2^21)
constexpr int kSiteTableFull = 211;   // no free slot (cannot happen at load <= 0.5)
constexpr int kCoordBits = 21;
constexpr int kCoordMax = (1 << kCoordBits) - 1;

__device__ __forceinline__ uint64_t pack_key(int x, int y, int z) {
  return ((uint64_t)x << (2 * kCoordBits)) | ((uint64_t)y << kCoordBits) | (uint64_t)z;
}

__device__ __forceinline__ uint32_t hash_key(uint64_t k) {
  k ^= k >> 33;
  k *= 0xff51afd7ed558ccdull;
  k ^= k >> 33;
  k *= 0xc4ceb9fe1a85ec53ull;
  k ^= k >> 33;
  return (uint32_t)k;
}

__global__ void hash_insert_kernel(const int32_t* __restrict__ coords, int64_t n, uint64_t* __restrict__ keys,
                                   int32_t* __restrict__ vals, uint32_t mask, int* __restrict__ overflow) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  const int x = coords[3 * i], y = coords[3 * i + 1], z = coords[3 * i + 2];
  if (x < 0 || y < 0 || z < 0 || x > kCoordMax || y > kCoordMax || z > kCoordMax) {
    // the row is left out of the table (its neighbours see it as absent) and the
    // first such row is reported through hi3d_device_status
    atomicExch(overflow, 2);
    report_error(HI3D_ERR_INVALID_ARGUMENT, kSiteCoordRange, (int)i);
    return;
  }
  const uint64_t key = pack_key(x, y, z);
  uint32_t slot = hash_key(key) & mask;
  for (uint32_t probe = 0; probe <= mask; ++probe) {
    const uint64_t prev = atomicCAS(reinterpret_cast<unsigned long long*>(keys + slot), (unsigned long long)kEmpty,
                                    (unsigned long long)key);
    if (prev == kEmpty || prev == key) {
      // duplicate coordinates: the last row wins, as the reference's grid assignment
      atomicMax(vals + slot, (int32_t)i);
      return;
    }
    slot = (slot + 1) & mask;
  }
  atomicExch(overflow, 1);
  report_error(HI3D_ERR_CAPACITY, kSiteTableFull, (int)i);
}

__global__ void hash_query_kernel(const int32_t* __restrict__ q, int64_t nq, int stride, const uint64_t* __restrict__ keys,
                                  const int32_t* __restrict__ vals, uint32_t mask, int32_t absent,
                                  int32_t* __restrict__ table) {
  const int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (t >= nq * 27) return;
  const int64_t o = t / 27;
  const int k = (int)(t % 27);
  const int x = q[3 * o] * stride + (k / 9 - 1);
  const int y = q[3 * o + 1] * stride + ((k / 3) % 3 - 1);
  const int z = q[3 * o + 2] * stride + (k % 3 - 1);
  int32_t r = absent;
  if (x >= 0 && y >= 0 && z >= 0 && x <= kCoordMax && y <= kCoordMax && z <= kCoordMax) {
    const uint64_t key = pack_key(x, y, z);
    uint32_t slot = hash_key(key) & mask;
    for (uint32_t probe = 0; probe <= mask; ++probe) {
      const uint64_t kk = keys[slot];
      if (kk == key) {
        r = vals[slot];
        break;
      }
      if (kk == kEmpty) break;
      slot = (slot + 1) & mask;
    }
  }
  table[t] = r;
}

// ---------------------------------------------------------------------------
// downsample structure
// ---------------------------------------------------------------------------
__global__ void half_keys_kernel(const int32_t* __restrict__ coords, int64_t n, uint64_t* __restrict__ keys,
                                 int32_t* __restrict__ rows) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  // coordinates are non-negative (checked by the caller's structure build); // 2 == >> 1
  keys[i] = pack_key(coords[3 * i] >> 1, coords[3 * i + 1] >> 1, coords[3 * i + 2] >> 1);
  rows[i] = (int32_t)i;
}

__global__ void unique_flags_kernel(const uint64_t* __restrict__ sorted, int64_t n, int32_t* __restrict__ flags) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  flags[i] = (i == 0 || sorted[i] != sorted[i - 1]) ? 1 : 0;
}

// group[i] = inclusive_scan(flags)[i] - 1 is the low index of sorted element i
// The radix sort is stable, so `rows` lists the children of each low voxel
// together and in ascending row order: with `children` set it is copied out and
// offsets[g] .. offsets[g + 1] delimit the children of low voxel g.
__global__ void downsample_scatter_kernel(const uint64_t* __restrict__ sorted, const int32_t* __restrict__ rows,
                                          const int32_t* __restrict__ scan, int64_t n, int32_t* __restrict__ low,
                                          int32_t* __restrict__ inverse, int32_t* __restrict__ counts,
                                          int32_t* __restrict__ num_low, int32_t* __restrict__ children,
                                          int32_t* __restrict__ offsets) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  const int g = scan[i] - 1;
  inverse[rows[i]] = g;
  atomicAdd(counts + g, 1);
  if (children) children[i] = rows[i];
  if (i == 0 || sorted[i] != sorted[i - 1]) {
    const uint64_t k = sorted[i];
    low[3 * g] = (int32_t)(k >> (2 * kCoordBits));
    low[3 * g + 1] = (int32_t)((k >> kCoordBits) & kCoordMax);
    low[3 * g + 2] = (int32_t)(k & kCoordMax);
    if (offsets) offsets[g] = (int32_t)i;
  }
  if (i == n - 1) {
    *num_low = g + 1;
    if (offsets) offsets[g + 1] = (int32_t)n;
  }
}

// ---------------------------------------------------------------------------
// Resampling between the fine and the downsampled level (the I/O stages of the
// transformer).  One thread per (row, 8-channel vector): consecutive threads read
// consecutive 16-byte pieces of a row.
// ---------------------------------------------------------------------------
struct alignas(16) Vec8h {
  uint32_t w[4];
};

template <typename T>
__device__ __forceinline__ void add8(float (&acc)[8], const Vec8h& v) {
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const T* e = reinterpret_cast<const T*>(&v.w[i]);
    acc[2 * i] += Cvt<T>::to_f(e[0]);
    acc[2 * i + 1] += Cvt<T>::to_f(e[1]);
  }
}

// out[g] = T(sum_{children i of g, ascending} float(x[i]) / (count_g + 1)):
// Geometry.downsample (transformer.py:261-263), whose scatter-add starts from the
// zero row and whose mean divides by children + 1 (upstream scatter_reduce(mean)
// includes the zero-initialised output, transformer.py:249-251).
template <typename T>
__global__ void downsample_mean_kernel(const T* __restrict__ x, const int32_t* __restrict__ children,
                                       const int32_t* __restrict__ offsets, int64_t m, int vecs,
                                       T* __restrict__ out) {
  const int64_t total = m * vecs;
  for (int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; t < total; t += (int64_t)gridDim.x * blockDim.x) {
    const int64_t g = t / vecs;
    const int v = (int)(t - g * vecs);
    const int b = offsets[g], e = offsets[g + 1];
    float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    for (int i = b; i < e; ++i)
      add8<T>(acc, *reinterpret_cast<const Vec8h*>(x + ((int64_t)children[i] * vecs + v) * 8));
    const float div = (float)(e - b + 1);
    Vec8h o;
#pragma unroll
    for (int i = 0; i < 4; ++i) o.w[i] = Cvt<T>::pack2(acc[2 * i] / div, acc[2 * i + 1] / div);
    *reinterpret_cast<Vec8h*>(out + (g * vecs + v) * 8) = o;
  }
}

// out[o] = T(sum_{k: table[o][k] present} float(proj[inverse[table[o][k]] * 27 + k]) + float(bias)):
// the convolution of the upsampled features without materialising them
// (Sparc3DTransformerMLX._up_conv, transformer.py:449-475): proj holds every low
// voxel projected through all 27 taps, rows p * 27 + k.
template <typename T>
__global__ void upconv_gather_kernel(const T* __restrict__ proj, const int32_t* __restrict__ table,
                                     const int32_t* __restrict__ inverse, int64_t n_fine, int vecs,
                                     const T* __restrict__ bias, T* __restrict__ out) {
  const int64_t total = n_fine * vecs;
  for (int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; t < total; t += (int64_t)gridDim.x * blockDim.x) {
    const int64_t o = t / vecs;
    const int v = (int)(t - o * vecs);
    float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    const int32_t* row = table + o * 27;
#pragma unroll 1
    for (int k = 0; k < 27; ++k) {
      const int32_t j = row[k];
      if (j >= n_fine) continue;  // absent neighbour (sentinel n_fine)
      const int64_t pr = (int64_t)inverse[j] * 27 + k;
      add8<T>(acc, *reinterpret_cast<const Vec8h*>(proj + (pr * vecs + v) * 8));
    }
    if (bias) {
      const Vec8h bv = *reinterpret_cast<const Vec8h*>(bias + v * 8);
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const T* e = reinterpret_cast<const T*>(&bv.w[i]);
        acc[2 * i] = __fadd_rn(acc[2 * i], Cvt<T>::to_f(e[0]));
        acc[2 * i + 1] = __fadd_rn(acc[2 * i + 1], Cvt<T>::to_f(e[1]));
      }
    }
    Vec8h ov;
#pragma unroll
    for (int i = 0; i < 4; ++i) ov.w[i] = Cvt<T>::pack2(acc[2 * i], acc[2 * i + 1]);
    *reinterpret_cast<Vec8h*>(out + (o * vecs + v) * 8) = ov;
  }
}

// out[o] = src[index[o]] (Geometry.upsample, transformer.py:265-266)
__global__ void gather_rows_kernel(const uint4* __restrict__ src, const int32_t* __restrict__ index, int64_t rows,
                                   int vecs, uint4* __restrict__ out) {
  const int64_t total = rows * vecs;
  for (int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; t < total; t += (int64_t)gridDim.x * blockDim.x) {
    const int64_t o = t / vecs;
    const int v = (int)(t - o * vecs);
    out[t] = src[(int64_t)index[o] * vecs + v];
  }
}

static unsigned stride_grid(int64_t total) {
  const int64_t blocks = (total + 255) / 256, cap = (int64_t)sm_count() * 8;
  return (unsigned)(blocks < cap ? blocks : cap);
}

__global__ void check_coords_kernel(const int32_t* __restrict__ coords, int64_t n, int* __restrict__ bad) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n * 3) return;
  const int v = coords[i];
  if (v < 0 || v > kCoordMax) atomicExch(bad, 1);
}

// ---------------------------------------------------------------------------
// gather-GEMM convolution
// ---------------------------------------------------------------------------
constexpr int CV_BM = 128;
constexpr int CV_BN = 256;
constexpr int CV_BKE = 64;  // input channels per stage (128 bytes of fp16)
constexpr int CV_NST = 4;
constexpr int CV_A = CV_BM * 128;
constexpr int CV_B = CV_BN * 128;
constexpr int CV_SMEM = CV_NST * (CV_A + CV_B) + 1024 + 256;
constexpr int CV_THREADS = 288;  // warps 0-3 gather (+ weight TMA), 4 MMA, 5-8 epilogue
constexpr int CV_LAG = 2;        // cp.async groups kept in flight per gather thread

struct ConvParams {
  const void* x;
  const int32_t* table;
  const uint32_t* tap_mask;  // [tiles_m] taps present in each 128-row tile
  const void* bias;
  void* out;
  int n_in, n_out, cin, cout;
  int tiles_m, tiles_n, kchunks;
  int act;  // 1: SiLU of the rounded output, rounded again (the conv2 -> SiLU of a res block)
};

struct ConvBarriers {
  uint64_t full[CV_NST];
  uint64_t empty[CV_NST];
  uint64_t acc_full[2];
  uint64_t acc_empty[2];
  uint32_t tmem_base;
  int abort;
};

__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src, uint32_t src_bytes) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(src_bytes) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}
__device__ __forceinline__ void fence_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

// 27-bit mask of taps with at least one present neighbour among the rows of each tile
__global__ void tap_mask_kernel(const int32_t* __restrict__ table, int n_out, int n_in, uint32_t* __restrict__ mask) {
  const int tile = blockIdx.x;
  uint32_t m = 0;
  for (int r = threadIdx.x; r < CV_BM; r += blockDim.x) {
    const int o = tile * CV_BM + r;
    if (o >= n_out) break;
    for (int k = 0; k < 27; ++k)
      if (table[(int64_t)o * 27 + k] < n_in) m |= 1u << k;
  }
  for (int s = 16; s > 0; s >>= 1) m |= __shfl_xor_sync(0xffffffffu, m, s);
  __shared__ uint32_t part[32];
  if ((threadIdx.x & 31) == 0) part[threadIdx.x >> 5] = m;
  __syncthreads();
  if (threadIdx.x == 0) {
    uint32_t all = 0;
    for (int w = 0; w < (int)(blockDim.x >> 5); ++w) all |= part[w];
    mask[tile] = all;
  }
}

template <typename T>
__global__ void __launch_bounds__(CV_THREADS, 1)
    conv_kernel(const __grid_constant__ CUtensorMap tmW, const ConvParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = smem;
  uint8_t* sB = smem + CV_NST * CV_A;
  ConvBarriers* bar = reinterpret_cast<ConvBarriers*>(sB + CV_NST * CV_B);
  const int warp = warp_id(), lane = lane_id();
  const int num_tiles = p.tiles_m * p.tiles_n;

  if (threadIdx.x == 0) {
    for (int s = 0; s < CV_NST; ++s) {
      mbar_init(&bar->full[s], 128 + 1);  // 128 gather threads + the weight TMA
      mbar_init(&bar->empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&bar->acc_full[a], 1);
      mbar_init(&bar->acc_empty[a], CV_BM);
    }
    bar->abort = 0;
    fence_barrier_init();
  }
  if (warp == 4) {
    tmem_alloc(&bar->tmem_base, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = bar->tmem_base;
  volatile int* abort = &bar->abort;

  if (warp < 4) {
    // ------------------------------------------------------------ gather producers
    const int t = threadIdx.x;          // 0..127
    const int chunk = t & 7;            // 16-byte chunk of a 128-byte row
    const int rsub = t >> 3;            // 0..15
    const T* x = reinterpret_cast<const T*>(p.x);
    if (t == 0) tma_prefetch_desc(&tmW);
    int it = 0;
    bool ok = true;
    int pending[CV_LAG + 1];
    int npend = 0;
    // Neighbour rows of this thread's eight tile rows for one tap, read from the table once
    // per tap (not per channel chunk); the next present tap's rows are requested while the
    // current tap's chunks are gathered, so the table latency is off the gather path.
    auto tap_rows = [&](int mt, int k, int (&dst)[8]) {
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const int o = mt * CV_BM + i * 16 + rsub;
        dst[i] = o < p.n_out ? p.table[(int64_t)o * 27 + k] : p.n_in;
      }
    };
    for (int tile = blockIdx.x; ok && tile < num_tiles; tile += gridDim.x) {
      const int mt = tile / p.tiles_n, nt = tile % p.tiles_n;
      const uint32_t taps = p.tap_mask[mt] & ((1u << 27) - 1);
      int cur[8], nxt[8];
      int k = taps ? __ffs(taps) - 1 : 27;
      if (k < 27) tap_rows(mt, k, cur);
      while (ok && k < 27) {
        const uint32_t later = taps & ~((2u << k) - 1);  // present taps after k
        const int kn = later ? __ffs(later) - 1 : 27;
        if (kn < 27) tap_rows(mt, kn, nxt);
        for (int c = 0; c < p.kchunks; ++c, ++it) {
          const int s = it % CV_NST, n = it / CV_NST;
          if (!(ok = mbar_wait(&bar->empty[s], (n & 1) ^ 1, abort, 201))) break;
          if (t == 0) {
            mbar_arrive_expect_tx(&bar->full[s], CV_B);
            tma_load_3d(sB + s * CV_B, &tmW, &bar->full[s], c * CV_BKE, k, nt * CV_BN);
          }
          const uint32_t dst0 = smem_u32(sA + s * CV_A);
          const int ch = c * CV_BKE + chunk * 8;
#pragma unroll
          for (int i = 0; i < 8; ++i) {
            const int row = i * 16 + rsub;
            const int src_row = cur[i];
            const bool present = src_row < p.n_in && ch < p.cin;
            const T* src = present ? x + (int64_t)src_row * p.cin + ch : x;
            const uint32_t dst = dst0 + row * 128 + ((chunk ^ (row & 7)) << 4);
            cp_async16(dst, src, present ? 16u : 0u);
          }
          cp_async_commit();
          pending[npend++] = s;
          if (npend > CV_LAG) {
            cp_async_wait<CV_LAG>();
            fence_async_smem();
            mbar_arrive(&bar->full[pending[0]]);
            for (int q = 1; q < npend; ++q) pending[q - 1] = pending[q];
            --npend;
          }
        }
        if (kn < 27) {
#pragma unroll
          for (int i = 0; i < 8; ++i) cur[i] = nxt[i];
        }
        k = kn;
      }
    }
    cp_async_wait<0>();
    fence_async_smem();
    for (int q = 0; q < npend; ++q) mbar_arrive(&bar->full[pending[q]]);
    if (ok && t == 0) {
      // tail: wait for the MMA warp's last stage releases before the CTA exits
      for (int j = (it > CV_NST ? it - CV_NST : 0); j < it; ++j)
        mbar_wait(&bar->empty[j % CV_NST], (j / CV_NST) & 1, abort, 202);
    }
  } else if (warp == 4) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t idesc = make_idesc(1, std::is_same<T, __nv_bfloat16>::value ? 1 : 0, 0, 0, CV_BM, CV_BN);
      const uint64_t dA = smem_desc(smem_u32(sA), 16, 1024, kLayoutSW128);
      const uint64_t dB = smem_desc(smem_u32(sB), 16, 1024, kLayoutSW128);
      int it = 0, local = 0;
      bool ok = true;
      for (int tile = blockIdx.x; ok && tile < num_tiles; tile += gridDim.x, ++local) {
        const int acc = local & 1, use = local >> 1;
        const uint32_t taps = p.tap_mask[tile / p.tiles_n];
        if (!(ok = mbar_wait(&bar->acc_empty[acc], (use & 1) ^ 1, abort, 210))) break;
        tc_fence_after();
        const uint32_t d = tmem + acc * CV_BN;
        bool first = true;
        for (int k = 0; ok && k < 27; ++k) {
          if (!(taps >> k & 1u)) continue;
          for (int c = 0; c < p.kchunks; ++c, ++it) {
            const int s = it % CV_NST, n = it / CV_NST;
            if (!(ok = mbar_wait(&bar->full[s], n & 1, abort, 211))) break;
            tc_fence_after();
            const uint64_t a = dA + (uint64_t)((s * CV_A) >> 4), b = dB + (uint64_t)((s * CV_B) >> 4);
#pragma unroll
            for (int q = 0; q < 4; ++q) {
              mma_f16_ss(d, a + (uint64_t)(q * 2), b + (uint64_t)(q * 2), idesc, first ? 0u : 1u);
              first = false;
            }
            tc_commit(&bar->empty[s]);
          }
        }
        if (!ok) break;
        if (first) {
          // no tap present in this tile: the accumulator stays undefined, the
          // epilogue writes the bias only
        }
        tc_commit(&bar->acc_full[acc]);
      }
    }
  } else {
    // ------------------------------------------------------------ epilogue
    const int sub = warp & 3;
    const int r = sub * 32 + lane;
    const uint32_t lane_addr = (uint32_t)(sub * 32) << 16;
    int local = 0;
    for (int tile = blockIdx.x; tile < num_tiles; tile += gridDim.x, ++local) {
      const int acc = local & 1, use = local >> 1;
      if (!mbar_wait(&bar->acc_full[acc], use & 1, abort, 220)) break;
      tc_fence_after();
      const int mt = tile / p.tiles_n, nt = tile % p.tiles_n;
      const bool any_tap = p.tap_mask[mt] != 0;
      const int o = mt * CV_BM + r;
      T* orow = reinterpret_cast<T*>(p.out) + (int64_t)o * p.cout;
      const T* bias = reinterpret_cast<const T*>(p.bias);
#pragma unroll 1
      for (int cc = 0; cc < CV_BN / 32; ++cc) {
        uint32_t v[32];
        __syncwarp();
        tmem_ld32(tmem + lane_addr + acc * CV_BN + cc * 32, v);
        tmem_wait_ld();
        const int n0 = nt * CV_BN + cc * 32;
        if (o >= p.n_out || n0 >= p.cout) continue;
#pragma unroll
        for (int e = 0; e < 32; e += 8) {
          const int n = n0 + e;
          if (n >= p.cout) break;
          float y[8];
#pragma unroll
          for (int q = 0; q < 8; ++q) {
            const int nn = min(n + q, p.cout - 1);
            float a = any_tap ? __uint_as_float(v[e + q]) : 0.0f;
            if (bias) a = __fadd_rn(a, Cvt<T>::to_f(bias[nn]));
            if (p.act) {
              a = Cvt<T>::to_f(Cvt<T>::from_f(a));
              a = a / (1.0f + __expf(-a));
            }
            y[q] = a;
          }
          if (n + 8 <= p.cout) {
            uint4 w;
            w.x = Cvt<T>::pack2(y[0], y[1]);
            w.y = Cvt<T>::pack2(y[2], y[3]);
            w.z = Cvt<T>::pack2(y[4], y[5]);
            w.w = Cvt<T>::pack2(y[6], y[7]);
            *reinterpret_cast<uint4*>(orow + n) = w;
          } else {
            for (int q = 0; q < 8 && n + q < p.cout; ++q) orow[n + q] = Cvt<T>::from_f(y[q]);
          }
        }
      }
      tc_fence_before();
      mbar_arrive(&bar->acc_empty[acc]);
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 4) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

static size_t align256(size_t v) { return (v + 255) & ~size_t(255); }

static uint32_t hash_capacity(int64_t n) {
  uint64_t cap = 1024;
  while (cap < (uint64_t)(2 * n)) cap <<= 1;
  return (uint32_t)cap;
}

}  // namespace sparse
}  // namespace hi3d

using namespace hi3d;
using namespace hi3d::sparse;

extern "C" int hi3d_neighbour_map_workspace_size(int64_t n, int64_t* bytes) {
  if (n < 0 || n > 0x3fffffff || !bytes) return set_error(HI3D_ERR_INVALID_ARGUMENT, "neighbour_map: bad n");
  const uint32_t cap = hash_capacity(n);
  *bytes = (int64_t)(align256((size_t)cap * 8) + align256((size_t)cap * 4) + 256);
  return HI3D_OK;
}

extern "C" int hi3d_neighbour_map_build(const int32_t* coords, int64_t n, const int32_t* query, int64_t nq,
                                        int stride, int32_t* table, void* workspace, int64_t workspace_bytes,
                                        void* stream) {
  if (n < 0 || nq < 0 || (stride != 1 && stride != 2) || (n > 0 && !coords) || !workspace)
    return set_error(HI3D_ERR_INVALID_ARGUMENT, "neighbour_map: bad arguments");
  if ((query ? nq : n) == 0) return HI3D_OK;
  if (!table) return set_error(HI3D_ERR_INVALID_ARGUMENT, "neighbour_map: null table");
  int64_t need = 0;
  int rc = hi3d_neighbour_map_workspace_size(n, &need);
  if (rc) return rc;
  if (workspace_bytes < need)
    return set_error(HI3D_ERR_CAPACITY, "neighbour_map: workspace %lld bytes, need %lld", (long long)workspace_bytes,
                     (long long)need);
  if (!query) {
    query = coords;
    nq = n;
  }
  if (nq == 0) return HI3D_OK;
  cudaStream_t st = as_stream(stream);
  const uint32_t cap = hash_capacity(n);
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  uint64_t* keys = reinterpret_cast<uint64_t*>(ws);
  int32_t* vals = reinterpret_cast<int32_t*>(ws + align256((size_t)cap * 8));
  int* flag = reinterpret_cast<int*>(ws + align256((size_t)cap * 8) + align256((size_t)cap * 4));
  cudaError_t e = cudaMemsetAsync(keys, 0xff, (size_t)cap * 8, st);
  if (e == cudaSuccess) e = cudaMemsetAsync(vals, 0xff, (size_t)cap * 4, st);  // -1: below every row
  if (e == cudaSuccess) e = cudaMemsetAsync(flag, 0, sizeof(int), st);
  if (e != cudaSuccess) return set_error(HI3D_ERR_CUDA, "neighbour_map: memset: %s", cudaGetErrorString(e));
  if (n > 0) hash_insert_kernel<<<(unsigned)((n + 255) / 256), 256, 0, st>>>(coords, n, keys, vals, cap - 1, flag);
  if ((rc = check_launch("neighbour_map insert"))) return rc;
  const int64_t total = nq * 27;
  hash_query_kernel<<<(unsigned)((total + 255) / 256), 256, 0, st>>>(query, nq, stride, keys, vals, cap - 1,
                                                                     (int32_t)n, table);
  return check_launch("neighbour_map query");
}

// ---------------------------------------------------------------------------
// neighbour map without a caller workspace
//
// For callers that cannot allocate device memory: the hash table lives in one
// file-scope device array sized for HI3D_NEIGHBOUR_MAP_NOALLOC_MAX_VOXELS
// voxels (6 MiB + 256 B), present on every GPU that loads this library until
// the process exits.  All calls on a GPU share it, so calls that overlap on
// that GPU (two streams, two host threads) race.
// ---------------------------------------------------------------------------
namespace hi3d {
namespace sparse {

constexpr uint32_t kNoAllocCap = 1u << 19;  // hash_capacity(HI3D_NEIGHBOUR_MAP_NOALLOC_MAX_VOXELS)
constexpr size_t kNoAllocValsOff = (size_t)kNoAllocCap * 8;
constexpr size_t kNoAllocFlagOff = kNoAllocValsOff + (size_t)kNoAllocCap * 4;
constexpr size_t kNoAllocBytes = kNoAllocFlagOff + 256;
static_assert(2 * (uint64_t)HI3D_NEIGHBOUR_MAP_NOALLOC_MAX_VOXELS <= kNoAllocCap, "scratch below the voxel limit");

// keys [cap] u64 at 0, vals [cap] i32 at kNoAllocValsOff, overflow flag at kNoAllocFlagOff
static __device__ __align__(256) uint8_t g_nmap_scratch[kNoAllocBytes];

// In host code `g_nmap_scratch` names a host-side stand-in, not device memory.
// The device address belongs to the context current at the lookup (it changes
// after cudaDeviceReset, and differs under a driver-API context other than the
// primary one), so every call outside stream capture looks it up again in the
// current context; that is a host-side table lookup once the module is loaded.
// The last address per device is kept only for calls made while `st` is
// capturing, where the lookup is not attempted.
constexpr int kMaxDevices = 64;
static std::mutex g_nmap_mu;
static uint8_t* g_nmap_ptr[kMaxDevices] = {};

static int nmap_scratch(cudaStream_t st, uint8_t** out) {
  int dev = -1;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return set_error(HI3D_ERR_CUDA, "neighbour_map_noalloc: cudaGetDevice: %s", cudaGetErrorString(e));
  if (dev < 0 || dev >= kMaxDevices)
    return set_error(HI3D_ERR_UNSUPPORTED, "neighbour_map_noalloc: device ordinal %d above %d", dev, kMaxDevices - 1);
  cudaStreamCaptureStatus capture = cudaStreamCaptureStatusNone;
  e = cudaStreamIsCapturing(st, &capture);
  if (e != cudaSuccess)
    return set_error(HI3D_ERR_CUDA, "neighbour_map_noalloc: cudaStreamIsCapturing: %s", cudaGetErrorString(e));
  std::lock_guard<std::mutex> lock(g_nmap_mu);
  if (capture == cudaStreamCaptureStatusNone) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_nmap_scratch);
    if (e != cudaSuccess)
      return set_error(HI3D_ERR_CUDA, "neighbour_map_noalloc: cudaGetSymbolAddress on device %d: %s", dev,
                       cudaGetErrorString(e));
    g_nmap_ptr[dev] = static_cast<uint8_t*>(p);
  } else if (!g_nmap_ptr[dev]) {
    return set_error(HI3D_ERR_INVALID_ARGUMENT,
                     "neighbour_map_noalloc: first call on device %d made during stream capture; "
                     "make one call on this device before capturing",
                     dev);
  }
  *out = g_nmap_ptr[dev];
  return HI3D_OK;
}

}  // namespace sparse
}  // namespace hi3d

extern "C" int hi3d_neighbour_map_build_noalloc(const int32_t* coords, int64_t n, const int32_t* query, int64_t nq,
                                                int stride, int32_t* table, void* stream) {
  if (n < 0 || nq < 0 || (stride != 1 && stride != 2) || (n > 0 && !coords))
    return set_error(HI3D_ERR_INVALID_ARGUMENT, "neighbour_map_noalloc: bad arguments");
  if (n > HI3D_NEIGHBOUR_MAP_NOALLOC_MAX_VOXELS)
    return set_error(HI3D_ERR_CAPACITY,
                     "neighbour_map_noalloc: %lld voxels exceed the fixed scratch limit of %d; "
                     "use hi3d_neighbour_map_build with a workspace",
                     (long long)n, HI3D_NEIGHBOUR_MAP_NOALLOC_MAX_VOXELS);
  if ((query ? nq : n) == 0) return HI3D_OK;
  if (!table) return set_error(HI3D_ERR_INVALID_ARGUMENT, "neighbour_map_noalloc: null table");
  if (!query) {
    query = coords;
    nq = n;
  }
  cudaStream_t st = as_stream(stream);
  uint8_t* ws = nullptr;
  int rc = nmap_scratch(st, &ws);
  if (rc) return rc;
  const uint32_t cap = hash_capacity(n);  // <= kNoAllocCap by the limit above
  uint64_t* keys = reinterpret_cast<uint64_t*>(ws);
  int32_t* vals = reinterpret_cast<int32_t*>(ws + kNoAllocValsOff);
  int* flag = reinterpret_cast<int*>(ws + kNoAllocFlagOff);
  // the array keeps the previous call's table: clear the slots this call probes
  cudaError_t e = cudaMemsetAsync(keys, 0xff, (size_t)cap * 8, st);
  if (e == cudaSuccess) e = cudaMemsetAsync(vals, 0xff, (size_t)cap * 4, st);
  if (e == cudaSuccess) e = cudaMemsetAsync(flag, 0, sizeof(int), st);
  if (e != cudaSuccess) return set_error(HI3D_ERR_CUDA, "neighbour_map_noalloc: memset: %s", cudaGetErrorString(e));
  if (n > 0) hash_insert_kernel<<<(unsigned)((n + 255) / 256), 256, 0, st>>>(coords, n, keys, vals, cap - 1, flag);
  if ((rc = check_launch("neighbour_map_noalloc insert"))) return rc;
  const int64_t total = nq * 27;
  hash_query_kernel<<<(unsigned)((total + 255) / 256), 256, 0, st>>>(query, nq, stride, keys, vals, cap - 1,
                                                                     (int32_t)n, table);
  return check_launch("neighbour_map_noalloc query");
}

extern "C" int hi3d_downsample_workspace_size(int64_t n, int64_t* bytes) {
  if (n < 0 || n > 0x3fffffff || !bytes) return set_error(HI3D_ERR_INVALID_ARGUMENT, "downsample: bad n");
  size_t sort_tmp = 0, scan_tmp = 0;
  cub::DeviceRadixSort::SortPairs(nullptr, sort_tmp, (const uint64_t*)nullptr, (uint64_t*)nullptr,
                                  (const int32_t*)nullptr, (int32_t*)nullptr, (int)n, 0, 3 * kCoordBits);
  cub::DeviceScan::InclusiveSum(nullptr, scan_tmp, (const int32_t*)nullptr, (int32_t*)nullptr, (int)n);
  const size_t nn = (size_t)(n > 0 ? n : 1);
  *bytes = (int64_t)(align256(nn * 8) * 2 + align256(nn * 4) * 4 + align256(sort_tmp > scan_tmp ? sort_tmp : scan_tmp) +
                     256);
  return HI3D_OK;
}

static int downsample_impl(const int32_t* coords, int64_t n, int32_t* low, int32_t* inverse, int32_t* counts,
                           int32_t* children, int32_t* offsets, int32_t* num_low, void* workspace,
                           int64_t workspace_bytes, void* stream) {
  if (n < 0 || !num_low || !workspace || (n > 0 && (!coords || !low || !inverse || !counts)))
    return set_error(HI3D_ERR_INVALID_ARGUMENT, "downsample_structure: bad arguments");
  int64_t need = 0;
  int rc = hi3d_downsample_workspace_size(n, &need);
  if (rc) return rc;
  if (workspace_bytes < need) return set_error(HI3D_ERR_CAPACITY, "downsample_structure: workspace too small");
  cudaStream_t st = as_stream(stream);
  cudaError_t e = cudaMemsetAsync(num_low, 0, sizeof(int32_t), st);
  if (e != cudaSuccess) return set_error(HI3D_ERR_CUDA, "downsample_structure: %s", cudaGetErrorString(e));
  if (n == 0) return HI3D_OK;
  const size_t nn = (size_t)n;
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  uint64_t* k_in = reinterpret_cast<uint64_t*>(ws);
  uint64_t* k_out = reinterpret_cast<uint64_t*>(ws + align256(nn * 8));
  uint8_t* p = ws + 2 * align256(nn * 8);
  int32_t* r_in = reinterpret_cast<int32_t*>(p);
  int32_t* r_out = reinterpret_cast<int32_t*>(p + align256(nn * 4));
  int32_t* flags = reinterpret_cast<int32_t*>(p + 2 * align256(nn * 4));
  int32_t* scan = reinterpret_cast<int32_t*>(p + 3 * align256(nn * 4));
  void* tmp = p + 4 * align256(nn * 4);
  size_t tmp_bytes = (size_t)(workspace_bytes - (int64_t)((uint8_t*)tmp - ws));
  int* bad = reinterpret_cast<int*>(flags);  // reused before the flags are written
  e = cudaMemsetAsync(bad, 0, sizeof(int), st);
  const unsigned g = (unsigned)((n + 255) / 256);
  check_coords_kernel<<<(unsigned)((3 * n + 255) / 256), 256, 0, st>>>(coords, n, bad);
  int host_bad = 0;
  // the structure is built once per sampling pass; validating the coordinates needs one sync
  e = cudaMemcpyAsync(&host_bad, bad, sizeof(int), cudaMemcpyDeviceToHost, st);
  if (e == cudaSuccess) e = cudaStreamSynchronize(st);
  if (e != cudaSuccess) return set_error(HI3D_ERR_CUDA, "downsample_structure: %s", cudaGetErrorString(e));
  if (host_bad) return set_error(HI3D_ERR_INVALID_ARGUMENT, "downsample_structure: coordinates must be in [0, 2^21)");
  half_keys_kernel<<<g, 256, 0, st>>>(coords, n, k_in, r_in);
  e = cub::DeviceRadixSort::SortPairs(tmp, tmp_bytes, k_in, k_out, r_in, r_out, (int)n, 0, 3 * kCoordBits, st);
  if (e != cudaSuccess) return set_error(HI3D_ERR_CUDA, "downsample_structure: sort: %s", cudaGetErrorString(e));
  unique_flags_kernel<<<g, 256, 0, st>>>(k_out, n, flags);
  e = cub::DeviceScan::InclusiveSum(tmp, tmp_bytes, flags, scan, (int)n, st);
  if (e != cudaSuccess) return set_error(HI3D_ERR_CUDA, "downsample_structure: scan: %s", cudaGetErrorString(e));
  e = cudaMemsetAsync(counts, 0, nn * sizeof(int32_t), st);
  if (e != cudaSuccess) return set_error(HI3D_ERR_CUDA, "downsample_structure: %s", cudaGetErrorString(e));
  downsample_scatter_kernel<<<g, 256, 0, st>>>(k_out, r_out, scan, n, low, inverse, counts, num_low, children,
                                               offsets);
  return check_launch("downsample_structure");
}

extern "C" int hi3d_downsample_structure(const int32_t* coords, int64_t n, int32_t* low, int32_t* inverse,
                                         int32_t* counts, int32_t* num_low, void* workspace, int64_t workspace_bytes,
                                         void* stream) {
  return downsample_impl(coords, n, low, inverse, counts, nullptr, nullptr, num_low, workspace, workspace_bytes,
                         stream);
}

extern "C" int hi3d_downsample_structure_children(const int32_t* coords, int64_t n, int32_t* low, int32_t* inverse,
                                                  int32_t* counts, int32_t* children, int32_t* offsets,
                                                  int32_t* num_low, void* workspace, int64_t workspace_bytes,
                                                  void* stream) {
  if (n > 0 && (!children || !offsets))
    return set_error(HI3D_ERR_INVALID_ARGUMENT, "downsample_structure_children: children and offsets required");
  if (n == 0 && offsets) {
    cudaError_t e = cudaMemsetAsync(offsets, 0, sizeof(int32_t), as_stream(stream));
    if (e != cudaSuccess) return set_error(HI3D_ERR_CUDA, "downsample_structure_children: %s", cudaGetErrorString(e));
  }
  return downsample_impl(coords, n, low, inverse, counts, children, offsets, num_low, workspace, workspace_bytes,
                         stream);
}

static int resample_args(const char* what, const void* a, const void* b, const void* out, int64_t rows,
                         int64_t channels, int dtype) {
  if (!a || !b || !out || rows < 0 || channels <= 0)
    return set_error(HI3D_ERR_INVALID_ARGUMENT, "%s: bad pointers or sizes", what);
  if (channels % 8) return set_error(HI3D_ERR_INVALID_ARGUMENT, "%s: channels must be a multiple of 8", what);
  if (channels / 8 > 0x7fffffff || rows > ((int64_t)1 << 40) / channels)
    return set_error(HI3D_ERR_INVALID_ARGUMENT, "%s: too many elements", what);
  if (!aligned16(a) || !aligned16(out))
    return set_error(HI3D_ERR_INVALID_ARGUMENT, "%s: feature pointers must be 16-byte aligned", what);
  if (dtype != HI3D_F16 && dtype != HI3D_BF16)
    return set_error(HI3D_ERR_INVALID_ARGUMENT, "%s: dtype must be f16 or bf16", what);
  return HI3D_OK;
}

extern "C" int hi3d_downsample_mean(const void* x, const int32_t* children, const int32_t* offsets, int64_t num_low,
                                    int64_t channels, void* out, int dtype, void* stream) {
  int rc = resample_args("downsample_mean", x, children, out, num_low, channels, dtype);
  if (rc) return rc;
  if (!offsets) return set_error(HI3D_ERR_INVALID_ARGUMENT, "downsample_mean: offsets required");
  if (num_low == 0) return HI3D_OK;
  const int vecs = (int)(channels / 8);
  const unsigned grid = stride_grid(num_low * vecs);
  cudaStream_t st = as_stream(stream);
  if (dtype == HI3D_F16)
    downsample_mean_kernel<__half><<<grid, 256, 0, st>>>((const __half*)x, children, offsets, num_low, vecs,
                                                         (__half*)out);
  else
    downsample_mean_kernel<__nv_bfloat16><<<grid, 256, 0, st>>>((const __nv_bfloat16*)x, children, offsets, num_low,
                                                                vecs, (__nv_bfloat16*)out);
  return check_launch("downsample_mean");
}

extern "C" int hi3d_upconv_gather_sum(const void* proj, const int32_t* table, const int32_t* inverse, int64_t n_fine,
                                      int64_t channels, const void* bias, void* out, int dtype, void* stream) {
  int rc = resample_args("upconv_gather_sum", proj, table, out, n_fine, channels, dtype);
  if (rc) return rc;
  if (!inverse) return set_error(HI3D_ERR_INVALID_ARGUMENT, "upconv_gather_sum: inverse required");
  if (bias && !aligned16(bias))
    return set_error(HI3D_ERR_INVALID_ARGUMENT, "upconv_gather_sum: bias must be 16-byte aligned");
  if (n_fine == 0) return HI3D_OK;
  const int vecs = (int)(channels / 8);
  const unsigned grid = stride_grid(n_fine * vecs);
  cudaStream_t st = as_stream(stream);
  if (dtype == HI3D_F16)
    upconv_gather_kernel<__half><<<grid, 256, 0, st>>>((const __half*)proj, table, inverse, n_fine, vecs,
                                                       (const __half*)bias, (__half*)out);
  else
    upconv_gather_kernel<__nv_bfloat16><<<grid, 256, 0, st>>>((const __nv_bfloat16*)proj, table, inverse, n_fine,
                                                              vecs, (const __nv_bfloat16*)bias,
                                                              (__nv_bfloat16*)out);
  return check_launch("upconv_gather_sum");
}

extern "C" int hi3d_gather_rows(const void* src, const int32_t* index, int64_t rows, int64_t channels, void* out,
                                int dtype, void* stream) {
  int rc = resample_args("gather_rows", src, index, out, rows, channels, dtype);
  if (rc) return rc;
  if (rows == 0) return HI3D_OK;
  const int vecs = (int)(channels / 8);
  gather_rows_kernel<<<stride_grid(rows * vecs), 256, 0, as_stream(stream)>>>(
      static_cast<const uint4*>(src), index, rows, vecs, static_cast<uint4*>(out));
  return check_launch("gather_rows");
}

extern "C" int hi3d_conv_tap_mask(const int32_t* table, int64_t n_out, int64_t n_in, uint32_t* tap_mask,
                                  void* stream) {
  if (!table || !tap_mask || n_out < 0 || n_in < 0)
    return set_error(HI3D_ERR_INVALID_ARGUMENT, "conv_tap_mask: bad arguments");
  if (n_out == 0) return HI3D_OK;
  const unsigned tiles = (unsigned)((n_out + CV_BM - 1) / CV_BM);
  tap_mask_kernel<<<tiles, 128, 0, as_stream(stream)>>>(table, (int)n_out, (int)n_in, tap_mask);
  return check_launch("conv_tap_mask");
}

static int num_sms_conv() {
  int dev = 0, n = 0;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
  return n > 0 ? n : 148;
}

extern "C" int hi3d_sparse_conv_act(const void* x, const int32_t* table, const uint32_t* tap_mask, const void* weight,
                                    const void* bias, void* out, int64_t n_in, int64_t n_out, int cin, int cout,
                                    int act, int dtype, void* stream) {
  if (!x || !table || !tap_mask || !weight || !out || n_in < 0 || n_out < 0 || cin <= 0 || cout <= 0)
    return set_error(HI3D_ERR_INVALID_ARGUMENT, "sparse_conv: bad arguments");
  if (act != 0 && act != 1) return set_error(HI3D_ERR_INVALID_ARGUMENT, "sparse_conv: act must be 0 or 1 (SiLU)");
  if (cin % 8 || cout % 8)
    return set_error(HI3D_ERR_INVALID_ARGUMENT, "sparse_conv: channels must be multiples of 8");
  if (!aligned16(x) || !aligned16(weight) || !aligned16(out))
    return set_error(HI3D_ERR_INVALID_ARGUMENT, "sparse_conv: pointers must be 16-byte aligned");
  if (n_in > 0x7ffffffe || n_out > 0x7fffffff)
    return set_error(HI3D_ERR_INVALID_ARGUMENT, "sparse_conv: too many rows");
  if (dtype != HI3D_F16 && dtype != HI3D_BF16)
    return set_error(HI3D_ERR_INVALID_ARGUMENT, "sparse_conv: dtype must be f16 or bf16");
  if (n_out == 0) return HI3D_OK;
  // weight [cout, 27, cin] (spconv (out, 3, 3, 3, in) layout): tap k is a K-major [cout, cin] matrix
  CUtensorMap mw;
  uint64_t dims[3] = {(uint64_t)cin, 27, (uint64_t)cout};
  uint64_t strides[2] = {(uint64_t)cin * 2, (uint64_t)cin * 27 * 2};
  uint32_t box[3] = {CV_BKE, 1, CV_BN};
  int rc = encode_tmap(&mw, dtype == HI3D_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3,
                       weight, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B);
  if (rc) return rc;
  ConvParams p;
  p.x = x;
  p.table = table;
  p.tap_mask = tap_mask;
  p.bias = bias;
  p.out = out;
  p.n_in = (int)n_in;
  p.n_out = (int)n_out;
  p.cin = cin;
  p.cout = cout;
  p.tiles_m = (int)((n_out + CV_BM - 1) / CV_BM);
  p.tiles_n = (cout + CV_BN - 1) / CV_BN;
  p.kchunks = (cin + CV_BKE - 1) / CV_BKE;
  p.act = act;
  const int tiles = p.tiles_m * p.tiles_n;
  const int grid = tiles < num_sms_conv() ? tiles : num_sms_conv();
  cudaStream_t st = as_stream(stream);
  if (dtype == HI3D_F16) {
    cudaError_t e = cudaFuncSetAttribute(conv_kernel<__half>, cudaFuncAttributeMaxDynamicSharedMemorySize, CV_SMEM);
    if (e != cudaSuccess) return set_error(HI3D_ERR_CUDA, "sparse_conv: %s", cudaGetErrorString(e));
    conv_kernel<__half><<<grid, CV_THREADS, CV_SMEM, st>>>(mw, p);
  } else {
    cudaError_t e =
        cudaFuncSetAttribute(conv_kernel<__nv_bfloat16>, cudaFuncAttributeMaxDynamicSharedMemorySize, CV_SMEM);
    if (e != cudaSuccess) return set_error(HI3D_ERR_CUDA, "sparse_conv: %s", cudaGetErrorString(e));
    conv_kernel<__nv_bfloat16><<<grid, CV_THREADS, CV_SMEM, st>>>(mw, p);
  }
  return check_launch("sparse_conv");
}

extern "C" int hi3d_sparse_conv(const void* x, const int32_t* table, const uint32_t* tap_mask, const void* weight,
                                const void* bias, void* out, int64_t n_in, int64_t n_out, int cin, int cout, int dtype,
                                void* stream) {
  return hi3d_sparse_conv_act(x, table, tap_mask, weight, bias, out, n_in, n_out, cin, cout, 0, dtype, stream);
}

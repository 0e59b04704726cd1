// Kernels of the sparse VAE decoder (PTv3 mesh decoder) around the sparse conv:
//
//  * GroupNorm statistics and the GroupNorm + swish prologue of conv(swish(GN(x)))
//    (SparconvVAEDecoderMLX.group_stats / conv_gn_swish, src/hi3d_mac/mlx_backend/
//    vae.py:142-192, kernel kernels.py:242-296).  The activated features are written
//    once, [N, C], and the conv gathers them; the reference instead materialises the
//    gathered [rows, 27 C] block per row block;
//  * the octree child neighbour table (sparse.child_neighbour_table,
//    src/hi3d_mac/mlx_backend/sparse.py:46-95): a child's neighbour at offset d has its
//    parent in the parent's 3x3x3 neighbourhood, so the child table follows from the
//    parent table and the occupancy masks without hashing;
//  * serialized window attention (SparconvVAEDecoderMLX.attention_block,
//    vae.py:249-266): every window of `window` consecutive points in space-filling-curve
//    order attends within itself (the last window is completed with the points before
//    it), heads of width 16..64 on CUDA cores in fp32.
#include <cub/cub.cuh>

#include "abi.h"
#include "common.cuh"

namespace hi3d {
namespace vae {

template <typename X>
__device__ __forceinline__ float load_f(const X* p) {
  return static_cast<float>(*p);
}
template <>
__device__ __forceinline__ float load_f<__half>(const __half* p) {
  return __half2float(*p);
}

template <typename T>
__device__ __forceinline__ T store_t(float v) {
  return static_cast<T>(v);
}
template <>
__device__ __forceinline__ __half store_t<__half>(float v) {
  return __float2half_rn(v);
}

// ---------------------------------------------------------------------------
// GroupNorm statistics.  Stage 1: block b sums rows [b * chunk, (b + 1) * chunk) per
// channel (fp32, rows in order) into partial[b][c] and partial_sq[b][c].  Stage 2 sums
// the partials of each column in a fixed order (deterministic), then per group
// mean = S1 / (count + eps), var = S2 / (count + eps) - mean^2, inv = 1 / sqrt(var + eps)
// with count = n * width (vae.py:142-164), written back per channel.
// ---------------------------------------------------------------------------
template <typename X>
__global__ void __launch_bounds__(256) gn_partial_kernel(const X* __restrict__ x, int64_t n, int c, int64_t chunk,
                                                         float* __restrict__ partial) {
  const int64_t r0 = (int64_t)blockIdx.x * chunk;
  const int64_t r1 = min(n, r0 + chunk);
  float* s1 = partial + (int64_t)blockIdx.x * 2 * c;
  float* s2 = s1 + c;
  for (int ch = threadIdx.x; ch < c; ch += blockDim.x) {
    float a = 0.f, b = 0.f;
    for (int64_t r = r0; r < r1; ++r) {
      const float v = load_f<X>(x + r * c + ch);
      a = __fadd_rn(a, v);
      b = __fmaf_rn(v, v, b);
    }
    s1[ch] = a;
    s2[ch] = b;
  }
}

// Stage 2a: column e of the [blocks][2 c] partials summed by a 32 x 32 thread block: segment y
// sums partials y, y + 32, ... in order (a warp reads 32 consecutive columns of one partial),
// then the 32 segment sums are added in segment order.
__global__ void __launch_bounds__(1024) gn_columns_kernel(const float* __restrict__ partial, int blocks, int cols,
                                                          float* __restrict__ colsum) {
  __shared__ float seg[32][33];
  const int e = blockIdx.x * 32 + threadIdx.x;
  float a = 0.f;
  if (e < cols) {
#pragma unroll 4
    for (int k = threadIdx.y; k < blocks; k += 32) a = __fadd_rn(a, partial[(int64_t)k * cols + e]);
  }
  seg[threadIdx.y][threadIdx.x] = a;
  __syncthreads();
  if (threadIdx.y == 0 && e < cols) {
    float t = 0.f;
    for (int y = 0; y < 32; ++y) t = __fadd_rn(t, seg[y][threadIdx.x]);
    colsum[e] = t;
  }
}

// Stage 2b: per group from the channel sums colsum[0, c) and sums of squares colsum[c, 2 c).
__global__ void __launch_bounds__(256) gn_finish_kernel(const float* __restrict__ colsum, int c, int groups,
                                                        int64_t n, float eps, float* __restrict__ mean,
                                                        float* __restrict__ inv) {
  extern __shared__ float sh[];  // [2 c]
  for (int e = threadIdx.x; e < 2 * c; e += blockDim.x) sh[e] = colsum[e];
  __syncthreads();
  const int width = c / groups;
  const float count = __fadd_rn((float)((double)n * width), eps);
  for (int g = threadIdx.x; g < groups; g += blockDim.x) {
    float a = 0.f, b = 0.f;
    for (int w = 0; w < width; ++w) {
      a = __fadd_rn(a, sh[g * width + w]);
      b = __fadd_rn(b, sh[c + g * width + w]);
    }
    const float m = __fdiv_rn(a, count);
    const float var = __fsub_rn(__fdiv_rn(b, count), __fmul_rn(m, m));
    const float iv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(var, eps)));
    for (int w = 0; w < width; ++w) {
      mean[g * width + w] = m;
      inv[g * width + w] = iv;
    }
  }
}

// swish(u) = u * sigmoid(u) with the stable sigmoid e = 1 / (1 + exp(|u|))
// (kernels.py:242-260): exp and the reciprocal on the MUFU unit (relative error ~1e-6 for
// |u| <= 20); an overflowed exp gives e = 0.
__device__ __forceinline__ float swish_stable(float u) {
  const float e = __fdividef(1.0f, 1.0f + __expf(fabsf(u)));
  return u < 0.0f ? u * e : u * (1.0f - e);
}

// u = (x - mean) * inv * w + b in fp32; swish(u) = u * sigmoid(u) with the stable
// sigmoid e = 1 / (1 + exp(|u|)) (kernels.py:242-260); rounded once to T.
template <typename X, typename T>
__global__ void __launch_bounds__(256) gn_swish_kernel(const X* __restrict__ x, int64_t n, int c,
                                                       const float* __restrict__ mean, const float* __restrict__ inv,
                                                       const float* __restrict__ w, const float* __restrict__ b,
                                                       T* __restrict__ out) {
  const int64_t total = n * c;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
    const int ch = (int)(i % c);
    const float u =
        __fadd_rn(__fmul_rn(__fmul_rn(__fsub_rn(load_f<X>(x + i), mean[ch]), inv[ch]), w[ch]), b[ch]);
    out[i] = store_t<T>(swish_stable(u));
  }
}

// 8 consecutive channels of one row as fp32 (16 bytes of fp16, 32 bytes of fp32)
template <typename X>
__device__ __forceinline__ void load8f(const X* p, float (&v)[8]);
template <>
__device__ __forceinline__ void load8f<__half>(const __half* p, float (&v)[8]) {
  const uint4 r = *reinterpret_cast<const uint4*>(p);
  const __half2* h = reinterpret_cast<const __half2*>(&r);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 f = __half22float2(h[i]);
    v[2 * i] = f.x;
    v[2 * i + 1] = f.y;
  }
}
template <>
__device__ __forceinline__ void load8f<float>(const float* p, float (&v)[8]) {
  const float4 a = *reinterpret_cast<const float4*>(p), b = *reinterpret_cast<const float4*>(p + 4);
  v[0] = a.x, v[1] = a.y, v[2] = a.z, v[3] = a.w, v[4] = b.x, v[5] = b.y, v[6] = b.z, v[7] = b.w;
}
template <typename T>
__device__ __forceinline__ void store8(T* p, const float (&v)[8]);
template <>
__device__ __forceinline__ void store8<__half>(__half* p, const float (&v)[8]) {
  uint4 r;
  __half2* h = reinterpret_cast<__half2*>(&r);
#pragma unroll
  for (int i = 0; i < 4; ++i) h[i] = __floats2half2_rn(v[2 * i], v[2 * i + 1]);
  *reinterpret_cast<uint4*>(p) = r;
}
template <>
__device__ __forceinline__ void store8<float>(float* p, const float (&v)[8]) {
  *reinterpret_cast<float4*>(p) = make_float4(v[0], v[1], v[2], v[3]);
  *reinterpret_cast<float4*>(p + 4) = make_float4(v[4], v[5], v[6], v[7]);
}

// Stage 1 with 8-channel vectors (channels % 8 == 0, <= 2048): thread (rr, v) of the block
// sums channels 8v .. 8v + 7 over rows r0 + rr, r0 + rr + R, ...; the R row lanes are then
// added in lane order through shared memory.
template <typename X>
__global__ void __launch_bounds__(256) gn_partial_v8_kernel(const X* __restrict__ x, int64_t n, int c, int64_t chunk,
                                                            float* __restrict__ partial) {
  extern __shared__ float red[];  // [R][2 c]
  const int vecs = c / 8, lanes = blockDim.x / vecs;
  const int v = threadIdx.x % vecs, rr = threadIdx.x / vecs;
  const int64_t r0 = (int64_t)blockIdx.x * chunk;
  const int64_t r1 = min(n, r0 + chunk);
  if (rr < lanes) {
    float a[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f}, b[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    int64_t r = r0 + rr;
    // four rows' loads in flight, summed in the same row order as one row at a time
    for (; r + 3 * lanes < r1; r += 4 * lanes) {
      float xv[4][8];
#pragma unroll
      for (int u = 0; u < 4; ++u) load8f<X>(x + (r + u * lanes) * c + v * 8, xv[u]);
#pragma unroll
      for (int u = 0; u < 4; ++u)
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          a[i] = __fadd_rn(a[i], xv[u][i]);
          b[i] = __fmaf_rn(xv[u][i], xv[u][i], b[i]);
        }
    }
    for (; r < r1; r += lanes) {
      float xv[8];
      load8f<X>(x + r * c + v * 8, xv);
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        a[i] = __fadd_rn(a[i], xv[i]);
        b[i] = __fmaf_rn(xv[i], xv[i], b[i]);
      }
    }
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      red[rr * 2 * c + v * 8 + i] = a[i];
      red[rr * 2 * c + c + v * 8 + i] = b[i];
    }
  }
  __syncthreads();
  float* out = partial + (int64_t)blockIdx.x * 2 * c;
  for (int e = threadIdx.x; e < 2 * c; e += blockDim.x) {
    float acc = 0.f;
    for (int l = 0; l < lanes; ++l) acc = __fadd_rn(acc, red[l * 2 * c + e]);
    out[e] = acc;
  }
}

template <typename X, typename T>
__global__ void __launch_bounds__(256) gn_swish_v8_kernel(const X* __restrict__ x, int64_t n, int c,
                                                          const float* __restrict__ mean,
                                                          const float* __restrict__ inv, const float* __restrict__ w,
                                                          const float* __restrict__ b, T* __restrict__ out) {
  const int vecs = c / 8;
  const int64_t total = n * vecs;
  for (int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; t < total; t += (int64_t)gridDim.x * blockDim.x) {
    const int ch = (int)(t % vecs) * 8;
    float xv[8], o[8];
    load8f<X>(x + t * 8, xv);
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const float u = __fadd_rn(
          __fmul_rn(__fmul_rn(__fsub_rn(xv[i], mean[ch + i]), inv[ch + i]), w[ch + i]), b[ch + i]);
      o[i] = swish_stable(u);
    }
    store8<T>(out + t * 8, o);
  }
}

// Row-blocked form (256 % (channels / 8) == 0): thread (rr, v) keeps the statistics and
// affine parameters of channels 8v .. 8v + 7 in registers and walks rows rr, rr + R, ... of
// its block's row stride with four rows' loads in flight; same arithmetic per element as
// gn_swish_v8_kernel.
template <typename X, typename T>
__global__ void __launch_bounds__(256, 2) gn_swish_rows_kernel(const X* __restrict__ x, int64_t n, int c,
                                                            const float* __restrict__ mean,
                                                            const float* __restrict__ inv,
                                                            const float* __restrict__ w,
                                                            const float* __restrict__ b, T* __restrict__ out) {
  const int vecs = c / 8, lanes = blockDim.x / vecs;
  const int v = threadIdx.x % vecs, rr = threadIdx.x / vecs;
  float mu[8], iv[8], ww[8], bb[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    mu[i] = mean[v * 8 + i];
    iv[i] = inv[v * 8 + i];
    ww[i] = w[v * 8 + i];
    bb[i] = b[v * 8 + i];
  }
  auto act8 = [&](const float (&xv)[8], float (&o)[8]) {
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const float u = __fadd_rn(__fmul_rn(__fmul_rn(__fsub_rn(xv[i], mu[i]), iv[i]), ww[i]), bb[i]);
      o[i] = swish_stable(u);
    }
  };
  const int64_t step = (int64_t)gridDim.x * lanes;
  int64_t r = (int64_t)blockIdx.x * lanes + rr;
  for (; r + 3 * step < n; r += 4 * step) {
    float xv[4][8];
#pragma unroll
    for (int u = 0; u < 4; ++u) load8f<X>(x + (r + u * step) * c + v * 8, xv[u]);
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      float o[8];
      act8(xv[u], o);
      store8<T>(out + (r + u * step) * c + v * 8, o);
    }
  }
  for (; r < n; r += step) {
    float xv[8], o[8];
    load8f<X>(x + r * c + v * 8, xv);
    act8(xv, o);
    store8<T>(out + r * c + v * 8, o);
  }
}

// ---------------------------------------------------------------------------
// Octree child neighbour table.  Child (p, s) sits at 2 p + bits(s), bits(s) =
// (s >> 2 & 1, s >> 1 & 1, s & 1); its neighbour at offset d = r_k - 1 is child
// (parent_table[p][pk], s') with t = bits + d, pk = the offset of floor(t / 2) and
// s' = the slot of t mod 2.  Children are numbered parent-major, slot-minor.
// ---------------------------------------------------------------------------
__global__ void child_flags_kernel(const uint8_t* __restrict__ mask, int64_t m, int32_t* __restrict__ flags) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i < m) flags[i] = mask[i] ? 1 : 0;
}

// lookup[i] = child id of slot i (i < 8 P) or `num` (unoccupied, and the 8 slots of the
// absent parent P); parent/slot of every child.
__global__ void child_lookup_kernel(const uint8_t* __restrict__ mask, const int32_t* __restrict__ scan, int64_t m,
                                    int32_t* __restrict__ lookup, int32_t* __restrict__ parent,
                                    int32_t* __restrict__ slot, int32_t* __restrict__ num) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  const int32_t total = scan[m - 1] + (mask[m - 1] ? 1 : 0);
  if (i == 0) *num = total;
  if (i < m) {
    if (mask[i]) {
      const int32_t id = scan[i];
      lookup[i] = id;
      parent[id] = (int32_t)(i >> 3);
      slot[id] = (int32_t)(i & 7);
    } else {
      lookup[i] = total;
    }
  } else if (i < m + 8) {
    lookup[i] = total;
  }
}

__global__ void child_table_kernel(const int32_t* __restrict__ parent_table, const int32_t* __restrict__ lookup,
                                   const int32_t* __restrict__ parent, const int32_t* __restrict__ slot,
                                   int64_t num_children, int32_t* __restrict__ table) {
  const int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (t >= num_children * 27) return;
  const int64_t cidx = t / 27;
  const int k = (int)(t - cidx * 27);
  const int s = slot[cidx];
  const int b0 = (s >> 2) & 1, b1 = (s >> 1) & 1, b2 = s & 1;
  const int t0 = b0 + k / 9 - 1, t1 = b1 + (k / 3) % 3 - 1, t2 = b2 + k % 3 - 1;  // in -1 .. 2
  const int pk = ((t0 >> 1) + 1) * 9 + ((t1 >> 1) + 1) * 3 + ((t2 >> 1) + 1);
  const int ss = (t0 & 1) * 4 + (t1 & 1) * 2 + (t2 & 1);
  const int64_t np = parent_table[(int64_t)parent[cidx] * 27 + pk];
  table[t] = lookup[np * 8 + ss];
}

// ---------------------------------------------------------------------------
// Window attention.  One block per (window, group of heads); thread (head, query row).
// Rows come from qkv [n, 3, heads, D] through gather[window * L + i]; the output row
// of window position p = w L + i is written to out[gather[p]] when p < n (later
// positions of the last window repeat rows that an earlier window writes).
// ---------------------------------------------------------------------------
template <typename T, int D>
__global__ void __launch_bounds__(256) window_attn_kernel(const T* __restrict__ qkv, const int32_t* __restrict__ gather,
                                                          int64_t n, int64_t n_pad, int L, int heads,
                                                          int heads_per_block, float scale, T* __restrict__ out) {
  extern __shared__ float kv[];  // [heads_per_block][L][2][D]
  const int64_t w = blockIdx.x;
  const int h0 = blockIdx.y * heads_per_block;
  const int64_t row_stride = (int64_t)3 * heads * D;
  const int64_t base = w * L;
  for (int e = threadIdx.x; e < heads_per_block * L * 2 * D; e += blockDim.x) {
    const int d = e % D;
    const int kvsel = (e / D) & 1;
    const int i = (e / (2 * D)) % L;
    const int hh = e / (2 * D * L);
    float v = 0.f;
    if (h0 + hh < heads && base + i < n_pad) {
      const int64_t r = gather[base + i];
      v = load_f<T>(qkv + r * row_stride + (int64_t)(1 + kvsel) * heads * D + (int64_t)(h0 + hh) * D + d);
    }
    kv[e] = v;
  }
  __syncthreads();
  const int hh = threadIdx.x / L, i = threadIdx.x % L;
  const int h = h0 + hh;
  if (hh >= heads_per_block || h >= heads) return;
  const int64_t p = base + i;
  if (p >= n) return;
  const int64_t r = gather[p];
  float q[D], o[D];
#pragma unroll
  for (int d = 0; d < D; ++d) {
    q[d] = load_f<T>(qkv + r * row_stride + (int64_t)h * D + d) * scale;
    o[d] = 0.f;
  }
  const float* kh = kv + (int64_t)hh * L * 2 * D;
  float mx = -INFINITY, l = 0.f;
  const int64_t left = n_pad - base;
  const int len = left < L ? (int)left : L;
  for (int j = 0; j < len; ++j) {
    const float* kj = kh + j * 2 * D;
    float s = 0.f;
#pragma unroll
    for (int d = 0; d < D; ++d) s = fmaf(q[d], kj[d], s);
    const float mnew = fmaxf(mx, s);
    const float corr = expf(mx - mnew);
    const float pj = expf(s - mnew);
    l = l * corr + pj;
#pragma unroll
    for (int d = 0; d < D; ++d) o[d] = o[d] * corr + pj * kj[D + d];
    mx = mnew;
  }
  const float il = 1.0f / l;
  T* orow = out + r * (int64_t)heads * D + (int64_t)h * D;
#pragma unroll
  for (int d = 0; d < D; ++d) orow[d] = store_t<T>(o[d] * il);
}

// Vectorised form (qkv and out 16-byte aligned): K/V of the block's heads staged with
// 16-byte loads, each thread's query row read the same way, keys taken eight at a time (one
// running-maximum correction per eight keys instead of one per key), the output row written
// as 16-byte vectors.
template <typename T, int D>
__global__ void __launch_bounds__(256, D <= 32 ? 2 : 1) window_attn_v8_kernel(const T* __restrict__ qkv,
                                                             const int32_t* __restrict__ gather, int64_t n,
                                                             int64_t n_pad, int L, int heads, int heads_per_block,
                                                             float scale, T* __restrict__ out) {
  extern __shared__ float kv[];  // [heads_per_block][L][2][D]
  constexpr int V = D / 8;       // 8-element vectors per head row
  const int64_t w = blockIdx.x;
  const int h0 = blockIdx.y * heads_per_block;
  const int64_t row_stride = (int64_t)3 * heads * D;
  const int64_t base = w * L;
  for (int e = threadIdx.x; e < heads_per_block * L * 2 * V; e += blockDim.x) {
    const int ch = e % V;
    int t = e / V;
    const int kvsel = t & 1;
    t >>= 1;
    const int i = t % L, hh = t / L;
    float v[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    if (h0 + hh < heads && base + i < n_pad) {
      const int64_t r = gather[base + i];
      load8f<T>(qkv + r * row_stride + (int64_t)(1 + kvsel) * heads * D + (int64_t)(h0 + hh) * D + ch * 8, v);
    }
    float* dst = kv + ((int64_t)(hh * L + i) * 2 + kvsel) * D + ch * 8;
    *reinterpret_cast<float4*>(dst) = make_float4(v[0], v[1], v[2], v[3]);
    *reinterpret_cast<float4*>(dst + 4) = make_float4(v[4], v[5], v[6], v[7]);
  }
  __syncthreads();
  const int hh = threadIdx.x / L, i = threadIdx.x % L;
  const int h = h0 + hh;
  if (hh >= heads_per_block || h >= heads) return;
  const int64_t p = base + i;
  if (p >= n) return;
  const int64_t r = gather[p];
  float q[D], o[D];
#pragma unroll
  for (int c = 0; c < V; ++c) {
    float v[8];
    load8f<T>(qkv + r * row_stride + (int64_t)h * D + c * 8, v);
#pragma unroll
    for (int u = 0; u < 8; ++u) {
      q[c * 8 + u] = v[u] * scale;
      o[c * 8 + u] = 0.f;
    }
  }
  const float* kh = kv + (int64_t)hh * L * 2 * D;
  float mx = -INFINITY, l = 0.f;
  const int64_t left = n_pad - base;
  const int len = left < L ? (int)left : L;
  for (int j = 0; j < len; j += 8) {
    float s[8];
    float cm = -INFINITY;
#pragma unroll
    for (int u = 0; u < 8; ++u) {
      s[u] = -INFINITY;
      if (j + u < len) {
        const float* kj = kh + (j + u) * 2 * D;
        float a = 0.f;
#pragma unroll
        for (int d = 0; d < D; ++d) a = fmaf(q[d], kj[d], a);
        s[u] = a;
      }
      cm = fmaxf(cm, s[u]);
    }
    const float mnew = fmaxf(mx, cm);
    const float corr = expf(mx - mnew);
    l *= corr;
#pragma unroll
    for (int d = 0; d < D; ++d) o[d] *= corr;
#pragma unroll
    for (int u = 0; u < 8; ++u) {
      if (j + u < len) {
        const float pj = expf(s[u] - mnew);
        const float* vj = kh + (j + u) * 2 * D + D;
        l += pj;
#pragma unroll
        for (int d = 0; d < D; ++d) o[d] = fmaf(pj, vj[d], o[d]);
      }
    }
    mx = mnew;
  }
  const float il = 1.0f / l;
  T* orow = out + r * (int64_t)heads * D + (int64_t)h * D;
#pragma unroll
  for (int c = 0; c < V; ++c) {
    float v[8];
#pragma unroll
    for (int u = 0; u < 8; ++u) v[u] = o[c * 8 + u] * il;
    store8<T>(orow + c * 8, v);
  }
}

// Space-filling-curve keys (vae.py:49-56): bit i of x, y, z goes to key bits 3i + 2,
// 3i + 1, 3i; `swap_xy` serializes (y, x, z) (the "z-trans" order).
__global__ void morton_kernel(const int32_t* __restrict__ coords, int64_t n, int depth, int swap_xy,
                              uint64_t* __restrict__ keys, int32_t* __restrict__ rows) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  uint64_t x = (uint32_t)coords[3 * i], y = (uint32_t)coords[3 * i + 1];
  const uint64_t z = (uint32_t)coords[3 * i + 2];
  if (swap_xy) {
    const uint64_t t = x;
    x = y;
    y = t;
  }
  uint64_t key = 0;
  for (int b = 0; b < depth; ++b)
    key |= ((x >> b) & 1) << (3 * b + 2) | ((y >> b) & 1) << (3 * b + 1) | ((z >> b) & 1) << (3 * b);
  keys[i] = key;
  rows[i] = (int32_t)i;
}

__global__ void inverse_perm_kernel(const int32_t* __restrict__ perm, int64_t n, int32_t* __restrict__ inverse) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) inverse[perm[i]] = (int32_t)i;
}

}  // namespace vae
}  // namespace hi3d

using namespace hi3d;
using namespace hi3d::vae;

static int gn_blocks(int64_t n) {
  const int64_t want = (int64_t)sm_count() * 4;
  return (int)(n < want ? (n > 0 ? n : 1) : want);
}

extern "C" int hi3d_group_norm_stats_workspace_size(int64_t n, int64_t channels, int64_t* bytes) {
  if (n < 0 || channels <= 0 || !bytes)
    return set_error(HI3D_ERR_INVALID_ARGUMENT, "group_norm_stats: bad sizes");
  *bytes = ((int64_t)gn_blocks(n) + 1) * 2 * channels * 4 + 256;  // partials + column sums
  return HI3D_OK;
}

extern "C" int hi3d_group_norm_stats(const void* x, int64_t n, int64_t channels, int groups, float eps, float* mean,
                                     float* inv, void* workspace, int64_t workspace_bytes, int dtype, void* stream) {
  if (!x || !mean || !inv || !workspace || n <= 0 || channels <= 0 || groups <= 0 || channels % groups)
    return set_error(HI3D_ERR_INVALID_ARGUMENT, "group_norm_stats: bad arguments (channels %% groups == 0, n > 0)");
  if (channels > 12288) return set_error(HI3D_ERR_UNSUPPORTED, "group_norm_stats: more than 12288 channels");
  int64_t need = 0;
  hi3d_group_norm_stats_workspace_size(n, channels, &need);
  if (workspace_bytes < need) return set_error(HI3D_ERR_CAPACITY, "group_norm_stats: workspace too small");
  const int blocks = gn_blocks(n);
  const int64_t chunk = (n + blocks - 1) / blocks;
  float* partial = static_cast<float*>(workspace);
  cudaStream_t st = as_stream(stream);
  const int c = (int)channels;
  if (dtype != HI3D_F16 && dtype != HI3D_F32)
    return set_error(HI3D_ERR_INVALID_ARGUMENT, "group_norm_stats: dtype must be f16 or f32");
  const bool vec = c % 8 == 0 && c <= 2048 && aligned16(x);
  if (vec) {
    const int vecs = c / 8, lanes = 256 / vecs;
    const int threads = lanes * vecs;
    const size_t red = (size_t)lanes * 2 * c * sizeof(float);  // <= 16 KB
    if (dtype == HI3D_F16)
      gn_partial_v8_kernel<__half><<<blocks, threads, red, st>>>((const __half*)x, n, c, chunk, partial);
    else
      gn_partial_v8_kernel<float><<<blocks, threads, red, st>>>((const float*)x, n, c, chunk, partial);
  } else if (dtype == HI3D_F16) {
    gn_partial_kernel<__half><<<blocks, 256, 0, st>>>((const __half*)x, n, c, chunk, partial);
  } else {
    gn_partial_kernel<float><<<blocks, 256, 0, st>>>((const float*)x, n, c, chunk, partial);
  }
  const size_t smem = (size_t)2 * c * sizeof(float);
  if (smem > 48 * 1024) {
    cudaError_t e = cudaFuncSetAttribute(gn_finish_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return set_error(HI3D_ERR_CUDA, "group_norm_stats: %s", cudaGetErrorString(e));
  }
  float* colsum = partial + (int64_t)blocks * 2 * c;
  gn_columns_kernel<<<(2 * c + 31) / 32, dim3(32, 32), 0, st>>>(partial, blocks, 2 * c, colsum);
  gn_finish_kernel<<<1, 256, smem, st>>>(colsum, c, groups, n, eps, mean, inv);
  return check_launch("group_norm_stats");
}

extern "C" int hi3d_group_norm_swish(const void* x, int64_t n, int64_t channels, const float* mean, const float* inv,
                                     const float* weight, const float* bias, void* out, int in_dtype, int out_dtype,
                                     void* stream) {
  if (!x || !mean || !inv || !weight || !bias || !out || n < 0 || channels <= 0)
    return set_error(HI3D_ERR_INVALID_ARGUMENT, "group_norm_swish: bad arguments");
  if ((in_dtype != HI3D_F16 && in_dtype != HI3D_F32) || (out_dtype != HI3D_F16 && out_dtype != HI3D_F32))
    return set_error(HI3D_ERR_INVALID_ARGUMENT, "group_norm_swish: dtypes must be f16 or f32");
  if (n == 0) return HI3D_OK;
  cudaStream_t st = as_stream(stream);
  const int c = (int)channels;
  if (c % 8 == 0 && c <= 2048 && 256 % (c / 8) == 0 && aligned16(x) && aligned16(out)) {
    const int lanes = 256 / (c / 8);
    const int64_t blocks = (n + lanes - 1) / lanes, cap = (int64_t)sm_count() * 2;  // two resident per SM
    const unsigned grid = (unsigned)(blocks < cap ? blocks : cap);
    if (in_dtype == HI3D_F16 && out_dtype == HI3D_F16)
      gn_swish_rows_kernel<__half, __half>
          <<<grid, 256, 0, st>>>((const __half*)x, n, c, mean, inv, weight, bias, (__half*)out);
    else if (in_dtype == HI3D_F16)
      gn_swish_rows_kernel<__half, float>
          <<<grid, 256, 0, st>>>((const __half*)x, n, c, mean, inv, weight, bias, (float*)out);
    else if (out_dtype == HI3D_F16)
      gn_swish_rows_kernel<float, __half>
          <<<grid, 256, 0, st>>>((const float*)x, n, c, mean, inv, weight, bias, (__half*)out);
    else
      gn_swish_rows_kernel<float, float>
          <<<grid, 256, 0, st>>>((const float*)x, n, c, mean, inv, weight, bias, (float*)out);
    return check_launch("group_norm_swish");
  }
  if (c % 8 == 0 && aligned16(x) && aligned16(out)) {
    const int64_t total = n * (c / 8), blocks = (total + 255) / 256, cap = (int64_t)sm_count() * 8;
    const unsigned grid = (unsigned)(blocks < cap ? blocks : cap);
    if (in_dtype == HI3D_F16 && out_dtype == HI3D_F16)
      gn_swish_v8_kernel<__half, __half>
          <<<grid, 256, 0, st>>>((const __half*)x, n, c, mean, inv, weight, bias, (__half*)out);
    else if (in_dtype == HI3D_F16)
      gn_swish_v8_kernel<__half, float>
          <<<grid, 256, 0, st>>>((const __half*)x, n, c, mean, inv, weight, bias, (float*)out);
    else if (out_dtype == HI3D_F16)
      gn_swish_v8_kernel<float, __half>
          <<<grid, 256, 0, st>>>((const float*)x, n, c, mean, inv, weight, bias, (__half*)out);
    else
      gn_swish_v8_kernel<float, float>
          <<<grid, 256, 0, st>>>((const float*)x, n, c, mean, inv, weight, bias, (float*)out);
    return check_launch("group_norm_swish");
  }
  const int64_t total = n * channels, blocks = (total + 255) / 256, cap = (int64_t)sm_count() * 8;
  const unsigned grid = (unsigned)(blocks < cap ? blocks : cap);
  if (in_dtype == HI3D_F16 && out_dtype == HI3D_F16)
    gn_swish_kernel<__half, __half><<<grid, 256, 0, st>>>((const __half*)x, n, c, mean, inv, weight, bias, (__half*)out);
  else if (in_dtype == HI3D_F16)
    gn_swish_kernel<__half, float><<<grid, 256, 0, st>>>((const __half*)x, n, c, mean, inv, weight, bias, (float*)out);
  else if (out_dtype == HI3D_F16)
    gn_swish_kernel<float, __half><<<grid, 256, 0, st>>>((const float*)x, n, c, mean, inv, weight, bias, (__half*)out);
  else
    gn_swish_kernel<float, float><<<grid, 256, 0, st>>>((const float*)x, n, c, mean, inv, weight, bias, (float*)out);
  return check_launch("group_norm_swish");
}

extern "C" int hi3d_child_table_workspace_size(int64_t num_parents, int64_t* bytes) {
  if (num_parents < 0 || num_parents > (int64_t)1 << 27 || !bytes)
    return set_error(HI3D_ERR_INVALID_ARGUMENT, "child_table: bad num_parents");
  const int64_t m = num_parents * 8;
  size_t tmp = 0;
  cub::DeviceScan::ExclusiveSum(nullptr, tmp, (const int32_t*)nullptr, (int32_t*)nullptr, (int)(m > 0 ? m : 1));
  // flags, scan and lookup regions of (8 P + 8) int32 each, 256-byte aligned, then the scan's
  // temporary storage
  *bytes = 3 * (((m + 8) * 4 + 255) / 256 * 256) + (int64_t)tmp + 256;
  return HI3D_OK;
}

extern "C" int hi3d_child_structure(const uint8_t* mask, int64_t num_parents, int32_t* parent, int32_t* slot,
                                    int32_t* num_children, void* workspace, int64_t workspace_bytes, void* stream) {
  if (!mask || !parent || !slot || !num_children || !workspace || num_parents <= 0)
    return set_error(HI3D_ERR_INVALID_ARGUMENT, "child_structure: bad arguments");
  int64_t need = 0;
  int rc = hi3d_child_table_workspace_size(num_parents, &need);
  if (rc) return rc;
  if (workspace_bytes < need) return set_error(HI3D_ERR_CAPACITY, "child_structure: workspace too small");
  const int64_t m = num_parents * 8;
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  int32_t* flags = reinterpret_cast<int32_t*>(ws);
  int32_t* scan = reinterpret_cast<int32_t*>(ws + ((m + 8) * 4 + 255) / 256 * 256);
  int32_t* lookup = reinterpret_cast<int32_t*>(ws + 2 * (((m + 8) * 4 + 255) / 256 * 256));
  void* tmp = ws + 3 * (((m + 8) * 4 + 255) / 256 * 256);
  size_t tmp_bytes = (size_t)(workspace_bytes - ((uint8_t*)tmp - ws));
  cudaStream_t st = as_stream(stream);
  const unsigned g = (unsigned)((m + 8 + 255) / 256);
  child_flags_kernel<<<g, 256, 0, st>>>(mask, m, flags);
  cudaError_t e = cub::DeviceScan::ExclusiveSum(tmp, tmp_bytes, flags, scan, (int)m, st);
  if (e != cudaSuccess) return set_error(HI3D_ERR_CUDA, "child_structure: scan: %s", cudaGetErrorString(e));
  child_lookup_kernel<<<g, 256, 0, st>>>(mask, scan, m, lookup, parent, slot, num_children);
  return check_launch("child_structure");
}

extern "C" int hi3d_child_table(const int32_t* parent_table, int64_t num_parents, const int32_t* parent,
                                const int32_t* slot, int64_t num_children, const void* workspace, int32_t* table,
                                void* stream) {
  if (num_children == 0) return HI3D_OK;
  if (!parent_table || !parent || !slot || !workspace || !table || num_parents <= 0 || num_children < 0)
    return set_error(HI3D_ERR_INVALID_ARGUMENT, "child_table: bad arguments");
  const int64_t m = num_parents * 8;
  const int32_t* lookup = reinterpret_cast<const int32_t*>(static_cast<const uint8_t*>(workspace) +
                                                           2 * (((m + 8) * 4 + 255) / 256 * 256));
  const int64_t total = num_children * 27;
  child_table_kernel<<<(unsigned)((total + 255) / 256), 256, 0, as_stream(stream)>>>(parent_table, lookup, parent,
                                                                                      slot, num_children, table);
  return check_launch("child_table");
}

template <typename T, int D>
static int launch_window(const void* qkv, const int32_t* gather, int64_t n, int64_t n_pad, int L, int heads,
                         float scale, void* out, cudaStream_t st) {
  const int hpb = max(1, min(heads, 256 / L));
  const size_t smem = (size_t)hpb * L * 2 * D * sizeof(float);
  const bool vec = aligned16(qkv) && aligned16(out);
  auto kern = vec ? window_attn_v8_kernel<T, D> : window_attn_kernel<T, D>;
  if (smem > 48 * 1024) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return set_error(HI3D_ERR_CUDA, "window_attention: %s", cudaGetErrorString(e));
  }
  dim3 grid((unsigned)(n_pad / L), (unsigned)((heads + hpb - 1) / hpb));
  kern<<<grid, hpb * L, smem, st>>>((const T*)qkv, gather, n, n_pad, L, heads, hpb, scale, (T*)out);
  return check_launch("window_attention");
}

extern "C" int hi3d_window_attention(const void* qkv, const int32_t* gather, int64_t n, int64_t n_pad, int window,
                                     int heads, int head_dim, float scale, void* out, int dtype, void* stream) {
  if (!qkv || !gather || !out || n <= 0 || heads <= 0 || window <= 0 || window > 256)
    return set_error(HI3D_ERR_INVALID_ARGUMENT, "window_attention: bad arguments (0 < window <= 256)");
  const bool whole = n <= window ? n_pad == n : (n_pad % window == 0 && n_pad >= n && n_pad - n < window);
  if (!whole)
    return set_error(HI3D_ERR_INVALID_ARGUMENT, "window_attention: n_pad must be n rounded up to whole windows");
  if (n <= window) window = (int)n;  // one window of all points
  cudaStream_t st = as_stream(stream);
  const bool f16 = dtype == HI3D_F16;
  if (dtype != HI3D_F16 && dtype != HI3D_F32)
    return set_error(HI3D_ERR_INVALID_ARGUMENT, "window_attention: dtype must be f16 or f32");
  switch (head_dim) {
    case 16: return f16 ? launch_window<__half, 16>(qkv, gather, n, n_pad, window, heads, scale, out, st)
                        : launch_window<float, 16>(qkv, gather, n, n_pad, window, heads, scale, out, st);
    case 32: return f16 ? launch_window<__half, 32>(qkv, gather, n, n_pad, window, heads, scale, out, st)
                        : launch_window<float, 32>(qkv, gather, n, n_pad, window, heads, scale, out, st);
    case 64: return f16 ? launch_window<__half, 64>(qkv, gather, n, n_pad, window, heads, scale, out, st)
                        : launch_window<float, 64>(qkv, gather, n, n_pad, window, heads, scale, out, st);
    default: return set_error(HI3D_ERR_UNSUPPORTED, "window_attention: head_dim must be 16, 32 or 64");
  }
}

extern "C" int hi3d_serialize_workspace_size(int64_t n, int64_t* bytes) {
  if (n < 0 || n > 0x7fffffff || !bytes) return set_error(HI3D_ERR_INVALID_ARGUMENT, "serialize: bad n");
  size_t tmp = 0;
  cub::DeviceRadixSort::SortPairs(nullptr, tmp, (const uint64_t*)nullptr, (uint64_t*)nullptr, (const int32_t*)nullptr,
                                  (int32_t*)nullptr, (int)(n > 0 ? n : 1), 0, 63);
  const int64_t nn = n > 0 ? n : 1;
  *bytes = 2 * ((nn * 8 + 255) / 256 * 256) + (nn * 4 + 255) / 256 * 256 + (int64_t)tmp + 256;
  return HI3D_OK;
}

extern "C" int hi3d_serialize(const int32_t* coords, int64_t n, int depth, int swap_xy, int32_t* perm,
                              int32_t* inverse, void* workspace, int64_t workspace_bytes, void* stream) {
  if (!coords || !perm || !inverse || !workspace || n <= 0 || depth < 0 || depth > 21)
    return set_error(HI3D_ERR_INVALID_ARGUMENT, "serialize: bad arguments (0 <= depth <= 21)");
  int64_t need = 0;
  int rc = hi3d_serialize_workspace_size(n, &need);
  if (rc) return rc;
  if (workspace_bytes < need) return set_error(HI3D_ERR_CAPACITY, "serialize: workspace too small");
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  const int64_t kb = (n * 8 + 255) / 256 * 256;
  uint64_t* k_in = reinterpret_cast<uint64_t*>(ws);
  uint64_t* k_out = reinterpret_cast<uint64_t*>(ws + kb);
  int32_t* r_in = reinterpret_cast<int32_t*>(ws + 2 * kb);
  void* tmp = ws + 2 * kb + (n * 4 + 255) / 256 * 256;
  size_t tmp_bytes = (size_t)(workspace_bytes - ((uint8_t*)tmp - ws));
  cudaStream_t st = as_stream(stream);
  const unsigned g = (unsigned)((n + 255) / 256);
  morton_kernel<<<g, 256, 0, st>>>(coords, n, depth, swap_xy, k_in, r_in);
  // LSD radix sort: stable, so equal keys keep their row order (numpy argsort kind="stable")
  cudaError_t e = cub::DeviceRadixSort::SortPairs(tmp, tmp_bytes, k_in, k_out, r_in, perm, (int)n, 0,
                                                  depth > 0 ? 3 * depth : 1, st);
  if (e != cudaSuccess) return set_error(HI3D_ERR_CUDA, "serialize: sort: %s", cudaGetErrorString(e));
  inverse_perm_kernel<<<g, 256, 0, st>>>(perm, n, inverse);
  return check_launch("serialize");
}

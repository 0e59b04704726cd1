// HBM-bound row kernels of the block: LayerNorm + adaLN modulation,
// RoPE + per-head QK RMS norm + head split, gate/residual and GELU epilogues.
//
// All of them move 16 bytes per lane per access and reduce with warp
// shuffles; none touches shared memory.  Rounding follows the reference
// operators exactly where it is specified (see each kernel).
#include "abi.h"
#include "common.cuh"

namespace hi3d {

// 16-byte vector of 8 I/O elements.
struct alignas(16) Vec8 {
  uint32_t w[4];
};

template <typename T>
__device__ __forceinline__ void unpack8(const Vec8& v, float (&f)[8]) {
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const T* h = reinterpret_cast<const T*>(&v.w[i]);
    f[2 * i] = Cvt<T>::to_f(h[0]);
    f[2 * i + 1] = Cvt<T>::to_f(h[1]);
  }
}

template <typename T>
__device__ __forceinline__ T round_t(float v) {
  return Cvt<T>::from_f(v);
}

// SiLU of a rounded pair, evaluated in fp32 and rounded once (F.silu on fp16,
// the activation after the res-block norms: sparc3d_transformer.py:137-141).
__device__ __forceinline__ float silu_f(float v) { return v / (1.0f + __expf(-v)); }
template <typename T>
__device__ __forceinline__ uint32_t silu2(uint32_t h) {
  const T* e = reinterpret_cast<const T*>(&h);
  return Cvt<T>::pack2(silu_f(Cvt<T>::to_f(e[0])), silu_f(Cvt<T>::to_f(e[1])));
}

// ---------------------------------------------------------------------------
// LayerNorm32 (+ affine) (+ modulation) (+ SiLU), one warp per row.
//
// Semantics of kernels.py:162-201: fp32 sum -> mean = sum / C; fp32 sum of
// squared deviations; inv = 1 / sqrt(sumsq / C + eps) (IEEE sqrt and divide);
// y = (x - mean) * inv; affine y = y * w + b without contraction; h = T(y);
// modulation h = T(float(h) * float(scale)); h = T(float(h) + float(shift));
// act: h = T(silu(float(h))).
// NCH = ceil(channels / 256) chunks of 8 elements per lane held in registers
// (channels % 8 == 0, <= 4352).
// ---------------------------------------------------------------------------
constexpr int kLnRowsPerBlock = 4;  // one warp per row: 128-thread blocks, 16 resident per SM

template <typename T, int NCH, bool AFFINE, bool MODULATE, bool ACT>
__global__ void __launch_bounds__(kLnRowsPerBlock * 32)
    ln_mod_kernel(const T* __restrict__ x, T* __restrict__ out, int64_t rows, int C, float eps,
                  const float* __restrict__ weight, const float* __restrict__ bias, const T* __restrict__ scale,
                  const T* __restrict__ shift, int64_t rows_per_batch, int64_t mod_stride) {
  const int lane = threadIdx.x & 31;
  // The fp32 affine parameters are the same for every row: staged once per block in
  // shared memory ([weight | bias], NCH * 256 each, zero past C), so the per-row
  // reads are short shared-memory loads instead of L1/L2 round trips.  Layout: the
  // channels c*256 + 8 l + 4 h + k (lane l, half h, k < 4) of chunk c sit at float4
  // (2c + h) * 32 + l, so each 16-byte load of a warp reads 512 contiguous bytes (4
  // shared-memory wavefronts instead of 8 for the natural order's 32-byte lane stride).
  extern __shared__ float ln_wb[];
  if constexpr (AFFINE) {
    for (int i = threadIdx.x; i < NCH * 256; i += blockDim.x) {
      const int c = i >> 8, l = (i >> 3) & 31, h = (i >> 2) & 1, k = i & 3;
      const int pos = (((c * 2 + h) * 32 + l) << 2) + k;
      ln_wb[pos] = i < C ? weight[i] : 0.f;
      ln_wb[NCH * 256 + pos] = i < C ? bias[i] : 0.f;
    }
    __syncthreads();
  }
  // grid-stride over rows (the grid is sized to whole waves), one warp per row
  for (int64_t row = (int64_t)blockIdx.x * kLnRowsPerBlock + (threadIdx.x >> 5); row < rows;
       row += (int64_t)gridDim.x * kLnRowsPerBlock) {
    const T* xr = x + row * C;
    T* yr = out + row * C;

    // chunk c covers channels [c*256, c*256+256); only the last chunk can be partial.
    // Pairs of channels travel as f32x2: one instruction per pair for each step.
    Vec8 raw[NCH];
#pragma unroll
    for (int c = 0; c < NCH; ++c) {
      raw[c] = Vec8{};
      if (c * 256 + lane * 8 < C) raw[c] = *reinterpret_cast<const Vec8*>(xr + c * 256 + lane * 8);
    }
    uint64_t d[NCH][4];
    uint64_t s2 = 0;  // (0.f, 0.f)
#pragma unroll
    for (int c = 0; c < NCH; ++c)
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        d[c][i] = Cvt<T>::to_f2(raw[c].w[i]);
        s2 = f2_add(s2, d[c][i]);
      }
    float slo, shi;
    f2_unpack(s2, slo, shi);
    float sum = slo + shi;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
    const float mean = __fdiv_rn(sum, (float)C);
    const uint64_t neg_mean = f2_splat(-mean);
    uint64_t q2 = 0;
#pragma unroll
    for (int c = 0; c < NCH; ++c) {
      if (c * 256 + lane * 8 < C) {
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          d[c][i] = f2_add(d[c][i], neg_mean);  // x - mean, exact as the scalar subtraction
          q2 = f2_fma(d[c][i], d[c][i], q2);
        }
      }
    }
    float qlo, qhi;
    f2_unpack(q2, qlo, qhi);
    float sq = qlo + qhi;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) sq += __shfl_xor_sync(0xffffffffu, sq, o);
    const uint64_t inv2 = f2_splat(__fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(sq, (float)C), eps))));

    const int64_t mb = MODULATE ? (row / rows_per_batch) * mod_stride : 0;
#pragma unroll
    for (int c = 0; c < NCH; ++c) {
      const int base = c * 256 + lane * 8;
      if (base >= C) continue;
      Vec8 o;
      Vec8 sc, sh;
      if (MODULATE) {
        sc = *reinterpret_cast<const Vec8*>(scale + mb + base);
        sh = *reinterpret_cast<const Vec8*>(shift + mb + base);
      }
      uint64_t wv[4], bv[4];
      if (AFFINE) {
        const float4* w4 = reinterpret_cast<const float4*>(ln_wb) + c * 64 + lane;
        const float4* b4 = reinterpret_cast<const float4*>(ln_wb + NCH * 256) + c * 64 + lane;
        const float4 w0 = w4[0], w1 = w4[32], b0 = b4[0], b1 = b4[32];
        wv[0] = f2_pack(w0.x, w0.y), wv[1] = f2_pack(w0.z, w0.w), wv[2] = f2_pack(w1.x, w1.y),
        wv[3] = f2_pack(w1.z, w1.w);
        bv[0] = f2_pack(b0.x, b0.y), bv[1] = f2_pack(b0.z, b0.w), bv[2] = f2_pack(b1.x, b1.y),
        bv[3] = f2_pack(b1.z, b1.w);
      }
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        uint64_t y = f2_mul(d[c][i], inv2);
        if (AFFINE) y = f2_add(f2_mul(y, wv[i]), bv[i]);
        uint32_t h = Cvt<T>::from_f2(y);
        // fp16/bf16 pair multiply and add are correctly rounded, so they equal
        // rounding the fp32 product / sum of the two rounded operands
        if (MODULATE) h = Cvt<T>::add2(Cvt<T>::mul2(h, sc.w[i]), sh.w[i]);
        if (ACT) h = silu2<T>(h);
        o.w[i] = h;
      }
      *reinterpret_cast<Vec8*>(yr + base) = o;
    }
  }
}

template <typename T, int NCH>
static void launch_ln(const void* x, void* out, int64_t rows, int C, float eps, const float* w, const float* b,
                      const void* sc, const void* sh, int64_t rpb, int64_t ms, int act, cudaStream_t st) {
  // at most 16 resident 128-thread blocks per SM (2048 threads): a grid of whole
  // waves, rows by grid stride
  const int64_t blocks = (rows + kLnRowsPerBlock - 1) / kLnRowsPerBlock,
                cap = (int64_t)sm_count() * (2048 / (kLnRowsPerBlock * 32));
  dim3 grid((unsigned)(blocks < cap ? blocks : cap)), block(kLnRowsPerBlock * 32);
  const T* xt = (const T*)x;
  T* ot = (T*)out;
  const T* s = (const T*)sc;
  const T* t = (const T*)sh;
  const size_t wb = (size_t)2 * NCH * 256 * sizeof(float);  // affine parameters in shared memory
  if (act && w)  // the res-block norm1: affine, then SiLU
    ln_mod_kernel<T, NCH, true, false, true><<<grid, block, wb, st>>>(xt, ot, rows, C, eps, w, b, s, t, rpb, ms);
  else if (act)  // the res-block norm2: modulation, then SiLU
    ln_mod_kernel<T, NCH, false, true, true><<<grid, block, 0, st>>>(xt, ot, rows, C, eps, w, b, s, t, rpb, ms);
  else if (w && sc)
    ln_mod_kernel<T, NCH, true, true, false><<<grid, block, wb, st>>>(xt, ot, rows, C, eps, w, b, s, t, rpb, ms);
  else if (w)
    ln_mod_kernel<T, NCH, true, false, false><<<grid, block, wb, st>>>(xt, ot, rows, C, eps, w, b, s, t, rpb, ms);
  else if (sc)
    ln_mod_kernel<T, NCH, false, true, false><<<grid, block, 0, st>>>(xt, ot, rows, C, eps, w, b, s, t, rpb, ms);
  else
    ln_mod_kernel<T, NCH, false, false, false><<<grid, block, 0, st>>>(xt, ot, rows, C, eps, w, b, s, t, rpb, ms);
}

template <typename T>
static int dispatch_ln(const void* x, void* out, int64_t rows, int C, float eps, const float* w, const float* b,
                       const void* sc, const void* sh, int64_t rpb, int64_t ms, int act, cudaStream_t st) {
  switch ((C + 255) / 256) {
#define HI3D_LN_CASE(n) \
  case n:               \
    launch_ln<T, n>(x, out, rows, C, eps, w, b, sc, sh, rpb, ms, act, st); break;
    HI3D_LN_CASE(1)
    HI3D_LN_CASE(2)
    HI3D_LN_CASE(3)
    HI3D_LN_CASE(4)
    HI3D_LN_CASE(5)
    HI3D_LN_CASE(6)
    HI3D_LN_CASE(7)
    HI3D_LN_CASE(8)
    HI3D_LN_CASE(9)
    HI3D_LN_CASE(10)
    HI3D_LN_CASE(11)
    HI3D_LN_CASE(12)
    HI3D_LN_CASE(13)
    HI3D_LN_CASE(14)
    HI3D_LN_CASE(15)
    HI3D_LN_CASE(16)
    HI3D_LN_CASE(17)
#undef HI3D_LN_CASE
    default:
      return set_error(HI3D_ERR_UNSUPPORTED, "layer_norm_modulate: channels %d not supported (multiple of 8, <= 4352)",
                       C);
  }
  return check_launch("layer_norm_modulate");
}

// ---------------------------------------------------------------------------
// RoPE + QK RMS norm + split.  A group of G lanes handles one (row, part,
// head); each active lane owns 8 W consecutive channels (W 16-byte vectors,
// 4 W rotation pairs).  Norm reduction by xor-shuffles in the group.
// kernels.py:22-57 semantics: re = x0 c - x1 s, im = x0 s + x1 c (fp32);
// nrm = max(sqrt(sum re^2 + im^2), 1e-12); y = re / nrm * g * sqrt(D), the
// division taken once per head as f = sqrt(D) / nrm (y = re * f * g).
// ---------------------------------------------------------------------------
// lanes per (row, part, head): D / (8 W) data lanes rounded up to a power of two (>= 2)
__host__ __device__ constexpr int rope_group(int D, int W) {
  return D / (8 * W) <= 2 ? 2 : (D / (8 * W) <= 4 ? 4 : (D / (8 * W) <= 8 ? 8 : 16));
}

template <typename T, int D, int W>
__global__ void __launch_bounds__(1024) qkv_rope_rms_kernel(const T* __restrict__ qkv, const float* __restrict__ cosv,
                                                            const float* __restrict__ sinv,
                                                            const float* __restrict__ gq,
                                                            const float* __restrict__ gk, T* __restrict__ q,
                                                            T* __restrict__ k, T* __restrict__ v, int N, int H,
                                                            int token_major) {
  constexpr int CH = 8 * W;        // channels per lane (W 16-byte vectors)
  constexpr int ACTIVE = D / CH;   // lanes per (row, part, head) that hold data
  constexpr int G = rope_group(D, W);
  const int lane = threadIdx.x & 31;
  const int sub = lane % G;
  const int m = blockIdx.x;  // token row of the [B*N, 3*H*D] projection
  const int b = m / N, n = m - b * N;
  const int units = 3 * H;
  const int per_block = (int)(blockDim.x / G);
  const T* row = qkv + (int64_t)m * units * D;
  const float* cs_row = cosv + (int64_t)n * (D / 2);
  const float* sn_row = sinv + (int64_t)n * (D / 2);
  const int c0 = sub * CH;
  // The loop bound is uniform across the block, so every lane reaches every
  // full-mask shuffle; lanes past the last unit contribute zero.
  for (int u0 = 0; u0 < units; u0 += per_block) {
    const int u = u0 + (int)(threadIdx.x / G);
    const bool in_range = u < units;
    const bool valid = in_range && sub < ACTIVE;
    const int part = in_range ? u / H : 0, h = in_range ? u - (u / H) * H : 0;
    Vec8 raw[W];
#pragma unroll
    for (int w = 0; w < W; ++w) {
      raw[w] = Vec8{};
      if (valid) raw[w] = *reinterpret_cast<const Vec8*>(row + (int64_t)u * D + c0 + 8 * w);  // ((m*3+part)*H+h)*D, kernels.py:31
    }
    float rr[CH];
    float ss = 0.f;
#pragma unroll
    for (int w = 0; w < W; ++w) {
      float x[8];
      unpack8<T>(raw[w], x);
#pragma unroll
      for (int i = 0; i < 8; ++i) rr[8 * w + i] = 0.f;
      if (valid && part != 2) {
        const float4 c4 = *reinterpret_cast<const float4*>(cs_row + (c0 + 8 * w) / 2);
        const float4 s4 = *reinterpret_cast<const float4*>(sn_row + (c0 + 8 * w) / 2);
        const float cc[4] = {c4.x, c4.y, c4.z, c4.w}, sv[4] = {s4.x, s4.y, s4.z, s4.w};
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          rr[8 * w + 2 * i] = x[2 * i] * cc[i] - x[2 * i + 1] * sv[i];
          rr[8 * w + 2 * i + 1] = x[2 * i] * sv[i] + x[2 * i + 1] * cc[i];
          ss += rr[8 * w + 2 * i] * rr[8 * w + 2 * i] + rr[8 * w + 2 * i + 1] * rr[8 * w + 2 * i + 1];
        }
      }
    }
#pragma unroll
    for (int o = G / 2; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    if (!valid) continue;
    const int64_t dst_off = token_major ? (((int64_t)b * N + n) * H + h) * D : (((int64_t)b * H + h) * N + n) * D;
    if (part == 2) {
#pragma unroll
      for (int w = 0; w < W; ++w) *reinterpret_cast<Vec8*>(v + dst_off + c0 + 8 * w) = raw[w];
      continue;
    }
    // y = re / nrm * g * sqrt(D), with one division per head: f = sqrt(D) / nrm
    const float f = __fdiv_rn(sqrtf((float)D), fmaxf(sqrtf(ss), 1e-12f));
    const float* g = (part == 0 ? gq : gk) + h * D + c0;
    T* dst = (part == 0 ? q : k) + dst_off + c0;
#pragma unroll
    for (int w = 0; w < W; ++w) {
      const float4 g0 = *reinterpret_cast<const float4*>(g + 8 * w), g1 = *reinterpret_cast<const float4*>(g + 8 * w + 4);
      const float gg[8] = {g0.x, g0.y, g0.z, g0.w, g1.x, g1.y, g1.z, g1.w};
      Vec8 o;
#pragma unroll
      for (int i = 0; i < 4; ++i)
        o.w[i] = Cvt<T>::pack2(rr[8 * w + 2 * i] * f * gg[2 * i], rr[8 * w + 2 * i + 1] * f * gg[2 * i + 1]);
      *reinterpret_cast<Vec8*>(dst + 8 * w) = o;
    }
  }
}

template <typename T>
static int dispatch_rope(const void* qkv, const float* c, const float* s, const float* gq, const float* gk, void* q,
                         void* k, void* v, int64_t M, int64_t N, int H, int D, int tm, cudaStream_t st) {
  if (M > 0x7fffffff || N > 0x7fffffff) return set_error(HI3D_ERR_INVALID_ARGUMENT, "qkv_rope_rms: too many rows");
  auto threads_for = [&](int G) {
    const int t = ((3 * H * G + 31) / 32) * 32;
    return t > 1024 ? 1024 : t;
  };
#ifndef HI3D_ROPE_VECS
#define HI3D_ROPE_VECS 2
#endif
  constexpr int W = HI3D_ROPE_VECS;  // 16-byte vectors per lane
#define HI3D_ROPE(DD)                                                                                      \
  qkv_rope_rms_kernel<T, DD, W><<<(unsigned)M, threads_for(rope_group(DD, W)), 0, st>>>((const T*)qkv, c, s, gq, gk, (T*)q, (T*)k, \
                                                                         (T*)v, (int)N, H, tm)
  switch (D) {
    case 32: HI3D_ROPE(32); break;
    case 64: HI3D_ROPE(64); break;
    case 96: HI3D_ROPE(96); break;
    case 128: HI3D_ROPE(128); break;
    default:
      return set_error(HI3D_ERR_UNSUPPORTED, "qkv_rope_rms: head_dim %d not supported (32, 64, 96, 128)", D);
  }
#undef HI3D_ROPE
  return check_launch("qkv_rope_rms");
}

// ---------------------------------------------------------------------------
// x <- T(x + T(y * gate)), 8 elements per thread.
// ---------------------------------------------------------------------------
template <typename T>
__global__ void gate_residual_kernel(T* __restrict__ x, const T* __restrict__ y, const T* __restrict__ gate,
                                     int64_t rows, int C, int64_t rows_per_batch, int64_t gate_stride) {
  const int64_t i = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) * 8;
  if (i >= rows * C) return;
  const int64_t row = i / C;
  const int c = (int)(i % C);
  Vec8 xv = *reinterpret_cast<const Vec8*>(x + i);
  Vec8 yv = *reinterpret_cast<const Vec8*>(y + i);
  Vec8 gv;
  if (gate) gv = *reinterpret_cast<const Vec8*>(gate + (row / rows_per_batch) * gate_stride + c);
  Vec8 o;
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const T* xa = reinterpret_cast<const T*>(&xv.w[j]);
    const T* ya = reinterpret_cast<const T*>(&yv.w[j]);
    T res[2];
#pragma unroll
    for (int e = 0; e < 2; ++e) {
      float yy = Cvt<T>::to_f(ya[e]);
      if (gate) yy = Cvt<T>::to_f(round_t<T>(__fmul_rn(yy, Cvt<T>::to_f(reinterpret_cast<const T*>(&gv.w[j])[e]))));
      res[e] = round_t<T>(__fadd_rn(Cvt<T>::to_f(xa[e]), yy));
    }
    o.w[j] = *reinterpret_cast<uint32_t*>(res);
  }
  *reinterpret_cast<Vec8*>(x + i) = o;
}

// gelu_tanh in fp32: 0.5 x (1 + tanh(sqrt(2/pi) (x + 0.044715 x^3))), rounded once.
template <typename T>
__global__ void gelu_kernel(const T* __restrict__ x, T* __restrict__ out, int64_t count) {
  const int64_t i = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) * 8;
  if (i >= count) return;
  Vec8 xv = *reinterpret_cast<const Vec8*>(x + i);
  float f[8];
  unpack8<T>(xv, f);
  Vec8 o;
  const float k0 = 0.7978845608028654f;  // sqrt(2 / pi)
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    float a = f[2 * j], b = f[2 * j + 1];
    float ga = 0.5f * a * (1.0f + tanhf(k0 * (a + 0.044715f * a * a * a)));
    float gb = 0.5f * b * (1.0f + tanhf(k0 * (b + 0.044715f * b * b * b)));
    o.w[j] = Cvt<T>::pack2(ga, gb);
  }
  *reinterpret_cast<Vec8*>(out + i) = o;
}

}  // namespace hi3d

using namespace hi3d;

static int layer_norm_entry(const void* x, void* out, int64_t rows, int64_t channels, float eps, const float* weight,
                            const float* bias, const void* scale, const void* shift, int64_t rows_per_batch,
                            int64_t mod_stride, int act, int dtype, void* stream) {
  if (!x || !out || rows < 0 || channels <= 0)
    return set_error(HI3D_ERR_INVALID_ARGUMENT, "layer_norm_modulate: bad pointers or sizes");
  if (channels % 8 || channels > 4352)
    return set_error(HI3D_ERR_UNSUPPORTED, "layer_norm_modulate: channels must be a multiple of 8 and <= 4352");
  if ((weight == nullptr) != (bias == nullptr) || (scale == nullptr) != (shift == nullptr))
    return set_error(HI3D_ERR_INVALID_ARGUMENT, "layer_norm_modulate: weight/bias and scale/shift come in pairs");
  if (act != 0 && act != 1) return set_error(HI3D_ERR_INVALID_ARGUMENT, "layer_norm: act must be 0 or 1 (SiLU)");
  if (act && (weight != nullptr) == (scale != nullptr))
    return set_error(HI3D_ERR_UNSUPPORTED, "layer_norm: SiLU follows either the affine or the modulation, not both");
  if (!aligned16(x) || !aligned16(out) || (scale && (!aligned16(scale) || !aligned16(shift))))
    return set_error(HI3D_ERR_INVALID_ARGUMENT, "layer_norm_modulate: pointers must be 16-byte aligned");
  if (scale && (rows_per_batch <= 0 || mod_stride % 8))
    return set_error(HI3D_ERR_INVALID_ARGUMENT, "layer_norm_modulate: bad rows_per_batch / mod_stride");
  if (rows == 0) return HI3D_OK;
  if (rows_per_batch <= 0) rows_per_batch = rows;
  cudaStream_t st = as_stream(stream);
  if (dtype == HI3D_F16)
    return dispatch_ln<__half>(x, out, rows, (int)channels, eps, weight, bias, scale, shift, rows_per_batch,
                               mod_stride, act, st);
  if (dtype == HI3D_BF16)
    return dispatch_ln<__nv_bfloat16>(x, out, rows, (int)channels, eps, weight, bias, scale, shift, rows_per_batch,
                                      mod_stride, act, st);
  return set_error(HI3D_ERR_INVALID_ARGUMENT, "layer_norm_modulate: dtype must be f16 or bf16");
}

extern "C" int hi3d_layer_norm_modulate(const void* x, void* out, int64_t rows, int64_t channels, float eps,
                                        const float* weight, const float* bias, const void* scale,
                                        const void* shift, int64_t rows_per_batch, int64_t mod_stride, int dtype,
                                        void* stream) {
  return layer_norm_entry(x, out, rows, channels, eps, weight, bias, scale, shift, rows_per_batch, mod_stride, 0,
                          dtype, stream);
}

extern "C" int hi3d_layer_norm_act(const void* x, void* out, int64_t rows, int64_t channels, float eps,
                                   const float* weight, const float* bias, const void* scale, const void* shift,
                                   int64_t rows_per_batch, int64_t mod_stride, int act, int dtype, void* stream) {
  return layer_norm_entry(x, out, rows, channels, eps, weight, bias, scale, shift, rows_per_batch, mod_stride,
                          act, dtype, stream);
}

extern "C" int hi3d_qkv_rope_rms(const void* qkv, const float* cos, const float* sin, const float* gamma_q,
                                 const float* gamma_k, void* q, void* k, void* v, int64_t batch, int64_t n, int heads,
                                 int head_dim, int out_layout, int dtype, void* stream) {
  if (!qkv || !cos || !sin || !gamma_q || !gamma_k || !q || !k || !v || batch < 0 || n < 0 || heads <= 0)
    return set_error(HI3D_ERR_INVALID_ARGUMENT, "qkv_rope_rms: bad pointers or sizes");
  if (head_dim % 2) return set_error(HI3D_ERR_INVALID_ARGUMENT, "qkv_rope_rms: head_dim must be even");
  if (out_layout != 0 && out_layout != 1)
    return set_error(HI3D_ERR_INVALID_ARGUMENT, "qkv_rope_rms: out_layout must be 0 ([B,H,N,D]) or 1 ([B,N,H,D])");
  if (!aligned16(qkv) || !aligned16(q) || !aligned16(k) || !aligned16(v))
    return set_error(HI3D_ERR_INVALID_ARGUMENT, "qkv_rope_rms: pointers must be 16-byte aligned");
  const int64_t M = batch * n;
  if (M == 0) return HI3D_OK;
  cudaStream_t st = as_stream(stream);
  if (dtype == HI3D_F16)
    return dispatch_rope<__half>(qkv, cos, sin, gamma_q, gamma_k, q, k, v, M, n, heads, head_dim, out_layout, st);
  if (dtype == HI3D_BF16)
    return dispatch_rope<__nv_bfloat16>(qkv, cos, sin, gamma_q, gamma_k, q, k, v, M, n, heads, head_dim, out_layout,
                                        st);
  return set_error(HI3D_ERR_INVALID_ARGUMENT, "qkv_rope_rms: dtype must be f16 or bf16");
}

extern "C" int hi3d_gate_residual(void* x, const void* y, const void* gate, int64_t rows, int64_t channels,
                                  int64_t rows_per_batch, int64_t gate_stride, int dtype, void* stream) {
  if (!x || !y || rows < 0 || channels <= 0 || channels % 8)
    return set_error(HI3D_ERR_INVALID_ARGUMENT, "gate_residual: bad pointers or sizes (channels % 8 == 0)");
  if (!aligned16(x) || !aligned16(y) || (gate && !aligned16(gate)) || gate_stride % 8)
    return set_error(HI3D_ERR_INVALID_ARGUMENT, "gate_residual: pointers must be 16-byte aligned");
  if (rows == 0) return HI3D_OK;
  if (rows_per_batch <= 0) rows_per_batch = rows;
  const int64_t threads = rows * channels / 8;
  dim3 grid((unsigned)((threads + 255) / 256));
  cudaStream_t st = as_stream(stream);
  if (dtype == HI3D_F16)
    gate_residual_kernel<__half><<<grid, 256, 0, st>>>((__half*)x, (const __half*)y, (const __half*)gate, rows,
                                                       (int)channels, rows_per_batch, gate_stride);
  else if (dtype == HI3D_BF16)
    gate_residual_kernel<__nv_bfloat16><<<grid, 256, 0, st>>>((__nv_bfloat16*)x, (const __nv_bfloat16*)y,
                                                              (const __nv_bfloat16*)gate, rows, (int)channels,
                                                              rows_per_batch, gate_stride);
  else
    return set_error(HI3D_ERR_INVALID_ARGUMENT, "gate_residual: dtype must be f16 or bf16");
  return check_launch("gate_residual");
}

extern "C" int hi3d_gelu_tanh(const void* x, void* out, int64_t count, int dtype, void* stream) {
  if (!x || !out || count < 0 || count % 8)
    return set_error(HI3D_ERR_INVALID_ARGUMENT, "gelu_tanh: bad pointers or count (multiple of 8)");
  if (!aligned16(x) || !aligned16(out))
    return set_error(HI3D_ERR_INVALID_ARGUMENT, "gelu_tanh: pointers must be 16-byte aligned");
  if (count == 0) return HI3D_OK;
  dim3 grid((unsigned)((count / 8 + 255) / 256));
  cudaStream_t st = as_stream(stream);
  if (dtype == HI3D_F16)
    gelu_kernel<__half><<<grid, 256, 0, st>>>((const __half*)x, (__half*)out, count);
  else if (dtype == HI3D_BF16)
    gelu_kernel<__nv_bfloat16><<<grid, 256, 0, st>>>((const __nv_bfloat16*)x, (__nv_bfloat16*)out, count);
  else
    return set_error(HI3D_ERR_INVALID_ARGUMENT, "gelu_tanh: dtype must be f16 or bf16");
  return check_launch("gelu_tanh");
}

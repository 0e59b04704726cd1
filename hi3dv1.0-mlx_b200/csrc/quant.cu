// Dynamic per-row int8 quantisation of activations with the signed 64-point
// Hadamard rotation of the reference W8A8 path (w8a8.py:25-58, :95-102).
//
// Per row and per 64-element block: y = H64(x * sign) / 8 with H64 the
// natural-order (Sylvester) Walsh-Hadamard transform, evaluated as six
// butterfly stages over the element index bits 0..5 in that order; stage b
// maps (u at bit clear, v at bit set) to (u + v, u - v), and the last stage
// also multiplies by 0.125.  This is the reference's operation order for every
// element (its five xor-shuffle stages over lane bits 0-4, then the (c, c+32)
// pair), so the fp32 values, and hence the int8 codes, are reproduced exactly.
// Then s = max(max|y|, 1e-8) / 127 and q = clamp(rint(y / s), -127, 127)
// (round half to even), all in IEEE fp32.
//
// Layout: one to eight warps per row (by width); each lane owns 8 consecutive
// elements of a 256-element chunk (16-byte loads, each warp instruction one
// contiguous 512-byte span), so bits 0-2 of the element index are in-register
// stages and bits 3-5 are xor-shuffles across lanes 1, 2 and 4 apart.  Warps of
// one row combine their maxima through shared memory.
#include "abi.h"
#include "common.cuh"

namespace hi3d {

template <typename T>
__device__ __forceinline__ void load8(const T* p, float (&f)[8]) {
  const uint4 raw = *reinterpret_cast<const uint4*>(p);
  const T* h = reinterpret_cast<const T*>(&raw);
#pragma unroll
  for (int i = 0; i < 8; ++i) f[i] = Cvt<T>::to_f(h[i]);
}

__device__ __forceinline__ uint64_t f2_sub(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("sub.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}

// Signed H64 of one lane's 8 elements v (element index bits 0-2), the lane's partners 1, 2
// and 4 lanes apart holding index bits 3-5 (g = lane % 8): the same operations in the same
// order as above, with the first two in-register stages on packed pairs (v[k], v[k + 4]),
// and each cross-lane stage as one exact fma(v, +-1, other) (x - v equals x + (-1) v).
__device__ __forceinline__ void h64_rotate(float (&v)[8], const float* __restrict__ sign, int g) {
  const float4 s0 = *reinterpret_cast<const float4*>(sign);
  const float4 s1 = *reinterpret_cast<const float4*>(sign + 4);
  uint64_t P[4];
  P[0] = f2_mul(f2_pack(v[0], v[4]), f2_pack(s0.x, s1.x));
  P[1] = f2_mul(f2_pack(v[1], v[5]), f2_pack(s0.y, s1.y));
  P[2] = f2_mul(f2_pack(v[2], v[6]), f2_pack(s0.z, s1.z));
  P[3] = f2_mul(f2_pack(v[3], v[7]), f2_pack(s0.w, s1.w));
  // element bit 0: (0,1), (2,3), (4,5), (6,7)
  uint64_t a = f2_add(P[0], P[1]), b = f2_sub(P[0], P[1]), c = f2_add(P[2], P[3]), d = f2_sub(P[2], P[3]);
  // element bit 1: (0,2), (1,3), (4,6), (5,7)
  P[0] = f2_add(a, c);
  P[2] = f2_sub(a, c);
  P[1] = f2_add(b, d);
  P[3] = f2_sub(b, d);
  // element bit 2: (k, k + 4) inside each pair
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    float lo, hi;
    f2_unpack(P[k], lo, hi);
    v[k] = __fadd_rn(lo, hi);
    v[k + 4] = __fsub_rn(lo, hi);
  }
  // element bits 3, 4, 5 across lanes; the last stage scales by 1/8 (exact)
  const float m1 = (g & 1) ? -1.0f : 1.0f, m2 = (g & 2) ? -1.0f : 1.0f, m4 = (g & 4) ? -1.0f : 1.0f;
#pragma unroll
  for (int i = 0; i < 8; ++i) v[i] = __fmaf_rn(v[i], m1, __shfl_xor_sync(0xffffffffu, v[i], 1));
#pragma unroll
  for (int i = 0; i < 8; ++i) v[i] = __fmaf_rn(v[i], m2, __shfl_xor_sync(0xffffffffu, v[i], 2));
#pragma unroll
  for (int i = 0; i < 8; ++i) v[i] = __fmul_rn(__fmaf_rn(v[i], m4, __shfl_xor_sync(0xffffffffu, v[i], 4)), 0.125f);
}

// rint(y / s) with y / s the correctly rounded IEEE quotient, clamped to
// [-127, 127] (|y / s| <= 127 for finite rows; NaN gives -127).
// z = y * rn(1 / s) is within |y / s| * 2^-23 <= 1.6e-5 of the true quotient;
// when z is farther than 3e-5 from a half-integer, the true quotient and its
// rounded value lie on the same side of it and rint(z) is the answer.  The few
// quotients closer to a rounding tie take the exact division.
// Codes of 8 values, packed little-endian into two words (a saturating conversion
// after the clamp at -127).
__device__ __forceinline__ uint2 quant_pack8(const float (&y)[8], float s, float inv) {
  int c[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const float z = __fmul_rn(y[i], inv);
    float r = rintf(z);
    if (fabsf(z - r) >= 0.5f - 3e-5f) r = rintf(__fdiv_rn(y[i], s));
    int q;
    asm("cvt.rni.sat.s8.f32 %0, %1;" : "=r"(q) : "f"(fmaxf(r, -127.0f)));
    c[i] = q;
  }
  const uint32_t w0 = __byte_perm(__byte_perm(c[0], c[1], 0x0040), __byte_perm(c[2], c[3], 0x0040), 0x5410);
  const uint32_t w1 = __byte_perm(__byte_perm(c[4], c[5], 0x0040), __byte_perm(c[6], c[7], 0x0040), 0x5410);
  return make_uint2(w0, w1);
}

// Codes of 8 values (4 f32x2 pairs), for the tiled and the LayerNorm-fused kernels: the quotient z = y * inv is rounded
// with the 1.5 * 2^23 shift, (z + 2^23 * 1.5) - 2^23 * 1.5, which is round-half-even to an
// integer for |z| < 2^22 (here |z| <= 127 * (1 + 3 * 2^-24)), on the FMA pipe and in pairs; the
// two's-complement low byte of the shifted value's bits is then the code.  As in quant_pack8,
// a quotient within 3e-5 of a rounding tie (or not finite) falls back to the exact division;
// any such value sends all 8 through quant_pack8, so the codes are those of quant_pack8.
__device__ __forceinline__ uint2 quant_pack8_pairs(const uint64_t (&Y)[4], float s, float inv) {
  const uint64_t INV = f2_splat(inv), SHIFT = f2_splat(12582912.0f), UNSHIFT = f2_splat(-12582912.0f);
  uint32_t tb[8];
  bool near_tie = false;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const uint64_t z = f2_mul(Y[i], INV);
    const uint64_t t = f2_add(z, SHIFT);
    const uint64_t d = f2_sub(z, f2_add(t, UNSHIFT));
    float d0, d1, t0, t1;
    f2_unpack(d, d0, d1);
    f2_unpack(t, t0, t1);
    near_tie |= !(fabsf(d0) < 0.5f - 3e-5f) || !(fabsf(d1) < 0.5f - 3e-5f);
    tb[2 * i] = __float_as_uint(t0);
    tb[2 * i + 1] = __float_as_uint(t1);
  }
  if (near_tie) {
    float y[8];
#pragma unroll
    for (int i = 0; i < 4; ++i) f2_unpack(Y[i], y[2 * i], y[2 * i + 1]);
    return quant_pack8(y, s, inv);
  }
  const uint32_t w0 = __byte_perm(__byte_perm(tb[0], tb[1], 0x0040), __byte_perm(tb[2], tb[3], 0x0040), 0x5410);
  const uint32_t w1 = __byte_perm(__byte_perm(tb[4], tb[5], 0x0040), __byte_perm(tb[6], tb[7], 0x0040), 0x5410);
  return make_uint2(w0, w1);
}

// One row per WPR warps of a 256-thread block; warp `part` of a row handles the
// 256-element chunks part, part + WPR, ... (IPW of them).
template <typename T, int IPW, int WPR, bool ROTATE>
__global__ void __launch_bounds__(256) quant_h64_kernel(const T* __restrict__ x, const float* __restrict__ sign,
                                                        int8_t* __restrict__ q, float* __restrict__ scale, int64_t rows,
                                                        int K) {
  constexpr int RPB = 8 / WPR;  // rows per block
  __shared__ float red[8];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int part = warp % WPR;
  // grid-stride over groups of RPB rows (the grid is sized to whole waves); the trip
  // count is uniform across the block, so every thread reaches the block barriers
  for (int64_t g = blockIdx.x; g * RPB < rows; g += gridDim.x) {
    const int64_t row = g * RPB + warp / WPR;
    const bool row_ok = row < rows;
    const T* xr = x + (row_ok ? row : 0) * K;
    float y[IPW][8];
    float amax = 0.f;
#pragma unroll
    for (int j = 0; j < IPW; ++j) {
      const int base = (part + j * WPR) * 256 + lane * 8;
      const bool active = row_ok && base < K;
      float v[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
      if (active) load8<T>(xr + base, v);
      if (ROTATE) {
        h64_rotate(v, sign + (active ? base : 0), lane & 7);
      }
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        y[j][i] = v[i];
        if (active) amax = fmaxf(amax, fabsf(v[i]));
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
    if (WPR > 1) {
      if (lane == 0) red[warp] = amax;
      __syncthreads();
      const int first = warp - part;
#pragma unroll
      for (int w = 0; w < WPR; ++w) amax = fmaxf(amax, red[first + w]);
    }
    if (row_ok) {
      const float s = __fdiv_rn(fmaxf(amax, 1e-8f), 127.0f);
      const float inv = __frcp_rn(s);
      if (lane == 0 && part == 0) scale[row] = s;
      int8_t* qr = q + row * K;
#pragma unroll
      for (int j = 0; j < IPW; ++j) {
        const int base = (part + j * WPR) * 256 + lane * 8;
        if (base >= K) continue;
        *reinterpret_cast<uint2*>(qr + base) = quant_pack8(y[j], s, inv);
      }
    }
    if (WPR > 1) __syncthreads();  // red[] is rewritten by the next group
  }
}

// ---------------------------------------------------------------------------
// LayerNorm-modulate fused with the signed-H64 quantiser: the input of the W8A8
// projections that follow a norm (QKV, cross-attention Q, MLP in).  Per row, one warp:
// the LayerNorm32 + affine / modulation of ln_mod_kernel (rowwise.cu; kernels.py:162-201)
// to the rounded 16-bit h, then exactly the quantiser above on h: sign, H64 (three
// in-register butterfly stages, three across lanes 1, 2 and 4 apart, / 8), row maximum,
// codes.  The 16-bit h is never written: bit-identical to quantize(layer_norm_modulate(x)).
// Lane l of the warp holds channels c * 256 + 8 l .. + 7 of chunk c (channels % 64 == 0).
// ---------------------------------------------------------------------------
// The LayerNorm32 (+ affine) (+ modulation) of one row by one warp, as ln_mod_kernel computes
// it (rowwise.cu; kernels.py:162-201): lane l gets the rounded 16-bit h of channels
// c * 256 + 8 l .. + 7 as four packed words per chunk c (zero past C).  `wb`: the fp32 affine
// parameters in shared memory in lane order (float4 (2c + h) * 32 + l), when AFFINE.
template <typename T, int NCH, bool AFFINE, bool MODULATE>
__device__ __forceinline__ void ln_row_words(const T* __restrict__ xr, int64_t row, int C, float eps,
                                             const float* wb, const T* __restrict__ scale,
                                             const T* __restrict__ shift, int64_t rows_per_batch,
                                             int64_t mod_stride, int lane, uint4 (&hw)[NCH]) {
  uint4 raw[NCH];
#pragma unroll
  for (int c = 0; c < NCH; ++c) {
    raw[c] = make_uint4(0, 0, 0, 0);
    if (c * 256 + lane * 8 < C) raw[c] = *reinterpret_cast<const uint4*>(xr + c * 256 + lane * 8);
  }
  uint64_t d[NCH][4];
  uint64_t s2 = 0;
#pragma unroll
  for (int c = 0; c < NCH; ++c) {
    const uint32_t* rw = reinterpret_cast<const uint32_t*>(&raw[c]);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      d[c][i] = Cvt<T>::to_f2(rw[i]);
      s2 = f2_add(s2, d[c][i]);
    }
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
        d[c][i] = f2_add(d[c][i], neg_mean);
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
    hw[c] = make_uint4(0, 0, 0, 0);
    if (base >= C) continue;
    uint4 sc = make_uint4(0, 0, 0, 0), sh = make_uint4(0, 0, 0, 0);
    if (MODULATE) {
      sc = *reinterpret_cast<const uint4*>(scale + mb + base);
      sh = *reinterpret_cast<const uint4*>(shift + mb + base);
    }
    const uint32_t* scw = reinterpret_cast<const uint32_t*>(&sc);
    const uint32_t* shw = reinterpret_cast<const uint32_t*>(&sh);
    uint64_t wv[4], bv[4];
    if (AFFINE) {
      const float4* w4 = reinterpret_cast<const float4*>(wb) + c * 64 + lane;
      const float4* b4 = reinterpret_cast<const float4*>(wb + NCH * 256) + c * 64 + lane;
      const float4 w0 = w4[0], w1 = w4[32], b0 = b4[0], b1 = b4[32];
      wv[0] = f2_pack(w0.x, w0.y), wv[1] = f2_pack(w0.z, w0.w), wv[2] = f2_pack(w1.x, w1.y),
      wv[3] = f2_pack(w1.z, w1.w);
      bv[0] = f2_pack(b0.x, b0.y), bv[1] = f2_pack(b0.z, b0.w), bv[2] = f2_pack(b1.x, b1.y),
      bv[3] = f2_pack(b1.z, b1.w);
    }
    uint32_t hv[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      uint64_t yy = f2_mul(d[c][i], inv2);
      if (AFFINE) yy = f2_add(f2_mul(yy, wv[i]), bv[i]);
      uint32_t h = Cvt<T>::from_f2(yy);
      if (MODULATE) h = Cvt<T>::add2(Cvt<T>::mul2(h, scw[i]), shw[i]);
      hv[i] = h;
    }
    hw[c] = make_uint4(hv[0], hv[1], hv[2], hv[3]);
  }
}

constexpr int kLnqRowsPerBlock = 4;

template <typename T, int NCH, bool AFFINE, bool MODULATE>
__global__ void __launch_bounds__(kLnqRowsPerBlock * 32)
    ln_quant_kernel(const T* __restrict__ x, int64_t rows, int C, float eps, const float* __restrict__ weight,
                    const float* __restrict__ bias, const T* __restrict__ scale, const T* __restrict__ shift,
                    int64_t rows_per_batch, int64_t mod_stride, const float* __restrict__ sign,
                    int8_t* __restrict__ q, float* __restrict__ qscale) {
  const int lane = threadIdx.x & 31;
  const int g = lane & 7;
  // fp32 affine parameters staged once per block in shared memory, in the lane order of
  // ln_mod_kernel (channel c*256 + 8 l + 4 h + k at float4 (2c + h) * 32 + l): each warp's
  // 16-byte loads read 512 contiguous bytes
  extern __shared__ float lnq_wb[];
  if constexpr (AFFINE) {
    for (int i = threadIdx.x; i < NCH * 256; i += blockDim.x) {
      const int c = i >> 8, l = (i >> 3) & 31, h = (i >> 2) & 1, k = i & 3;
      const int pos = (((c * 2 + h) * 32 + l) << 2) + k;
      lnq_wb[pos] = i < C ? weight[i] : 0.f;
      lnq_wb[NCH * 256 + pos] = i < C ? bias[i] : 0.f;
    }
    __syncthreads();
  }
  for (int64_t row = (int64_t)blockIdx.x * kLnqRowsPerBlock + (threadIdx.x >> 5); row < rows;
       row += (int64_t)gridDim.x * kLnqRowsPerBlock) {
    uint4 hw[NCH];
    ln_row_words<T, NCH, AFFINE, MODULATE>(x + row * C, row, C, eps, lnq_wb, scale, shift, rows_per_batch,
                                           mod_stride, lane, hw);
    // ---- the rotation per 64-block of h
    float y[NCH][8];
    float amax = 0.f;
#pragma unroll
    for (int c = 0; c < NCH; ++c) {
      const int base = c * 256 + lane * 8;
      const bool active = base < C;
      float v[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
      if (active) {
        const uint32_t* hv = reinterpret_cast<const uint32_t*>(&hw[c]);
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const T* hp = reinterpret_cast<const T*>(&hv[i]);
          v[2 * i] = Cvt<T>::to_f(hp[0]);
          v[2 * i + 1] = Cvt<T>::to_f(hp[1]);
        }
      }
      h64_rotate(v, sign + (active ? base : 0), g);
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        y[c][i] = v[i];
        if (active) amax = fmaxf(amax, fabsf(v[i]));
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
    const float sc = __fdiv_rn(fmaxf(amax, 1e-8f), 127.0f);
    const float inv = __frcp_rn(sc);
    if (lane == 0) qscale[row] = sc;
    int8_t* qr = q + row * C;
#pragma unroll
    for (int c = 0; c < NCH; ++c) {
      const int base = c * 256 + lane * 8;
      if (base >= C) continue;
      const uint64_t yp[4] = {f2_pack(y[c][0], y[c][1]), f2_pack(y[c][2], y[c][3]), f2_pack(y[c][4], y[c][5]),
                              f2_pack(y[c][6], y[c][7])};
      *reinterpret_cast<uint2*>(qr + base) = quant_pack8_pairs(yp, sc, inv);
    }
  }
}

template <typename T, int NCH>
static void launch_lnq(const void* x, int64_t rows, int C, float eps, const float* w, const float* b, const void* sc,
                       const void* sh, int64_t rpb, int64_t ms, const float* sign, int8_t* q, float* qs,
                       cudaStream_t st) {
  const int64_t blocks = (rows + kLnqRowsPerBlock - 1) / kLnqRowsPerBlock,
                cap = (int64_t)sm_count() * (2048 / (kLnqRowsPerBlock * 32));
  const unsigned grid = (unsigned)(blocks < cap ? blocks : cap);
  const T* xt = (const T*)x;
  const T* s = (const T*)sc;
  const T* t = (const T*)sh;
  const size_t wb = (size_t)2 * NCH * 256 * sizeof(float);  // affine parameters in shared memory
  if (w && sc)
    ln_quant_kernel<T, NCH, true, true><<<grid, kLnqRowsPerBlock * 32, wb, st>>>(xt, rows, C, eps, w, b, s, t, rpb,
                                                                                ms, sign, q, qs);
  else if (w)
    ln_quant_kernel<T, NCH, true, false><<<grid, kLnqRowsPerBlock * 32, wb, st>>>(xt, rows, C, eps, w, b, s, t, rpb,
                                                                                 ms, sign, q, qs);
  else if (sc)
    ln_quant_kernel<T, NCH, false, true><<<grid, kLnqRowsPerBlock * 32, 0, st>>>(xt, rows, C, eps, w, b, s, t, rpb,
                                                                                ms, sign, q, qs);
  else
    ln_quant_kernel<T, NCH, false, false><<<grid, kLnqRowsPerBlock * 32, 0, st>>>(xt, rows, C, eps, w, b, s, t, rpb,
                                                                                 ms, sign, q, qs);
}

template <typename T>
static int dispatch_lnq(const void* x, int64_t rows, int C, float eps, const float* w, const float* b, const void* sc,
                        const void* sh, int64_t rpb, int64_t ms, const float* sign, int8_t* q, float* qs,
                        cudaStream_t st) {
  switch ((C + 255) / 256) {
#define HI3D_LNQ_CASE(n) \
  case n:                \
    launch_lnq<T, n>(x, rows, C, eps, w, b, sc, sh, rpb, ms, sign, q, qs, st); break;
    HI3D_LNQ_CASE(1)
    HI3D_LNQ_CASE(2)
    HI3D_LNQ_CASE(3)
    HI3D_LNQ_CASE(4)
    HI3D_LNQ_CASE(5)
    HI3D_LNQ_CASE(6)
    HI3D_LNQ_CASE(7)
    HI3D_LNQ_CASE(8)
    HI3D_LNQ_CASE(9)
    HI3D_LNQ_CASE(10)
    HI3D_LNQ_CASE(11)
    HI3D_LNQ_CASE(12)
    HI3D_LNQ_CASE(13)
    HI3D_LNQ_CASE(14)
    HI3D_LNQ_CASE(15)
    HI3D_LNQ_CASE(16)
#undef HI3D_LNQ_CASE
    default:
      return set_error(HI3D_ERR_UNSUPPORTED, "layer_norm_quantize: channels %d not supported (<= 4096)", C);
  }
  return check_launch("layer_norm_quantize");
}

template <typename T, int IPW, int WPR, bool ROTATE>
static void launch_q(const void* x, const float* sign, int8_t* q, float* scale, int64_t rows, int K, cudaStream_t st) {
  constexpr int RPB = 8 / WPR;
  // at most 8 resident 256-thread blocks per SM: a grid of whole waves
  const int64_t blocks = (rows + RPB - 1) / RPB, cap = (int64_t)sm_count() * 8;
  quant_h64_kernel<T, IPW, WPR, ROTATE>
      <<<(unsigned)(blocks < cap ? blocks : cap), 256, 0, st>>>((const T*)x, sign, q, scale, rows, K);
}

template <typename T, int WPR, bool ROTATE>
static void launch_w(int ipw, const void* x, const float* sign, int8_t* q, float* scale, int64_t rows, int K,
                     cudaStream_t st) {
  switch (ipw) {
    case 1: launch_q<T, 1, WPR, ROTATE>(x, sign, q, scale, rows, K, st); break;
    case 2: launch_q<T, 2, WPR, ROTATE>(x, sign, q, scale, rows, K, st); break;
    case 3: launch_q<T, 3, WPR, ROTATE>(x, sign, q, scale, rows, K, st); break;
    case 4: launch_q<T, 4, WPR, ROTATE>(x, sign, q, scale, rows, K, st); break;
    default: launch_q<T, 5, WPR, ROTATE>(x, sign, q, scale, rows, K, st); break;
  }
}

// ---------------------------------------------------------------------------
// The rotating quantiser with one thread per 64-element block.
//
// A tile is R whole rows, viewed as R * K/64 blocks of 128 bytes (at most 256: one
// per thread).  One TMA load brings the tile into shared memory with the 128-byte
// swizzle (16-byte chunk j of block b lands at chunk j ^ (b % 8)), so thread b
// reads its own block with eight conflict-free 16-byte loads; two tile buffers
// alternate, the next-but-one tile loading while the current one is computed.
// The thread then runs the whole signed H64 in registers: the multiply, the six
// butterfly stages in index-bit order 0..5 (stage 0 on scalars, stages 1-5 on
// f32x2 pairs), the final * 0.125 - the same IEEE operations on the same values
// as the warp-shuffle kernel above, so the codes are identical - with no
// cross-lane traffic.  Row maxima meet in shared memory (atomicMax on the
// non-negative floats' bits, NaN excluded as fmaxf excludes it), three slots
// rotating over the tiles so that one block barrier per tile suffices.
// The multipliers sit in shared memory transposed ([K/256][K/64] float4), so a
// warp's threads, which hold consecutive blocks of a row, read consecutive float4.
// ---------------------------------------------------------------------------
// The signed H64 of one 64-element block held by one thread: block `b` of a swizzled shared
// tile (16-byte chunk j of block b at chunk j ^ (b % 8) of its 128-byte row), times the
// multipliers (`m4[e4 * stride]`, e4 = element / 4), the six butterfly stages in index-bit
// order 0..5 (stage 0 on scalars, stages 1-5 on f32x2 pairs), * 0.125: the IEEE operations
// of h64_rotate on the same values.  Leaves (y[2k], y[2k+1]) in P[k]; returns max |y|.
template <typename T>
__device__ __forceinline__ float h64_block(const uint8_t* tile, int b, const float4* m4, int stride,
                                           uint64_t (&P)[32]) {
  const uint8_t* src = tile + b * 128;
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    const uint4 raw = *reinterpret_cast<const uint4*>(src + ((j ^ (b & 7)) << 4));
    P[4 * j] = Cvt<T>::to_f2(raw.x);
    P[4 * j + 1] = Cvt<T>::to_f2(raw.y);
    P[4 * j + 2] = Cvt<T>::to_f2(raw.z);
    P[4 * j + 3] = Cvt<T>::to_f2(raw.w);
  }
  // y = x * multiplier
#pragma unroll
  for (int e4 = 0; e4 < 16; ++e4) {
    const float4 m = m4[e4 * stride];
    P[2 * e4] = f2_mul(P[2 * e4], f2_pack(m.x, m.y));
    P[2 * e4 + 1] = f2_mul(P[2 * e4 + 1], f2_pack(m.z, m.w));
  }
  // stage 0 (index bit 0): the two halves of each pair
#pragma unroll
  for (int k = 0; k < 32; ++k) {
    float a, c;
    f2_unpack(P[k], a, c);
    P[k] = f2_pack(__fadd_rn(a, c), __fsub_rn(a, c));
  }
  // stages 1..5 (index bits 1..5): pairs k and k + 2^(bit-1)
#pragma unroll
  for (int h = 1; h < 32; h <<= 1) {
#pragma unroll
    for (int k = 0; k < 32; ++k) {
      if (k & h) continue;
      const uint64_t u = P[k], v = P[k + h];
      P[k] = f2_add(u, v);
      P[k + h] = f2_sub(u, v);
    }
  }
  float amax = 0.f;
#pragma unroll
  for (int k = 0; k < 32; ++k) {
    P[k] = f2_mul(P[k], f2_splat(0.125f));
    float lo, hi;
    f2_unpack(P[k], lo, hi);
    amax = fmaxf(amax, fmaxf(fabsf(lo), fabsf(hi)));
  }
  return amax;
}

// Codes of one block (P from h64_block) into 64 bytes at dst (16-byte aligned).
__device__ __forceinline__ void store_block_codes(const uint64_t (&P)[32], float sc, float inv, int8_t* dst) {
  uint4* d4 = reinterpret_cast<uint4*>(dst);
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const uint64_t(&lo)[4] = *reinterpret_cast<const uint64_t(*)[4]>(&P[8 * j]);
    const uint64_t(&hi)[4] = *reinterpret_cast<const uint64_t(*)[4]>(&P[8 * j + 4]);
    const uint2 a = quant_pack8_pairs(lo, sc, inv), b = quant_pack8_pairs(hi, sc, inv);
    d4[j] = make_uint4(a.x, a.y, b.x, b.y);
  }
}

constexpr int kQtThreads = 256;
constexpr int kQtMaxRows = 256;  // rows per tile (a tile of 64-wide rows)
constexpr int kSiteQuantTile = 960;

template <typename T>
__global__ void __launch_bounds__(kQtThreads, 2)
    quant_h64_tile_kernel(const __grid_constant__ CUtensorMap tm, const float* __restrict__ mult,
                          int8_t* __restrict__ q, float* __restrict__ scale, int64_t rows, int K, int R,
                          int64_t ntiles) {
  extern __shared__ uint8_t qt_smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(qt_smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* stage0 = smem;  // two tiles of 256 x 128 bytes
  float* ms = reinterpret_cast<float*>(smem + 2 * kQtThreads * 128);
  __shared__ __align__(8) uint64_t full[2];
  __shared__ uint32_t rmax[3][kQtMaxRows];
  __shared__ int abort_flag;
  const int t = threadIdx.x;
  const int bpr = K >> 6, tb = R * bpr;
  const int bc = t % bpr, rl = t / bpr;  // this thread's block column and row within the tile
  if (t == 0) {
    mbar_init(&full[0], 1);
    mbar_init(&full[1], 1);
    abort_flag = 0;
    fence_barrier_init();
  }
  for (int i = t; i < K; i += kQtThreads) {
    const int e = i & 63;
    ms[(((e >> 2) * bpr + (i >> 6)) << 2) + (e & 3)] = mult[i];
  }
  for (int i = t; i < 3 * kQtMaxRows; i += kQtThreads) (&rmax[0][0])[i] = 0u;
  __syncthreads();
  const int64_t step = gridDim.x;
  const uint32_t tile_bytes = (uint32_t)tb * 128u;
  if (t == 0) {
    tma_prefetch_desc(&tm);
    for (int s = 0; s < 2; ++s) {
      const int64_t tile = blockIdx.x + s * step;
      if (tile < ntiles) {
        mbar_arrive_expect_tx(&full[s], tile_bytes);
        tma_load_2d(stage0 + s * kQtThreads * 128, &tm, &full[s], 0, (int)(tile * tb));
      }
    }
  }
  const float4* ms4 = reinterpret_cast<const float4*>(ms);
  int it = 0;
  for (int64_t tile = blockIdx.x; tile < ntiles; tile += step, ++it) {
    const int s = it & 1;
    const bool ok = mbar_wait(&full[s], (it >> 1) & 1, &abort_flag, kSiteQuantTile);
    if (__syncthreads_or(!ok)) break;  // every thread leaves together on a time-out
    const int64_t row = tile * R + rl;
    const bool active = t < tb && row < rows;
    uint64_t P[32];  // (y[2k], y[2k+1])
    const float amax = h64_block<T>(stage0 + s * kQtThreads * 128, t, ms4 + bc, bpr, P);
    if (active) atomicMax(&rmax[it % 3][rl], __float_as_uint(amax));
    if (t < R) rmax[(it + 1) % 3][t] = 0u;  // the next tile's slot (its readers finished two tiles ago)
    __syncthreads();  // the tile buffer is read and the row maxima are complete
    if (t == 0 && tile + 2 * step < ntiles) {
      // generic-proxy reads of the buffer above, then the TMA (async proxy) refills it
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      mbar_arrive_expect_tx(&full[s], tile_bytes);
      tma_load_2d(stage0 + s * kQtThreads * 128, &tm, &full[s], 0, (int)((tile + 2 * step) * tb));
    }
    if (active) {
      const float sc = __fdiv_rn(fmaxf(__uint_as_float(rmax[it % 3][rl]), 1e-8f), 127.0f);
      const float inv = __frcp_rn(sc);
      if (bc == 0) scale[row] = sc;
      store_block_codes(P, sc, inv, q + (tile * tb + t) * 64);
    }
  }
}

template <typename T>
static int launch_quant_tiles(const void* x, const float* sign, int8_t* q, float* scale, int64_t rows, int K,
                              cudaStream_t st) {
  const int bpr = K / 64, R = kQtThreads / bpr;
  const int64_t nblocks = rows * bpr, ntiles = (rows + R - 1) / R;
  CUtensorMap tm;
  const uint64_t dims[2] = {64, (uint64_t)nblocks}, strides[1] = {128};
  const uint32_t box[2] = {64, (uint32_t)(R * bpr)};
  int rc = encode_tmap(&tm, std::is_same<T, __half>::value ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16
                                                           : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16,
                       2, x, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B);
  if (rc) return rc;
  const size_t smem = 1024 + 2 * kQtThreads * 128 + (size_t)K * sizeof(float);
  auto kern = quant_h64_tile_kernel<T>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return set_error(HI3D_ERR_CUDA, "quantize_act_i8: smem attribute: %s", cudaGetErrorString(e));
  const int64_t cap = 2 * (int64_t)sm_count();  // two resident CTAs per SM
  const int grid = (int)(ntiles < cap ? ntiles : cap);
  kern<<<grid, kQtThreads, smem, st>>>(tm, sign, q, scale, rows, K, R, ntiles);
  return check_launch("quantize_act_i8");
}

// ---------------------------------------------------------------------------
// LayerNorm(-modulate) + quantiser with the rotation of the tiled kernel, for rows of at most
// 1024 channels.  A tile is R = 256 / (C / 64) whole rows.  Phase 1: each warp computes the
// LayerNorm of its rows (ln_row_words: the rounded 16-bit h of ln_mod_kernel) and writes h
// into a swizzled shared tile of 64-element blocks.  Phase 2: one thread per block runs the
// signed H64 in registers (h64_block), row maxima meet in shared memory, codes and scales
// follow.  Same h, same rotation arithmetic, same rounding as quantize(layer_norm(x)).
// ---------------------------------------------------------------------------
template <typename T, int NCH, bool AFFINE, bool MODULATE>
__global__ void __launch_bounds__(kQtThreads, 2)
    ln_quant_tile_kernel(const T* __restrict__ x, int64_t rows, int C, float eps, const float* __restrict__ weight,
                         const float* __restrict__ bias, const T* __restrict__ scale, const T* __restrict__ shift,
                         int64_t rows_per_batch, int64_t mod_stride, const float* __restrict__ sign,
                         int8_t* __restrict__ q, float* __restrict__ qscale, int R, int64_t ntiles) {
  extern __shared__ __align__(16) uint8_t lqt_smem[];
  uint8_t* hs = lqt_smem;                                             // [256 blocks][128 B], swizzled
  float* ms = reinterpret_cast<float*>(lqt_smem + kQtThreads * 128);  // multipliers, transposed
  float* wb = ms + NCH * 256;                                         // affine parameters, lane order
  __shared__ uint32_t rmax[2][kQtMaxRows];
  const int t = threadIdx.x, lane = t & 31, warp = t >> 5;
  const int bpr = C >> 6;
  const int bc = t % bpr, rl = t / bpr;
  for (int i = t; i < C; i += kQtThreads) {
    const int e = i & 63;
    ms[(((e >> 2) * bpr + (i >> 6)) << 2) + (e & 3)] = sign[i];
  }
  if constexpr (AFFINE) {
    for (int i = t; i < NCH * 256; i += kQtThreads) {
      const int c = i >> 8, l = (i >> 3) & 31, h = (i >> 2) & 1, k = i & 3;
      const int pos = (((c * 2 + h) * 32 + l) << 2) + k;
      wb[pos] = i < C ? weight[i] : 0.f;
      wb[NCH * 256 + pos] = i < C ? bias[i] : 0.f;
    }
  }
  __syncthreads();
  const float4* ms4 = reinterpret_cast<const float4*>(ms);
  int it = 0;
  for (int64_t tile = blockIdx.x; tile < ntiles; tile += gridDim.x, ++it) {
    // phase 1: LayerNorm rows -> swizzled h blocks; this tile's row-maximum slot cleared (its
    // last readers, two tiles back, passed the previous tile's barriers)
    if (t < R) rmax[it & 1][t] = 0u;
    for (int r = warp; r < R; r += kQtThreads / 32) {
      const int64_t row = tile * R + r;
      if (row >= rows) break;
      uint4 hw[NCH];
      ln_row_words<T, NCH, AFFINE, MODULATE>(x + row * C, row, C, eps, wb, scale, shift, rows_per_batch,
                                             mod_stride, lane, hw);
#pragma unroll
      for (int c = 0; c < NCH; ++c) {
        const int base = c * 256 + lane * 8;
        if (base >= C) continue;
        const int b = r * bpr + (base >> 6), j = lane & 7;
        *reinterpret_cast<uint4*>(hs + b * 128 + ((j ^ (b & 7)) << 4)) = hw[c];
      }
    }
    __syncthreads();
    // phase 2: one thread per 64-element block
    const int64_t row = tile * R + rl;
    const bool active = t < R * bpr && row < rows;
    uint64_t P[32];
    const float amax = h64_block<T>(hs, t, ms4 + bc, bpr, P);
    if (active) atomicMax(&rmax[it & 1][rl], __float_as_uint(amax));
    __syncthreads();  // row maxima complete; the h tile is read
    if (active) {
      const float sc = __fdiv_rn(fmaxf(__uint_as_float(rmax[it & 1][rl]), 1e-8f), 127.0f);
      const float inv = __frcp_rn(sc);
      if (bc == 0) qscale[row] = sc;
      store_block_codes(P, sc, inv, q + row * C + bc * 64);
    }
  }
}

template <typename T, int NCH, bool AFFINE, bool MODULATE>
static int launch_lnq_tiles_t(const void* x, int64_t rows, int C, float eps, const float* w, const float* b,
                              const void* sc, const void* sh, int64_t rpb, int64_t ms, const float* sign, int8_t* q,
                              float* qs, cudaStream_t st) {
  const int bpr = C / 64, R = kQtThreads / bpr;
  const int64_t ntiles = (rows + R - 1) / R, cap = 2 * (int64_t)sm_count();
  const int grid = (int)(ntiles < cap ? ntiles : cap);
  const size_t smem = kQtThreads * 128 + (size_t)NCH * 256 * sizeof(float) * (AFFINE ? 3 : 1);
  ln_quant_tile_kernel<T, NCH, AFFINE, MODULATE><<<grid, kQtThreads, smem, st>>>(
      (const T*)x, rows, C, eps, w, b, (const T*)sc, (const T*)sh, rpb, ms, sign, q, qs, R, ntiles);
  return check_launch("layer_norm_quantize");
}

template <typename T, int NCH>
static int launch_lnq_tiles(const void* x, int64_t rows, int C, float eps, const float* w, const float* b,
                            const void* sc, const void* sh, int64_t rpb, int64_t ms, const float* sign, int8_t* q,
                            float* qs, cudaStream_t st) {
  if (w && sc) return launch_lnq_tiles_t<T, NCH, true, true>(x, rows, C, eps, w, b, sc, sh, rpb, ms, sign, q, qs, st);
  if (w) return launch_lnq_tiles_t<T, NCH, true, false>(x, rows, C, eps, w, b, sc, sh, rpb, ms, sign, q, qs, st);
  if (sc) return launch_lnq_tiles_t<T, NCH, false, true>(x, rows, C, eps, w, b, sc, sh, rpb, ms, sign, q, qs, st);
  return launch_lnq_tiles_t<T, NCH, false, false>(x, rows, C, eps, w, b, sc, sh, rpb, ms, sign, q, qs, st);
}

template <typename T, bool ROTATE>
static int launch_quant(const void* x, const float* sign, int8_t* q, float* scale, int64_t rows, int K,
                        cudaStream_t st) {
  const int chunks = (K + 255) / 256;  // 256-element chunks per row
  if (chunks > 40) return set_error(HI3D_ERR_UNSUPPORTED, "quantize_act_i8: width %d above 10240 not supported", K);
  const int wpr = chunks <= 4 ? 1 : chunks <= 8 ? 2 : chunks <= 16 ? 4 : 8;
  const int ipw = (chunks + wpr - 1) / wpr;
  switch (wpr) {
    case 1: launch_w<T, 1, ROTATE>(ipw, x, sign, q, scale, rows, K, st); break;
    case 2: launch_w<T, 2, ROTATE>(ipw, x, sign, q, scale, rows, K, st); break;
    case 4: launch_w<T, 4, ROTATE>(ipw, x, sign, q, scale, rows, K, st); break;
    default: launch_w<T, 8, ROTATE>(ipw, x, sign, q, scale, rows, K, st); break;
  }
  return check_launch("quantize_act_i8");
}

}  // namespace hi3d

using namespace hi3d;

extern "C" int hi3d_quantize_act_i8(const void* x, const float* multiplier, int8_t* q, float* scale, int64_t rows,
                                    int64_t k, int rotate, int dtype, void* stream) {
  if (!x || !q || !scale || rows < 0 || k <= 0)
    return set_error(HI3D_ERR_INVALID_ARGUMENT, "quantize_act_i8: bad pointers or sizes");
  if (k % 64) return set_error(HI3D_ERR_INVALID_ARGUMENT, "signed H64 requires width divisible by 64");
  if (rotate && !multiplier)
    return set_error(HI3D_ERR_INVALID_ARGUMENT, "quantize_act_i8: the rotation needs the sign multiplier");
  if (!aligned16(x) || !aligned16(q) || (multiplier && !aligned16(multiplier)))
    return set_error(HI3D_ERR_INVALID_ARGUMENT, "quantize_act_i8: pointers must be 16-byte aligned");
  if (rows == 0) return HI3D_OK;
  cudaStream_t st = as_stream(stream);
  const int K = (int)k;
  // the block-per-thread kernel for rotated rows of up to 16384 (256 blocks of 64)
  const bool tiles = rotate && K <= 64 * kQtThreads && rows * (K / 64) < (int64_t)1 << 31;
  if (dtype == HI3D_F16)
    return tiles ? launch_quant_tiles<__half>(x, multiplier, q, scale, rows, K, st)
           : rotate ? launch_quant<__half, true>(x, multiplier, q, scale, rows, K, st)
                    : launch_quant<__half, false>(x, multiplier, q, scale, rows, K, st);
  if (dtype == HI3D_BF16)
    return tiles ? launch_quant_tiles<__nv_bfloat16>(x, multiplier, q, scale, rows, K, st)
           : rotate ? launch_quant<__nv_bfloat16, true>(x, multiplier, q, scale, rows, K, st)
                    : launch_quant<__nv_bfloat16, false>(x, multiplier, q, scale, rows, K, st);
  return set_error(HI3D_ERR_INVALID_ARGUMENT, "quantize_act_i8: dtype must be f16 or bf16");
}

extern "C" int hi3d_layer_norm_quantize(const void* x, int8_t* q, float* qscale, int64_t rows, int64_t channels,
                                        float eps, const float* weight, const float* bias, const void* scale,
                                        const void* shift, int64_t rows_per_batch, int64_t mod_stride,
                                        const float* sign, int dtype, void* stream) {
  if (!x || !q || !qscale || !sign || rows < 0 || channels <= 0)
    return set_error(HI3D_ERR_INVALID_ARGUMENT, "layer_norm_quantize: bad pointers or sizes");
  if (channels % 64) return set_error(HI3D_ERR_INVALID_ARGUMENT, "signed H64 requires width divisible by 64");
  if (channels > 4096)
    return set_error(HI3D_ERR_UNSUPPORTED, "layer_norm_quantize: channels above 4096 not supported");
  if ((weight == nullptr) != (bias == nullptr) || (scale == nullptr) != (shift == nullptr))
    return set_error(HI3D_ERR_INVALID_ARGUMENT, "layer_norm_quantize: weight/bias and scale/shift come in pairs");
  if (!aligned16(x) || !aligned16(sign) || (reinterpret_cast<uintptr_t>(q) & 7) ||
      (scale && (!aligned16(scale) || !aligned16(shift))))
    return set_error(HI3D_ERR_INVALID_ARGUMENT, "layer_norm_quantize: misaligned pointers");
  if (scale && (rows_per_batch <= 0 || mod_stride % 8))
    return set_error(HI3D_ERR_INVALID_ARGUMENT, "layer_norm_quantize: bad rows_per_batch / mod_stride");
  if (rows == 0) return HI3D_OK;
  if (rows_per_batch <= 0) rows_per_batch = rows;
  cudaStream_t st = as_stream(stream);
  const int C = (int)channels;
  if (C <= 1024 && aligned16(q)) {  // the tiled rotation (codes stored 16 bytes at a time)
    const int nch = (C + 255) / 256;
#define HI3D_LNQT(TT, n) \
  if (nch == n) return launch_lnq_tiles<TT, n>(x, rows, C, eps, weight, bias, scale, shift, rows_per_batch, \
                                               mod_stride, sign, q, qscale, st);
    if (dtype == HI3D_F16) {
      HI3D_LNQT(__half, 1) HI3D_LNQT(__half, 2) HI3D_LNQT(__half, 3) HI3D_LNQT(__half, 4)
    } else if (dtype == HI3D_BF16) {
      HI3D_LNQT(__nv_bfloat16, 1) HI3D_LNQT(__nv_bfloat16, 2) HI3D_LNQT(__nv_bfloat16, 3)
      HI3D_LNQT(__nv_bfloat16, 4)
    }
#undef HI3D_LNQT
  }
  if (dtype == HI3D_F16)
    return dispatch_lnq<__half>(x, rows, C, eps, weight, bias, scale, shift, rows_per_batch, mod_stride, sign, q,
                                qscale, st);
  if (dtype == HI3D_BF16)
    return dispatch_lnq<__nv_bfloat16>(x, rows, C, eps, weight, bias, scale, shift, rows_per_batch, mod_stride, sign,
                                       q, qscale, st);
  return set_error(HI3D_ERR_INVALID_ARGUMENT, "layer_norm_quantize: dtype must be f16 or bf16");
}

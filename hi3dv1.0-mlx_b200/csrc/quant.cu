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
constexpr int kLnqRowsPerBlock = 4;

template <typename T, int NCH, bool AFFINE, bool MODULATE>
__global__ void __launch_bounds__(kLnqRowsPerBlock * 32)
    ln_quant_kernel(const T* __restrict__ x, int64_t rows, int C, float eps, const float* __restrict__ weight,
                    const float* __restrict__ bias, const T* __restrict__ scale, const T* __restrict__ shift,
                    int64_t rows_per_batch, int64_t mod_stride, const float* __restrict__ sign,
                    int8_t* __restrict__ q, float* __restrict__ qscale) {
  const int lane = threadIdx.x & 31;
  const int g = lane & 7;
  for (int64_t row = (int64_t)blockIdx.x * kLnqRowsPerBlock + (threadIdx.x >> 5); row < rows;
       row += (int64_t)gridDim.x * kLnqRowsPerBlock) {
    const T* xr = x + row * C;
    // ---- LayerNorm statistics (as ln_mod_kernel)
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

    // ---- h (rounded as the separate kernel rounds it), then the rotation per 64-block
    float y[NCH][8];
    float amax = 0.f;
#pragma unroll
    for (int c = 0; c < NCH; ++c) {
      const int base = c * 256 + lane * 8;
      const bool active = base < C;
      float v[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
      if (active) {
        uint4 sc = make_uint4(0, 0, 0, 0), sh = make_uint4(0, 0, 0, 0);
        if (MODULATE) {
          sc = *reinterpret_cast<const uint4*>(scale + mb + base);
          sh = *reinterpret_cast<const uint4*>(shift + mb + base);
        }
        const uint32_t* scw = reinterpret_cast<const uint32_t*>(&sc);
        const uint32_t* shw = reinterpret_cast<const uint32_t*>(&sh);
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          uint64_t yy = f2_mul(d[c][i], inv2);
          if (AFFINE) {
            const uint64_t w2 = f2_pack(weight[base + 2 * i], weight[base + 2 * i + 1]);
            const uint64_t b2 = f2_pack(bias[base + 2 * i], bias[base + 2 * i + 1]);
            yy = f2_add(f2_mul(yy, w2), b2);
          }
          uint32_t h = Cvt<T>::from_f2(yy);
          if (MODULATE) h = Cvt<T>::add2(Cvt<T>::mul2(h, scw[i]), shw[i]);
          const T* hp = reinterpret_cast<const T*>(&h);
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
      *reinterpret_cast<uint2*>(qr + base) = quant_pack8(y[c], sc, inv);
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
  if (w && sc)
    ln_quant_kernel<T, NCH, true, true><<<grid, kLnqRowsPerBlock * 32, 0, st>>>(xt, rows, C, eps, w, b, s, t, rpb, ms,
                                                                               sign, q, qs);
  else if (w)
    ln_quant_kernel<T, NCH, true, false><<<grid, kLnqRowsPerBlock * 32, 0, st>>>(xt, rows, C, eps, w, b, s, t, rpb,
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
  if (dtype == HI3D_F16)
    return rotate ? launch_quant<__half, true>(x, multiplier, q, scale, rows, K, st)
                  : launch_quant<__half, false>(x, multiplier, q, scale, rows, K, st);
  if (dtype == HI3D_BF16)
    return rotate ? launch_quant<__nv_bfloat16, true>(x, multiplier, q, scale, rows, K, st)
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
  if (dtype == HI3D_F16)
    return dispatch_lnq<__half>(x, rows, C, eps, weight, bias, scale, shift, rows_per_batch, mod_stride, sign, q,
                                qscale, st);
  if (dtype == HI3D_BF16)
    return dispatch_lnq<__nv_bfloat16>(x, rows, C, eps, weight, bias, scale, shift, rows_per_batch, mod_stride, sign,
                                       q, qscale, st);
  return set_error(HI3D_ERR_INVALID_ARGUMENT, "layer_norm_quantize: dtype must be f16 or bf16");
}

// Persistent tcgen05 GEMM for the block's projections: C = A W^T with fused
// epilogues.  One kernel template serves
//   * the W8A8 path: int8 A [M,K] x int8 W [N,K] -> exact int32 accumulators in
//     TMEM, dequantised in the epilogue as half(float(acc) * sa[m] * sw[n] + bias[n])
//     (w8a8.py:61-80 of the reference, evaluated left to right without FMA);
//   * the 16-bit path: f16/bf16 A x W -> fp32 accumulators, half(acc + bias[n])
//     (mx.addmm, transformer.py:119).
// Epilogue variants on the rounded 16-bit result y: store y; store gelu_tanh(y)
// (GELU in fp32, transformer.py:176-179); or update a residual stream in place,
// x = round(x + round(y * gate)) (transformer.py:570, :588).
//
// CTA (320 threads), one per SM, looping over 128 x 256 output tiles (16-bit GEMMs run
// as CTA pairs, cta_group::2, over 256 x 256 tiles: see PAIR below):
//   warp 0     TMA producer: A [128 x 128 B] and W [256 x 128 B] per stage
//   warp 1     MMA issuer (one lane), TMEM owner; two 256-column accumulators
//              so the epilogue of one tile overlaps the MMAs of the next
//   warps 2-9  epilogue: two warps per TMEM lane quarter (one per 128-column
//              half), results staged through shared memory for coalesced
//              16-byte global accesses
#include <type_traits>

#include "abi.h"
#include "common.cuh"

namespace hi3d {
namespace gemm {

constexpr int kThreads = 320;
constexpr int BM = 128;
constexpr int BN = 256;
constexpr int BKB = 128;  // K bytes per stage (one 128-byte swizzle row)
constexpr int NST = 4;
constexpr int A_STAGE = BM * BKB;
constexpr int B_STAGE = BN * BKB;
constexpr int EPI_WARPS = 8;
constexpr int STAGE_BYTES = 32 * 64;  // per epilogue warp: 32 rows x 32 16-bit columns
constexpr int VEC = 384;  // per epilogue warp: bias, weight scales, QK-norm gains of its 128 columns
constexpr int SMEM = NST * (A_STAGE + B_STAGE) + EPI_WARPS * (STAGE_BYTES + VEC * 4) + 1024 + 256;
// CTA pairs (cta_group::2): a 256 x 256 output tile per pair, each CTA holding 128 rows of A,
// 128 rows of W and its 128 x 256 accumulator rows.  A pair stage holds KSUB = 2 of the 64-deep
// K blocks (64 KB per CTA, a 3-deep ring): eight MMAs per stage handshake and commit instead of
// four (block projections 907 -> 881 us, bit-identical).
constexpr int KSUB = 2;
constexpr int NST_PAIR = 3;
constexpr int SMEM_PAIR =
    NST_PAIR * KSUB * (A_STAGE + B_STAGE / 2) + EPI_WARPS * (STAGE_BYTES + VEC * 4) + 1024 + 256;

enum Kind { KIND_F16 = 0, KIND_BF16 = 1, KIND_I8 = 2 };

enum Epi { EPI_STORE = 0, EPI_GELU = 1, EPI_RESIDUAL = 2, EPI_QKV_ROPE = 3 };
constexpr int kMaxPeers = 7;  // peer GPUs of one node

struct Params {
  void* out;          // [M, ldo] output (or the residual stream for EPI_RESIDUAL)
  int64_t ldo;
  const void* bias;   // [N] in the output type, or null
  const float* sa;    // [M] per-row activation scales (int8 path)
  const float* sw;    // [N] per-column weight scales (int8 path)
  const void* gate;   // [N] per batch element (EPI_RESIDUAL), or null
  int64_t rows_per_batch, gate_stride;
  int M, N, K;        // K in elements
  int tiles_m, tiles_n;
  int vec;            // 1 when output rows (and gate rows) allow 16-byte accesses
  // EPI_QKV_ROPE: the fused projection [B*N, 3*H*D] is split into q, k, v with
  // RoPE + QK RMS norm on q and k (head_dim 64)
  const float* cosv;  // [N, D/2]
  const float* sinv;  // [N, D/2]
  const float* gq;    // [H, D]
  const float* gk;    // [H, D]
  void* q;
  void* k;
  void* v;
  int seq_n, heads, token_major;
  // EPI_QKV_ROPE: every k / v store is repeated at address + peer_off[i] (the same rows of
  // the peers' gather buffers, mapped into this process), so the projection itself
  // all-gathers K and V over NVLink
  int npeers;
  int64_t peer_off[kMaxPeers];
  // or, when non-zero, every k / v store goes to address + mcast_off instead: an NVLink
  // multicast mapping of the gather buffers, so one multimem store reaches every GPU bound to
  // it (this one included) and NVSwitch does the fan-out
  int64_t mcast_off;
};

struct Barriers {
  uint64_t full[NST];
  uint64_t empty[NST];
  uint64_t acc_full[2];
  uint64_t acc_empty[2];
  uint32_t tmem_base;
  int abort;
};

// 16 bytes to every GPU bound to the multicast address `mc` (relaxed, system scope)
__device__ __forceinline__ void multimem_st16(void* mc, uint4 v) {
  asm volatile("multimem.st.relaxed.sys.global.v4.f32 [%0], {%1, %2, %3, %4};" ::"l"(mc), "r"(v.x), "r"(v.y),
               "r"(v.z), "r"(v.w)
               : "memory");
}

template <typename OutT>
__device__ __forceinline__ float gelu_tanh_f(float a) {
  const float k0 = 0.7978845608028654f;  // sqrt(2 / pi)
  return 0.5f * a * (1.0f + tanhf(k0 * (a + 0.044715f * a * a * a)));
}

// Coalesced residual loads of one 32 x 32 chunk: row group i covers rows
// m0 + i*8 + lane/4, columns n + (lane%4)*8 .. +7 (zero where not 16-byte loadable;
// the scalar path reloads those).
template <typename OutT>
__device__ __forceinline__ void prefetch_residual(const Params& p, uint4 (&r)[4], int m0, int n, int lane) {
  if constexpr (std::is_same<OutT, int32_t>::value) {
    return;
  } else {
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int m = m0 + i * 8 + (lane >> 2), nn = n + (lane & 3) * 8;
      r[i] = make_uint4(0, 0, 0, 0);
      if (p.vec && m < p.M && nn + 8 <= p.N)
        r[i] = *reinterpret_cast<const uint4*>(reinterpret_cast<const OutT*>(p.out) + (int64_t)m * p.ldo + nn);
    }
  }
}

// PAIR: launched as clusters of two CTAs.  Both CTAs load their halves of the operands
// (completion counted on the first CTA's barriers); the first CTA's MMA warp issues the
// cta_group::2 MMAs and releases stages and accumulators to both CTAs with one commit;
// each CTA runs the epilogue of its 128 accumulator rows and hands the accumulator back to
// the first CTA.
template <int KIND, int EPI, typename OutT, bool PAIR>
__global__ void __launch_bounds__(kThreads, 1)
    gemm_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB, const Params p) {
  constexpr int NSTX = PAIR ? NST_PAIR : NST;              // ring depth
  constexpr int KS = PAIR ? KSUB : 1;                       // 64-deep K blocks per stage
  constexpr int A_STAGE_L = KS * A_STAGE;                   // A bytes per stage and CTA
  constexpr int B_STAGE_L = PAIR ? KS * B_STAGE / 2 : B_STAGE;  // W bytes per stage and CTA
  constexpr int B_SUB = PAIR ? B_STAGE / 2 : B_STAGE;       // W bytes per 64-deep K block
  constexpr int TM = PAIR ? 2 * BM : BM;                   // output rows per tile
  const uint32_t rank = PAIR ? cluster_rank() : 0u;
  const int tile0 = PAIR ? (int)(blockIdx.x >> 1) : (int)blockIdx.x;
  const int tstep = PAIR ? (int)(gridDim.x >> 1) : (int)gridDim.x;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = smem;
  uint8_t* sB = smem + NSTX * A_STAGE_L;
  uint8_t* sStage = sB + NSTX * B_STAGE_L;
  float* sVec = reinterpret_cast<float*>(sStage + EPI_WARPS * STAGE_BYTES);
  Barriers* bar = reinterpret_cast<Barriers*>(sVec + EPI_WARPS * VEC);
  constexpr int ESZ = KIND == KIND_I8 ? 1 : 2;
  constexpr int BKE = BKB / ESZ;  // K elements per stage

  const int warp = warp_id(), lane = lane_id();
  const int num_tiles = p.tiles_m * p.tiles_n;
  const int kblocks = (p.K + BKE * KS - 1) / (BKE * KS);  // stages per tile
  if (threadIdx.x == 0) {
    for (int s = 0; s < NSTX; ++s) {
      mbar_init(&bar->full[s], 1);
      mbar_init(&bar->empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&bar->acc_full[a], 1);
      mbar_init(&bar->acc_empty[a], PAIR ? 2 * EPI_WARPS : EPI_WARPS);
    }
    bar->abort = 0;
    fence_barrier_init();
  }
  if (warp == 1) {
    if constexpr (PAIR) {
      tmem_alloc_pair(&bar->tmem_base, 512);
      tmem_relinquish_pair();
    } else {
      tmem_alloc(&bar->tmem_base, 512);
      tmem_relinquish();
    }
  }
  tc_fence_before();
  if constexpr (PAIR)
    cluster_sync();  // both CTAs' barriers are initialised before any cross-CTA signal
  else
    __syncthreads();
  tc_fence_after();
  const uint32_t tmem = bar->tmem_base;
  volatile int* abort = &bar->abort;

  if (warp == 0) {
    if (lane == 0) {
      tma_prefetch_desc(&tmA);
      tma_prefetch_desc(&tmB);
      int it = 0;  // global k-block counter (ring position)
      bool ok = true;
      for (int tile = tile0; ok && tile < num_tiles; tile += tstep) {
        const int m0 = (tile / p.tiles_n) * TM + (int)rank * BM;
        const int n0 = (tile % p.tiles_n) * BN + (int)rank * (BN / 2) * (PAIR ? 1 : 0);
        for (int kb = 0; kb < kblocks; ++kb, ++it) {
          const int s = it % NSTX, n = it / NSTX;
          if (!(ok = mbar_wait(&bar->empty[s], (n & 1) ^ 1, abort, 101))) break;
          if constexpr (PAIR) {
            // the first CTA expects both CTAs' bytes on its barrier
            if (rank == 0) mbar_arrive_expect_tx(&bar->full[s], 2 * (A_STAGE_L + B_STAGE_L));
            const uint32_t fb = cluster_addr(&bar->full[s], 0);
            for (int u = 0; u < KS; ++u) {
              tma_load_2d_pair(sA + s * A_STAGE_L + u * A_STAGE, &tmA, fb, (kb * KS + u) * BKE, m0);
              tma_load_2d_pair(sB + s * B_STAGE_L + u * B_SUB, &tmB, fb, (kb * KS + u) * BKE, n0);
            }
          } else {
            mbar_arrive_expect_tx(&bar->full[s], A_STAGE + B_STAGE);
            tma_load_2d(sA + s * A_STAGE, &tmA, &bar->full[s], kb * BKE, m0);
            tma_load_2d(sB + s * B_STAGE, &tmB, &bar->full[s], kb * BKE, n0);
          }
        }
      }
      volatile int no_abort = 0;
      if (!ok) {
        // drain the copies already in flight before leaving (in a pair the first CTA's
        // barriers count both CTAs' copies, and the final cluster barrier holds the second)
        if (!PAIR || rank == 0)
          for (int j = (it > NSTX ? it - NSTX : 0); j < it; ++j)
            mbar_wait(&bar->full[j % NSTX], (j / NSTX) & 1, &no_abort, 102);
      } else {
        // producer tail: wait for the MMA warp's last releases of each stage, so
        // no barrier arrive is still in flight when the CTA exits
        for (int j = (it > NSTX ? it - NSTX : 0); j < it; ++j)
          mbar_wait(&bar->empty[j % NSTX], (j / NSTX) & 1, abort, 103);
      }
    }
  } else if (warp == 1) {
    if (lane == 0 && rank == 0) {
      constexpr uint32_t idesc = KIND == KIND_I8 ? make_idesc(2, 1, 0, 0, TM, BN)
                                                 : make_idesc(1, KIND == KIND_BF16 ? 1 : 0, 0, 0, TM, BN);
      const uint32_t sAa = smem_u32(sA), sBa = smem_u32(sB);
      int it = 0, local = 0;
      bool ok = true;
      for (int tile = tile0; ok && tile < num_tiles; tile += tstep, ++local) {
        const int acc = local & 1, use = local >> 1;
        if (!(ok = mbar_wait(&bar->acc_empty[acc], (use & 1) ^ 1, abort, 110))) break;
        tc_fence_after();
        const uint32_t d = tmem + acc * BN;
        for (int kb = 0; kb < kblocks; ++kb, ++it) {
          const int s = it % NSTX, n = it / NSTX;
          if (!(ok = mbar_wait(&bar->full[s], n & 1, abort, 111))) break;
          tc_fence_after();
#pragma unroll
          for (int k = 0; k < KS * (BKB / 32); ++k) {
            const int u = k / (BKB / 32), kk = k % (BKB / 32);
            const uint64_t da = smem_desc(sAa + s * A_STAGE_L + u * A_STAGE + kk * 32, 16, 1024, kLayoutSW128);
            const uint64_t db = smem_desc(sBa + s * B_STAGE_L + u * B_SUB + kk * 32, 16, 1024, kLayoutSW128);
            const uint32_t accum = (kb > 0 || k > 0) ? 1u : 0u;
            if constexpr (PAIR) {
              if (KIND == KIND_I8)
                mma_i8_ss_pair(d, da, db, idesc, accum);
              else
                mma_f16_ss_pair(d, da, db, idesc, accum);
            } else {
              if (KIND == KIND_I8)
                mma_i8_ss(d, da, db, idesc, accum);
              else
                mma_f16_ss(d, da, db, idesc, accum);
            }
          }
          if constexpr (PAIR)
            tc_commit_pair(&bar->empty[s], 3);
          else
            tc_commit(&bar->empty[s]);
        }
        if (!ok) break;
        if constexpr (PAIR)
          tc_commit_pair(&bar->acc_full[acc], 3);
        else
          tc_commit(&bar->acc_full[acc]);
      }
    }
  } else {
    // ------------------------------------------------------------ epilogue
    // Warp w (2..9) reads TMEM lanes 32 (w % 4) .. +31 (rows q*32.. of the tile)
    // and columns 128 h .. 128 h + 127 with h = (w - 2) / 4.  Per 32-column chunk:
    //   phase 1, thread = row: accumulators -> rounded 16-bit y (bias, dequant,
    //            GELU) -> the warp's swizzled 32 x 64 B staging tile;
    //   phase 2, coalesced: lane -> (row i*8 + lane/4, 16-byte column group
    //            lane%4): residual/gate update and 16-byte global stores, eight
    //            rows x 64 contiguous bytes per instruction.
    // The residual tile is prefetched with coalesced loads before the
    // accumulator wait.
    const int q = warp & 3, h = (warp - 2) >> 2, ew = warp - 2;
    uint8_t* stage = sStage + ew * STAGE_BYTES;
    // [0, 128): bias of this warp's columns; [128, 256): weight scales; [256, 384): QK-norm gains
    float* vec = sVec + ew * VEC;
    const uint32_t lane_addr = (uint32_t)(q * 32) << 16;
    constexpr bool kRaw = std::is_same<OutT, int32_t>::value;
    // Residual rows of this warp's strip, [chunk][row group]: loaded for the first
    // tile before its accumulator wait, and for each next tile chunk by chunk as
    // the current tile's chunks finish, so the loads overlap the current tile.
    uint4 res[4][4];
    int local = 0;
    for (int tile = tile0; tile < num_tiles; tile += tstep, ++local) {
      const int acc = local & 1, use = local >> 1;
      const int m0 = (tile / p.tiles_n) * TM + (int)rank * BM + q * 32;  // this warp's first row
      const int nh = (tile % p.tiles_n) * BN + h * 128;  // this warp's first column
      if constexpr (!kRaw) {
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int nn = nh + lane * 4 + e;
          float b = 0.0f, sw = 1.0f;
          if (nn < p.N) {
            if (p.bias) b = Cvt<OutT>::to_f(reinterpret_cast<const OutT*>(p.bias)[nn]);
            if (KIND == KIND_I8) sw = p.sw[nn];
          }
          vec[lane * 4 + e] = b;
          vec[128 + lane * 4 + e] = sw;
          if (EPI == EPI_QKV_ROPE) {
            // gain of channel nn: part = nn / (H D) (q, k or v), head channel nn % (H D)
            const int hd = p.heads * 64, part = nn / hd;
            vec[256 + lane * 4 + e] = nn < p.N && part < 2 ? (part == 0 ? p.gq : p.gk)[nn - part * hd] : 1.0f;
          }
        }
      }
      if (EPI == EPI_RESIDUAL && local == 0) {
#pragma unroll
        for (int c = 0; c < 4; ++c) prefetch_residual<OutT>(p, res[c], m0, nh + c * 32, lane);
      }
      __syncwarp();
      if (!mbar_wait(&bar->acc_full[acc], use & 1, abort, 120)) break;
      tc_fence_after();
      const int mr = m0 + lane;  // phase-1 row
      float sa = 1.0f;
      if (KIND == KIND_I8 && mr < p.M && !kRaw) sa = p.sa[mr];
      if constexpr (EPI == EPI_QKV_ROPE && !kRaw) {
        // Two 64-channel heads per warp strip.  Phase 1 (thread = row): the
        // projection output y = round(acc [* sa * sw] + bias) exactly as the
        // store epilogue writes it, then for q and k heads RoPE on adjacent
        // pairs and the RMS norm in fp32 (re = y0 c - y1 s, im = y0 s + y1 c,
        // out = re * (sqrt(64) / max(|r|, 1e-12)) * g); v heads pass through.
        // Phase 2 stores each 32-channel half through the staging tile into
        // q/k/v [B, H, N, 64] (or token-major [B, N, H, 64]).
        const int hd = p.heads * 64;
        const int tok = mr < p.M ? mr : 0;
        const int tb = tok / p.seq_n, tn = tok - tb * p.seq_n;
#pragma unroll 1
        for (int hh = 0; hh < 2; ++hh) {
          const int col0 = nh + hh * 64;  // first channel of this head in the projection
          const int part = col0 / hd, head = (col0 - part * hd) >> 6;
          float yv[64];
#pragma unroll
          for (int c = 0; c < 2; ++c) {
            uint32_t v[32];
            tmem_ld32(tmem + lane_addr + acc * BN + h * 128 + hh * 64 + c * 32, v);
            tmem_wait_ld();
#pragma unroll
            for (int e = 0; e < 32; ++e) {
              const int col = hh * 64 + c * 32 + e;
              float t;
              if (KIND == KIND_I8)
                t = __fmul_rn(__fmul_rn(__int2float_rn((int)v[e]), sa), vec[128 + col]);
              else
                t = __uint_as_float(v[e]);
              if (p.bias) t = __fadd_rn(t, vec[col]);
              yv[c * 32 + e] = Cvt<OutT>::to_f(Cvt<OutT>::from_f(t));
            }
          }
          uint32_t outw[32];  // 64 rounded outputs as 16-bit pairs
          if (part < 2) {
            const float4* cs4 = reinterpret_cast<const float4*>(p.cosv + (int64_t)tn * 32);
            const float4* sn4 = reinterpret_cast<const float4*>(p.sinv + (int64_t)tn * 32);
            float ss = 0.f;
#pragma unroll
            for (int i4 = 0; i4 < 8; ++i4) {
              const float4 c4 = __ldg(cs4 + i4), s4 = __ldg(sn4 + i4);
              const float cc[4] = {c4.x, c4.y, c4.z, c4.w}, sv[4] = {s4.x, s4.y, s4.z, s4.w};
#pragma unroll
              for (int i = 0; i < 4; ++i) {
                const int pi = i4 * 4 + i;
                const float x0 = yv[2 * pi], x1 = yv[2 * pi + 1];
                const float re = x0 * cc[i] - x1 * sv[i], im = x0 * sv[i] + x1 * cc[i];
                yv[2 * pi] = re;
                yv[2 * pi + 1] = im;
                ss += re * re + im * im;
              }
            }
            const float f = __fdiv_rn(8.0f, fmaxf(sqrtf(ss), 1e-12f));  // sqrt(64) / nrm
#pragma unroll
            for (int i = 0; i < 32; ++i)
              outw[i] = Cvt<OutT>::pack2(yv[2 * i] * f * vec[256 + hh * 64 + 2 * i],
                                         yv[2 * i + 1] * f * vec[256 + hh * 64 + 2 * i + 1]);
          } else {
#pragma unroll
            for (int i = 0; i < 32; ++i) outw[i] = Cvt<OutT>::pack2(yv[2 * i], yv[2 * i + 1]);
          }
          OutT* dst_base = reinterpret_cast<OutT*>(part == 0 ? p.q : part == 1 ? p.k : p.v);
#pragma unroll
          for (int half = 0; half < 2; ++half) {
#pragma unroll
            for (int j = 0; j < 4; ++j)
              *reinterpret_cast<uint4*>(stage + lane * 64 + ((j ^ ((lane >> 1) & 3)) << 4)) =
                  make_uint4(outw[half * 16 + 4 * j], outw[half * 16 + 4 * j + 1], outw[half * 16 + 4 * j + 2],
                             outw[half * 16 + 4 * j + 3]);
            __syncwarp();
#pragma unroll
            for (int i = 0; i < 4; ++i) {
              const int rl = i * 8 + (lane >> 2), j = lane & 3;
              const int m = m0 + rl;
              const uint4 yq = *reinterpret_cast<const uint4*>(stage + rl * 64 + ((j ^ ((rl >> 1) & 3)) << 4));
              if (m < p.M) {
                const int b2 = m / p.seq_n, n2 = m - b2 * p.seq_n;
                const int64_t row = p.token_major ? ((int64_t)b2 * p.seq_n + n2) * p.heads + head
                                                  : ((int64_t)b2 * p.heads + head) * p.seq_n + n2;
                OutT* dst = dst_base + row * 64 + half * 32 + j * 8;
                if (part > 0 && p.mcast_off) {  // K and V rows into every GPU's gather buffer at once
                  multimem_st16(reinterpret_cast<char*>(dst) + p.mcast_off, yq);
                } else {
                  *reinterpret_cast<uint4*>(dst) = yq;
                  if (part > 0) {  // K and V rows also into every peer's gather buffer (NVLink stores)
#pragma unroll 1
                    for (int pp = 0; pp < p.npeers; ++pp)
                      *reinterpret_cast<uint4*>(reinterpret_cast<char*>(dst) + p.peer_off[pp]) = yq;
                  }
                }
              }
            }
            __syncwarp();
          }
        }
      } else {
        // Gate vectors of this warp's four column chunks, loaded once per tile when every row
        // of the 32-row strip belongs to one batch element (else per row group below):
        // gated residual projection 93 -> 88 us at T = 32768.
        uint4 gate_pre[4];
        // rows_per_batch is at most M (the host clamps it), so the batch index takes a 32-bit division
        const int rpb = (int)p.rows_per_batch;
        const bool gated = EPI == EPI_RESIDUAL && p.gate != nullptr;
        const bool gate_hoist = gated && p.vec && (rpb % 32) == 0;
        if (EPI == EPI_RESIDUAL && gate_hoist) {
          const OutT* g0 = reinterpret_cast<const OutT*>(p.gate) + (int64_t)(m0 / rpb) * p.gate_stride;
#pragma unroll
          for (int c = 0; c < 4; ++c) {
            const int n = nh + c * 32 + (lane & 3) * 8;
            gate_pre[c] = n + 8 <= p.N ? __ldg(reinterpret_cast<const uint4*>(g0 + n)) : make_uint4(0, 0, 0, 0);
          }
        }
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          uint32_t v[32];
          tmem_ld32(tmem + lane_addr + acc * BN + h * 128 + c * 32, v);
          tmem_wait_ld();
          const int nb = nh + c * 32;
          if constexpr (kRaw) {
            // raw exact int32 accumulators (verification / custom dequantisation), thread = row
            OutT* orow = reinterpret_cast<OutT*>(p.out) + (int64_t)mr * p.ldo;
            if (mr < p.M) {
#pragma unroll
              for (int e = 0; e < 32; e += 8) {
                const int n = nb + e;
                if (n >= p.N) break;
                if (p.vec && n + 8 <= p.N) {
                  *reinterpret_cast<uint4*>(orow + n) = make_uint4(v[e], v[e + 1], v[e + 2], v[e + 3]);
                  *reinterpret_cast<uint4*>(orow + n + 4) = make_uint4(v[e + 4], v[e + 5], v[e + 6], v[e + 7]);
                } else {
                  for (int qq = 0; qq < 8 && n + qq < p.N; ++qq) orow[n + qq] = (int32_t)v[e + qq];
                }
              }
            }
            continue;
          } else {
            // phase 1
#pragma unroll
            for (int e = 0; e < 32; e += 8) {
              float y[8];
#pragma unroll
              for (int qq = 0; qq < 8; ++qq) {
                const int col = c * 32 + e + qq;
                float t;
                if (KIND == KIND_I8)
                  t = __fmul_rn(__fmul_rn(__int2float_rn((int)v[e + qq]), sa), vec[128 + col]);
                else
                  t = __uint_as_float(v[e + qq]);
                if (p.bias) t = __fadd_rn(t, vec[col]);
                if (EPI == EPI_GELU)  // GELU of the value rounded to the output type
                  y[qq] = gelu_tanh_f<OutT>(Cvt<OutT>::to_f(Cvt<OutT>::from_f(t)));
                else
                  y[qq] = t;  // pack2 below rounds to the output type
              }
              uint4 w;
              w.x = Cvt<OutT>::pack2(y[0], y[1]);
              w.y = Cvt<OutT>::pack2(y[2], y[3]);
              w.z = Cvt<OutT>::pack2(y[4], y[5]);
              w.w = Cvt<OutT>::pack2(y[6], y[7]);
              const int j = e >> 3;
              *reinterpret_cast<uint4*>(stage + lane * 64 + ((j ^ ((lane >> 1) & 3)) << 4)) = w;
            }
            __syncwarp();
            // phase 2
#pragma unroll
            for (int i = 0; i < 4; ++i) {
              const int rl = i * 8 + (lane >> 2), j = lane & 3;
              const int m = m0 + rl, n = nb + j * 8;
              const uint4 yv = *reinterpret_cast<const uint4*>(stage + rl * 64 + ((j ^ ((rl >> 1) & 3)) << 4));
              if (m >= p.M || n >= p.N) continue;
              OutT* orow = reinterpret_cast<OutT*>(p.out) + (int64_t)m * p.ldo;
              const OutT* ya = reinterpret_cast<const OutT*>(&yv);
              // this row's gate vector (per batch element), unless hoisted for the whole strip
              const OutT* grow = gated && !gate_hoist
                                     ? reinterpret_cast<const OutT*>(p.gate) + (int64_t)(m / rpb) * p.gate_stride
                                     : nullptr;
              if (p.vec && n + 8 <= p.N) {
                if constexpr (EPI == EPI_RESIDUAL) {
                  // x + round(y * gate), rounded, on 16-bit pairs: the product of two 16-bit values
                  // is exact in fp32, and the fp32 sum of two 16-bit values rounds to the same
                  // 16-bit value as the exact sum, so the correctly rounded pair instructions give
                  // the scalar fp32 path's bits with an eighth of the instructions
                  const uint4 gv = gate_hoist ? gate_pre[c]
                                   : grow ? __ldg(reinterpret_cast<const uint4*>(grow + n)) : make_uint4(0, 0, 0, 0);
                  const uint4 xv = res[c][i];
                  uint4 w;
                  if (gated) {
                    w.x = Cvt<OutT>::add2(xv.x, Cvt<OutT>::mul2(yv.x, gv.x));
                    w.y = Cvt<OutT>::add2(xv.y, Cvt<OutT>::mul2(yv.y, gv.y));
                    w.z = Cvt<OutT>::add2(xv.z, Cvt<OutT>::mul2(yv.z, gv.z));
                    w.w = Cvt<OutT>::add2(xv.w, Cvt<OutT>::mul2(yv.w, gv.w));
                  } else {
                    w.x = Cvt<OutT>::add2(xv.x, yv.x);
                    w.y = Cvt<OutT>::add2(xv.y, yv.y);
                    w.z = Cvt<OutT>::add2(xv.z, yv.z);
                    w.w = Cvt<OutT>::add2(xv.w, yv.w);
                  }
                  *reinterpret_cast<uint4*>(orow + n) = w;
                } else {
                  *reinterpret_cast<uint4*>(orow + n) = yv;
                }
              } else {
                const OutT* gr =
                    gated ? reinterpret_cast<const OutT*>(p.gate) + (int64_t)(m / rpb) * p.gate_stride : nullptr;
                for (int qq = 0; qq < 8 && n + qq < p.N; ++qq) {
                  if (EPI == EPI_RESIDUAL) {
                    float g = Cvt<OutT>::to_f(ya[qq]);
                    if (gr) g = Cvt<OutT>::to_f(Cvt<OutT>::from_f(__fmul_rn(g, Cvt<OutT>::to_f(gr[n + qq]))));
                    orow[n + qq] = Cvt<OutT>::from_f(__fadd_rn(Cvt<OutT>::to_f(orow[n + qq]), g));
                  } else {
                    orow[n + qq] = ya[qq];
                  }
                }
              }
            }
            __syncwarp();  // the staging tile is rewritten by the next chunk
            if (EPI == EPI_RESIDUAL) {
              const int nt = tile + tstep;
              if (nt < num_tiles)
                prefetch_residual<OutT>(p, res[c], (nt / p.tiles_n) * TM + (int)rank * BM + q * 32,
                                        (nt % p.tiles_n) * BN + h * 128 + c * 32, lane);
            }
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) {
        // the accumulator belongs to the first CTA's MMA warp
        if (PAIR && rank != 0)
          mbar_arrive_remote(cluster_addr(&bar->acc_empty[acc], 0));
        else
          mbar_arrive(&bar->acc_empty[acc]);
      }
    }
    // stores into the peers' gather buffers are performed at system scope before this grid
    // completes, hence before the cross-GPU barrier that follows it on the stream signals them
    if (EPI == EPI_QKV_ROPE && (p.npeers > 0 || p.mcast_off)) __threadfence_system();
  }

  tc_fence_before();
  if constexpr (PAIR) {
    // no CTA of the pair leaves while the other may still signal its barriers
    cluster_sync();
    if (warp == 1) {
      tc_fence_after();
      tmem_dealloc_pair(tmem, 512);
    }
  } else {
    __syncthreads();
    if (warp == 1) {
      tc_fence_after();
      tmem_dealloc(tmem, 512);
    }
  }
}

}  // namespace gemm

static int num_sms() {
  static int n = 0;
  if (n == 0) {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    if (n <= 0) n = 148;
  }
  return n;
}

#ifndef HI3D_GEMM_PAIR
#define HI3D_GEMM_PAIR 1
#endif

template <int KIND, int EPI, typename OutT>
static int launch_gemm(const void* a, const void* w, int M, int N, int K, const gemm::Params& prm, cudaStream_t st) {
  using namespace gemm;
  const int esz = KIND == KIND_I8 ? 1 : 2;
  // CTA pairs for the 16-bit GEMMs with at least two 128-row blocks: each SM reads 32 KB of
  // operands per 64-deep K step instead of 48 KB (block projections 927 -> 902 us at
  // T = 32768, bit-identical).  The int8 GEMM measured slower in pairs (199 -> 208 us).
  const bool pair = HI3D_GEMM_PAIR && KIND != KIND_I8 && M > BM;
  const CUtensorMapDataType t = KIND == KIND_I8 ? CU_TENSOR_MAP_DATA_TYPE_UINT8
                                : KIND == KIND_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16
                                                    : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  CUtensorMap ma, mb;
  uint64_t da[2] = {(uint64_t)K, (uint64_t)M}, db[2] = {(uint64_t)K, (uint64_t)N};
  uint64_t sa[1] = {(uint64_t)K * esz}, sb[1] = {(uint64_t)K * esz};
  uint32_t ba[2] = {(uint32_t)(BKB / esz), BM}, bb[2] = {(uint32_t)(BKB / esz), (uint32_t)(pair ? BN / 2 : BN)};
  int rc;
  if ((rc = encode_tmap(&ma, t, 2, a, da, sa, ba, CU_TENSOR_MAP_SWIZZLE_128B))) return rc;
  if ((rc = encode_tmap(&mb, t, 2, w, db, sb, bb, CU_TENSOR_MAP_SWIZZLE_128B))) return rc;
  Params p = prm;
  const int out_esz = std::is_same<OutT, int32_t>::value ? 4 : 2;
  p.vec = ((p.ldo * out_esz) % 16 == 0 && (reinterpret_cast<uintptr_t>(p.out) & 15) == 0 &&
           (!p.gate || ((p.gate_stride * 2) % 16 == 0 && (reinterpret_cast<uintptr_t>(p.gate) & 15) == 0)))
              ? 1
              : 0;
  p.M = M;
  p.N = N;
  p.K = K;
  const int tm = pair ? 2 * BM : BM;
  p.tiles_m = (M + tm - 1) / tm;
  p.tiles_n = (N + BN - 1) / BN;
  const int tiles = p.tiles_m * p.tiles_n;
  if (!pair) {
    const int grid = tiles < num_sms() ? tiles : num_sms();
    auto kern = gemm_kernel<KIND, EPI, OutT, false>;
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM);
    if (e != cudaSuccess) return set_error(HI3D_ERR_CUDA, "gemm: smem attribute: %s", cudaGetErrorString(e));
    kern<<<grid, kThreads, SMEM, st>>>(ma, mb, p);
    return check_launch("gemm");
  }
  if constexpr (KIND == KIND_I8) {
    return set_error(HI3D_ERR_UNSUPPORTED, "gemm: int8 CTA pairs are not built");
  } else {
  auto kern = gemm_kernel<KIND, EPI, OutT, true>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_PAIR);
  if (e != cudaSuccess) return set_error(HI3D_ERR_CUDA, "gemm: smem attribute: %s", cudaGetErrorString(e));
  cudaLaunchConfig_t cfg = {};
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = SMEM_PAIR;
  cfg.stream = st;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  static int max_pairs = 0;  // co-resident pairs (one CTA per SM)
  if (max_pairs == 0) {
    cfg.gridDim = dim3(2 * (num_sms() / 2));
    int n = 0;
    e = cudaOccupancyMaxActiveClusters(&n, kern, &cfg);
    max_pairs = (e == cudaSuccess && n > 0) ? n : num_sms() / 2;
  }
  const int pairs = tiles < max_pairs ? tiles : max_pairs;
  cfg.gridDim = dim3(2 * pairs);
  e = cudaLaunchKernelEx(&cfg, kern, ma, mb, p);
  if (e != cudaSuccess) return set_error(HI3D_ERR_CUDA, "gemm: pair launch: %s", cudaGetErrorString(e));
  return check_launch("gemm");
  }
}

template <int KIND, typename OutT>
static int dispatch_epi(int epi, const void* a, const void* w, int M, int N, int K, const gemm::Params& p,
                        cudaStream_t st) {
  switch (epi) {
    case gemm::EPI_STORE: return launch_gemm<KIND, gemm::EPI_STORE, OutT>(a, w, M, N, K, p, st);
    case gemm::EPI_GELU: return launch_gemm<KIND, gemm::EPI_GELU, OutT>(a, w, M, N, K, p, st);
    case gemm::EPI_RESIDUAL: return launch_gemm<KIND, gemm::EPI_RESIDUAL, OutT>(a, w, M, N, K, p, st);
    case gemm::EPI_QKV_ROPE: return launch_gemm<KIND, gemm::EPI_QKV_ROPE, OutT>(a, w, M, N, K, p, st);
  }
  return set_error(HI3D_ERR_INVALID_ARGUMENT, "gemm: unknown epilogue %d", epi);
}

static int check_common(const char* what, const void* a, const void* w, const void* out, int64_t m, int64_t n,
                        int64_t k, int64_t ldo, int epi, const void* gate, int64_t rows_per_batch, int64_t gate_stride) {
  if (!a || !w || !out) return set_error(HI3D_ERR_INVALID_ARGUMENT, "%s: null pointer", what);
  if (m < 0 || n <= 0 || k <= 0 || m > 0x7fffffff || n > 0x7fffffff || k > 0x7fffffff)
    return set_error(HI3D_ERR_INVALID_ARGUMENT, "%s: bad sizes m=%lld n=%lld k=%lld", what, (long long)m,
                     (long long)n, (long long)k);
  if (ldo < n || !aligned16(a) || !aligned16(w))
    return set_error(HI3D_ERR_INVALID_ARGUMENT, "%s: ldo must be >= n; A and W 16-byte aligned", what);
  if (epi < 0 || epi > 2) return set_error(HI3D_ERR_INVALID_ARGUMENT, "%s: unknown epilogue %d", what, epi);
  if (gate && (epi != gemm::EPI_RESIDUAL || rows_per_batch <= 0))
    return set_error(HI3D_ERR_INVALID_ARGUMENT, "%s: gate needs the residual epilogue and rows_per_batch > 0", what);
  return HI3D_OK;
}

}  // namespace hi3d

using namespace hi3d;

extern "C" int hi3d_gemm_w8a8(const int8_t* a, const int8_t* w, const float* sa, const float* sw, const void* bias,
                              void* out, int64_t m, int64_t n, int64_t k, int64_t ldo, int epilogue,
                              const void* gate, int64_t rows_per_batch, int64_t gate_stride, int out_dtype,
                              void* stream) {
  int rc = check_common("gemm_w8a8", a, w, out, m, n, k, ldo, epilogue, gate, rows_per_batch, gate_stride);
  if (rc) return rc;
  if ((!sa || !sw) && out_dtype != HI3D_I32)
    return set_error(HI3D_ERR_INVALID_ARGUMENT, "gemm_w8a8: activation and weight scales are required");
  if (k % 16) return set_error(HI3D_ERR_INVALID_ARGUMENT, "gemm_w8a8: K must be a multiple of 16");

  if (m == 0) return HI3D_OK;
  gemm::Params p = {};
  p.out = out;
  p.ldo = ldo;
  p.bias = bias;
  p.sa = sa;
  p.sw = sw;
  p.gate = gate;
  p.rows_per_batch = rows_per_batch > 0 && rows_per_batch < m ? rows_per_batch : m;  // <= m: fits 32 bits
  p.gate_stride = gate_stride;
  cudaStream_t st = as_stream(stream);
  if (out_dtype == HI3D_F16)
    return dispatch_epi<gemm::KIND_I8, __half>(epilogue, a, w, (int)m, (int)n, (int)k, p, st);
  if (out_dtype == HI3D_BF16)
    return dispatch_epi<gemm::KIND_I8, __nv_bfloat16>(epilogue, a, w, (int)m, (int)n, (int)k, p, st);
  if (out_dtype == HI3D_I32) {
    if (epilogue != gemm::EPI_STORE)
      return set_error(HI3D_ERR_INVALID_ARGUMENT, "gemm_w8a8: int32 output stores raw accumulators only");
    return launch_gemm<gemm::KIND_I8, gemm::EPI_STORE, int32_t>(a, w, (int)m, (int)n, (int)k, p, st);
  }
  return set_error(HI3D_ERR_INVALID_ARGUMENT, "gemm_w8a8: out dtype must be f16, bf16 or i32");
}

extern "C" int hi3d_gemm(const void* a, const void* w, const void* bias, void* out, int64_t m, int64_t n, int64_t k,
                         int64_t ldo, int epilogue, const void* gate, int64_t rows_per_batch, int64_t gate_stride,
                         int dtype, void* stream) {
  int rc = check_common("gemm", a, w, out, m, n, k, ldo, epilogue, gate, rows_per_batch, gate_stride);
  if (rc) return rc;
  if (k % 8) return set_error(HI3D_ERR_INVALID_ARGUMENT, "gemm: K must be a multiple of 8");

  if (m == 0) return HI3D_OK;
  gemm::Params p = {};
  p.out = out;
  p.ldo = ldo;
  p.bias = bias;
  p.gate = gate;
  p.rows_per_batch = rows_per_batch > 0 && rows_per_batch < m ? rows_per_batch : m;  // <= m: fits 32 bits
  p.gate_stride = gate_stride;
  cudaStream_t st = as_stream(stream);
  if (dtype == HI3D_F16) return dispatch_epi<gemm::KIND_F16, __half>(epilogue, a, w, (int)m, (int)n, (int)k, p, st);
  if (dtype == HI3D_BF16)
    return dispatch_epi<gemm::KIND_BF16, __nv_bfloat16>(epilogue, a, w, (int)m, (int)n, (int)k, p, st);
  return set_error(HI3D_ERR_INVALID_ARGUMENT, "gemm: dtype must be f16 or bf16");
}

// ---------------------------------------------------------------------------
// QKV projection with RoPE + QK RMS norm + head split in the epilogue
// ---------------------------------------------------------------------------
static int qkv_rope_params(const char* what, const void* a, const void* w, const void* cosv, const void* sinv,
                           const float* gq, const float* gk, void* q, void* k, void* v, int64_t m, int64_t n_seq,
                           int heads, int head_dim, int64_t kdim, int token_major, gemm::Params* p) {
  if (!a || !w || !cosv || !sinv || !gq || !gk || !q || !k || !v)
    return set_error(HI3D_ERR_INVALID_ARGUMENT, "%s: null pointer", what);
  if (m < 0 || n_seq <= 0 || heads <= 0 || kdim <= 0 || m > 0x7fffffff || kdim > 0x7fffffff || m % n_seq)
    return set_error(HI3D_ERR_INVALID_ARGUMENT, "%s: bad sizes (rows must be batch * n_seq)", what);
  if (head_dim != 64 || (heads * 64) % gemm::BN)
    return set_error(HI3D_ERR_UNSUPPORTED, "%s: needs head_dim 64 and heads * 64 divisible by %d", what, gemm::BN);
  if (!aligned16(a) || !aligned16(w) || !aligned16(cosv) || !aligned16(sinv) || !aligned16(q) || !aligned16(k) ||
      !aligned16(v))
    return set_error(HI3D_ERR_INVALID_ARGUMENT, "%s: pointers must be 16-byte aligned", what);
  *p = gemm::Params{};
  p->out = q;
  p->ldo = 3 * (int64_t)heads * 64;
  p->rows_per_batch = m > 0 ? m : 1;
  p->cosv = static_cast<const float*>(cosv);
  p->sinv = static_cast<const float*>(sinv);
  p->gq = gq;
  p->gk = gk;
  p->q = q;
  p->k = k;
  p->v = v;
  p->seq_n = (int)n_seq;
  p->heads = heads;
  p->token_major = token_major ? 1 : 0;
  return HI3D_OK;
}

static int set_peers(const char* what, const int64_t* peer_offsets, int num_peers, int64_t multicast_offset,
                     gemm::Params* p) {
  if (num_peers < 0 || num_peers > gemm::kMaxPeers || (num_peers > 0 && !peer_offsets))
    return set_error(HI3D_ERR_INVALID_ARGUMENT, "%s: num_peers must be in [0, %d] with the offsets given", what,
                     gemm::kMaxPeers);
  if (multicast_offset % 16 || (multicast_offset && num_peers))
    return set_error(HI3D_ERR_INVALID_ARGUMENT,
                     "%s: multicast_offset must be a multiple of 16 bytes, and excludes peer offsets", what);
  p->mcast_off = multicast_offset;
  p->npeers = num_peers;
  for (int i = 0; i < num_peers; ++i) {
    if (peer_offsets[i] % 16 || peer_offsets[i] == 0)
      return set_error(HI3D_ERR_INVALID_ARGUMENT, "%s: peer offset %d must be a non-zero multiple of 16 bytes", what,
                       i);
    p->peer_off[i] = peer_offsets[i];
  }
  return HI3D_OK;
}

extern "C" int hi3d_gemm_qkv_rope(const void* a, const void* w, const void* bias, const float* cosv,
                                  const float* sinv, const float* gamma_q, const float* gamma_k, void* q, void* k,
                                  void* v, int64_t m, int64_t n_seq, int heads, int head_dim, int64_t kdim,
                                  int token_major, int dtype, void* stream) {
  return hi3d_gemm_qkv_rope_peers(a, w, bias, cosv, sinv, gamma_q, gamma_k, q, k, v, m, n_seq, heads, head_dim, kdim,
                                  token_major, dtype, nullptr, 0, 0, stream);
}

extern "C" int hi3d_gemm_qkv_rope_peers(const void* a, const void* w, const void* bias, const float* cosv,
                                        const float* sinv, const float* gamma_q, const float* gamma_k, void* q,
                                        void* k, void* v, int64_t m, int64_t n_seq, int heads, int head_dim,
                                        int64_t kdim, int token_major, int dtype, const int64_t* peer_offsets,
                                        int num_peers, int64_t multicast_offset, void* stream) {
  gemm::Params p;
  int rc = qkv_rope_params("gemm_qkv_rope", a, w, cosv, sinv, gamma_q, gamma_k, q, k, v, m, n_seq, heads, head_dim,
                           kdim, token_major, &p);
  if (rc) return rc;
  if ((rc = set_peers("gemm_qkv_rope", peer_offsets, num_peers, multicast_offset, &p))) return rc;
  if (kdim % 8) return set_error(HI3D_ERR_INVALID_ARGUMENT, "gemm_qkv_rope: K must be a multiple of 8");
  if (m == 0) return HI3D_OK;
  p.bias = bias;
  const int n = 3 * heads * 64;
  cudaStream_t st = as_stream(stream);
  if (dtype == HI3D_F16)
    return launch_gemm<gemm::KIND_F16, gemm::EPI_QKV_ROPE, __half>(a, w, (int)m, n, (int)kdim, p, st);
  if (dtype == HI3D_BF16)
    return launch_gemm<gemm::KIND_BF16, gemm::EPI_QKV_ROPE, __nv_bfloat16>(a, w, (int)m, n, (int)kdim, p, st);
  return set_error(HI3D_ERR_INVALID_ARGUMENT, "gemm_qkv_rope: dtype must be f16 or bf16");
}

extern "C" int hi3d_gemm_w8a8_qkv_rope(const int8_t* a, const int8_t* w, const float* sa, const float* sw,
                                       const void* bias, const float* cosv, const float* sinv, const float* gamma_q,
                                       const float* gamma_k, void* q, void* k, void* v, int64_t m, int64_t n_seq,
                                       int heads, int head_dim, int64_t kdim, int token_major, int out_dtype,
                                       void* stream) {
  return hi3d_gemm_w8a8_qkv_rope_peers(a, w, sa, sw, bias, cosv, sinv, gamma_q, gamma_k, q, k, v, m, n_seq, heads,
                                       head_dim, kdim, token_major, out_dtype, nullptr, 0, 0, stream);
}

extern "C" int hi3d_gemm_w8a8_qkv_rope_peers(const int8_t* a, const int8_t* w, const float* sa, const float* sw,
                                             const void* bias, const float* cosv, const float* sinv,
                                             const float* gamma_q, const float* gamma_k, void* q, void* k, void* v,
                                             int64_t m, int64_t n_seq, int heads, int head_dim, int64_t kdim,
                                             int token_major, int out_dtype, const int64_t* peer_offsets,
                                             int num_peers, int64_t multicast_offset, void* stream) {
  gemm::Params p;
  int rc = qkv_rope_params("gemm_w8a8_qkv_rope", a, w, cosv, sinv, gamma_q, gamma_k, q, k, v, m, n_seq, heads,
                           head_dim, kdim, token_major, &p);
  if (rc) return rc;
  if ((rc = set_peers("gemm_w8a8_qkv_rope", peer_offsets, num_peers, multicast_offset, &p))) return rc;
  if (!sa || !sw) return set_error(HI3D_ERR_INVALID_ARGUMENT, "gemm_w8a8_qkv_rope: scales are required");
  if (kdim % 16) return set_error(HI3D_ERR_INVALID_ARGUMENT, "gemm_w8a8_qkv_rope: K must be a multiple of 16");
  if (m == 0) return HI3D_OK;
  p.bias = bias;
  p.sa = sa;
  p.sw = sw;
  const int n = 3 * heads * 64;
  cudaStream_t st = as_stream(stream);
  if (out_dtype == HI3D_F16)
    return launch_gemm<gemm::KIND_I8, gemm::EPI_QKV_ROPE, __half>(a, w, (int)m, n, (int)kdim, p, st);
  if (out_dtype == HI3D_BF16)
    return launch_gemm<gemm::KIND_I8, gemm::EPI_QKV_ROPE, __nv_bfloat16>(a, w, (int)m, n, (int)kdim, p, st);
  return set_error(HI3D_ERR_INVALID_ARGUMENT, "gemm_w8a8_qkv_rope: out dtype must be f16 or bf16");
}

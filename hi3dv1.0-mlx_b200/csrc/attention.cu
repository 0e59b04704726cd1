// Flash attention forward for sm_100a: tcgen05 MMAs with TMEM accumulators,
// TMA-fed K/V ring, two 128-row query tiles per CTA whose softmax warps run
// continuously while the tensor core computes the other products.
//
// Numerics (attention.py:84-233 of the reference): S = Q K^T in fp32; online
// softmax in the exp2 domain (scale * log2 e folded into one multiplier);
// P = exp2(s - m) summed unrounded into l, rounded to the I/O type for the
// P V product, which accumulates in fp32; output O / l rounded once.
//
// CTA layout (352 threads):
//   warp 0      TMA producer (one lane): Q tiles once, then K/V blocks into
//               an NST-stage ring
//   warp 1      MMA issuer of query tile 0 (one lane); owns the TMEM allocation
//   warp 10     MMA issuer of query tile 1 (one lane)
//   warps 2-5   softmax + O correction + epilogue of query tile 0
//   warps 6-9   the same for query tile 1
// A warp reaches TMEM lanes 32*(warp % 4) .. +31, so each group of four
// consecutive warps covers the 128 rows of its tile.
// TMEM (512 columns): tile i at column 256*i holds S [BK cols, fp32],
// P [BK/2 cols, packed 16-bit pairs] and O [D cols, fp32].
// Per tile and key block j: the softmax signals s_free once S(j) is in its
// registers, and the tile's issuer immediately computes S(j+1) into the same
// columns; P(j) V is issued when the softmax publishes P(j) (p_full).  Each
// tile's softmax therefore finds its next scores ready, and the two issuers
// wait only on their own tile, so neither tile's P V queues behind the other.
#include <type_traits>

#include "abi.h"
#include "common.cuh"

namespace hi3d {
namespace attn {

constexpr int kThreads = 352;
constexpr int kRowsPerTile = 128;
// Exponentials per 16-pair chunk of a score row evaluated by the FMA-pipe
// polynomial (the rest use the MUFU ex2 unit), balancing the two pipes.
#ifndef HI3D_ATTN_EMU_PAIRS
#define HI3D_ATTN_EMU_PAIRS 4
#endif
constexpr int kEmuPairs = HI3D_ATTN_EMU_PAIRS;
// Row maximum growth (log2 units) tolerated before O and l are rescaled.
#ifndef HI3D_ATTN_RESCALE_LOG2
#define HI3D_ATTN_RESCALE_LOG2 8.0f
#endif
constexpr float kRescaleLog2 = HI3D_ATTN_RESCALE_LOG2;

template <int D>
struct Cfg {
  static constexpr int NCH = (D + 63) / 64;           // 64-element (128-byte) chunks per row
  static constexpr int BK = D <= 64 ? 128 : 64;       // keys per block
  static constexpr int NST = D <= 64 ? 4 : 4;         // K/V ring stages
  static constexpr int Q_CHUNK = kRowsPerTile * 128;  // bytes of one Q chunk
  static constexpr int KV_CHUNK = BK * 128;           // bytes of one K or V chunk
  static constexpr int Q_BYTES = 2 * NCH * Q_CHUNK;
  static constexpr int KV_STAGE = NCH * KV_CHUNK;
  static constexpr int S_COL = 0;
  static constexpr int P_COL = BK;
  static constexpr int O_COL = BK + BK / 2;
  static constexpr int SMEM = Q_BYTES + 2 * NST * KV_STAGE + 1024 /*align*/ + 256 /*barriers*/;
  static_assert(O_COL + D <= 256, "TMEM budget per tile");
};

struct Params {
  void* out;
  int64_t o_row, o_head, o_batch;
  const int32_t* cu_q;
  const int32_t* cu_k;
  int64_t nq, nk;
  int num_seqs, heads, tiles_per_seq;
  int kv_batched;  // 0: one K/V set shared by all sequences
  float scale2;  // softmax scale * log2(e)
  // Partial mode (part_o set): CTA `split` covers key blocks
  // [split * nb / k_splits, (split + 1) * nb / k_splits) of its sequence and writes
  // O / l (fp32) to part_o[slot0 + split][row][head][d] and the log2-sum-exp
  // m + log2(l) (in units of scale2 * s) to part_lse[slot0 + split][row][head];
  // row = packed query row (varlen) or b * nq + query row (dense).  Without
  // part_o there is one key range and O / l is written to `out`.
  int k_splits;
  int slot0;  // partial slot of split 0 (several launches can fill one partial buffer)
  float* part_o;
  float* part_lse;
  int64_t part_rows;
  // Partial mode with k_splits == 1 only: instead of writing its partial, this launch
  // folds the partials of slots [0, slot0) into its own result (merge_kernel's
  // arithmetic, slots in order with this range last) and writes the final rows to `out`.
  int merge_final;
};

// out row (b, qrow, h) of the final result
template <typename T>
__device__ __forceinline__ T* out_row(const Params& p, int b, int64_t q_start, int64_t qrow, int h) {
  return reinterpret_cast<T*>(p.out) + (int64_t)(p.cu_q ? 0 : b) * p.o_batch + (q_start + qrow) * p.o_row +
         (int64_t)h * p.o_head;
}

__device__ __forceinline__ float slot_lse(const Params& p, int s, int64_t prow, int h) {
  return p.part_lse[((int64_t)s * p.part_rows + prow) * p.heads + h];
}

struct Barriers {
  uint64_t q_full;
  uint64_t k_full[4];
  uint64_t v_full[4];
  uint64_t kv_empty[4];
  uint64_t s_full[2];
  uint64_t s_free[2];  // the tile's softmax has read its scores into registers
  uint64_t p_full[2];
  uint64_t o_done[2];
  uint32_t tmem_base;
  int abort;
};

// PARTIAL: key-split launch writing partial O / l and log2-sum-exp (Params::part_o);
// otherwise one pass over all keys writing `out`.  Two instantiations keep the
// single-pass kernel free of the split bookkeeping.
template <typename T, int D, bool PARTIAL>
__global__ void __launch_bounds__(kThreads, 1)
    flash_fwd_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                     const __grid_constant__ CUtensorMap tmV, const Params p) {
  using C = Cfg<D>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sQ = smem;                         // [2][NCH][128 rows][128 B]
  uint8_t* sK = smem + C::Q_BYTES;            // [NST][NCH][BK][128 B]
  uint8_t* sV = sK + C::NST * C::KV_STAGE;    // [NST][NCH][BK][128 B]
  Barriers* bar = reinterpret_cast<Barriers*>(sV + C::NST * C::KV_STAGE);

  // ---- work decode: (head, sequence, 256-row query block[, key split]) ----
  const int split = PARTIAL ? (int)(blockIdx.x % p.k_splits) : 0;
  const int bid = PARTIAL ? (int)(blockIdx.x / p.k_splits) : (int)blockIdx.x;
  const int t = bid % p.tiles_per_seq;
  const int rest = bid / p.tiles_per_seq;
  const int b = rest % p.num_seqs;
  const int h = rest / p.num_seqs;
  int64_t q_start = 0, q_len = p.nq, k_start = 0, k_len = p.nk;
  int bq = b, bk = p.kv_batched ? b : 0;
  if (p.cu_q) {
    q_start = p.cu_q[b];
    q_len = p.cu_q[b + 1] - q_start;
    bq = 0;
  }
  if (p.cu_k) {
    k_start = p.cu_k[b];
    k_len = p.cu_k[b + 1] - k_start;
    bk = 0;
  }
  const int64_t q_row0 = (int64_t)t * 2 * kRowsPerTile;
  if (q_row0 >= q_len) return;  // uniform across the CTA
  int nblk;  // key blocks of this CTA
  if constexpr (PARTIAL) {
    const int nblk_all = k_len > 0 ? (int)((k_len + C::BK - 1) / C::BK) : 0;
    const int kb0 = (int)((int64_t)split * nblk_all / p.k_splits);
    nblk = (int)((int64_t)(split + 1) * nblk_all / p.k_splits) - kb0;
    if (nblk <= 0) {
      // no keys for this CTA: its rows are marked empty (log2-sum-exp -inf), or, when
      // merging, the final rows come from the earlier slots alone
      for (int e = threadIdx.x; e < 2 * kRowsPerTile; e += blockDim.x) {
        const int64_t qr = q_row0 + e;
        if (qr >= q_len) continue;
        const int64_t prow = p.cu_q ? q_start + qr : (int64_t)b * p.nq + qr;
        if (!p.merge_final) {
          p.part_lse[((int64_t)(p.slot0 + split) * p.part_rows + prow) * p.heads + h] = -INFINITY;
          continue;
        }
        float mx = -INFINITY;
        for (int s = 0; s < p.slot0; ++s) mx = fmaxf(mx, slot_lse(p, s, prow, h));
        if (mx == -INFINITY) continue;  // no keys at all: the row is left untouched
        float wsum = 0.f;
        for (int s = 0; s < p.slot0; ++s) {
          const float ls = slot_lse(p, s, prow, h);
          if (ls != -INFINITY) wsum += exp2f(ls - mx);
        }
        const float iw = 1.0f / wsum;
        T* dst = out_row<T>(p, b, q_start, qr, h);
        for (int d0 = 0; d0 < D; d0 += 8) {
          float acc[8] = {};
          for (int s = 0; s < p.slot0; ++s) {
            const float ls = slot_lse(p, s, prow, h);
            if (ls == -INFINITY) continue;
            const float w = exp2f(ls - mx);
            const float* po = p.part_o + (((int64_t)s * p.part_rows + prow) * p.heads + h) * D + d0;
#pragma unroll
            for (int u = 0; u < 8; ++u) acc[u] += w * po[u];
          }
          uint4 o;
          o.x = Cvt<T>::pack2(acc[0] * iw, acc[1] * iw);
          o.y = Cvt<T>::pack2(acc[2] * iw, acc[3] * iw);
          o.z = Cvt<T>::pack2(acc[4] * iw, acc[5] * iw);
          o.w = Cvt<T>::pack2(acc[6] * iw, acc[7] * iw);
          *reinterpret_cast<uint4*>(dst + d0) = o;
        }
      }
      return;
    }
    // key blocks are numbered from the first block of this CTA's range
    k_start += (int64_t)kb0 * C::BK;
    k_len -= (int64_t)kb0 * C::BK;
  } else {
    if (k_len <= 0) return;
    nblk = (int)((k_len + C::BK - 1) / C::BK);
  }

  const int warp = warp_id(), lane = lane_id();
  if (threadIdx.x == 0) {
    mbar_init(&bar->q_full, 1);
    for (int s = 0; s < C::NST; ++s) {
      mbar_init(&bar->k_full[s], 1);
      mbar_init(&bar->v_full[s], 1);
      mbar_init(&bar->kv_empty[s], 2);  // released by both tiles' MMA issuers
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&bar->s_full[i], 1);
      mbar_init(&bar->s_free[i], 4);  // one arrival per softmax warp of the tile
      mbar_init(&bar->p_full[i], kRowsPerTile);
      mbar_init(&bar->o_done[i], 1);
    }
    bar->abort = 0;
    fence_barrier_init();
  }
  if (warp == 1) {
    tmem_alloc(&bar->tmem_base, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = bar->tmem_base;
  volatile int* abort = &bar->abort;

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      tma_prefetch_desc(&tmQ);
      tma_prefetch_desc(&tmK);
      tma_prefetch_desc(&tmV);
      mbar_arrive_expect_tx(&bar->q_full, C::Q_BYTES);
      for (int i = 0; i < 2; ++i)
        for (int c = 0; c < C::NCH; ++c)
          tma_load_4d(sQ + (i * C::NCH + c) * C::Q_CHUNK, &tmQ, &bar->q_full, c * 64,
                      (int)(q_start + q_row0 + i * kRowsPerTile), h, bq);
      int issued = 0;
      for (int j = 0; j < nblk; ++j) {
        const int s = j % C::NST, n = j / C::NST;
        if (!mbar_wait(&bar->kv_empty[s], (n & 1) ^ 1, abort, 1)) break;
        const int krow = (int)(k_start + (int64_t)j * C::BK);
        mbar_arrive_expect_tx(&bar->k_full[s], C::KV_STAGE);
        for (int c = 0; c < C::NCH; ++c)
          tma_load_4d(sK + s * C::KV_STAGE + c * C::KV_CHUNK, &tmK, &bar->k_full[s], c * 64, krow, h, bk);
        mbar_arrive_expect_tx(&bar->v_full[s], C::KV_STAGE);
        for (int c = 0; c < C::NCH; ++c)
          tma_load_4d(sV + s * C::KV_STAGE + c * C::KV_CHUNK, &tmV, &bar->v_full[s], c * 64, krow, h, bk);
        issued = j + 1;
      }
      if (*abort) {
        // Drain: let every copy already issued land before the CTA exits.
        mbar_wait(&bar->q_full, 0, abort, 2);
        for (int j = (issued > C::NST ? issued - C::NST : 0); j < issued; ++j) {
          const int s = j % C::NST, n = j / C::NST;
          volatile int no_abort = 0;
          mbar_wait(&bar->k_full[s], n & 1, &no_abort, 3);
          mbar_wait(&bar->v_full[s], n & 1, &no_abort, 3);
        }
      }
    }
  } else if (warp == 1 || warp == 10) {
    // ------------------------------------------------------------ MMA issuers
    // Warp 1 issues tile 0's MMAs, warp 10 tile 1's: each waits (suspended)
    // only on its own tile's events, so neither tile's P V queues behind the
    // other tile's softmax.
    if (lane == 0) {
      constexpr uint32_t fmt = std::is_same<T, __nv_bfloat16>::value ? 1u : 0u;
      constexpr uint32_t idesc_s = make_idesc(1, fmt, 0, 0, kRowsPerTile, C::BK);
      constexpr uint32_t idesc_pv = make_idesc(1, fmt, 0, 1, kRowsPerTile, D);
      // Base descriptors, built once.  Moving a descriptor by `off` bytes adds
      // off >> 4 to its start-address field (no carry: shared addresses < 2^18).
      const uint64_t dQ = smem_desc(smem_u32(sQ), 16, 1024, kLayoutSW128);
      const uint64_t dK = smem_desc(smem_u32(sK), 16, 1024, kLayoutSW128);
      const uint64_t dV = smem_desc(smem_u32(sV), C::KV_CHUNK, 1024, kLayoutSW128);
      auto issue_s = [&](int i, int s) {
        const uint64_t dKs = dK + (uint64_t)((s * C::KV_STAGE) >> 4);
        const uint32_t d = tmem + 256 * i + C::S_COL;
#pragma unroll
        for (int ks = 0; ks < D / 16; ++ks) {
          const uint32_t off_q = ((i * C::NCH + (ks >> 2)) * C::Q_CHUNK + (ks & 3) * 32) >> 4;
          const uint32_t off_k = ((ks >> 2) * C::KV_CHUNK + (ks & 3) * 32) >> 4;
          mma_f16_ss(d, dQ + off_q, dKs + off_k, idesc_s, ks > 0 ? 1u : 0u);
        }
        tc_commit(&bar->s_full[i]);
      };
      const int i = warp == 1 ? 0 : 1;
      bool ok = mbar_wait(&bar->q_full, 0, abort, 10) && mbar_wait(&bar->k_full[0], 0, abort, 11);
      if (ok) {
        tc_fence_after();
        issue_s(i, 0);
      }
      // Per block j: S_i(j+1) as soon as softmax i has read S_i(j) (s_free), then
      // P_i(j) V once it has published P_i(j).
      for (int j = 0; ok && j < nblk; ++j) {
        const int s = j % C::NST, n = j / C::NST;
        const int s1 = (j + 1) % C::NST, n1 = (j + 1) / C::NST;
        if (j + 1 < nblk) {
          if (!(ok = mbar_wait(&bar->k_full[s1], n1 & 1, abort, 11))) break;
          if (!(ok = mbar_wait(&bar->s_free[i], j & 1, abort, 15))) break;
          tc_fence_after();
          issue_s(i, s1);
        }
        if (!(ok = mbar_wait(&bar->v_full[s], n & 1, abort, 13))) break;
        if (!(ok = mbar_wait(&bar->p_full[i], j & 1, abort, 14))) break;
        tc_fence_after();
        const uint64_t dVs = dV + (uint64_t)((s * C::KV_STAGE) >> 4);
        const uint32_t dO = tmem + 256 * i + C::O_COL, aP = tmem + 256 * i + C::P_COL;
#pragma unroll
        for (int ks = 0; ks < C::BK / 16; ++ks)
          mma_f16_ts(dO, aP + ks * 8, dVs + (uint64_t)(ks * (2048 >> 4)), idesc_pv, (j > 0 || ks > 0) ? 1u : 0u);
        tc_commit(&bar->o_done[i]);
        // Release the stage only when a later block will be loaded into it, so
        // that every commit has a waiter before the CTA exits.
        if (j + C::NST < nblk) tc_commit(&bar->kv_empty[s]);
      }
    }
  } else {
    // ------------------------------------------------------------ softmax
    const int i = (warp - 2) >> 2;   // query tile
    const int sub = warp & 3;        // TMEM lane quarter
    const int row = sub * 32 + lane; // row within the tile
    const uint32_t lane_addr = (uint32_t)(sub * 32) << 16;
    const uint32_t tS = tmem + lane_addr + 256 * i + C::S_COL;
    const uint32_t tP = tmem + lane_addr + 256 * i + C::P_COL;
    const uint32_t tO = tmem + lane_addr + 256 * i + C::O_COL;
    const float scale2 = p.scale2;
    const uint64_t scale2x2 = f2_pack(scale2, scale2);
    float m_run = -INFINITY, l_run = 0.f;
    bool ok = true;
    for (int j = 0; j < nblk; ++j) {
      if (!(ok = mbar_wait(&bar->s_full[i], j & 1, abort, 20))) break;
      tc_fence_after();
      uint32_t sv[C::BK];
#pragma unroll
      for (int c = 0; c < C::BK / 32; ++c) tmem_ld32(tS + c * 32, *reinterpret_cast<uint32_t(*)[32]>(&sv[c * 32]));
      tmem_wait_ld();
      // scores are in registers: the next block's S may overwrite them
      if (j + 1 < nblk) {
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&bar->s_free[i]);
      }

      const int klim = (int)(k_len - (int64_t)j * C::BK);  // valid keys in this block
      if (klim < C::BK) {
#pragma unroll
        for (int e = 0; e < C::BK; ++e)
          if (e >= klim) sv[e] = __float_as_uint(-INFINITY);
      }
      // Row maximum with four independent chains (a single chain of BK dependent
      // max operations would leave the two softmax warps of each sub-partition
      // waiting on latency).
      float mq[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
#pragma unroll
      for (int e = 0; e < C::BK; e += 8) {
#pragma unroll
        for (int u = 0; u < 4; ++u)
          mq[u] = fmax3(mq[u], __uint_as_float(sv[e + 2 * u]), __uint_as_float(sv[e + 2 * u + 1]));
      }
      const float mx = fmaxf(fmaxf(mq[0], mq[1]), fmaxf(mq[2], mq[3]));
      // Running maximum in the scaled log2 domain.  The maximum used for the
      // exponentials (m_run) only moves when a row's maximum grows by more than
      // kRescaleLog2; until then P may reach 2^kRescaleLog2 (exact in the 16-bit
      // P and in fp32 l), and O needs no correction.  O / l is unchanged.
      const float m_blk = mx * scale2;
      const bool grow = m_blk > m_run + kRescaleLog2;
      const bool warp_grow = __any_sync(0xffffffffu, grow);
      const float m_new = grow ? m_blk : m_run;
      // the correction factor needs the MUFU unit only in the rare blocks where
      // a row of this warp moves its maximum
      float alpha = 1.0f;
      if (warp_grow) alpha = grow ? ex2_approx(m_run - m_new) : 1.0f;
      const uint64_t negm = f2_pack(-m_new, -m_new);
      uint64_t acc[4] = {0ull, 0ull, 0ull, 0ull};  // four independent packed row-sum chains
#pragma unroll
      for (int c = 0; c < C::BK / 32; ++c) {
        uint32_t pk[16];
#pragma unroll
        for (int e = 0; e < 16; ++e) {
          const uint64_t sx = f2_pack(__uint_as_float(sv[c * 32 + 2 * e]), __uint_as_float(sv[c * 32 + 2 * e + 1]));
          const uint64_t xx = f2_fma(sx, scale2x2, negm);
          uint64_t pp;
          if (e < kEmuPairs) {
            pp = f2_exp2_poly(xx);
          } else {
            float x0, x1;
            f2_unpack(xx, x0, x1);
            pp = f2_pack(ex2_approx(x0), ex2_approx(x1));
          }
          acc[e & 3] = f2_add(acc[e & 3], pp);
          float p0, p1;
          f2_unpack(pp, p0, p1);
          pk[e] = Cvt<T>::pack2(p0, p1);
        }
        // P of block j overwrites P of block j-1: wait until P V of block
        // j-1 has completed (which also makes O final for the correction).
        if (c == 0 && j > 0) {
          if (!(ok = mbar_wait(&bar->o_done[i], (j - 1) & 1, abort, 21))) break;
          tc_fence_after();
        }
        tmem_st16(tP + c * 16, pk);
      }
      if (!ok) break;
      // O *= alpha, only when a row of this warp moved its maximum
      if (j > 0 && warp_grow) {
#pragma unroll
        for (int oc = 0; oc < (D + 31) / 32; ++oc) {
          uint32_t r[32];
          tmem_ld32(tO + oc * 32, r);
          tmem_wait_ld();
#pragma unroll
          for (int e = 0; e < 32; ++e) r[e] = __float_as_uint(__uint_as_float(r[e]) * alpha);
          tmem_st32(tO + oc * 32, r);
        }
      }
      m_run = m_new;
      tmem_wait_st();
      tc_fence_before();
      mbar_arrive(&bar->p_full[i]);
      // the row sum is not needed by P V: update it after publishing P
      float a0, a1, a2, a3;
      f2_unpack(f2_add(acc[0], acc[1]), a0, a1);
      f2_unpack(f2_add(acc[2], acc[3]), a2, a3);
      l_run = l_run * alpha + ((a0 + a1) + (a2 + a3));
    }
    // ---- epilogue: O / l -> out[row, h*D + d]
    if (ok && mbar_wait(&bar->o_done[i], (nblk - 1) & 1, abort, 22)) {
      tc_fence_after();
      const int64_t qrow = q_row0 + i * kRowsPerTile + row;
      const float inv = 1.0f / l_run;
      if constexpr (PARTIAL) {
        const int64_t prow = p.cu_q ? q_start + qrow : (int64_t)b * p.nq + qrow;
        if (p.merge_final) {
          // this range's O / l and log2-sum-exp folded with the earlier slots' partials
          const float lse_own = m_run + log2f(l_run);
          float mx = lse_own, wsum = 0.f;
          if (qrow < q_len) {
            for (int s = 0; s < p.slot0; ++s) mx = fmaxf(mx, slot_lse(p, s, prow, h));
            for (int s = 0; s < p.slot0; ++s) {
              const float ls = slot_lse(p, s, prow, h);
              if (ls != -INFINITY) wsum += exp2f(ls - mx);
            }
          }
          const float w_own = exp2f(lse_own - mx);
          wsum += w_own;
          const float iw = 1.0f / wsum;
          T* dst = out_row<T>(p, b, q_start, qrow, h);
#pragma unroll
          for (int oc = 0; oc < (D + 31) / 32; ++oc) {
            uint32_t r[32];
            __syncwarp();
            tmem_ld32(tO + oc * 32, r);
            tmem_wait_ld();
            if (qrow < q_len) {
              float acc[32];
#pragma unroll
              for (int e = 0; e < 32; ++e) acc[e] = 0.f;
              for (int s = 0; s < p.slot0; ++s) {
                const float ls = slot_lse(p, s, prow, h);
                if (ls == -INFINITY) continue;
                const float w = exp2f(ls - mx);
                const float* po = p.part_o + (((int64_t)s * p.part_rows + prow) * p.heads + h) * D + oc * 32;
#pragma unroll
                for (int e = 0; e < 32 && oc * 32 + e < D; e += 4) {
                  const float4 v4 = *reinterpret_cast<const float4*>(po + e);
                  acc[e] += w * v4.x;
                  acc[e + 1] += w * v4.y;
                  acc[e + 2] += w * v4.z;
                  acc[e + 3] += w * v4.w;
                }
              }
#pragma unroll
              for (int e = 0; e < 32 && oc * 32 + e < D; e += 8) {
                float o[8];
#pragma unroll
                for (int u = 0; u < 8; ++u) o[u] = (acc[e + u] + w_own * (__uint_as_float(r[e + u]) * inv)) * iw;
                uint4 w4;
                w4.x = Cvt<T>::pack2(o[0], o[1]);
                w4.y = Cvt<T>::pack2(o[2], o[3]);
                w4.z = Cvt<T>::pack2(o[4], o[5]);
                w4.w = Cvt<T>::pack2(o[6], o[7]);
                *reinterpret_cast<uint4*>(dst + oc * 32 + e) = w4;
              }
            }
          }
        } else {
        // partial result of this key range: O / l in fp32 and the log2-sum-exp
        float* po = p.part_o + (((int64_t)(p.slot0 + split) * p.part_rows + prow) * p.heads + h) * D;
        if (qrow < q_len) p.part_lse[((int64_t)(p.slot0 + split) * p.part_rows + prow) * p.heads + h] = m_run + log2f(l_run);
#pragma unroll
        for (int oc = 0; oc < (D + 31) / 32; ++oc) {
          uint32_t r[32];
          __syncwarp();
          tmem_ld32(tO + oc * 32, r);
          tmem_wait_ld();
          if (qrow < q_len) {
#pragma unroll
            for (int e = 0; e < 32 && oc * 32 + e < D; e += 4)
              *reinterpret_cast<float4*>(po + oc * 32 + e) =
                  make_float4(__uint_as_float(r[e]) * inv, __uint_as_float(r[e + 1]) * inv,
                              __uint_as_float(r[e + 2]) * inv, __uint_as_float(r[e + 3]) * inv);
          }
        }
        }
      } else {
        T* dst = reinterpret_cast<T*>(p.out) + (int64_t)(p.cu_q ? 0 : b) * p.o_batch + (q_start + qrow) * p.o_row +
                 (int64_t)h * p.o_head;
#pragma unroll
        for (int oc = 0; oc < (D + 31) / 32; ++oc) {
          uint32_t r[32];
          __syncwarp();
          tmem_ld32(tO + oc * 32, r);
          tmem_wait_ld();
          if (qrow < q_len) {
#pragma unroll
            for (int e = 0; e < 32 && oc * 32 + e < D; e += 8) {
              uint4 w;
              w.x = Cvt<T>::pack2(__uint_as_float(r[e]) * inv, __uint_as_float(r[e + 1]) * inv);
              w.y = Cvt<T>::pack2(__uint_as_float(r[e + 2]) * inv, __uint_as_float(r[e + 3]) * inv);
              w.z = Cvt<T>::pack2(__uint_as_float(r[e + 4]) * inv, __uint_as_float(r[e + 5]) * inv);
              w.w = Cvt<T>::pack2(__uint_as_float(r[e + 6]) * inv, __uint_as_float(r[e + 7]) * inv);
              *reinterpret_cast<uint4*>(dst + oc * 32 + e) = w;
            }
          }
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

// Combines the key-split partials of one (row, head) per warp:
// out = sum_s 2^(lse_s - max) O_s / sum_s 2^(lse_s - max), rounded once.  Rows
// whose splits all saw no keys are left untouched, as in the single-pass kernel.
template <typename T, int D>
__global__ void __launch_bounds__(256) merge_kernel(const float* __restrict__ part_o,
                                                    const float* __restrict__ part_lse, T* __restrict__ out,
                                                    int64_t rows, int heads, int splits, int64_t nq, int dense,
                                                    int64_t o_row, int64_t o_head, int64_t o_batch) {
  constexpr int E = D / 32;  // elements per lane
  const int64_t wid = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (wid >= rows * heads) return;
  const int64_t r = wid / heads;
  const int h = (int)(wid - r * heads);
  float mx = -INFINITY;
  for (int s = 0; s < splits; ++s) mx = fmaxf(mx, part_lse[((int64_t)s * rows + r) * heads + h]);
  if (mx == -INFINITY) return;
  float acc[E] = {};
  float wsum = 0.f;
  for (int s = 0; s < splits; ++s) {
    const float ls = part_lse[((int64_t)s * rows + r) * heads + h];
    if (ls == -INFINITY) continue;
    const float wgt = exp2f(ls - mx);
    wsum += wgt;
    const float* po = part_o + (((int64_t)s * rows + r) * heads + h) * D + lane * E;
#pragma unroll
    for (int e = 0; e < E; ++e) acc[e] += wgt * po[e];
  }
  const float inv = 1.0f / wsum;
  const int64_t b = dense ? r / nq : 0, qr = dense ? r - b * nq : r;
  T* dst = out + b * o_batch + qr * o_row + (int64_t)h * o_head + lane * E;
#pragma unroll
  for (int e = 0; e < E; ++e) dst[e] = Cvt<T>::from_f(acc[e] * inv);
}

}  // namespace attn

static int make_attn_map(CUtensorMap* map, const void* base, int dtype, int D, int64_t rows, int heads,
                         int64_t batch, int64_t row_stride, int64_t head_stride, int64_t batch_stride, int box_rows) {
  const uint64_t esz = 2;
  uint64_t dims[4] = {(uint64_t)D, (uint64_t)rows, (uint64_t)heads, (uint64_t)batch};
  uint64_t strides[3] = {(uint64_t)row_stride * esz, (uint64_t)head_stride * esz,
                         (uint64_t)(batch_stride ? batch_stride : rows * row_stride) * esz};
  uint32_t box[4] = {64, (uint32_t)box_rows, 1, 1};
  CUtensorMapDataType t = dtype == HI3D_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  return encode_tmap(map, t, 4, base, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B);
}

// Single pass (part_o == nullptr) or partial results of k_splits key ranges into
// slots [slot0, slot0 + k_splits) of part_o / part_lse (no merge).
template <typename T, int D>
static int launch_attn(const hi3d_attn_args* a, cudaStream_t st, int k_splits = 1, float* part_o = nullptr,
                       float* part_lse = nullptr, int slot0 = 0, bool merge_final = false) {
  using C = attn::Cfg<D>;
  const bool varlen_q = a->cu_seqlens_q != nullptr, varlen_k = a->cu_seqlens_k != nullptr;
  const int64_t qb = varlen_q ? 1 : a->num_seqs;
  const int64_t kb = varlen_k ? 1 : (a->k_batch == 0 ? 1 : a->num_seqs);
  CUtensorMap mq, mk, mv;
  int rc;
  if ((rc = make_attn_map(&mq, a->q, a->dtype, D, a->nq, a->heads, qb, a->q_row, a->q_head, a->q_batch,
                          attn::kRowsPerTile)))
    return rc;
  if ((rc = make_attn_map(&mk, a->k, a->dtype, D, a->nk, a->heads, kb, a->k_row, a->k_head, a->k_batch, C::BK)))
    return rc;
  if ((rc = make_attn_map(&mv, a->v, a->dtype, D, a->nk, a->heads, kb, a->v_row, a->v_head, a->v_batch, C::BK)))
    return rc;
  attn::Params p;
  p.out = a->out;
  p.o_row = a->o_row;
  p.o_head = a->o_head;
  p.o_batch = a->o_batch;
  p.cu_q = a->cu_seqlens_q;
  p.cu_k = a->cu_seqlens_k;
  p.nq = a->nq;
  p.nk = a->nk;
  p.num_seqs = a->num_seqs;
  p.heads = a->heads;
  p.kv_batched = (!varlen_k && a->k_batch != 0) ? 1 : 0;
  const int64_t qlen_max = varlen_q ? a->max_seqlen_q : a->nq;
  p.tiles_per_seq = (int)((qlen_max + 2 * attn::kRowsPerTile - 1) / (2 * attn::kRowsPerTile));
  p.scale2 = a->scale * 1.4426950408889634f;
  p.k_splits = k_splits;
  p.slot0 = slot0;
  p.part_o = part_o;
  p.part_lse = part_lse;
  p.part_rows = varlen_q ? a->nq : (int64_t)a->num_seqs * a->nq;
  p.merge_final = merge_final ? 1 : 0;
  const int64_t grid = (int64_t)p.tiles_per_seq * a->num_seqs * a->heads * k_splits;
  if (grid == 0) return HI3D_OK;
  if (grid > 0x7fffffff) return set_error(HI3D_ERR_INVALID_ARGUMENT, "flash_attn: too many tiles");
  auto kern = part_o ? attn::flash_fwd_kernel<T, D, true> : attn::flash_fwd_kernel<T, D, false>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM);
  if (e != cudaSuccess) return set_error(HI3D_ERR_CUDA, "flash_attn: smem attribute: %s", cudaGetErrorString(e));
  kern<<<(unsigned)grid, attn::kThreads, C::SMEM, st>>>(mq, mk, mv, p);
  return check_launch("flash_attn_fwd");
}

template <typename T, int D>
static int launch_merge(const hi3d_attn_args* a, cudaStream_t st, int num_slots, const float* part_o,
                        const float* part_lse) {
  const bool varlen_q = a->cu_seqlens_q != nullptr;
  const int64_t rows = varlen_q ? a->nq : (int64_t)a->num_seqs * a->nq;
  const int64_t warps = rows * a->heads;
  if (warps == 0) return HI3D_OK;
  attn::merge_kernel<T, D><<<(unsigned)((warps + 7) / 8), 256, 0, st>>>(
      part_o, part_lse, static_cast<T*>(a->out), rows, a->heads, num_slots, a->nq, varlen_q ? 0 : 1, a->o_row,
      a->o_head, a->o_batch);
  return check_launch("flash_attn_merge");
}

static int64_t split_part_bytes(const hi3d_attn_args* a, int k_splits) {
  const int64_t rows = a->cu_seqlens_q ? a->nq : (int64_t)a->num_seqs * a->nq;
  return (int64_t)k_splits * rows * a->heads * a->head_dim * 4;
}

static int check_attn_args(const hi3d_attn_args* a) {
  if (!a || !a->q || !a->k || !a->v || !a->out)
    return set_error(HI3D_ERR_INVALID_ARGUMENT, "flash_attn: null pointer");
  if (a->dtype != HI3D_F16 && a->dtype != HI3D_BF16)
    return set_error(HI3D_ERR_INVALID_ARGUMENT, "flash_attn: dtype must be f16 or bf16");
  if (a->head_dim != 64 && a->head_dim != 96 && a->head_dim != 128)
    return set_error(HI3D_ERR_UNSUPPORTED, "flash_attn: head_dim %d not supported (64, 96, 128)", a->head_dim);
  if (a->num_seqs < 0 || a->heads <= 0 || a->nq < 0 || a->nk < 0)
    return set_error(HI3D_ERR_INVALID_ARGUMENT, "flash_attn: negative sizes");
  if (!aligned16(a->q) || !aligned16(a->k) || !aligned16(a->v) || !aligned16(a->out))
    return set_error(HI3D_ERR_INVALID_ARGUMENT, "flash_attn: pointers must be 16-byte aligned");
  const int64_t strides[] = {a->q_row, a->q_head, a->q_batch, a->k_row, a->k_head, a->k_batch,
                             a->v_row, a->v_head, a->v_batch, a->o_row, a->o_head, a->o_batch};
  for (int64_t s : strides)
    if (s < 0 || s % 8) return set_error(HI3D_ERR_INVALID_ARGUMENT, "flash_attn: strides must be multiples of 8");
  if (a->cu_seqlens_q && a->max_seqlen_q <= 0 && a->nq > 0)
    return set_error(HI3D_ERR_INVALID_ARGUMENT, "flash_attn: varlen needs max_seqlen_q");
  if (a->nq > 0x7fffffff || a->nk > 0x7fffffff)
    return set_error(HI3D_ERR_INVALID_ARGUMENT, "flash_attn: more than 2^31 rows");
  return HI3D_OK;
}

template <typename T>
static int dispatch_attn(const hi3d_attn_args* a, cudaStream_t st, int k_splits, float* part_o, float* part_lse,
                         int slot0, bool merge_final = false) {
  switch (a->head_dim) {
    case 64: return launch_attn<T, 64>(a, st, k_splits, part_o, part_lse, slot0, merge_final);
    case 96: return launch_attn<T, 96>(a, st, k_splits, part_o, part_lse, slot0, merge_final);
    default: return launch_attn<T, 128>(a, st, k_splits, part_o, part_lse, slot0, merge_final);
  }
}

template <typename T>
static int dispatch_merge(const hi3d_attn_args* a, cudaStream_t st, int num_slots, const float* part_o,
                          const float* part_lse) {
  switch (a->head_dim) {
    case 64: return launch_merge<T, 64>(a, st, num_slots, part_o, part_lse);
    case 96: return launch_merge<T, 96>(a, st, num_slots, part_o, part_lse);
    default: return launch_merge<T, 128>(a, st, num_slots, part_o, part_lse);
  }
}

}  // namespace hi3d

using namespace hi3d;

extern "C" int hi3d_flash_attn_fwd(const hi3d_attn_args* a, void* stream) {
  int rc = check_attn_args(a);
  if (rc) return rc;
  if (a->nq == 0 || a->num_seqs == 0) return HI3D_OK;
  cudaStream_t st = as_stream(stream);
  return a->dtype == HI3D_BF16 ? dispatch_attn<__nv_bfloat16>(a, st, 1, nullptr, nullptr, 0)
                               : dispatch_attn<__half>(a, st, 1, nullptr, nullptr, 0);
}

extern "C" int hi3d_flash_attn_split_workspace_size(const hi3d_attn_args* a, int k_splits, int64_t* bytes) {
  int rc = check_attn_args(a);
  if (rc) return rc;
  if (!bytes || k_splits < 1 || k_splits > 64)
    return set_error(HI3D_ERR_INVALID_ARGUMENT, "flash_attn_split: k_splits must be in [1, 64]");
  const int64_t po = split_part_bytes(a, k_splits);
  *bytes = ((po + 255) & ~int64_t(255)) + po / a->head_dim + 256;
  return HI3D_OK;
}

extern "C" int hi3d_flash_attn_fwd_split(const hi3d_attn_args* a, int k_splits, void* workspace,
                                         int64_t workspace_bytes, void* stream) {
  int64_t need = 0;
  int rc = hi3d_flash_attn_split_workspace_size(a, k_splits, &need);
  if (rc) return rc;
  if (a->nq == 0 || a->num_seqs == 0) return HI3D_OK;
  cudaStream_t st = as_stream(stream);
  if (k_splits == 1)
    return a->dtype == HI3D_BF16 ? dispatch_attn<__nv_bfloat16>(a, st, 1, nullptr, nullptr, 0)
                                 : dispatch_attn<__half>(a, st, 1, nullptr, nullptr, 0);
  if (!workspace || !aligned16(workspace) || workspace_bytes < need)
    return set_error(HI3D_ERR_CAPACITY, "flash_attn_split: workspace %lld bytes, need %lld (16-byte aligned)",
                     (long long)workspace_bytes, (long long)need);
  float* part_o = static_cast<float*>(workspace);
  float* part_lse = reinterpret_cast<float*>(static_cast<uint8_t*>(workspace) +
                                             ((split_part_bytes(a, k_splits) + 255) & ~int64_t(255)));
  rc = a->dtype == HI3D_BF16 ? dispatch_attn<__nv_bfloat16>(a, st, k_splits, part_o, part_lse, 0)
                             : dispatch_attn<__half>(a, st, k_splits, part_o, part_lse, 0);
  if (rc) return rc;
  return a->dtype == HI3D_BF16 ? dispatch_merge<__nv_bfloat16>(a, st, k_splits, part_o, part_lse)
                               : dispatch_merge<__half>(a, st, k_splits, part_o, part_lse);
}

extern "C" int hi3d_flash_attn_fwd_partial(const hi3d_attn_args* a, int k_splits, int slot0, float* part_o,
                                           float* part_lse, int64_t part_rows, void* stream) {
  int rc = check_attn_args(a);
  if (rc) return rc;
  if (k_splits < 1 || k_splits > 64 || slot0 < 0)
    return set_error(HI3D_ERR_INVALID_ARGUMENT, "flash_attn_partial: k_splits in [1, 64] and slot0 >= 0");
  if (!part_o || !part_lse || !aligned16(part_o))
    return set_error(HI3D_ERR_INVALID_ARGUMENT, "flash_attn_partial: partial buffers (part_o 16-byte aligned)");
  const int64_t rows = a->cu_seqlens_q ? a->nq : (int64_t)a->num_seqs * a->nq;
  if (part_rows != rows)
    return set_error(HI3D_ERR_INVALID_ARGUMENT, "flash_attn_partial: part_rows %lld, the query rows are %lld",
                     (long long)part_rows, (long long)rows);
  if (a->nq == 0 || a->num_seqs == 0) return HI3D_OK;
  cudaStream_t st = as_stream(stream);
  return a->dtype == HI3D_BF16 ? dispatch_attn<__nv_bfloat16>(a, st, k_splits, part_o, part_lse, slot0)
                               : dispatch_attn<__half>(a, st, k_splits, part_o, part_lse, slot0);
}

extern "C" int hi3d_flash_attn_fwd_partial_merge(const hi3d_attn_args* a, int slot0, const float* part_o,
                                                 const float* part_lse, int64_t part_rows, void* stream) {
  int rc = check_attn_args(a);
  if (rc) return rc;
  if (slot0 < 0 || slot0 > 64 || (slot0 > 0 && (!part_o || !part_lse || !aligned16(part_o))))
    return set_error(HI3D_ERR_INVALID_ARGUMENT,
                     "flash_attn_partial_merge: slot0 in [0, 64] and the partial buffers (part_o 16-byte aligned)");
  const int64_t rows = a->cu_seqlens_q ? a->nq : (int64_t)a->num_seqs * a->nq;
  if (slot0 > 0 && part_rows != rows)
    return set_error(HI3D_ERR_INVALID_ARGUMENT, "flash_attn_partial_merge: part_rows %lld, the query rows are %lld",
                     (long long)part_rows, (long long)rows);
  if (a->nq == 0 || a->num_seqs == 0) return HI3D_OK;
  cudaStream_t st = as_stream(stream);
  // the partial instantiation with merge_final reads part_o / part_lse only below slot0
  float* po = const_cast<float*>(part_o);
  float* pl = const_cast<float*>(part_lse);
  return a->dtype == HI3D_BF16 ? dispatch_attn<__nv_bfloat16>(a, st, 1, po, pl, slot0, true)
                               : dispatch_attn<__half>(a, st, 1, po, pl, slot0, true);
}

extern "C" int hi3d_flash_attn_merge(const hi3d_attn_args* a, int num_slots, const float* part_o,
                                     const float* part_lse, void* stream) {
  int rc = check_attn_args(a);
  if (rc) return rc;
  if (num_slots < 1 || !part_o || !part_lse)
    return set_error(HI3D_ERR_INVALID_ARGUMENT, "flash_attn_merge: num_slots >= 1 and partial buffers required");
  if (a->nq == 0 || a->num_seqs == 0) return HI3D_OK;
  cudaStream_t st = as_stream(stream);
  return a->dtype == HI3D_BF16 ? dispatch_merge<__nv_bfloat16>(a, st, num_slots, part_o, part_lse)
                               : dispatch_merge<__half>(a, st, num_slots, part_o, part_lse);
}

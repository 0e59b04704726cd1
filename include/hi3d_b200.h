/*
 * hi3d_b200 C ABI: the sparse-voxel refinement-transformer block of Hi3D v1.0
 * (Sparc3D) on NVIDIA B200 (sm_100a).
 *
 * Every entry point takes raw device pointers, sizes and a CUDA stream
 * (`void* stream`, a cudaStream_t; NULL = legacy default stream), enqueues its
 * work asynchronously and returns an int status (HI3D_OK = 0).  No entry point
 * synchronises the host or allocates device memory: the caller owns inputs,
 * outputs and workspaces.  On failure `hi3d_last_error_string()` describes the
 * problem (thread-local, valid until the next call on that thread).
 *
 * Kernels never trap.  Waits inside kernels are bounded; a wait that runs out
 * (which only a library bug can cause) records HI3D_ERR_DEVICE_TIMEOUT in the
 * library's device status word, read with hi3d_device_status().
 *
 * Each declaration cites the reference interface it replaces, as
 * path:line inside the devin-lai/Hi3Dv1.0-mlx source tree.
 */
#ifndef HI3D_B200_H_
#define HI3D_B200_H_

#include <stdint.h>

#if defined(__GNUC__)
#define HI3D_API __attribute__((visibility("default")))
#else
#define HI3D_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* ---- status codes ------------------------------------------------------ */
#define HI3D_OK 0
#define HI3D_ERR_INVALID_ARGUMENT 1 /* shape/dtype/layout violation (Python: ValueError) */
#define HI3D_ERR_UNSUPPORTED 2      /* valid but not implemented (Python: NotImplementedError) */
#define HI3D_ERR_CUDA 3             /* a CUDA runtime/driver call failed */
#define HI3D_ERR_DEVICE_TIMEOUT 4   /* a bounded device-side wait ran out */
#define HI3D_ERR_CAPACITY 5         /* a caller-provided workspace is too small */
#define HI3D_ERR_NCCL 6             /* an NCCL call failed (or libnccl.so.2 is not available) */

/* ---- element types ----------------------------------------------------- */
#define HI3D_F16 0
#define HI3D_BF16 1
#define HI3D_F32 2
#define HI3D_I32 3 /* raw int32 accumulators (hi3d_gemm_w8a8 output only) */

/* ---- library ----------------------------------------------------------- */
HI3D_API int hi3d_version(void);
HI3D_API const char* hi3d_last_error_string(void);

/* Copies the device status word (first device-side error) to the host; with
 * reset != 0 clears it afterwards.  Synchronises the current device. */
HI3D_API int hi3d_device_status(int* code, int* where, int* block, int* detail, int reset);

/* No counterpart in the reference (it has no device-side waits): a check of the library's
 * time-out path.  Launches one CTA whose thread waits on an mbarrier that nothing arrives at,
 * through the same bounded wait every kernel of the library uses, but with a limit of
 * limit_ns (1e3 .. 1e9 ns) instead of the library's 2 s.  The kernel returns normally; the
 * status word then holds HI3D_ERR_DEVICE_TIMEOUT with where = 900, and the context stays
 * usable. */
HI3D_API int hi3d_wait_timeout_selftest(int64_t limit_ns, void* stream);

/* ---- LayerNorm32 + adaLN modulation ------------------------------------- */
/* Replaces kernels.layer_norm_modulate (src/hi3d_mac/mlx_backend/kernels.py:206-237,
 * kernel :162-201) and upstream LayerNorm32 (src/sparc3d/nn/norm.py:12-17).
 * Per row of x [rows, channels]: fp32 mean, two-pass fp32 variance,
 * inv = 1/sqrt(var + eps); y = (x - mean) * inv; optional fp32 affine
 * (weight/bias, NULL to skip); round to the I/O type; optional modulation
 * (scale/shift in the I/O type, both NULL to skip) with two roundings:
 * h = round(h * scale); h = round(h + shift).  `mod_stride` is the element
 * stride between the scale/shift vectors of consecutive batch elements
 * (0 = one vector for all rows); `rows_per_batch` maps rows to batch elements. */
HI3D_API int hi3d_layer_norm_modulate(const void* x, void* out, int64_t rows, int64_t channels, float eps,
                             const float* weight, const float* bias, const void* scale, const void* shift,
                             int64_t rows_per_batch, int64_t mod_stride, int dtype, void* stream);

/* hi3d_layer_norm_modulate followed by SiLU (act = 1; act = 0 is the plain form): the norms of
 * the transformer's sparse res blocks, h = silu(LN32(x; weight, bias)) (norm1) and
 * h = silu(LN(x) * (1 + scale) + shift) (norm2; pass the rounded 1 + scale as `scale`)
 * (src/hi3d_mac/mlx_backend/transformer.py:418-437; upstream SparseResBlock3d.forward,
 * src/sparc3d/models/transformers/sparc3d_transformer.py:132-144).  SiLU is evaluated in fp32 on
 * the rounded value and rounded once.  With act = 1 exactly one of weight/bias and scale/shift
 * is given.  Channels up to 4352 (the 2 x 2112-channel input of the upsampling block). */
HI3D_API int hi3d_layer_norm_act(const void* x, void* out, int64_t rows, int64_t channels, float eps,
                                 const float* weight, const float* bias, const void* scale, const void* shift,
                                 int64_t rows_per_batch, int64_t mod_stride, int act, int dtype, void* stream);

/* ---- RoPE + per-head QK RMS norm + head split --------------------------- */
/* Replaces kernels.qkv_rope_rms / qkv_rope_rms_simd
 * (src/hi3d_mac/mlx_backend/kernels.py:62-90, :137-157; kernels :22-57, :93-133) and the upstream
 * pair RotaryPositionEmbedder + SparseMultiHeadRMSNorm (src/sparc3d/nn/rope.py:14-93,
 * src/sparc3d/nn/sparse/attention/modules.py:17-32).
 * qkv [batch*n, 3*heads*head_dim] (channel = part*H*D + h*D + d); cos/sin [n, head_dim/2] fp32;
 * gamma_q/gamma_k [heads, head_dim] fp32.  Q and K: rotate adjacent pairs in fp32, then
 * r / max(||r||_2, 1e-12) * gamma * sqrt(head_dim); V copied bit-exactly.
 * Outputs q, k, v in the input type, [batch, heads, n, head_dim] (out_layout 0, the reference's
 * layout) or token-major [batch, n, heads, head_dim] (out_layout 1, rows ready to be gathered
 * across ranks). */
HI3D_API int hi3d_qkv_rope_rms(const void* qkv, const float* cos, const float* sin, const float* gamma_q,
                      const float* gamma_k, void* q, void* k, void* v, int64_t batch, int64_t n, int heads,
                      int head_dim, int out_layout, int dtype, void* stream);

/* ---- flash attention (tcgen05 / TMEM, TMA-fed) --------------------------- */
/* Replaces attention.flash_attention (src/hi3d_mac/mlx_backend/attention.py:238-277,
 * kernel :84-233) and the upstream flash_attn varlen API as called at
 * src/sparc3d/nn/sparse/attention/full_attn.py:56-76 (shimmed at
 * src/hi3d_mac/torch_backend/attention.py:77-109).
 *
 * out = softmax(scale * Q K^T) V per sequence, non-causal.  S and the online
 * softmax in fp32 (exp2 domain), P rounded to the I/O type for P V, fp32 PV
 * accumulation, output O / l rounded once.
 *
 * Sequence b reads query rows [q_start, q_start + q_len) of batch slice b:
 *   cu_seqlens_q == NULL: q_start = 0, q_len = nq, batch offset b * q_batch_stride
 *   cu_seqlens_q != NULL: q_start = cu_seqlens_q[b], q_len = cu_seqlens_q[b+1] - q_start,
 *                         batch offset 0 (packed varlen).  Same for keys/values.
 * Element (row r, head h, dim d) of tensor X is at X + b*X_batch + r*X_row + h*X_head + d
 * (strides in elements; d is contiguous).  All pointers 16-byte aligned, all strides
 * multiples of 8 elements.  head_dim in {64, 96, 128}; dtype F16 or BF16.
 * cu_seqlens_* are device int32 arrays of num_seqs + 1 entries; max_seqlen_q bounds q_len.
 * Keys/values may be shared by all sequences (k_batch_stride = 0, cu_seqlens_k = NULL). */
typedef struct hi3d_attn_args {
  const void* q;
  const void* k;
  const void* v;
  void* out;
  int64_t q_row, q_head, q_batch;
  int64_t k_row, k_head, k_batch;
  int64_t v_row, v_head, v_batch;
  int64_t o_row, o_head, o_batch;
  const int32_t* cu_seqlens_q;
  const int32_t* cu_seqlens_k;
  int64_t nq;           /* rows per sequence (dense) or total rows (varlen) */
  int64_t nk;
  int64_t max_seqlen_q; /* varlen: longest query sequence */
  int32_t num_seqs;     /* batch (dense) or number of packed sequences (varlen) */
  int32_t heads;
  int32_t head_dim;
  int32_t dtype;
  float scale;
} hi3d_attn_args;

HI3D_API int hi3d_flash_attn_fwd(const hi3d_attn_args* args, void* stream);

/* The same attention with each (sequence, head, 256-row query block) split into k_splits key
 * ranges processed by separate CTAs, then merged: out = sum_s 2^(lse_s - max) O_s / sum_s
 * 2^(lse_s - max) with O_s = O / l and lse_s the log2-sum-exp of key range s (fp32), rounded
 * once.  Same contract as hi3d_flash_attn_fwd (attention.py:238-277 of the reference); splitting
 * keeps all SMs busy when the query blocks alone do not fill whole waves (a query shard per GPU).
 * Results agree with the single-pass kernel to within 16-bit output rounding.  The workspace
 * (partials, fp32) comes from the caller; k_splits in [1, 64]. */
HI3D_API int hi3d_flash_attn_split_workspace_size(const hi3d_attn_args* args, int k_splits, int64_t* bytes);
HI3D_API int hi3d_flash_attn_fwd_split(const hi3d_attn_args* args, int k_splits, void* workspace,
                                       int64_t workspace_bytes, void* stream);

/* Partial results for combining attention over disjoint key sets of the same queries (key sets
 * that become available at different times): k_splits key ranges of
 * args' keys, written as O / l (fp32) to part_o[slot0 + s][row][head][head_dim] and the
 * log2-sum-exp to part_lse[slot0 + s][row][head], row = query row (dense: b * nq + row;
 * varlen: packed row) with part_rows the number of query rows.  args->out is not touched.
 * hi3d_flash_attn_merge then writes args->out from slots [0, num_slots) as in
 * hi3d_flash_attn_fwd_split.  No counterpart in the reference (attention.py:238-277 computes all
 * keys in one pass); it serves the sharded block. */
HI3D_API int hi3d_flash_attn_fwd_partial(const hi3d_attn_args* args, int k_splits, int slot0, float* part_o,
                                         float* part_lse, int64_t part_rows, void* stream);
HI3D_API int hi3d_flash_attn_merge(const hi3d_attn_args* args, int num_slots, const float* part_o,
                                   const float* part_lse, void* stream);
/* The last key range of a split attention in one pass, merged on the fly: attends the keys of
 * `args` (one split) and, instead of writing a partial, combines its O / l and log2-sum-exp with
 * the partials already in slots [0, slot0) (the arithmetic of hi3d_flash_attn_merge, slots in
 * order with this range last) and writes the final rows to args->out.  Replaces a
 * hi3d_flash_attn_fwd_partial(k_splits = 1) + hi3d_flash_attn_merge pair; part_o / part_lse are
 * only read (may be NULL when slot0 == 0). */
HI3D_API int hi3d_flash_attn_fwd_partial_merge(const hi3d_attn_args* args, int slot0, const float* part_o,
                                               const float* part_lse, int64_t part_rows, void* stream);

/* ---- query-sharded self-attention over NCCL ------------------------------ */
/* One process per GPU.  hi3d_nccl_unique_id fills a 128-byte id on one rank, which the caller
 * hands to the others; hi3d_nccl_comm_init creates the communicator on the current device
 * (NCCL is loaded at run time from libnccl.so.2).  It is the one entry that allocates: NCCL's
 * own buffers, plus a side stream and two events for the gather, released by
 * hi3d_nccl_comm_destroy.
 *
 * hi3d_sharded_attn: the partitioned self-attention of the sharded block (the reference runs
 * one GPU and has no counterpart; it replaces attention.flash_attention, attention.py:238-277,
 * over all T rows).  This rank holds rows [rank * s_rows, (rank + 1) * s_rows) of one sequence:
 * q, k, v [s_rows, heads, head_dim] token-major.  The K/V slices of all ranks are all-gathered
 * into k_all, v_all [world * s_rows, heads, head_dim] on a high-priority side stream, which
 * `stream` then waits for; the queries attend all keys in one launch (key-split when the grid
 * is short of waves) into out [s_rows, heads * head_dim].  Same numerics as
 * hi3d_flash_attn_fwd_split over the gathered keys. */
HI3D_API int hi3d_nccl_unique_id(void* id);
HI3D_API int hi3d_nccl_comm_init(const void* id, int world, int rank, void** comm);
HI3D_API int hi3d_nccl_comm_destroy(void* comm);

/* Failure handling of the communicator (no counterpart in the reference, which has no
 * distributed code).  hi3d_nccl_comm_check: HI3D_ERR_NCCL when NCCL reports an asynchronous
 * error (a peer failed, a network error), without waiting.  hi3d_nccl_comm_wait: waits on the
 * host, up to timeout_ms, for the work enqueued on `stream` and on the gather's side stream,
 * polling ncclCommGetAsyncError meanwhile; on an asynchronous error or at the limit it calls
 * ncclCommAbort (which ends NCCL kernels still waiting for a peer) and returns HI3D_ERR_NCCL.
 * hi3d_nccl_comm_abort: the same abort, for a caller that learnt on the host (a store, a
 * heartbeat) that a peer is gone.  An aborted communicator refuses hi3d_sharded_attn and is
 * only destroyed. */
HI3D_API int hi3d_nccl_comm_check(void* comm);
HI3D_API int hi3d_nccl_comm_wait(void* comm, void* stream, int64_t timeout_ms);
HI3D_API int hi3d_nccl_comm_abort(void* comm);
HI3D_API int hi3d_sharded_attn_workspace_size(void* comm, int64_t s_rows, int heads, int head_dim, int64_t* bytes);
HI3D_API int hi3d_sharded_attn(void* comm, const void* q, const void* k, const void* v, void* k_all, void* v_all,
                               void* out, int64_t s_rows, int heads, int head_dim, float scale, int dtype,
                               void* workspace, int64_t workspace_bytes, void* stream);

/* ---- projections (tcgen05 GEMM with fused epilogues) --------------------- */
/* out = epilogue(A W^T): A [m, k] and W [n, k] row-major (K-major, as nn.Linear weights),
 * out [m, ldo] row-major.  Epilogues act on y = round(acc + bias) (bias [n] in the output
 * type, may be NULL):
 *   0  store y
 *   1  store gelu_tanh(y) (GELU in fp32, rounded once; transformer.py:176-179)
 *   2  residual update in place: out[m, n] = round(out[m, n] + round(y * gate[n])) with
 *      gate [n] per batch element (gate_stride apart, rows_per_batch rows each), or
 *      out += y when gate is NULL (transformer.py:570, :584, :588)
 * hi3d_gemm replaces the fp16 projection mx.addmm (src/hi3d_mac/mlx_backend/transformer.py:111-119,
 * 501-516): 16-bit A and W, fp32 accumulation.  k % 8 == 0. */
HI3D_API int hi3d_gemm(const void* a, const void* w, const void* bias, void* out, int64_t m, int64_t n, int64_t k,
                       int64_t ldo, int epilogue, const void* gate, int64_t rows_per_batch, int64_t gate_stride,
                       int dtype, void* stream);

/* Replaces w8a8.linear's GEMM (src/hi3d_mac/mlx_backend/w8a8.py:61-80, :105-119): int8 A [m, k]
 * x int8 W [n, k] with exact int32 accumulation, dequantised as
 * y = round(float(acc) * sa[m] * sw[n] + float(bias[n])) evaluated left to right without FMA,
 * then the epilogue above.  out_dtype HI3D_I32 stores the raw accumulators (epilogue 0,
 * scales and bias ignored).  k % 16 == 0. */
HI3D_API int hi3d_gemm_w8a8(const int8_t* a, const int8_t* w, const float* sa, const float* sw, const void* bias,
                            void* out, int64_t m, int64_t n, int64_t k, int64_t ldo, int epilogue,
                            const void* gate, int64_t rows_per_batch, int64_t gate_stride, int out_dtype,
                            void* stream);

/* The attention input projection with RoPE + QK RMS norm + head split in its epilogue: replaces
 * the fused QKV mx.addmm (src/hi3d_mac/mlx_backend/transformer.py:501-516) followed by
 * kernels.qkv_rope_rms (src/hi3d_mac/mlx_backend/kernels.py:22-90).  The projection
 * y = round(A W^T + bias) ([m, 3 * heads * 64], channel = part * H * 64 + h * 64 + d) is not
 * written out: q and k get the rotation of adjacent pairs with cos/sin [n_seq, 32] of the row's
 * position and r / max(|r|, 1e-12) * gamma * 8 in fp32 (gamma_q/gamma_k [heads, 64] fp32), v the
 * rounded projection itself.  Outputs [batch, heads, n_seq, 64] (token_major 0) or
 * [batch, n_seq, heads, 64] (token_major 1); m = batch * n_seq.  head_dim must be 64 and
 * heads * 64 a multiple of 256 (HI3D_ERR_UNSUPPORTED otherwise: use hi3d_gemm + hi3d_qkv_rope_rms). */
HI3D_API int hi3d_gemm_qkv_rope(const void* a, const void* w, const void* bias, const float* cos, const float* sin,
                                const float* gamma_q, const float* gamma_k, void* q, void* k, void* v, int64_t m,
                                int64_t n_seq, int heads, int head_dim, int64_t k_dim, int token_major, int dtype,
                                void* stream);

/* The same through int8: activation codes and scales from hi3d_quantize_act_i8, int8 weights with
 * per-channel scales, y = round(float(acc) * sa * sw + bias) as in hi3d_gemm_w8a8
 * (src/hi3d_mac/mlx_backend/w8a8.py:105-119), then the epilogue of hi3d_gemm_qkv_rope. */
HI3D_API int hi3d_gemm_w8a8_qkv_rope(const int8_t* a, const int8_t* w, const float* sa, const float* sw,
                                     const void* bias, const float* cos, const float* sin, const float* gamma_q,
                                     const float* gamma_k, void* q, void* k, void* v, int64_t m, int64_t n_seq,
                                     int heads, int head_dim, int64_t k_dim, int token_major, int out_dtype,
                                     void* stream);

/* The two projections above fused with the K/V all-gather of the query-sharded block (no
 * counterpart in the reference, which runs one GPU): every k and v store is repeated at
 * address + peer_offsets[i] for i < num_peers (<= 7; non-zero multiples of 16 bytes), i.e. into
 * the same rows of each peer GPU's gather buffer, mapped into this process (symmetric memory over
 * NVLink).  Or, with multicast_offset != 0 (a multiple of 16; no peer offsets then), every k
 * and v store goes once to address + multicast_offset, an NVLink multicast mapping of the
 * gather buffers (multimem.st: NVSwitch writes it into every bound GPU's buffer, this one
 * included).  The stores are relaxed: the caller orders them before the peers' reads with
 * hi3d_peer_barrier on the same stream.  num_peers = 0 and multicast_offset = 0 is the plain
 * projection. */
HI3D_API int hi3d_gemm_qkv_rope_peers(const void* a, const void* w, const void* bias, const float* cos,
                                      const float* sin, const float* gamma_q, const float* gamma_k, void* q, void* k,
                                      void* v, int64_t m, int64_t n_seq, int heads, int head_dim, int64_t k_dim,
                                      int token_major, int dtype, const int64_t* peer_offsets, int num_peers,
                                      int64_t multicast_offset, void* stream);
HI3D_API int hi3d_gemm_w8a8_qkv_rope_peers(const int8_t* a, const int8_t* w, const float* sa, const float* sw,
                                           const void* bias, const float* cos, const float* sin,
                                           const float* gamma_q, const float* gamma_k, void* q, void* k, void* v,
                                           int64_t m, int64_t n_seq, int heads, int head_dim, int64_t k_dim,
                                           int token_major, int out_dtype, const int64_t* peer_offsets,
                                           int num_peers, int64_t multicast_offset, void* stream);

/* Cross-GPU barrier of the peer-store gather: flags_dev is a device array of `world` pointers
 * to each rank's int32 flag words [world] (symmetric memory, zeroed before the first use); this
 * rank writes `epoch` into word `rank` of every peer's flags (release, system scope; ordered
 * after all earlier work on `stream`), then waits until every peer's word in its own flags has
 * reached `epoch` (acquire).  epoch increases by one per barrier (wrap-around safe).  The wait is
 * bounded by limit_ns (1e3 .. 6e10): when it runs out the device status word holds
 * HI3D_ERR_DEVICE_TIMEOUT with where = 950, detail = the peer, and the kernel returns. */
HI3D_API int hi3d_peer_barrier(void* const* flags_dev, int rank, int world, uint32_t epoch, int64_t limit_ns,
                               void* stream);

/* Replaces w8a8.quantize_activation (src/hi3d_mac/mlx_backend/w8a8.py:25-58, :95-102):
 * per row of x [rows, k] (k % 64 == 0), y = H64(x * multiplier) / 8 per 64-block (signed
 * natural-order Walsh-Hadamard, rotate != 0) or y = x (rotate == 0); s = max(max|y|, 1e-8) / 127;
 * q = clamp(rint(y / s), -127, 127).  Writes q [rows, k] int8 and scale [rows] fp32.
 * The fp32 butterfly follows the reference's operation order, so codes are reproducible. */
HI3D_API int hi3d_quantize_act_i8(const void* x, const float* multiplier, int8_t* q, float* scale, int64_t rows,
                                  int64_t k, int rotate, int dtype, void* stream);

/* ---- sparse voxel structure and convolution ------------------------------ */
/* Bytes of workspace hi3d_neighbour_map_build needs for n voxels (hash table). */
HI3D_API int hi3d_neighbour_map_workspace_size(int64_t n, int64_t* bytes);

/* Replaces sparse.neighbour_table (src/hi3d_mac/mlx_backend/sparse.py:29-43; OFFSETS :20) and the
 * pair search of the spconv shim (src/hi3d_mac/torch_backend/sparse_conv.py:115-149).
 * coords [n, 3] int32 (x, y, z) in [0, 2^21); query [nq, 3] (NULL = coords, nq ignored);
 * table [nq, 27] int32: table[o, k] = row of coords equal to query[o] * stride + d_k, or n
 * when absent, d_k = (k / 9 - 1, k / 3 % 3 - 1, k % 3 - 1).  stride 1 (submanifold) or 2
 * (query = downsampled coordinates).  Duplicate coordinates resolve to the last row.
 * A coords row outside [0, 2^21) is left out of the table (its neighbours see it as absent)
 * and reported without a host synchronisation: hi3d_device_status then gives
 * HI3D_ERR_INVALID_ARGUMENT, where = 210, detail = the first such row seen. */
HI3D_API int hi3d_neighbour_map_build(const int32_t* coords, int64_t n, const int32_t* query, int64_t nq,
                                      int stride, int32_t* table, void* workspace, int64_t workspace_bytes,
                                      void* stream);

/* No counterpart in the reference: an addition of this library for callers that cannot
 * allocate device memory, such as a host whose own memory pool has already reserved the
 * GPU's memory (so a cudaMalloc would fail or compete with it), a C host that binds only this
 * ABI and has no allocator for a workspace, or a latency-bound caller that cannot accept the
 * device-wide synchronisation that cudaMalloc and cudaFree imply.
 *
 * Same arguments and result as hi3d_neighbour_map_build, without the workspace: the hash table
 * lives in a fixed device array inside the library, sized for at most
 * HI3D_NEIGHBOUR_MAP_NOALLOC_MAX_VOXELS voxels (n); 6 MiB + 256 bytes of it are held on every
 * GPU that loads the library until the process exits.  A larger n returns HI3D_ERR_CAPACITY;
 * nq is not limited.  Nothing is allocated, at set-up or per call.
 *
 * Every call outside stream capture looks up the array's address in the context current at the
 * call (so a cudaDeviceReset or a driver-API context of its own is followed); a call made while
 * `stream` is capturing reuses the address of the last call on that device, so make one call
 * on a device before capturing.  `stream` must belong to the current device.  Every call on a device shares the one array, and each call clears the part
 * it uses before building, so calls in sequence are independent, but calls that overlap on the
 * GPU (on two streams, or from two host threads) race and give wrong tables. */
#define HI3D_NEIGHBOUR_MAP_NOALLOC_MAX_VOXELS 262144
HI3D_API int hi3d_neighbour_map_build_noalloc(const int32_t* coords, int64_t n, const int32_t* query, int64_t nq,
                                              int stride, int32_t* table, void* stream);

/* Bytes of workspace hi3d_downsample_structure needs for n voxels. */
HI3D_API int hi3d_downsample_workspace_size(int64_t n, int64_t* bytes);

/* Replaces sparse.downsample_structure (src/hi3d_mac/mlx_backend/sparse.py:217-233): unique
 * coords // 2 in lexicographic (x, y, z) order -> low [num_low, 3], inverse [n] (parent of each
 * row), counts [num_low] (children per parent); *num_low (device int32) receives the count.
 * low and counts must hold n rows.  Validates the coordinates with one stream synchronisation. */
HI3D_API int hi3d_downsample_structure(const int32_t* coords, int64_t n, int32_t* low, int32_t* inverse,
                                       int32_t* counts, int32_t* num_low, void* workspace, int64_t workspace_bytes,
                                       void* stream);

/* hi3d_downsample_structure that also lists the children of every low voxel: children [n] holds
 * the fine rows grouped by parent, each group in ascending row order, and offsets [n + 1]
 * delimits group g as children[offsets[g] .. offsets[g + 1]) (offsets[num_low] = n).  This is the
 * row set the reference's scatter-add visits for each parent (Geometry.downsample,
 * src/hi3d_mac/mlx_backend/transformer.py:261-263), kept so the mean is summed in a fixed order. */
HI3D_API int hi3d_downsample_structure_children(const int32_t* coords, int64_t n, int32_t* low, int32_t* inverse,
                                                int32_t* counts, int32_t* children, int32_t* offsets,
                                                int32_t* num_low, void* workspace, int64_t workspace_bytes,
                                                void* stream);

/* Replaces Geometry.downsample (src/hi3d_mac/mlx_backend/transformer.py:261-263; upstream
 * SparseDownsample, src/sparc3d/nn/sparse/spatial.py:34-82): out[g] = round(sum of x over the
 * children of g, fp32 in ascending row order, / (children + 1)) -- the upstream mean includes the
 * zero-initialised output row.  x [n, channels]; out [num_low, channels]; channels % 8 == 0. */
HI3D_API int hi3d_downsample_mean(const void* x, const int32_t* children, const int32_t* offsets, int64_t num_low,
                                  int64_t channels, void* out, int dtype, void* stream);

/* Replaces the gather-sum of Sparc3DTransformerMLX._up_conv (src/hi3d_mac/mlx_backend/transformer.py:
 * 449-475): the 3x3x3 convolution of upsampled features computed from the low level.
 * proj [num_low * 27, channels] holds every low voxel projected through each tap (row p * 27 + k,
 * a GEMM of the low features with the taps' weights); for each fine voxel o
 * out[o] = round(sum_k proj[inverse[table[o, k]] * 27 + k] + bias) over the present taps k
 * (table [n_fine, 27] of the fine level, sentinel n_fine), fp32 in tap order, bias [channels] or
 * NULL.  Upstream this is SparseUpsample followed by the conv (sparc3d_transformer.py:135-139). */
HI3D_API int hi3d_upconv_gather_sum(const void* proj, const int32_t* table, const int32_t* inverse, int64_t n_fine,
                                    int64_t channels, const void* bias, void* out, int dtype, void* stream);

/* Replaces Geometry.upsample (src/hi3d_mac/mlx_backend/transformer.py:265-266; upstream
 * SparseUpsample, src/sparc3d/nn/sparse/spatial.py:85-124): out[o] = src[index[o]] for
 * rows o of out [rows, channels]; channels % 8 == 0. */
HI3D_API int hi3d_gather_rows(const void* src, const int32_t* index, int64_t rows, int64_t channels, void* out,
                              int dtype, void* stream);

/* 27-bit mask per 128-row output tile of the taps with at least one present neighbour
 * (tap_mask [ceil(n_out / 128)]); hi3d_sparse_conv skips the others. */
HI3D_API int hi3d_conv_tap_mask(const int32_t* table, int64_t n_out, int64_t n_in, uint32_t* tap_mask, void* stream);

/* Replaces sparse.sparse_conv (src/hi3d_mac/mlx_backend/sparse.py:191-214) and the upstream
 * SubMConv3d (src/sparc3d/ops/sparse_backend.py:130-148): out[o] = bias + sum_k x[table[o, k]] W_k^T
 * (rows equal to n_in contribute zero), fp32 accumulation, output rounded once.
 * x [n_in, cin]; table [n_out, 27] from hi3d_neighbour_map_build; weight [cout, 27, cin]
 * (spconv's (out, 3, 3, 3, in) layout); bias [cout] or NULL; out [n_out, cout]; cin, cout % 8 == 0. */
HI3D_API int hi3d_sparse_conv(const void* x, const int32_t* table, const uint32_t* tap_mask, const void* weight,
                              const void* bias, void* out, int64_t n_in, int64_t n_out, int cin, int cout, int dtype,
                              void* stream);

/* hi3d_sparse_conv with an activation: act = 1 applies SiLU to the rounded output (fp32, rounded
 * again), the conv2 -> SiLU of the transformer's sparse res blocks
 * (src/hi3d_mac/mlx_backend/transformer.py:418-424; upstream sparc3d_transformer.py:142-143). */
HI3D_API int hi3d_sparse_conv_act(const void* x, const int32_t* table, const uint32_t* tap_mask, const void* weight,
                                  const void* bias, void* out, int64_t n_in, int64_t n_out, int cin, int cout, int act,
                                  int dtype, void* stream);

/* hi3d_layer_norm_modulate followed by hi3d_quantize_act_i8 (signed H64, `sign` [channels]) in one
 * pass: the input of a W8A8 projection that follows a norm (the block's QKV, cross-attention Q
 * and MLP-in projections, src/hi3d_mac/mlx_backend/transformer.py:543-588 with the w8a8 hook
 * :504-507).  q [rows, channels] int8 and qscale [rows] fp32 equal those of quantising the
 * rounded layer_norm_modulate output, which is never written.  channels % 64 == 0, <= 4096. */
HI3D_API int hi3d_layer_norm_quantize(const void* x, int8_t* q, float* qscale, int64_t rows, int64_t channels,
                                      float eps, const float* weight, const float* bias, const void* scale,
                                      const void* shift, int64_t rows_per_batch, int64_t mod_stride,
                                      const float* sign, int dtype, void* stream);

/* ---- sparse VAE decoder ---------------------------------------------------- */
/* Bytes of workspace hi3d_group_norm_stats needs. */
HI3D_API int hi3d_group_norm_stats_workspace_size(int64_t n, int64_t channels, int64_t* bytes);

/* Replaces SparconvVAEDecoderMLX.group_stats (src/hi3d_mac/mlx_backend/vae.py:142-164; upstream
 * PointGroupNorm): per-channel fp32 sums S1, S2 of x [n, channels] (f16 or f32), then per group of
 * channels / groups channels mean = S1 / (count + eps), var = S2 / (count + eps) - mean^2,
 * inv = 1 / sqrt(var + eps) with count = n * width; mean, inv [channels] (each group's values
 * repeated over its channels).  Deterministic (fixed summation order). */
HI3D_API int hi3d_group_norm_stats(const void* x, int64_t n, int64_t channels, int groups, float eps, float* mean,
                                   float* inv, void* workspace, int64_t workspace_bytes, int dtype, void* stream);

/* Replaces the normalise + swish part of kernels.gather_group_norm_swish
 * (src/hi3d_mac/mlx_backend/kernels.py:242-296): out = swish(u), u = (x - mean) * inv * weight + bias
 * in fp32, swish(u) = u * sigmoid(u) with sigmoid from e = 1 / (1 + exp(|u|)), rounded once to
 * out_dtype (f16 or f32).  The convolution then gathers `out` (hi3d_sparse_conv): the activated
 * features are written once instead of once per gathered neighbour. */
HI3D_API int hi3d_group_norm_swish(const void* x, int64_t n, int64_t channels, const float* mean, const float* inv,
                                   const float* weight, const float* bias, void* out, int in_dtype, int out_dtype,
                                   void* stream);

/* Bytes of workspace hi3d_child_structure / hi3d_child_table need for num_parents parents. */
HI3D_API int hi3d_child_table_workspace_size(int64_t num_parents, int64_t* bytes);

/* First half of sparse.child_neighbour_table (src/hi3d_mac/mlx_backend/sparse.py:64-95): from the
 * occupancy mask [num_parents, 8] (uint8, nonzero = kept) the kept children in parent-major,
 * slot-minor order: parent, slot [capacity >= 8 * num_parents] and *num_children (device int32).
 * Fills `workspace` with the child lookup hi3d_child_table reads. */
HI3D_API int hi3d_child_structure(const uint8_t* mask, int64_t num_parents, int32_t* parent, int32_t* slot,
                                  int32_t* num_children, void* workspace, int64_t workspace_bytes, void* stream);

/* Second half of sparse.child_neighbour_table (sparse.py:64-95, offsets :46-58): table [num_children, 27]
 * of the children from the parent table [num_parents, 27] (sentinel num_parents): the neighbour of
 * child (p, s) at offset k is child (parent_table[p][pk], s') with t = bits(s) + d_k,
 * pk = offset of floor(t / 2), s' = slot of t mod 2; absent -> num_children.  `workspace` as filled
 * by hi3d_child_structure. */
HI3D_API int hi3d_child_table(const int32_t* parent_table, int64_t num_parents, const int32_t* parent,
                              const int32_t* slot, int64_t num_children, const void* workspace, int32_t* table,
                              void* stream);

/* Bytes of workspace hi3d_serialize needs for n points. */
HI3D_API int hi3d_serialize_workspace_size(int64_t n, int64_t* bytes);

/* Replaces vae.serialization for one order (src/hi3d_mac/mlx_backend/vae.py:49-69; upstream
 * Point.serialization): Morton keys of coords [n, 3] with `depth` bits per axis (x -> key bit
 * 3i + 2, y -> 3i + 1, z -> 3i; swap_xy = 1 for the "z-trans" order), perm = the stable argsort of
 * the keys, inverse[perm[i]] = i. */
HI3D_API int hi3d_serialize(const int32_t* coords, int64_t n, int depth, int swap_xy, int32_t* perm,
                            int32_t* inverse, void* workspace, int64_t workspace_bytes, void* stream);

/* Replaces the windowed attention of SparconvVAEDecoderMLX.attention_block
 * (src/hi3d_mac/mlx_backend/vae.py:249-266, windows :72-88; upstream SerializedAttention): qkv
 * [n, 3, heads, head_dim] (f16 or f32); gather [n_pad] = the rows in padded window order
 * (window_index); each window of `window` rows attends within itself (softmax(q k^T * scale) v,
 * fp32), and the result of window position p < n is written to out[gather[p]] ([n, heads *
 * head_dim]).  n <= window: one window of all rows (n_pad = n).  head_dim 16, 32 or 64. */
HI3D_API int hi3d_window_attention(const void* qkv, const int32_t* gather, int64_t n, int64_t n_pad, int window,
                                   int heads, int head_dim, float scale, void* out, int dtype, void* stream);

/* ---- elementwise epilogues of the block --------------------------------- */
/* x <- x + y * gate (all in the I/O type, two roundings: round(y*gate), then round(x + .)).
 * Replaces the residual/gate expressions at src/hi3d_mac/mlx_backend/transformer.py:570,588
 * (upstream src/sparc3d/nn/sparse/transformer/modulated.py:59-65).
 * x, y [rows, channels]; gate [channels] per batch element (gate_stride apart), NULL = 1.
 * rows_per_batch maps rows to batch elements. */
HI3D_API int hi3d_gate_residual(void* x, const void* y, const void* gate, int64_t rows, int64_t channels,
                       int64_t rows_per_batch, int64_t gate_stride, int dtype, void* stream);

/* out = gelu_tanh(x) computed in fp32 and rounded once.
 * Replaces gelu_tanh, src/hi3d_mac/mlx_backend/transformer.py:176-179. */
HI3D_API int hi3d_gelu_tanh(const void* x, void* out, int64_t count, int dtype, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* HI3D_B200_H_ */

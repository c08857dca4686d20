/*
 * tilequant_b200 -- C ABI of the B200 (sm_100a) mixed-precision 64x64 tile GEMM path.
 *
 * Drop-in boundary for the reference's Triton path (HanzhiZhang-Ulrica/TileQuant,
 * src/kernels/triton/ and the torch paths of src/kernels/quant_utils.py and
 * src/kernels/pack.py).  Every entry point takes plain device pointers, element
 * strides and a cudaStream_t passed as void*; nothing here allocates device memory
 * except tq_peer_alloc (the exchange buffer of the tensor-parallel peer sum).
 * Kernel launches are asynchronous on `stream`.  The quantizer, GEMM (tq_gemm_mixed,
 * tq_gemm_mixed_fused_quant, tq_gemm_mixed_peer_sum), packer and calibration entry
 * points may be captured in a CUDA graph; the tq_peer_* set-up calls are synchronous
 * host calls, and this statement does not cover tq_gemm_mixed_peer_sum_noalloc.
 *
 * Return value: TQ_OK (0) or a TQ_ERR_* code; tq_last_error() gives a message for
 * the calling thread's last failure.  Shape/argument problems are detected on the
 * host before any launch.  Device-side waits are bounded: a wait that gives up
 * writes TQ_ERR_TIMEOUT into the optional `err` word (a device int the caller
 * zeroes and reads back) instead of hanging.
 *
 * Tile layout (the reference's Pack, src/kernels/pack.py:11-29, unchanged):
 *   tile id = r * n_tc + c for the 64x64 tile at output rows [64r, 64r+64) and input
 *   columns [64c, 64c+64) of the zero-padded weight W (M_pad x K_pad);
 *   int8_tiles  int8[T8][64][64], tile[i][j] = W[64r+i][64c+j] quantized;
 *   int8_scales f32[T8];  int8_tile_ids int32[T8] ascending;  int8_row_ptr int32[n_tr+1];
 *   fp16_tiles  bf16/f16[T16][64][64]; fp16_tile_ids int32[T16]; fp16_row_ptr int32[n_tr+1].
 */
#ifndef TILEQUANT_B200_H
#define TILEQUANT_B200_H

#include <stdint.h>

#if defined(__GNUC__)
#define TQ_API __attribute__((visibility("default")))
#else
#define TQ_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

enum {
  TQ_OK = 0,
  TQ_ERR_INVALID = 1,     /* bad shape / stride / dtype / alignment argument      */
  TQ_ERR_UNSUPPORTED = 2, /* valid request this build does not implement          */
  TQ_ERR_CUDA = 3,        /* a CUDA runtime call failed                           */
  TQ_ERR_TIMEOUT = 4      /* written to the device error word by a bounded wait   */
};

enum { TQ_DTYPE_BF16 = 0, TQ_DTYPE_F16 = 1 };

enum {
  TQ_ALGO_AUTO = 0,  /* pick by problem shape                                     */
  TQ_ALGO_ROWS = 1,  /* split-K row-owned kernel: bulk-copy weight stream, cluster
                        (DSMEM) split reduction; decode and general fallback      */
  TQ_ALGO_UMMA = 2,  /* persistent TMA + tcgen05 (kind::i8 / kind::f16) kernel    */
  TQ_ALGO_GEMV = 3,  /* decode kernel: operands straight into MMA fragments, split-K
                        across the warps of a CTA; chosen automatically for 9..16
                        rows when its grid fits one wave and each warp holds few
                        tiles, by name for up to 64 rows (16-row blocks); the form
                        the row-parallel peer sum uses                           */
  TQ_ALGO_STREAM = 4 /* decode kernel for <= 16 rows: one CTA per (split, row tile),
                        the splits of a row tile a cluster (DSMEM reduction), INT8
                        tiles in 16 KB bulk copies, activations resident in shared
                        memory; the automatic choice for <= 8 rows where it fits,
                        else the row kernel at the same split                    */
};

/* ABI version of this header (bumped on any signature change). */
TQ_API int tq_abi_version(void);

/* Message for the calling thread's last non-OK return. */
TQ_API const char* tq_last_error(void);

/* Static name of a status code. */
TQ_API const char* tq_status_string(int status);

/* Number of kernels this library has launched in the process so far (all devices,
 * all streams).  Lets a caller count the native launches of a region of work. */
TQ_API int64_t tq_kernel_launches(void);

/* ---------------------------------------------------------------- quantizer
 * x is (n_rows, k) of x_dtype with element strides (ld_row, ld_col).
 * sx[c] = f32(dtype(f32(absmax(x[:, 64c:64c+64])) / 127)), 1.0 for an all-zero
 * column tile; q = clamp(rint(f32(x) / sx[col/64]), -127, 127), contiguous rows of
 * stride ldq (>= k).
 */

/* replaces activation_tile_absmax_scales (src/kernels/quant_utils.py:41-74) and the
 * Triton _activation_tile_absmax_scales_64_kernel (triton/quantize_activation.py:13-44,
 * host :158-176). */
TQ_API int tq_act_scales(const void* x, int x_dtype, int64_t n_rows, int64_t k, int64_t ld_row, int64_t ld_col,
                  float* sx, void* stream);

/* replaces quantize_activation_tile_with_scales (src/kernels/quant_utils.py:78-115) and
 * _quantize_activation_with_scales_64_kernel (triton/quantize_activation.py:47-74,
 * host :179-203). */
TQ_API int tq_quantize_with_scales(const void* x, int x_dtype, int64_t n_rows, int64_t k, int64_t ld_row,
                            int64_t ld_col, const float* sx, int8_t* q, int64_t ldq, void* stream);

/* replaces quantize_activation_tile_absmax (src/kernels/quant_utils.py:119-134) and the
 * one-pass _quantize_activation_64_kernel (triton/quantize_activation.py:77-112,
 * host :118-155); any n_rows. */
TQ_API int tq_quantize_act(const void* x, int x_dtype, int64_t n_rows, int64_t k, int64_t ld_row, int64_t ld_col,
                    int8_t* q, int64_t ldq, float* sx, void* stream);

/* ---------------------------------------------------------------- mixed GEMM
 * out[n, o] for n < n_rows, o < m (out features), k in features:
 *   per row tile r and split s (of split_k), INT8 tiles in ascending column order:
 *     acc = acc + f32(i32 tile dot) * (sx[c] * sw[t])
 *   (the row kernel rounds the multiply and the add separately, as the reference's
 *   kernel does under the Triton interpreter; the tcgen05 kernel fuses them, as
 *   compiled Triton does; the two differ by at most 1 ulp of the output dtype)
 *   then BF16/F16 tiles: acc += f32 dot(x_fp tile, W tile);
 *   split partials summed in split order; out = dtype(acc); with bias:
 *   out = dtype(f32(out) + f32(bias[o])).
 * x_i8 (n_rows, k) row stride ld_x8 bytes; x_fp (n_rows, k) of fp_dtype (the dtype of
 * the 16-bit tiles too), row stride ld_xfp elements (may be NULL when t16 == 0);
 * out (n_rows, m) of out_dtype, row stride ldo; bias (m) of out_dtype or NULL.
 * split_k: 0 = automatic, else 1..16 (the result depends on split_k exactly as the
 * reference's does).  algo: TQ_ALGO_*.  err: optional device error word.
 *
 * replaces gemm_mixed_rows_splitk / _gemm_mixed_rows_splitk_kernel
 * (src/kernels/triton/gemm_rows_splitk_64x64.py:78-190, host :225-323).
 */
TQ_API int tq_gemm_mixed(const int8_t* x_i8, int64_t ld_x8, const float* sx, const int8_t* int8_tiles,
                  const float* int8_scales, const int32_t* int8_tile_ids, const int32_t* int8_row_ptr,
                  int64_t t8, const void* x_fp, int64_t ld_xfp, const void* fp16_tiles,
                  const int32_t* fp16_tile_ids, const int32_t* fp16_row_ptr, int64_t t16, int fp_dtype,
                  void* out, int64_t ldo, int out_dtype, const void* bias, int64_t n_rows, int64_t m, int64_t k,
                  int n_tr, int n_tc, int split_k, int algo, int* err, void* stream);

/* Decode form with the activation quantizer fused into the GEMM prologue: the same
 * result as tq_quantize_act followed by tq_gemm_mixed, in one launch.  n_rows <= 64; up
 * to 8 rows it runs the stream kernel, whose splits each quantize their own columns.
 * replaces quantize_activation_tile_absmax + gemm_mixed_rows_splitk as called by
 * MixedLinear.forward for small row counts (src/models/mixed_linear.py:232-239). */
TQ_API int tq_gemm_mixed_fused_quant(const void* x_fp, int64_t ld_xfp, int fp_dtype, const int8_t* int8_tiles,
                              const float* int8_scales, const int32_t* int8_tile_ids,
                              const int32_t* int8_row_ptr, int64_t t8, const void* fp16_tiles,
                              const int32_t* fp16_tile_ids, const int32_t* fp16_row_ptr, int64_t t16,
                              void* out, int64_t ldo, int out_dtype, const void* bias, int64_t n_rows, int64_t m,
                              int64_t k, int n_tr, int n_tc, int split_k, int* err, void* stream);

/* Launch geometry the decode kernels use when split_k = 0 on this device: *split
 * (1..16) and *rows_per_cta (row tiles one CTA streams when split is 1).
 * Up to 8 rows (with or without fused quantization) this is the split of TQ_ALGO_STREAM:
 * the most splits (at most 8, at least 4 INT8 tiles each) whose n_tr clusters of split
 * CTAs are all resident on this device at once, 1 if none is; the automatic choice also
 * gives it to the row kernel when the stream kernel cannot take a call.  For 9..16 rows
 * it is the split of TQ_ALGO_GEMV where the automatic choice takes that kernel (its grid
 * fits one wave and each warp holds few tiles).  Otherwise the split of the row kernel
 * (TQ_ALGO_ROWS).
 * The split fixes the FP32 summation order of the result; passing it back as split_k
 * reproduces the same result.  (The reference picks its split from a fixed rule,
 * select_split_k, gemm_rows_splitk_64x64.py:52-67; this one sizes the grid to one
 * wave of resident CTAs on the B200.) */
TQ_API int tq_gemm_rows_plan(int64_t n_rows, int n_tr, int n_tc, int fp_dtype, int fused, int* split,
                             int* rows_per_cta);

/* Debug: the exact INT32 tile products the GEMM kernels form, partials[t][n][j] =
 * sum_k x_i8[n, 64c+k] * int8_tiles[t][j][k] for every INT8 tile t (int32[t8][n_rows][64]).
 * The reference computes the same value inside its kernel (gemm_rows_splitk_64x64.py:134)
 * without exposing it. */
TQ_API int tq_gemm_int8_partials(const int8_t* x_i8, int64_t ld_x8, const int8_t* int8_tiles,
                          const int32_t* int8_tile_ids, const int32_t* int8_row_ptr, int64_t t8,
                          int64_t n_rows, int64_t k, int n_tr, int n_tc, int32_t* partials, int algo,
                          void* stream);

/* ---------------------------------------------------------------- packer
 * W (m, k) of w_dtype, row stride ldw elements, zero padded to (64 n_tr, 64 n_tc).
 */

/* INT8 codes and scales of the tiles `ids` (sorted): scale = f32(absmax)/127 (1.0 for
 * an all-zero tile); with col_importance (f32[64 n_tc], may be NULL) the IAA search
 * over {0.75, 1.0, 1.25} x scale by importance-weighted squared error, first best kept.
 * replaces src/kernels/pack.py:119-167 (inside _pack_weight_with_tile_ids :65-203). */
TQ_API int tq_pack_int8_tiles(const void* w, int w_dtype, int64_t m, int64_t k, int64_t ldw, int n_tc,
                       const int32_t* ids, int64_t t8, const float* col_importance, int8_t* tiles,
                       float* scales, void* stream);

/* Gather the 16-bit tiles `ids` unchanged (zero padded).  replaces pack.py:172-177. */
TQ_API int tq_gather_fp_tiles(const void* w, int w_dtype, int64_t m, int64_t k, int64_t ldw, int n_tc,
                       const int32_t* ids, int64_t t16, void* tiles, void* stream);

/* ---------------------------------------------------------------- tensor-parallel peer sum
 * No counterpart in the reference, which runs on one GPU: for a row-parallel projection
 * (K split across the ranks of one node, one process per GPU) the decode GEMM sums the
 * ranks' partial outputs itself, over NVLink, instead of a separate all-reduce after
 * it.  Each rank allocates one exchange buffer, exports it (tq_peer_ipc_handle), maps
 * every peer's (tq_peer_ipc_open) and passes the device array of the world pointers
 * (its own at index rank) plus its per-CTA call counters (uint32[slots], zeroed once). */

#define TQ_PEER_MAX_WORLD 8
#define TQ_PEER_MAX_SLOTS 65536
#define TQ_IPC_HANDLE_BYTES 64

/* Bytes of one exchange buffer for `world` ranks and `slots` CTA slots (0 if out of range). */
TQ_API int64_t tq_peer_buffer_bytes(int world, int slots);

/* cudaMalloc'd, zeroed exchange buffer on the current device; tq_peer_free releases it. */
TQ_API int tq_peer_alloc(int world, int slots, void** buf);
TQ_API int tq_peer_free(void* buf);

/* The buffer's CUDA IPC handle (TQ_IPC_HANDLE_BYTES bytes) and its mapping in another
 * process on another GPU of the node; tq_peer_ipc_close unmaps. */
TQ_API int tq_peer_ipc_handle(void* buf, void* handle);
TQ_API int tq_peer_ipc_open(const void* handle, void** buf);
TQ_API int tq_peer_ipc_close(void* buf);

/* Zero the buffer and the counters (stream-ordered).  Every rank must reset before any
 * rank's next peer-sum call, e.g. after a timeout. */
TQ_API int tq_peer_reset(void* buf, int world, int slots, uint32_t* epochs, void* stream);

/* tq_gemm_mixed on the decode kernel (1..64 rows as 16-row blocks, split_k 0..8) for this
 * rank's K slice, with the world ranks' FP32 partials summed in rank order 0..world-1
 * inside the kernel before the output rounding and the bias: every rank gets the same
 * (n_rows, m) output.
 * Every rank must make the same sequence of calls (same n_rows, m, n_tr).  Needs
 * 4 * n_tr * ceil(n_rows / 16) <= slots and all those CTAs resident at once (else
 * TQ_ERR_UNSUPPORTED).
 * A wait for a peer that exceeds timeout_ns writes TQ_ERR_TIMEOUT to `err` and the
 * output is then undefined; reset the exchange on every rank before going on. */
TQ_API int tq_gemm_mixed_peer_sum(const int8_t* x_i8, int64_t ld_x8, const float* sx, const int8_t* int8_tiles,
                                  const float* int8_scales, const int32_t* int8_tile_ids,
                                  const int32_t* int8_row_ptr, int64_t t8, const void* x_fp, int64_t ld_xfp,
                                  const void* fp16_tiles, const int32_t* fp16_tile_ids,
                                  const int32_t* fp16_row_ptr, int64_t t16, int fp_dtype, void* out, int64_t ldo,
                                  int out_dtype, const void* bias, int64_t n_rows, int64_t m, int64_t k, int n_tr,
                                  int n_tc, int split_k, float* const* peer_bufs, uint32_t* epochs, int world,
                                  int rank, int slots, int64_t timeout_ns, int* err, void* stream);

/* No counterpart in the reference.  tq_gemm_mixed_peer_sum for callers that cannot call
 * cudaMalloc: serving runtimes that give all free device memory to their own pools at
 * start-up, and real-time host loops that cannot take the device synchronization an
 * allocation may cause.  Nothing is allocated: the exchange words, call counters and
 * exchange-address table live in one file-scope __device__ array of
 * TQ_NOALLOC_SCRATCH_BYTES (about 4 MB) that every GPU loading the library holds until
 * the process exits.  A world of one GPU (the current device): that array cannot be
 * reached from other GPUs, so sums across GPUs need tq_peer_alloc's buffers.  Limits,
 * checked before anything runs: more than 16 rows returns TQ_ERR_UNSUPPORTED (not a
 * decode call), m > 16384 (more than 256 row tiles, beyond the array's 1024 CTA slots)
 * returns TQ_ERR_INVALID.  Every call looks up the array's address; the first call on a
 * device writes the array's table with a synchronous copy, so make it before any stream
 * capture.  Every call shares the array, which keeps the last call's state (the call
 * counters advance; each call's words carry its number, so nothing needs clearing
 * between calls): calls whose kernels overlap on the GPU race.  reset_only != 0 zeroes
 * the counters and words and rewrites the table (stream-ordered, no launch): use it
 * after a timeout, and after a cudaDeviceReset before the next call.  Otherwise the
 * contract and the result of tq_gemm_mixed_peer_sum with world 1 (the same bits as
 * tq_gemm_mixed on the decode kernel). */
#define TQ_NOALLOC_SLOTS 1024
#define TQ_NOALLOC_SCRATCH_BYTES 4198656
TQ_API int tq_gemm_mixed_peer_sum_noalloc(const int8_t* x_i8, int64_t ld_x8, const float* sx,
                                          const int8_t* int8_tiles, const float* int8_scales,
                                          const int32_t* int8_tile_ids, const int32_t* int8_row_ptr, int64_t t8,
                                          const void* x_fp, int64_t ld_xfp, const void* fp16_tiles,
                                          const int32_t* fp16_tile_ids, const int32_t* fp16_row_ptr, int64_t t16,
                                          int fp_dtype, void* out, int64_t ldo, int out_dtype, const void* bias,
                                          int64_t n_rows, int64_t m, int64_t k, int n_tr, int n_tc, int split_k,
                                          int64_t timeout_ns, int reset_only, int* err, void* stream);

/* ---------------------------------------------------------------- decode step
 *
 * The non-GEMM work of one greedy decode step of a Llama/Qwen2 decoder layer, fused.
 * The reference runs these as torch operators inside its CUDA graph
 * (src/runtime/graph_decode.py:172-214, the decoder layers of transformers) and its
 * decode attention as aten._flash_attention_forward with seqused_k
 * (src/runtime/graph_decode.py:58-70).  16-bit tensors are bf16 or f16 (dtype). */

/* resid_out = resid + delta (16-bit; delta may be NULL: no add, resid_out unused),
 * y = weight * round16(h * rsqrt(mean(h^2) + eps)) per row: the decoder layer's
 * residual add and RMSNorm (f32 statistics).  resid_out may alias resid.  hidden is a
 * multiple of 8 up to 16384; every row starts on a 16-byte boundary. */
TQ_API int tq_add_rmsnorm(const void* resid, int64_t ld_r, const void* delta, int64_t ld_d, const void* weight,
                          void* resid_out, int64_t ld_ro, void* y, int64_t ld_y, int64_t n_rows, int64_t hidden,
                          float eps, int dtype, void* stream);

/* h = round16(round16(silu(gate)) * up) for n_rows <= 128 rows of k columns (gate and
 * up share the row stride ld_gu), then h's INT8 codes q and per-64-column scales sx
 * exactly as tq_quantize_act makes them. */
TQ_API int tq_silu_mul_quant(const void* gate, const void* up, int64_t ld_gu, int64_t n_rows, int64_t k, void* h,
                             int64_t ld_h, int8_t* q, int64_t ldq, float* sx, int dtype, void* stream);

/* One query token per sequence against a head-major KV cache [B][Hkv][L][D]
 * (16-byte aligned, contiguous).  q/k/v: the projections' outputs for the token (row
 * b, head h at + b * ld + h * D; every row, and cos/sin, on 16-byte boundaries).  The
 * kernel applies RoPE (cos/sin: D values of the
 * current position) to q and k, writes the rotated k and v into cache slot *pos, and
 * attends over slots [0, *pos] in S splits (ws_*: f32 scratch of B*Hq*S, B*Hq*S,
 * B*Hq*S*D); *pos is read on the device, so one launch serves every step of a graph. */
typedef struct tq_attn_args {
  const void* q;
  const void* k;
  const void* v;
  const void* cos;
  const void* sin;
  void* k_cache;
  void* v_cache;
  const int64_t* pos;
  float* ws_m;
  float* ws_l;
  float* ws_o;
  int* err; /* TQ_ERR_TIMEOUT when a TMA load never lands (NULL: not reported) */
  int64_t ld_q, ld_k, ld_v;
  int B, Hq, Hkv, D, L, S;
  float scale_log2; /* softmax scale * log2(e) */
  int reserved;
} tq_attn_args;

/* Splits tq_attn_decode should use for this shape on this device: as many as keep every
 * CTA resident at once (two per SM). */
TQ_API int tq_attn_decode_splits(int batch, int kv_heads, int max_len);

/* out[b, h*D + d] = softmax(q_h k^T * scale) v (16-bit); with q_out, also its INT8 codes
 * and per-64-column scales sx, as tq_quantize_act would make them from out. */
TQ_API int tq_attn_decode(const tq_attn_args* args, void* out, int64_t ld_out, int8_t* q_out, int64_t ldq, float* sx,
                          int dtype, void* stream);

/* Greedy pick of a decode step: next[b] = token[b] = argmax of logits row b (the first
 * index of the maximum, as torch.argmax), generated[b, *position - prompt_tokens + 1] =
 * that id (skipped outside 0..gen_cols-1), then *position += 1 -- the bookkeeping of the
 * reference's decode body (src/runtime/graph_decode.py:428-452).  keys: n_rows uint64 of
 * scratch, zero before the first call; each call leaves them zero.  next, token and
 * generated may be NULL. */
TQ_API int tq_greedy_pick(const void* logits, int64_t ld, int64_t n_rows, int64_t vocab, int dtype,
                          unsigned long long* keys, int64_t* next, int64_t* token, int64_t* generated,
                          int64_t gen_ld, int64_t gen_cols, int64_t* position, int64_t prompt_tokens, void* stream);

/* ---------------------------------------------------------------- calibration */

/* tile_scores[r, c] += sum over the tile of |f32(W) * f32(G)| (f32 [n_tr][n_tc]).
 * replaces the GI reduction of collect_gi_tile_scores (src/kernels/calibrate.py:153-164). */
TQ_API int tq_calib_gi_accumulate(const void* w, const void* g, int dtype, int64_t m, int64_t k, int64_t ldw,
                           int64_t ldg, int n_tr, int n_tc, float* tile_scores, void* stream);

/* act_sum[j] += sum over rows of |f32(x[i, j])| accumulated in f64.
 * replaces the IAA forward pre-hook (src/kernels/calibrate.py:244-255). */
TQ_API int tq_calib_iaa_channel_accumulate(const void* x, int dtype, int64_t rows, int64_t k, int64_t ld_row,
                                    double* act_sum, void* stream);

/* mean[j] = f32(act_sum[j] / count); tile_scores[r, c] = sum over the tile of
 * |f32(W)| * mean[col] (f32 [n_tr][n_tc]).
 * replaces src/kernels/calibrate.py:346-367. */
TQ_API int tq_calib_iaa_tile_scores(const void* w, int dtype, int64_t m, int64_t k, int64_t ldw,
                             const double* act_sum, int64_t count, float* mean, float* tile_scores,
                             void* stream);

#ifdef __cplusplus
}
#endif

#endif /* TILEQUANT_B200_H */

// C-ABI entry points of the mixed tile GEMM: argument checks and kernel dispatch.
#include <algorithm>

#include "common.cuh"
#include "gemm_args.cuh"

int tq_launch_rows(tq::RowsArgs& a, int n_tr, int fp_dtype, cudaStream_t st, int64_t t16);
int tq_umma_supported(int64_t n_rows, int64_t m, int64_t k, const int8_t* x_i8, int64_t ld_x8, const void* x_fp,
                      int64_t ld_xfp, const void* w8, const void* w16);
int tq_launch_umma(const tq::RowsArgs& a, int n_tr, int fp_dtype, cudaStream_t st);
int tq_gemv_supported(const tq::RowsArgs& a);
int tq_gemv_peer_supported(const tq::RowsArgs& a);
int tq_gemv_preferred(const tq::RowsArgs& a, int n_tr);
int tq_launch_gemv(tq::RowsArgs& a, int n_tr, int fp_dtype, cudaStream_t st);
int tq_stream_split(int n_tr, int n_tc, int n_rows);
int tq_stream_supported(const tq::RowsArgs& a);
int tq_launch_stream(tq::RowsArgs& a, int n_tr, int fp_dtype, cudaStream_t st);

static bool aligned16(const void* p) { return ((uintptr_t)p & 15) == 0; }

static int check_pack(const int8_t* w8, const float* s8, const int32_t* ids8, const int32_t* rp8, int64_t t8,
                      const void* w16, const int32_t* ids16, const int32_t* rp16, int64_t t16, int64_t m, int64_t k,
                      int n_tr, int n_tc) {
  if (m <= 0 || k <= 0) return tq_set_error(TQ_ERR_INVALID, "m and k must be positive");
  if (n_tr != (m + 63) / 64 || n_tc != (k + 63) / 64)
    return tq_set_error(TQ_ERR_INVALID, "tile grid (n_tr, n_tc) does not match (m, k)");
  if (t8 < 0 || t16 < 0 || t8 + t16 != (int64_t)n_tr * n_tc)
    return tq_set_error(TQ_ERR_INVALID, "t8 + t16 must equal n_tr * n_tc");
  if (!rp8) return tq_set_error(TQ_ERR_INVALID, "null int8_row_ptr");
  if (t8 > 0 && (!w8 || !s8 || !ids8)) return tq_set_error(TQ_ERR_INVALID, "null INT8 tile arrays");
  if (t16 > 0 && (!w16 || !ids16 || !rp16)) return tq_set_error(TQ_ERR_INVALID, "null 16-bit tile arrays");
  if ((t8 > 0 && !aligned16(w8)) || (t16 > 0 && !aligned16(w16)))
    return tq_set_error(TQ_ERR_INVALID, "tile arenas must be 16-byte aligned");
  return TQ_OK;
}

// Validates the operands of a mixed GEMM and fills the kernel arguments.
static int gemm_args(tq::RowsArgs& a, const int8_t* x_i8, int64_t ld_x8, const float* sx, const int8_t* int8_tiles,
                     const float* int8_scales, const int32_t* int8_tile_ids, const int32_t* int8_row_ptr, int64_t t8,
                     const void* x_fp, int64_t ld_xfp, const void* fp16_tiles, const int32_t* fp16_tile_ids,
                     const int32_t* fp16_row_ptr, int64_t t16, int fp_dtype, void* out, int64_t ldo, int out_dtype,
                     const void* bias, int64_t n_rows, int64_t m, int64_t k, int n_tr, int n_tc, int split_k, int* err) {
  int rc = check_pack(int8_tiles, int8_scales, int8_tile_ids, int8_row_ptr, t8, fp16_tiles, fp16_tile_ids,
                      fp16_row_ptr, t16, m, k, n_tr, n_tc);
  if (rc) return rc;
  if (fp_dtype != TQ_DTYPE_BF16 && fp_dtype != TQ_DTYPE_F16) return tq_set_error(TQ_ERR_INVALID, "bad fp dtype");
  if (out_dtype != TQ_DTYPE_BF16 && out_dtype != TQ_DTYPE_F16) return tq_set_error(TQ_ERR_INVALID, "bad out dtype");
  if (n_rows < 0) return tq_set_error(TQ_ERR_INVALID, "negative n_rows");
  if (n_rows > INT32_MAX / 2) return tq_set_error(TQ_ERR_INVALID, "n_rows too large");
  if (n_rows > 0 && (!out || ldo < m)) return tq_set_error(TQ_ERR_INVALID, "out must be (n_rows, m) with row stride >= m");
  if (n_rows > 0 && t8 > 0 && (!x_i8 || !sx || ld_x8 < k)) return tq_set_error(TQ_ERR_INVALID, "x_int8 must be (n_rows, k)");
  if (n_rows > 0 && t16 > 0 && (!x_fp || ld_xfp < k)) return tq_set_error(TQ_ERR_INVALID, "x_fp must be (n_rows, k)");
  if (split_k < 0 || split_k > 16) return tq_set_error(TQ_ERR_INVALID, "split_k must be 0 (auto) or 1..16");
  a = tq::RowsArgs{};
  a.x_i8 = x_i8;
  a.ld_x8 = ld_x8;
  a.sx = sx;
  a.w8 = int8_tiles;
  a.s8 = int8_scales;
  a.ids8 = int8_tile_ids;
  a.rp8 = int8_row_ptr;
  a.x_fp = x_fp;
  a.ld_xfp = ld_xfp;
  a.w16 = fp16_tiles;
  a.ids16 = fp16_tile_ids;
  a.rp16 = fp16_row_ptr;
  a.out = out;
  a.ldo = ldo;
  a.out_dtype = out_dtype;
  a.bias = bias;
  a.err = err;
  a.n_rows = (int)n_rows;
  a.M = (int)m;
  a.K = (int)k;
  a.n_tc = n_tc;
  a.split = split_k;
  a.has_fp16 = t16 > 0;
  a.w8_rows = t8 * 64;
  a.w16_rows = t16 * 64;
  return TQ_OK;
}

extern "C" int tq_gemm_mixed(const int8_t* x_i8, int64_t ld_x8, const float* sx, const int8_t* int8_tiles,
                             const float* int8_scales, const int32_t* int8_tile_ids, const int32_t* int8_row_ptr,
                             int64_t t8, const void* x_fp, int64_t ld_xfp, const void* fp16_tiles,
                             const int32_t* fp16_tile_ids, const int32_t* fp16_row_ptr, int64_t t16, int fp_dtype,
                             void* out, int64_t ldo, int out_dtype, const void* bias, int64_t n_rows, int64_t m,
                             int64_t k, int n_tr, int n_tc, int split_k, int algo, int* err, void* stream) {
  tq::RowsArgs a;
  int rc = gemm_args(a, x_i8, ld_x8, sx, int8_tiles, int8_scales, int8_tile_ids, int8_row_ptr, t8, x_fp, ld_xfp,
                     fp16_tiles, fp16_tile_ids, fp16_row_ptr, t16, fp_dtype, out, ldo, out_dtype, bias, n_rows, m, k,
                     n_tr, n_tc, split_k, err);
  if (rc) return rc;
  if (n_rows == 0) return TQ_OK;
  cudaStream_t st = (cudaStream_t)stream;
  if (algo == TQ_ALGO_UMMA || (algo == TQ_ALGO_AUTO && n_rows > 64 && t8 > 0 &&
                               tq_umma_supported(n_rows, m, k, x_i8, ld_x8, x_fp, ld_xfp, int8_tiles, fp16_tiles))) {
    if (!tq_umma_supported(n_rows, m, k, x_i8, ld_x8, x_fp, ld_xfp, int8_tiles, fp16_tiles))
      return tq_set_error(TQ_ERR_UNSUPPORTED, "tcgen05 GEMM: unsupported shape or alignment");
    return tq_launch_umma(a, n_tr, fp_dtype, st);
  }
  if (algo == TQ_ALGO_STREAM || (algo == TQ_ALGO_AUTO && n_rows <= 8)) {
    // decode up to 8 rows: the stream kernel at its split; where it cannot take the call
    // (alignment, shared memory), the row kernel at the same split gives the same bits
    if (a.split == 0) a.split = tq_stream_split(n_tr, n_tc, (int)n_rows);
    if (tq_stream_supported(a)) return tq_launch_stream(a, n_tr, fp_dtype, st);
    if (algo == TQ_ALGO_STREAM) return tq_set_error(TQ_ERR_UNSUPPORTED, "stream decode kernel: unsupported call");
    return tq_launch_rows(a, n_tr, fp_dtype, st, t16);
  }
  if (algo == TQ_ALGO_GEMV || (algo == TQ_ALGO_AUTO && tq_gemv_preferred(a, n_tr))) {
    // asked for by name, the decode kernel also runs 17..64 rows as 16-row blocks
    if (!tq_gemv_peer_supported(a))
      return tq_set_error(TQ_ERR_UNSUPPORTED, "decode kernel: needs <= 64 rows and split_k <= 8");
    return tq_launch_gemv(a, n_tr, fp_dtype, st);
  }
  if (algo != TQ_ALGO_AUTO && algo != TQ_ALGO_ROWS) return tq_set_error(TQ_ERR_INVALID, "unknown algo");
  return tq_launch_rows(a, n_tr, fp_dtype, st, t16);
}

extern "C" int tq_gemm_mixed_peer_sum(const int8_t* x_i8, int64_t ld_x8, const float* sx, const int8_t* int8_tiles,
                                      const float* int8_scales, const int32_t* int8_tile_ids,
                                      const int32_t* int8_row_ptr, int64_t t8, const void* x_fp, int64_t ld_xfp,
                                      const void* fp16_tiles, const int32_t* fp16_tile_ids,
                                      const int32_t* fp16_row_ptr, int64_t t16, int fp_dtype, void* out, int64_t ldo,
                                      int out_dtype, const void* bias, int64_t n_rows, int64_t m, int64_t k, int n_tr,
                                      int n_tc, int split_k, float* const* peer_bufs, uint32_t* epochs, int world,
                                      int rank, int slots, int64_t timeout_ns, int* err, void* stream) {
  tq::RowsArgs a;
  int rc = gemm_args(a, x_i8, ld_x8, sx, int8_tiles, int8_scales, int8_tile_ids, int8_row_ptr, t8, x_fp, ld_xfp,
                     fp16_tiles, fp16_tile_ids, fp16_row_ptr, t16, fp_dtype, out, ldo, out_dtype, bias, n_rows, m, k,
                     n_tr, n_tc, split_k, err);
  if (rc) return rc;
  if (world < 1 || world > TQ_PEER_MAX_WORLD || rank < 0 || rank >= world)
    return tq_set_error(TQ_ERR_INVALID, "peer sum: need 1 <= world <= 8 and 0 <= rank < world");
  if (!peer_bufs || !epochs || slots < 1 || timeout_ns <= 0)
    return tq_set_error(TQ_ERR_INVALID, "peer sum: exchange buffers, counters, slots and timeout are required");
  if (n_rows == 0) return TQ_OK;  // every rank sees the same n_rows, so all skip together
  if (!tq_gemv_peer_supported(a)) return tq_set_error(TQ_ERR_UNSUPPORTED, "peer sum: needs 1..64 rows and split_k <= 8");
  a.peer_bufs = peer_bufs;
  a.peer_epochs = epochs;
  a.world = world;
  a.rank = rank;
  a.peer_slots = slots;
  a.peer_timeout_ns = timeout_ns;
  return tq_launch_gemv(a, n_tr, fp_dtype, (cudaStream_t)stream);
}

extern "C" int tq_gemm_mixed_fused_quant(const void* x_fp, int64_t ld_xfp, int fp_dtype, const int8_t* int8_tiles,
                                         const float* int8_scales, const int32_t* int8_tile_ids,
                                         const int32_t* int8_row_ptr, int64_t t8, const void* fp16_tiles,
                                         const int32_t* fp16_tile_ids, const int32_t* fp16_row_ptr, int64_t t16,
                                         void* out, int64_t ldo, int out_dtype, const void* bias, int64_t n_rows,
                                         int64_t m, int64_t k, int n_tr, int n_tc, int split_k, int* err,
                                         void* stream) {
  int rc = check_pack(int8_tiles, int8_scales, int8_tile_ids, int8_row_ptr, t8, fp16_tiles, fp16_tile_ids,
                      fp16_row_ptr, t16, m, k, n_tr, n_tc);
  if (rc) return rc;
  if (fp_dtype != TQ_DTYPE_BF16 && fp_dtype != TQ_DTYPE_F16) return tq_set_error(TQ_ERR_INVALID, "bad fp dtype");
  if (out_dtype != TQ_DTYPE_BF16 && out_dtype != TQ_DTYPE_F16) return tq_set_error(TQ_ERR_INVALID, "bad out dtype");
  if (n_rows < 0 || n_rows > 64) return tq_set_error(TQ_ERR_INVALID, "fused quantization needs 0 <= n_rows <= 64");
  if (n_rows == 0) return TQ_OK;
  if (!out || ldo < m) return tq_set_error(TQ_ERR_INVALID, "out must be (n_rows, m) with row stride >= m");
  if (!x_fp || ld_xfp < k) return tq_set_error(TQ_ERR_INVALID, "x_fp must be (n_rows, k)");
  if (split_k < 0 || split_k > 16) return tq_set_error(TQ_ERR_INVALID, "split_k must be 0 (auto) or 1..16");
  tq::RowsArgs a = {};
  a.w8 = int8_tiles;
  a.s8 = int8_scales;
  a.ids8 = int8_tile_ids;
  a.rp8 = int8_row_ptr;
  a.x_fp = x_fp;
  a.ld_xfp = ld_xfp;
  a.w16 = fp16_tiles;
  a.ids16 = fp16_tile_ids;
  a.rp16 = fp16_row_ptr;
  a.out = out;
  a.ldo = ldo;
  a.out_dtype = out_dtype;
  a.bias = bias;
  a.err = err;
  a.n_rows = (int)n_rows;
  a.M = (int)m;
  a.K = (int)k;
  a.n_tc = n_tc;
  a.split = split_k;
  a.has_fp16 = t16 > 0;
  a.fused = 1;
  a.w8_rows = t8 * 64;
  a.w16_rows = t16 * 64;
  if (n_rows <= 8) {  // decode: the stream kernel quantizes in its prologue; else the row kernel at its split
    if (a.split == 0) a.split = tq_stream_split(n_tr, n_tc, (int)n_rows);
    if (tq_stream_supported(a)) return tq_launch_stream(a, n_tr, fp_dtype, (cudaStream_t)stream);
  }
  return tq_launch_rows(a, n_tr, fp_dtype, (cudaStream_t)stream, t16);
}

extern "C" int tq_gemm_int8_partials(const int8_t* x_i8, int64_t ld_x8, const int8_t* int8_tiles,
                                     const int32_t* int8_tile_ids, const int32_t* int8_row_ptr, int64_t t8,
                                     int64_t n_rows, int64_t k, int n_tr, int n_tc, int32_t* partials, int algo,
                                     void* stream) {
  if (k <= 0 || n_tc != (k + 63) / 64 || n_tr <= 0) return tq_set_error(TQ_ERR_INVALID, "bad tile grid");
  if (t8 < 0 || (t8 > 0 && (!int8_tiles || !int8_tile_ids || !int8_row_ptr || !partials)))
    return tq_set_error(TQ_ERR_INVALID, "null INT8 arrays");
  if (t8 > 0 && !aligned16(int8_tiles)) return tq_set_error(TQ_ERR_INVALID, "tile arena must be 16-byte aligned");
  if (n_rows < 0 || (n_rows > 0 && (!x_i8 || ld_x8 < k))) return tq_set_error(TQ_ERR_INVALID, "bad x_int8");
  if (n_rows == 0 || t8 == 0) return TQ_OK;
  tq::RowsArgs a = {};
  a.x_i8 = x_i8;
  a.ld_x8 = ld_x8;
  a.w8 = int8_tiles;
  a.ids8 = int8_tile_ids;
  a.rp8 = int8_row_ptr;
  a.partials = partials;
  a.w8_rows = t8 * 64;
  a.n_rows = (int)n_rows;
  a.M = n_tr * 64;
  a.K = (int)k;
  a.n_tc = n_tc;
  a.split = 1;
  if (algo == TQ_ALGO_UMMA) {
    if (!tq_umma_supported(n_rows, (int64_t)n_tr * 64, k, x_i8, ld_x8, nullptr, 0, int8_tiles, nullptr))
      return tq_set_error(TQ_ERR_UNSUPPORTED, "tcgen05 GEMM: unsupported shape or alignment");
    return tq_launch_umma(a, n_tr, TQ_DTYPE_BF16, (cudaStream_t)stream);
  }
  return tq_launch_rows(a, n_tr, TQ_DTYPE_BF16, (cudaStream_t)stream, 0);
}

/*
 * TEST INFRASTRUCTURE ONLY -- the CPU oracle for the TileQuant mixed 64x64 tile
 * GEMM path.  Only tests/, __graft_entry__.smoke() and bench.py's cpu_baseline /
 * reference arm may load this library, and only as the checker (or the timed CPU
 * baseline).  The product path (tilequant_b200/) never calls it.
 *
 * Plain C restatement of the reference algorithm (HanzhiZhang-Ulrica/TileQuant):
 *   activation scales   src/kernels/quant_utils.py:41-74,
 *                       src/kernels/triton/quantize_activation.py:13-44
 *   activation codes    src/kernels/quant_utils.py:78-115,
 *                       src/kernels/triton/quantize_activation.py:47-74
 *   weight packer       src/kernels/pack.py:65-203 (GI absmax and IAA search)
 *   mixed GEMM          src/kernels/triton/gemm_rows_splitk_64x64.py:78-190
 *   GI tile scores      src/kernels/calibrate.py:153-164
 *   IAA channel sums    src/kernels/calibrate.py:244-255
 *   IAA tile scores     src/kernels/calibrate.py:346-367
 *
 * Parity of this restatement is pinned against fixtures produced by running the
 * reference itself (tests/golden/make_golden.py).
 *
 * 16-bit float inputs are passed as raw uint16 bit patterns; dtype 0 = bfloat16,
 * dtype 1 = float16.  Strides are in elements.
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

#define TQO_BF16 0
#define TQO_F16 1

/* Threads of the OpenMP loops of the calling thread (n > 0 sets them, whatever
 * OMP_NUM_THREADS the process inherited; n <= 0 leaves them); returns the count the
 * next parallel loop will use. */
int tqo_set_threads(int n) {
#ifdef _OPENMP
  if (n > 0) omp_set_num_threads(n);
  return omp_get_max_threads();
#else
  (void)n;
  return 1;
#endif
}

/* ---------------------------------------------------------------- 16-bit floats */

static inline float bf16_to_f32(uint16_t h) {
  uint32_t u = ((uint32_t)h) << 16;
  float f;
  memcpy(&f, &u, 4);
  return f;
}

static inline uint16_t f32_to_bf16(float f) {
  uint32_t u;
  memcpy(&u, &f, 4);
  if ((u & 0x7f800000u) == 0x7f800000u && (u & 0x007fffffu)) return (uint16_t)((u >> 16) | 0x40);
  u += 0x7fffu + ((u >> 16) & 1u); /* round to nearest, ties to even */
  return (uint16_t)(u >> 16);
}

static inline float f16_to_f32(uint16_t h) {
  _Float16 v;
  memcpy(&v, &h, 2);
  return (float)v;
}

static inline uint16_t f32_to_f16(float f) {
  _Float16 v = (_Float16)f; /* IEEE round to nearest even */
  uint16_t h;
  memcpy(&h, &v, 2);
  return h;
}

static inline float h_to_f32(uint16_t h, int dtype) {
  return dtype == TQO_BF16 ? bf16_to_f32(h) : f16_to_f32(h);
}

static inline uint16_t f32_to_h(float f, int dtype) {
  return dtype == TQO_BF16 ? f32_to_bf16(f) : f32_to_f16(f);
}

/* Round-trip through the 16-bit type: the value `x.to(dtype)` would hold. */
static inline float round_h(float f, int dtype) { return h_to_f32(f32_to_h(f, dtype), dtype); }

/* ------------------------------------------------------- activation quantizer */

/* sx[c] = f32(dtype(f32(absmax over all rows of x[:, 64c:64c+64]) / 127)), 1.0 when
 * the absmax is 0.  quant_utils.py:61-74 (the absmax is exact in the 16-bit type and
 * the division is done in f32 then rounded to the activation dtype). */
void tqo_act_scales(const uint16_t* x, int dtype, int64_t n, int64_t k, int64_t ld_row,
                    int64_t ld_col, float* sx) {
  int64_t n_tc = (k + 63) / 64;
  for (int64_t c = 0; c < n_tc; ++c) {
    float amax = 0.0f;
    for (int64_t i = 0; i < n; ++i) {
      for (int64_t j = c * 64; j < c * 64 + 64 && j < k; ++j) {
        float v = fabsf(h_to_f32(x[i * ld_row + j * ld_col], dtype));
        if (v > amax || isnan(v)) amax = v;
      }
    }
    sx[c] = amax > 0.0f ? round_h(amax / 127.0f, dtype) : 1.0f;
  }
}

static inline int8_t quant_code(float v, float s) {
  float q = rintf(v / s); /* IEEE division, ties to even */
  if (q > 127.0f) q = 127.0f;
  if (q < -127.0f) q = -127.0f;
  return (int8_t)q;
}

/* q[i, j] = clamp(rint(f32(x[i, j]) / sx[j / 64]), -127, 127); q is contiguous (n, k).
 * quant_utils.py:103-115. */
void tqo_quantize_with_scales(const uint16_t* x, int dtype, int64_t n, int64_t k, int64_t ld_row,
                              int64_t ld_col, const float* sx, int8_t* q) {
  for (int64_t i = 0; i < n; ++i)
    for (int64_t j = 0; j < k; ++j)
      q[i * k + j] = quant_code(h_to_f32(x[i * ld_row + j * ld_col], dtype), sx[j / 64]);
}

/* -------------------------------------------------------------- weight packer */

/* Tile t of the (zero-padded) weight: element (i, j) of tile id = r * n_tc + c is
 * W[64 r + i, 64 c + j], 0 outside the original (m, k) extent (pad_to_multiple,
 * quant_utils.py:152-164). */
static inline float w_at(const uint16_t* w, int dtype, int64_t m, int64_t k, int64_t ldw, int64_t row,
                         int64_t col) {
  if (row >= m || col >= k) return 0.0f;
  return h_to_f32(w[row * ldw + col], dtype);
}

/* INT8 tiles and scales for the given (already sorted) tile ids.  pack.py:119-167:
 *   base = absmax(tile) / 127 in f32 (1.0 for an all-zero tile);
 *   IAA (col_imp != NULL): candidates {0.75, 1.0, 1.25} * base, clamp_min 1e-12,
 *     err = mean((clamp(rint(W / s), +-127) * s - W)^2 * max(col_imp[col], 1e-8)),
 *     strictly smaller error wins, 0.75 is tried first;
 *   codes = clamp(rint(W / s), +-127).
 * The weighted error is summed in double here (the reference sums f32); the
 * candidate order and the strict comparison are the reference's. */
void tqo_pack_int8(const uint16_t* w, int dtype, int64_t m, int64_t k, int64_t ldw, int n_tc,
                   const int32_t* ids, int64_t t8, const float* col_imp, int8_t* tiles,
                   float* scales) {
  static const float mults[3] = {0.75f, 1.0f, 1.25f};
  for (int64_t t = 0; t < t8; ++t) {
    int64_t r = ids[t] / n_tc, c = ids[t] % n_tc;
    float amax = 0.0f;
    for (int i = 0; i < 64; ++i)
      for (int j = 0; j < 64; ++j) {
        float v = fabsf(w_at(w, dtype, m, k, ldw, r * 64 + i, c * 64 + j));
        if (v > amax) amax = v;
      }
    float base = amax == 0.0f ? 1.0f : amax / 127.0f;
    float s = base;
    if (col_imp) {
      double best = 0.0;
      for (int cand = 0; cand < 3; ++cand) {
        float sc = base * mults[cand];
        if (sc < 1e-12f) sc = 1e-12f;
        double err = 0.0;
        for (int i = 0; i < 64; ++i)
          for (int j = 0; j < 64; ++j) {
            float v = w_at(w, dtype, m, k, ldw, r * 64 + i, c * 64 + j);
            float dq = (float)quant_code(v, sc) * sc;
            float d = dq - v;
            float wm = col_imp[c * 64 + j];
            if (wm < 1e-8f) wm = 1e-8f;
            err += (double)(d * d * wm);
          }
        err /= 4096.0;
        if (cand == 0 || err < best) {
          best = err;
          s = sc;
        }
      }
    }
    scales[t] = s;
    for (int i = 0; i < 64; ++i)
      for (int j = 0; j < 64; ++j)
        tiles[t * 4096 + i * 64 + j] = quant_code(w_at(w, dtype, m, k, ldw, r * 64 + i, c * 64 + j), s);
  }
}

/* ----------------------------------------------------------------- mixed GEMM */

/* out[n, 64 r + j] for every row tile r, following gemm_rows_splitk_64x64.py:108-190:
 * per split s of SPLIT_K, the INT8 range [b + cnt*s/S, b + cnt*(s+1)/S) of row r in
 * ascending order: acc = fma(f32(i32 tile dot), sx[c] * sw[pos], acc) (use_fma = 0
 * gives mul-then-add); then the BF16 range: acc += f32 dot (summed in double here);
 * partials summed in split order 0..S-1, rounded to the output type, then
 * out = round(f32(y) + f32(bias)) when bias is given.
 *
 * x_i8 is (n_rows, K) with row stride ld_x8; x_fp (16-bit, xdtype) with row stride
 * ld_xfp; out (16-bit, odtype) with row stride ldo.  partials (optional) receives
 * the exact INT32 tile products as [t8][n_rows][64] (i32[pos][row][j]); acc_f32
 * (optional, row stride ldo) receives the FP32 sum of the splits before the rounding,
 * the quantity a row-parallel (K-split) sum across GPUs adds up.
 * Parallel over row tiles with OpenMP when compiled with -fopenmp. */
void tqo_gemm_mixed(const int8_t* x_i8, int64_t ld_x8, const float* sx, const int8_t* w8,
                    const float* s8, const int32_t* ids8, const int32_t* rowptr8,
                    const uint16_t* x_fp, int64_t ld_xfp, int xdtype, const uint16_t* w16,
                    const int32_t* ids16, const int32_t* rowptr16, uint16_t* out, int64_t ldo,
                    int odtype, const uint16_t* bias, int64_t n_rows, int64_t M, int64_t K,
                    int n_tr, int n_tc, int split_k, int use_fma, int32_t* partials, float* acc_f32) {
  if (split_k < 1) split_k = 1;
#pragma omp parallel for schedule(dynamic, 1)
  for (int r = 0; r < n_tr; ++r) {
    float* acc = (float*)malloc(sizeof(float) * 64 * (size_t)split_k);
    float* xrow = (float*)malloc(sizeof(float) * 64);
    for (int64_t n = 0; n < n_rows; ++n) {
      for (int s = 0; s < split_k; ++s) {
        float* a = acc + 64 * s;
        for (int j = 0; j < 64; ++j) a[j] = 0.0f;
        int64_t b = rowptr8[r], cnt = rowptr8[r + 1] - rowptr8[r];
        int64_t lo = b + cnt * s / split_k, hi = b + cnt * (s + 1) / split_k;
        for (int64_t pos = lo; pos < hi; ++pos) {
          int64_t c = ids8[pos] % n_tc;
          const int8_t* xr = x_i8 + n * ld_x8 + c * 64;
          int kmax = (int)((K - c * 64) < 64 ? (K - c * 64) : 64);
          float scale = sx[c] * s8[pos];
          for (int j = 0; j < 64; ++j) {
            const int8_t* wr = w8 + pos * 4096 + j * 64;
            int32_t dot = 0;
            for (int kk = 0; kk < kmax; ++kk) dot += (int32_t)xr[kk] * (int32_t)wr[kk];
            if (partials) partials[(pos * n_rows + n) * 64 + j] = dot;
            a[j] = use_fma ? fmaf((float)dot, scale, a[j]) : a[j] + (float)dot * scale;
          }
        }
        if (w16 && rowptr16) {
          b = rowptr16[r];
          cnt = rowptr16[r + 1] - rowptr16[r];
          lo = b + cnt * s / split_k;
          hi = b + cnt * (s + 1) / split_k;
          for (int64_t pos = lo; pos < hi; ++pos) {
            int64_t c = ids16[pos] % n_tc;
            for (int kk = 0; kk < 64; ++kk)
              xrow[kk] = (c * 64 + kk < K) ? h_to_f32(x_fp[n * ld_xfp + c * 64 + kk], xdtype) : 0.0f;
            for (int j = 0; j < 64; ++j) {
              const uint16_t* wr = w16 + pos * 4096 + j * 64;
              double d = 0.0;
              for (int kk = 0; kk < 64; ++kk) d += (double)xrow[kk] * (double)h_to_f32(wr[kk], xdtype);
              a[j] += (float)d;
            }
          }
        }
      }
      for (int j = 0; j < 64; ++j) {
        int64_t col = (int64_t)r * 64 + j;
        if (col >= M) break;
        float t = acc[j];
        for (int s = 1; s < split_k; ++s) t += acc[64 * s + j];
        if (acc_f32) acc_f32[n * ldo + col] = t;
        uint16_t y = f32_to_h(t, odtype);
        if (bias) y = f32_to_h(h_to_f32(y, odtype) + h_to_f32(bias[col], odtype), odtype);
        out[n * ldo + col] = y;
      }
    }
    free(acc);
    free(xrow);
  }
}

/* ---------------------------------------------------------------- calibration */

/* tile_scores[r, c] += sum over the tile of |f32(W) * f32(G)|  (calibrate.py:153-164).
 * Tile sums are accumulated in double here, then added in f32. */
void tqo_calib_gi_accumulate(const uint16_t* w, const uint16_t* g, int dtype, int64_t m, int64_t k,
                             int n_tr, int n_tc, float* tile_scores) {
  for (int r = 0; r < n_tr; ++r)
    for (int c = 0; c < n_tc; ++c) {
      double s = 0.0;
      for (int i = 0; i < 64; ++i)
        for (int j = 0; j < 64; ++j) {
          int64_t row = (int64_t)r * 64 + i, col = (int64_t)c * 64 + j;
          if (row >= m || col >= k) continue;
          float p = h_to_f32(w[row * k + col], dtype) * h_to_f32(g[row * k + col], dtype);
          s += fabsf(p);
        }
      tile_scores[r * n_tc + c] += (float)s;
    }
}

/* act_sum[j] += sum_i |f32(x[i, j])| in double  (calibrate.py:244-255). */
void tqo_iaa_channel_accumulate(const uint16_t* x, int dtype, int64_t rows, int64_t k, double* act_sum) {
  for (int64_t i = 0; i < rows; ++i)
    for (int64_t j = 0; j < k; ++j) act_sum[j] += (double)fabsf(h_to_f32(x[i * k + j], dtype));
}

/* mean[j] = f32(act_sum[j] / count); tile_scores[r, c] = sum over the tile of
 * |f32(W)| * mean[col]  (calibrate.py:346-367), summed in double here. */
void tqo_iaa_tile_scores(const uint16_t* w, int dtype, int64_t m, int64_t k, int n_tr, int n_tc,
                         const double* act_sum, int64_t count, float* mean_out, float* tile_scores) {
  for (int64_t j = 0; j < k; ++j) mean_out[j] = (float)(act_sum[j] / (double)count);
  for (int r = 0; r < n_tr; ++r)
    for (int c = 0; c < n_tc; ++c) {
      double s = 0.0;
      for (int i = 0; i < 64; ++i)
        for (int j = 0; j < 64; ++j) {
          int64_t row = (int64_t)r * 64 + i, col = (int64_t)c * 64 + j;
          if (row >= m || col >= k) continue;
          s += (double)(fabsf(h_to_f32(w[row * k + col], dtype)) * mean_out[col]);
        }
      tile_scores[r * n_tc + c] = (float)s;
    }
}

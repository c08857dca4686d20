// Load-time tile packer (sm_100a): INT8 codes + per-tile scales, and the 16-bit tile
// gather, written straight into the reference's Pack layout (int8[T8][64][64],
// f32[T8], 16-bit [T16][64][64]).
//
// Reference: src/kernels/pack.py:65-203 (_pack_weight_with_tile_ids), padding from
// src/kernels/quant_utils.py:152-164.
//   base  = f32(absmax(tile)) / 127, 1.0 for an all-zero tile           (:125-130)
//   IAA   = candidates {0.75, 1.0, 1.25} * base, clamp_min 1e-12;
//           err = mean((clamp(rint(W/s), +-127) * s - W)^2 * max(imp[col], 1e-8));
//           the first strictly smaller error wins                        (:132-159)
//   codes = clamp(rint(f32(W) / s), -127, 127)                            (:163-167)
// One CTA per tile; 256 threads x 16 elements; the squared error is summed in f64.
#include "common.cuh"

namespace tq {

template <int WT>
__device__ __forceinline__ void load_tile16(const void* w, int64_t m, int64_t k, int64_t ldw, int64_t r, int64_t c,
                                            int tid, float (&v)[16]) {
  const int i = tid >> 2, j0 = (tid & 3) * 16;
  const int64_t row = r * 64 + i, col0 = c * 64 + j0;
  const uint16_t* src = reinterpret_cast<const uint16_t*>(w) + row * ldw + col0;
  const bool full = row < m && col0 + 16 <= k && ((uintptr_t)src % 16) == 0;
  if (full) {
    const uint4 a = *reinterpret_cast<const uint4*>(src);
    const uint4 b = *reinterpret_cast<const uint4*>(src + 8);
    const uint32_t words[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      v[2 * e] = h2f((uint16_t)(words[e] & 0xffffu), WT);
      v[2 * e + 1] = h2f((uint16_t)(words[e] >> 16), WT);
    }
  } else {
#pragma unroll
    for (int e = 0; e < 16; ++e) v[e] = (row < m && col0 + e < k) ? h2f(src[e], WT) : 0.0f;
  }
}

__device__ __forceinline__ float block_max256(float v, float* red) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
  __syncthreads();
  float m = red[0];
#pragma unroll
  for (int w = 1; w < 8; ++w) m = fmaxf(m, red[w]);
  __syncthreads();
  return m;
}

__device__ __forceinline__ double block_sum256(double v, double* red) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
  __syncthreads();
  double s = 0.0;
#pragma unroll
  for (int w = 0; w < 8; ++w) s += red[w];
  __syncthreads();
  return s;
}

template <int WT>
__global__ void __launch_bounds__(256) pack_int8_kernel(const void* __restrict__ w, int64_t m, int64_t k, int64_t ldw,
                                                        int n_tc, const int32_t* __restrict__ ids,
                                                        const float* __restrict__ imp, int8_t* __restrict__ tiles,
                                                        float* __restrict__ scales) {
  __shared__ float redf[8];
  __shared__ double redd[8];
  const int64_t t = blockIdx.x;
  const int id = ids[t];
  const int64_t r = id / n_tc, c = id % n_tc;
  const int tid = threadIdx.x;
  float v[16];
  load_tile16<WT>(w, m, k, ldw, r, c, tid, v);
  float amax = 0.0f;
#pragma unroll
  for (int e = 0; e < 16; ++e) amax = fmaxf(amax, fabsf(v[e]));
  amax = block_max256(amax, redf);
  const float base = amax == 0.0f ? 1.0f : __fdiv_rn(amax, 127.0f);
  float s = base;
  if (imp) {
    const int j0 = (tid & 3) * 16;
    float wm[16];
#pragma unroll
    for (int e = 0; e < 16; ++e) wm[e] = fmaxf(imp[c * 64 + j0 + e], 1e-8f);
    const float mults[3] = {0.75f, 1.0f, 1.25f};
    double best = 0.0;
#pragma unroll 1
    for (int cand = 0; cand < 3; ++cand) {
      const float sc = fmaxf(__fmul_rn(base, mults[cand]), 1e-12f);
      const float rc = __frcp_rn(sc);
      double err = 0.0;
#pragma unroll
      for (int e = 0; e < 16; ++e) {
        const float dq = __fmul_rn((float)quant_code_fast(v[e], sc, rc), sc);
        const float d = __fsub_rn(dq, v[e]);
        err += (double)__fmul_rn(__fmul_rn(d, d), wm[e]);
      }
      err = block_sum256(err, redd) / 4096.0;
      if (cand == 0 || err < best) {
        best = err;
        s = sc;
      }
    }
  }
  const float rc = __frcp_rn(s);
  uint32_t words[4];
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    uint32_t wv = 0;
#pragma unroll
    for (int e = 0; e < 4; ++e) wv |= ((uint32_t)(quant_code_fast(v[4 * q + e], s, rc) & 0xff)) << (8 * e);
    words[q] = wv;
  }
  *reinterpret_cast<uint4*>(tiles + t * 4096 + (tid >> 2) * 64 + (tid & 3) * 16) =
      make_uint4(words[0], words[1], words[2], words[3]);
  if (tid == 0) scales[t] = s;
}

__global__ void __launch_bounds__(256) gather_fp_kernel(const uint16_t* __restrict__ w, int64_t m, int64_t k,
                                                        int64_t ldw, int n_tc, const int32_t* __restrict__ ids,
                                                        uint16_t* __restrict__ tiles) {
  const int64_t t = blockIdx.x;
  const int id = ids[t];
  const int64_t r = id / n_tc, c = id % n_tc;
  for (int e = threadIdx.x; e < 4096; e += 256) {
    const int64_t row = r * 64 + (e >> 6), col = c * 64 + (e & 63);
    tiles[t * 4096 + e] = (row < m && col < k) ? w[row * ldw + col] : (uint16_t)0;
  }
}

}  // namespace tq

using namespace tq;

static int check_w(const void* w, int dtype, int64_t m, int64_t k, int64_t ldw, int n_tc) {
  if (dtype != TQ_DTYPE_BF16 && dtype != TQ_DTYPE_F16) return tq_set_error(TQ_ERR_INVALID, "weight dtype must be bf16 or f16");
  if (m <= 0 || k <= 0 || ldw < k || !w) return tq_set_error(TQ_ERR_INVALID, "weight must be a non-empty (m, k) matrix");
  if (n_tc != (k + 63) / 64) return tq_set_error(TQ_ERR_INVALID, "n_tc does not match k");
  return TQ_OK;
}

extern "C" int tq_pack_int8_tiles(const void* w, int w_dtype, int64_t m, int64_t k, int64_t ldw, int n_tc,
                                  const int32_t* ids, int64_t t8, const float* col_importance, int8_t* tiles,
                                  float* scales, void* stream) {
  int rc = check_w(w, w_dtype, m, k, ldw, n_tc);
  if (rc) return rc;
  if (t8 < 0) return tq_set_error(TQ_ERR_INVALID, "negative tile count");
  if (t8 == 0) return TQ_OK;
  if (!ids || !tiles || !scales) return tq_set_error(TQ_ERR_INVALID, "null output or id array");
  if (((uintptr_t)tiles & 15) != 0) return tq_set_error(TQ_ERR_INVALID, "tile arena must be 16-byte aligned");
  if (t8 > 0x7fffffff) return tq_set_error(TQ_ERR_INVALID, "too many tiles");
  cudaStream_t st = (cudaStream_t)stream;
  if (w_dtype == TQ_DTYPE_BF16)
    pack_int8_kernel<TQ_DTYPE_BF16><<<(unsigned)t8, 256, 0, st>>>(w, m, k, ldw, n_tc, ids, col_importance, tiles, scales);
  else
    pack_int8_kernel<TQ_DTYPE_F16><<<(unsigned)t8, 256, 0, st>>>(w, m, k, ldw, n_tc, ids, col_importance, tiles, scales);
  TQ_LAUNCHED();
  return TQ_OK;
}

extern "C" int tq_gather_fp_tiles(const void* w, int w_dtype, int64_t m, int64_t k, int64_t ldw, int n_tc,
                                  const int32_t* ids, int64_t t16, void* tiles, void* stream) {
  int rc = check_w(w, w_dtype, m, k, ldw, n_tc);
  if (rc) return rc;
  if (t16 < 0) return tq_set_error(TQ_ERR_INVALID, "negative tile count");
  if (t16 == 0) return TQ_OK;
  if (!ids || !tiles) return tq_set_error(TQ_ERR_INVALID, "null output or id array");
  gather_fp_kernel<<<(unsigned)t16, 256, 0, (cudaStream_t)stream>>>(reinterpret_cast<const uint16_t*>(w), m, k, ldw,
                                                                    n_tc, ids, reinterpret_cast<uint16_t*>(tiles));
  TQ_LAUNCHED();
  return TQ_OK;
}

// GI / IAA calibration reductions (sm_100a).
//
// Reference: src/kernels/calibrate.py
//   GI   tile_scores += sum_tile |f32(W) * f32(dL/dW)|                     (:153-164)
//   IAA  act_sum[j] += sum_rows |f32(x[:, j])| (f64 running sum)             (:244-255)
//        mean = f32(act_sum / count); tile score = sum_tile |f32(W)| * mean  (:346-367)
// The reference forms these with dense torch temporaries (|W*G| and |W|*mean are full
// f32 copies of the weight) and, for GI, a host copy every batch; here each is one
// pass over the 16-bit operands, accumulated on the device.
#include <algorithm>

#include "common.cuh"

namespace tq {

__device__ __forceinline__ float block_sum256f(float v, float* red) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
  __syncthreads();
  float s = 0.0f;
  if (threadIdx.x == 0)
#pragma unroll
    for (int w = 0; w < 8; ++w) s += red[w];
  return s;
}

// One CTA per tile; each thread covers 16 elements of one tile row.
template <int DT>
__global__ void __launch_bounds__(256) gi_kernel(const uint16_t* __restrict__ w, const uint16_t* __restrict__ g, int64_t m,
                                                 int64_t k, int64_t ldw, int64_t ldg, int n_tc, float* __restrict__ scores) {
  __shared__ float red[8];
  const int64_t r = blockIdx.x / n_tc, c = blockIdx.x % n_tc;
  const int i = threadIdx.x >> 2, j0 = (threadIdx.x & 3) * 16;
  const int64_t row = r * 64 + i;
  float s = 0.0f;
  if (row < m) {
#pragma unroll 4
    for (int e = 0; e < 16; ++e) {
      const int64_t col = c * 64 + j0 + e;
      if (col < k) s += fabsf(__fmul_rn(h2f(w[row * ldw + col], DT), h2f(g[row * ldg + col], DT)));
    }
  }
  s = block_sum256f(s, red);
  if (threadIdx.x == 0) scores[blockIdx.x] += s;
}

// Column sums of |x| in f64: thread = column, CTA = (column block, row slice).
template <int DT>
__global__ void __launch_bounds__(256) iaa_channel_kernel(const uint16_t* __restrict__ x, int64_t rows, int64_t k,
                                                          int64_t ld_row, double* __restrict__ act_sum) {
  const int64_t j = (int64_t)blockIdx.x * 256 + threadIdx.x;
  if (j >= k) return;
  const int64_t per = (rows + gridDim.y - 1) / gridDim.y;
  const int64_t r0 = (int64_t)blockIdx.y * per, r1 = min(rows, r0 + per);
  double s = 0.0;
  for (int64_t r = r0; r < r1; ++r) s += (double)fabsf(h2f(x[r * ld_row + j], DT));
  if (r1 > r0) atomicAdd(act_sum + j, s);
}

__global__ void iaa_mean_kernel(const double* __restrict__ act_sum, int64_t k, int64_t count, float* __restrict__ mean) {
  const int64_t j = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (j < k) mean[j] = (float)(act_sum[j] / (double)count);
}

template <int DT>
__global__ void __launch_bounds__(256) iaa_tile_kernel(const uint16_t* __restrict__ w, int64_t m, int64_t k, int64_t ldw,
                                                       int n_tc, const float* __restrict__ mean, float* __restrict__ scores) {
  __shared__ float red[8];
  const int64_t r = blockIdx.x / n_tc, c = blockIdx.x % n_tc;
  const int i = threadIdx.x >> 2, j0 = (threadIdx.x & 3) * 16;
  const int64_t row = r * 64 + i;
  float s = 0.0f;
  if (row < m) {
#pragma unroll 4
    for (int e = 0; e < 16; ++e) {
      const int64_t col = c * 64 + j0 + e;
      if (col < k) s += __fmul_rn(fabsf(h2f(w[row * ldw + col], DT)), mean[col]);
    }
  }
  s = block_sum256f(s, red);
  if (threadIdx.x == 0) scores[blockIdx.x] = s;
}

}  // namespace tq

using namespace tq;

extern "C" int tq_calib_gi_accumulate(const void* w, const void* g, int dtype, int64_t m, int64_t k, int64_t ldw,
                                      int64_t ldg, int n_tr, int n_tc, float* tile_scores, void* stream) {
  if (dtype != TQ_DTYPE_BF16 && dtype != TQ_DTYPE_F16) return tq_set_error(TQ_ERR_INVALID, "dtype must be bf16 or f16");
  if (m <= 0 || k <= 0 || !w || !g || !tile_scores || ldw < k || ldg < k)
    return tq_set_error(TQ_ERR_INVALID, "bad GI operands");
  if (n_tr != (m + 63) / 64 || n_tc != (k + 63) / 64) return tq_set_error(TQ_ERR_INVALID, "tile grid mismatch");
  const auto W = reinterpret_cast<const uint16_t*>(w);
  const auto G = reinterpret_cast<const uint16_t*>(g);
  const unsigned blocks = (unsigned)((int64_t)n_tr * n_tc);
  cudaStream_t st = (cudaStream_t)stream;
  if (dtype == TQ_DTYPE_BF16)
    gi_kernel<TQ_DTYPE_BF16><<<blocks, 256, 0, st>>>(W, G, m, k, ldw, ldg, n_tc, tile_scores);
  else
    gi_kernel<TQ_DTYPE_F16><<<blocks, 256, 0, st>>>(W, G, m, k, ldw, ldg, n_tc, tile_scores);
  TQ_LAUNCHED();
  return TQ_OK;
}

extern "C" int tq_calib_iaa_channel_accumulate(const void* x, int dtype, int64_t rows, int64_t k, int64_t ld_row,
                                               double* act_sum, void* stream) {
  if (dtype != TQ_DTYPE_BF16 && dtype != TQ_DTYPE_F16) return tq_set_error(TQ_ERR_INVALID, "dtype must be bf16 or f16");
  if (rows < 0 || k <= 0 || !act_sum || ld_row < k || (rows > 0 && !x)) return tq_set_error(TQ_ERR_INVALID, "bad IAA operands");
  if (rows == 0) return TQ_OK;
  const unsigned cb = (unsigned)((k + 255) / 256);
  int64_t splits = std::max<int64_t>(1, std::min<int64_t>((int64_t)tq_sm_count() * 4 / cb, rows / 64));
  splits = std::min<int64_t>(splits, 65535);
  const auto X = reinterpret_cast<const uint16_t*>(x);
  cudaStream_t st = (cudaStream_t)stream;
  if (dtype == TQ_DTYPE_BF16)
    iaa_channel_kernel<TQ_DTYPE_BF16><<<dim3(cb, (unsigned)splits), 256, 0, st>>>(X, rows, k, ld_row, act_sum);
  else
    iaa_channel_kernel<TQ_DTYPE_F16><<<dim3(cb, (unsigned)splits), 256, 0, st>>>(X, rows, k, ld_row, act_sum);
  TQ_LAUNCHED();
  return TQ_OK;
}

extern "C" int tq_calib_iaa_tile_scores(const void* w, int dtype, int64_t m, int64_t k, int64_t ldw,
                                        const double* act_sum, int64_t count, float* mean, float* tile_scores,
                                        void* stream) {
  if (dtype != TQ_DTYPE_BF16 && dtype != TQ_DTYPE_F16) return tq_set_error(TQ_ERR_INVALID, "dtype must be bf16 or f16");
  if (m <= 0 || k <= 0 || !w || !act_sum || !mean || !tile_scores || ldw < k)
    return tq_set_error(TQ_ERR_INVALID, "bad IAA operands");
  if (count <= 0) return tq_set_error(TQ_ERR_INVALID, "no activation samples captured (count <= 0)");
  const int n_tr = (int)((m + 63) / 64), n_tc = (int)((k + 63) / 64);
  cudaStream_t st = (cudaStream_t)stream;
  iaa_mean_kernel<<<(unsigned)((k + 255) / 256), 256, 0, st>>>(act_sum, k, count, mean);
  TQ_LAUNCHED();
  const auto W = reinterpret_cast<const uint16_t*>(w);
  if (dtype == TQ_DTYPE_BF16)
    iaa_tile_kernel<TQ_DTYPE_BF16><<<(unsigned)((int64_t)n_tr * n_tc), 256, 0, st>>>(W, m, k, ldw, n_tc, mean, tile_scores);
  else
    iaa_tile_kernel<TQ_DTYPE_F16><<<(unsigned)((int64_t)n_tr * n_tc), 256, 0, st>>>(W, m, k, ldw, n_tc, mean, tile_scores);
  TQ_LAUNCHED();
  return TQ_OK;
}

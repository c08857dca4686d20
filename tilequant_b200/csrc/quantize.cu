// Per-64-column activation INT8 quantizer (sm_100a).
//
// Reference semantics (HanzhiZhang-Ulrica/TileQuant):
//   src/kernels/quant_utils.py:41-134, src/kernels/triton/quantize_activation.py:13-203.
//   sx[c] = f32(dtype(f32(absmax over ALL rows of x[:, 64c:64c+64]) / 127)), 1.0 if 0
//   q     = clamp(rint(f32(x) / sx[c]), -127, 127)          (IEEE quotient, ties-to-even)
//
// Kernels:
//   act_scales_kernel      column-tile absmax.  Large row counts split the rows of one
//                          column tile over a thread-block cluster; the partial maxima
//                          meet in distributed shared memory (no global scratch, no
//                          atomics), so the grid fills all 148 SMs even for n_tc = 48.
//   quantize_kernel        elementwise codes, 16-byte loads / 8-byte stores.
//   quantize_small_kernel  one pass for n_rows <= 128: the column tile stays in shared
//                          memory between the absmax and the codes (x read once).
#include <cooperative_groups.h>

#include <algorithm>

#include "common.cuh"
#include "tma.cuh"

namespace cg = cooperative_groups;

namespace tq {

template <int XT>
__device__ __forceinline__ float ld16(const void* base, int64_t idx) {
  return h2f(reinterpret_cast<const uint16_t*>(base)[idx], XT);
}

// absmax of 8 packed 16-bit values
template <int XT>
__device__ __forceinline__ float absmax8(uint4 v) {
  const uint32_t w[4] = {v.x, v.y, v.z, v.w};
  float m = 0.0f;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    m = fmaxf(m, fabsf(h2f((uint16_t)(w[i] & 0xffffu), XT)));
    m = fmaxf(m, fabsf(h2f((uint16_t)(w[i] >> 16), XT)));
  }
  return m;
}

// Absmax of column tile blockIdx.x over rows [row0, row1).  vec: 16-byte path allowed.
template <int XT>
__device__ float tile_absmax(const void* x, int64_t n_rows, int64_t k, int64_t ld_row, int64_t ld_col,
                             int64_t row0, int64_t row1, bool vec) {
  const int64_t c = blockIdx.x;
  float m = 0.0f;
  if (vec) {
    // 8 chunks of 16 bytes per row; blockDim/8 rows per pass, 4 passes in flight
    const int chunk = threadIdx.x & 7;
    const int64_t rstep = blockDim.x >> 3;
    const char* base = reinterpret_cast<const char*>(x) + (c * 64 + chunk * 8) * 2;
    int64_t r = row0 + (threadIdx.x >> 3);
    for (; r + 3 * rstep < row1; r += 4 * rstep) {
      uint4 v0 = __ldg(reinterpret_cast<const uint4*>(base + (r)*ld_row * 2));
      uint4 v1 = __ldg(reinterpret_cast<const uint4*>(base + (r + rstep) * ld_row * 2));
      uint4 v2 = __ldg(reinterpret_cast<const uint4*>(base + (r + 2 * rstep) * ld_row * 2));
      uint4 v3 = __ldg(reinterpret_cast<const uint4*>(base + (r + 3 * rstep) * ld_row * 2));
      m = fmaxf(m, fmaxf(fmaxf(absmax8<XT>(v0), absmax8<XT>(v1)), fmaxf(absmax8<XT>(v2), absmax8<XT>(v3))));
    }
    for (; r < row1; r += rstep) m = fmaxf(m, absmax8<XT>(__ldg(reinterpret_cast<const uint4*>(base + r * ld_row * 2))));
  } else {
    const int64_t width = min((int64_t)64, k - c * 64);
    for (int64_t e = threadIdx.x; e < (row1 - row0) * 64; e += blockDim.x) {
      const int64_t r = row0 + e / 64, j = e % 64;
      if (j < width) m = fmaxf(m, fabsf(ld16<XT>(x, r * ld_row + (c * 64 + j) * ld_col)));
    }
  }
  return m;
}

template <int XT, bool CLUSTER>
__global__ void __launch_bounds__(256) act_scales_kernel(const void* __restrict__ x, int64_t n_rows, int64_t k,
                                                         int64_t ld_row, int64_t ld_col, float* __restrict__ sx,
                                                         int vec) {
  grid_dep_launch();  // a dependent GEMM may start streaming its weights
  __shared__ float red[32];
  __shared__ float cta_max;
  const int64_t parts = gridDim.y;
  const int64_t per = (n_rows + parts - 1) / parts;
  const int64_t row0 = min(n_rows, (int64_t)blockIdx.y * per);
  const int64_t row1 = min(n_rows, row0 + per);
  const bool v = vec && (blockIdx.x * 64 + 64 <= k);
  float m = block_max(tile_absmax<XT>(x, n_rows, k, ld_row, ld_col, row0, row1, v), red);
  if constexpr (CLUSTER) {
    cg::cluster_group cluster = cg::this_cluster();
    if (threadIdx.x == 0) cta_max = m;
    cluster.sync();
    if (cluster.block_rank() == 0 && threadIdx.x == 0) {
      float total = 0.0f;
      for (unsigned p = 0; p < cluster.num_blocks(); ++p) total = fmaxf(total, *cluster.map_shared_rank(&cta_max, p));
      sx[blockIdx.x] = scale_from_absmax<XT>(total);
    }
    cluster.sync();  // peers keep their shared memory alive until rank 0 has read it
  } else {
    if (threadIdx.x == 0) sx[blockIdx.x] = scale_from_absmax<XT>(m);
  }
}

// Codes of 8 consecutive 16-bit values that share the scale s (r = 1/s).
template <int XT>
__device__ __forceinline__ uint2 codes8(uint4 v, float s, float r) {
  const uint32_t w[4] = {v.x, v.y, v.z, v.w};
  uint32_t out[2] = {0u, 0u};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int lo = quant_code_fast(h2f((uint16_t)(w[i] & 0xffffu), XT), s, r);
    const int hi = quant_code_fast(h2f((uint16_t)(w[i] >> 16), XT), s, r);
    out[i >> 1] |= ((uint32_t)(lo & 0xff) | ((uint32_t)(hi & 0xff) << 8)) << ((i & 1) * 16);
  }
  return make_uint2(out[0], out[1]);
}

template <int XT>
__global__ void __launch_bounds__(256) quantize_kernel(const void* __restrict__ x, int64_t n_rows, int64_t k,
                                                       int64_t ld_row, int64_t ld_col, const float* __restrict__ sx,
                                                       int8_t* __restrict__ q, int64_t ldq, int vec) {
  grid_dep_launch();
  if (vec) {
    const int64_t chunks = k / 8;  // k % 8 == 0 on this path
    const int64_t total = n_rows * chunks;
    for (int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; e < total; e += (int64_t)gridDim.x * blockDim.x) {
      const int64_t r = e / chunks, ch = e % chunks;
      const float s = __ldg(sx + (ch * 8) / 64);
      const float rc = __frcp_rn(s);
      const uint4 v = __ldg(reinterpret_cast<const uint4*>(reinterpret_cast<const uint16_t*>(x) + r * ld_row + ch * 8));
      *reinterpret_cast<uint2*>(q + r * ldq + ch * 8) = codes8<XT>(v, s, rc);
    }
  } else {
    const int64_t total = n_rows * k;
    for (int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; e < total; e += (int64_t)gridDim.x * blockDim.x) {
      const int64_t r = e / k, j = e % k;
      q[r * ldq + j] = (int8_t)quant_code(ld16<XT>(x, r * ld_row + j * ld_col), __ldg(sx + j / 64));
    }
  }
}

// One pass for n_rows <= 128: column tile blockIdx.x is staged in shared memory.
template <int XT>
__global__ void __launch_bounds__(256) quantize_small_kernel(const void* __restrict__ x, int64_t n_rows, int64_t k,
                                                             int64_t ld_row, int64_t ld_col, int8_t* __restrict__ q,
                                                             int64_t ldq, float* __restrict__ sx) {
  grid_dep_wait();  // x comes from the preceding kernel (launched with programmatic serialization)
  grid_dep_launch();
  __shared__ float tile[128 * 64];
  __shared__ float red[32];
  const int64_t c = blockIdx.x;
  const int64_t width = min((int64_t)64, k - c * 64);
  float m = 0.0f;
  for (int e = threadIdx.x; e < n_rows * 64; e += blockDim.x) {
    const int r = e >> 6, j = e & 63;
    const float v = j < width ? ld16<XT>(x, r * ld_row + (c * 64 + j) * ld_col) : 0.0f;
    tile[e] = v;
    m = fmaxf(m, fabsf(v));
  }
  m = block_max(m, red);
  const float s = scale_from_absmax<XT>(m);
  const float rc = __frcp_rn(s);
  for (int e = threadIdx.x; e < n_rows * 64; e += blockDim.x) {
    const int r = e >> 6, j = e & 63;
    if (j < width) q[r * ldq + c * 64 + j] = (int8_t)quant_code_fast(tile[e], s, rc);
  }
  if (threadIdx.x == 0) sx[c] = s;
}

}  // namespace tq

using namespace tq;

static int check_x(const void* x, int dtype, int64_t n_rows, int64_t k, int64_t ld_row, int64_t ld_col) {
  if (dtype != TQ_DTYPE_BF16 && dtype != TQ_DTYPE_F16) return tq_set_error(TQ_ERR_INVALID, "x dtype must be bf16 or f16");
  if (n_rows < 0 || k < 0) return tq_set_error(TQ_ERR_INVALID, "negative shape");
  if ((n_rows > 0 && k > 0) && !x) return tq_set_error(TQ_ERR_INVALID, "null activation pointer");
  if (ld_row < 0 || ld_col < 0) return tq_set_error(TQ_ERR_INVALID, "negative stride");
  return TQ_OK;
}

static bool vec_ok(const void* x, int64_t ld_row, int64_t ld_col) {
  return ld_col == 1 && ((uintptr_t)x % 16) == 0 && (ld_row * 2) % 16 == 0;
}

static int launch_scales(const void* x, int dtype, int64_t n_rows, int64_t k, int64_t ld_row, int64_t ld_col,
                         float* sx, cudaStream_t st) {
  const int n_tc = (int)((k + 63) / 64);
  const int vec = vec_ok(x, ld_row, ld_col) ? 1 : 0;
  int parts = 1;
  if (n_rows > 256) {
    // aim for ~2 CTAs per SM overall, at most 8 CTAs (one portable cluster) per tile
    const int sms = tq_sm_count();
    while (parts < 8 && (int64_t)n_tc * parts < 2 * sms && n_rows / (parts * 2) >= 128) parts *= 2;
  }
  if (parts == 1) {
    if (dtype == TQ_DTYPE_BF16)
      act_scales_kernel<TQ_DTYPE_BF16, false><<<dim3(n_tc, 1), 256, 0, st>>>(x, n_rows, k, ld_row, ld_col, sx, vec);
    else
      act_scales_kernel<TQ_DTYPE_F16, false><<<dim3(n_tc, 1), 256, 0, st>>>(x, n_rows, k, ld_row, ld_col, sx, vec);
    TQ_LAUNCHED();
    return TQ_OK;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(n_tc, parts, 1);
  cfg.blockDim = dim3(256, 1, 1);
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 1;
  attr[0].val.clusterDim.y = parts;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  if (dtype == TQ_DTYPE_BF16)
    TQ_CUDA_TRY(cudaLaunchKernelEx(&cfg, act_scales_kernel<TQ_DTYPE_BF16, true>, x, n_rows, k, ld_row, ld_col, sx, vec));
  else
    TQ_CUDA_TRY(cudaLaunchKernelEx(&cfg, act_scales_kernel<TQ_DTYPE_F16, true>, x, n_rows, k, ld_row, ld_col, sx, vec));
  tq_count_launch();
  return TQ_OK;
}

static int launch_quantize(const void* x, int dtype, int64_t n_rows, int64_t k, int64_t ld_row, int64_t ld_col,
                           const float* sx, int8_t* q, int64_t ldq, cudaStream_t st) {
  const int vec = (vec_ok(x, ld_row, ld_col) && k % 8 == 0 && ((uintptr_t)q % 8) == 0 && ldq % 8 == 0) ? 1 : 0;
  const int64_t work = vec ? n_rows * (k / 8) : n_rows * k;
  const int64_t blocks = std::min<int64_t>((work + 255) / 256, (int64_t)tq_sm_count() * 16);
  if (blocks <= 0) return TQ_OK;
  if (dtype == TQ_DTYPE_BF16)
    quantize_kernel<TQ_DTYPE_BF16><<<(unsigned)blocks, 256, 0, st>>>(x, n_rows, k, ld_row, ld_col, sx, q, ldq, vec);
  else
    quantize_kernel<TQ_DTYPE_F16><<<(unsigned)blocks, 256, 0, st>>>(x, n_rows, k, ld_row, ld_col, sx, q, ldq, vec);
  TQ_LAUNCHED();
  return TQ_OK;
}

extern "C" int tq_act_scales(const void* x, int x_dtype, int64_t n_rows, int64_t k, int64_t ld_row, int64_t ld_col,
                             float* sx, void* stream) {
  int rc = check_x(x, x_dtype, n_rows, k, ld_row, ld_col);
  if (rc) return rc;
  if (k == 0) return TQ_OK;
  if (!sx) return tq_set_error(TQ_ERR_INVALID, "null sx");
  return launch_scales(x, x_dtype, n_rows, k, ld_row, ld_col, sx, (cudaStream_t)stream);
}

extern "C" int tq_quantize_with_scales(const void* x, int x_dtype, int64_t n_rows, int64_t k, int64_t ld_row,
                                       int64_t ld_col, const float* sx, int8_t* q, int64_t ldq, void* stream) {
  int rc = check_x(x, x_dtype, n_rows, k, ld_row, ld_col);
  if (rc) return rc;
  if (n_rows == 0 || k == 0) return TQ_OK;
  if (!sx || !q) return tq_set_error(TQ_ERR_INVALID, "null sx or q");
  if (ldq < k) return tq_set_error(TQ_ERR_INVALID, "ldq < k");
  return launch_quantize(x, x_dtype, n_rows, k, ld_row, ld_col, sx, q, ldq, (cudaStream_t)stream);
}

extern "C" int tq_quantize_act(const void* x, int x_dtype, int64_t n_rows, int64_t k, int64_t ld_row, int64_t ld_col,
                               int8_t* q, int64_t ldq, float* sx, void* stream) {
  int rc = check_x(x, x_dtype, n_rows, k, ld_row, ld_col);
  if (rc) return rc;
  if (k == 0) return TQ_OK;
  if (!sx || (n_rows > 0 && !q)) return tq_set_error(TQ_ERR_INVALID, "null sx or q");
  if (ldq < k) return tq_set_error(TQ_ERR_INVALID, "ldq < k");
  cudaStream_t st = (cudaStream_t)stream;
  if (n_rows <= 128) {
    const int n_tc = (int)((k + 63) / 64);
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)n_tc, 1, 1);
    cfg.blockDim = dim3(256, 1, 1);
    cfg.stream = st;
    cfg.attrs = attr;
    cfg.numAttrs = tq_pdl_enabled() ? 1 : 0;
    if (x_dtype == TQ_DTYPE_BF16)
      TQ_CUDA_TRY(cudaLaunchKernelEx(&cfg, quantize_small_kernel<TQ_DTYPE_BF16>, x, n_rows, k, ld_row, ld_col, q, ldq, sx));
    else
      TQ_CUDA_TRY(cudaLaunchKernelEx(&cfg, quantize_small_kernel<TQ_DTYPE_F16>, x, n_rows, k, ld_row, ld_col, q, ldq, sx));
    tq_count_launch();
    return TQ_OK;
  }
  rc = launch_scales(x, x_dtype, n_rows, k, ld_row, ld_col, sx, st);
  if (rc) return rc;
  return launch_quantize(x, x_dtype, n_rows, k, ld_row, ld_col, sx, q, ldq, st);
}

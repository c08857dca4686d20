// Row-owned mixed INT8/BF16 64x64 tile GEMM, split-K over each row's tile list
// (sm_100a).  Decode-sized row counts and the general fallback.
//
// Reference: src/kernels/triton/gemm_rows_splitk_64x64.py:78-190 (kernel) and
// :225-323 (host).  Same arithmetic, same split partition and same split order:
//   split s of S owns positions [b + cnt*s/S, b + cnt*(s+1)/S) of row r's INT8 list
//   and of its BF16 list;  acc = acc + f32(i32 tile dot) * (sx[c] * sw[pos]) (mul and
//   add rounded separately, ascending column order), then acc += dot(x, W16^T);
//   the split partials are added in split order 0..S-1.
//
// B200 design (one CTA = row tile r x 8*NB activation rows x split s):
//   * warp-specialized: a producer warp streams each step's operands into a ring of
//     NS shared-memory stages with the TMA engine (the 4 KB INT8 weight tile as one
//     1-D bulk copy; the activation tile, and each 32-column half of a BF16 weight
//     tile, as 2-D tensor-map copies that zero-fill past the matrix edge), and four
//     compute warps consume them.  full/empty mbarriers per stage replace CTA-wide
//     barriers, so the compute warps never wait for each other;
//   * programmatic dependent launch: the weight stream of the first NS steps starts
//     before the kernel that produced the INT8 activations has finished;
//   * swap-AB: the 64 weight rows of a tile are the MMA's M side, the activation rows
//     its N side (8 per block), so decode batches of 1..8 tokens pay for 8, not 16;
//   * exact INT32 tile products with mma.sync m16n8k32 s8 (k order permuted identically
//     for both operands, so every thread reads 16 contiguous bytes per row: the integer
//     dot does not depend on the order), converted to f32 with an exact integer-add /
//     float-subtract pair instead of the quarter-rate I2F; 16-bit tiles with m16n8k16
//     straight into the FP32 accumulator;
//   * split-K partials meet in distributed shared memory: the S CTAs of one
//     (r, row block) form a thread-block cluster, each publishes its FP32 partial in its
//     own shared memory and sums a 1/S slice over ranks 0..S-1.  No global workspace,
//     no arrival counters;
//   * optional fused activation quantization (decode): the compute warps quantize the
//     16-bit activation tile of each INT8 step, bit-identical to the quantizer kernel.
#include <cooperative_groups.h>
#include <string.h>

#include <algorithm>

#include "common.cuh"
#include "gemm_args.cuh"
#include "tma.cuh"

namespace cg = cooperative_groups;

namespace tq {

struct RowsMaps {
  CUtensorMap x8;        // x_int8, box 64 x BN bytes
  CUtensorMap xfp_half;  // x_fp,   box 32 x BN elements
  CUtensorMap xfp_full;  // x_fp,   box 64 x BN elements (fused quantization)
  CUtensorMap w16_half;  // 16-bit tile arena [T16*64][64], box 32 x 64
};

template <int NB>
struct RowsCfg {
  static constexpr int BN = 8 * NB;  // activation rows (tokens) per CTA
  static constexpr int NS = NB <= 4 ? 8 : (NB == 8 ? 6 : 4);
  static constexpr int W_BYTES = 4096;  // INT8 tile, or half of a 16-bit tile
  // stage: weight tile, activation tile (BN x 64 bytes; BN x 128 for the fused
  // quantizer's 16-bit input) and, fused only, the quantized INT8 activation tile
  __host__ __device__ static constexpr int stage_bytes(bool fused) { return W_BYTES + (fused ? BN * 192 : BN * 64); }
  static constexpr int PART_BYTES = BN * 64 * 4;
  __host__ __device__ static constexpr int ring_bytes(bool fused) {
    return NS * stage_bytes(fused) > PART_BYTES ? NS * stage_bytes(fused) : PART_BYTES;
  }
  // ring + barriers + per-stage scale + per-row and per-step metadata + sx table
  static size_t smem_bytes(bool fused, int n_tc, int rows_per_cta) {
    return ring_bytes(fused) + 20 * NS + (size_t)(rows_per_cta + 1) * 16 + (size_t)rows_per_cta * 2 * n_tc * 12 +
           (size_t)n_tc * 4 + 256;
  }
};

__device__ __forceinline__ uint4 lds128(const void* p) { return *reinterpret_cast<const uint4*>(p); }

// Exact f32 of an int32 |v| < 2^22 without the quarter-rate I2F: the integer add
// places v in the mantissa of 2^23 + 2^22, the float subtract removes the offset.
__device__ __forceinline__ float i2f_exact(int v) { return __fsub_rn(__int_as_float(v + 0x4B400000), 12582912.0f); }

template <int NB, int XT>
__global__ void __launch_bounds__(160) rows_kernel(const RowsArgs a, const __grid_constant__ RowsMaps maps) {
  using C = RowsCfg<NB>;
  constexpr int BN = C::BN, NS = C::NS;
  extern __shared__ __align__(128) uint8_t smem[];
  const bool fused = a.fused != 0;
  const int SB = C::stage_bytes(fused);
  const int R = a.rows_per_cta;
  uint8_t* stages = smem;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + C::ring_bytes(fused));
  uint64_t* empty = full + NS;
  float* st_scale = reinterpret_cast<float*>(empty + NS);  // NS: sx*sw of the step in each stage
  int* row_start = reinterpret_cast<int*>(st_scale + NS);  // R+1: first step of each row tile
  int* row_lo8 = row_start + (R + 1);                      // R: first INT8 list position
  int* row_n8 = row_lo8 + R;                               // R: INT8 steps
  int* row_lo16 = row_n8 + R;                              // R: first 16-bit list position
  int* it_c = row_lo16 + R;                                // steps: column tile
  int* it_pos = it_c + R * 2 * a.n_tc;                     // steps: >= 0 INT8 position, < 0 16-bit half
  float* it_s = reinterpret_cast<float*>(it_pos + R * 2 * a.n_tc);  // steps: sw of INT8 steps
  float* sx_s = it_s + R * 2 * a.n_tc;                              // n_tc
  __shared__ float red[4];

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, g = lane >> 2, t = lane & 3;
  const int r0 = blockIdx.x * R;
  const int rows = min(R, a.n_tr - r0);  // row tiles of this CTA
  const int n0 = blockIdx.y * BN;
  const int s = blockIdx.z, S = a.split;
  const bool tma_x = a.tma_x != 0;

  // ---- this CTA's slice of each row tile's INT8 and 16-bit lists (reference
  //      :121-124, :140-143); 16-bit tiles are streamed in two 32-column halves
  if (tid < rows) {
    const int r = r0 + tid;
    const int b8 = __ldg(a.rp8 + r), c8 = __ldg(a.rp8 + r + 1) - b8;
    const int lo8 = b8 + (c8 * s) / S, hi8 = b8 + (c8 * (s + 1)) / S;
    int lo16 = 0, n16 = 0;
    if (a.has_fp16) {
      const int b16 = __ldg(a.rp16 + r), c16 = __ldg(a.rp16 + r + 1) - b16;
      lo16 = b16 + (c16 * s) / S;
      n16 = b16 + (c16 * (s + 1)) / S - lo16;
    }
    row_lo8[tid] = lo8;
    row_n8[tid] = hi8 - lo8;
    row_lo16[tid] = lo16;
    row_start[tid + 1] = (hi8 - lo8) + 2 * n16;  // step count, turned into offsets below
  }
  __syncthreads();
  if (tid == 0) {
    row_start[0] = 0;
    for (int j = 0; j < rows; ++j) row_start[j + 1] += row_start[j];
  }
  __syncthreads();
  const int nitems = row_start[rows];

  auto item_pos = [&](int i) {  // list position of step i: >= 0 INT8, < 0 16-bit half
    int j = 0;
    while (i >= row_start[j + 1]) ++j;
    const int li = i - row_start[j];
    if (li < row_n8[j]) return row_lo8[j] + li;
    const int h = li - row_n8[j];
    return -((row_lo16[j] + (h >> 1)) * 2 + (h & 1)) - 1;
  };
  auto issue_w = [&](int pos, int stg) {  // one lane
    uint8_t* wdst = stages + stg * SB;
    mbar_add_tx(&full[stg], 4096);
    if (pos >= 0) {
      bulk_g2s(wdst, a.w8 + (int64_t)pos * 4096, 4096, &full[stg]);
    } else {
      const int hp = -pos - 1;
      tma_load_2d(wdst, &maps.w16_half, (hp & 1) * 32, (hp >> 1) * 64, &full[stg]);
    }
  };

  if (warp == 4 && lane == 0) {
    const int cnt = 1 + (tma_x ? 0 : 32);
    for (int i = 0; i < NS; ++i) {
      mbar_init(&full[i], cnt);
      mbar_init(&empty[i], 4);
    }
    fence_mbar_init();
    if (tma_x) {  // only the maps the host encoded
      if (a.x_i8 && !fused) prefetch_tensormap(&maps.x8);
      if (a.x_fp) prefetch_tensormap(&maps.xfp_half);
      if (a.x_fp && fused) prefetch_tensormap(&maps.xfp_full);
    }
    if (a.has_fp16) prefetch_tensormap(&maps.w16_half);
    // weights do not depend on the preceding kernel: start streaming them now
    for (int i = 0; i < NS && i < nitems; ++i) issue_w(item_pos(i), i);
  }
  // ---- per-step metadata
  for (int i = tid; i < nitems; i += 160) {
    const int pos = item_pos(i);
    it_pos[i] = pos;
    if (pos >= 0) {
      it_c[i] = __ldg(a.ids8 + pos) % a.n_tc;
      it_s[i] = a.s8 ? __ldg(a.s8 + pos) : 1.0f;
    } else {
      it_c[i] = __ldg(a.ids16 + ((-pos - 1) >> 1)) % a.n_tc;
    }
  }
  __syncthreads();

  const int rows_here = min(BN, a.n_rows - n0);
  bool ok = true;

  if (warp == 4) {
    // ================================================================ producer
    grid_dep_wait();  // activations and their scales come from the preceding kernel
    // With tensor maps, the activation copies of the first ring's worth of steps go out
    // before the scales are read, so the two global round trips overlap; the stage's
    // arrival (which publishes its scale) follows the scale.
    const int early = tma_x ? min(nitems, NS) : 0;
    if (lane == 0) {
      for (int i = 0; i < early; ++i) {
        const int pos = it_pos[i], c = it_c[i];
        uint8_t* adst = stages + i * SB + C::W_BYTES;
        if (pos >= 0 && fused) {
          mbar_add_tx(&full[i], BN * 128);
          tma_load_2d(adst, &maps.xfp_full, c * 64, n0, &full[i]);
        } else if (pos >= 0) {
          mbar_add_tx(&full[i], BN * 64);
          tma_load_2d(adst, &maps.x8, c * 64, n0, &full[i]);
        } else {
          mbar_add_tx(&full[i], BN * 64);
          tma_load_2d(adst, &maps.xfp_half, c * 64 + ((-pos - 1) & 1) * 32, n0, &full[i]);
        }
      }
    }
    if (!fused) {
      for (int c = lane; c < a.n_tc; c += 32) sx_s[c] = a.sx ? __ldg(a.sx + c) : 1.0f;
      __syncwarp();
    }
    if (lane == 0) {
      for (int i = 0; i < early; ++i) {
        if (it_pos[i] >= 0 && !fused) st_scale[i] = sx_s[it_c[i]] * it_s[i];  // (sx * sw) in f32, ref :135-137
        mbar_arrive(&full[i]);
      }
    }
#pragma unroll 1
    for (int i = early; i < nitems; ++i) {
      const int stg = i % NS;
      const int pos = it_pos[i];
      if (i >= NS) {
        if (ok && !mbar_wait_bounded(&empty[stg], (uint32_t)(((i / NS) - 1) & 1), a.err)) ok = false;
        if (lane == 0) issue_w(pos, stg);
      }
      uint8_t* adst = stages + stg * SB + C::W_BYTES;
      const int c = it_c[i];
      const bool q8 = pos >= 0;
      const int half = q8 ? 0 : ((-pos - 1) & 1);
      if (lane == 0 && q8 && !fused) st_scale[stg] = sx_s[c] * it_s[i];  // (sx * sw) in f32, ref :135-137
      if (tma_x) {
        if (lane == 0) {
          if (q8 && fused) {
            mbar_expect_tx(&full[stg], BN * 128);
            tma_load_2d(adst, &maps.xfp_full, c * 64, n0, &full[stg]);
          } else if (q8) {
            mbar_expect_tx(&full[stg], BN * 64);
            tma_load_2d(adst, &maps.x8, c * 64, n0, &full[stg]);
          } else {
            mbar_expect_tx(&full[stg], BN * 64);
            tma_load_2d(adst, &maps.xfp_half, c * 64 + half * 32, n0, &full[stg]);
          }
        }
      } else {
        // lanes copy the activation tile: 16-byte cp.async with zero fill when rows are
        // 16-byte aligned (the copies arrive on the barrier as they land), byte copies
        // otherwise (then a plain arrival)
        const int bpr = (q8 && fused) ? 128 : 64;  // bytes per activation row
        const bool vec = (q8 && !fused) ? a.a8_vec != 0 : a.afp_vec != 0;
        for (int ch = lane; ch < BN * bpr / 16; ch += 32) {
          const int row = ch / (bpr / 16), off = (ch % (bpr / 16)) * 16;
          int nb = 0;
          const uint8_t* src;
          if (q8 && !fused) {
            const int col = c * 64 + off;
            nb = (row < rows_here) ? max(0, min(16, a.K - col)) : 0;
            src = reinterpret_cast<const uint8_t*>(a.x_i8) + (int64_t)(n0 + (nb ? row : 0)) * a.ld_x8 + (nb ? col : 0);
          } else {
            const int col = c * 64 + half * 32 + off / 2;
            nb = (row < rows_here) ? 2 * max(0, min(8, a.K - col)) : 0;
            src = reinterpret_cast<const uint8_t*>(a.x_fp) +
                  ((int64_t)(n0 + (nb ? row : 0)) * a.ld_xfp + (nb ? col : 0)) * 2;
          }
          if (vec) {
            cp_async16(adst + row * bpr + off, src, nb);
          } else {
            for (int e = 0; e < 16; ++e) adst[row * bpr + off + e] = e < nb ? src[e] : (uint8_t)0;
          }
        }
        if (vec) {
          cp_async_arrive_noinc(&full[stg]);
        } else {
          mbar_arrive(&full[stg]);
        }
        if (lane == 0) mbar_arrive(&full[stg]);
      }
    }
  } else {
    // ================================================================ consumers
    // Swap-AB: the weight tile is the MMA's M side (warp w owns weight rows 16w..16w+15
    // = output columns), the activation rows are the N side in NB blocks of 8.  Thread
    // (g, t) holds output columns 16w+g and 16w+g+8 for activation rows 8nb+2t, +1.
    grid_dep_wait();  // the output may still be read by the preceding kernel
    const int wr = 16 * warp + g;  // this thread's first weight row within the tile
    int i = 0;
#pragma unroll 1
    for (int j = 0; j < rows; ++j) {
      float acc[NB][4];
#pragma unroll
      for (int nb = 0; nb < NB; ++nb)
#pragma unroll
        for (int q = 0; q < 4; ++q) acc[nb][q] = 0.0f;
#pragma unroll 1
      for (; i < row_start[j + 1]; ++i) {
        const int stg = i % NS;
        const uint8_t* st = stages + stg * SB;
        if (ok && !mbar_wait_bounded(&full[stg], (uint32_t)((i / NS) & 1), a.err)) ok = false;
        const int pos = it_pos[i];
        if (pos >= 0) {
          const uint8_t* ax = st + C::W_BYTES;
          float scale;
          if (fused) {
            // quantize the 16-bit activation tile: absmax over all rows (zero fill does
            // not count), scale dtype(absmax/127), codes (quantize_activation.py:100-109)
            const uint8_t* af = st + C::W_BYTES;
            float m = 0.0f;
            for (int ch = tid; ch < BN * 8; ch += 128) {
              const uint4 raw = lds128(af + ch * 16);
              const uint32_t w4[4] = {raw.x, raw.y, raw.z, raw.w};
#pragma unroll
              for (int e = 0; e < 4; ++e) {
                m = fmaxf(m, fabsf(h2f((uint16_t)(w4[e] & 0xffffu), XT)));
                m = fmaxf(m, fabsf(h2f((uint16_t)(w4[e] >> 16), XT)));
              }
            }
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
            if (lane == 0) red[warp] = m;
            named_bar_sync(1, 128);
            m = fmaxf(fmaxf(red[0], red[1]), fmaxf(red[2], red[3]));
            const float sxc = m > 0.0f ? round16(__fdiv_rn(m, 127.0f), XT) : 1.0f;
            const float rc = __frcp_rn(sxc);
            uint8_t* aqw = const_cast<uint8_t*>(st) + C::W_BYTES + BN * 128;
            for (int ch = tid; ch < BN * 8; ch += 128) {
              const uint4 raw = lds128(af + ch * 16);
              const uint32_t w4[4] = {raw.x, raw.y, raw.z, raw.w};
              uint32_t o2[2] = {0u, 0u};
#pragma unroll
              for (int e = 0; e < 4; ++e) {
                const int lo = quant_code_fast(h2f((uint16_t)(w4[e] & 0xffffu), XT), sxc, rc);
                const int hi = quant_code_fast(h2f((uint16_t)(w4[e] >> 16), XT), sxc, rc);
                o2[e >> 1] |= ((uint32_t)(lo & 0xff) | ((uint32_t)(hi & 0xff) << 8)) << ((e & 1) * 16);
              }
              *reinterpret_cast<uint2*>(aqw + (ch >> 3) * 64 + (ch & 7) * 8) = make_uint2(o2[0], o2[1]);
            }
            named_bar_sync(1, 128);
            ax = aqw;
            scale = sxc * it_s[i];  // (sx * sw) in f32, reference :135-137
          } else {
            scale = st_scale[stg];
          }
          // A = weight rows wr and wr+8, B = activation row 8nb+g; 16 bytes per row per thread
          const uint4 wlo = lds128(st + wr * 64 + 16 * t);
          const uint4 whi = lds128(st + (wr + 8) * 64 + 16 * t);
#pragma unroll
          for (int nb = 0; nb < NB; ++nb) {
            const uint4 xb = lds128(ax + (nb * 8 + g) * 64 + 16 * t);
            int d[4] = {0, 0, 0, 0};
            mma_s8_16832(d, wlo.x, whi.x, wlo.y, whi.y, xb.x, xb.y);
            mma_s8_16832(d, wlo.z, whi.z, wlo.w, whi.w, xb.z, xb.w);
#pragma unroll
            for (int q = 0; q < 4; ++q) acc[nb][q] = __fadd_rn(acc[nb][q], __fmul_rn(i2f_exact(d[q]), scale));
            if (a.partials) {
              // d[q]: weight row wr + 8*(q>>1), activation row n0 + 8nb + 2t + (q&1)
              int32_t* base = a.partials + (int64_t)pos * a.n_rows * 64;
#pragma unroll
              for (int q = 0; q < 4; ++q) {
                const int row = n0 + nb * 8 + 2 * t + (q & 1);
                if (row < a.n_rows) base[(int64_t)row * 64 + wr + 8 * (q >> 1)] = d[q];
              }
            }
          }
        } else {
          // one 32-column half of a 16-bit tile: W rows and activation rows are 64 bytes
          const uint8_t* af = st + C::W_BYTES;
          const uint4 wlo = lds128(st + wr * 64 + 16 * t);
          const uint4 whi = lds128(st + (wr + 8) * 64 + 16 * t);
#pragma unroll
          for (int nb = 0; nb < NB; ++nb) {
            const uint4 xb = lds128(af + (nb * 8 + g) * 64 + 16 * t);
            mma_16816<XT>(acc[nb], wlo.x, whi.x, wlo.y, whi.y, xb.x, xb.y);
            mma_16816<XT>(acc[nb], wlo.z, whi.z, wlo.w, whi.w, xb.z, xb.w);
          }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[stg]);
      }
      const int r = r0 + j;
      if (S == 1) {
#pragma unroll
        for (int nb = 0; nb < NB; ++nb)
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            const int rr = n0 + nb * 8 + 2 * t + (q & 1), cc = r * 64 + wr + 8 * (q >> 1);
            if (rr < a.n_rows && cc < a.M && a.out) {
              const int ot = a.out_dtype;
              uint16_t y = f2h(acc[nb][q], ot);
              if (a.bias) y = f2h(h2f(y, ot) + h2f(reinterpret_cast<const uint16_t*>(a.bias)[cc], ot), ot);
              reinterpret_cast<uint16_t*>(a.out)[(int64_t)rr * a.ldo + cc] = y;
            }
          }
      } else {
        named_bar_sync(1, 128);  // every consumer is done reading the ring
        float* part = reinterpret_cast<float*>(stages);
#pragma unroll
        for (int nb = 0; nb < NB; ++nb)
#pragma unroll
          for (int q = 0; q < 4; ++q) part[(nb * 8 + 2 * t + (q & 1)) * 64 + wr + 8 * (q >> 1)] = acc[nb][q];
      }
    }
  }

  if (S > 1) {  // one row tile per CTA here
    cg::cluster_group cluster = cg::this_cluster();
    cluster.sync();
    const int rank = (int)cluster.block_rank();
    const float* part = reinterpret_cast<const float*>(stages);
    const int E = rows_here * 64;
    const int e0 = (E * rank) / S, e1 = (E * (rank + 1)) / S;
    for (int e = e0 + tid; e < e1; e += 160) {
      float v = *cluster.map_shared_rank(part + e, 0);
      for (int p = 1; p < S; ++p) v += *cluster.map_shared_rank(part + e, p);
      const int rr = n0 + e / 64, cc = r0 * 64 + (e % 64);
      if (cc < a.M && a.out) {
        const int ot = a.out_dtype;
        uint16_t y = f2h(v, ot);
        if (a.bias) y = f2h(h2f(y, ot) + h2f(reinterpret_cast<const uint16_t*>(a.bias)[cc], ot), ot);
        reinterpret_cast<uint16_t*>(a.out)[(int64_t)rr * a.ldo + cc] = y;
      }
    }
    cluster.sync();  // keep this CTA's partial alive until every peer has read it
  }
}

template <int NB, int XT>
static int configure_rows() {
  static uint64_t configured = 0;  // one bit per device
  int dev = 0;
  TQ_CUDA_TRY(cudaGetDevice(&dev));
  if (dev < 64 && !(configured & (1ull << dev))) {
    TQ_CUDA_TRY(cudaFuncSetAttribute(rows_kernel<NB, XT>, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024));
    TQ_CUDA_TRY(cudaFuncSetAttribute(rows_kernel<NB, XT>, cudaFuncAttributeNonPortableClusterSizeAllowed, 1));
    configured |= 1ull << dev;
  }
  return TQ_OK;
}

// Resident CTAs per SM of one kernel instance (cached per device and shared-memory size).
template <int NB, int XT>
static int rows_occupancy(size_t smem) {
  static int dev_cached = -1;
  static size_t smem_cached = 0;
  static int occ_cached = 1;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return 1;
  if (dev != dev_cached || smem != smem_cached) {
    int occ = 1;
    if (configure_rows<NB, XT>() != TQ_OK ||
        cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, rows_kernel<NB, XT>, 160, smem) != cudaSuccess || occ < 1)
      occ = 1;
    dev_cached = dev;
    smem_cached = smem;
    occ_cached = occ;
  }
  return occ_cached;
}

// Launch geometry: split S and row tiles per CTA R.  An explicit split is kept (R = 1).
// Otherwise the grid is sized to one wave of resident CTAs: with at least a wave of
// (row tile, row block) units, S = 1 and each CTA streams R consecutive row tiles; with
// fewer, S splits each row's list (power of two <= 16, >= 4 tiles per split) and the S
// CTAs of a row reduce through distributed shared memory.
template <int NB, int XT>
static void rows_plan(int n_tr, int n_blocks, int n_tc, bool fused, int& split, int& rpc) {
  using C = RowsCfg<NB>;
  const int units = n_tr * n_blocks;
  const int cap = rows_occupancy<NB, XT>(C::smem_bytes(fused, n_tc, 1)) * tq_sm_count();
  if (split > 0) {
    rpc = 1;
    return;
  }
  if (units >= cap) {
    split = 1;
    rpc = (units + cap - 1) / cap;
    // the larger per-CTA metadata must still leave the same residency
    while (rpc > 1 && rows_occupancy<NB, XT>(C::smem_bytes(fused, n_tc, rpc)) * tq_sm_count() * rpc < units) ++rpc;
    return;
  }
  rpc = 1;
  split = 1;
  while (split < 16 && units * split * 2 <= cap && n_tc / (split * 2) >= 4) split *= 2;
}

template <int NB, int XT>
static int launch_rows(RowsArgs& a, const RowsMaps& maps, int n_blocks, cudaStream_t st) {
  using C = RowsCfg<NB>;
  int rc = configure_rows<NB, XT>();
  if (rc) return rc;
  rows_plan<NB, XT>(a.n_tr, n_blocks, a.n_tc, a.fused != 0, a.split, a.rows_per_cta);
  if (a.split > 16) return tq_set_error(TQ_ERR_INVALID, "split_k must be in 1..16");
  const size_t smem = C::smem_bytes(a.fused != 0, a.n_tc, a.rows_per_cta);
  if (smem > 200 * 1024) return tq_set_error(TQ_ERR_UNSUPPORTED, "rows kernel: too many column tiles for shared memory");
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((a.n_tr + a.rows_per_cta - 1) / a.rows_per_cta, n_blocks, a.split);
  cfg.blockDim = dim3(160, 1, 1);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[2];
  int na = 0;
  if (a.split > 1) {
    attr[na].id = cudaLaunchAttributeClusterDimension;
    attr[na].val.clusterDim.x = 1;
    attr[na].val.clusterDim.y = 1;
    attr[na].val.clusterDim.z = a.split;
    ++na;
  }
  if (tq_pdl_enabled()) {
    attr[na].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[na].val.programmaticStreamSerializationAllowed = 1;
    ++na;
  }
  cfg.attrs = attr;
  cfg.numAttrs = na;
  TQ_CUDA_TRY(cudaLaunchKernelEx(&cfg, rows_kernel<NB, XT>, a, maps));
  tq_count_launch();
  return TQ_OK;
}

}  // namespace tq

using namespace tq;

// Token blocks of 8 per CTA (the MMA's N side): 8, 16, 32, 64 or 128 rows.
static int rows_nb(int64_t n_rows) {
  if (n_rows <= 8) return 1;
  if (n_rows <= 16) return 2;
  if (n_rows <= 32) return 4;
  if (n_rows <= 64) return 8;
  return 16;
}

// Tensor maps of the activation operands (absent -> lanes copy them) and of the 16-bit
// tile arena.
static int rows_maps(RowsArgs& a, int bn, int64_t t16, RowsMaps& m) {
  memset(&m, 0, sizeof(m));
  bool x_ok = true;
  if (a.x_i8 && !a.fused)
    x_ok = x_ok && tq_encode_2d(&m.x8, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, a.x_i8, a.K, a.n_rows, a.ld_x8, 64, bn,
                                CU_TENSOR_MAP_SWIZZLE_NONE) == TQ_OK;
  if (a.x_fp) {
    x_ok = x_ok && tq_encode_2d(&m.xfp_half, CU_TENSOR_MAP_DATA_TYPE_UINT16, 2, a.x_fp, a.K, a.n_rows, a.ld_xfp * 2, 32,
                                bn, CU_TENSOR_MAP_SWIZZLE_NONE) == TQ_OK;
    if (a.fused)
      x_ok = x_ok && tq_encode_2d(&m.xfp_full, CU_TENSOR_MAP_DATA_TYPE_UINT16, 2, a.x_fp, a.K, a.n_rows, a.ld_xfp * 2,
                                  64, bn, CU_TENSOR_MAP_SWIZZLE_NONE) == TQ_OK;
  }
  a.tma_x = x_ok ? 1 : 0;
  a.a8_vec = a.x_i8 && ((uintptr_t)a.x_i8 & 15) == 0 && a.ld_x8 % 16 == 0;
  a.afp_vec = a.x_fp && ((uintptr_t)a.x_fp & 15) == 0 && (a.ld_xfp * 2) % 16 == 0;
  if (t16 > 0 && tq_encode_2d(&m.w16_half, CU_TENSOR_MAP_DATA_TYPE_UINT16, 2, a.w16, 64, (uint64_t)t16 * 64, 128, 32,
                              64, CU_TENSOR_MAP_SWIZZLE_NONE) != TQ_OK)
    return tq_set_error(TQ_ERR_INVALID, "16-bit tile arena must be 16-byte aligned");
  return TQ_OK;
}

int tq_launch_rows(RowsArgs& a, int n_tr, int fp_dtype, cudaStream_t st, int64_t t16) {
  const int nb = rows_nb(a.n_rows);
  const int bn = 8 * nb;
  const int n_blocks = (a.n_rows + bn - 1) / bn;
  a.n_tr = n_tr;
  if (a.split < 0 || a.split > 16) return tq_set_error(TQ_ERR_INVALID, "split_k must be in 1..16");
  if (n_blocks > 65535) return tq_set_error(TQ_ERR_INVALID, "too many activation rows");
  RowsMaps maps;
  int rc = rows_maps(a, bn, t16, maps);
  if (rc) return rc;
#define TQ_ROWS_CASE(NB)                                                                      \
  case NB:                                                                                    \
    return fp_dtype == TQ_DTYPE_BF16 ? launch_rows<NB, TQ_DTYPE_BF16>(a, maps, n_blocks, st) \
                                     : launch_rows<NB, TQ_DTYPE_F16>(a, maps, n_blocks, st);
  switch (nb) {
    TQ_ROWS_CASE(1)
    TQ_ROWS_CASE(2)
    TQ_ROWS_CASE(4)
    TQ_ROWS_CASE(8)
    TQ_ROWS_CASE(16)
  }
#undef TQ_ROWS_CASE
  return tq_set_error(TQ_ERR_INVALID, "bad row block");
}

// The split and row tiles per CTA the rows kernel picks for a shape (split_k = 0).
int tq_stream_split(int n_tr, int n_tc, int n_rows);
int tq_gemv_split(int n_tc);
int tq_gemv_preferred(const tq::RowsArgs& a, int n_tr);

extern "C" int tq_gemm_rows_plan(int64_t n_rows, int n_tr, int n_tc, int fp_dtype, int fused, int* split, int* rows_per_cta) {
  if (n_rows <= 0 || n_tr <= 0 || n_tc <= 0 || !split || !rows_per_cta) return tq_set_error(TQ_ERR_INVALID, "bad plan query");
  if (n_rows <= 8) {  // the stream decode kernel (TQ_ALGO_STREAM), or the row kernel at its split
    *split = tq_stream_split(n_tr, n_tc, (int)n_rows);
    *rows_per_cta = 1;
    return TQ_OK;
  }
  if (n_rows <= 16 && !fused) {  // the register-fragment decode kernel (TQ_ALGO_GEMV) where it is chosen
    tq::RowsArgs a = {};
    a.n_rows = (int)n_rows;
    a.n_tc = n_tc;
    if (tq_gemv_preferred(a, n_tr)) {
      *split = tq_gemv_split(n_tc);
      *rows_per_cta = 1;
      return TQ_OK;
    }
  }
  const int nb = rows_nb(n_rows);
  const int n_blocks = (int)((n_rows + 8 * nb - 1) / (8 * nb));
  int sp = 0, rpc = 1;
#define TQ_PLAN_CASE(NB)                                                                         \
  case NB:                                                                                       \
    if (fp_dtype == TQ_DTYPE_BF16)                                                               \
      rows_plan<NB, TQ_DTYPE_BF16>(n_tr, n_blocks, n_tc, fused != 0, sp, rpc);                   \
    else                                                                                         \
      rows_plan<NB, TQ_DTYPE_F16>(n_tr, n_blocks, n_tc, fused != 0, sp, rpc);                    \
    break;
  switch (nb) {
    TQ_PLAN_CASE(1)
    TQ_PLAN_CASE(2)
    TQ_PLAN_CASE(4)
    TQ_PLAN_CASE(8)
    TQ_PLAN_CASE(16)
  }
#undef TQ_PLAN_CASE
  *split = sp;
  *rows_per_cta = rpc;
  return TQ_OK;
}

// Persistent TMA + tcgen05 mixed INT8/BF16 64x64 tile GEMM for prefill-sized row
// counts (sm_100a).
//
// Reference semantics: src/kernels/triton/gemm_rows_splitk_64x64.py:108-190 with
// SPLIT_K = 1: per output tile (128 activation rows x one 64-wide row tile r), the
// INT8 tiles of row r in ascending column order contribute
//     acc = fma(f32(i32 tile dot), sx[c] * sw[pos], acc)
// (the FP32 multiply-add the reference's `acc += tile_acc * (sx * sw)` compiles to
// with Triton's default FP contraction), then the 16-bit tiles add their FP32 dot,
// then the output rounding and bias of the reference.  The INT32 tile dot is exact.
//
// Design (at most two CTAs per SM, persistent over output tiles):
//   warp 0      TMA producer: per step a 128 x 64-byte activation tile and a 64 x
//               64-byte weight tile (an INT8 tile, or one 32-column half of a 16-bit
//               tile) land in a 6-stage shared-memory ring (1024-byte aligned,
//               SWIZZLE_64B, the UMMA canonical K-major layout);
//   warp 1      MMA issuer (one thread): two tcgen05.mma per step (K = 32 bytes each),
//               kind::i8 into one of two INT32 TMEM tiles (128 lanes x 64 columns), or
//               kind::f16 into an FP32 TMEM tile that accumulates all 16-bit tiles of
//               the output tile; tcgen05.commit frees the smem stage and publishes the
//               TMEM tile;
//   warps 2-9   epilogue: the INT32 TMEM tile is preset to the bits of 2^23 + 2^22, so
//               after the MMA adds the tile dot, the 32 bits read back ARE the float
//               2^23 + 2^22 + dot (exact for |dot| < 2^22; |dot| <= 64*128*128); one
//               packed f32x2 add recovers the dot, one packed f32x2 FMA rescales it
//               into the FP32 accumulator held in registers.  The epilogue rewrites the
//               preset after reading, so no integer conversion is ever needed.
//               8 warps = two per TMEM lane quadrant, each owning 32 of the 64 columns.
// TMEM: 256 columns per CTA: [0,64) and [64,128) INT32 tiles, [128,192) FP32 16-bit sum.
#include <string.h>

#include <algorithm>

#include "common.cuh"
#include "gemm_args.cuh"
#include "tma.cuh"

namespace tq {

namespace um {
constexpr int BM = 128;            // activation rows per output tile (MMA M)
constexpr int NS = 6;              // shared-memory stages
constexpr int A_BYTES = BM * 64;   // 8 KB
constexpr int B_BYTES = 64 * 64;   // 4 KB
constexpr int STAGE = A_BYTES + B_BYTES;
constexpr int THREADS = 320;       // 10 warps
constexpr int TMEM_COLS = 256;
constexpr uint32_t MAGIC = 0x4B400000u;  // bits of 2^23 + 2^22
constexpr float MAGIC_F = 12582912.0f;

// tcgen05 instruction descriptors: M = 128, N = 64, K-major A and B.
constexpr uint32_t idesc(uint32_t c_fmt, uint32_t ab_fmt) {
  return (c_fmt << 4) | (ab_fmt << 7) | (ab_fmt << 10) | ((64u >> 3) << 17) | ((128u >> 4) << 24);
}
constexpr uint32_t IDESC_I8 = idesc(2 /*S32*/, 1 /*S8*/);
constexpr uint32_t IDESC_BF16 = idesc(1 /*F32*/, 1 /*BF16*/);
constexpr uint32_t IDESC_F16 = idesc(1 /*F32*/, 0 /*F16*/);

inline size_t smem_bytes(int n_tc) {
  return 1024 /*alignment*/ + (size_t)NS * STAGE + 256 /*barriers*/ + (size_t)n_tc * 4 * 4 + 256;
}
}  // namespace um

struct UmmaMaps {
  CUtensorMap x8;   // x_int8 [n_rows][K], box 64 x 128, SWIZZLE_64B
  CUtensorMap xfp;  // x_fp   [n_rows][K], box 32 x 128 elements, SWIZZLE_64B
  CUtensorMap w8;   // INT8 arena [T8*64][64], box 64 x 64, SWIZZLE_64B
  CUtensorMap w16;  // 16-bit arena [T16*64][64], box 32 x 64 elements, SWIZZLE_64B
};

// K-major, SWIZZLE_64B shared-memory matrix descriptor: rows of 64 bytes, 8-row groups
// 512 bytes apart (SBO), leading offset 1 (unused by swizzled K-major), version 1.
__device__ __forceinline__ uint64_t sw64_desc(uint32_t saddr) {
  return (uint64_t)((saddr >> 4) & 0x3FFFu) | ((uint64_t)1 << 16) | ((uint64_t)(512 >> 4) << 32) | ((uint64_t)1 << 46) |
         ((uint64_t)4 << 61);
}

__device__ __forceinline__ void umma(uint32_t d_tmem, uint64_t a, uint64_t b, uint32_t idesc, uint32_t accumulate,
                                     bool i8) {
  if (i8) {
    asm volatile(
        "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
        " tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, {%5, %6, %7, %8}, p;\n}\n" ::"r"(d_tmem),
        "l"(a), "l"(b), "r"(idesc), "r"(accumulate), "r"(0), "r"(0), "r"(0), "r"(0));
  } else {
    asm volatile(
        "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
        " tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, {%5, %6, %7, %8}, p;\n}\n" ::"r"(d_tmem),
        "l"(a), "l"(b), "r"(idesc), "r"(accumulate), "r"(0), "r"(0), "r"(0), "r"(0));
  }
}

__device__ __forceinline__ void umma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// 16 consecutive TMEM columns of this thread's lane.
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&v)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]), "=r"(v[8]),
        "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

// Write the same 32-bit value into 32 consecutive TMEM columns of this thread's lane.
__device__ __forceinline__ void tmem_fill32(uint32_t taddr, uint32_t x) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,"
      "%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1};" ::"r"(taddr),
      "r"(x)
      : "memory");
  asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}

template <int XT>
__global__ void __launch_bounds__(um::THREADS, 2) umma_kernel(const RowsArgs a, const __grid_constant__ UmmaMaps maps) {
  using namespace um;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
  uint8_t* stages = smem;  // NS x (A 8 KB | B 4 KB), every tile 1024-byte aligned
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + NS * STAGE);
  uint64_t* sempty = full + NS;
  uint64_t* tfull = sempty + NS;  // [2]
  uint64_t* tempty = tfull + 2;   // [2]
  uint64_t* bfull = tempty + 2;
  uint64_t* bempty = bfull + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bempty + 1);
  float* sx_s = reinterpret_cast<float*>(smem + NS * STAGE + 256);  // n_tc
  int* pr_c = reinterpret_cast<int*>(sx_s + a.n_tc);                // 2 * n_tc: producer's column per step
  float* ep_s = reinterpret_cast<float*>(pr_c + 2 * a.n_tc);        // n_tc: epilogue's scale per INT8 step

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int n_tb = (a.n_rows + BM - 1) / BM;
  const int tiles = n_tb * a.n_tr;

  if (tid == 0) {
    for (int i = 0; i < NS; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&sempty[i], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&tfull[b], 1);
      mbar_init(&tempty[b], 8);
    }
    mbar_init(bfull, 1);
    mbar_init(bempty, 8);
    fence_mbar_init();
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"(TMEM_COLS)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  if (warp == 0 && lane == 0) {
    prefetch_tensormap(&maps.w8);
    if (a.has_fp16) prefetch_tensormap(&maps.w16);
    if (a.x_i8) prefetch_tensormap(&maps.x8);
    if (a.has_fp16) prefetch_tensormap(&maps.xfp);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  grid_dep_wait();  // activations and scales come from the preceding kernel
  for (int c = tid; c < a.n_tc; c += um::THREADS) sx_s[c] = a.sx ? __ldg(a.sx + c) : 1.0f;
  __syncthreads();
  bool ok = true;

  if (warp == 0) {
    // ================================================================ TMA producer
    uint32_t g = 0;  // global step counter
    for (int tile = blockIdx.x; tile < tiles; tile += gridDim.x) {
      const int r = tile % a.n_tr, tb = tile / a.n_tr;
      const int b8 = __ldg(a.rp8 + r), n8 = __ldg(a.rp8 + r + 1) - b8;
      int b16 = 0, n16 = 0;
      if (a.has_fp16) {
        b16 = __ldg(a.rp16 + r);
        n16 = __ldg(a.rp16 + r + 1) - b16;
      }
      const int nit = n8 + 2 * n16;
      __syncwarp();  // lane 0 has issued every step of the previous tile
      for (int i = lane; i < nit; i += 32)
        pr_c[i] = (i < n8 ? __ldg(a.ids8 + b8 + i) : __ldg(a.ids16 + b16 + ((i - n8) >> 1))) % a.n_tc;
      __syncwarp();
      if (lane == 0) {
        for (int i = 0; i < nit; ++i, ++g) {
          const int stg = g % NS;
          if (ok && !mbar_wait_bounded(&sempty[stg], ((g / NS) & 1) ^ 1, a.err)) ok = false;
          uint8_t* sa = stages + stg * STAGE;
          uint8_t* sb = sa + A_BYTES;
          mbar_expect_tx(&full[stg], STAGE);
          const int c = pr_c[i];
          if (i < n8) {
            tma_load_2d(sa, &maps.x8, c * 64, tb * BM, &full[stg]);
            tma_load_2d(sb, &maps.w8, 0, (b8 + i) * 64, &full[stg]);
          } else {
            const int j = i - n8, h = j & 1;
            tma_load_2d(sa, &maps.xfp, c * 64 + h * 32, tb * BM, &full[stg]);
            tma_load_2d(sb, &maps.w16, h * 32, (b16 + (j >> 1)) * 64, &full[stg]);
          }
        }
      }
    }
  } else if (warp == 1) {
    // ================================================================ MMA issuer
    if (lane == 0) {
      uint32_t g = 0, k8 = 0, nbf = 0;
      const uint32_t idesc16 = XT == TQ_DTYPE_BF16 ? IDESC_BF16 : IDESC_F16;
      for (int tile = blockIdx.x; tile < tiles; tile += gridDim.x) {
        const int r = tile % a.n_tr;
        const int n8 = __ldg(a.rp8 + r + 1) - __ldg(a.rp8 + r);
        const int n16 = a.has_fp16 ? __ldg(a.rp16 + r + 1) - __ldg(a.rp16 + r) : 0;
        const int nit = n8 + 2 * n16;
        for (int i = 0; i < nit; ++i, ++g) {
          const int stg = g % NS;
          if (ok && !mbar_wait_bounded(&full[stg], (g / NS) & 1, a.err)) ok = false;
          tc_fence_after();
          const uint32_t sa = smem_u32(stages + stg * STAGE);
          const uint64_t da = sw64_desc(sa), db = sw64_desc(sa + A_BYTES);
          if (i < n8) {
            const uint32_t b = k8 & 1;
            if (ok && !mbar_wait_bounded(&tempty[b], (k8 >> 1) & 1, a.err)) ok = false;
            tc_fence_after();
            // the TMEM tile holds the preset; both K halves accumulate onto it
            umma(tmem + b * 64, da, db, IDESC_I8, 1, true);
            umma(tmem + b * 64, da + 2, db + 2, IDESC_I8, 1, true);
            umma_commit(&sempty[stg]);
            umma_commit(&tfull[b]);
            ++k8;
          } else {
            if (i == n8) {
              if (ok && !mbar_wait_bounded(bempty, nbf & 1, a.err)) ok = false;
              tc_fence_after();
            }
            umma(tmem + 128, da, db, idesc16, i == n8 ? 0 : 1, false);
            umma(tmem + 128, da + 2, db + 2, idesc16, 1, false);
            umma_commit(&sempty[stg]);
            if (i == nit - 1) {
              umma_commit(bfull);
              ++nbf;
            }
          }
        }
      }
    }
  } else {
    // ================================================================ epilogue
    const int ew = warp - 2;    // 0..7
    const int q = warp & 3;     // TMEM lane quadrant this warp may access
    const int half = ew >> 2;   // which 32 of the 64 columns
    const uint32_t lane_base = (uint32_t)(q * 32) << 16;
    const int et = tid - 64;    // 0..255
    // preset both INT32 tiles, then hand them (and the FP32 tile) to the MMA issuer
    tmem_fill32(tmem + lane_base + 0 * 64 + half * 32, MAGIC);
    tmem_fill32(tmem + lane_base + 1 * 64 + half * 32, MAGIC);
    tc_fence_before();
    __syncwarp();
    if (lane == 0) {
      mbar_arrive(&tempty[0]);
      mbar_arrive(&tempty[1]);
      mbar_arrive(bempty);
    }
    uint32_t k8 = 0, nbf = 0;
    const float2 neg_magic = make_float2(-MAGIC_F, -MAGIC_F);
    for (int tile = blockIdx.x; tile < tiles; tile += gridDim.x) {
      const int r = tile % a.n_tr, tb = tile / a.n_tr;
      const int b8 = __ldg(a.rp8 + r), n8 = __ldg(a.rp8 + r + 1) - b8;
      const int n16 = a.has_fp16 ? __ldg(a.rp16 + r + 1) - __ldg(a.rp16 + r) : 0;
      named_bar_sync(1, 256);  // every epilogue thread is done with the previous tile's scales
      for (int i = et; i < n8; i += 256)
        ep_s[i] = sx_s[__ldg(a.ids8 + b8 + i) % a.n_tc] * (a.s8 ? __ldg(a.s8 + b8 + i) : 1.0f);
      named_bar_sync(1, 256);
      float2 acc[16];
#pragma unroll
      for (int j = 0; j < 16; ++j) acc[j] = make_float2(0.0f, 0.0f);
      const int row = tb * BM + q * 32 + lane;  // this thread's activation row
      for (int i = 0; i < n8; ++i, ++k8) {
        const uint32_t b = k8 & 1;
        if (ok && !mbar_wait_bounded(&tfull[b], (k8 >> 1) & 1, a.err)) ok = false;
        tc_fence_after();
        const uint32_t taddr = tmem + lane_base + b * 64 + half * 32;
        const float s = ep_s[i];
        const float2 s2 = make_float2(s, s);
#pragma unroll
        for (int part = 0; part < 2; ++part) {
          uint32_t v[16];
          tmem_ld16(taddr + part * 16, v);
#pragma unroll
          for (int j = 0; j < 8; ++j) {
            const float2 m = make_float2(__uint_as_float(v[2 * j]), __uint_as_float(v[2 * j + 1]));
            const float2 d = __fadd2_rn(m, neg_magic);  // exact: the tile dot as f32
            acc[part * 8 + j] = __ffma2_rn(d, s2, acc[part * 8 + j]);
          }
          if (a.partials && row < a.n_rows) {
            int32_t* base = a.partials + ((int64_t)(b8 + i) * a.n_rows + row) * 64 + half * 32 + part * 16;
#pragma unroll
            for (int j = 0; j < 16; ++j) base[j] = (int32_t)(v[j] - MAGIC);
          }
        }
        tmem_fill32(taddr, MAGIC);
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&tempty[b]);
      }
      if (n16 > 0) {
        if (ok && !mbar_wait_bounded(bfull, nbf & 1, a.err)) ok = false;
        tc_fence_after();
#pragma unroll
        for (int part = 0; part < 2; ++part) {
          uint32_t v[16];
          tmem_ld16(tmem + lane_base + 128 + half * 32 + part * 16, v);
#pragma unroll
          for (int j = 0; j < 8; ++j)
            acc[part * 8 + j] =
                __fadd2_rn(acc[part * 8 + j], make_float2(__uint_as_float(v[2 * j]), __uint_as_float(v[2 * j + 1])));
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(bempty);
        ++nbf;
      }
      if (row < a.n_rows && a.out) {
        const int col0 = r * 64 + half * 32;
        const int ot = a.out_dtype;
        uint16_t* orow = reinterpret_cast<uint16_t*>(a.out) + (int64_t)row * a.ldo + col0;
        const uint16_t* brow = a.bias ? reinterpret_cast<const uint16_t*>(a.bias) + col0 : nullptr;
        uint32_t packed[16];
#pragma unroll
        for (int j = 0; j < 16; ++j) {
          uint16_t y0 = f2h(acc[j].x, ot), y1 = f2h(acc[j].y, ot);
          if (brow) {
            if (col0 + 2 * j < a.M) y0 = f2h(h2f(y0, ot) + h2f(brow[2 * j], ot), ot);
            if (col0 + 2 * j + 1 < a.M) y1 = f2h(h2f(y1, ot) + h2f(brow[2 * j + 1], ot), ot);
          }
          packed[j] = (uint32_t)y0 | ((uint32_t)y1 << 16);
        }
        const bool full_row = col0 + 32 <= a.M && (((uintptr_t)orow) & 15) == 0;
        if (full_row) {
#pragma unroll
          for (int j = 0; j < 4; ++j)
            reinterpret_cast<uint4*>(orow)[j] =
                make_uint4(packed[4 * j], packed[4 * j + 1], packed[4 * j + 2], packed[4 * j + 3]);
        } else {
          for (int j = 0; j < 32 && col0 + j < a.M; ++j) orow[j] = (uint16_t)(packed[j >> 1] >> ((j & 1) * 16));
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(TMEM_COLS) : "memory");
  }
}

template <int XT>
static int launch_umma_t(const RowsArgs& a, const UmmaMaps& maps, cudaStream_t st) {
  static uint64_t configured = 0;
  int dev = 0;
  TQ_CUDA_TRY(cudaGetDevice(&dev));
  if (dev < 64 && !(configured & (1ull << dev))) {
    TQ_CUDA_TRY(cudaFuncSetAttribute(umma_kernel<XT>, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024));
    configured |= 1ull << dev;
  }
  // at least 100 KB so no more than two CTAs (2 x 256 TMEM columns) share an SM
  const size_t smem = std::max<size_t>(um::smem_bytes(a.n_tc), 100 * 1024);
  if (smem > 200 * 1024) return tq_set_error(TQ_ERR_UNSUPPORTED, "tcgen05 GEMM: too many column tiles");
  const int n_tb = (a.n_rows + um::BM - 1) / um::BM;
  const int64_t tiles = (int64_t)n_tb * a.n_tr;
  int occ = 1;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, umma_kernel<XT>, um::THREADS, smem) != cudaSuccess || occ < 1)
    occ = 1;
  occ = std::min(occ, 2);
  const int64_t grid = std::min<int64_t>(tiles, (int64_t)occ * tq_sm_count());
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)grid, 1, 1);
  cfg.blockDim = dim3(um::THREADS, 1, 1);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  int na = 0;
  if (tq_pdl_enabled()) {
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    na = 1;
  }
  cfg.attrs = attr;
  cfg.numAttrs = na;
  TQ_CUDA_TRY(cudaLaunchKernelEx(&cfg, umma_kernel<XT>, a, maps));
  tq_count_launch();
  return TQ_OK;
}

}  // namespace tq

using namespace tq;

int tq_umma_supported(int64_t n_rows, int64_t m, int64_t k, const int8_t* x_i8, int64_t ld_x8, const void* x_fp,
                      int64_t ld_xfp, const void* w8, const void* w16) {
  (void)m;
  if (n_rows <= 0 || k <= 0 || n_rows > (int64_t)INT32_MAX / 2) return 0;
  if (x_i8 && ((((uintptr_t)x_i8) & 15) || (ld_x8 & 15))) return 0;
  if (x_fp && ((((uintptr_t)x_fp) & 15) || ((ld_xfp * 2) & 15))) return 0;
  if ((w8 && (((uintptr_t)w8) & 15)) || (w16 && (((uintptr_t)w16) & 15))) return 0;
  if (um::smem_bytes((int)((k + 63) / 64)) > 200 * 1024) return 0;
  return 1;
}

int tq_launch_umma(const RowsArgs& a_in, int n_tr, int fp_dtype, cudaStream_t st) {
  RowsArgs a = a_in;
  a.n_tr = n_tr;
  a.split = 1;
  UmmaMaps maps;
  memset(&maps, 0, sizeof(maps));
  if (a.x_i8 && tq_encode_2d(&maps.x8, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, a.x_i8, a.K, a.n_rows, a.ld_x8, 64, um::BM,
                             CU_TENSOR_MAP_SWIZZLE_64B) != TQ_OK)
    return tq_set_error(TQ_ERR_UNSUPPORTED, "tcgen05 GEMM: x_int8 tensor map");
  if (a.has_fp16 && tq_encode_2d(&maps.xfp, CU_TENSOR_MAP_DATA_TYPE_UINT16, 2, a.x_fp, a.K, a.n_rows, a.ld_xfp * 2,
                                 32, um::BM, CU_TENSOR_MAP_SWIZZLE_64B) != TQ_OK)
    return tq_set_error(TQ_ERR_UNSUPPORTED, "tcgen05 GEMM: x_fp tensor map");
  if (a.w8_rows > 0 && tq_encode_2d(&maps.w8, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, a.w8, 64, (uint64_t)a.w8_rows, 64, 64,
                                    64, CU_TENSOR_MAP_SWIZZLE_64B) != TQ_OK)
    return tq_set_error(TQ_ERR_UNSUPPORTED, "tcgen05 GEMM: INT8 tile tensor map");
  if (a.has_fp16 && tq_encode_2d(&maps.w16, CU_TENSOR_MAP_DATA_TYPE_UINT16, 2, a.w16, 64, (uint64_t)a.w16_rows, 128,
                                 32, 64, CU_TENSOR_MAP_SWIZZLE_64B) != TQ_OK)
    return tq_set_error(TQ_ERR_UNSUPPORTED, "tcgen05 GEMM: 16-bit tile tensor map");
  return fp_dtype == TQ_DTYPE_BF16 ? launch_umma_t<TQ_DTYPE_BF16>(a, maps, st) : launch_umma_t<TQ_DTYPE_F16>(a, maps, st);
}

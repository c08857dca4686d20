// Persistent TMA + tcgen05 mixed INT8/BF16 64x64 tile GEMM for prefill-sized row
// counts (sm_100a).
//
// Reference semantics: src/kernels/triton/gemm_rows_splitk_64x64.py:108-190 with
// SPLIT_K = 1: for every output row tile r, its INT8 tiles in ascending column order
// contribute  acc = fma(f32(i32 tile dot), sx[c] * sw[pos], acc)  (the FP32
// multiply-add the reference's `acc += tile_acc * (sx * sw)` compiles to with Triton's
// default FP contraction); then the 16-bit tiles add their FP32 dot; then the output
// rounding and bias of the reference.  The INT32 tile dot is exact.
//
// Output tile = 128 activation rows x two row tiles (128 output columns).  The K loop
// runs over the n_tc input-column tiles: one 128 x 64-byte activation tile and, stacked,
// the two row tiles' 64 x 64 INT8 weight tiles make one N = 128 tcgen05.mma step (a
// row tile whose tile at that column is 16-bit, or that does not exist, is loaded as an
// out-of-bounds TMA box, i.e. zeros, and its step is skipped in the rescale, so each row
// tile still sees exactly its own INT8 tiles in ascending order).  The 16-bit tiles of
// each row tile then run as N = 64 kind::f16 MMAs into an FP32 TMEM accumulator.
//
// Warp roles (one CTA per SM, persistent over output tiles, 11 warps):
//   warp 0      TMA producer (one thread): 10-stage shared-memory ring, 16 KB per stage,
//               SWIZZLE_64B (the UMMA canonical K-major layout);
//   warp 1      MMA issuer (one thread); tcgen05.commit frees stages and publishes tiles;
//   warp 2      scheduler: builds each output tile's column table (INT8 list position
//               and combined scale sx*sw of both row tiles at every column, 16-bit tile
//               columns) one tile ahead into a 2-slot ring, so no role stalls on the
//               id lists;
//   warps 3-10  epilogue: two per TMEM lane quadrant, one per row tile (64 columns).
//               The INT32 TMEM tiles are preset to the bits of 2^23 + 2^22, so after the
//               MMA adds the tile dot the 32 bits read back ARE the float 2^23 + 2^22 +
//               dot (exact: |dot| <= 64*128*128 < 2^22); a packed f32x2 add recovers the
//               dot, a packed f32x2 FMA rescales it into the FP32 accumulator held in
//               registers; the preset is rewritten after every read.
// TMEM (512 columns): [0,128) and [128,256) INT32 tiles (double buffer), [256,384) FP32
// 16-bit sums of the two row tiles.
#include <string.h>

#include <algorithm>

#include "common.cuh"
#include "gemm_args.cuh"
#include "tma.cuh"

namespace tq {

namespace um {
constexpr int BM = 128;             // activation rows per output tile (MMA M)
constexpr int NS = 10;              // shared-memory stages
constexpr int A_BYTES = BM * 64;    // 8 KB activation tile
constexpr int W_BYTES = 64 * 64;    // 4 KB weight tile
constexpr int STAGE = A_BYTES + 2 * W_BYTES;
constexpr int THREADS = 352;        // 11 warps
constexpr int EPI_WARP0 = 3;
constexpr int TMEM_COLS = 512;
constexpr uint32_t MAGIC = 0x4B400000u;  // bits of 2^23 + 2^22
constexpr float MAGIC_F = 12582912.0f;

// tcgen05 instruction descriptors: M = 128, K-major A and B.
constexpr uint32_t idesc(uint32_t c_fmt, uint32_t ab_fmt, uint32_t n) {
  return (c_fmt << 4) | (ab_fmt << 7) | (ab_fmt << 10) | ((n >> 3) << 17) | ((128u >> 4) << 24);
}
constexpr uint32_t IDESC_I8 = idesc(2 /*S32*/, 1 /*S8*/, 128);
constexpr uint32_t IDESC_BF16 = idesc(1 /*F32*/, 1 /*BF16*/, 64);
constexpr uint32_t IDESC_F16 = idesc(1 /*F32*/, 0 /*F16*/, 64);

// column table slot: pos[2][n_tc] int, scale[2][n_tc] float, bcol[2][n_tc] int, header
__host__ __device__ inline size_t table_bytes(int n_tc) { return (size_t)n_tc * 24 + 64; }
inline size_t smem_bytes(int n_tc) { return 1024 + (size_t)NS * STAGE + 512 + 2 * table_bytes(n_tc) + (size_t)n_tc * 4; }
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

// 16 consecutive TMEM columns of this thread's lane (no wait).
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t* v) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]), "=r"(v[8]),
        "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15])
      : "r"(taddr));
}
__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }
__device__ __forceinline__ void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// The same 32-bit value into 32 consecutive TMEM columns of this thread's lane (no wait).
__device__ __forceinline__ void tmem_fill32(uint32_t taddr, uint32_t x) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,"
      "%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1};" ::"r"(taddr),
      "r"(x)
      : "memory");
}

struct TileHdr {
  int tb, r0, n_r;    // token block, first row tile, row tiles present (1 or 2)
  int n16[2];         // 16-bit tiles of each row tile
  int b16[2];         // first 16-bit list position of each row tile
};

template <int XT>
__global__ void __launch_bounds__(um::THREADS, 1) umma_kernel(const RowsArgs a, const __grid_constant__ UmmaMaps maps) {
  using namespace um;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
  const int n_tc = a.n_tc;
  uint8_t* stages = smem;  // NS x (A 8 KB | W0 4 KB | W1 4 KB), 1024-byte aligned
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + NS * STAGE);
  uint64_t* sempty = full + NS;
  uint64_t* tfull = sempty + NS;   // [2]
  uint64_t* tempty = tfull + 2;    // [2]
  uint64_t* bfull = tempty + 2;
  uint64_t* bempty = bfull + 1;
  uint64_t* qfull = bempty + 1;    // [2] column table ready
  uint64_t* qempty = qfull + 2;    // [2] column table consumed
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(qempty + 2);
  uint8_t* tables = smem + NS * STAGE + 512;
  float* sx_s = reinterpret_cast<float*>(tables + 2 * table_bytes(n_tc));
  auto t_hdr = [&](int slot) { return reinterpret_cast<TileHdr*>(tables + slot * table_bytes(n_tc)); };
  auto t_pos = [&](int slot) { return reinterpret_cast<int*>(tables + slot * table_bytes(n_tc) + 64); };  // [2][n_tc]
  auto t_scl = [&](int slot) { return reinterpret_cast<float*>(t_pos(slot) + 2 * n_tc); };             // [2][n_tc]
  auto t_bcol = [&](int slot) { return reinterpret_cast<int*>(t_scl(slot) + 2 * n_tc); };              // [2][n_tc]

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int n_tb = (a.n_rows + BM - 1) / BM;
  const int n_rp = (a.n_tr + 1) / 2;  // row-tile pairs
  const int tiles = n_tb * n_rp;
  const int oob_row = (int)a.w8_rows;  // a weight-tile row past the INT8 arena: TMA fills zeros

  if (tid == 0) {
    for (int i = 0; i < NS; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&sempty[i], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&tfull[b], 1);
      mbar_init(&tempty[b], 8);
      mbar_init(&qfull[b], 32);
      mbar_init(&qempty[b], 3);
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
    if (a.w8_rows > 0) prefetch_tensormap(&maps.w8);
    if (a.x_i8) prefetch_tensormap(&maps.x8);
    if (a.has_fp16) {
      prefetch_tensormap(&maps.w16);
      prefetch_tensormap(&maps.xfp);
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  grid_dep_wait();  // activations and scales come from the preceding kernel
  for (int c = tid; c < n_tc; c += THREADS) sx_s[c] = a.sx ? __ldg(a.sx + c) : 1.0f;
  __syncthreads();
  bool ok = true;

  if (warp == 2) {
    // ================================================================ scheduler
    uint32_t k = 0;
    for (int tile = blockIdx.x; tile < tiles; tile += gridDim.x, ++k) {
      const int slot = k & 1;
      if (ok && !mbar_wait_bounded(&qempty[slot], ((k >> 1) & 1) ^ 1, a.err)) ok = false;
      TileHdr* h = t_hdr(slot);
      int* pos = t_pos(slot);
      float* scl = t_scl(slot);
      int* bcol = t_bcol(slot);
      const int rp = tile % n_rp, tb = tile / n_rp;
      const int r0 = rp * 2, n_r = min(2, a.n_tr - r0);
      for (int i = lane; i < 2 * n_tc; i += 32) {
        pos[i] = -1;
        scl[i] = 0.0f;
      }
      __syncwarp();
      int n16[2] = {0, 0}, b16[2] = {0, 0};
      for (int j = 0; j < n_r; ++j) {
        const int r = r0 + j;
        const int b8 = __ldg(a.rp8 + r), n8 = __ldg(a.rp8 + r + 1) - b8;
        for (int i = lane; i < n8; i += 32) {
          const int p = b8 + i;
          const int c = __ldg(a.ids8 + p) % n_tc;
          pos[j * n_tc + c] = p;
          scl[j * n_tc + c] = sx_s[c] * (a.s8 ? __ldg(a.s8 + p) : 1.0f);  // (sx * sw) in f32, ref :135-137
        }
        if (a.has_fp16) {
          b16[j] = __ldg(a.rp16 + r);
          n16[j] = __ldg(a.rp16 + r + 1) - b16[j];
          for (int i = lane; i < n16[j]; i += 32) bcol[j * n_tc + i] = __ldg(a.ids16 + b16[j] + i) % n_tc;
        }
      }
      if (lane == 0) {
        h->tb = tb;
        h->r0 = r0;
        h->n_r = n_r;
        h->n16[0] = n16[0];
        h->n16[1] = n16[1];
        h->b16[0] = b16[0];
        h->b16[1] = b16[1];
      }
      __syncwarp();
      mbar_arrive(&qfull[slot]);  // every lane publishes its writes
    }
  } else if (warp == 0) {
    // ================================================================ TMA producer
    if (lane == 0) {
      uint32_t g = 0, k = 0;
      for (int tile = blockIdx.x; tile < tiles; tile += gridDim.x, ++k) {
        const int slot = k & 1;
        if (ok && !mbar_wait_bounded(&qfull[slot], (k >> 1) & 1, a.err)) ok = false;
        const TileHdr h = *t_hdr(slot);
        const int* pos = t_pos(slot);
        const int* bcol = t_bcol(slot);
        for (int c = 0; c < n_tc; ++c, ++g) {
          const int stg = g % NS;
          if (ok && !mbar_wait_bounded(&sempty[stg], ((g / NS) & 1) ^ 1, a.err)) ok = false;
          uint8_t* sa = stages + stg * STAGE;
          mbar_expect_tx(&full[stg], STAGE);
          tma_load_2d(sa, &maps.x8, c * 64, h.tb * BM, &full[stg]);
          const int p0 = pos[c], p1 = pos[n_tc + c];
          tma_load_2d(sa + A_BYTES, &maps.w8, 0, p0 >= 0 ? p0 * 64 : oob_row, &full[stg]);
          tma_load_2d(sa + A_BYTES + W_BYTES, &maps.w8, 0, p1 >= 0 ? p1 * 64 : oob_row, &full[stg]);
        }
        for (int j = 0; j < h.n_r; ++j) {
          for (int i = 0; i < 2 * h.n16[j]; ++i, ++g) {
            const int stg = g % NS;
            if (ok && !mbar_wait_bounded(&sempty[stg], ((g / NS) & 1) ^ 1, a.err)) ok = false;
            uint8_t* sa = stages + stg * STAGE;
            const int c = bcol[j * n_tc + (i >> 1)], half = i & 1;
            mbar_expect_tx(&full[stg], A_BYTES + W_BYTES);
            tma_load_2d(sa, &maps.xfp, c * 64 + half * 32, h.tb * BM, &full[stg]);
            tma_load_2d(sa + A_BYTES, &maps.w16, half * 32, (h.b16[j] + (i >> 1)) * 64, &full[stg]);
          }
        }
        mbar_arrive(&qempty[slot]);
      }
    }
  } else if (warp == 1) {
    // ================================================================ MMA issuer
    if (lane == 0) {
      uint32_t g = 0, k = 0, k8 = 0, nbf = 0;
      const uint32_t idesc16 = XT == TQ_DTYPE_BF16 ? IDESC_BF16 : IDESC_F16;
      for (int tile = blockIdx.x; tile < tiles; tile += gridDim.x, ++k) {
        const int slot = k & 1;
        if (ok && !mbar_wait_bounded(&qfull[slot], (k >> 1) & 1, a.err)) ok = false;
        const TileHdr h = *t_hdr(slot);
        mbar_arrive(&qempty[slot]);  // only the header was needed
        for (int c = 0; c < n_tc; ++c, ++g, ++k8) {
          const int stg = g % NS;
          const uint32_t b = k8 & 1;
          if (ok && !mbar_wait_bounded(&full[stg], (g / NS) & 1, a.err)) ok = false;
          if (ok && !mbar_wait_bounded(&tempty[b], (k8 >> 1) & 1, a.err)) ok = false;
          tc_fence_after();
          const uint32_t sa = smem_u32(stages + stg * STAGE);
          const uint64_t da = sw64_desc(sa), db = sw64_desc(sa + A_BYTES);
          // the TMEM tile holds the preset; both K halves accumulate onto it
          umma(tmem + b * 128, da, db, IDESC_I8, 1, true);
          umma(tmem + b * 128, da + 2, db + 2, IDESC_I8, 1, true);
          umma_commit(&sempty[stg]);
          umma_commit(&tfull[b]);
        }
        const int nb = 2 * (h.n16[0] + h.n16[1]);
        if (nb > 0) {
          if (ok && !mbar_wait_bounded(bempty, nbf & 1, a.err)) ok = false;
          tc_fence_after();
          for (int j = 0; j < h.n_r; ++j) {
            for (int i = 0; i < 2 * h.n16[j]; ++i, ++g) {
              const int stg = g % NS;
              if (ok && !mbar_wait_bounded(&full[stg], (g / NS) & 1, a.err)) ok = false;
              tc_fence_after();
              const uint32_t sa = smem_u32(stages + stg * STAGE);
              const uint64_t da = sw64_desc(sa), db = sw64_desc(sa + A_BYTES);
              umma(tmem + 256 + j * 64, da, db, idesc16, i == 0 ? 0 : 1, false);
              umma(tmem + 256 + j * 64, da + 2, db + 2, idesc16, 1, false);
              umma_commit(&sempty[stg]);
            }
          }
          umma_commit(bfull);
          ++nbf;
        }
      }
    }
  } else {
    // ================================================================ epilogue
    const int ew = warp - EPI_WARP0;  // 0..7
    const int q = warp & 3;           // TMEM lane quadrant this warp may access
    const int j = ew >> 2;            // row tile of the pair: columns [64j, 64j+64)
    const uint32_t lane_base = (uint32_t)(q * 32) << 16;
    // preset both INT32 tiles, then hand them (and the FP32 sums) to the MMA issuer
    for (int b = 0; b < 2; ++b) {
      tmem_fill32(tmem + lane_base + b * 128 + j * 64, MAGIC);
      tmem_fill32(tmem + lane_base + b * 128 + j * 64 + 32, MAGIC);
    }
    tmem_wait_st();
    tc_fence_before();
    __syncwarp();
    if (lane == 0) {
      mbar_arrive(&tempty[0]);
      mbar_arrive(&tempty[1]);
      mbar_arrive(bempty);
    }
    uint32_t k = 0, k8 = 0, nbf = 0;
    const float2 neg_magic = make_float2(-MAGIC_F, -MAGIC_F);
    for (int tile = blockIdx.x; tile < tiles; tile += gridDim.x, ++k) {
      const int slot = k & 1;
      if (ok && !mbar_wait_bounded(&qfull[slot], (k >> 1) & 1, a.err)) ok = false;
      const TileHdr h = *t_hdr(slot);
      const float* scl = t_scl(slot) + j * n_tc;
      const int* pos = t_pos(slot) + j * n_tc;
      const int row = h.tb * BM + q * 32 + lane;  // this thread's activation row
      float2 acc[32];
#pragma unroll
      for (int e = 0; e < 32; ++e) acc[e] = make_float2(0.0f, 0.0f);
      for (int c = 0; c < n_tc; ++c, ++k8) {
        const uint32_t b = k8 & 1;
        if (ok && !mbar_wait_bounded(&tfull[b], (k8 >> 1) & 1, a.err)) ok = false;
        tc_fence_after();
        const uint32_t taddr = tmem + lane_base + b * 128 + j * 64;
        uint32_t v[64];
        tmem_ld16(taddr, v);
        tmem_ld16(taddr + 16, v + 16);
        tmem_ld16(taddr + 32, v + 32);
        tmem_ld16(taddr + 48, v + 48);
        tmem_wait_ld();
        tmem_fill32(taddr, MAGIC);
        tmem_fill32(taddr + 32, MAGIC);
        const float s = scl[c];
        if (pos[c] >= 0) {  // this row tile's tile at column c is INT8
          const float2 s2 = make_float2(s, s);
#pragma unroll
          for (int e = 0; e < 32; ++e) {
            const float2 m = make_float2(__uint_as_float(v[2 * e]), __uint_as_float(v[2 * e + 1]));
            acc[e] = __ffma2_rn(__fadd2_rn(m, neg_magic), s2, acc[e]);  // the add is exact: the tile dot
          }
          if (a.partials && row < a.n_rows) {
            int32_t* base = a.partials + ((int64_t)pos[c] * a.n_rows + row) * 64;
#pragma unroll
            for (int e = 0; e < 64; ++e) base[e] = (int32_t)(v[e] - MAGIC);
          }
        }
        tmem_wait_st();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&tempty[b]);
      }
      const int nb = 2 * (h.n16[0] + h.n16[1]);
      if (nb > 0) {
        if (ok && !mbar_wait_bounded(bfull, nbf & 1, a.err)) ok = false;
        tc_fence_after();
        if (j < h.n_r && h.n16[j] > 0) {
          uint32_t v[64];
          const uint32_t taddr = tmem + lane_base + 256 + j * 64;
          tmem_ld16(taddr, v);
          tmem_ld16(taddr + 16, v + 16);
          tmem_ld16(taddr + 32, v + 32);
          tmem_ld16(taddr + 48, v + 48);
          tmem_wait_ld();
#pragma unroll
          for (int e = 0; e < 32; ++e)
            acc[e] = __fadd2_rn(acc[e], make_float2(__uint_as_float(v[2 * e]), __uint_as_float(v[2 * e + 1])));
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(bempty);
        ++nbf;
      }
      named_bar_sync(1, 256);  // all epilogue threads are done with this table slot
      if (tid == EPI_WARP0 * 32) mbar_arrive(&qempty[slot]);
      const int r = h.r0 + j;
      if (j < h.n_r && row < a.n_rows && a.out) {
        const int col0 = r * 64;
        const int ot = a.out_dtype;
        uint16_t* orow = reinterpret_cast<uint16_t*>(a.out) + (int64_t)row * a.ldo + col0;
        const uint16_t* brow = a.bias ? reinterpret_cast<const uint16_t*>(a.bias) + col0 : nullptr;
        const bool vec = col0 + 64 <= a.M && (((uintptr_t)orow) & 15) == 0;
#pragma unroll
        for (int part = 0; part < 4; ++part) {
          uint32_t packed[8];
#pragma unroll
          for (int e = 0; e < 8; ++e) {
            const int cc = part * 16 + 2 * e;
            uint16_t y0 = f2h(acc[part * 8 + e].x, ot), y1 = f2h(acc[part * 8 + e].y, ot);
            if (brow) {
              if (col0 + cc < a.M) y0 = f2h(h2f(y0, ot) + h2f(brow[cc], ot), ot);
              if (col0 + cc + 1 < a.M) y1 = f2h(h2f(y1, ot) + h2f(brow[cc + 1], ot), ot);
            }
            packed[e] = (uint32_t)y0 | ((uint32_t)y1 << 16);
          }
          if (vec) {
            reinterpret_cast<uint4*>(orow + part * 16)[0] = make_uint4(packed[0], packed[1], packed[2], packed[3]);
            reinterpret_cast<uint4*>(orow + part * 16)[1] = make_uint4(packed[4], packed[5], packed[6], packed[7]);
          } else {
            for (int e = 0; e < 16 && col0 + part * 16 + e < a.M; ++e)
              orow[part * 16 + e] = (uint16_t)(packed[e >> 1] >> ((e & 1) * 16));
          }
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
    TQ_CUDA_TRY(cudaFuncSetAttribute(umma_kernel<XT>, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024));
    configured |= 1ull << dev;
  }
  // more than half the SM's shared memory: one CTA (and its 512 TMEM columns) per SM
  const size_t smem = std::max<size_t>(um::smem_bytes(a.n_tc), 120 * 1024);
  if (smem > 227 * 1024) return tq_set_error(TQ_ERR_UNSUPPORTED, "tcgen05 GEMM: too many column tiles");
  const int64_t tiles = (int64_t)((a.n_rows + um::BM - 1) / um::BM) * ((a.n_tr + 1) / 2);
  const int64_t grid = std::min<int64_t>(tiles, tq_sm_count());
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
  if (!x_i8 || (((uintptr_t)x_i8) & 15) || (ld_x8 & 15)) return 0;
  if (x_fp && ((((uintptr_t)x_fp) & 15) || ((ld_xfp * 2) & 15))) return 0;
  if ((w8 && (((uintptr_t)w8) & 15)) || (w16 && (((uintptr_t)w16) & 15))) return 0;
  if (um::smem_bytes((int)((k + 63) / 64)) > 227 * 1024) return 0;
  return 1;
}

int tq_launch_umma(const RowsArgs& a_in, int n_tr, int fp_dtype, cudaStream_t st) {
  RowsArgs a = a_in;
  a.n_tr = n_tr;
  a.split = 1;
  if (a.w8_rows <= 0) return tq_set_error(TQ_ERR_UNSUPPORTED, "tcgen05 GEMM: needs at least one INT8 tile");
  if (a.w8_rows + 64 > (int64_t)INT32_MAX) return tq_set_error(TQ_ERR_UNSUPPORTED, "tcgen05 GEMM: INT8 arena too large");
  UmmaMaps maps;
  memset(&maps, 0, sizeof(maps));
  if (tq_encode_2d(&maps.x8, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, a.x_i8, a.K, a.n_rows, a.ld_x8, 64, um::BM,
                   CU_TENSOR_MAP_SWIZZLE_64B) != TQ_OK)
    return tq_set_error(TQ_ERR_UNSUPPORTED, "tcgen05 GEMM: x_int8 tensor map");
  if (a.has_fp16 && tq_encode_2d(&maps.xfp, CU_TENSOR_MAP_DATA_TYPE_UINT16, 2, a.x_fp, a.K, a.n_rows, a.ld_xfp * 2,
                                 32, um::BM, CU_TENSOR_MAP_SWIZZLE_64B) != TQ_OK)
    return tq_set_error(TQ_ERR_UNSUPPORTED, "tcgen05 GEMM: x_fp tensor map");
  // weight rows past the INT8 arena are the zero boxes of 16-bit / missing row tiles
  if (tq_encode_2d(&maps.w8, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, a.w8, 64, (uint64_t)a.w8_rows, 64, 64, 64,
                   CU_TENSOR_MAP_SWIZZLE_64B) != TQ_OK)
    return tq_set_error(TQ_ERR_UNSUPPORTED, "tcgen05 GEMM: INT8 tile tensor map");
  if (a.has_fp16 && tq_encode_2d(&maps.w16, CU_TENSOR_MAP_DATA_TYPE_UINT16, 2, a.w16, 64, (uint64_t)a.w16_rows, 128,
                                 32, 64, CU_TENSOR_MAP_SWIZZLE_64B) != TQ_OK)
    return tq_set_error(TQ_ERR_UNSUPPORTED, "tcgen05 GEMM: 16-bit tile tensor map");
  return fp_dtype == TQ_DTYPE_BF16 ? launch_umma_t<TQ_DTYPE_BF16>(a, maps, st) : launch_umma_t<TQ_DTYPE_F16>(a, maps, st);
}

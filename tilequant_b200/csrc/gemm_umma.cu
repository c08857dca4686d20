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
// Output tile = 128 activation rows x RT row tiles (64 RT output columns; the kernel
// is written for RT = 2 or 4, the launcher uses RT = 2, which measured faster).  The K
// loop runs over the n_tc input-column tiles: one 128 x 64-byte activation tile and,
// stacked, the RT row tiles' 64 x 64 INT8 weight tiles make one N = 64 RT tcgen05.mma
// step (a row tile whose tile at that column is 16-bit, or that does not exist, is
// loaded as an out-of-bounds TMA box, i.e. zeros, and its step is skipped in the
// rescale, so each row tile still sees exactly its own INT8 tiles in ascending order).
// The 16-bit tiles of each row tile then run as N = 64 kind::f16 MMAs into an FP32 TMEM
// accumulator, as one more step of the same TMEM ring.
//
// Warp roles (one CTA per SM, persistent over output tiles, 12 warps):
//   warp 0      TMA producer (one thread): shared-memory ring of 192 KB, each stage two
//               K steps of 16 KB (RT = 2) or one of 24 KB (RT = 4), SWIZZLE_64B (the
//               UMMA canonical K-major layout);
//   warp 1      MMA issuer (one thread); tcgen05.commit frees stages and publishes groups;
//   warp 2      scheduler: builds each output tile's column table (INT8 list position
//               and combined scale sx*sw of the RT row tiles at every column, 16-bit tile
//               columns) one tile ahead into a 2-slot ring, so no role stalls on the
//               id lists;
//   warp 3      second TMA producer (the other half of the weight tiles);
//   warps 4-11  epilogue: two per TMEM lane quadrant, each over half of the step's
//               columns.  Every K step's first MMA overwrites its INT32 TMEM tile (the
//               second accumulates), so each word read back is that step's tile dot; it
//               converts to FP32 exactly (|dot| <= 64*128*128 < 2^24) and a packed
//               f32x2 FMA rescales it into the FP32 accumulator held in registers.
// TMEM (512 columns): two groups of step buffers (two of 128 columns, or one of 256).
// Every barrier hand-off (stage full / empty, group full / empty) covers a whole group:
// an mbarrier round trip and the tcgen05 fences around it cost about as much as one
// step's MMA, so per-step hand-offs at RT = 2 left the tensor pipe idle most of the time.
// The per-step read-back and rescale (a 64 KB TMEM read, one conversion and one FMA per
// output element and K step, at least twice the step's MMA time) is the bound of this
// kernel; an earlier form preset the tiles to 2^23 + 2^22 so the bits read back were
// already a float, but rewriting the preset (a 64 KB TMEM store per step) cost more than
// the conversions.
#include <string.h>

#include <algorithm>

#include "common.cuh"
#include "gemm_args.cuh"
#include "tma.cuh"

namespace tq {

__device__ __forceinline__ bool mbar_test(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile("{\n .reg .pred p;\n mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
               : "=r"(ok)
               : "r"(smem_u32(bar)), "r"(parity)
               : "memory");
  return ok != 0;
}

// Spin on an mbarrier phase without suspending, bounded by about two seconds (then
// TQ_ERR_TIMEOUT).  Used for the MMA <-> epilogue hand-offs, whose wake-up latency is
// on the kernel's critical path (1-1.5 % faster than the sleeping wait on the prefill
// shapes); the other roles keep the sleeping wait.
__device__ __forceinline__ bool mbar_wait_spin(uint64_t* bar, uint32_t parity, int* err) {
  const uint64_t t0 = global_ns();
#pragma unroll 1
  for (uint32_t i = 0; i < (1u << 31); ++i) {
    if (mbar_test(bar, parity)) return true;
    if ((i & 1023u) == 1023u && global_ns() - t0 > kWaitLimitNs) break;
  }
  report(err, TQ_ERR_TIMEOUT);
  return false;
}

namespace um {
constexpr int BM = 128;             // activation rows per output tile (MMA M)
constexpr int A_BYTES = BM * 64;    // 8 KB activation tile of one K step
constexpr int W_BYTES = 64 * 64;    // 4 KB weight tile
constexpr int EPI_WARP0 = 4;        // warpgroup 0: producer, MMA issuer, scheduler, one idle warp
constexpr int NEPI = 8;             // epilogue warps: 4 lane quadrants x (NEPI / 4) column slices
constexpr int THREADS = (EPI_WARP0 + NEPI) * 32;
// Registers after the role split (setmaxnreg works per warpgroup): warpgroup 0 drops to
// AUX_REGS and the two epilogue warpgroups grow to EPI_REGS.  With one CTA per SM in the
// launch bounds and the setmaxnreg at the top of each warpgroup's branch, ptxas compiles
// each branch for its own count.  setmaxnreg.inc draws on the registers the CTA was
// launched with and waits until they are free, so the launcher checks the compiled
// register count covers the split (SPLIT_REGS) before launching.
constexpr int AUX_REGS = 56;
constexpr int EPI_REGS = 224;
constexpr int SPLIT_REGS = 128 * AUX_REGS + NEPI * 32 * EPI_REGS;
static_assert(SPLIT_REGS <= 65536, "register split");
constexpr int TMEM_COLS = 512;

// tcgen05 instruction descriptors: M = 128, K-major A and B.
constexpr uint32_t idesc(uint32_t c_fmt, uint32_t ab_fmt, uint32_t n) {
  return (c_fmt << 4) | (ab_fmt << 7) | (ab_fmt << 10) | ((n >> 3) << 17) | ((128u >> 4) << 24);
}
constexpr uint32_t IDESC_BF16 = idesc(1 /*F32*/, 1 /*BF16*/, 64);
constexpr uint32_t IDESC_F16 = idesc(1 /*F32*/, 0 /*F16*/, 64);

// Tile geometry by the number RT of 64-row weight tiles an output tile spans (its N =
// 64 RT output columns): RT = 2 streams two K steps per stage and per TMEM group (two
// groups of two 128-column buffers), RT = 4 one K step (two 256-column buffers) with
// 24 KB per step for twice the MMA work of RT = 2, so fewer bytes per MAC come from L2.
template <int RT>
struct Geo {
  static constexpr int BN = 64 * RT;
  static constexpr int STEP_BYTES = A_BYTES + RT * W_BYTES;
  static constexpr int GS = RT == 2 ? 2 : 1;
  static constexpr int STAGE = GS * STEP_BYTES;
  static constexpr int NS = (192 * 1024) / STAGE;
  static constexpr int NG = TMEM_COLS / (GS * BN);
  static constexpr int CW = BN / (NEPI / 4);  // columns of a step one epilogue warp rescales
  static constexpr int CH = RT == 4 ? 16 : 32;  // columns per TMEM load of the rescale pipeline
  static constexpr uint32_t IDESC = idesc(2 /*S32*/, 1 /*S8*/, BN);
  static_assert(NG == 2 && CW % 64 == 0, "geometry");
  // column table slot: pos[RT][n_tc] int, scale[RT][n_tc] float, bcol[RT][n_tc] int, header
  __host__ __device__ static constexpr size_t table_bytes(int n_tc) { return (size_t)n_tc * 12 * RT + 64; }
  static size_t smem_bytes(int n_tc) {
    return 1024 + (size_t)NS * STAGE + 512 + 2 * table_bytes(n_tc) + (size_t)n_tc * 4;
  }
};
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

// One lane of the (converged) warp, chosen by the hardware.
__device__ __forceinline__ bool elect_one() {
  uint32_t pred;
  asm volatile("{\n .reg .pred p;\n elect.sync _|p, 0xffffffff;\n selp.u32 %0, 1, 0, p;\n}\n" : "=r"(pred));
  return pred != 0;
}

__device__ __forceinline__ void umma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// 32 consecutive TMEM columns of this thread's lane (no wait).
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t* v) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,%17,%18,%19,"
      "%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]), "=r"(v[8]),
        "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15]), "=r"(v[16]),
        "=r"(v[17]), "=r"(v[18]), "=r"(v[19]), "=r"(v[20]), "=r"(v[21]), "=r"(v[22]), "=r"(v[23]), "=r"(v[24]),
        "=r"(v[25]), "=r"(v[26]), "=r"(v[27]), "=r"(v[28]), "=r"(v[29]), "=r"(v[30]), "=r"(v[31])
      : "r"(taddr));
}
__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }
template <int CH>
__device__ __forceinline__ void tmem_ld_chunk(uint32_t taddr, uint32_t* v);
template <int CH>
__device__ __forceinline__ void tmem_wait_ld_chunk(uint32_t* v);

// 16 consecutive TMEM columns of this thread's lane (no wait).
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t* v) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]), "=r"(v[8]),
        "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15])
      : "r"(taddr));
}
// Wait for this thread's TMEM loads; the 16 destination registers of the last load are
// operands so no use of them can be scheduled ahead of the wait.
__device__ __forceinline__ void tmem_wait_ld_regs16(uint32_t* v) {
  asm volatile("tcgen05.wait::ld.sync.aligned;"
               : "+r"(v[0]), "+r"(v[1]), "+r"(v[2]), "+r"(v[3]), "+r"(v[4]), "+r"(v[5]), "+r"(v[6]), "+r"(v[7]),
                 "+r"(v[8]), "+r"(v[9]), "+r"(v[10]), "+r"(v[11]), "+r"(v[12]), "+r"(v[13]), "+r"(v[14]), "+r"(v[15])
               :
               : "memory");
}
// Wait for this thread's TMEM loads, with the 32 destination registers of the last load
// as operands so no use of them can be scheduled ahead of the wait.
__device__ __forceinline__ void tmem_wait_ld_regs(uint32_t* v) {
  asm volatile("tcgen05.wait::ld.sync.aligned;"
               : "+r"(v[0]), "+r"(v[1]), "+r"(v[2]), "+r"(v[3]), "+r"(v[4]), "+r"(v[5]), "+r"(v[6]), "+r"(v[7]),
                 "+r"(v[8]), "+r"(v[9]), "+r"(v[10]), "+r"(v[11]), "+r"(v[12]), "+r"(v[13]), "+r"(v[14]), "+r"(v[15]),
                 "+r"(v[16]), "+r"(v[17]), "+r"(v[18]), "+r"(v[19]), "+r"(v[20]), "+r"(v[21]), "+r"(v[22]),
                 "+r"(v[23]), "+r"(v[24]), "+r"(v[25]), "+r"(v[26]), "+r"(v[27]), "+r"(v[28]), "+r"(v[29]),
                 "+r"(v[30]), "+r"(v[31])
               :
               : "memory");
}

template <>
__device__ __forceinline__ void tmem_ld_chunk<16>(uint32_t taddr, uint32_t* v) { tmem_ld16(taddr, v); }
template <>
__device__ __forceinline__ void tmem_ld_chunk<32>(uint32_t taddr, uint32_t* v) { tmem_ld32(taddr, v); }
template <>
__device__ __forceinline__ void tmem_wait_ld_chunk<16>(uint32_t* v) { tmem_wait_ld_regs16(v); }
template <>
__device__ __forceinline__ void tmem_wait_ld_chunk<32>(uint32_t* v) { tmem_wait_ld_regs(v); }

// acc[e] = fma(f32(dot), s, acc[e]) for 16 columns whose TMEM words hold INT32 tile dots;
// with DUMP, also writes the INT32 dots of an INT8 tile (p >= 0) to `partials`.
template <bool DUMP>
__device__ __forceinline__ void rescale16(float2* acc, const uint32_t* v, float s, int32_t* partials, int p, int row,
                                          int n_rows, int col) {
  const float2 s2 = make_float2(s, s);
#pragma unroll
  for (int e = 0; e < 8; ++e) {
    const float2 d = make_float2(__int2float_rn((int)v[2 * e]), __int2float_rn((int)v[2 * e + 1]));  // exact
    acc[e] = __ffma2_rn(d, s2, acc[e]);
  }
  if (DUMP && p >= 0 && row < n_rows) {
    int32_t* base = partials + ((int64_t)p * n_rows + row) * 64 + col;
#pragma unroll
    for (int e = 0; e < 16; ++e) base[e] = (int32_t)v[e];
  }
}

struct TileHdr {
  int tb, r0, n_r;    // token block, first row tile, row tiles present (1 .. RT)
  int n16[4];         // 16-bit tiles of each row tile
  int b16[4];         // first 16-bit list position of each row tile
};

template <int XT, bool DUMP, int RT>
__global__ void __launch_bounds__(um::THREADS, 1) umma_kernel(const RowsArgs a, const __grid_constant__ UmmaMaps maps) {
  using namespace um;
  using G = Geo<RT>;
  constexpr int NS = G::NS, STAGE = G::STAGE, STEP_BYTES = G::STEP_BYTES, GS = G::GS, NG = G::NG, CW = G::CW;
  constexpr int BN = G::BN, CH = G::CH;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
  const int n_tc = a.n_tc;
  uint8_t* stages = smem;  // NS x GS x (A 8 KB | W0 .. W[RT-1] 4 KB each), 1024-byte aligned
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + NS * STAGE);
  uint64_t* sempty = full + NS;
  uint64_t* tfull = sempty + NS;   // [NG] TMEM group written by the MMA
  uint64_t* tempty = tfull + NG;   // [NG] TMEM group read
  uint64_t* qfull = tempty + NG;   // [2] column table ready
  uint64_t* qempty = qfull + 2;    // [2] column table consumed
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(qempty + 2);
  uint8_t* tables = smem + NS * STAGE + 512;
  float* sx_s = reinterpret_cast<float*>(tables + 2 * G::table_bytes(n_tc));
  auto t_hdr = [&](int slot) { return reinterpret_cast<TileHdr*>(tables + slot * G::table_bytes(n_tc)); };
  auto t_pos = [&](int slot) { return reinterpret_cast<int*>(tables + slot * G::table_bytes(n_tc) + 64); };  // [RT][n_tc]
  auto t_scl = [&](int slot) { return reinterpret_cast<float*>(t_pos(slot) + RT * n_tc); };                // [RT][n_tc]
  auto t_bcol = [&](int slot) { return reinterpret_cast<int*>(t_scl(slot) + RT * n_tc); };                 // [RT][n_tc]

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int n_tb = (a.n_rows + BM - 1) / BM;
  const int n_rp = (a.n_tr + RT - 1) / RT;  // groups of RT row tiles
  const int tiles = n_tb * n_rp;
  const int oob_row = (int)a.w8_rows;  // a weight-tile row past the INT8 arena: TMA fills zeros

  if (tid == 0) {
    for (int i = 0; i < NS; ++i) {
      mbar_init(&full[i], 2);  // the two producers
      mbar_init(&sempty[i], 1);
    }
    for (int b = 0; b < NG; ++b) {
      mbar_init(&tfull[b], 1);
      mbar_init(&tempty[b], NEPI);
    }
    for (int s = 0; s < 2; ++s) {
      mbar_init(&qfull[s], 32);
      mbar_init(&qempty[s], 4);  // two producers, MMA issuer, epilogue
    }
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
  // The register split sits at the top of each warpgroup's branch so that every role's
  // code is compiled under its warpgroup's register count.
  if (warp < EPI_WARP0) {
    asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(AUX_REGS));
    if (warp == 2) {
      // ================================================================ scheduler
      uint32_t k = 0;
      for (int tile = blockIdx.x; tile < tiles; tile += gridDim.x, ++k) {
        const int slot = k & 1;
        if (ok && !mbar_wait_sleep(&qempty[slot], ((k >> 1) & 1) ^ 1, a.err)) ok = false;
        TileHdr* h = t_hdr(slot);
        int* pos = t_pos(slot);
        float* scl = t_scl(slot);
        int* bcol = t_bcol(slot);
        const int rp = tile % n_rp, tb = tile / n_rp;
        const int r0 = rp * RT, n_r = min(RT, a.n_tr - r0);
        for (int i = lane; i < RT * n_tc; i += 32) {
          pos[i] = -1;
          scl[i] = 0.0f;
        }
        if (lane < 4) {
          h->n16[lane] = 0;
          h->b16[lane] = 0;
        }
        __syncwarp();
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
            const int b16 = __ldg(a.rp16 + r), n16 = __ldg(a.rp16 + r + 1) - b16;
            for (int i = lane; i < n16; i += 32) bcol[j * n_tc + i] = __ldg(a.ids16 + b16 + i) % n_tc;
            if (lane == 0) {
              h->n16[j] = n16;
              h->b16[j] = b16;
            }
          }
        }
        if (lane == 0) {
          h->tb = tb;
          h->r0 = r0;
          h->n_r = n_r;
        }
        __syncwarp();
        mbar_arrive(&qfull[slot]);  // every lane publishes its writes
      }
    } else if (warp == 0 || warp == 3) {
      // ================================================================ TMA producers
      // P0 (warp 0): the activation box and the first half of the row tiles' weight
      // tiles of every K step, and the 16-bit tiles; P1 (warp 3): the other half of the
      // weight tiles.  Both arrive on every stage's full barrier.  The whole warp runs the
      // loop (warp-uniform control flow keeps the TMA operands in uniform registers, which
      // more than halves the cost of issuing a box); one elected lane issues.
      const bool leader = elect_one();
      const bool p0 = warp == 0;
      const int j_lo = p0 ? 0 : RT / 2, j_hi = p0 ? RT / 2 : RT;
      const uint32_t step_bytes = (p0 ? A_BYTES : 0) + (j_hi - j_lo) * W_BYTES;
      uint32_t g = 0, k = 0;
      for (int tile = blockIdx.x; tile < tiles; tile += gridDim.x, ++k) {
        const int slot = k & 1;
        if (ok && !mbar_wait_sleep(&qfull[slot], (k >> 1) & 1, a.err)) ok = false;
        const TileHdr* h = t_hdr(slot);
        const int tb = h->tb, n_r = h->n_r;
        const int* pos = t_pos(slot);
        const int* bcol = t_bcol(slot);
        for (int c0 = 0; c0 < n_tc; c0 += GS, ++g) {  // GS INT8 K steps per stage
          const int stg = g % NS, ns = min(GS, n_tc - c0);
          if (ok && !mbar_wait_sleep(&sempty[stg], ((g / NS) & 1) ^ 1, a.err)) ok = false;
          if (leader) {
            mbar_expect_tx(&full[stg], ns * step_bytes);
            for (int s = 0; s < ns; ++s) {
              const int c = c0 + s;
              uint8_t* sa = stages + stg * STAGE + s * STEP_BYTES;
              if (p0) tma_load_2d(sa, &maps.x8, c * 64, tb * BM, &full[stg]);
              for (int j = j_lo; j < j_hi; ++j) {
                const int p = pos[j * n_tc + c];
                tma_load_2d(sa + A_BYTES + j * W_BYTES, &maps.w8, 0, p >= 0 ? p * 64 : oob_row, &full[stg]);
              }
            }
          }
        }
        for (int j = 0; j < n_r; ++j) {  // one 16-bit tile (two 32-column halves) per stage
          const int n16 = h->n16[j], b16 = h->b16[j];
          for (int i = 0; i < n16; ++i, ++g) {
            const int stg = g % NS;
            if (ok && !mbar_wait_sleep(&sempty[stg], ((g / NS) & 1) ^ 1, a.err)) ok = false;
            if (!leader) continue;
            if (!p0) {
              mbar_arrive(&full[stg]);
              continue;
            }
            const int c = bcol[j * n_tc + i];
            mbar_expect_tx(&full[stg], 2 * (A_BYTES + W_BYTES));
            for (int half = 0; half < 2; ++half) {
              uint8_t* sa = stages + stg * STAGE + half * (A_BYTES + W_BYTES);
              tma_load_2d(sa, &maps.xfp, c * 64 + half * 32, tb * BM, &full[stg]);
              tma_load_2d(sa + A_BYTES, &maps.w16, half * 32, (b16 + i) * 64, &full[stg]);
            }
          }
        }
        __syncwarp();
        if (leader) mbar_arrive(&qempty[slot]);
      }
    } else if (warp == 1) {
      // ================================================================ MMA issuer
      // The whole warp runs the loop; one elected lane issues the tcgen05 instructions.
      {
        const bool leader = elect_one();
        uint32_t g = 0, k = 0, grp = 0;
        const uint32_t idesc16 = XT == TQ_DTYPE_BF16 ? IDESC_BF16 : IDESC_F16;
        for (int tile = blockIdx.x; tile < tiles; tile += gridDim.x, ++k) {
          const int slot = k & 1;
          if (ok && !mbar_wait_sleep(&qfull[slot], (k >> 1) & 1, a.err)) ok = false;
          const TileHdr* h = t_hdr(slot);
          const int n_r = h->n_r;
          int n16s[RT];
          int n16_all = 0;
  #pragma unroll
          for (int j = 0; j < RT; ++j) {
            n16s[j] = h->n16[j];
            n16_all += n16s[j];
          }
          if (leader) mbar_arrive(&qempty[slot]);  // only the header was needed
          for (int c0 = 0; c0 < n_tc; c0 += GS, ++g, ++grp) {
            const int stg = g % NS, ns = min(GS, n_tc - c0);
            const uint32_t gb = grp % NG;
            if (ok && !mbar_wait_spin(&full[stg], (g / NS) & 1, a.err)) ok = false;
            if (ok && !mbar_wait_spin(&tempty[gb], (grp / NG) & 1, a.err)) ok = false;
            tc_fence_after();
            for (int s = 0; s < ns; ++s) {
              const uint32_t sa = smem_u32(stages + stg * STAGE + s * STEP_BYTES);
              const uint64_t da = sw64_desc(sa), db = sw64_desc(sa + A_BYTES);
              const uint32_t d = tmem + (gb * GS + s) * BN;
              // the first K half overwrites the step buffer, the second accumulates
              if (leader) {
                umma(d, da, db, G::IDESC, 0, true);
                umma(d, da + 2, db + 2, G::IDESC, 1, true);
              }
            }
            if (leader) {
              umma_commit(&sempty[stg]);
              umma_commit(&tfull[gb]);
            }
          }
          if (n16_all > 0) {  // the 16-bit tiles: one more group, first buffer only
            const uint32_t gb = grp % NG;
            if (ok && !mbar_wait_sleep(&tempty[gb], (grp / NG) & 1, a.err)) ok = false;
            tc_fence_after();
  #pragma unroll
            for (int j = 0; j < RT; ++j) {
              const int n16 = j < n_r ? n16s[j] : 0;
              for (int i = 0; i < n16; ++i, ++g) {
                const int stg = g % NS;
                if (ok && !mbar_wait_sleep(&full[stg], (g / NS) & 1, a.err)) ok = false;
                tc_fence_after();
                for (int half = 0; half < 2; ++half) {
                  const uint32_t sa = smem_u32(stages + stg * STAGE + half * (A_BYTES + W_BYTES));
                  const uint64_t da = sw64_desc(sa), db = sw64_desc(sa + A_BYTES);
                  const uint32_t d = tmem + gb * GS * BN + j * 64;
                  // the first MMA of a row tile overwrites the buffer
                  if (leader) {
                    umma(d, da, db, idesc16, (i == 0 && half == 0) ? 0 : 1, false);
                    umma(d, da + 2, db + 2, idesc16, 1, false);
                  }
                }
                if (leader) umma_commit(&sempty[stg]);
              }
            }
            if (leader) umma_commit(&tfull[gb]);
            ++grp;
          }
        }
      }
    }
  } else {
    asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(EPI_REGS));
    // ================================================================ epilogue
    const int ew = warp - EPI_WARP0;
    const int q = warp & 3;           // TMEM lane quadrant this warp may access
    const int cs = ew >> 2;           // CW-column slice of the BN-column step
    const uint32_t col = cs * CW;
    const int j0 = col >> 6;          // first row tile of the slice
    constexpr int NJ = (CW + 63) / 64;  // row tiles the slice spans
    const uint32_t tbase = tmem + ((uint32_t)(q * 32) << 16) + col;
    // hand the empty groups to the MMA issuer
    if (lane == 0)
      for (int b = 0; b < NG; ++b) mbar_arrive(&tempty[b]);
    uint32_t k = 0, grp = 0;
    for (int tile = blockIdx.x; tile < tiles; tile += gridDim.x, ++k) {
      const int slot = k & 1;
      if (ok && !mbar_wait_sleep(&qfull[slot], (k >> 1) & 1, a.err)) ok = false;
      const TileHdr* h = t_hdr(slot);
      const float* scl = t_scl(slot) + j0 * n_tc;
      const int* pos = t_pos(slot) + j0 * n_tc;
      const int row = h->tb * BM + q * 32 + lane;  // this thread's activation row
      float2 acc[CW / 2];
#pragma unroll
      for (int e = 0; e < CW / 2; ++e) acc[e] = make_float2(0.0f, 0.0f);
      static_assert(CW % CH == 0 && (CH <= 64 || NJ == 1), "chunks must not straddle row tiles");
      for (int c0 = 0; c0 < n_tc; c0 += GS, ++grp) {
        const uint32_t gb = grp % NG;
        // A step whose tile at this column is 16-bit or missing was an MMA with a zero
        // box: its buffer reads dot 0, and with scale 0 the FMA leaves the accumulator
        // bit-identical (it is never -0), so every step of the group runs the same
        // branch-free sequence.
        float sc[GS][NJ];
        int pp[GS][NJ];
#pragma unroll
        for (int s = 0; s < GS; ++s)
#pragma unroll
          for (int t = 0; t < NJ; ++t) {
            const bool in = GS == 1 || c0 + s < n_tc;
            sc[s][t] = in ? scl[t * n_tc + c0 + s] : 0.0f;
            pp[s][t] = DUMP && in ? pos[t * n_tc + c0 + s] : -1;
          }
        const uint32_t t0 = tbase + gb * GS * BN;  // step s, chunk u at t0 + s * BN + u * CH
        if (ok && !mbar_wait_spin(&tfull[gb], (grp / NG) & 1, a.err)) ok = false;
        tc_fence_after();
        // CH-column chunks (step s = i / CPS, columns CH * (i % CPS)), each chunk's load
        // issued before the previous chunk's rescale so the TMEM latency overlaps FP work
        constexpr int CPS = CW / CH;  // chunks per step
        uint32_t v[2][CH];
        tmem_ld_chunk<CH>(t0, v[0]);
        tmem_wait_ld_chunk<CH>(v[0]);
#pragma unroll
        for (int i = 0; i < GS * CPS; ++i) {
          const int s = i / CPS, cc = (i % CPS) * CH, t = cc >> 6;
          if (i + 1 < GS * CPS) tmem_ld_chunk<CH>(t0 + ((i + 1) / CPS) * BN + ((i + 1) % CPS) * CH, v[(i + 1) & 1]);
#pragma unroll
          for (int hh = 0; hh < CH / 16; ++hh) {
            rescale16<DUMP>(acc + cc / 2 + hh * 8, v[i & 1] + hh * 16, sc[s][t], a.partials, pp[s][t], row, a.n_rows,
                            ((col + cc) & 63) + hh * 16);
          }
          if (i + 1 < GS * CPS) tmem_wait_ld_chunk<CH>(v[(i + 1) & 1]);
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&tempty[gb]);
      }
      int n16_all = 0;
#pragma unroll
      for (int jj = 0; jj < RT; ++jj) n16_all += h->n16[jj];
      if (n16_all > 0) {
        const uint32_t gb = grp % NG;
        if (ok && !mbar_wait_sleep(&tfull[gb], (grp / NG) & 1, a.err)) ok = false;
        tc_fence_after();
#pragma unroll
        for (int t = 0; t < NJ; ++t) {
          if (j0 + t < h->n_r && h->n16[j0 + t] > 0) {  // (other row tiles' columns were not written)
#pragma unroll
            for (int u = 0; u < 64 && u < CW; u += 32) {
              const uint32_t taddr = tbase + gb * GS * BN + t * 64 + u;
              uint32_t v[32];
              tmem_ld32(taddr, v);
              tmem_wait_ld_regs(v);
#pragma unroll
              for (int e = 0; e < 16; ++e)
                acc[(t * 64 + u) / 2 + e] =
                    __fadd2_rn(acc[(t * 64 + u) / 2 + e], make_float2(__uint_as_float(v[2 * e]), __uint_as_float(v[2 * e + 1])));
            }
          }
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&tempty[gb]);
        ++grp;
      }
      const int r = h->r0 + j0, n_r = h->n_r;
      named_bar_sync(1, NEPI * 32);  // all epilogue threads are done with this table slot
      if (tid == EPI_WARP0 * 32) mbar_arrive(&qempty[slot]);
      // the slice's row tiles are adjacent in the output; columns past the last row tile
      // present are at or past M
      if (j0 < n_r && row < a.n_rows && a.out) {
        const int col0 = r * 64 + (col & 63);
        const int ot = a.out_dtype;
        uint16_t* orow = reinterpret_cast<uint16_t*>(a.out) + (int64_t)row * a.ldo + col0;
        const uint16_t* brow = a.bias ? reinterpret_cast<const uint16_t*>(a.bias) + col0 : nullptr;
        const bool vec = col0 + CW <= a.M && (((uintptr_t)orow) & 15) == 0;
#pragma unroll
        for (int part = 0; part < CW / 16; ++part) {
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

template <int XT, bool DUMP, int RT>
static int launch_umma_t(const RowsArgs& a, const UmmaMaps& maps, cudaStream_t st) {
  static uint64_t configured = 0;
  int dev = 0;
  TQ_CUDA_TRY(cudaGetDevice(&dev));
  if (dev < 64 && !(configured & (1ull << dev))) {
    TQ_CUDA_TRY(cudaFuncSetAttribute(umma_kernel<XT, DUMP, RT>, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024));
    cudaFuncAttributes fa;
    TQ_CUDA_TRY(cudaFuncGetAttributes(&fa, umma_kernel<XT, DUMP, RT>));
    if ((int64_t)fa.numRegs * um::THREADS < um::SPLIT_REGS)  // the register split could never complete
      return tq_set_error(TQ_ERR_UNSUPPORTED, "tcgen05 GEMM: compiled register count too small for the warp split");
    configured |= 1ull << dev;
  }
  // more than half the SM's shared memory: one CTA (and its 512 TMEM columns) per SM
  const size_t smem = std::max<size_t>(um::Geo<RT>::smem_bytes(a.n_tc), 120 * 1024);
  if (smem > 227 * 1024) return tq_set_error(TQ_ERR_UNSUPPORTED, "tcgen05 GEMM: too many column tiles");
  const int64_t tiles = (int64_t)((a.n_rows + um::BM - 1) / um::BM) * ((a.n_tr + RT - 1) / RT);
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
  TQ_CUDA_TRY(cudaLaunchKernelEx(&cfg, umma_kernel<XT, DUMP, RT>, a, maps));
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
  if (um::Geo<2>::smem_bytes((int)((k + 63) / 64)) > 227 * 1024) return 0;
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
  // 128-column output tiles (RT = 2): 256-column tiles (RT = 4) give each epilogue
  // thread 128 accumulator columns and half the TMEM steps in flight, and measured
  // 10-25 % slower on every prefill shape, although they cut the L2 -> SM bytes per MAC
  if (a.partials) return launch_umma_t<TQ_DTYPE_BF16, true, 2>(a, maps, st);  // INT8 only: no 16-bit tiles
  return fp_dtype == TQ_DTYPE_BF16 ? launch_umma_t<TQ_DTYPE_BF16, false, 2>(a, maps, st)
                                   : launch_umma_t<TQ_DTYPE_F16, false, 2>(a, maps, st);
}

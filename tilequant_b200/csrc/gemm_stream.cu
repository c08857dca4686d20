// Decode-sized mixed INT8/16-bit 64x64 tile GEMM, streamed (sm_100a): up to 16
// activation rows against a packed weight.
//
// Reference: src/kernels/triton/gemm_rows_splitk_64x64.py:78-190 with SPLIT_K = S.  Same
// partition and arithmetic as the other decode kernels (gemm_rows.cu, gemm_gemv.cu), so
// the result is bit-identical to theirs at the same split:
//   split s of row tile r owns positions [b + cnt*s/S, b + cnt*(s+1)/S) of the row's
//   INT8 list and of its 16-bit list; acc = acc + f32(i32 tile dot) * (sx[c] * sw[pos])
//   (multiply and add rounded separately) in list order, then acc += dot(x, W16^T); the
//   split partials are added in split order 0..S-1, rounded, then the bias.
//
// At decode a projection is a stream of weight bytes read once, so the kernel is built
// to keep HBM busy with as few instructions per byte as possible:
//   * CTA = (split s, row tile r); the S CTAs of a row tile form a thread-block cluster:
//     at the end every split but the first stores its partial into split 0's shared
//     memory (distributed shared memory) and signals split 0's barrier, then exits,
//     and split 0 adds the partials in split order (no global scratch, no arrival
//     counters, no cluster-wide wait at the end).  The host picks S so that all n_tr * S CTAs are
//     resident at once (as many splits as fit, up to 8 and at least 4 tiles each);
//   * the INT8 positions of a split are contiguous in the tile arena, so its weights
//     arrive as 16 KB bulk copies (four tiles each) into a ring of up to eight chunks
//     (as deep as leaves room for two CTAs per SM), issued by
//     one elected lane of a producer warp; the first ring's worth goes out before the
//     wait on the kernel that produced the activations (programmatic dependent launch),
//     so the weight stream starts while that kernel finishes;
//   * the INT8 activations of the split's column range are copied into shared memory
//     once (one bulk copy per row, rows padded so the operand loads are free of bank
//     conflicts) and stay there; with fused quantization the consumers make those
//     codes and scales from the 16-bit activations instead, bit-identical to the
//     activation quantizer (one launch instead of two); each 16-bit tile arrives as an 8 KB bulk copy plus a TMA box of
//     its 16-bit activation columns, in a separate one-slot ring;
//   * four consumer warps split every tile by weight rows (warp w: rows 16w..16w+15,
//     swap-AB mma.sync m16n8k32 with the k order permuted identically for both
//     operands, as in gemm_rows.cu), and synchronise with the producer once per chunk.
#include <string.h>

#include <algorithm>

#include "common.cuh"
#include "gemm_args.cuh"
#include "tma.cuh"


namespace tq {

namespace sk {
constexpr int CONS = 4;                    // consumer warps
constexpr int THREADS = (CONS + 1) * 32;   // + the producer warp
constexpr int CHK = 4;                     // INT8 tiles per bulk copy
constexpr int MAX_NCH = 8;                 // chunks in the ring: sized per launch (RowsArgs::ring_chunks)
constexpr int CHUNK = CHK * 4096;
constexpr int NS16 = 1;                    // 16-bit tile slots (16-bit tiles are the rare ones)
constexpr int W16B = 8192;
constexpr int XB16 = 16 * 128;             // TMA box of 16-bit activations: 16 rows x 64 values
constexpr int SLOT16 = W16B + XB16;
constexpr int PART_ROW = 64 * 4;           // a split's partial: 64 outputs per activation row, f32
constexpr int MAX_S = 8;                   // portable cluster size
}  // namespace sk

struct StreamMaps {
  CUtensorMap xfp;  // x_fp [n_rows][K] 16-bit, box 64 x 16 (only when the weight has 16-bit tiles)
};

__device__ __forceinline__ uint4 lds16(const void* p) { return *reinterpret_cast<const uint4*>(p); }

__device__ __forceinline__ float i2f_stream(int v) {
  return __fsub_rn(__int_as_float(v + 0x4B400000), 12582912.0f);  // exact for |v| < 2^22
}

// Address of the same shared-memory location in cluster CTA `rank`.
__device__ __forceinline__ uint32_t mapa_rank(uint32_t addr, uint32_t rank) {
  uint32_t out;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(out) : "r"(addr), "r"(rank));
  return out;
}
__device__ __forceinline__ void st_cluster_f32(uint32_t addr, float v) {
  asm volatile("st.shared::cluster.f32 [%0], %1;" ::"r"(addr), "f"(v) : "memory");
}
__device__ __forceinline__ void mbar_arrive_remote(uint32_t addr) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(addr) : "memory");
}
// Bounded wait on a local barrier phase completed by arrivals from other CTAs of the
// cluster (acquire at cluster scope, so their stores before the arrival are visible).
__device__ __forceinline__ bool mbar_wait_cluster(uint64_t* bar, uint32_t parity, int* err) {
  for (uint32_t i = 0; i < kSpinLimit; ++i) {
    uint32_t done;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
        : "=r"(done)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    if (done) return true;
  }
  report(err, TQ_ERR_TIMEOUT);
  return false;
}

__device__ __forceinline__ bool elect_lane() {
  uint32_t pred;
  asm volatile(
      "{\n .reg .b32 r;\n .reg .pred p;\n elect.sync r|p, 0xffffffff;\n selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(pred));
  return pred != 0;
}

// Shared-memory bytes of the stream kernel for n_rows activation rows of K values and a
// ring of nch chunks.
__host__ __device__ constexpr int stream_smem(int n_rows, int K, int n_tc, int nch) {
  return 128 + nch * sk::CHUNK + sk::NS16 * sk::SLOT16 + sk::MAX_S * n_rows * sk::PART_ROW +
         n_rows * (((K + 15) & ~15) + 16) + n_tc * 12;
}

// Ring chunks for a call: as many as leave room for two CTAs per SM (at least 2, at
// most MAX_NCH); with activations too large for that, the ring of a single CTA per SM.
__host__ __device__ constexpr int stream_chunks(int n_rows, int K, int n_tc) {
  const int two = (113 * 1024 - stream_smem(n_rows, K, n_tc, 0)) / sk::CHUNK;
  const int one = (226 * 1024 - stream_smem(n_rows, K, n_tc, 0)) / sk::CHUNK;
  const int n = two >= 3 ? two : one;
  return n < 2 ? 2 : (n > sk::MAX_NCH ? sk::MAX_NCH : n);
}

// Fused activation quantization (the consumers, after the wait): column tiles
// [c_lo, c_hi) of the 16-bit activations, all n_rows rows, become INT8 codes in `act`
// (row stride act_ld, column c at (c - c_lo) * 64) and scales in sxs[c], exactly as the
// activation quantizer makes them: scale = dtype(absmax / 127) over the tile's rows
// and columns, code = rint(x / scale) clamped (quantize.cu).  Warp w takes tiles
// c_lo + w, c_lo + w + 4, ...; lane l reads the 16-byte piece l % 8 of rows l / 8,
// l / 8 + 4, ...; up to four tiles' loads are in flight at once.
template <int XT>
__device__ __forceinline__ void quantize_columns(const RowsArgs& a, int8_t* act, int act_ld, float* sxs, int c_lo,
                                                 int c_hi, int warp, int lane) {
  constexpr int GRP = 4, RPL = 4;  // tiles per group, rows per lane (16 rows / 4)
  const int piece = lane & 7, r0 = lane >> 3;
  const uint16_t* x = reinterpret_cast<const uint16_t*>(a.x_fp);
  for (int c0 = c_lo + warp; c0 < c_hi; c0 += GRP * sk::CONS) {
    uint4 v[GRP][RPL];
#pragma unroll
    for (int gi = 0; gi < GRP; ++gi) {
      const int c = c0 + gi * sk::CONS, col = c * 64 + piece * 8;
#pragma unroll
      for (int k = 0; k < RPL; ++k) {
        const int row = r0 + 4 * k;
        v[gi][k] = (c < c_hi && row < a.n_rows && col < a.K)
                       ? *reinterpret_cast<const uint4*>(x + (int64_t)row * a.ld_xfp + col)
                       : make_uint4(0u, 0u, 0u, 0u);
      }
    }
#pragma unroll
    for (int gi = 0; gi < GRP; ++gi) {
      const int c = c0 + gi * sk::CONS;
      if (c >= c_hi) break;  // warp-uniform
      float m = 0.0f;
#pragma unroll
      for (int k = 0; k < RPL; ++k) {
        const uint32_t w4[4] = {v[gi][k].x, v[gi][k].y, v[gi][k].z, v[gi][k].w};
#pragma unroll
        for (int e = 0; e < 4; ++e)
          m = fmaxf(m, fmaxf(fabsf(h2f((uint16_t)(w4[e] & 0xffffu), XT)), fabsf(h2f((uint16_t)(w4[e] >> 16), XT))));
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
      const float sc = scale_from_absmax<XT>(m);
      const float rc = __frcp_rn(sc);
#pragma unroll
      for (int k = 0; k < RPL; ++k) {
        const int row = r0 + 4 * k;
        if (row >= a.n_rows) continue;
        const uint32_t w4[4] = {v[gi][k].x, v[gi][k].y, v[gi][k].z, v[gi][k].w};
        uint32_t o2[2] = {0u, 0u};
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int lo = quant_code_fast(h2f((uint16_t)(w4[e] & 0xffffu), XT), sc, rc);
          const int hi = quant_code_fast(h2f((uint16_t)(w4[e] >> 16), XT), sc, rc);
          o2[e >> 1] |= ((uint32_t)(lo & 0xff) | ((uint32_t)(hi & 0xff) << 8)) << ((e & 1) * 16);
        }
        *reinterpret_cast<uint2*>(act + row * act_ld + (c - c_lo) * 64 + piece * 8) = make_uint2(o2[0], o2[1]);
      }
      if (lane == 0) sxs[c] = sc;
    }
  }
}

template <int NB, int XT>
__global__ void __launch_bounds__(sk::THREADS) stream_kernel(const RowsArgs a, const __grid_constant__ StreamMaps maps) {
  using namespace sk;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 127) & ~uintptr_t(127));
  // activation rows padded by 16 bytes: the 8 rows one 16-byte load spans fall in distinct banks
  const int K = a.K, n_tc = a.n_tc, act_ld = ((K + 15) & ~15) + 16;
  const int NCH = a.ring_chunks;
  uint8_t* ring8 = smem;
  uint8_t* ring16 = ring8 + NCH * CHUNK;
  float* part = reinterpret_cast<float*>(ring16 + NS16 * SLOT16);  // MAX_S slots of n_rows x 64 (rank 0's)
  int8_t* act = reinterpret_cast<int8_t*>(part + MAX_S * a.n_rows * 64);
  float* sxs = reinterpret_cast<float*>(act + a.n_rows * act_ld);  // n_tc
  int* mcol = reinterpret_cast<int*>(sxs + n_tc);                 // column of each INT8 tile, from the first
  float* msw = reinterpret_cast<float*>(mcol + n_tc);             // its weight scale
  __shared__ __align__(8) uint64_t full8[MAX_NCH], empty8[MAX_NCH], full16[NS16], empty16[NS16], act_bar, red_bar;

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, g = lane >> 2, t = lane & 3;
  const int s = blockIdx.x, r = blockIdx.y, S = a.split;
  const int b8 = __ldg(a.rp8 + r), c8 = __ldg(a.rp8 + r + 1) - b8;
  const int lo8 = b8 + (c8 * s) / S, n8 = b8 + (c8 * (s + 1)) / S - lo8;
  int lo16 = 0, n16 = 0;
  if (a.has_fp16) {
    const int b16 = __ldg(a.rp16 + r), c16 = __ldg(a.rp16 + r + 1) - b16;
    lo16 = b16 + (c16 * s) / S;
    n16 = b16 + (c16 * (s + 1)) / S - lo16;
  }
  const int nchk = (n8 + CHK - 1) / CHK;

  if (tid == 0) {
    for (int i = 0; i < NCH; ++i) {
      mbar_init(&full8[i], 1);
      mbar_init(&empty8[i], CONS);
    }
    for (int i = 0; i < NS16; ++i) {
      mbar_init(&full16[i], 1);
      mbar_init(&empty16[i], CONS);
    }
    mbar_init(&act_bar, 1);
    mbar_init(&red_bar, S > 1 ? S - 1 : 1);  // rank 0: one arrival per other split
    fence_mbar_init();
  }
  __syncthreads();
  // every CTA of the cluster has initialised its barriers once this phase completes;
  // waited for only before the first remote access, at the end
  if (S > 1) asm volatile("barrier.cluster.arrive.relaxed.aligned;" ::: "memory");
  grid_dep_launch();  // the next kernel may start its own weight-side prologue

  bool ok = true;
  float acc[NB][4];  // consumers: this thread's outputs (rows wr, wr + 8 of the tile)
#pragma unroll
  for (int nb = 0; nb < NB; ++nb) acc[nb][0] = acc[nb][1] = acc[nb][2] = acc[nb][3] = 0.0f;
  if (warp == CONS) {
    // ================================================================ producer
    const bool leader = elect_lane();
    auto issue8 = [&](int q) {
      const int nt = min(CHK, n8 - q * CHK);
      const uint32_t bytes = (uint32_t)nt * 4096u;
      uint64_t* bar = &full8[q % NCH];
      mbar_expect_tx(bar, bytes);
      bulk_g2s(ring8 + (q % NCH) * CHUNK, a.w8 + (int64_t)(lo8 + q * CHK) * 4096, bytes, bar);
    };
    auto issue16_w = [&](int j) {
      uint64_t* bar = &full16[j % NS16];
      mbar_expect_tx(bar, SLOT16);  // the weight tile and its activation box
      bulk_g2s(ring16 + (j % NS16) * SLOT16, reinterpret_cast<const uint8_t*>(a.w16) + (int64_t)(lo16 + j) * W16B,
               W16B, bar);
    };
    auto issue16_x = [&](int j) {
      const int c = __ldg(a.ids16 + lo16 + j) % n_tc;
      tma_load_2d(ring16 + (j % NS16) * SLOT16 + W16B, &maps.xfp, c * 64, 0, &full16[j % NS16]);
    };
    // weights first: they do not depend on the preceding kernel
    if (leader) {
      if (n16) prefetch_tensormap(&maps.xfp);
      for (int q = 0; q < min(NCH, nchk); ++q) issue8(q);
      for (int j = 0; j < min(NS16, n16); ++j) issue16_w(j);
    }
    // the split's INT8 columns are one ascending range: only those activations are copied
    const int c_first = n8 ? __ldg(a.ids8 + lo8) % n_tc : 0;
    const int c_end = n8 ? __ldg(a.ids8 + lo8 + n8 - 1) % n_tc + 1 : 0;
    const uint32_t span = (uint32_t)(n8 ? min(c_end * 64, K) - c_first * 64 : 0);
    grid_dep_wait();  // activations come from the preceding kernel
    if (leader) {
      mbar_expect_tx(&act_bar, a.fused ? 0u : (uint32_t)a.n_rows * span);
      if (span && !a.fused)
        for (int row = 0; row < a.n_rows; ++row)
          bulk_g2s(act + row * act_ld, a.x_i8 + (int64_t)row * a.ld_x8 + c_first * 64, span, &act_bar);
      for (int j = 0; j < min(NS16, n16); ++j) issue16_x(j);
    }
#pragma unroll 1
    for (int q = NCH; q < nchk && ok; ++q) {
      ok = mbar_wait_bounded(&empty8[q % NCH], (uint32_t)(((q / NCH) - 1) & 1), a.err);
      if (ok && leader) issue8(q);
    }
#pragma unroll 1
    for (int j = NS16; j < n16 && ok; ++j) {
      ok = mbar_wait_bounded(&empty16[j % NS16], (uint32_t)(((j / NS16) - 1) & 1), a.err);
      if (ok && leader) {
        issue16_w(j);
        issue16_x(j);
      }
    }
  } else {
    // ================================================================ consumers
    const int c_first = n8 ? __ldg(a.ids8 + lo8) % n_tc : 0;  // activations in shared memory start here
    for (int i = tid; i < n8; i += CONS * 32) {  // weight-side metadata, before the wait
      mcol[i] = __ldg(a.ids8 + lo8 + i) % n_tc - c_first;
      msw[i] = a.s8 ? __ldg(a.s8 + lo8 + i) : 1.0f;
    }
    grid_dep_wait();  // activations come from the preceding kernel, which may also still read `out`
    if (a.fused) {
      if (n8) quantize_columns<XT>(a, act, act_ld, sxs, c_first, __ldg(a.ids8 + lo8 + n8 - 1) % n_tc + 1, warp, lane);
    } else {
      for (int c = tid; c < n_tc; c += CONS * 32) sxs[c] = a.sx ? __ldg(a.sx + c) : 1.0f;
    }
    named_bar_sync(1, CONS * 32);
    ok = mbar_wait_bounded(&act_bar, 0, a.err);

    const int wr = 16 * warp + g;  // this thread's weight rows: wr and wr + 8
#pragma unroll 1
    for (int q = 0; q < nchk && ok; ++q) {
      const int slot = q % NCH;
      ok = mbar_wait_bounded(&full8[slot], (uint32_t)((q / NCH) & 1), a.err);
      if (!ok) break;
      const uint8_t* chunk = ring8 + slot * CHUNK;
      const int nt = min(CHK, n8 - q * CHK), i0 = q * CHK;
      // the chunk's four tiles in stages, so their loads and MMAs overlap: metadata,
      // operands, INT32 tile dots, then the fold in list order
      int c[CHK];
      float sc[CHK];
#pragma unroll
      for (int u = 0; u < CHK; ++u) c[u] = u < nt ? mcol[i0 + u] : 0;
#pragma unroll
      for (int u = 0; u < CHK; ++u) sc[u] = u < nt ? sxs[c_first + c[u]] * msw[i0 + u] : 0.0f;  // (sx * sw) in f32, ref :135-137
      uint4 wl[CHK], wh[CHK], xa[CHK][NB];
#pragma unroll
      for (int u = 0; u < CHK; ++u) {
        const uint8_t* tile = chunk + u * 4096;
        wl[u] = lds16(tile + wr * 64 + 16 * t);
        wh[u] = lds16(tile + (wr + 8) * 64 + 16 * t);
#pragma unroll
        for (int nb = 0; nb < NB; ++nb) {
          const int row = nb * 8 + g;  // activation rows past n_rows count as zero
          xa[u][nb] = row < a.n_rows ? lds16(act + row * act_ld + c[u] * 64 + 16 * t) : make_uint4(0u, 0u, 0u, 0u);
        }
      }
      int d[CHK][NB][4];
#pragma unroll
      for (int u = 0; u < CHK; ++u)
#pragma unroll
        for (int nb = 0; nb < NB; ++nb) {
          d[u][nb][0] = d[u][nb][1] = d[u][nb][2] = d[u][nb][3] = 0;
          mma_s8_16832(d[u][nb], wl[u].x, wh[u].x, wl[u].y, wh[u].y, xa[u][nb].x, xa[u][nb].y);
          mma_s8_16832(d[u][nb], wl[u].z, wh[u].z, wl[u].w, wh[u].w, xa[u][nb].z, xa[u][nb].w);
        }
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty8[slot]);  // the operands are in registers now
#pragma unroll
      for (int u = 0; u < CHK; ++u)
        if (u < nt)
#pragma unroll
          for (int nb = 0; nb < NB; ++nb)
#pragma unroll
            for (int e = 0; e < 4; ++e) acc[nb][e] = __fadd_rn(acc[nb][e], __fmul_rn(i2f_stream(d[u][nb][e]), sc[u]));
    }
    // the split's 16-bit tiles, each as two 32-column halves (m16n8k16, FP32 accumulate)
#pragma unroll 1
    for (int j = 0; j < n16 && ok; ++j) {
      const int slot = j % NS16;
      ok = mbar_wait_bounded(&full16[slot], (uint32_t)((j / NS16) & 1), a.err);
      if (!ok) break;
      const uint8_t* wt = ring16 + slot * SLOT16;
      const uint8_t* xb = wt + W16B;
#pragma unroll
      for (int half = 0; half < 2; ++half) {
        const uint4 wlo = lds16(wt + (wr * 64 + half * 32 + 8 * t) * 2);
        const uint4 whi = lds16(wt + ((wr + 8) * 64 + half * 32 + 8 * t) * 2);
#pragma unroll
        for (int nb = 0; nb < NB; ++nb) {
          const uint4 xv = lds16(xb + ((nb * 8 + g) * 64 + half * 32 + 8 * t) * 2);
          mma_16816<XT>(acc[nb], wlo.x, whi.x, wlo.y, whi.y, xv.x, xv.y);
          mma_16816<XT>(acc[nb], wlo.z, whi.z, wlo.w, whi.w, xv.z, xv.w);
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty16[slot]);
    }
    // acc[nb][e]: output column r * 64 + wr + 8 (e >> 1), activation row 8 nb + 2 t + (e & 1)
    if (S == 1) {
#pragma unroll
      for (int nb = 0; nb < NB; ++nb)
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int rr = nb * 8 + 2 * t + (e & 1), cc = r * 64 + wr + 8 * (e >> 1);
          if (ok && rr < a.n_rows && cc < a.M && a.out) {
            const int ot = a.out_dtype;
            uint16_t y = f2h(acc[nb][e], ot);
            if (a.bias) y = f2h(h2f(y, ot) + h2f(reinterpret_cast<const uint16_t*>(a.bias)[cc], ot), ot);
            reinterpret_cast<uint16_t*>(a.out)[(int64_t)rr * a.ldo + cc] = y;
          }
        }
    }
  }

  if (S > 1) {
    // The splits of row tile r meet in rank 0 (split 0): every other split stores its
    // partial into its slot of rank 0's shared memory and arrives on rank 0's barrier,
    // then exits; rank 0 adds the slots in split order and writes the output.
    asm volatile("barrier.cluster.wait.aligned;" ::: "memory");
    const int E = a.n_rows * 64;
    if (warp < CONS) {
      const int wr = 16 * warp + g;
      float* slot = part + s * E;
      const uint32_t base = s == 0 ? smem_u32(slot) : mapa_rank(smem_u32(slot), 0);
#pragma unroll
      for (int nb = 0; nb < NB; ++nb)
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int rr = nb * 8 + 2 * t + (e & 1);
          if (rr < a.n_rows) st_cluster_f32(base + (uint32_t)(rr * 64 + wr + 8 * (e >> 1)) * 4u, acc[nb][e]);
        }
    }
    __syncthreads();
    if (s != 0) {
      if (tid == 0) {
        asm volatile("fence.acq_rel.cluster;" ::: "memory");
        mbar_arrive_remote(mapa_rank(smem_u32(&red_bar), 0));
      }
      return;
    }
    ok = mbar_wait_cluster(&red_bar, 0, a.err) && ok;
    for (int e = tid; e < E; e += THREADS) {
      float v = part[e];
#pragma unroll
      for (int p = 1; p < MAX_S; ++p)
        if (p < S) v += part[p * E + e];  // split order, reference :170-176
      const int rr = e / 64, cc = r * 64 + (e % 64);
      if (ok && cc < a.M && a.out) {
        const int ot = a.out_dtype;
        uint16_t y = f2h(v, ot);
        if (a.bias) y = f2h(h2f(y, ot) + h2f(reinterpret_cast<const uint16_t*>(a.bias)[cc], ot), ot);
        reinterpret_cast<uint16_t*>(a.out)[(int64_t)rr * a.ldo + cc] = y;
      }
    }
  }
}

}  // namespace tq

using namespace tq;

// Clusters of `split` CTAs the stream kernel can hold resident at once for this shape
// (cached per shared-memory size and split: the same answer on every B200).
static int stream_max_clusters(int split, int smem, bool two) {
  static int cache[2][sk::MAX_S + 1][64] = {};  // [two][split][smem in 4 KB steps]
  const int key = std::min(63, smem >> 12);
  int& c = cache[two][split][key];
  if (c) return c;
  auto kern = two ? stream_kernel<2, TQ_DTYPE_BF16> : stream_kernel<1, TQ_DTYPE_BF16>;
  if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) != cudaSuccess) return 0;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)split, 1, 1);
  cfg.blockDim = dim3(sk::THREADS, 1, 1);
  cfg.dynamicSmemBytes = (size_t)smem;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = (unsigned)split;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  int n = 0;
  if (cudaOccupancyMaxActiveClusters(&n, kern, &cfg) != cudaSuccess || n <= 0) {
    cudaGetLastError();
    return 0;
  }
  return c = n;
}

// The split the stream kernel uses when none is given: the most splits (up to the
// portable cluster size, at least 4 INT8 tiles each) whose n_tr clusters are all
// resident at once; 1 when even that takes more than one wave.
int tq_stream_split(int n_tr, int n_tc, int n_rows) {
  const int rows = std::max(1, std::min(16, n_rows)), K = n_tc * 64;
  const int smem = stream_smem(rows, K, n_tc, stream_chunks(rows, K, n_tc));
  const bool two = n_rows > 8;
  int best = 1;
  for (int s = 2; s <= sk::MAX_S && s * 4 <= n_tc; ++s) {
    if (stream_max_clusters(s, smem, two) < n_tr) break;
    best = s;
  }
  return best;
}

// Whether the stream kernel takes this call: <= 16 rows, split 1..8, K a multiple of 16,
// 16-byte aligned INT8 activation rows (or, with fused quantization, 16-bit ones), 16-bit
// activation rows a tensor map can address, and the activations fitting in shared
// memory with the rings.
int tq_stream_supported(const RowsArgs& a) {
  if (a.n_rows <= 0 || a.n_rows > 16 || a.partials) return 0;
  if (a.split < 0 || a.split > sk::MAX_S || (a.K & 15)) return 0;
  if (!a.fused && (!a.x_i8 || ((uintptr_t)a.x_i8 & 15) || (a.ld_x8 & 15))) return 0;
  const bool need_fp = a.has_fp16 || a.fused;  // the 16-bit activations are read (TMA box / quantizer)
  if (need_fp && (!a.x_fp || ((uintptr_t)a.x_fp & 15) || ((a.ld_xfp * 2) & 15))) return 0;
  if (a.has_fp16 && (((uintptr_t)a.w16 & 15) || a.K < 64)) return 0;
  return stream_smem(a.n_rows, a.K, a.n_tc, stream_chunks(a.n_rows, a.K, a.n_tc)) <= 227 * 1024;
}

template <int NB, int XT>
static int launch_stream_t(const RowsArgs& a, const StreamMaps& maps, int n_tr, cudaStream_t st) {
  const int smem = stream_smem(a.n_rows, a.K, a.n_tc, a.ring_chunks);
  TQ_CUDA_TRY(cudaFuncSetAttribute(stream_kernel<NB, XT>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)a.split, (unsigned)n_tr, 1);
  cfg.blockDim = dim3(sk::THREADS, 1, 1);
  cfg.dynamicSmemBytes = (size_t)smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[2];
  int na = 0;
  if (a.split > 1) {
    attr[na].id = cudaLaunchAttributeClusterDimension;
    attr[na].val.clusterDim.x = (unsigned)a.split;
    attr[na].val.clusterDim.y = 1;
    attr[na].val.clusterDim.z = 1;
    ++na;
  }
  if (tq_pdl_enabled()) {
    attr[na].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[na].val.programmaticStreamSerializationAllowed = 1;
    ++na;
  }
  cfg.attrs = attr;
  cfg.numAttrs = na;
  TQ_CUDA_TRY(cudaLaunchKernelEx(&cfg, stream_kernel<NB, XT>, a, maps));
  tq_count_launch();
  return TQ_OK;
}

int tq_launch_stream(RowsArgs& a, int n_tr, int fp_dtype, cudaStream_t st) {
  a.n_tr = n_tr;
  if (a.split == 0) a.split = tq_stream_split(n_tr, a.n_tc, a.n_rows);
  if (!tq_stream_supported(a)) return tq_set_error(TQ_ERR_UNSUPPORTED, "stream decode kernel: unsupported call");
  a.ring_chunks = stream_chunks(a.n_rows, a.K, a.n_tc);
  StreamMaps maps;
  memset(&maps, 0, sizeof(maps));
  if (a.has_fp16) {
    const CUtensorMapDataType dt = fp_dtype == TQ_DTYPE_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16
                                                               : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
    const int rc = tq_encode_2d(&maps.xfp, dt, 2, a.x_fp, (uint64_t)a.K, (uint64_t)a.n_rows, (uint64_t)a.ld_xfp * 2, 64,
                                16, CU_TENSOR_MAP_SWIZZLE_NONE);
    if (rc != TQ_OK) return rc;
  }
  const bool two = a.n_rows > 8;
  if (fp_dtype == TQ_DTYPE_BF16)
    return two ? launch_stream_t<2, TQ_DTYPE_BF16>(a, maps, n_tr, st) : launch_stream_t<1, TQ_DTYPE_BF16>(a, maps, n_tr, st);
  return two ? launch_stream_t<2, TQ_DTYPE_F16>(a, maps, n_tr, st) : launch_stream_t<1, TQ_DTYPE_F16>(a, maps, n_tr, st);
}

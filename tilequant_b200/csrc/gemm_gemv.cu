// Decode-sized mixed INT8/BF16 64x64 tile GEMM (up to 16 activation rows), sm_100a.
//
// Reference: src/kernels/triton/gemm_rows_splitk_64x64.py:78-190 with SPLIT_K = S:
// split s of row tile r owns positions [b + cnt*s/S, b + cnt*(s+1)/S) of the row's INT8
// list and of its 16-bit list; acc = acc + f32(i32 tile dot) * (sx[c] * sw[pos]) (mul
// and add rounded separately) in ascending column order, then acc += dot(x, W16^T);
// the split partials are added in split order 0..S-1, rounded, then the bias.
//
// Decode is a latency problem: a 3072 x 3072 layer streams 9.75 MB, about 1.5 us of
// HBM time, so every dependent round trip to memory counts.  Layout for that:
//   * one CTA per (row tile r, 16-column slice m of its 64 output columns): n_tr * 4
//     CTAs, and warp s of the CTA is split s -- the reference's split-K becomes a
//     warp split with an in-CTA, in-order shared-memory reduction, no clusters;
//   * operands go from global memory straight into MMA fragments: a thread's share of
//     a 64x64 INT8 tile slice is two 16-byte loads, so all of a warp's tiles are in
//     flight at once with no shared-memory staging, no barriers and no bulk-copy
//     engine round trip (a plain 16-byte load returns in about a quarter of the time
//     of a bulk copy here);
//   * everything that depends only on the weights (row pointers, tile ids, scales and
//     the weight fragments themselves) is loaded before griddepcontrol.wait, so under
//     programmatic dependent launch it overlaps the kernel that produces the
//     activations; only the activation loads follow the wait;
//   * swap-AB mma.sync m16n8k32 (weights = M side, tokens = N side in two blocks of 8)
//     with the k order permuted identically for both operands (every thread holds 16
//     contiguous bytes of a row), so the exact INT32 dot is unchanged.
// Quantization stays a separate launch: quantizing inside this kernel repeats it in
// every CTA (n_tr * 4 times per column tile), which cost more than the launch saved.
// The results are bit-identical to the split-K row kernel at the same split.
//
// Row-parallel peer sum (PEER): for a tensor-parallel projection split along K, the
// partial outputs of the ranks are summed inside this kernel instead of by a separate
// all-reduce.  CTA b writes its FP32 partial (16 rows x 16 columns) into slot b of every
// rank's exchange buffer over NVLink (the buffers are CUDA IPC mappings), one 64-bit
// word per value: the value's bits and the CTA's call number, stored with one relaxed
// system-scope 64-bit store.  A 64-bit scalar access is single-copy atomic, so a reader
// that sees the current call number in a word sees that call's value with it: no fence
// or separate flag is needed.  A reader polls each word of its own buffer until it holds
// the current call number (bounded by a timeout that sets an error word, never
// forever), adds the partials of ranks 0..world-1 in that order, rounds and adds the bias
// -- the same bits on every rank.  Partials alternate between two halves
// of the buffer by call parity: a rank can only write call e + 2 after finishing call
// e + 1, which needed every rank's call e + 1 partial, so every rank has read its call
// e partials by then.  All CTAs of the grid must be resident at once (the launcher
// checks), so a waiting CTA never holds the SM a peer's partial needs.  (A first form
// published each slot with a release flag after the data; the fence behind the release
// and the flag round trip cost about 10 us per call on two B200s, as much as the NCCL
// all-reduce it replaced.)
#include "common.cuh"
#include "gemm_args.cuh"
#include "tma.cuh"

namespace tq {

namespace gv {
constexpr int U = 6;        // INT8 tiles per warp the automatic split aims for
constexpr int MAX_S = 8;    // splits (warps) per CTA
constexpr int PSTRIDE = 260;  // floats per split partial (16 columns x 16 tokens, padded)
}  // namespace gv

__device__ __forceinline__ uint4 ldg16(const void* p) { return *reinterpret_cast<const uint4*>(p); }

// 16 bytes at byte offset `off` of a row of `len` valid bytes; zeros past the end.
// `vec`: the row start is 16-byte aligned (else bytes are read one by one).
__device__ __forceinline__ uint4 ldg16_row(const uint8_t* row, int off, int len, bool vec) {
  if (vec && off + 16 <= len) return ldg16(row + off);
  uint32_t w[4] = {0u, 0u, 0u, 0u};
  for (int e = 0; e < 16 && off + e < len; ++e) w[e >> 2] |= (uint32_t)row[off + e] << ((e & 3) * 8);
  return make_uint4(w[0], w[1], w[2], w[3]);
}

__device__ __forceinline__ uint64_t globaltimer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}
// Exchange words: {call number (high 32 bits), value bits (low 32 bits)}, written and read
// with relaxed system-scope 64-bit scalar accesses (single-copy atomic; peer buffers
// change under the reader, so every read goes to memory).
__device__ __forceinline__ void st_word(uint64_t* p, uint64_t v) {
  asm volatile("st.relaxed.sys.global.b64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ uint64_t ld_word(const uint64_t* p) {
  uint64_t v;
  asm volatile("ld.relaxed.sys.global.b64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ float i2f_exact_gv(int v) {
  return __fsub_rn(__int_as_float(v + 0x4B400000), 12582912.0f);  // exact for |v| < 2^22
}

// Weight fragments, column ids and weight scales of up to N consecutive INT8 tiles.
template <int N>
struct WChunk {
  uint4 wl[N], wh[N];
  int col[N];
  float sw[N];
  int n;
};

template <int N>
__device__ __forceinline__ void load_w(const RowsArgs& a, WChunk<N>& c, int p0, int hi8, int wr, int t) {
  c.n = max(0, min(N, hi8 - p0));
#pragma unroll
  for (int u = 0; u < N; ++u) {
    if (u < c.n) {
      const int8_t* tile = a.w8 + (int64_t)(p0 + u) * 4096;
      c.wl[u] = ldg16(tile + wr * 64 + 16 * t);
      c.wh[u] = ldg16(tile + (wr + 8) * 64 + 16 * t);
      c.col[u] = __ldg(a.ids8 + p0 + u);  // tile id; the column is taken when it is needed
      c.sw[u] = a.s8 ? __ldg(a.s8 + p0 + u) : 1.0f;
    }
  }
}

// Activations of a chunk and its MMAs.
template <int N>
__device__ __forceinline__ void run_chunk(const RowsArgs& a, const WChunk<N>& c, float (&acc)[2][4], int g, int t,
                                          int rb) {
  uint4 xa[N][2];
  float sc[N];
  int col[N];  // the loads of the whole chunk are issued before any of them is used
#pragma unroll
  for (int u = 0; u < N; ++u) col[u] = c.col[u] % a.n_tc;
#pragma unroll
  for (int u = 0; u < N; ++u) {
    if (u < c.n) {
#pragma unroll
        for (int nb = 0; nb < 2; ++nb) {
          const int row = rb + nb * 8 + g;
          xa[u][nb] = row < a.n_rows ? ldg16_row(reinterpret_cast<const uint8_t*>(a.x_i8) + (int64_t)row * a.ld_x8,
                                                 col[u] * 64 + 16 * t, a.K, a.a8_vec != 0)
                                     : make_uint4(0u, 0u, 0u, 0u);
        }
        sc[u] = (a.sx ? __ldg(a.sx + col[u]) : 1.0f) * c.sw[u];  // (sx * sw) in f32, reference :135-137
    }
  }
#pragma unroll
  for (int u = 0; u < N; ++u) {
    if (u < c.n) {
#pragma unroll
      for (int nb = 0; nb < 2; ++nb) {
        int d[4] = {0, 0, 0, 0};
        mma_s8_16832(d, c.wl[u].x, c.wh[u].x, c.wl[u].y, c.wh[u].y, xa[u][nb].x, xa[u][nb].y);
        mma_s8_16832(d, c.wl[u].z, c.wh[u].z, c.wl[u].w, c.wh[u].w, xa[u][nb].z, xa[u][nb].w);
#pragma unroll
        for (int q = 0; q < 4; ++q) acc[nb][q] = __fadd_rn(acc[nb][q], __fmul_rn(i2f_exact_gv(d[q]), sc[u]));
      }
    }
  }
}

template <int XT, bool PEER>
__global__ void __launch_bounds__(gv::MAX_S * 32, 2) gemv_kernel(const RowsArgs a) {
  constexpr int UC = 6;  // INT8 tiles per chunk

  using namespace gv;
  __shared__ float part[MAX_S * PSTRIDE];
  const int S = blockDim.x >> 5;
  const int r = blockIdx.x >> 2, m = blockIdx.x & 3;
  const int rb = blockIdx.y * 16;  // first activation row of this CTA's 16-row block
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, g = lane >> 2, t = lane & 3;
  const int wr = 16 * m + g;  // this thread's weight rows in the tile: wr and wr + 8

  grid_dep_launch();  // the next kernel may start its own weight-side prologue

  const int b8 = __ldg(a.rp8 + r), c8 = __ldg(a.rp8 + r + 1) - b8;
  const int lo8 = b8 + (c8 * warp) / S, hi8 = b8 + (c8 * (warp + 1)) / S;
  int lo16 = 0, hi16 = 0;
  if (a.has_fp16) {
    const int b16 = __ldg(a.rp16 + r), c16 = __ldg(a.rp16 + r + 1) - b16;
    lo16 = b16 + (c16 * warp) / S;
    hi16 = b16 + (c16 * (warp + 1)) / S;
  }

  float acc[2][4];
#pragma unroll
  for (int nb = 0; nb < 2; ++nb)
#pragma unroll
    for (int q = 0; q < 4; ++q) acc[nb][q] = 0.0f;

  // INT8 tiles in chunks of UC per warp, every load of a chunk in flight together; the
  // first chunk's weights are requested before the wait for the preceding kernel.
  WChunk<UC> ch;
  load_w(a, ch, lo8, hi8, wr, t);
  grid_dep_wait();  // activations (and their scales) come from the preceding kernel
  run_chunk(a, ch, acc, g, t, rb);
#pragma unroll 1
  for (int p0 = lo8 + UC; p0 < hi8; p0 += UC) {
    load_w(a, ch, p0, hi8, wr, t);
    run_chunk(a, ch, acc, g, t, rb);
  }

  // 16-bit tiles of this split, each as two 32-column halves (m16n8k16, FP32 accumulate)
#pragma unroll 1
  for (int p = lo16; p < hi16; ++p) {
    const uint16_t* tile = reinterpret_cast<const uint16_t*>(a.w16) + (int64_t)p * 4096;
    const int c = __ldg(a.ids16 + p) % a.n_tc;
#pragma unroll
    for (int half = 0; half < 2; ++half) {
      const uint4 wlo = ldg16(tile + wr * 64 + half * 32 + 8 * t);
      const uint4 whi = ldg16(tile + (wr + 8) * 64 + half * 32 + 8 * t);
#pragma unroll
      for (int nb = 0; nb < 2; ++nb) {
        const int row = rb + nb * 8 + g;
        uint4 xb = make_uint4(0u, 0u, 0u, 0u);
        if (row < a.n_rows)
          xb = ldg16_row(reinterpret_cast<const uint8_t*>(a.x_fp) + (int64_t)row * a.ld_xfp * 2,
                         (c * 64 + half * 32 + 8 * t) * 2, a.K * 2, a.afp_vec != 0);
        mma_16816<XT>(acc[nb], wlo.x, whi.x, wlo.y, whi.y, xb.x, xb.y);
        mma_16816<XT>(acc[nb], wlo.z, whi.z, wlo.w, whi.w, xb.z, xb.w);
      }
    }
  }

  // split partials: column j = g + 8 (q >> 1) of the slice, token 8 nb + 2 t + (q & 1)
  float* mine = part + warp * PSTRIDE;
#pragma unroll
  for (int nb = 0; nb < 2; ++nb)
#pragma unroll
    for (int q = 0; q < 4; ++q) mine[(g + 8 * (q >> 1)) * 16 + nb * 8 + 2 * t + (q & 1)] = acc[nb][q];
  __syncthreads();
  if constexpr (PEER) {
    __shared__ __align__(16) float red[256];
    __shared__ uint32_t s_ep;
    for (int e = tid; e < 256; e += blockDim.x) {
      float v = part[e];
      for (int s = 1; s < S; ++s) v += part[s * PSTRIDE + e];  // split order, reference :170-176
      red[e] = v;
    }
    const int b = blockIdx.y * gridDim.x + blockIdx.x, W = a.world, slots = a.peer_slots;
    if (tid == 0) {  // only this CTA of this rank touches its counter; launches are stream-ordered
      const uint32_t ep = a.peer_epochs[b] + 1u;
      a.peer_epochs[b] = ep;
      s_ep = ep;
    }
    __syncthreads();
    const uint32_t ep = s_ep;
    // element e of a slot is word e: {call, value bits}
    constexpr int ELEMS = 2 * PEER_WORDS;  // 256 values per slot, 8 bytes each (the slot's 2 KB)
    const int64_t par_base = (int64_t)(ep & 1u) * W * slots * ELEMS;
    for (int i = tid; i < ELEMS * W; i += blockDim.x) {
      const int p = i / ELEMS, e = i % ELEMS;
      uint64_t* dst = reinterpret_cast<uint64_t*>(a.peer_bufs[p]) + par_base + ((int64_t)a.rank * slots + b) * ELEMS + e;
      st_word(dst, ((uint64_t)ep << 32) | __float_as_uint(red[e]));
    }
    // this CTA's slot of every source rank, in this rank's own buffer
    const uint64_t* src = reinterpret_cast<const uint64_t*>(a.peer_bufs[a.rank]) + par_base + (int64_t)b * ELEMS;
    const int64_t src_stride = (int64_t)slots * ELEMS;
    bool gave_up = false;
    for (int e = tid; e < ELEMS; e += blockDim.x) {
      float v = 0.0f;
      for (int p = 0; p < W; ++p) {  // rank order
        uint64_t q = ld_word(src + p * src_stride + e);
        if ((uint32_t)(q >> 32) != ep && !gave_up) {
          const uint64_t t0 = globaltimer_ns();
          while ((uint32_t)(q >> 32) != ep) {
            if ((int64_t)(globaltimer_ns() - t0) > a.peer_timeout_ns) {
              report(a.err, TQ_ERR_TIMEOUT);
              gave_up = true;
              break;
            }
            q = ld_word(src + p * src_stride + e);
          }
        }
        const float x = __uint_as_float((uint32_t)q);
        v = p == 0 ? x : v + x;
      }
      const int j = e >> 4, tok = e & 15;
      const int cc = r * 64 + 16 * m + j;
      if (rb + tok < a.n_rows && cc < a.M && a.out) {
        const int ot = a.out_dtype;
        uint16_t y = f2h(v, ot);
        if (a.bias) y = f2h(h2f(y, ot) + h2f(reinterpret_cast<const uint16_t*>(a.bias)[cc], ot), ot);
        reinterpret_cast<uint16_t*>(a.out)[(int64_t)(rb + tok) * a.ldo + cc] = y;
      }
    }
    return;
  }
  for (int e = tid; e < 256; e += blockDim.x) {
    const int j = e >> 4, tok = e & 15;
    float v = part[e];
    for (int s = 1; s < S; ++s) v += part[s * PSTRIDE + e];  // split order, reference :170-176
    const int cc = r * 64 + 16 * m + j;
    if (rb + tok < a.n_rows && cc < a.M && a.out) {
      const int ot = a.out_dtype;
      uint16_t y = f2h(v, ot);
      if (a.bias) y = f2h(h2f(y, ot) + h2f(reinterpret_cast<const uint16_t*>(a.bias)[cc], ot), ot);
      reinterpret_cast<uint16_t*>(a.out)[(int64_t)(rb + tok) * a.ldo + cc] = y;
    }
  }
}

}  // namespace tq

using namespace tq;

// Split the decode kernel uses when none is given: enough warps that each holds at most
// gv::U INT8 tiles of a full row (all its loads in flight at once), a power of two.
int tq_gemv_split(int n_tc) {
  int s = 1;
  while (s < gv::MAX_S && (n_tc + s - 1) / s > gv::U) s *= 2;
  return s;
}

int tq_gemv_supported(const RowsArgs& a) {
  return a.n_rows > 0 && a.n_rows <= 16 && !a.partials && !a.fused && a.split >= 0 && a.split <= gv::MAX_S;
}

// Whether the automatic choice for <= 16 rows is this kernel rather than the split-K
// row kernel: measured on B200, it wins while its grid (4 CTAs per row tile) fits in one
// wave and each warp holds at most 2 * U INT8 tiles (e.g. 3584 x 3584: 8.3 against
// 10.7 us at 4 rows), and loses beyond (37888 x 3584: 69 against 40 us; 3584 x 18944:
// 34 against 28 us), where the row kernel's bulk-copy stream keeps more bytes in flight.
int tq_gemv_preferred(const RowsArgs& a, int n_tr) {
  if (!tq_gemv_supported(a)) return 0;
  const int split = a.split ? a.split : tq_gemv_split(a.n_tc);
  if ((a.n_tc + split - 1) / split > 2 * gv::U) return 0;
  static int per_sm[gv::MAX_S + 1] = {};  // resident CTAs per SM by split (the same on every B200)
  if (!per_sm[split]) {
    int n = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, gemv_kernel<TQ_DTYPE_BF16, false>, 32 * split, 0) !=
            cudaSuccess || n <= 0)
      return 0;
    per_sm[split] = n;
  }
  return (int64_t)n_tr * 4 <= (int64_t)per_sm[split] * tq_sm_count();
}

// The peer-sum form also takes up to 64 rows, as 16-row blocks along the grid's y.
int tq_gemv_peer_supported(const RowsArgs& a) {
  return a.n_rows > 0 && a.n_rows <= 64 && !a.partials && !a.fused && a.split >= 0 && a.split <= gv::MAX_S;
}

template <int XT, bool PEER>
static int launch_gemv_t(const RowsArgs& a, const cudaLaunchConfig_t& cfg) {
  if (PEER) {  // a waiting CTA must never hold the SM a later CTA of its grid needs
    int per_sm = 0;
    TQ_CUDA_TRY(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, gemv_kernel<XT, PEER>, cfg.blockDim.x, 0));
    if ((int64_t)per_sm * tq_sm_count() < (int64_t)cfg.gridDim.x * cfg.gridDim.y)
      return tq_set_error(TQ_ERR_UNSUPPORTED, "peer sum: the decode grid does not fit on the GPU at once");
  }
  TQ_CUDA_TRY(cudaLaunchKernelEx(&cfg, gemv_kernel<XT, PEER>, a));
  return TQ_OK;
}

int tq_launch_gemv(RowsArgs& a, int n_tr, int fp_dtype, cudaStream_t st) {
  a.n_tr = n_tr;
  a.a8_vec = a.x_i8 && ((uintptr_t)a.x_i8 & 15) == 0 && (a.ld_x8 & 15) == 0;
  a.afp_vec = a.x_fp && ((uintptr_t)a.x_fp & 15) == 0 && ((a.ld_xfp * 2) & 15) == 0;
  if (a.split == 0) a.split = tq_gemv_split(a.n_tc);
  if (a.split < 1 || a.split > gv::MAX_S) return tq_set_error(TQ_ERR_UNSUPPORTED, "decode kernel: split_k must be in 1..8");
  if ((int64_t)n_tr * 4 > INT32_MAX) return tq_set_error(TQ_ERR_INVALID, "too many row tiles");
  cudaLaunchConfig_t cfg = {};
  const int row_blocks = (a.n_rows + 15) / 16;  // 1 on the plain decode path (<= 16 rows)
  cfg.gridDim = dim3((unsigned)(n_tr * 4), (unsigned)row_blocks, 1);
  cfg.blockDim = dim3(32 * a.split, 1, 1);
  cfg.dynamicSmemBytes = 0;
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
  if (a.world > 0 && (int64_t)n_tr * 4 * row_blocks > a.peer_slots)
    return tq_set_error(TQ_ERR_INVALID, "peer sum: more decode CTAs than exchange slots");
  const bool peer = a.world > 0;
  int rc;
  if (fp_dtype == TQ_DTYPE_BF16)
    rc = peer ? launch_gemv_t<TQ_DTYPE_BF16, true>(a, cfg) : launch_gemv_t<TQ_DTYPE_BF16, false>(a, cfg);
  else
    rc = peer ? launch_gemv_t<TQ_DTYPE_F16, true>(a, cfg) : launch_gemv_t<TQ_DTYPE_F16, false>(a, cfg);
  if (rc != TQ_OK) return rc;
  tq_count_launch();
  return TQ_OK;
}

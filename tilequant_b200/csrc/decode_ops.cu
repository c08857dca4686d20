// Fused decode-step kernels of the CUDA-graph greedy decoder (sm_100a).
//
// One decode step of a Llama/Qwen2 decoder layer is, besides its four projection GEMMs,
// a residual add, two RMSNorms, RoPE on Q and K, a KV-cache write, one query token's
// attention over the cache, SiLU(gate) * up and the INT8 quantization of each
// projection's input.  Run as framework operators that is about forty small launches
// per layer; here it is five kernels, each reading its operands once:
//
//   add_rmsnorm_kernel      h = resid + delta (16-bit), y = w * rmsnorm(h)
//   attn_partial_kernel     RoPE of the query heads of one KV head, the new token's K/V
//                           into the cache, then a split of the valid cache prefix
//                           streamed through shared memory by TMA and reduced on the
//                           tensor cores with an online softmax
//   attn_combine_kernel     the splits of one 64-column tile of a query head merged, the
//                           output rounded to 16 bits and quantized for the O projection
//   silu_mul_quant_kernel   a = silu(gate), h = a * up (16-bit), quantized per tile
//
// Elementwise arithmetic follows the decoder's own torch code operation by operation
// (each 16-bit op computed in f32 and rounded): the residual add, RoPE
// (q * cos + rotate_half(q) * sin with every product and the sum rounded), the RMSNorm's
// 16-bit round before the weight multiply, silu(x) = x / (1 + exp(-x)) rounded before the
// multiply by up.  The RMSNorm's f32 sum of squares and the attention's reductions are
// exact up to their summation order.  The INT8 codes and scales are those of the
// activation quantizer (quantize.cu) for the same 16-bit values.
#include <algorithm>

#include "common.cuh"
#include "tma.cuh"

namespace tq {

using AttnArgs = tq_attn_args;

template <int XT>
__device__ __forceinline__ float ldh(const void* p, int64_t i) {
  return h2f(reinterpret_cast<const uint16_t*>(p)[i], XT);
}
template <int XT>
__device__ __forceinline__ void sth(void* p, int64_t i, float v) {
  reinterpret_cast<uint16_t*>(p)[i] = f2h(v, XT);
}

__device__ __forceinline__ float block_sum(float v, float* red) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  __syncthreads();
  if (lane == 0) red[warp] = v;
  __syncthreads();
  if (warp == 0) {
    v = lane < (int)(blockDim.x >> 5) ? red[lane] : 0.0f;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    if (lane == 0) red[0] = v;
  }
  __syncthreads();
  return red[0];
}

// ------------------------------------------------------------------ residual + RMSNorm
// One CTA per row, 256 threads; thread t owns the 16-byte pieces t, t + 256, ... of the
// row (NVT of them at most), all loaded before any is used.  delta may be null (the first
// layer's input is the embedding).  resid_out may alias resid (each piece is read, then
// written, by one thread).
template <int XT, int NVT>
__global__ void __launch_bounds__(256) add_rmsnorm_kernel(const void* resid, int64_t ld_r, const void* delta,
                                                          int64_t ld_d, const void* __restrict__ w,
                                                          void* resid_out, int64_t ld_ro, void* __restrict__ y,
                                                          int64_t ld_y, int H, float eps) {
  __shared__ float red[32];
  grid_dep_wait();
  grid_dep_launch();
  const int64_t row = blockIdx.x;
  const int nvec = H / 8;
  uint4 rv[NVT], dv[NVT];
#pragma unroll
  for (int i = 0; i < NVT; ++i) {
    const int v = threadIdx.x + i * 256;
    rv[i] = dv[i] = make_uint4(0u, 0u, 0u, 0u);
    if (v < nvec) {
      rv[i] = *reinterpret_cast<const uint4*>(reinterpret_cast<const uint16_t*>(resid) + row * ld_r + v * 8);
      if (delta) dv[i] = *reinterpret_cast<const uint4*>(reinterpret_cast<const uint16_t*>(delta) + row * ld_d + v * 8);
    }
  }
  float h[NVT][8];
  float ss = 0.0f;
#pragma unroll
  for (int i = 0; i < NVT; ++i) {
    const uint32_t r4[4] = {rv[i].x, rv[i].y, rv[i].z, rv[i].w};
    const uint32_t d4[4] = {dv[i].x, dv[i].y, dv[i].z, dv[i].w};
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      float x = h2f((uint16_t)(r4[e >> 1] >> ((e & 1) * 16)), XT);
      if (delta) x = round16(__fadd_rn(x, h2f((uint16_t)(d4[e >> 1] >> ((e & 1) * 16)), XT)), XT);
      h[i][e] = x;
      if (threadIdx.x + i * 256 < nvec) ss = __fadd_rn(ss, __fmul_rn(x, x));
    }
  }
  const float total = block_sum(ss, red);
  const float inv = rsqrtf(__fadd_rn(__fmul_rn(total, 1.0f / (float)H), eps));
#pragma unroll
  for (int i = 0; i < NVT; ++i) {
    const int v = threadIdx.x + i * 256;
    if (v < nvec) {
      const uint4 wv = *reinterpret_cast<const uint4*>(reinterpret_cast<const uint16_t*>(w) + v * 8);
      const uint32_t w4[4] = {wv.x, wv.y, wv.z, wv.w};
      uint32_t ho[4], yo[4];
#pragma unroll
      for (int e = 0; e < 8; e += 2) {
        const float n0 = round16(__fmul_rn(h[i][e], inv), XT), n1 = round16(__fmul_rn(h[i][e + 1], inv), XT);
        const float y0 = __fmul_rn(h2f((uint16_t)(w4[e >> 1] & 0xffffu), XT), n0);
        const float y1 = __fmul_rn(h2f((uint16_t)(w4[e >> 1] >> 16), XT), n1);
        ho[e >> 1] = (uint32_t)f2h(h[i][e], XT) | ((uint32_t)f2h(h[i][e + 1], XT) << 16);
        yo[e >> 1] = (uint32_t)f2h(y0, XT) | ((uint32_t)f2h(y1, XT) << 16);
      }
      if (delta)
        *reinterpret_cast<uint4*>(reinterpret_cast<uint16_t*>(resid_out) + row * ld_ro + v * 8) =
            make_uint4(ho[0], ho[1], ho[2], ho[3]);
      *reinterpret_cast<uint4*>(reinterpret_cast<uint16_t*>(y) + row * ld_y + v * 8) =
          make_uint4(yo[0], yo[1], yo[2], yo[3]);
    }
  }
}

// ------------------------------------------------------------------ SiLU(gate) * up
// One CTA per 64-column tile, every row (<= 128): the tile stays in shared memory
// between its absmax and its codes.
template <int XT>
__global__ void __launch_bounds__(256) silu_mul_quant_kernel(const void* __restrict__ gate,
                                                             const void* __restrict__ up, int64_t ld_gu,
                                                             int n_rows, int k, void* __restrict__ h, int64_t ld_h,
                                                             int8_t* __restrict__ q, int64_t ldq,
                                                             float* __restrict__ sx) {
  __shared__ float tile[128 * 64];
  __shared__ float red[32];
  grid_dep_wait();
  grid_dep_launch();
  const int c = blockIdx.x;
  const int width = min(64, k - c * 64);
  float m = 0.0f;
  for (int e = threadIdx.x; e < n_rows * 64; e += blockDim.x) {
    const int r = e >> 6, j = e & 63;
    float v = 0.0f;
    if (j < width) {
      const int64_t col = (int64_t)c * 64 + j;
      const float g = ldh<XT>(gate, r * ld_gu + col), u = ldh<XT>(up, r * ld_gu + col);
      const float a = round16(__fdiv_rn(g, __fadd_rn(1.0f, expf(-g))), XT);
      v = round16(__fmul_rn(a, u), XT);
      sth<XT>(h, r * ld_h + col, v);
    }
    tile[e] = v;
    m = fmaxf(m, fabsf(v));
  }
  m = block_max(m, red);
  const float s = scale_from_absmax<XT>(m);
  const float rc = __frcp_rn(s);
  for (int e = threadIdx.x; e < n_rows * 64; e += blockDim.x) {
    const int r = e >> 6, j = e & 63;
    if (j < width) q[r * ldq + (int64_t)c * 64 + j] = (int8_t)quant_code_fast(tile[e], s, rc);
  }
  if (threadIdx.x == 0) sx[c] = s;
}

// ------------------------------------------------------------------ decode attention
// Split-KV attention of one query token per sequence (FlashAttention-2's online
// softmax, published form, scores kept in the log2 domain: p = 2^(s * scale * log2 e - m)).
//
// CTA = (split s, KV head, batch row); its split is a run of 64-slot chunks of the valid
// prefix [0, pos].  Each chunk of K and of V is brought into shared memory by 2-D TMA
// loads (64-column boxes, 128-byte swizzle), three chunks in flight; chunks that do not
// hold the new token are requested before the wait for the QKV projection, so they
// stream while it finishes.  Warp w takes slots [16w, 16w + 16) of every chunk:
//   S = Q K^T   mma m16n8k16, A = the (up to 8) rotated query heads of the KV head
//               (rows >= G zero), B = K rows via ldmatrix (conflict-free on the swizzle)
//   O += P V    A = P straight from S's accumulator registers (rounded to 16 bits, as
//               flash attention does), B = V via ldmatrix.trans
// and keeps its own running max / sum / output; the four warps merge at the end and
// the CTA writes its split's partial.  attn_combine_kernel merges the splits.
namespace at {
constexpr int CH = 64;            // cache slots per chunk (16 per warp)
constexpr int NSTG = 3;           // chunks in flight per CTA
constexpr int WARPS = 4;
constexpr int BOXB = CH * 128;    // one 64-column box of a chunk
constexpr int MAXG = 8;           // query heads per KV head
}  // namespace at

struct AttnMaps {
  CUtensorMap k, v;  // [B*Hkv*L rows][D] 16-bit, box 64 x CH, 128-byte swizzle
};

__device__ __forceinline__ void ldsm_x4(uint32_t (&r)[4], uint32_t addr) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t (&r)[4], uint32_t addr) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr));
}
// Shared address of 16-byte piece c (0 .. D/8-1) of chunk row r: box c / 8, and within
// the box the 128-byte swizzle (piece index XOR row mod 8).
__device__ __forceinline__ uint32_t swz(uint32_t base, int r, int c) {
  return base + (uint32_t)((c >> 3) * at::BOXB + r * 128 + (((c & 7) ^ (r & 7)) << 4));
}
// 8 rotated values d0..d0+7 of one head x[0..D) (16-byte aligned pieces):
// round(round(x * cos) + round(rotate_half(x) * sin)), rotate_half(x)[d] = -x[d + D/2]
// for d < D/2 and x[d - D/2] above.
template <int XT>
__device__ __forceinline__ uint4 rope8(const uint16_t* x, int d0, int D, const void* cosp, const void* sinp) {
  const bool lower = d0 < D / 2;
  const uint4 xv = *reinterpret_cast<const uint4*>(x + d0);
  const uint4 rv = *reinterpret_cast<const uint4*>(x + (lower ? d0 + D / 2 : d0 - D / 2));
  const uint4 cv = *reinterpret_cast<const uint4*>(reinterpret_cast<const uint16_t*>(cosp) + d0);
  const uint4 sv = *reinterpret_cast<const uint4*>(reinterpret_cast<const uint16_t*>(sinp) + d0);
  const uint32_t x4[4] = {xv.x, xv.y, xv.z, xv.w}, r4[4] = {rv.x, rv.y, rv.z, rv.w};
  const uint32_t c4[4] = {cv.x, cv.y, cv.z, cv.w}, s4[4] = {sv.x, sv.y, sv.z, sv.w};
  uint32_t o4[4];
#pragma unroll
  for (int e = 0; e < 4; ++e) {
    float o[2];
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const float xx = h2f((uint16_t)(x4[e] >> (16 * h)), XT);
      float rr = h2f((uint16_t)(r4[e] >> (16 * h)), XT);
      if (lower) rr = -rr;
      const float cc = h2f((uint16_t)(c4[e] >> (16 * h)), XT), ss = h2f((uint16_t)(s4[e] >> (16 * h)), XT);
      o[h] = round16(__fadd_rn(round16(__fmul_rn(xx, cc), XT), round16(__fmul_rn(rr, ss), XT)), XT);
    }
    o4[e] = (uint32_t)f2h(o[0], XT) | ((uint32_t)f2h(o[1], XT) << 16);
  }
  return make_uint4(o4[0], o4[1], o4[2], o4[3]);
}

template <int XT>
__device__ __forceinline__ uint32_t pack2(float lo, float hi) {
  return (uint32_t)f2h(lo, XT) | ((uint32_t)f2h(hi, XT) << 16);
}

template <int XT, int D>
__global__ void __launch_bounds__(at::WARPS * 32) attn_partial_kernel(const AttnArgs a,
                                                                      const __grid_constant__ AttnMaps maps) {
  using namespace at;
  constexpr int NBX = D / 64, STB = NBX * BOXB, KS = D / 16, NBLK = D / 8;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* ks = smem;                                                // NSTG x STB
  uint8_t* vs = smem + NSTG * STB;                                   // NSTG x STB
  uint16_t* qh = reinterpret_cast<uint16_t*>(vs + NSTG * STB);       // MAXG x D rotated query heads
  __shared__ __align__(8) uint64_t full[NSTG];
  __shared__ float mrg_m[WARPS * MAXG], mrg_l[WARPS * MAXG];

  const int s = blockIdx.x, kvh = blockIdx.y, b = blockIdx.z;
  const int G = a.Hq / a.Hkv;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, g = lane >> 2, t = lane & 3;
  const int64_t pos = *a.pos;  // advanced by an earlier step, not by the kernel this one follows
  const int n = (int)pos + 1;  // valid slots, the new token's included
  const int chunks = (n + CH - 1) / CH;
  const int per = (chunks + a.S - 1) / a.S;
  const int lo = min(n, s * per * CH), hi = min(n, (s + 1) * per * CH);
  const int nch = hi > lo ? (hi - lo + CH - 1) / CH : 0;
  const int pos_chunk = (pos >= lo && pos < hi) ? (int)(pos - lo) / CH : -1;
  const int row0 = (b * a.Hkv + kvh) * a.L;  // first cache row of this (b, kv head)

  if (tid == 0) {
    prefetch_tensormap(&maps.k);
    prefetch_tensormap(&maps.v);
    for (int i = 0; i < NSTG; ++i) mbar_init(&full[i], 1);
    fence_mbar_init();
  }
  __syncthreads();
  auto issue = [&](int ci) {  // chunk ci into stage ci % NSTG (one thread)
    const int st = ci % NSTG, y = row0 + lo + ci * CH;
    mbar_expect_tx(&full[st], 2 * STB);
#pragma unroll
    for (int x = 0; x < NBX; ++x) {
      tma_load_2d(ks + st * STB + x * BOXB, &maps.k, x * 64, y, &full[st]);
      tma_load_2d(vs + st * STB + x * BOXB, &maps.v, x * 64, y, &full[st]);
    }
  };
  int issued = 0;
  const int first = min(NSTG, nch);
  if (tid == 0)
    while (issued < first && issued != pos_chunk) issue(issued++);

  grid_dep_wait();  // q, k, v come from the preceding projection
  grid_dep_launch();

  // RoPE of the query heads: round(round(q * cos) + round(rotate_half(q) * sin)) (the
  // decoder's apply_rotary_pos_emb, op by op); rows G..7 zero.  One 16-byte piece (8
  // values, all in one half of the head) per thread: every load in one round.
  for (int pc = tid; pc < MAXG * D / 8; pc += blockDim.x) {
    const int hh = pc / (D / 8), d0 = (pc % (D / 8)) * 8;
    uint4 outv = make_uint4(0u, 0u, 0u, 0u);
    if (hh < G) {
      const int64_t base = (int64_t)b * a.ld_q + (int64_t)(kvh * G + hh) * D;
      outv = rope8<XT>(reinterpret_cast<const uint16_t*>(a.q) + base, d0, D, a.cos, a.sin);
    }
    *reinterpret_cast<uint4*>(qh + hh * D + d0) = outv;
  }
  // the split holding slot pos writes the new token's rotated K and its V there; its
  // TMA loads of that chunk read them after the proxy fence and the barrier
  if (pos_chunk >= 0) {
    const int64_t kb = (int64_t)b * a.ld_k + (int64_t)kvh * D, vb = (int64_t)b * a.ld_v + (int64_t)kvh * D;
    const int64_t dst = ((int64_t)row0 + pos) * D;
    for (int pc = tid; pc < D / 8; pc += blockDim.x) {
      const int d0 = pc * 8;
      *reinterpret_cast<uint4*>(reinterpret_cast<uint16_t*>(a.k_cache) + dst + d0) =
          rope8<XT>(reinterpret_cast<const uint16_t*>(a.k) + kb, d0, D, a.cos, a.sin);
      *reinterpret_cast<uint4*>(reinterpret_cast<uint16_t*>(a.v_cache) + dst + d0) =
          *reinterpret_cast<const uint4*>(reinterpret_cast<const uint16_t*>(a.v) + vb + d0);
    }
    asm volatile("fence.proxy.async.global;" ::: "memory");
  }
  __syncthreads();
  if (tid == 0)
    while (issued < first) issue(issued++);

  // the query heads as the A operand of S = Q K^T (rows g + 8 are empty)
  uint32_t qa[KS][2];
#pragma unroll
  for (int kp = 0; kp < KS; ++kp) {
    qa[kp][0] = *reinterpret_cast<const uint32_t*>(qh + g * D + kp * 16 + 2 * t);
    qa[kp][1] = *reinterpret_cast<const uint32_t*>(qh + g * D + kp * 16 + 8 + 2 * t);
  }
  float o[NBLK][4];
#pragma unroll
  for (int j = 0; j < NBLK; ++j) o[j][0] = o[j][1] = o[j][2] = o[j][3] = 0.0f;
  float m_run = -INFINITY, l_part = 0.0f;  // head g: running max (log2 domain), this lane's sum
  const float sl2 = a.scale_log2;
  const int r0 = warp * 16;
  bool ok = true;
#pragma unroll 1
  for (int ci = 0; ci < nch; ++ci) {
    const int st = ci % NSTG;
    ok = ok && mbar_wait_sleep(&full[st], (uint32_t)((ci / NSTG) & 1), a.err);
    const int slot0 = lo + ci * CH + r0;
    if (ok && slot0 < hi) {
      const uint32_t kb = smem_u32(ks + st * STB), vb = smem_u32(vs + st * STB);
      const int mat = lane >> 3;
      const int valid = hi - slot0;  // rows of this warp's 16 that hold slots of the split
      if (valid < 16) {  // the box also brought rows past the split: zero their V (P is 0 there)
        for (int e = lane; e < (16 - valid) * NBX * 8; e += 32) {
          const int rr = r0 + valid + e / (NBX * 8), pc = e % (NBX * 8);
          *reinterpret_cast<uint4*>(vs + st * STB + (pc >> 3) * BOXB + rr * 128 + (pc & 7) * 16) =
              make_uint4(0u, 0u, 0u, 0u);
        }
        fence_proxy_async();  // before any later bulk copy into this stage
        __syncwarp();
      }
      float sc[2][4] = {{0.0f, 0.0f, 0.0f, 0.0f}, {0.0f, 0.0f, 0.0f, 0.0f}};
#pragma unroll
      for (int kp = 0; kp < KS; ++kp) {
        uint32_t r[4];
        ldsm_x4(r, swz(kb, r0 + (mat >> 1) * 8 + (lane & 7), 2 * kp + (mat & 1)));
        mma_16816<XT>(sc[0], qa[kp][0], 0u, qa[kp][1], 0u, r[0], r[1]);
        mma_16816<XT>(sc[1], qa[kp][0], 0u, qa[kp][1], 0u, r[2], r[3]);
      }
      // head g, slots slot0 + 8 nb + 2t + j
      float v[4];
#pragma unroll
      for (int nb = 0; nb < 2; ++nb)
#pragma unroll
        for (int j = 0; j < 2; ++j)
          v[nb * 2 + j] = slot0 + nb * 8 + 2 * t + j < hi ? sc[nb][j] * sl2 : -INFINITY;
      float cm = fmaxf(fmaxf(v[0], v[1]), fmaxf(v[2], v[3]));
      cm = fmaxf(cm, __shfl_xor_sync(0xffffffffu, cm, 1));
      cm = fmaxf(cm, __shfl_xor_sync(0xffffffffu, cm, 2));
      const float mn = fmaxf(m_run, cm);
      const float base = mn == -INFINITY ? 0.0f : mn;
      float p[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) p[i] = exp2f(v[i] - base);
      const float corr = exp2f(m_run - base);
      m_run = mn;
      l_part = l_part * corr + ((p[0] + p[1]) + (p[2] + p[3]));
#pragma unroll
      for (int j = 0; j < NBLK; ++j) {
        o[j][0] *= corr;
        o[j][1] *= corr;
      }
      const uint32_t pa0 = pack2<XT>(p[0], p[1]), pa2 = pack2<XT>(p[2], p[3]);
#pragma unroll
      for (int jp = 0; jp < NBLK / 2; ++jp) {
        uint32_t r[4];
        ldsm_x4_t(r, swz(vb, r0 + (mat & 1) * 8 + (lane & 7), 2 * jp + (mat >> 1)));
        mma_16816<XT>(o[2 * jp], pa0, 0u, pa2, 0u, r[0], r[1]);
        mma_16816<XT>(o[2 * jp + 1], pa0, 0u, pa2, 0u, r[2], r[3]);
      }
    }
    // a stage is refilled only when a later chunk goes into it (ci + NSTG < nch, the same
    // for every thread): only then must every warp be done with it first
    if (ci + NSTG < nch) {
      __syncthreads();
      if (tid == 0 && ok) issue(ci + NSTG);
    }
  }
  l_part += __shfl_xor_sync(0xffffffffu, l_part, 1);
  l_part += __shfl_xor_sync(0xffffffffu, l_part, 2);

  // merge the four warps in the K stages: every load issued was awaited, and after this
  // barrier no warp still reads a stage
  __syncthreads();
  float* mrg_o = reinterpret_cast<float*>(ks);  // WARPS x MAXG x D
  if (g < G) {
    if (t == 0) {
      mrg_m[warp * MAXG + g] = m_run;
      mrg_l[warp * MAXG + g] = l_part;
    }
#pragma unroll
    for (int j = 0; j < NBLK; ++j) {
      mrg_o[(warp * MAXG + g) * D + j * 8 + 2 * t] = o[j][0];
      mrg_o[(warp * MAXG + g) * D + j * 8 + 2 * t + 1] = o[j][1];
    }
  }
  __syncthreads();
  for (int e = tid; e < G * D; e += blockDim.x) {
    const int hh = e / D, d = e % D;
    float mx = -INFINITY;
#pragma unroll
    for (int w = 0; w < WARPS; ++w) mx = fmaxf(mx, mrg_m[w * MAXG + hh]);
    float lsum = 0.0f, acc = 0.0f;
    if (mx != -INFINITY) {
#pragma unroll
      for (int w = 0; w < WARPS; ++w) {
        const float f = exp2f(mrg_m[w * MAXG + hh] - mx);
        lsum = fmaf(mrg_l[w * MAXG + hh], f, lsum);
        acc = fmaf(mrg_o[(w * MAXG + hh) * D + d], f, acc);
      }
    }
    const int64_t idx = ((int64_t)b * a.Hq + kvh * G + hh) * a.S + s;
    a.ws_o[idx * D + d] = ok ? acc : 0.0f;
    if (d == 0) {
      a.ws_m[idx] = ok ? mx : -INFINITY;
      a.ws_l[idx] = ok ? lsum : 0.0f;
    }
  }
}

// One CTA per 64-column tile of a query head (D / 64 per head), every batch row: merge
// the splits (a warp per row computes the row's max and the split weights; then each
// thread sums the weighted partials of one output, the split loads in flight together),
// round to 16 bits, then the tile's INT8 codes and scale (all rows share a scale).
template <int XT, int D>
__global__ void __launch_bounds__(256) attn_combine_kernel(const AttnArgs a, void* __restrict__ out, int64_t ld_out,
                                                           int8_t* __restrict__ q, int64_t ldq,
                                                           float* __restrict__ sx) {
  extern __shared__ float sm[];
  float* vals = sm;                   // B x 64 outputs of this tile
  float* wts = sm + a.B * 64;         // B x S split weights
  float* inv_l = wts + a.B * a.S;     // B: 1 / total sum (0 for an empty row)
  __shared__ float red[32];
  grid_dep_wait();
  grid_dep_launch();
  constexpr int TPH = D / 64;  // column tiles per head
  const int h = blockIdx.x / TPH, tile = blockIdx.x % TPH, S = a.S, B = a.B;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = blockDim.x >> 5;
  for (int b = warp; b < B; b += nw) {
    const int64_t base = ((int64_t)b * a.Hq + h) * S;
    const float m0 = lane < S ? a.ws_m[base + lane] : -INFINITY;
    const float m1 = lane + 32 < S ? a.ws_m[base + lane + 32] : -INFINITY;
    float mx = fmaxf(m0, m1);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    const float w0 = m0 == -INFINITY ? 0.0f : exp2f(m0 - mx), w1 = m1 == -INFINITY ? 0.0f : exp2f(m1 - mx);
    float ls = (lane < S ? a.ws_l[base + lane] * w0 : 0.0f) + (lane + 32 < S ? a.ws_l[base + lane + 32] * w1 : 0.0f);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) ls += __shfl_xor_sync(0xffffffffu, ls, o);
    if (lane < S) wts[b * S + lane] = w0;
    if (lane + 32 < S) wts[b * S + lane + 32] = w1;
    if (lane == 0) inv_l[b] = ls > 0.0f ? 1.0f / ls : 0.0f;
  }
  __syncthreads();
  float mv = 0.0f;
  for (int e = threadIdx.x; e < B * 64; e += blockDim.x) {
    const int b = e >> 6, d = tile * 64 + (e & 63);
    const float* po = a.ws_o + (((int64_t)b * a.Hq + h) * S) * D + d;
    const float* wb = wts + b * S;
    float acc = 0.0f;
#pragma unroll 8
    for (int s = 0; s < S; ++s) acc = fmaf(po[(int64_t)s * D], wb[s], acc);
    const float v = round16(acc * inv_l[b], XT);
    vals[e] = v;
    mv = fmaxf(mv, fabsf(v));
    sth<XT>(out, (int64_t)b * ld_out + (int64_t)h * D + d, v);
  }
  if (!q) return;
  mv = block_max(mv, red);  // also orders the vals writes before the reads below
  const float sc = scale_from_absmax<XT>(mv);
  const float rc = __frcp_rn(sc);
  for (int e = threadIdx.x; e < B * 64; e += blockDim.x) {
    const int b = e >> 6, j = e & 63;
    q[(int64_t)b * ldq + (int64_t)h * D + tile * 64 + j] = (int8_t)quant_code_fast(vals[e], sc, rc);
  }
  if (threadIdx.x == 0) sx[h * TPH + tile] = sc;
}

// ------------------------------------------------------------------ greedy pick
// argmax over each row of the logits (the first index of the maximum, as torch.argmax),
// then the decoder's bookkeeping: the token becomes the next input, is stored in the
// generated ids at column (position - prompt + 1), and the position advances.
// Pass 1 (grid: chunks x rows): each CTA's (max, first index) of its chunk, folded into
// a per-row 64-bit key with atomicMax: high word the value's bits made order-preserving,
// low word ~index, so the larger value wins and, among equal values, the smaller index.
__device__ __forceinline__ uint64_t pick_key(float v, uint32_t idx) {
  const uint32_t u = __float_as_uint(v);
  const uint32_t ord = (u & 0x80000000u) ? ~u : (u | 0x80000000u);
  return ((uint64_t)ord << 32) | (uint64_t)(0xFFFFFFFFu - idx);
}

template <int XT>
__global__ void __launch_bounds__(256) argmax_partial_kernel(const void* __restrict__ logits, int64_t ld, int V,
                                                             int chunk, unsigned long long* __restrict__ keys) {
  __shared__ unsigned long long red[8];
  grid_dep_wait();
  grid_dep_launch();
  const int row = blockIdx.y;
  const int lo = blockIdx.x * chunk, hi = min(V, lo + chunk);
  uint64_t best = 0;
  for (int j = lo + threadIdx.x; j < hi; j += blockDim.x) {
    const uint64_t k = pick_key(ldh<XT>(logits, (int64_t)row * ld + j), (uint32_t)j);
    best = k > best ? k : best;
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const uint64_t other = __shfl_xor_sync(0xffffffffu, best, o);
    best = other > best ? other : best;
  }
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = best;
  __syncthreads();
  if (threadIdx.x == 0) {
    for (int w = 1; w < (int)(blockDim.x >> 5); ++w) best = red[w] > best ? red[w] : best;
    atomicMax(keys + row, (unsigned long long)best);
  }
}

// Pass 2 (one CTA): decode the keys, write the bookkeeping, clear the keys for the next call.
__global__ void argmax_finish_kernel(unsigned long long* __restrict__ keys, int B, int64_t* __restrict__ next,
                                     int64_t* __restrict__ token, int64_t* __restrict__ generated, int64_t gen_ld,
                                     int64_t gen_cols, int64_t* __restrict__ position, int64_t prompt_tokens) {
  grid_dep_wait();
  grid_dep_launch();
  const int64_t col = *position - prompt_tokens + 1;
  for (int b = threadIdx.x; b < B; b += blockDim.x) {
    const int64_t id = (int64_t)(0xFFFFFFFFu - (uint32_t)(keys[b] & 0xFFFFFFFFull));
    keys[b] = 0ull;
    if (next) next[b] = id;
    if (token) token[b] = id;
    if (generated && col >= 0 && col < gen_cols) generated[(int64_t)b * gen_ld + col] = id;
  }
  __syncthreads();
  if (threadIdx.x == 0 && position) *position += 1;
}

}  // namespace tq

using namespace tq;

static int attn_smem(int D) { return 1024 + 2 * at::NSTG * (D / 64) * at::BOXB + at::MAXG * D * 2; }

template <int XT>
static int launch_norm(int nvt, const void* resid, int64_t ld_r, const void* delta, int64_t ld_d, const void* weight,
                       void* resid_out, int64_t ld_ro, void* y, int64_t ld_y, int64_t n_rows, int H, float eps,
                       cudaStream_t st) {
  auto kern = nvt == 1 ? add_rmsnorm_kernel<XT, 1>
                       : nvt == 2 ? add_rmsnorm_kernel<XT, 2> : nvt == 4 ? add_rmsnorm_kernel<XT, 4> : add_rmsnorm_kernel<XT, 8>;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)n_rows, 1, 1);
  cfg.blockDim = dim3(256, 1, 1);
  cfg.stream = st;
  cfg.attrs = attr;
  cfg.numAttrs = tq_pdl_enabled() ? 1 : 0;
  TQ_CUDA_TRY(cudaLaunchKernelEx(&cfg, kern, resid, ld_r, delta, ld_d, weight, resid_out, ld_ro, y, ld_y, H, eps));
  tq_count_launch();
  return TQ_OK;
}

extern "C" int tq_add_rmsnorm(const void* resid, int64_t ld_r, const void* delta, int64_t ld_d, const void* weight,
                              void* resid_out, int64_t ld_ro, void* y, int64_t ld_y, int64_t n_rows, int64_t hidden,
                              float eps, int dtype, void* stream) {
  if (dtype != TQ_DTYPE_BF16 && dtype != TQ_DTYPE_F16) return tq_set_error(TQ_ERR_INVALID, "dtype must be bf16 or f16");
  if (n_rows < 0 || hidden <= 0 || hidden > 16384 || hidden % 8)
    return tq_set_error(TQ_ERR_INVALID, "hidden must be a multiple of 8 in 8..16384");
  if (n_rows == 0) return TQ_OK;
  if (!resid || !weight || !y || (delta && !resid_out)) return tq_set_error(TQ_ERR_INVALID, "null pointer");
  if (ld_r < hidden || ld_y < hidden || (delta && (ld_d < hidden || ld_ro < hidden)))
    return tq_set_error(TQ_ERR_INVALID, "row stride smaller than hidden");
  const uintptr_t al = (uintptr_t)resid | (uintptr_t)weight | (uintptr_t)y | (uintptr_t)delta | (uintptr_t)resid_out;
  if ((al & 15) || ((ld_r | ld_y | (delta ? ld_d | ld_ro : 0)) & 7))
    return tq_set_error(TQ_ERR_INVALID, "rows must start on 16-byte boundaries");
  const int nvec = (int)(hidden / 8);
  const int nvt = nvec <= 256 ? 1 : nvec <= 512 ? 2 : nvec <= 1024 ? 4 : 8;
  cudaStream_t st = (cudaStream_t)stream;
  return dtype == TQ_DTYPE_BF16
             ? launch_norm<TQ_DTYPE_BF16>(nvt, resid, ld_r, delta, ld_d, weight, resid_out, ld_ro, y, ld_y, n_rows,
                                          (int)hidden, eps, st)
             : launch_norm<TQ_DTYPE_F16>(nvt, resid, ld_r, delta, ld_d, weight, resid_out, ld_ro, y, ld_y, n_rows,
                                         (int)hidden, eps, st);
}

extern "C" int tq_silu_mul_quant(const void* gate, const void* up, int64_t ld_gu, int64_t n_rows, int64_t k, void* h,
                                 int64_t ld_h, int8_t* q, int64_t ldq, float* sx, int dtype, void* stream) {
  if (dtype != TQ_DTYPE_BF16 && dtype != TQ_DTYPE_F16) return tq_set_error(TQ_ERR_INVALID, "dtype must be bf16 or f16");
  if (n_rows < 0 || n_rows > 128 || k < 0) return tq_set_error(TQ_ERR_INVALID, "n_rows must be in 0..128");
  if (n_rows == 0 || k == 0) return TQ_OK;
  if (!gate || !up || !h || !q || !sx) return tq_set_error(TQ_ERR_INVALID, "null pointer");
  if (ld_gu < k || ld_h < k || ldq < k) return tq_set_error(TQ_ERR_INVALID, "row stride smaller than k");
  const unsigned n_tc = (unsigned)((k + 63) / 64);
  cudaStream_t st = (cudaStream_t)stream;
  if (dtype == TQ_DTYPE_BF16)
    silu_mul_quant_kernel<TQ_DTYPE_BF16><<<n_tc, 256, 0, st>>>(gate, up, ld_gu, (int)n_rows, (int)k, h, ld_h, q, ldq, sx);
  else
    silu_mul_quant_kernel<TQ_DTYPE_F16><<<n_tc, 256, 0, st>>>(gate, up, ld_gu, (int)n_rows, (int)k, h, ld_h, q, ldq, sx);
  TQ_LAUNCHED();
  return TQ_OK;
}

extern "C" int tq_attn_decode_splits(int batch, int kv_heads, int max_len) {
  if (batch <= 0 || kv_heads <= 0 || max_len <= 0) return 1;
  // as many splits as keep every CTA resident at once (two per SM at this kernel's
  // shared memory), so no split waits for a second wave
  const int want = (2 * tq_sm_count()) / (batch * kv_heads);
  const int chunks = (max_len + at::CH - 1) / at::CH;
  return std::max(1, std::min({want, chunks, 64}));
}

template <int XT, int D>
static int launch_attn(const AttnArgs& a, const AttnMaps& maps, void* out, int64_t ld_out, int8_t* q_out, int64_t ldq,
                       float* sx, cudaStream_t st) {
  const int smem = attn_smem(D);
  TQ_CUDA_TRY(cudaFuncSetAttribute(attn_partial_kernel<XT, D>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)a.S, (unsigned)a.Hkv, (unsigned)a.B);
  cfg.blockDim = dim3(at::WARPS * 32, 1, 1);
  cfg.dynamicSmemBytes = (size_t)smem;
  cfg.stream = st;
  cfg.attrs = attr;
  cfg.numAttrs = tq_pdl_enabled() ? 1 : 0;
  TQ_CUDA_TRY(cudaLaunchKernelEx(&cfg, attn_partial_kernel<XT, D>, a, maps));
  tq_count_launch();
  cfg.gridDim = dim3((unsigned)(a.Hq * (D / 64)), 1, 1);
  cfg.blockDim = dim3(256, 1, 1);
  cfg.dynamicSmemBytes = ((size_t)a.B * 64 + (size_t)a.B * a.S + a.B) * 4;
  TQ_CUDA_TRY(cudaLaunchKernelEx(&cfg, attn_combine_kernel<XT, D>, a, out, ld_out, q_out, ldq, sx));
  tq_count_launch();
  return TQ_OK;
}

extern "C" int tq_attn_decode(const AttnArgs* args, void* out, int64_t ld_out, int8_t* q_out, int64_t ldq,
                              float* sx, int dtype, void* stream) {
  if (!args) return tq_set_error(TQ_ERR_INVALID, "null arguments");
  const AttnArgs a = *args;
  if (dtype != TQ_DTYPE_BF16 && dtype != TQ_DTYPE_F16) return tq_set_error(TQ_ERR_INVALID, "dtype must be bf16 or f16");
  if (a.D != 64 && a.D != 128) return tq_set_error(TQ_ERR_UNSUPPORTED, "head_dim must be 64 or 128");
  if (a.B <= 0 || a.B > 64 || a.Hkv <= 0 || a.Hq <= 0 || a.Hq % a.Hkv || a.Hq / a.Hkv > at::MAXG)
    return tq_set_error(TQ_ERR_UNSUPPORTED, "decode attention: batch 1..64, up to 8 query heads per KV head");
  if (a.L <= 0 || a.S < 1 || a.S > 64 || (int64_t)a.B * a.Hkv * a.L > INT32_MAX)
    return tq_set_error(TQ_ERR_INVALID, "decode attention: bad cache length or split");
  if (!a.q || !a.k || !a.v || !a.cos || !a.sin || !a.k_cache || !a.v_cache || !a.pos || !a.ws_m || !a.ws_l ||
      !a.ws_o || !out)
    return tq_set_error(TQ_ERR_INVALID, "null pointer");
  if ((((uintptr_t)a.k_cache) | ((uintptr_t)a.v_cache)) & 15)
    return tq_set_error(TQ_ERR_INVALID, "KV cache must be 16-byte aligned");
  if ((((uintptr_t)a.q) | ((uintptr_t)a.k) | ((uintptr_t)a.v) | ((uintptr_t)a.cos) | ((uintptr_t)a.sin)) & 15 ||
      ((a.ld_q | a.ld_k | a.ld_v) & 7))
    return tq_set_error(TQ_ERR_INVALID, "q, k, v, cos and sin must start (and their rows) on 16-byte boundaries");
  if (ld_out < (int64_t)a.Hq * a.D || (q_out && (!sx || ldq < (int64_t)a.Hq * a.D)))
    return tq_set_error(TQ_ERR_INVALID, "bad output stride or quantized output");
  const uint64_t rows = (uint64_t)a.B * a.Hkv * a.L;
  const CUtensorMapDataType tdt = dtype == TQ_DTYPE_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  AttnMaps maps;
  int rc = tq_encode_2d(&maps.k, tdt, 2, a.k_cache, (uint64_t)a.D, rows, (uint64_t)a.D * 2, 64, at::CH,
                        CU_TENSOR_MAP_SWIZZLE_128B);
  if (rc == TQ_OK)
    rc = tq_encode_2d(&maps.v, tdt, 2, a.v_cache, (uint64_t)a.D, rows, (uint64_t)a.D * 2, 64, at::CH,
                      CU_TENSOR_MAP_SWIZZLE_128B);
  if (rc != TQ_OK) return rc;
  cudaStream_t st = (cudaStream_t)stream;
  if (dtype == TQ_DTYPE_BF16)
    return a.D == 128 ? launch_attn<TQ_DTYPE_BF16, 128>(a, maps, out, ld_out, q_out, ldq, sx, st)
                      : launch_attn<TQ_DTYPE_BF16, 64>(a, maps, out, ld_out, q_out, ldq, sx, st);
  return a.D == 128 ? launch_attn<TQ_DTYPE_F16, 128>(a, maps, out, ld_out, q_out, ldq, sx, st)
                    : launch_attn<TQ_DTYPE_F16, 64>(a, maps, out, ld_out, q_out, ldq, sx, st);
}

extern "C" int tq_greedy_pick(const void* logits, int64_t ld, int64_t n_rows, int64_t vocab, int dtype,
                              unsigned long long* keys, int64_t* next, int64_t* token, int64_t* generated,
                              int64_t gen_ld, int64_t gen_cols, int64_t* position, int64_t prompt_tokens,
                              void* stream) {
  if (dtype != TQ_DTYPE_BF16 && dtype != TQ_DTYPE_F16) return tq_set_error(TQ_ERR_INVALID, "dtype must be bf16 or f16");
  if (n_rows <= 0 || n_rows > 1024 || vocab <= 0 || vocab > INT32_MAX / 2 || ld < vocab)
    return tq_set_error(TQ_ERR_INVALID, "greedy pick: 1..1024 rows of vocab <= ld logits");
  if (!logits || !keys || !position) return tq_set_error(TQ_ERR_INVALID, "null pointer");
  cudaStream_t st = (cudaStream_t)stream;
  const int chunk = 4096;
  const dim3 grid((unsigned)((vocab + chunk - 1) / chunk), (unsigned)n_rows, 1);
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = dim3(256, 1, 1);
  cfg.stream = st;
  cfg.attrs = attr;
  cfg.numAttrs = tq_pdl_enabled() ? 1 : 0;
  if (dtype == TQ_DTYPE_BF16)
    TQ_CUDA_TRY(cudaLaunchKernelEx(&cfg, argmax_partial_kernel<TQ_DTYPE_BF16>, logits, ld, (int)vocab, chunk, keys));
  else
    TQ_CUDA_TRY(cudaLaunchKernelEx(&cfg, argmax_partial_kernel<TQ_DTYPE_F16>, logits, ld, (int)vocab, chunk, keys));
  tq_count_launch();
  cfg.gridDim = dim3(1, 1, 1);
  cfg.blockDim = dim3(128, 1, 1);
  TQ_CUDA_TRY(cudaLaunchKernelEx(&cfg, argmax_finish_kernel, keys, (int)n_rows, next, token, generated, gen_ld, gen_cols,
                                 position, prompt_tokens));
  tq_count_launch();
  return TQ_OK;
}

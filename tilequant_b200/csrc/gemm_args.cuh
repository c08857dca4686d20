// Launch arguments shared by the mixed tile GEMM kernels.
#pragma once

#include <stdint.h>

namespace tq {

struct RowsArgs {
  const int8_t* x_i8;  // (n_rows, K) INT8 activations, row stride ld_x8 bytes
  int64_t ld_x8;
  const float* sx;     // f32[n_tc] activation scales
  const int8_t* w8;    // int8[T8][64][64]
  const float* s8;     // f32[T8]
  const int32_t* ids8;
  const int32_t* rp8;
  const void* x_fp;    // (n_rows, K) 16-bit activations, row stride ld_xfp elements
  int64_t ld_xfp;
  const void* w16;     // 16-bit [T16][64][64]
  const int32_t* ids16;
  const int32_t* rp16;
  void* out;           // (n_rows, M) 16-bit, row stride ldo; null = no output
  int64_t ldo;
  int out_dtype;       // TQ_DTYPE_* of out and bias
  const void* bias;
  int32_t* partials;   // debug dump of INT32 tile products, or null
  int* err;            // device error word, or null
  int n_rows, M, K, n_tc, split;
  int n_tr;            // row tiles of the weight
  int rows_per_cta;    // row tiles one CTA streams (rows kernel, split 1)
  int ring_chunks;     // 16 KB chunks in the weight ring (stream kernel)
  int64_t w8_rows;     // 64 * T8 (rows of the INT8 arena)
  int64_t w16_rows;    // 64 * T16
  int has_fp16;
  int a8_vec;          // x_i8 rows are 16-byte addressable
  int afp_vec;         // x_fp rows are 16-byte addressable
  int fused;           // quantize x_fp in the kernel (x_i8 / sx unused)
  int tma_x;           // activation tensor maps are valid (set by the launcher)
  // Row-parallel peer sum (decode kernel only; world 0 = off): CTA b of every rank
  // writes its FP32 partial tile into slot b of every rank's exchange buffer, then sums
  // the world partials found in its own buffer in rank order.
  float* const* peer_bufs;  // device array [world] of the exchange buffers, mapped on this GPU
  uint32_t* peer_epochs;    // this rank's per-CTA call counters [peer_slots]
  int world, rank, peer_slots;
  int64_t peer_timeout_ns;  // bound of every wait for a peer's partial
};

// Exchange buffer of the peer sum: [2 (call parity)][world (source rank)][slots] slots of
// 2 KB; a slot holds the 256 partial values (16 rows x 16 columns) of one CTA, one 64-bit
// word each: {call number (high 32 bits), value bits (low 32 bits)}.  PEER_WORDS counts
// the slot in 16-byte units.
constexpr int PEER_WORDS = 128;
__host__ __device__ constexpr int64_t peer_buffer_bytes(int world, int slots) {
  return (int64_t)2 * world * slots * PEER_WORDS * 16;
}

}  // namespace tq

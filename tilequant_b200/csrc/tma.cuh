// TMA tensor maps, programmatic dependent launch and named barriers (sm_100a).
#pragma once

#include <cudaTypedefs.h>

#include "common.cuh"

namespace tq {

// 2-D tiled TMA load of box (x, y) into shared memory, completion on `bar`.
// x * element size must be a multiple of 16 bytes (callers pass 64-byte multiples).
__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, int x, int y, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::
          "r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_u32(bar))
      : "memory");
}

// 3-D tiled TMA load of box (x, y, z) into shared memory, completion on `bar`.
__device__ __forceinline__ void tma_load_3d(void* dst, const CUtensorMap* map, int x, int y, int z, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4}], "
      "[%5];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(z), "r"(smem_u32(bar))
      : "memory");
}

__device__ __forceinline__ void prefetch_tensormap(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

// Adds tx bytes to the current phase without arriving.
__device__ __forceinline__ void mbar_add_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.expect_tx.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes) : "memory");
}

// The executing thread's prior cp.async copies arrive on `bar` when they complete
// (the arrival is part of the barrier's expected count).
__device__ __forceinline__ void cp_async_arrive_noinc(uint64_t* bar) {
  asm volatile("cp.async.mbarrier.arrive.noinc.shared::cta.b64 [%0];" ::"r"(smem_u32(bar)) : "memory");
}

// Programmatic dependent launch: wait for the preceding grid's memory, or let the
// next grid start its prologue.
__device__ __forceinline__ void grid_dep_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void grid_dep_launch() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

__device__ __forceinline__ void named_bar_sync(int id, int threads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(threads) : "memory");
}

}  // namespace tq

// Host: encode a 2-D row-major tensor map (inner dim `cols` elements, `rows` rows,
// row stride `ld_bytes`), box (box_cols, box_rows), zero fill out of bounds.
// Returns TQ_OK or TQ_ERR_UNSUPPORTED when the layout cannot be expressed.
int tq_encode_2d(CUtensorMap* map, CUtensorMapDataType dtype, int elem_bytes, const void* base, uint64_t cols,
                 uint64_t rows, uint64_t ld_bytes, uint32_t box_cols, uint32_t box_rows, CUtensorMapSwizzle swizzle);

// Host: encode a 3-D uint8 tensor map (dims d0 innermost .. d2, byte strides of dims 1
// and 2), box (b0, b1, b2), zero fill out of bounds.
int tq_encode_3d_u8(CUtensorMap* map, const void* base, uint64_t d0, uint64_t d1, uint64_t d2, uint64_t stride1,
                    uint64_t stride2, uint32_t b0, uint32_t b1, uint32_t b2, CUtensorMapSwizzle swizzle);

// Whether programmatic dependent launch is enabled (environment TQ_PDL, default on).
bool tq_pdl_enabled();

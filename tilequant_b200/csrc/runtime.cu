// Status codes, per-thread error messages and device queries of the C ABI.
#include <stdio.h>
#include <string.h>

#include "common.cuh"

static thread_local char g_last_error[512] = "";

int tq_set_error(int code, const char* msg) {
  snprintf(g_last_error, sizeof(g_last_error), "%s", msg);
  return code;
}

int tq_set_cuda_error(cudaError_t e) {
  snprintf(g_last_error, sizeof(g_last_error), "CUDA error %d: %s", (int)e, cudaGetErrorString(e));
  return TQ_ERR_CUDA;
}

int tq_sm_count() {
  static int cached[64] = {0};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return 148;
  if (dev < 0 || dev >= 64) return 148;
  if (!cached[dev]) {
    int n = 0;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) n = 148;
    cached[dev] = n;
  }
  return cached[dev];
}

#include <atomic>

static std::atomic<int64_t> g_launches{0};

void tq_count_launch(int n) { g_launches.fetch_add(n, std::memory_order_relaxed); }

extern "C" int64_t tq_kernel_launches(void) { return g_launches.load(std::memory_order_relaxed); }

extern "C" int tq_abi_version(void) { return 1; }

extern "C" const char* tq_last_error(void) { return g_last_error; }

extern "C" const char* tq_status_string(int status) {
  switch (status) {
    case TQ_OK: return "TQ_OK";
    case TQ_ERR_INVALID: return "TQ_ERR_INVALID";
    case TQ_ERR_UNSUPPORTED: return "TQ_ERR_UNSUPPORTED";
    case TQ_ERR_CUDA: return "TQ_ERR_CUDA";
    case TQ_ERR_TIMEOUT: return "TQ_ERR_TIMEOUT";
    default: return "TQ_ERR_UNKNOWN";
  }
}

// ------------------------------------------------------------ tensor maps

#include <stdlib.h>

#include "tma.cuh"

static PFN_cuTensorMapEncodeTiled_v12000 g_encode = nullptr;

static int load_encoder() {
  if (!g_encode) {
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult q;
    cudaError_t e = cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q);
    if (e != cudaSuccess || q != cudaDriverEntryPointSuccess || !fn)
      return tq_set_error(TQ_ERR_UNSUPPORTED, "cuTensorMapEncodeTiled is not available");
    g_encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
  }
  return TQ_OK;
}

int tq_encode_3d_u8(CUtensorMap* map, const void* base, uint64_t d0, uint64_t d1, uint64_t d2, uint64_t stride1,
                    uint64_t stride2, uint32_t b0, uint32_t b1, uint32_t b2, CUtensorMapSwizzle swizzle) {
  if (load_encoder() != TQ_OK) return TQ_ERR_UNSUPPORTED;
  if (((uintptr_t)base & 15) || (stride1 & 15) || (stride2 & 15) || !d0 || !d1 || !d2)
    return tq_set_error(TQ_ERR_UNSUPPORTED, "tensor map needs 16-byte aligned base and strides");
  cuuint64_t dims[3] = {d0, d1, d2};
  cuuint64_t strides[2] = {stride1, stride2};
  cuuint32_t box[3] = {b0, b1, b2};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = g_encode(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, const_cast<void*>(base), dims, strides, box, estr,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_128B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return tq_set_error(TQ_ERR_UNSUPPORTED, "cuTensorMapEncodeTiled rejected the 3-D layout");
  return TQ_OK;
}

int tq_encode_2d(CUtensorMap* map, CUtensorMapDataType dtype, int elem_bytes, const void* base, uint64_t cols,
                 uint64_t rows, uint64_t ld_bytes, uint32_t box_cols, uint32_t box_rows, CUtensorMapSwizzle swizzle) {
  if (load_encoder() != TQ_OK) return TQ_ERR_UNSUPPORTED;
  if (((uintptr_t)base & 15) || (ld_bytes & 15) || rows == 0 || cols == 0)
    return tq_set_error(TQ_ERR_UNSUPPORTED, "tensor map needs 16-byte aligned base and row stride");
  cuuint64_t dims[2] = {cols, rows};
  cuuint64_t strides[1] = {ld_bytes};
  cuuint32_t box[2] = {box_cols, box_rows};
  cuuint32_t estr[2] = {1, 1};
  (void)elem_bytes;
  CUresult r = g_encode(map, dtype, 2, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                        swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_128B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return tq_set_error(TQ_ERR_UNSUPPORTED, "cuTensorMapEncodeTiled rejected the layout");
  return TQ_OK;
}

bool tq_pdl_enabled() {
  static int v = -1;
  if (v < 0) {
    const char* s = getenv("TQ_PDL");
    v = (s && s[0] == '0') ? 0 : 1;
  }
  return v == 1;
}

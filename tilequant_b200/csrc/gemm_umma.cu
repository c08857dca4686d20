// Persistent TMA + tcgen05 mixed tile GEMM (prefill shapes).  Not built yet: the
// dispatcher never selects it.
#include "common.cuh"
#include "gemm_args.cuh"

int tq_umma_supported(int64_t, int64_t, int64_t, const int8_t*, int64_t, const void*, int64_t, const void*,
                      const void*) {
  return 0;
}

int tq_launch_umma(const tq::RowsArgs&, int, int, cudaStream_t) {
  return tq_set_error(TQ_ERR_UNSUPPORTED, "tcgen05 GEMM not available");
}

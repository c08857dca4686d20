// The peer-sum decode GEMM without any device allocation: tq_gemm_mixed_peer_sum_noalloc.
//
// For callers that cannot call cudaMalloc -- serving runtimes that hand all free device
// memory to their own pools at start-up (a late cudaMalloc fails or fragments them),
// and real-time host loops that cannot afford the device-wide synchronization a
// cudaMalloc / cudaFree may imply -- this form of the peer-sum decode kernel keeps all
// of its scratch (the exchange words, the per-CTA call counters and the one-entry table
// of exchange addresses) in one file-scope __device__ array.  Every GPU that loads the
// library holds that array (TQ_NOALLOC_SCRATCH_BYTES) until the process exits.
//
// It serves a world of one GPU: module-scope device memory is not reachable from other
// GPUs (CUDA IPC export needs cudaMalloc'd memory, and a kernel of another GPU in the
// same process faulted on it here even with peer access enabled), so the sums across
// GPUs stay with tq_gemm_mixed_peer_sum and its tq_peer_alloc buffers.
//
// Set-up, per device and with that device current: the array's device address
// (cudaGetSymbolAddress; in host code the array's name only stands for it) is looked up
// on every call, which is cheap, and the table entry that holds it is written with a
// synchronous copy whenever that address is new for the device -- so the first call on
// a device does that copy and should come before any stream capture.  Every call shares
// the array and it keeps the last call's state (the counters advance call by call; the
// exchange words of a call carry its number, so nothing has to be cleared between
// calls), so calls whose kernels overlap on one GPU race.  reset_only zeroes the
// counters and words again and rewrites the table entry, without a launch: use it after
// a timeout, and after a cudaDeviceReset (which reloads the array as zeros, possibly at
// the same address) before the next call.
#include <mutex>

#include "common.cuh"
#include "gemm_args.cuh"

namespace {
// scratch layout: [0, 256) the exchange-address table (one entry); then the call
// counters u32[TQ_NOALLOC_SLOTS] (padded to 256 bytes); then the exchange words
// [2][1][TQ_NOALLOC_SLOTS][PEER_WORDS] x 16 bytes.
constexpr size_t kTableOff = 0;
constexpr size_t kCountOff = 256;
constexpr size_t kWordsOff = kCountOff + ((TQ_NOALLOC_SLOTS * 4 + 255) / 256) * 256;
constexpr size_t kBytes = kWordsOff + (size_t)tq::peer_buffer_bytes(1, TQ_NOALLOC_SLOTS);
static_assert(kBytes == TQ_NOALLOC_SCRATCH_BYTES, "scratch size in the header");
}  // namespace

// The scratch: one copy per GPU that loads the library, zero at load.
static __device__ __align__(256) unsigned char tq_noalloc_scratch[kBytes];

namespace {
constexpr int kMaxDevices = 64;
std::mutex g_mu;
unsigned char* g_addr[kMaxDevices] = {};  // device address of the scratch, per device

// The scratch's address on the current device `dev`; the table entry is (re)written
// when the address differs from the one recorded for the device.
int scratch_of(int dev, unsigned char** out) {
  if (dev < 0 || dev >= kMaxDevices) return tq_set_error(TQ_ERR_INVALID, "no-alloc peer sum: device ordinal out of range");
  void* p = nullptr;
  if (cudaGetSymbolAddress(&p, tq_noalloc_scratch) != cudaSuccess || !p)
    return tq_set_error(TQ_ERR_CUDA, "no-alloc peer sum: cudaGetSymbolAddress of the scratch array failed");
  unsigned char* base = static_cast<unsigned char*>(p);
  std::lock_guard<std::mutex> lock(g_mu);
  if (g_addr[dev] != base) {
    float* words = reinterpret_cast<float*>(base + kWordsOff);
    TQ_CUDA_TRY(cudaMemcpy(base + kTableOff, &words, sizeof(words), cudaMemcpyHostToDevice));
    g_addr[dev] = base;
  }
  *out = base;
  return TQ_OK;
}
}  // namespace

extern "C" int tq_gemm_mixed_peer_sum_noalloc(
    const int8_t* x_i8, int64_t ld_x8, const float* sx, const int8_t* int8_tiles, const float* int8_scales,
    const int32_t* int8_tile_ids, const int32_t* int8_row_ptr, int64_t t8, const void* x_fp, int64_t ld_xfp,
    const void* fp16_tiles, const int32_t* fp16_tile_ids, const int32_t* fp16_row_ptr, int64_t t16, int fp_dtype,
    void* out, int64_t ldo, int out_dtype, const void* bias, int64_t n_rows, int64_t m, int64_t k, int n_tr, int n_tc,
    int split_k, int64_t timeout_ns, int reset_only, int* err, void* stream) {
  int dev = 0;
  TQ_CUDA_TRY(cudaGetDevice(&dev));
  unsigned char* base = nullptr;
  const int rc = scratch_of(dev, &base);
  if (rc) return rc;
  if (reset_only) {  // counters and words zero, the table entry rewritten (stream-ordered)
    float* words = reinterpret_cast<float*>(base + kWordsOff);
    TQ_CUDA_TRY(cudaMemcpyAsync(base + kTableOff, &words, sizeof(words), cudaMemcpyHostToDevice,
                                (cudaStream_t)stream));
    TQ_CUDA_TRY(cudaMemsetAsync(base + kCountOff, 0, kBytes - kCountOff, (cudaStream_t)stream));
    return TQ_OK;
  }
  if (n_rows > 16) return tq_set_error(TQ_ERR_UNSUPPORTED, "no-alloc peer sum: needs 1..16 rows");
  if ((int64_t)n_tr * 4 > TQ_NOALLOC_SLOTS)
    return tq_set_error(TQ_ERR_INVALID, "no-alloc peer sum: more than 256 row tiles (m > 16384) exceeds the "
                                        "scratch array's 1024 CTA slots");
  // the allocating entry point's checks and launch, on the scratch array
  return tq_gemm_mixed_peer_sum(x_i8, ld_x8, sx, int8_tiles, int8_scales, int8_tile_ids, int8_row_ptr, t8, x_fp,
                                ld_xfp, fp16_tiles, fp16_tile_ids, fp16_row_ptr, t16, fp_dtype, out, ldo, out_dtype,
                                bias, n_rows, m, k, n_tr, n_tc, split_k,
                                reinterpret_cast<float* const*>(base + kTableOff),
                                reinterpret_cast<uint32_t*>(base + kCountOff), 1, 0, TQ_NOALLOC_SLOTS, timeout_ns,
                                err, stream);
}

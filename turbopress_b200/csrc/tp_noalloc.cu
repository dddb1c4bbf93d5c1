// Allocation-free variant of the fused GEMV entry point.
//
// Some callers cannot allocate device memory at all: plugins that run inside
// a host engine which owns every allocation and hands out only input and
// output buffers, or decode loops where a cudaMalloc (which may synchronize
// the device) is not allowed.  For them tp_tcq_gemv_noalloc takes the same
// inputs and outputs as tp_tcq_gemv but runs on a scratch area that is part
// of this library's device image instead of a caller-provided workspace.
#include <mutex>

#include "tp_gemv_sk.cuh"

using namespace tp;

namespace {

// GEMV scratch (split-K counters, rotated activations, partial sums).  Every
// GPU that loads the library keeps these bytes until the process exits.
constexpr int64_t kNoAllocScratchBytes = int64_t(8) << 20;
static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

std::mutex g_mu;
void* g_scratch_seen[64] = {nullptr};

// Device address of the scratch array for the current device, looked up on
// every call (cheap on the host) so a reset device or another context never
// gets a stale pointer.  The host-side name g_noalloc_scratch is only a
// stand-in and must never reach a kernel.  The first time an address is seen
// the counter block (tp_gemv_sk.cuh: counters and status word, which every
// completed call leaves zero) is cleared on `stream`.
tp_status scratch_for_current_device(void** out, cudaStream_t stream) {
  int dev = 0;
  TP_CUDA_TRY(cudaGetDevice(&dev), "cudaGetDevice");
  if (dev < 0 || dev >= 64) return fail(TP_ERR_UNSUPPORTED, "device index %d out of range", dev);
  void* p = nullptr;
  TP_CUDA_TRY(cudaGetSymbolAddress(&p, g_noalloc_scratch), "cudaGetSymbolAddress(noalloc scratch)");
  std::lock_guard<std::mutex> lk(g_mu);
  if (g_scratch_seen[dev] != p) {
    TP_CUDA_TRY(cudaMemsetAsync(p, 0, kCounterBytes, stream), "cudaMemsetAsync(noalloc counters)");
    g_scratch_seen[dev] = p;
  }
  *out = p;
  return TP_OK;
}

}  // namespace

extern "C" tp_status tp_tcq_gemv_noalloc(const void* x, int x_dtype, const uint16_t* rot_scale,
                                         const uint8_t* tcq_stream, const uint16_t* scales, const uint16_t* codebook,
                                         const uint16_t* bias, void* y, int y_dtype, int64_t B, int64_t n, int64_t d,
                                         int64_t block, int bits, int n_states, void* stream) {
  if (B < 0 || n < 0 || d < 0) return fail(TP_ERR_ARG, "tp_tcq_gemv_noalloc: bad arguments");
  if (B == 0 || n == 0) return clear_ok();
  const int64_t need = tp_gemv_workspace_bytes(B, n, d, bits);
  if (need < 0) return fail(TP_ERR_UNSUPPORTED, "tp_tcq_gemv_noalloc: unsupported shape or bits");
  if (need > kNoAllocScratchBytes)
    return fail(TP_ERR_UNSUPPORTED,
                "tp_tcq_gemv_noalloc: problem needs %lld scratch bytes, above the built-in maximum of %lld "
                "(use tp_tcq_gemv with a workspace, or fewer rows in the batch)",
                (long long)need, (long long)kNoAllocScratchBytes);
  void* scratch = nullptr;
  if (tp_status s = scratch_for_current_device(&scratch, as_stream(stream))) return s;
  return tp_tcq_gemv(x, x_dtype, rot_scale, tcq_stream, scales, codebook, bias, y, y_dtype, B, n, d, block, bits,
                     n_states, scratch, kNoAllocScratchBytes, stream);
}

extern "C" tp_status tp_gemv_noalloc_status(void* stream) {
  void* scratch = nullptr;
  cudaStream_t st = as_stream(stream);
  if (tp_status s = scratch_for_current_device(&scratch, st)) return s;
  return gemv_status_at(static_cast<const unsigned char*>(scratch), st, "tp_tcq_gemv_noalloc");
}

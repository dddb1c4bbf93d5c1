// Host interface between the GEMV entry points (tp_gemv.cu, tp_noalloc.cu)
// and the stream-K GEMV kernel (tp_gemv_sk.cu).
#pragma once

#include "tp_common.cuh"

namespace tp {

// Workspace layout shared by every GEMV kernel: a fixed block of per-row-tile
// counters (zero at rest; each call leaves them zero), one status word, then
// the per-call regions (pre-rotated activations, partial sums).
constexpr int64_t kMaxRowBlocks = 16384;
constexpr int64_t kStatusOff = kMaxRowBlocks * 4;
constexpr int64_t kCounterBytes = kStatusOff + 256;

// Status bits a GEMV kernel may leave in the workspace's status word.
constexpr unsigned kStatusLayout = 1u;   // shared-memory layout check failed: outputs not written
constexpr unsigned kStatusTimeout = 2u;  // a bounded wait ran out: outputs are NaN

inline int64_t align256(int64_t v) { return (v + 255) / 256 * 256; }

int sm_count();

// Reads the status word of the workspace at `ws` (synchronizing `st`); a
// nonzero status clears the counter block and is reported as TP_ERR_DEVICE.
tp_status gemv_status_at(const unsigned char* ws, cudaStream_t st, const char* who);

// One fused rotate + decode + GEMV problem (batch <= kSkMaxBatch).
struct SkRequest {
  const void* x;
  int x_dtype;
  const uint16_t* rot_scale;
  const uint8_t* stream;
  const uint16_t* scales;
  const uint16_t* codebook;
  const uint16_t* bias;
  void* y;
  int y_dtype;
  int B;
  int64_t n, d, block;
  int bits, n_states;
  unsigned char* workspace;  // kCounterBytes + sk_workspace_extra(...) bytes, 256-byte aligned
};

constexpr int kSkMaxBatch = 8;

// Workspace bytes past the counter block, or -1 when the stream-K kernel does
// not take this problem (the caller then uses the cluster split-K kernel).
int64_t sk_workspace_extra(int64_t B, int64_t n, int64_t d, int bits, int64_t block);

tp_status sk_gemv(const SkRequest& r, cudaStream_t stream);

}  // namespace tp

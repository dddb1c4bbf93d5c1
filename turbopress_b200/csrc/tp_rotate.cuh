// Rotation kernel interface shared by tp_rotate.cu and the GEMV host code.
#pragma once

#include "tp_common.cuh"

namespace tp {

constexpr int kMaxRotateBlock = 32768;  // fp32 block in shared memory: 128 KB

struct RotateArgs {
  const void* x;
  int x_dtype;
  const uint16_t* scale;  // rot_scale (pre-scale) or post-scale, fp16 [d]
  void* z;
  int z_dtype;
  int64_t d;
  int64_t d_pad;
  int64_t block;
  int lg_block;
  int per;  // Hadamard blocks per CTA
  float norm;
  int mode;  // 0 rotate, 1 fold (post-scale), 2 permuted fp16 for the GEMV, 3 stream-K GEMV order
};

// Butterfly stages for index bits [0, lg) over s[0, count) (count a multiple
// of 2^lg).  Called by the whole CTA.
__device__ __forceinline__ void fwht_shared(float* s, int count, int lg) {
  for (int b0 = 0; b0 < lg; b0 += 3) {
    const int nb = lg - b0 < 3 ? lg - b0 : 3;
    const int G = 1 << nb;
    const int groups = count >> nb;
    for (int grp = threadIdx.x; grp < groups; grp += blockDim.x) {
      const int lo = grp & ((1 << b0) - 1);
      const int hi = grp >> b0;
      const int base = (hi << (b0 + nb)) | lo;
      float v[8];
#pragma unroll
      for (int e = 0; e < 8; ++e)
        if (e < G) v[e] = s[base + (e << b0)];
#pragma unroll
      for (int h = 1; h < 8; h <<= 1) {
        if (h >= G) break;
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          if (e < G && !(e & h)) {
            const float a = v[e], b = v[e + h];
            v[e] = a + b;
            v[e + h] = a - b;
          }
        }
      }
#pragma unroll
      for (int e = 0; e < 8; ++e)
        if (e < G) s[base + (e << b0)] = v[e];
    }
    __syncthreads();
  }
}

tp_status launch_rotate(RotateArgs a, int64_t rows, cudaStream_t stream);

}  // namespace tp

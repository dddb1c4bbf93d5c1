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
  int mode;  // 0 rotate, 1 fold (post-scale), 2 permuted fp16 for the GEMV
};

tp_status launch_rotate(RotateArgs a, int64_t rows, cudaStream_t stream);

}  // namespace tp

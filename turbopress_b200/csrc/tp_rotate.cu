// Seeded randomized Hadamard rotation of activations: z = blockFWHT(x * rs).
//
// One CTA owns a run of whole Hadamard blocks of one activation row, holds
// them in shared memory in fp32 and applies the butterfly stages in register
// groups of up to 3 index bits (8 elements per thread per group, one
// __syncthreads per group).  The Walsh-Hadamard stages commute, so the
// grouping order is free; the orthonormal 1/sqrt(block) factor is applied
// once on the way out (turbopress/runtime.py:192-208).
#include "tp_rotate.cuh"

using namespace tp;

namespace tp {

// mode 0: z = FWHT(x * scale) in z_dtype, row stride d        (tp_rotate)
// mode 1: z = fp16(FWHT(x) * scale), row stride d             (tp_fold_rows)
// mode 2: z = fp16(FWHT(x * scale)) in the permuted pair layout of the
//         native GEMV, row stride d_pad, columns [d, d_pad) zeroed
// mode 3: as mode 2 in the stream-K GEMV's order (sk_zpos)
__global__ void rotate_kernel(RotateArgs a) {
  extern __shared__ float s[];
  const int64_t row = blockIdx.y;
  const int64_t nblocks = a.d / a.block;
  const int64_t blk0 = (int64_t)blockIdx.x * a.per;
  const int64_t nb = (blk0 + a.per <= nblocks) ? a.per : nblocks - blk0;
  const int count = static_cast<int>(nb * a.block);
  const int64_t col0 = blk0 * a.block;
  for (int i = threadIdx.x; i < count; i += blockDim.x) {
    float v = load_as_float(a.x, row * a.d + col0 + i, a.x_dtype);
    if (a.mode != 1) v *= h2f_bits(a.scale[col0 + i]);
    s[i] = v;
  }
  __syncthreads();
  fwht_shared(s, count, a.lg_block);
  for (int i = threadIdx.x; i < count; i += blockDim.x) {
    float v = s[i] * a.norm;
    const int64_t c = col0 + i;
    if (a.mode == 0) {
      store_from_float(a.z, row * a.d + c, a.z_dtype, v);
    } else if (a.mode == 1) {
      v *= h2f_bits(a.scale[c]);
      reinterpret_cast<__half*>(a.z)[row * a.d + c] = __float2half_rn(v);
    } else {
      const int64_t pos = a.mode == 3 ? sk_zpos(c) : (c & ~int64_t(31)) + zperm_pos(static_cast<int>(c & 31));
      reinterpret_cast<__half*>(a.z)[row * a.d_pad + pos] = __float2half_rn(v);
    }
  }
  if (a.mode >= 2 && blockIdx.x == gridDim.x - 1) {
    for (int64_t c = a.d + threadIdx.x; c < a.d_pad; c += blockDim.x) {
      const int64_t pos = a.mode == 3 ? sk_zpos(c) : (c & ~int64_t(31)) + zperm_pos(static_cast<int>(c & 31));
      reinterpret_cast<__half*>(a.z)[row * a.d_pad + pos] = __float2half_rn(0.f);
    }
  }
}

tp_status launch_rotate(RotateArgs a, int64_t rows, cudaStream_t stream) {
  if (a.block < 1 || (a.block & (a.block - 1)) || a.d % a.block)
    return fail(TP_ERR_ARG, "block must be a power of two dividing d (d=%lld, block=%lld)", (long long)a.d,
                (long long)a.block);
  if (a.block > kMaxRotateBlock)
    return fail(TP_ERR_UNSUPPORTED, "Hadamard block %lld exceeds the supported maximum %d", (long long)a.block,
                kMaxRotateBlock);
  int lg = 0;
  while ((int64_t(1) << lg) < a.block) ++lg;
  a.lg_block = lg;
  a.norm = static_cast<float>(1.0 / __builtin_sqrt(static_cast<double>(a.block)));
  const int64_t nblocks = a.d / a.block;
  int64_t per = a.block >= 2048 ? 1 : 2048 / a.block;
  if (per > nblocks) per = nblocks;
  a.per = static_cast<int>(per);
  const int64_t count = per * a.block;
  const size_t smem = static_cast<size_t>(count) * sizeof(float);
  static int smem_set[64] = {0};
  if (tp_status s = ensure_smem(rotate_kernel, smem, smem_set, "cudaFuncSetAttribute(rotate)")) return s;
  int threads = static_cast<int>(count / 8);
  if (threads < 32) threads = 32;
  if (threads > 1024) threads = 1024;
  dim3 grid(static_cast<unsigned>((nblocks + per - 1) / per), static_cast<unsigned>(rows));
  rotate_kernel<<<grid, threads, smem, stream>>>(a);
  return check_launch("rotate_kernel");
}

}  // namespace tp

extern "C" tp_status tp_rotate(const void* x, int x_dtype, const uint16_t* rot_scale, void* z, int z_dtype,
                               int64_t B, int64_t d, int64_t block, void* stream) {
  if (!x || !rot_scale || !z || B < 0 || d < 0) return fail(TP_ERR_ARG, "tp_rotate: bad arguments");
  if (!valid_dtype(x_dtype) || !valid_dtype(z_dtype)) return fail(TP_ERR_ARG, "tp_rotate: bad dtype");
  if (B == 0 || d == 0) return clear_ok();
  if (B > 65535) return fail(TP_ERR_UNSUPPORTED, "tp_rotate: at most 65535 rows per call");
  RotateArgs a{};
  a.x = x;
  a.x_dtype = x_dtype;
  a.scale = rot_scale;
  a.z = z;
  a.z_dtype = z_dtype;
  a.d = d;
  a.d_pad = d;
  a.block = block;
  a.mode = 0;
  return launch_rotate(a, B, as_stream(stream));
}

extern "C" tp_status tp_fold_rows(const uint16_t* w_rot, const uint16_t* post_scale, uint16_t* w_out, int64_t n,
                                  int64_t d, int64_t block, void* stream) {
  if (!w_rot || !post_scale || !w_out || n < 0 || d < 0) return fail(TP_ERR_ARG, "tp_fold_rows: bad arguments");
  if (n == 0 || d == 0) return clear_ok();
  RotateArgs a{};
  a.x = w_rot;
  a.x_dtype = TP_F16;
  a.scale = post_scale;
  a.z = w_out;
  a.z_dtype = TP_F16;
  a.d = d;
  a.d_pad = d;
  a.block = block;
  a.mode = 1;
  for (int64_t r0 = 0; r0 < n; r0 += 65535) {
    const int64_t rows = n - r0 < 65535 ? n - r0 : 65535;
    RotateArgs b = a;
    b.x = w_rot + r0 * d;
    b.z = w_out + r0 * d;
    if (tp_status s = launch_rotate(b, rows, as_stream(stream))) return s;
  }
  return clear_ok();
}

// Greedy LM head: fp16 GEMV over the vocabulary fused with argmax.
//
// The reference's decode loops pick the next token as
// `logits[:, -1:].argmax(-1)` after the tied fp16 lm_head F.linear
// (scripts/run_packed.py:164,178,190; scripts/graph_decode_bench.py:55-112).
// Here one kernel streams the weight matrix once (HBM-bound: V*h*2 bytes),
// keeps the running argmax in registers and never needs the logits in HBM
// (they are written only when the caller asks for them).
//
// Layout: W row-major fp16 [V][h] (16-byte aligned, h % 8 == 0), x fp16
// [B][h].  Each warp owns R consecutive rows per iteration and walks their
// columns 256 at a time (one 16-byte load per lane per row), with U column
// chunks in flight, so every lane has R*U independent 16-byte loads
// outstanding.  x is converted to fp32 once per CTA into shared memory.
// Products accumulate in fp32; sums are reduced across the warp by
// shuffles.  The argmax key of a logit is its order-preserving 32-bit image
// in the high word and (0xFFFFFFFF - index) in the low word, so a 64-bit
// atomicMax selects the largest logit and, among equal logits, the first
// index (torch.argmax's rule; a NaN logit maps above +inf and wins, as there).
// The last CTA to finish (counter in the workspace) turns the keys into
// (index, value) and leaves the workspace zeroed for the next call.
#include <algorithm>

#include "tp_common.cuh"

using namespace tp;

namespace {

constexpr int kLhThreads = 256;
constexpr int kLhWarps = kLhThreads / 32;
constexpr int kLhMaxB = 8;
constexpr int64_t kLhMaxSmem = 100 * 1024;  // fp32 copy of x; two CTAs per SM

__device__ __forceinline__ uint4 ld_stream16(const uint16_t* p) {
  uint4 v;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p));
  return v;
}

// The reference's logits are fp16 (F.linear in fp16, then argmax): the key
// ranks the fp16-rounded logit, so values that round together tie and the
// first index wins.  Like torch.argmax, a NaN ranks above everything and -0
// equals +0.
__device__ __forceinline__ unsigned long long argmax_key(float v, unsigned idx) {
  float r = __half2float(__float2half_rn(v));
  unsigned u;
  if (r != r) {
    u = 0xFFFFFFFFu;
  } else {
    if (r == 0.f) r = 0.f;
    u = __float_as_uint(r);
    u = (u & 0x80000000u) ? ~u : (u | 0x80000000u);
  }
  return (static_cast<unsigned long long>(u) << 32) | (0xFFFFFFFFu - idx);
}

__device__ __forceinline__ float key_value(unsigned long long k) {
  unsigned u = static_cast<unsigned>(k >> 32);
  u = (u & 0x80000000u) ? (u & 0x7FFFFFFFu) : ~u;
  return __uint_as_float(u);
}

__device__ __forceinline__ void fma8(float& acc, uint4 w, const float4& xa, const float4& xb) {
  const float2 w0 = __half22float2(*reinterpret_cast<const __half2*>(&w.x));
  const float2 w1 = __half22float2(*reinterpret_cast<const __half2*>(&w.y));
  const float2 w2 = __half22float2(*reinterpret_cast<const __half2*>(&w.z));
  const float2 w3 = __half22float2(*reinterpret_cast<const __half2*>(&w.w));
  acc = fmaf(w0.x, xa.x, acc);
  acc = fmaf(w0.y, xa.y, acc);
  acc = fmaf(w1.x, xa.z, acc);
  acc = fmaf(w1.y, xa.w, acc);
  acc = fmaf(w2.x, xb.x, acc);
  acc = fmaf(w2.y, xb.y, acc);
  acc = fmaf(w3.x, xb.z, acc);
  acc = fmaf(w3.y, xb.w, acc);
}

struct LhWorkspace {
  unsigned long long key[kLhMaxB];
  unsigned done;
};

template <int B, int R, int U>
__global__ void __launch_bounds__(kLhThreads, 2)
    lm_head_kernel(const uint16_t* __restrict__ x, const uint16_t* __restrict__ w, int V, int h,
                   float* __restrict__ logits, int64_t* __restrict__ idx_out, float* __restrict__ val_out,
                   LhWorkspace* __restrict__ ws) {
  extern __shared__ __align__(16) float xs[];  // [B][h]
  __shared__ unsigned long long s_best[kLhWarps][B];
  __shared__ bool s_last;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  for (int i = threadIdx.x; i < B * h / 2; i += kLhThreads) {
    const float2 f = __half22float2(reinterpret_cast<const __half2*>(x)[i]);
    xs[2 * i] = f.x;
    xs[2 * i + 1] = f.y;
  }
  __syncthreads();

  unsigned long long best[B];
#pragma unroll
  for (int b = 0; b < B; ++b) best[b] = 0ull;

  const int stride = gridDim.x * kLhWarps * R;
  for (int row0 = (blockIdx.x * kLhWarps + warp) * R; row0 < V; row0 += stride) {
    float acc[R][B];
#pragma unroll
    for (int r = 0; r < R; ++r)
#pragma unroll
      for (int b = 0; b < B; ++b) acc[r][b] = 0.f;
    const uint16_t* wrow[R];
#pragma unroll
    for (int r = 0; r < R; ++r) wrow[r] = w + (size_t)min(row0 + r, V - 1) * h;  // rows past V: a valid row, dropped
    for (int c0 = lane * 8; c0 < h; c0 += 256 * U) {
      uint4 wv[U][R];
#pragma unroll
      for (int u = 0; u < U; ++u)
#pragma unroll
        for (int r = 0; r < R; ++r)
          wv[u][r] = c0 + u * 256 < h ? ld_stream16(wrow[r] + c0 + u * 256) : make_uint4(0u, 0u, 0u, 0u);
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const int c = c0 + u * 256;
        if (c < h) {
#pragma unroll
          for (int b = 0; b < B; ++b) {
            const float4 xa = *reinterpret_cast<const float4*>(xs + b * h + c);
            const float4 xb = *reinterpret_cast<const float4*>(xs + b * h + c + 4);
#pragma unroll
            for (int r = 0; r < R; ++r) fma8(acc[r][b], wv[u][r], xa, xb);
          }
        }
      }
    }
#pragma unroll
    for (int r = 0; r < R; ++r)
#pragma unroll
      for (int b = 0; b < B; ++b) {
        float s = acc[r][b];
#pragma unroll
        for (int m = 16; m >= 1; m >>= 1) s += __shfl_xor_sync(0xffffffffu, s, m);
        const int row = row0 + r;
        if (row < V) {
          const unsigned long long k = argmax_key(s, static_cast<unsigned>(row));
          best[b] = k > best[b] ? k : best[b];
          if (logits && lane == ((r * B + b) & 31)) logits[(size_t)b * V + row] = s;
        }
      }
  }
  if (lane == 0)
#pragma unroll
    for (int b = 0; b < B; ++b) s_best[warp][b] = best[b];
  __syncthreads();
  if (threadIdx.x < B) {
    unsigned long long k = s_best[0][threadIdx.x];
    for (int i = 1; i < kLhWarps; ++i) k = s_best[i][threadIdx.x] > k ? s_best[i][threadIdx.x] : k;
    atomicMax(&ws->key[threadIdx.x], k);
  }
  __threadfence();
  __syncthreads();
  if (threadIdx.x == 0) s_last = atomicAdd(&ws->done, 1u) == gridDim.x - 1;
  __syncthreads();
  if (s_last && threadIdx.x < B) {
    __threadfence();
    const unsigned long long k = atomicExch(&ws->key[threadIdx.x], 0ull);
    idx_out[threadIdx.x] = static_cast<int64_t>(0xFFFFFFFFu - static_cast<unsigned>(k & 0xFFFFFFFFull));
    if (val_out) val_out[threadIdx.x] = key_value(k);
    if (threadIdx.x == 0) ws->done = 0u;
  }
}

__device__ __forceinline__ void mma_f16_16816(float* c, uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                              uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// Batches 2..8: the batch is the n=8 side of m16n8k16 MMAs (fp32
// accumulate).  A warp owns 16 rows per iteration; lane (g = lane/4,
// t = lane%4) loads 16 bytes of rows g and g+8 at columns c + 8t.. of each
// 32-column chunk, and since a dot product may visit K in any order shared
// by both operands, those eight columns are the lane's A-fragment K slots of
// two MMAs (columns 8t+0..3 the first, 8t+4..7 the second); the matching B
// fragments are one 16-byte load of x row g (zero for g >= B).  No cross-lane
// reduction: lane (g, t) ends with rows g, g+8 of batch rows 2t, 2t+1.
template <int B, int U>
__global__ void __launch_bounds__(kLhThreads, 2)
    lm_head_mma_kernel(const uint16_t* __restrict__ x, const uint16_t* __restrict__ w, int V, int h,
                       float* __restrict__ logits, int64_t* __restrict__ idx_out, float* __restrict__ val_out,
                       LhWorkspace* __restrict__ ws) {
  extern __shared__ __align__(16) uint16_t xh[];  // [B][h] fp16
  __shared__ unsigned long long s_best[kLhWarps][8];
  __shared__ bool s_last;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
  for (int i = threadIdx.x; i < B * h / 8; i += kLhThreads)
    reinterpret_cast<uint4*>(xh)[i] = reinterpret_cast<const uint4*>(x)[i];
  __syncthreads();

  unsigned long long best0 = 0ull, best1 = 0ull;  // batch rows 2t, 2t+1
  const uint16_t* xrow = xh + (size_t)(g < B ? g : 0) * h;
  const int stride = gridDim.x * kLhWarps * 16;
  for (int row0 = (blockIdx.x * kLhWarps + warp) * 16; row0 < V; row0 += stride) {
    float c1[4] = {0.f, 0.f, 0.f, 0.f}, c2[4] = {0.f, 0.f, 0.f, 0.f};
    const uint16_t* wg = w + (size_t)min(row0 + g, V - 1) * h;
    const uint16_t* wq = w + (size_t)min(row0 + g + 8, V - 1) * h;
    // the trip count must be the same in every lane: mma.sync is a
    // warp-collective (.aligned) instruction
    for (int cb = 0; cb < h; cb += 32 * U) {
      const int c0 = cb + 8 * t;
      uint4 ag[U], aq[U];
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const int c = c0 + 32 * u;
        ag[u] = c < h ? ld_stream16(wg + c) : make_uint4(0u, 0u, 0u, 0u);
        aq[u] = c < h ? ld_stream16(wq + c) : make_uint4(0u, 0u, 0u, 0u);
      }
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const int c = c0 + 32 * u;
        const uint4 xb = (g < B && c < h) ? *reinterpret_cast<const uint4*>(xrow + c) : make_uint4(0u, 0u, 0u, 0u);
        mma_f16_16816(c1, ag[u].x, aq[u].x, ag[u].y, aq[u].y, xb.x, xb.y);
        mma_f16_16816(c2, ag[u].z, aq[u].z, ag[u].w, aq[u].w, xb.z, xb.w);
      }
    }
    // c[0], c[1]: row g, batch 2t, 2t+1; c[2], c[3]: row g + 8
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const int row = row0 + g + (e >= 2 ? 8 : 0), bn = 2 * t + (e & 1);
      const float v = c1[e] + c2[e];
      if (row < V && bn < B) {
        const unsigned long long k = argmax_key(v, static_cast<unsigned>(row));
        if (e & 1) best1 = k > best1 ? k : best1;
        else best0 = k > best0 ? k : best0;
        if (logits) logits[(size_t)bn * V + row] = v;
      }
    }
  }
  // lanes with the same t hold the same batch rows: reduce over g
#pragma unroll
  for (int m = 4; m < 32; m <<= 1) {
    const unsigned long long o0 = __shfl_xor_sync(0xffffffffu, best0, m);
    const unsigned long long o1 = __shfl_xor_sync(0xffffffffu, best1, m);
    best0 = o0 > best0 ? o0 : best0;
    best1 = o1 > best1 ? o1 : best1;
  }
  if (lane < 4) {
    s_best[warp][2 * lane] = best0;
    s_best[warp][2 * lane + 1] = best1;
  }
  __syncthreads();
  if (threadIdx.x < B) {
    unsigned long long k = s_best[0][threadIdx.x];
    for (int i = 1; i < kLhWarps; ++i) k = s_best[i][threadIdx.x] > k ? s_best[i][threadIdx.x] : k;
    atomicMax(&ws->key[threadIdx.x], k);
  }
  __threadfence();
  __syncthreads();
  if (threadIdx.x == 0) s_last = atomicAdd(&ws->done, 1u) == gridDim.x - 1;
  __syncthreads();
  if (s_last && threadIdx.x < B) {
    __threadfence();
    const unsigned long long k = atomicExch(&ws->key[threadIdx.x], 0ull);
    idx_out[threadIdx.x] = static_cast<int64_t>(0xFFFFFFFFu - static_cast<unsigned>(k & 0xFFFFFFFFull));
    if (val_out) val_out[threadIdx.x] = key_value(k);
    if (threadIdx.x == 0) ws->done = 0u;
  }
}

template <int B>
tp_status launch_lm_head_mma(const uint16_t* x, const uint16_t* w, int V, int h, float* logits, int64_t* idx,
                             float* val, LhWorkspace* ws, cudaStream_t st) {
  auto kern = lm_head_mma_kernel<B, 4>;
  const int smem = B * h * 2;
  static int smem_set[64];
  // the default dynamic limit is 48 KB minus the kernel's static shared
  // memory, so raise it from 47 KB of dynamic shared memory on
  const tp_status s = ensure_smem(kern, smem > 47 * 1024 ? smem + 1024 : smem, smem_set,
                                  "lm_head: shared memory attribute");
  if (s != TP_OK) return s;
  int dev = 0, sms = 0;
  TP_CUDA_TRY(cudaGetDevice(&dev), "lm_head: device");
  TP_CUDA_TRY(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev), "lm_head: SM count");
  const int64_t need = ((int64_t)V + kLhWarps * 16 - 1) / (kLhWarps * 16);
  const int grid = static_cast<int>(std::min<int64_t>(need, 2 * sms));
  kern<<<grid, kLhThreads, smem, st>>>(x, w, V, h, logits, idx, val, ws);
  return check_launch("lm_head launch");
}

template <int B>
tp_status launch_lm_head(const uint16_t* x, const uint16_t* w, int V, int h, float* logits, int64_t* idx,
                         float* val, LhWorkspace* ws, cudaStream_t st) {
  // R rows x U chunks of 16-byte loads in flight per lane: 8 at small
  // batches, 4 rows x 1 chunk at large ones (accumulator registers)
  constexpr int R = B <= 2 ? 4 : (B <= 4 ? 4 : 2);
  constexpr int U = B <= 2 ? 2 : 1;
  auto kern = lm_head_kernel<B, R, U>;
  const int smem = B * h * 4;
  static int smem_set[64];  // per device: dynamic shared memory limit already raised to
  // the default dynamic limit is 48 KB minus the kernel's static shared
  // memory, so raise it from 47 KB of dynamic shared memory on
  const tp_status s = ensure_smem(kern, smem > 47 * 1024 ? smem + 1024 : smem, smem_set,
                                  "lm_head: shared memory attribute");
  if (s != TP_OK) return s;
  int dev = 0, sms = 0;
  TP_CUDA_TRY(cudaGetDevice(&dev), "lm_head: device");
  TP_CUDA_TRY(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev), "lm_head: SM count");
  const int64_t need = ((int64_t)V + kLhWarps * R - 1) / (kLhWarps * R);
  const int grid = static_cast<int>(std::min<int64_t>(need, 2 * sms));
  kern<<<grid, kLhThreads, smem, st>>>(x, w, V, h, logits, idx, val, ws);
  return check_launch("lm_head launch");
}

}  // namespace

extern "C" {

TP_API int64_t tp_lm_head_workspace_bytes(int64_t B) {
  (void)B;
  return (int64_t)((sizeof(LhWorkspace) + 127) / 128 * 128);
}

TP_API tp_status tp_lm_head_argmax(const uint16_t* x, const uint16_t* w, int64_t B, int64_t V, int64_t h,
                                   float* logits, int64_t* idx, float* val, void* workspace,
                                   int64_t workspace_bytes, void* stream) {
  if (!x || !w || !idx) return fail(TP_ERR_ARG, "tp_lm_head_argmax: null pointer");
  if (B < 1 || B > kLhMaxB) return fail(TP_ERR_UNSUPPORTED, "tp_lm_head_argmax: batch %lld not in 1..8", (long long)B);
  if (V < 1 || V > 0x7FFFFFFF || h < 8 || h % 8)
    return fail(TP_ERR_ARG, "tp_lm_head_argmax: need 1 <= V < 2^31 and h a positive multiple of 8");
  if (B * h * 4 > kLhMaxSmem)
    return fail(TP_ERR_UNSUPPORTED, "tp_lm_head_argmax: B*h = %lld exceeds %lld", (long long)(B * h),
                (long long)(kLhMaxSmem / 4));
  if (reinterpret_cast<uintptr_t>(x) % 16 || reinterpret_cast<uintptr_t>(w) % 16)
    return fail(TP_ERR_ALIGN, "tp_lm_head_argmax: x and w must be 16-byte aligned");
  if (!workspace || workspace_bytes < tp_lm_head_workspace_bytes(B) || reinterpret_cast<uintptr_t>(workspace) % 8)
    return fail(TP_ERR_WORKSPACE, "tp_lm_head_argmax: workspace missing, unaligned or smaller than %lld bytes",
                (long long)tp_lm_head_workspace_bytes(B));
  auto* ws = static_cast<LhWorkspace*>(workspace);
  auto st = static_cast<cudaStream_t>(stream);
  const int Vi = static_cast<int>(V), hi = static_cast<int>(h);
  switch (B) {
    case 1: return launch_lm_head<1>(x, w, Vi, hi, logits, idx, val, ws, st);
    case 2: return launch_lm_head_mma<2>(x, w, Vi, hi, logits, idx, val, ws, st);
    case 3: return launch_lm_head_mma<3>(x, w, Vi, hi, logits, idx, val, ws, st);
    case 4: return launch_lm_head_mma<4>(x, w, Vi, hi, logits, idx, val, ws, st);
    case 5: return launch_lm_head_mma<5>(x, w, Vi, hi, logits, idx, val, ws, st);
    case 6: return launch_lm_head_mma<6>(x, w, Vi, hi, logits, idx, val, ws, st);
    case 7: return launch_lm_head_mma<7>(x, w, Vi, hi, logits, idx, val, ws, st);
    default: return launch_lm_head_mma<8>(x, w, Vi, hi, logits, idx, val, ws, st);
  }
}

}  // extern "C"

// Skinny GEMM (batch 16..64 per launch) on the 5th-generation tensor cores:
// decode packed TCQ weights into shared memory, tcgen05.mma into TMEM.
//
// y[B, n] = z[B, d] @ W^T with z = blockFWHT(x * rot_scale) (rotated first by
// rotate_kernel into the permuted fp16 layout the native decoder uses) and W
// the fp16 dequant of the native stream (scale applied in the epilogue).
//
// CTA = 128 output rows (8 row tiles, one decode warp each) x a K range of
// whole units (split-K over CTAs, fp32 atomics into a workspace).  Per half
// unit (128 columns) the decode warps write the weight pairs straight into a
// K-major UMMA operand (no-swizzle canonical layout: 8-row x 16-byte core
// matrices, K in the same permuted order as z), the activations are copied in
// with cp.async, and one thread issues 8 tcgen05.mma (M=128, N=B, K=16)
// accumulating in TMEM; two half-unit buffers alternate, a tcgen05.commit
// per step releases its buffer.  Epilogue: tcgen05.ld rows -> scale -> add.
#include "tp_decode.cuh"
#include "tp_rotate.cuh"

using namespace tp;

namespace {

constexpr int kUWarps = 8;               // decode warps (one row tile each)
constexpr int kUDecThreads = kUWarps * 32;
constexpr int kUThreads = kUDecThreads + 32;  // + one MMA-issue warp
constexpr int kUMaxN = 64;               // batch rows per launch (32 for 4-bit weights)
constexpr uint32_t kATile = 128 * 128 * 2;   // one half unit of A: 32 KB
constexpr uint32_t kCoreK = 128;             // bytes between K-adjacent core matrices
constexpr uint32_t kCoreRows = 16 * 128;     // bytes between 8-row groups (16 core columns)

// weight units in flight per decode warp (bulk-copy ring); 4-bit weights use
// register prefetch (their 128 KB pair table leaves no room for a ring)
template <int BITS>
struct UDepth {
  static constexpr int kDepth = BITS <= 3 ? 4 : 0;
};

struct UArgs {
  const uint4* stream;
  const uint16_t* scales;
  const uint16_t* codebook;
  const __half* z;     // [NB][d_pad] permuted fp16 (rows >= B zero)
  float* y32;          // [B][n] fp32, zero before the launch
  int B, NB, n, d_pad, units_k, row_tiles, ksplit;
  uint32_t lut_off, a_off, b_off, w_off, bar_off, smem;
};

#ifndef TP_UMMA_SW128
#define TP_UMMA_SW128 1
#endif
// Operand tiles (rows x 128 K halves, K-major).  Byte offset of 16-byte
// chunk kc (0..15) of `row` in a tile of `rows` rows:
//  no swizzle : 8-row x 16-byte core matrices, K-adjacent ones 128 B apart,
//               8-row groups 2048 B apart;
//  128B swizzle: two 64-element K halves of `rows` x 128 B each; inside a
//               row the chunk index is XORed with row % 8 (the hardware's
//               128-byte swizzle; measured 5-13 % faster than no swizzle).
__device__ __forceinline__ uint32_t opnd_off(int row, int kc, int rows) {
  if (TP_UMMA_SW128)
    return (uint32_t)((kc >> 3) * rows * 128 + row * 128 + (((kc & 7) ^ (row & 7)) << 4));
  return (uint32_t)((row >> 3) * kCoreRows + kc * kCoreK + (row & 7) * 16);
}
// descriptor of MMA k-step s (16 K elements) of a tile at `base` with `rows` rows
__device__ __forceinline__ uint64_t umma_desc(uint32_t base, int s, int rows) {
  // start >> 4 | LBO >> 4 << 16 | SBO >> 4 << 32 | version 1 << 46 | layout << 61
  if (TP_UMMA_SW128) {
    const uint32_t a = base + (uint32_t)((s >> 2) * rows * 128 + (s & 3) * 32);
    return (uint64_t)((a >> 4) & 0x3FFFu) | (1ull << 16) | ((uint64_t)(1024 >> 4) << 32) | (1ull << 46) |
           (2ull << 61);
  }
  const uint32_t a = base + (uint32_t)s * 2 * kCoreK;
  return (uint64_t)((a >> 4) & 0x3FFFu) | ((uint64_t)(kCoreK >> 4) << 16) | ((uint64_t)(kCoreRows >> 4) << 32) |
         (1ull << 46);
}

__device__ __forceinline__ void umma_f16(uint32_t tmem_d, uint64_t a, uint64_t b, uint32_t idesc, uint32_t acc) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, {%5, %6, %7, %8}, p;\n}" ::"r"(tmem_d),
      "l"(a), "l"(b), "r"(idesc), "r"(acc), "r"(0u), "r"(0u), "r"(0u), "r"(0u)  // no output lanes disabled
      : "memory");
}

__device__ __forceinline__ void umma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}

// one half unit (cgi) of one row tile -> A operand rows [16*rt_local, +16)
template <int BITS, int S>
__device__ __forceinline__ void decode_half_store(const unsigned char* lut, uint32_t lanew, uint32_t Pg, uint32_t Hg,
                                                  uint32_t Pq, uint32_t Hq, uint32_t Mg0, uint32_t Mg1,
                                                  uint32_t Mg2, uint32_t Mq0, uint32_t Mq1, uint32_t Mq2,
                                                  unsigned char* A, int rg, int t) {
  uint32_t Lg[4], Lq[4];
  {
    uint32_t A, Bm, Cw, Dm;
    member_words<BITS>(Mg0, Mg1, A, Bm, Cw, Dm);
    level_words<S>(Pg, Hg, A, Bm, Cw, Dm, Lg);
    member_words<BITS>(Mq0, Mq1, A, Bm, Cw, Dm);
    level_words<S>(Pq, Hq, A, Bm, Cw, Dm, Lq);
  }
  uint32_t r[4][2][4];  // [w][row g / g+8][a0 q0, a2 q0, a0 q1, a2 q1]
#pragma unroll
  for (int w = 0; w < 4; ++w) {
#pragma unroll
    for (int q = 0; q < 2; ++q) {
      if (BITS <= 3) {
        const uint32_t s0 = 0x5504u | ((2u * q) << 4), s1 = 0x5504u | ((2u * q + 1u) << 4);
        r[w][0][2 * q] = lds32(lut, prmt(Lg[w], lanew, s0));
        r[w][0][2 * q + 1] = lds32(lut, prmt(Lg[w], lanew, s1));
        r[w][1][2 * q] = lds32(lut, prmt(Lq[w], lanew, s0));
        r[w][1][2 * q + 1] = lds32(lut, prmt(Lq[w], lanew, s1));
      } else {
        const uint32_t xg = x4(Mg2, w, q, lanew), xq = x4(Mq2, w, q, lanew);
        const uint32_t s0 = 0xD504u | ((2u * q) << 4), s1 = 0xF706u | ((2u * q + 1u) << 4);
        r[w][0][2 * q] = lds32(lut, prmt(Lg[w], xg, s0));
        r[w][0][2 * q + 1] = lds32(lut, prmt(Lg[w], xg, s1));
        r[w][1][2 * q] = lds32(lut, prmt(Lq[w], xq, s0));
        r[w][1][2 * q + 1] = lds32(lut, prmt(Lq[w], xq, s1));
      }
    }
  }
  // K chunk (8 halves) t*4 + w of this half unit is operand chunk t*4 + w
#pragma unroll
  for (int w = 0; w < 4; ++w) {
    const int kc = t * 4 + w;
    *reinterpret_cast<uint4*>(A + opnd_off(rg, kc, 128)) = make_uint4(r[w][0][0], r[w][0][1], r[w][0][2], r[w][0][3]);
    *reinterpret_cast<uint4*>(A + opnd_off(rg + 8, kc, 128)) =
        make_uint4(r[w][1][0], r[w][1][1], r[w][1][2], r[w][1][3]);
  }
}

template <int BITS, int S>
__global__ void __launch_bounds__(kUThreads, 1) tcq_umma_kernel(UArgs a) {
  extern __shared__ __align__(1024) unsigned char smem[];
  __shared__ uint32_t s_tmem;
  __shared__ int s_bad;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int g = lane >> 2, t = lane & 3;
  unsigned char* lut = smem + a.lut_off;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + a.bar_off);  // [2] MMA done per buffer, [2] final
  const int mt = blockIdx.x, ks = blockIdx.y;
  const int u0 = (int)((int64_t)ks * a.units_k / a.ksplit), u1 = (int)((int64_t)(ks + 1) * a.units_k / a.ksplit);
  const int rt = mt * 8 + warp;  // this warp's row tile
  const bool have_rows = rt < a.row_tiles;
  const uint32_t ncols = a.NB <= 32 ? 32u : 64u;

  constexpr int D = UDepth<BITS>::kDepth;
  constexpr unsigned kUB = 512u * BITS;  // bytes of one unit
  // bars: [0,2) A buffer free (tcgen05.commit), [2,4) A buffer ready (every
  // decode thread arrives), then the weight-ring slots [kUWarps][D]
  uint64_t* fullb = bars + 4;
  if (tid == 0) {
    s_bad = 0;
    mbar_init(&bars[0], 1);
    mbar_init(&bars[1], 1);
    mbar_init(&bars[2], kUDecThreads);
    mbar_init(&bars[3], kUDecThreads);
  }
  if (D > 0 && tid < kUWarps * D) mbar_init(&fullb[tid], 1);
  fence_mbar_init();
  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&s_tmem)),
                 "r"(ncols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  const uint32_t cbv = lane < (1 << (BITS + 1)) ? a.codebook[lane] : 0u;
  build_lut<BITS>(lut, cbv, warp, lane, kUWarps + 1);
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  const uint32_t tmem = s_tmem;
  const uint32_t lanew = BITS <= 3 ? (uint32_t)lane * 4u : (uint32_t)lane * 4u * 0x10001u;
  const int src = (lane & ~3) | ((t + 3) & 3);
  const uint32_t idesc = (1u << 4) | ((uint32_t)(a.NB >> 3) << 17) | ((128u >> 4) << 24);

  const int steps = 2 * (u1 - u0);
  const uint32_t btile = (uint32_t)(a.NB * 256);
  unsigned char* wring = smem + a.w_off + (uint32_t)(warp < kUWarps ? warp : 0) * (D > 0 ? D : 1) * kUB;
  const uint4* wsrc = a.stream + ((int64_t)rt * a.units_k) * 32 * BITS;  // unit u at wsrc + u * 32 * BITS
  if (D > 0) {
    __syncthreads();  // ring barriers initialised
    if (warp < kUWarps && have_rows && lane == 0)
      for (int i = 0; i < D && u0 + i < u1; ++i)
        bulk_load(wring + i * kUB, wsrc + (int64_t)(u0 + i) * 32 * BITS, kUB, &fullb[warp * D + i]);
  }
  if (warp < kUWarps) {
    // ===================== decode warps =====================
    // activations of step h (rows b < NB, the 16 core columns of its half
    // unit) into activation buffer h % 3, one cp.async group per step
    auto copy_z = [&](int h) {
      const int u = u0 + (h >> 1), cgi = h & 1;
      unsigned char* Bt = smem + a.b_off + (uint32_t)(h % 3) * btile;
      for (int i = tid; i < a.NB * 16; i += kUDecThreads) {
        const int b = i >> 4, kc = i & 15;
        const __half* srcp = a.z + (size_t)b * a.d_pad + (size_t)(u * 32 + cgi * 16 + kc) * 8;
        asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(Bt + opnd_off(b, kc, a.NB))),
                     "l"(srcp)
                     : "memory");
      }
      asm volatile("cp.async.commit_group;" ::: "memory");
    };
    // halo for the first unit of the range (from the previous unit of the row tile)
    uint32_t prevg = 0u, prevq = 0u;
    if (have_rows && u0 > 0) {
      const uint4 pv = ldg_stream(wsrc + ((int64_t)(u0 - 1) * 32 + lane) * BITS);
      prevg = pv.z;
      prevq = pv.w;
    }
    uint4 cur[BITS], nxt[BITS];
    if (D == 0 && have_rows && u0 < u1) {
#pragma unroll
      for (int k = 0; k < BITS; ++k) cur[k] = ldg_stream(wsrc + ((int64_t)u0 * 32 + lane) * BITS + k);
    }
    if (steps > 0) copy_z(0);
    for (int h = 0; h < steps; ++h) {
      const int buf = h & 1, u = u0 + (h >> 1), cgi = h & 1;
      unsigned char* A = smem + a.a_off + buf * kATile;
      // A buffer h % 2 and activation buffer (h + 1) % 3 == (h - 2) % 3 are
      // free once the MMAs of step h - 2 completed
      if (h >= 2 && !mbar_wait(&bars[buf], (unsigned)(((h - 2) >> 1) & 1))) s_bad = 1;
      if (h + 1 < steps) copy_z(h + 1);  // in flight while this step decodes
      if (have_rows) {
        if (D > 0 && cgi == 0) {
          // this unit from its ring slot; refill the slot with unit u + D
          const int i = u - u0, slot = i % (D > 0 ? D : 1);
          if (!mbar_wait(&fullb[warp * D + slot], (unsigned)((i / (D > 0 ? D : 1)) & 1))) s_bad = 1;
          const uint4* su = reinterpret_cast<const uint4*>(wring + slot * kUB) + lane * BITS;
#pragma unroll
          for (int k = 0; k < BITS; ++k) cur[k] = su[k];
          __syncwarp();
          if (lane == 0 && u + D < u1) {
            fence_proxy_async();
            bulk_load(wring + slot * kUB, wsrc + (int64_t)(u + D) * 32 * BITS, kUB, &fullb[warp * D + slot]);
          }
        } else if (D == 0 && cgi == 0 && u + 1 < u1) {  // prefetch the next unit of this row tile
#pragma unroll
          for (int k = 0; k < BITS; ++k) nxt[k] = ldg_stream(wsrc + ((int64_t)(u + 1) * 32 + lane) * BITS + k);
        }
        const uint32_t P0g = cur[0].x, P0q = cur[0].y, P1g = cur[0].z, P1q = cur[0].w;
        const uint32_t Pg = cgi ? P1g : P0g, Pq = cgi ? P1q : P0q;
        const uint32_t Hg = __shfl_sync(0xffffffffu, t == 3 ? (cgi ? P0g : prevg) : Pg, src);
        const uint32_t Hq = __shfl_sync(0xffffffffu, t == 3 ? (cgi ? P0q : prevq) : Pq, src);
        uint32_t Mg0 = 0u, Mq0 = 0u, Mg1 = 0u, Mq1 = 0u, Mg2 = 0u, Mq2 = 0u;
        if (BITS >= 2) {
          Mg0 = cgi ? cur[1].z : cur[1].x;
          Mq0 = cgi ? cur[1].w : cur[1].y;
        }
        if (BITS >= 3) {
          Mg1 = cgi ? cur[2].z : cur[2].x;
          Mq1 = cgi ? cur[2].w : cur[2].y;
        }
        if (BITS >= 4) {
          Mg2 = cgi ? cur[3].z : cur[3].x;
          Mq2 = cgi ? cur[3].w : cur[3].y;
        }
        const int rg = warp * 16 + g;  // A rows of this lane: rg and rg + 8
        decode_half_store<BITS, S>(lut, lanew, Pg, Hg, Pq, Hq, Mg0, Mg1, Mg2, Mq0, Mq1, Mq2, A, rg, t);
        if (cgi == 1) {
          prevg = P1g;
          prevq = P1q;
          if (D == 0 && u + 1 < u1) {
#pragma unroll
            for (int k = 0; k < BITS; ++k) cur[k] = nxt[k];
          }
        }
      }
      // this step's activations landed (the next step's group may still be in flight)
      if (h + 1 < steps) asm volatile("cp.async.wait_group 1;" ::: "memory");
      else asm volatile("cp.async.wait_group 0;" ::: "memory");
      fence_proxy_async();  // generic-proxy writes of A and B -> visible to the tensor core
      mbar_arrive(&bars[2 + buf]);
    }
  } else if (lane == 0) {
    // ===================== MMA warp =====================
    for (int h = 0; h < steps; ++h) {
      const int buf = h & 1;
      if (!mbar_wait(&bars[2 + buf], (unsigned)((h >> 1) & 1))) {
        s_bad = 1;
        break;
      }
      asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
      const uint32_t a0 = smem_u32(smem + a.a_off + buf * kATile);
      const uint32_t b0 = smem_u32(smem + a.b_off + (uint32_t)(h % 3) * btile);
#pragma unroll
      for (int s = 0; s < 8; ++s)  // K = 16 per MMA: two core columns
        umma_f16(tmem, umma_desc(a0, s, 128), umma_desc(b0, s, a.NB), idesc,
                 (h > 0 || s > 0) ? 1u : 0u);
      umma_commit(&bars[buf]);
    }
  }
  // all MMAs done: the last commit of each buffer
  if (steps > 0) {
    const int hl = steps - 1;
    if (!mbar_wait(&bars[hl & 1], (unsigned)((hl >> 1) & 1))) s_bad = 1;
    if (steps > 1 && !mbar_wait(&bars[(hl - 1) & 1], (unsigned)(((hl - 1) >> 1) & 1))) s_bad = 1;
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();  // s_bad final and the same in every thread (tcgen05.ld below is warp-aligned)
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  const bool bad = s_bad != 0;
  // epilogue: warps 0..3 read TMEM lanes 32w.. (output rows), NB fp32 columns
  if (warp < 4 && steps > 0 && !bad) {
    const int row = mt * 128 + warp * 32 + lane;
    const uint32_t taddr = tmem + ((uint32_t)(warp * 32) << 16);
    const float sc = row < a.n ? h2f_bits(a.scales[row]) : 0.f;
    for (int c0 = 0; c0 < a.NB; c0 += 16) {
      uint32_t v[16];
      asm volatile(
          "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
          : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]),
            "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15])
          : "r"(taddr + (uint32_t)c0));
      asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
      if (row < a.n)
#pragma unroll
        for (int j = 0; j < 16; ++j)
          if (c0 + j < a.B) atomicAdd(a.y32 + (int64_t)(c0 + j) * a.n + row, __uint_as_float(v[j]) * sc);
    }
  }
  if (bad && tid == 0) {
    // a bounded wait gave up: poison this CTA's rows so the failure is visible
    for (int b = 0; b < a.B; ++b)
      for (int r = 0; r < 128 && mt * 128 + r < a.n; ++r) a.y32[(int64_t)b * a.n + mt * 128 + r] = __int_as_float(0x7fc00000);
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  if (warp == 0) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(ncols) : "memory");
  }
}

// y (dtype) = y32 (+ bias)
__global__ void finish_kernel(const float* y32, const uint16_t* bias, void* y, int y_dtype, int B, int n) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= (int64_t)B * n) return;
  float v = y32[i];
  if (bias) v += h2f_bits(bias[i % n]);
  store_from_float(y, i, y_dtype, v);
}

template <int BITS, int S>
tp_status launch_umma_t(const UArgs& a, int m_tiles, cudaStream_t st) {
  auto kern = tcq_umma_kernel<BITS, S>;
  static int smem_set[64] = {0};
  if (tp_status s = ensure_smem(kern, a.smem, smem_set, "cudaFuncSetAttribute(umma)")) return s;
  dim3 grid((unsigned)m_tiles, (unsigned)a.ksplit);
  kern<<<grid, kUThreads, a.smem, st>>>(a);
  return check_launch("tcq_umma_kernel");
}

template <int BITS>
tp_status launch_umma_s(const UArgs& a, int m_tiles, int n_states, cudaStream_t st) {
  switch (n_states) {
    case 4: return launch_umma_t<BITS, 4>(a, m_tiles, st);
    case 8: return launch_umma_t<BITS, 8>(a, m_tiles, st);
    case 16: return launch_umma_t<BITS, 16>(a, m_tiles, st);
    default: return launch_umma_t<BITS, 64>(a, m_tiles, st);
  }
}

int sm_count_u() {
  int dev = 0, v = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return 148;
  if (cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || v <= 0) return 148;
  return v;
}

}  // namespace

extern "C" int64_t tp_gemm_tc_workspace_bytes(int64_t B, int64_t n, int64_t d) {
  if (B < 0 || n < 0 || d < 0) return -1;
  const int64_t nb = B < kUMaxN ? B : kUMaxN;
  const int64_t NB = (nb + 15) / 16 * 16;
  return pad_to(NB * pad_to(d, kUnitCols) * 2, 256) + pad_to(nb * n * 4, 256);
}

extern "C" tp_status tp_tcq_gemm_tc(const void* x, int x_dtype, const uint16_t* rot_scale, const uint8_t* tcq_stream,
                                    const uint16_t* scales, const uint16_t* codebook, const uint16_t* bias, void* y,
                                    int y_dtype, int64_t B, int64_t n, int64_t d, int64_t block, int bits,
                                    int n_states, void* workspace, int64_t workspace_bytes, void* stream) {
  if (!x || !rot_scale || !tcq_stream || !scales || !codebook || !y || B < 0 || n < 0 || d < 0)
    return fail(TP_ERR_ARG, "tp_tcq_gemm_tc: bad arguments");
  if (B == 0 || n == 0) return clear_ok();
  if (bits < 1 || bits > 4) return fail(TP_ERR_UNSUPPORTED, "tp_tcq_gemm_tc: bits must be 1..4");
  if (log2_states(n_states) < 0) return fail(TP_ERR_UNSUPPORTED, "n_states must be 4, 8, 16 or 64");
  if (!valid_dtype(x_dtype) || !valid_dtype(y_dtype)) return fail(TP_ERR_ARG, "tp_tcq_gemm_tc: bad dtype");
  if (!aligned(tcq_stream, 16) || !aligned(workspace, 256))
    return fail(TP_ERR_ALIGN, "tp_tcq_gemm_tc: stream 16-byte and workspace 256-byte alignment required");
  if (workspace_bytes < tp_gemm_tc_workspace_bytes(B, n, d))
    return fail(TP_ERR_WORKSPACE, "tp_tcq_gemm_tc: workspace too small");
  if (n > (int64_t)1 << 30 || d > (int64_t)1 << 22) return fail(TP_ERR_UNSUPPORTED, "tp_tcq_gemm_tc: shape too big");
  cudaStream_t st = as_stream(stream);
  const int64_t d_pad = pad_to(d, kUnitCols);
  const int64_t n_pad = pad_to(n, kTileRows);
  const int units_k = (int)(d_pad / kUnitCols);
  const int row_tiles = (int)(n_pad / kTileRows);
  const int m_tiles = (int)((n + 127) / 128);
  const int G = sm_count_u();
  int ksplit = G / m_tiles;  // one CTA per SM: keep the grid within one wave
  if (ksplit > units_k) ksplit = units_k;
  if (ksplit < 1) ksplit = 1;
  const uint32_t lut = bits == 4 ? LutCfg<4>::kLutBytes : LutCfg<3>::kLutBytes;
  const int64_t max_n = bits == 4 ? 32 : kUMaxN;
  for (int64_t b0 = 0; b0 < B; b0 += max_n) {
    const int nb = (int)(B - b0 < max_n ? B - b0 : max_n);
    const int NB = (nb + 15) / 16 * 16;
    __half* z = static_cast<__half*>(workspace);
    float* y32 = reinterpret_cast<float*>(static_cast<unsigned char*>(workspace) + pad_to((int64_t)NB * d_pad * 2, 256));
    // rotated activations of this batch chunk, zero rows up to NB
    TP_CUDA_TRY(cudaMemsetAsync(z, 0, (size_t)NB * d_pad * 2, st), "cudaMemsetAsync(z)");
    RotateArgs ra{};
    ra.x = static_cast<const unsigned char*>(x) + (size_t)b0 * d * (x_dtype == TP_F32 ? 4 : 2);
    ra.x_dtype = x_dtype;
    ra.scale = rot_scale;
    ra.z = z;
    ra.z_dtype = TP_F16;
    ra.d = d;
    ra.d_pad = d_pad;
    ra.block = block;
    ra.mode = 2;
    if (tp_status s = launch_rotate(ra, nb, st)) return s;
    TP_CUDA_TRY(cudaMemsetAsync(y32, 0, (size_t)nb * n * 4, st), "cudaMemsetAsync(y32)");
    UArgs a{};
    a.stream = reinterpret_cast<const uint4*>(tcq_stream);
    a.scales = scales;
    a.codebook = codebook;
    a.z = z;
    a.y32 = y32;
    a.B = nb;
    a.NB = NB;
    a.n = (int)n;
    a.d_pad = (int)d_pad;
    a.units_k = units_k;
    a.row_tiles = row_tiles;
    a.ksplit = ksplit;
    a.lut_off = 0;
    a.a_off = lut;
    a.b_off = a.a_off + 2 * kATile;
    a.w_off = a.b_off + 3 * (uint32_t)(NB * 256);
    const uint32_t depth = bits <= 3 ? 4u : 0u;
    a.bar_off = a.w_off + (uint32_t)kUWarps * depth * 512u * (uint32_t)bits;
    a.smem = a.bar_off + 8u * (4u + (uint32_t)kUWarps * depth);
    tp_status s;
    switch (bits) {
      case 1: s = launch_umma_s<1>(a, m_tiles, n_states, st); break;
      case 2: s = launch_umma_s<2>(a, m_tiles, n_states, st); break;
      case 3: s = launch_umma_s<3>(a, m_tiles, n_states, st); break;
      default: s = launch_umma_s<4>(a, m_tiles, n_states, st); break;
    }
    if (s) return s;
    const int64_t total = (int64_t)nb * n;
    finish_kernel<<<(unsigned)((total + 255) / 256), 256, 0, st>>>(
        y32, bias, static_cast<unsigned char*>(y) + (size_t)b0 * n * (y_dtype == TP_F32 ? 4 : 2), y_dtype, nb, (int)n);
    if (tp_status s2 = check_launch("finish_kernel")) return s2;
  }
  return clear_ok();
}

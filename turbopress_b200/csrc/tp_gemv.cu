// Fused packed-TCQ GEMV / skinny GEMM for batch 1..32 on sm_100a.
//
// y[b, r] = scale[r] * sum_c codebook[level(r, c)] * z[b, c]  (+ bias[r])
//
// Data path per warp (16 output rows, see tp_common.cuh for the stream
// layout):
//   1. coalesced 16-byte non-allocating loads of the true-rate stream
//      (bits words per row per 32 columns), prefetched one unit ahead;
//   2. the 6-bit trellis halo of every 32-column chunk comes from the
//      neighbouring lane by one warp shuffle;
//   3. register bit-slicing: the two subset bit-planes are GF(2)
//      convolutions of the path word (funnel shifts + XOR), merged with the
//      member bits into four "level words" of 8 nibbles (LOP3 selects);
//   4. each byte of a level word (two 4-bit levels) is turned into a shared
//      memory address by ONE byte permute (byte | lane*4) and looked up in a
//      lane-replicated pair table holding half2(codebook[lo], codebook[hi]),
//      so 32 lanes hit 32 distinct banks;
//   5. the half2 weight pairs are the A fragments of a warp-level
//      m16n8k16 tensor-core MMA (fp32 accumulate) against the rotated
//      activations held in shared memory (B fragments), so the reduction
//      over columns costs one MMA per 256 weights instead of 128 HFMA2;
//   6. split-K over CTAs, reduced deterministically by the last CTA of each
//      row block (counter in the workspace), scale/bias/cast fused.
//
// 4-bit payloads (5-bit levels) use a 1024-entry pair table: the two fifth
// level bits are carried in bit 7 and bit 16 of the address via a second
// permute source (see build_lut / lut_addr4).
#include <algorithm>
#include <mutex>

#include "tp_rotate.cuh"

using namespace tp;

namespace {

constexpr int kMaxBatchPerLaunch = 32;  // 4 n-tiles of the m16n8k16 MMA
// The workspace starts with a fixed-size block of split-K counters, so calls
// of different shapes sharing one workspace never overlap each other's
// counters with their activation or partial-sum regions.
constexpr int64_t kMaxRowBlocks = 16384;
constexpr int64_t kCounterBytes = kMaxRowBlocks * 4;

template <int BITS>
struct Cfg {
  static constexpr int kLutBytes = BITS == 4 ? 131072 : 65536;
  static constexpr int kWarps = BITS == 4 ? 16 : 8;
};

struct GemvParams {
  const uint4* stream;
  const uint16_t* scales;
  const uint16_t* bias;
  const uint16_t* codebook;
  const uint4* zperm;  // [B][d_pad] fp16, permuted pair order
  void* y;
  float* partial;      // [ksplit][B][n_pad]
  unsigned* counters;  // [row_blocks]
  int y_dtype;
  int B;
  int64_t n;
  int64_t n_pad;
  int64_t d_pad;
  int units_k;
  int ksplit;
};

__device__ __forceinline__ uint4 ldg_stream(const uint4* p) {
  uint4 v;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p));
  return v;
}

__device__ __forceinline__ uint32_t prmt(uint32_t a, uint32_t b, uint32_t sel) {
  uint32_t r;
  asm("prmt.b32 %0, %1, %2, %3;" : "=r"(r) : "r"(a), "r"(b), "r"(sel));
  return r;
}

__device__ __forceinline__ void mma16816(float* c, uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0,
                                         uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// Pair table.  bits <= 3: entry e (byte of a level word) at byte offset
// e*256 + lane*4 holds half2(cb[lo(e)], cb[hi(e)]); levels ignore nibble bits
// above the level width.  bits == 4: entry key k = m2lo<<7 | byte<<8 |
// m2hi<<16 (word offset k + lane*4), levels (byte nibble | m2 << 4).
template <int BITS>
__device__ void build_lut(uint32_t* lut, const uint16_t* __restrict__ cb, int tid, int nthreads) {
  const int lane = tid & 31;
  const int warp = tid >> 5, nwarps = nthreads >> 5;
  if (BITS <= 3) {
    const unsigned lmask = (1u << (BITS + 1)) - 1u;
    for (int e = warp; e < 256; e += nwarps) {
      const uint32_t lo = cb[e & 15 & lmask], hi = cb[(e >> 4) & lmask];
      lut[e * 64 + lane] = lo | (hi << 16);
    }
  } else {
    for (int k = warp; k < 1024; k += nwarps) {
      const int byte = k & 255, m2lo = (k >> 8) & 1, m2hi = k >> 9;
      const uint32_t lo = cb[(byte & 15) | (m2lo << 4)], hi = cb[(byte >> 4) | (m2hi << 4)];
      const int off = (m2lo << 7) | (byte << 8) | (m2hi << 16);
      lut[(off >> 2) + lane] = lo | (hi << 16);
    }
  }
}

// Subset bit-planes of one 32-column chunk and the four level words.
template <int S>
__device__ __forceinline__ void level_words(uint32_t P, uint32_t H, uint32_t A, uint32_t Bm, uint32_t Cw, uint32_t Dm,
                                            uint32_t* L) {
  constexpr int m = mlog(S);
  constexpr unsigned K0 = kmask(gen0(S), m), K1 = kmask(gen1(S), m);
  uint32_t s0 = 0, s1 = 0;
#pragma unroll
  for (int k = 0; k <= m; ++k) {
    const uint32_t dk = k == 0 ? P : __funnelshift_l(H, P, k);  // bit t = b_{t-k}
    if ((K0 >> k) & 1u) s0 ^= dk;
    if ((K1 >> k) & 1u) s1 ^= dk;
  }
  // E: subsets of even columns in 2-bit fields, O: odd columns
  const uint32_t E = (s0 & 0x55555555u) | ((s1 << 1) & 0xAAAAAAAAu);
  const uint32_t O = ((s0 >> 1) & 0x55555555u) | (s1 & 0xAAAAAAAAu);
  L[0] = (E & 0x33333333u) | (A & 0xCCCCCCCCu);
  L[1] = ((E >> 2) & 0x33333333u) | (Bm & 0xCCCCCCCCu);
  L[2] = (O & 0x33333333u) | (Cw & 0xCCCCCCCCu);
  L[3] = ((O >> 2) & 0x33333333u) | (Dm & 0xCCCCCCCCu);
}

// member words of one row-chunk for the level-word merge
template <int BITS>
__device__ __forceinline__ void member_words(uint32_t M0, uint32_t M1, uint32_t& A, uint32_t& Bm, uint32_t& Cw,
                                             uint32_t& Dm) {
  if (BITS == 1) {
    A = Bm = Cw = Dm = 0u;
  } else if (BITS == 2) {
    A = M0;
    Bm = M0 >> 1;
    Cw = M0 << 2;
    Dm = M0 << 1;
  } else {
    A = M0;
    Bm = M0 << 2;
    Cw = M1;
    Dm = M1 << 2;
  }
}

__device__ __forceinline__ uint32_t lds32(const unsigned char* base, uint32_t off) {
  return *reinterpret_cast<const uint32_t*>(base + off);
}

// 4-bit address word for level word w, byte pair q (bytes 2q, 2q+1).
__device__ __forceinline__ uint32_t x4(uint32_t M2, int w, int q, uint32_t lanepat) {
  const int s = 2 * (2 * w + q);
  return (__funnelshift_r(M2, M2, s) & 0x01800180u) | lanepat;
}

template <int BITS, int S, int NT>
__device__ __forceinline__ void process_chunk(const unsigned char* lut, uint32_t lanew, const uint4* zq_base,
                                              uint32_t Pg, uint32_t Hg, uint32_t Pq, uint32_t Hq, uint32_t Mg0,
                                              uint32_t Mg1, uint32_t Mg2, uint32_t Mq0, uint32_t Mq1, uint32_t Mq2,
                                              const int* zoff, float (*acc)[4]) {
  uint32_t Lg[4], Lq[4];
  {
    uint32_t A, Bm, Cw, Dm;
    member_words<BITS>(Mg0, Mg1, A, Bm, Cw, Dm);
    level_words<S>(Pg, Hg, A, Bm, Cw, Dm, Lg);
    member_words<BITS>(Mq0, Mq1, A, Bm, Cw, Dm);
    level_words<S>(Pq, Hq, A, Bm, Cw, Dm, Lq);
  }
#pragma unroll
  for (int w = 0; w < 4; ++w) {
    uint4 zv[NT];
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) zv[nt] = zq_base[zoff[nt] + w];
#pragma unroll
    for (int q = 0; q < 2; ++q) {
      uint32_t a0, a1, a2, a3;
      if (BITS <= 3) {
        const uint32_t s0 = 0x5504u | ((2u * q) << 4), s1 = 0x5504u | ((2u * q + 1u) << 4);
        a0 = lds32(lut, prmt(Lg[w], lanew, s0));
        a2 = lds32(lut, prmt(Lg[w], lanew, s1));
        a1 = lds32(lut, prmt(Lq[w], lanew, s0));
        a3 = lds32(lut, prmt(Lq[w], lanew, s1));
      } else {
        const uint32_t xg = x4(Mg2, w, q, lanew), xq = x4(Mq2, w, q, lanew);
        const uint32_t s0 = 0xD504u | ((2u * q) << 4), s1 = 0xF706u | ((2u * q + 1u) << 4);
        a0 = lds32(lut, prmt(Lg[w], xg, s0));
        a2 = lds32(lut, prmt(Lg[w], xg, s1));
        a1 = lds32(lut, prmt(Lq[w], xq, s0));
        a3 = lds32(lut, prmt(Lq[w], xq, s1));
      }
#pragma unroll
      for (int nt = 0; nt < NT; ++nt) {
        const uint32_t b0 = q == 0 ? zv[nt].x : zv[nt].z;
        const uint32_t b1 = q == 0 ? zv[nt].y : zv[nt].w;
        mma16816(acc[nt], a0, a1, a2, a3, b0, b1);
      }
    }
  }
}

template <int BITS, int S, int NT>
__global__ void __launch_bounds__(Cfg<BITS>::kWarps * 32) tcq_gemv_kernel(GemvParams p) {
  constexpr int WARPS = Cfg<BITS>::kWarps;
  extern __shared__ __align__(16) unsigned char smem[];
  unsigned char* lut = smem;
  uint4* zs = reinterpret_cast<uint4*>(smem + Cfg<BITS>::kLutBytes);
  __shared__ unsigned s_last;

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int g = lane >> 2, t = lane & 3;
  const int ks = blockIdx.y;
  const int u0 = static_cast<int>((int64_t)ks * p.units_k / p.ksplit);
  const int u1 = static_cast<int>((int64_t)(ks + 1) * p.units_k / p.ksplit);
  const int nunits = u1 - u0;
  const int64_t rt = (int64_t)blockIdx.x * WARPS + warp;
  const bool active = rt * kTileRows < p.n_pad;

  // ---- prologue: first stream loads in flight before the table build ----
  const uint4* wp = p.stream + ((rt * p.units_k + u0) * 32 + lane) * BITS;
  const int64_t ustride = 32 * BITS;
  uint4 cur[BITS];
  uint32_t prevP1g = 0u, prevP1q = 0u;
  if (active && nunits > 0) {
#pragma unroll
    for (int i = 0; i < BITS; ++i) cur[i] = ldg_stream(wp + i);
    if (u0 > 0) {
      const uint4 pv = ldg_stream(wp - ustride);
      prevP1g = pv.z;
      prevP1q = pv.w;
    }
  }

  build_lut<BITS>(reinterpret_cast<uint32_t*>(lut), p.codebook, tid, WARPS * 32);
  const int zchunk = nunits * 32;  // uint4 per batch row in the slice
  for (int i = tid; i < p.B * zchunk; i += WARPS * 32) {
    const int b = i / zchunk, r = i - b * zchunk;
    zs[i] = p.zperm[(int64_t)b * (p.d_pad / 8) + (int64_t)u0 * 32 + r];
  }
  if (tid < 4) zs[p.B * zchunk + tid] = make_uint4(0, 0, 0, 0);
  __syncthreads();

  float acc[NT][4];
#pragma unroll
  for (int nt = 0; nt < NT; ++nt) acc[nt][0] = acc[nt][1] = acc[nt][2] = acc[nt][3] = 0.f;

  if (active) {
    // per n-tile z pointers: batch row nt*8+g, or the zero block
    int zbase[NT], zunit[NT];
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
      const int bn = nt * 8 + g;
      zbase[nt] = bn < p.B ? bn * zchunk + t * 4 : p.B * zchunk;
      zunit[nt] = bn < p.B ? 1 : 0;
    }
    const uint32_t lanew = BITS <= 3 ? (uint32_t)lane * 4u : (uint32_t)lane * 4u * 0x10001u;
    const int src = (lane & ~3) | ((t + 3) & 3);
    for (int i = 0; i < nunits; ++i) {
      uint4 nxt[BITS];
      if (i + 1 < nunits) {
#pragma unroll
        for (int k = 0; k < BITS; ++k) nxt[k] = ldg_stream(wp + (i + 1) * ustride + k);
      }
      const uint32_t P0g = cur[0].x, P0q = cur[0].y, P1g = cur[0].z, P1q = cur[0].w;
      // halos: neighbour lane's chunk (t-1), lane t=0 takes lane 3's
      const uint32_t H0g = __shfl_sync(0xffffffffu, t == 3 ? prevP1g : P0g, src);
      const uint32_t H0q = __shfl_sync(0xffffffffu, t == 3 ? prevP1q : P0q, src);
      const uint32_t H1g = __shfl_sync(0xffffffffu, t == 3 ? P0g : P1g, src);
      const uint32_t H1q = __shfl_sync(0xffffffffu, t == 3 ? P0q : P1q, src);
      prevP1g = P1g;
      prevP1q = P1q;
      const uint32_t z0 = 0u;
#pragma unroll
      for (int cg = 0; cg < 2; ++cg) {
        int zoff[NT];
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) zoff[nt] = zbase[nt] + zunit[nt] * (i * 32 + cg * 16);
        const uint32_t Pg = cg ? P1g : P0g, Pq = cg ? P1q : P0q;
        const uint32_t Hg = cg ? H1g : H0g, Hq = cg ? H1q : H0q;
        uint32_t Mg0 = z0, Mq0 = z0, Mg1 = z0, Mq1 = z0, Mg2 = z0, Mq2 = z0;
        if (BITS >= 2) {
          Mg0 = cg ? cur[1].z : cur[1].x;
          Mq0 = cg ? cur[1].w : cur[1].y;
        }
        if (BITS >= 3) {
          Mg1 = cg ? cur[2].z : cur[2].x;
          Mq1 = cg ? cur[2].w : cur[2].y;
        }
        if (BITS >= 4) {
          Mg2 = cg ? cur[3].z : cur[3].x;
          Mq2 = cg ? cur[3].w : cur[3].y;
        }
        process_chunk<BITS, S, NT>(lut, lanew, zs, Pg, Hg, Pq, Hq, Mg0, Mg1, Mg2, Mq0, Mq1, Mq2, zoff, acc);
      }
      if (i + 1 < nunits) {
#pragma unroll
        for (int k = 0; k < BITS; ++k) cur[k] = nxt[k];
      }
    }
  }

  // ---- epilogue ----
  const int64_t row_g = rt * kTileRows + g, row_q = row_g + 8;
  if (p.ksplit == 1) {
    if (active) {
#pragma unroll
      for (int nt = 0; nt < NT; ++nt) {
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int bn = nt * 8 + 2 * t + (e & 1);
          const int64_t row = (e < 2) ? row_g : row_q;
          if (bn < p.B && row < p.n) {
            float v = acc[nt][e] * h2f_bits(p.scales[row]);
            if (p.bias) v += h2f_bits(p.bias[row]);
            store_from_float(p.y, (int64_t)bn * p.n + row, p.y_dtype, v);
          }
        }
      }
    }
    return;
  }
  if (active) {
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int bn = nt * 8 + 2 * t + (e & 1);
        const int64_t row = (e < 2) ? row_g : row_q;
        if (bn < p.B) p.partial[((int64_t)ks * p.B + bn) * p.n_pad + row] = acc[nt][e];
      }
    }
  }
  __threadfence();
  __syncthreads();
  if (tid == 0) {
    const unsigned prev = atomicAdd(&p.counters[blockIdx.x], 1u);
    s_last = (prev == (unsigned)p.ksplit - 1u) ? 1u : 0u;
  }
  __syncthreads();
  if (!s_last) return;
  __threadfence();
  const int64_t row0 = (int64_t)blockIdx.x * WARPS * kTileRows;
  const int rows = WARPS * kTileRows;
  for (int i = tid; i < rows * p.B; i += WARPS * 32) {
    const int bn = i / rows;
    const int64_t row = row0 + (i - bn * rows);
    if (row >= p.n) continue;
    float v = 0.f;
    for (int k = 0; k < p.ksplit; ++k) v += __ldcg(&p.partial[((int64_t)k * p.B + bn) * p.n_pad + row]);
    v *= h2f_bits(p.scales[row]);
    if (p.bias) v += h2f_bits(p.bias[row]);
    store_from_float(p.y, (int64_t)bn * p.n + row, p.y_dtype, v);
  }
  if (tid == 0) p.counters[blockIdx.x] = 0u;
}

// ---------------------------------------------------------------------------
// launch configuration
// ---------------------------------------------------------------------------
struct Plan {
  int warps;
  int64_t row_blocks;
  int units_k;
  int ksplit;
  size_t smem;
  int64_t ws_counters, ws_z, ws_partial, ws_total;
};

int sm_count() {
  static std::mutex mu;
  static int cache[64] = {0};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return 148;
  std::lock_guard<std::mutex> lk(mu);
  if (dev >= 64) return 148;
  if (!cache[dev]) {
    int v = 0;
    if (cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || v <= 0) v = 148;
    cache[dev] = v;
  }
  return cache[dev];
}

inline int64_t align256(int64_t v) { return (v + 255) / 256 * 256; }

Plan make_plan(int64_t B, int64_t n, int64_t d, int bits, int sms) {
  Plan pl{};
  const int64_t Bc = B < kMaxBatchPerLaunch ? B : kMaxBatchPerLaunch;
  pl.warps = bits == 4 ? Cfg<4>::kWarps : Cfg<3>::kWarps;
  const int64_t n_pad = pad_to(n, kTileRows), d_pad = pad_to(d, kUnitCols);
  const int64_t row_tiles = n_pad / kTileRows;
  pl.row_blocks = (row_tiles + pl.warps - 1) / pl.warps;
  pl.units_k = static_cast<int>(d_pad / kUnitCols);
  const int ctas_per_sm = bits == 4 ? 1 : 3;
  const int64_t target = (int64_t)sms * ctas_per_sm;
  int64_t ks = (target + pl.row_blocks - 1) / pl.row_blocks;
  // keep the activation slice in shared memory modest: <= 64 KB
  const int64_t max_units_smem = std::max<int64_t>(1, (64 * 1024) / (Bc * 512));
  const int64_t min_ks = (pl.units_k + max_units_smem - 1) / max_units_smem;
  ks = std::max(ks, min_ks);
  ks = std::min<int64_t>(ks, 32);
  ks = std::min<int64_t>(ks, pl.units_k);
  ks = std::max<int64_t>(ks, 1);
  pl.ksplit = static_cast<int>(ks);
  const int64_t slice_units = (pl.units_k + pl.ksplit - 1) / pl.ksplit;
  const int lut = bits == 4 ? Cfg<4>::kLutBytes : Cfg<3>::kLutBytes;
  pl.smem = static_cast<size_t>(lut + (Bc * slice_units * 32 + 4) * 16);
  pl.ws_counters = kCounterBytes;
  pl.ws_z = align256(Bc * d_pad * 2);
  pl.ws_partial = pl.ksplit > 1 ? align256((int64_t)pl.ksplit * Bc * n_pad * 4) : 0;
  pl.ws_total = pl.ws_counters + pl.ws_z + pl.ws_partial;
  return pl;
}

template <int BITS, int S, int NT>
tp_status launch_gemv_t(const GemvParams& p, const Plan& pl, cudaStream_t stream) {
  auto kern = tcq_gemv_kernel<BITS, S, NT>;
  static int smem_set[64] = {0};
  if (tp_status s = ensure_smem(kern, pl.smem, smem_set, "cudaFuncSetAttribute(gemv)")) return s;
  dim3 grid(static_cast<unsigned>(pl.row_blocks), static_cast<unsigned>(pl.ksplit));
  kern<<<grid, Cfg<BITS>::kWarps * 32, pl.smem, stream>>>(p);
  return check_launch("tcq_gemv_kernel");
}

template <int BITS, int S>
tp_status launch_gemv_nt(const GemvParams& p, const Plan& pl, cudaStream_t stream) {
  const int nt = (p.B + 7) / 8;
  switch (nt) {
    case 1: return launch_gemv_t<BITS, S, 1>(p, pl, stream);
    case 2: return launch_gemv_t<BITS, S, 2>(p, pl, stream);
    case 3: return launch_gemv_t<BITS, S, 3>(p, pl, stream);
    default: return launch_gemv_t<BITS, S, 4>(p, pl, stream);
  }
}

template <int BITS>
tp_status launch_gemv_s(const GemvParams& p, const Plan& pl, int n_states, cudaStream_t stream) {
  switch (n_states) {
    case 4: return launch_gemv_nt<BITS, 4>(p, pl, stream);
    case 8: return launch_gemv_nt<BITS, 8>(p, pl, stream);
    case 16: return launch_gemv_nt<BITS, 16>(p, pl, stream);
    default: return launch_gemv_nt<BITS, 64>(p, pl, stream);
  }
}

tp_status launch_gemv(const GemvParams& p, const Plan& pl, int bits, int n_states, cudaStream_t stream) {
  switch (bits) {
    case 1: return launch_gemv_s<1>(p, pl, n_states, stream);
    case 2: return launch_gemv_s<2>(p, pl, n_states, stream);
    case 3: return launch_gemv_s<3>(p, pl, n_states, stream);
    default: return launch_gemv_s<4>(p, pl, n_states, stream);
  }
}

// ---------------------------------------------------------------------------
// reference-order GEMV straight from format-v2 streams (any bits 1..7)
// ---------------------------------------------------------------------------
__global__ void gemv_v2_kernel(const float* __restrict__ z, const uint8_t* __restrict__ path,
                               const uint8_t* __restrict__ member, const uint16_t* __restrict__ scales,
                               const uint16_t* __restrict__ codebook, const uint16_t* __restrict__ bias, void* y,
                               int y_dtype, int B, int64_t n, int64_t d, int bits, unsigned k0, unsigned k1, int m) {
  const int lane = threadIdx.x & 31;
  const int64_t row = (int64_t)blockIdx.x * (blockDim.x / 32) + (threadIdx.x >> 5);
  if (row >= n) return;
  const int64_t prb = (d + 7) / 8, mrb = (d * (bits - 1) + 7) / 8;
  const uint8_t* pr = path + row * prb;
  const uint8_t* mr = bits > 1 ? member + row * mrb : nullptr;
  const float sc = h2f_bits(scales[row]);
  float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
  for (int64_t c = lane; c < d; c += 32) {
    unsigned win = 0;
    for (int k = 0; k <= m; ++k)
      if (c - k >= 0) win |= ((pr[(c - k) >> 3] >> ((c - k) & 7)) & 1u) << k;
    unsigned mv = 0;
    for (int j = 0; j < bits - 1; ++j) {
      const int64_t bit = c * (bits - 1) + j;
      mv |= ((mr[bit >> 3] >> (bit & 7)) & 1u) << j;
    }
    const unsigned level = mv * 4u + subset_of_window(win, k0, k1);
    // the reference multiplies by the fp16-rounded dequantized weight
    const float w = __half2float(__float2half_rn(h2f_bits(codebook[level]) * sc));
#pragma unroll
    for (int b = 0; b < 8; ++b)
      if (b < B) acc[b] = fmaf(w, z[(int64_t)b * d + c], acc[b]);
  }
#pragma unroll
  for (int b = 0; b < 8; ++b) {
    if (b >= B) break;
    float v = acc[b];
    for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    if (lane == 0) {
      if (bias) v += h2f_bits(bias[row]);
      store_from_float(y, (int64_t)b * n + row, y_dtype, v);
    }
  }
}

}  // namespace

extern "C" int64_t tp_gemv_workspace_bytes(int64_t B, int64_t n, int64_t d, int bits) {
  if (B < 1 || n < 1 || d < 1 || bits < 1 || bits > 4) return -1;
  return make_plan(B, n, d, bits, sm_count()).ws_total;
}

extern "C" tp_status tp_tcq_gemv(const void* x, int x_dtype, const uint16_t* rot_scale, const uint8_t* tcq_stream,
                                 const uint16_t* scales, const uint16_t* codebook, const uint16_t* bias, void* y,
                                 int y_dtype, int64_t B, int64_t n, int64_t d, int64_t block, int bits, int n_states,
                                 void* workspace, int64_t workspace_bytes, void* stream) {
  if (!x || !rot_scale || !tcq_stream || !scales || !codebook || !y || B < 0 || n < 0 || d < 0)
    return fail(TP_ERR_ARG, "tp_tcq_gemv: bad arguments");
  if (!valid_dtype(x_dtype) || !valid_dtype(y_dtype)) return fail(TP_ERR_ARG, "tp_tcq_gemv: bad dtype");
  if (bits < 1 || bits > 4) return fail(TP_ERR_UNSUPPORTED, "tp_tcq_gemv: bits must be 1..4 (got %d)", bits);
  if (log2_states(n_states) < 0) return fail(TP_ERR_UNSUPPORTED, "n_states must be 4, 8, 16 or 64 (got %d)", n_states);
  if (!aligned(tcq_stream, 16)) return fail(TP_ERR_ALIGN, "tp_tcq_gemv: stream must be 16-byte aligned");
  if (B == 0 || n == 0) return clear_ok();
  if (d == 0) return fail(TP_ERR_ARG, "tp_tcq_gemv: d must be positive");
  const Plan pl = make_plan(B, n, d, bits, sm_count());
  if (pl.row_blocks > kMaxRowBlocks)
    return fail(TP_ERR_UNSUPPORTED, "tp_tcq_gemv: n=%lld exceeds the supported maximum row count", (long long)n);
  if (!workspace || workspace_bytes < pl.ws_total)
    return fail(TP_ERR_WORKSPACE, "tp_tcq_gemv: workspace of %lld bytes required (got %lld)", (long long)pl.ws_total,
                (long long)workspace_bytes);
  if (!aligned(workspace, 256)) return fail(TP_ERR_ALIGN, "tp_tcq_gemv: workspace must be 256-byte aligned");
  cudaStream_t st = as_stream(stream);
  unsigned char* ws = static_cast<unsigned char*>(workspace);
  const int64_t d_pad = pad_to(d, kUnitCols), n_pad = pad_to(n, kTileRows);
  const size_t xel = x_dtype == TP_F32 ? 4 : 2, yel = y_dtype == TP_F32 ? 4 : 2;
  for (int64_t b0 = 0; b0 < B; b0 += kMaxBatchPerLaunch) {
    const int64_t Bc = std::min<int64_t>(kMaxBatchPerLaunch, B - b0);
    const Plan pc = make_plan(Bc, n, d, bits, sm_count());
    RotateArgs ra{};
    ra.x = static_cast<const unsigned char*>(x) + b0 * d * xel;
    ra.x_dtype = x_dtype;
    ra.scale = rot_scale;
    ra.z = ws + pl.ws_counters;
    ra.z_dtype = TP_F16;
    ra.d = d;
    ra.d_pad = d_pad;
    ra.block = block;
    ra.mode = 2;
    if (tp_status s = launch_rotate(ra, Bc, st)) return s;
    GemvParams p{};
    p.stream = reinterpret_cast<const uint4*>(tcq_stream);
    p.scales = scales;
    p.bias = bias;
    p.codebook = codebook;
    p.zperm = reinterpret_cast<const uint4*>(ws + pl.ws_counters);
    p.y = static_cast<unsigned char*>(y) + b0 * n * yel;
    p.partial = reinterpret_cast<float*>(ws + pl.ws_counters + pl.ws_z);
    p.counters = reinterpret_cast<unsigned*>(ws);
    p.y_dtype = y_dtype;
    p.B = static_cast<int>(Bc);
    p.n = n;
    p.n_pad = n_pad;
    p.d_pad = d_pad;
    p.units_k = pc.units_k;
    p.ksplit = pc.ksplit;
    if (tp_status s = launch_gemv(p, pc, bits, n_states, st)) return s;
  }
  return clear_ok();
}

extern "C" tp_status tp_gemv_v2(const float* z, const uint8_t* path_packed, const uint8_t* member_packed,
                                const uint16_t* scales, const uint16_t* codebook, const uint16_t* bias, void* y,
                                int y_dtype, int64_t B, int64_t n, int64_t d, int bits, int n_states, void* stream) {
  if (!z || !path_packed || !scales || !codebook || !y || B < 0 || n < 0 || d < 0)
    return fail(TP_ERR_ARG, "tp_gemv_v2: bad arguments");
  if (bits < 1 || bits > 7) return fail(TP_ERR_UNSUPPORTED, "tp_gemv_v2: bits must be 1..7 (got %d)", bits);
  if (bits > 1 && !member_packed) return fail(TP_ERR_ARG, "tp_gemv_v2: member stream required for bits > 1");
  if (!valid_dtype(y_dtype)) return fail(TP_ERR_ARG, "tp_gemv_v2: bad dtype");
  unsigned k0, k1;
  int m;
  if (log2_states(n_states) < 0) return fail(TP_ERR_UNSUPPORTED, "n_states must be 4, 8, 16 or 64 (got %d)", n_states);
  tap_masks(n_states, k0, k1, m);
  if (B == 0 || n == 0) return clear_ok();
  const int rows_per_cta = 8;
  for (int64_t b0 = 0; b0 < B; b0 += 8) {
    const int Bc = static_cast<int>(std::min<int64_t>(8, B - b0));
    const size_t yel = y_dtype == TP_F32 ? 4 : 2;
    gemv_v2_kernel<<<static_cast<unsigned>((n + rows_per_cta - 1) / rows_per_cta), rows_per_cta * 32, 0,
                     as_stream(stream)>>>(z + b0 * d, path_packed, member_packed, scales, codebook, bias,
                                          static_cast<unsigned char*>(y) + b0 * n * yel, y_dtype, Bc, n, d, bits, k0,
                                          k1, m);
    if (tp_status s = check_launch("gemv_v2_kernel")) return s;
  }
  return clear_ok();
}

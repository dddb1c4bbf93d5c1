// Decode core of the stream-K packed-TCQ kernels (per-call GEMV in
// tp_gemv_sk.cu, persistent decode step in tp_step.cu): the flat split of
// weight units over warps, the GF(2) trellis decode into level words, the
// pair tables and the lookup + MMA step.
#pragma once

#include "tp_decode.cuh"

namespace tp {
namespace sk {

constexpr uint32_t kLutAbs = 0x10000u;  // shared-window address of the bits <= 3 pair table
// Activation rows in shared memory are padded by 64 bytes so that rows g and
// g+1 (and the zero row) start in different bank halves.
constexpr int kZPad = 32;

// q = x / d for 0 <= x < 2^31 by multiply-high (divisor fixed per launch).
struct FastDiv {
  uint32_t m, l;
  __device__ __forceinline__ uint32_t operator()(uint32_t x) const { return (__umulhi(x, m) + x) >> l; }
};

inline FastDiv make_fastdiv(uint32_t d) {
  uint32_t l = 0;
  while ((uint64_t(1) << l) < d) ++l;
  const uint64_t m = ((uint64_t(1) << 32) * ((uint64_t(1) << l) - d)) / d + 1;
  return FastDiv{static_cast<uint32_t>(m), l};
}

// One K-slice's split of its flat unit index space x in [0, row_tiles * us):
// warp w < nw runs [w*r + min(w, rem), (w+1)*r + min(w+1, rem)) (the first
// `rem` warps take r+1 units).
struct SliceSplit {
  int us;     // units per row tile in this slice
  int r, rem;
  int nw;     // warps with work (the others' runs are empty)
  FastDiv div_us, div_r, div_r1;
  __device__ __forceinline__ int start(int w) const { return w * r + min(w, rem); }
  // the warp whose run holds flat index x
  __device__ __forceinline__ int warp_of(int x) const {
    const int b = rem * (r + 1);
    return x < b ? static_cast<int>(div_r1(x)) : rem + static_cast<int>(div_r(x - b));
  }
  __device__ __forceinline__ int row_tile(int x) const { return static_cast<int>(div_us(x)); }
};

// Subset bit-planes of one 32-column chunk: the taps both generators share
// are XORed once.
template <int S>
__device__ __forceinline__ void subset_planes(uint32_t P, uint32_t H, uint32_t& s0, uint32_t& s1) {
  constexpr int m = mlog(S);
  constexpr unsigned K0 = kmask(gen0(S), m), K1 = kmask(gen1(S), m), C = K0 & K1;
  uint32_t c = 0u, x0 = 0u, x1 = 0u;
#pragma unroll
  for (int k = 0; k <= m; ++k) {
    const uint32_t dk = k == 0 ? P : __funnelshift_l(H, P, k);  // bit t = b_{t-k}
    if ((C >> k) & 1u) c ^= dk;
    else if ((K0 >> k) & 1u) x0 ^= dk;
    else if ((K1 >> k) & 1u) x1 ^= dk;
  }
  s0 = c ^ x0;
  s1 = c ^ x1;
}

// Four level words of a row-chunk.  Byte j of word w holds two levels (see
// tp_common.cuh); for BITS == 3, words 1 and 3 keep each nibble rotated by
// two bits (member in bits 0-1, subset in bits 2-3) and use the second table.
template <int BITS, int S>
__device__ __forceinline__ void level_words_sk(uint32_t P, uint32_t H, uint32_t M0, uint32_t M1, uint32_t* L) {
  uint32_t s0, s1;
  subset_planes<S>(P, H, s0, s1);
  const uint32_t E = (s0 & 0x55555555u) | ((s1 << 1) & 0xAAAAAAAAu);
  const uint32_t O = ((s0 >> 1) & 0x55555555u) | (s1 & 0xAAAAAAAAu);
  if (BITS == 3) {
    L[0] = (E & 0x33333333u) | (M0 & 0xCCCCCCCCu);
    L[1] = (E & 0xCCCCCCCCu) | (M0 & 0x33333333u);
    L[2] = (O & 0x33333333u) | (M1 & 0xCCCCCCCCu);
    L[3] = (O & 0xCCCCCCCCu) | (M1 & 0x33333333u);
  } else {
    uint32_t A, Bm, Cw, Dm;
    member_words<BITS>(M0, M1, A, Bm, Cw, Dm);
    L[0] = (E & 0x33333333u) | (A & 0xCCCCCCCCu);
    L[1] = ((E >> 2) & 0x33333333u) | (Bm & 0xCCCCCCCCu);
    L[2] = (O & 0x33333333u) | (Cw & 0xCCCCCCCCu);
    L[3] = ((O >> 2) & 0x33333333u) | (Dm & 0xCCCCCCCCu);
  }
}

__device__ __forceinline__ uint32_t lds_abs_v(uint32_t addr) {
  uint32_t v;
  asm volatile("ld.shared.b32 %0, [%1];" : "=r"(v) : "r"(addr));
  return v;
}

__device__ __forceinline__ uint32_t lds_rel_v(const unsigned char* base, uint32_t off) {
  return *reinterpret_cast<const volatile uint32_t*>(base + off);
}

__device__ __forceinline__ void prefetch_l2(const void* p, unsigned bytes) {
  asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(p), "r"(bytes) : "memory");
}

// Pair tables.  bits <= 3: table A (entry e at e*256 + lane*4) holds
// half2(cb[lo nibble], cb[hi nibble]); for bits == 3 table B (same entry +128)
// holds the nibble-rotated form.  bits == 4: the 1024-entry table of
// build_lut<4>.
template <int BITS>
__device__ __forceinline__ void build_tables(unsigned char* lut, uint32_t cbv, int warp, int lane, int nwarps) {
  if (BITS == 4) {
    build_lut<4>(lut, cbv, warp, lane, nwarps);
    return;
  }
  constexpr int kTabs = BITS == 3 ? 2 : 1;
  constexpr unsigned lmask = (1u << (BITS + 1)) - 1u;
  const int row = lane >> 3, col = lane & 7;
  for (int r0 = warp * 4; r0 < 256 * kTabs; r0 += nwarps * 4) {
    const int r = r0 + row;
    const int tab = kTabs == 2 ? (r & 1) : 0;
    const int e = kTabs == 2 ? (r >> 1) : r;
    unsigned lo = e & 15u, hi = (e >> 4) & 15u;
    if (tab) {
      lo = ((lo >> 2) | (lo << 2)) & 15u;
      hi = ((hi >> 2) | (hi << 2)) & 15u;
    }
    const uint32_t vlo = __shfl_sync(0xffffffffu, cbv, lo & lmask);
    const uint32_t vhi = __shfl_sync(0xffffffffu, cbv, hi & lmask);
    const uint32_t v = vlo | (vhi << 16);
    *reinterpret_cast<uint4*>(lut + e * 256 + tab * 128 + col * 16) = make_uint4(v, v, v, v);
  }
}

// Activation fragment: a 16-byte shared load for the lanes whose batch row
// exists; the other lanes keep the zeros they start with (predicated, so the
// shared-memory pipe serves only the active quarter-warps).
__device__ __forceinline__ void lds_z(uint4& v, const uint4* p, bool on) {
  asm volatile(
      "{\n .reg .pred q;\n setp.ne.b32 q, %4, 0;\n @q ld.shared.v4.b32 {%0,%1,%2,%3}, [%5];\n}"
      : "+r"(v.x), "+r"(v.y), "+r"(v.z), "+r"(v.w)
      : "r"((int)on), "r"(smem_u32(p)));
}

// Pair lookups and MMAs of one 32-column chunk pair (rows g and g+8): 8 MMAs.
// Lg / Lq: the chunk's level words of rows g and g+8; M2g / M2q: the fifth
// level bits (4-bit payloads only).
template <int BITS>
__device__ __forceinline__ void sk_mma_chunk(uint32_t lwA, uint32_t lwB, const unsigned char* lut, const uint4* zp,
                                             bool zon, uint4& zv, const uint32_t* Lg, const uint32_t* Lq,
                                             uint32_t M2g, uint32_t M2q, float (*acc)[4]) {
#pragma unroll
  for (int w = 0; w < 4; ++w) {
    lds_z(zv, zp + w * 8, zon);
#pragma unroll
    for (int q = 0; q < 2; ++q) {
      uint32_t a0, a1, a2, a3;
      if (BITS <= 3) {
        const uint32_t lw = (BITS == 3 && (w & 1)) ? lwB : lwA;
        // [lane*4 (| 0x80 for table B), level byte, 0x01, 0] = 0x10000 + byte*256 + lane*4
        const uint32_t s0 = 0x7604u | ((2u * q) << 4), s1 = 0x7604u | ((2u * q + 1u) << 4);
        a0 = lds_abs_v(prmt(Lg[w], lw, s0));
        a2 = lds_abs_v(prmt(Lg[w], lw, s1));
        a1 = lds_abs_v(prmt(Lq[w], lw, s0));
        a3 = lds_abs_v(prmt(Lq[w], lw, s1));
      } else {
        const uint32_t xg = x4(M2g, w, q, lwA), xq = x4(M2q, w, q, lwA);
        const uint32_t s0 = 0xD504u | ((2u * q) << 4), s1 = 0xF706u | ((2u * q + 1u) << 4);
        a0 = lds_rel_v(lut, prmt(Lg[w], xg, s0));
        a2 = lds_rel_v(lut, prmt(Lg[w], xg, s1));
        a1 = lds_rel_v(lut, prmt(Lq[w], xq, s0));
        a3 = lds_rel_v(lut, prmt(Lq[w], xq, s1));
      }
      mma16816(acc[q], a0, a1, a2, a3, q == 0 ? zv.x : zv.z, q == 0 ? zv.y : zv.w);
    }
  }
}

// butterflies over index bits [0, LG) of v[0, 2^LG)
template <int LG>
__device__ __forceinline__ void fwht_regs(float* v) {
#pragma unroll
  for (int h = 1; h < (1 << LG); h <<= 1)
#pragma unroll
    for (int e = 0; e < (1 << LG); ++e)
      if (!(e & h)) {
        const float a = v[e], b = v[e + h];
        v[e] = a + b;
        v[e + h] = a - b;
      }
}

}  // namespace sk
}  // namespace tp

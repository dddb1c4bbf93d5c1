// Device building blocks of the packed-TCQ decoder shared by the per-call
// GEMV (tp_gemv.cu) and the persistent decode engine (tp_engine.cu):
// weight staging (bulk copies + mbarriers), the pair table, the GF(2)
// trellis decode into level words, the MMA inner step and the warp FWHT.
#pragma once

#include "tp_common.cuh"

namespace tp {

// Bounded mbarrier wait: ~2^26 polls (seconds); the copies complete in
// microseconds, so running out means the hardware misbehaved.
constexpr unsigned kMaxPolls = 1u << 26;

template <int BITS>
struct LutCfg {
  static constexpr int kLutBytes = BITS == 4 ? 131072 : 65536;
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

// --- bulk-copy staging (TMA engine, no multicast) --------------------------
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ void mbar_init(uint64_t* bar, unsigned count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void fence_proxy_async() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}
// arrive + expect `bytes`, then copy global -> shared completing on `bar`
__device__ __forceinline__ void bulk_load(void* dst, const void* src, unsigned bytes, uint64_t* bar) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
               : "memory");
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}
// one arrival on `bar`
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
// non-blocking: true when the phase with `parity` has completed
__device__ __forceinline__ bool mbar_test(uint64_t* bar, unsigned parity) {
  uint32_t done;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}"
      : "=r"(done)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return done != 0;
}
// true when the phase with `parity` completed; false after kMaxPolls polls
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, unsigned parity) {
  const uint32_t a = smem_u32(bar);
  for (unsigned i = 0; i < kMaxPolls; ++i) {
    uint32_t done;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}"
        : "=r"(done)
        : "r"(a), "r"(parity)
        : "memory");
    if (done) return true;
  }
  return false;
}

__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" :::); }

// Pair table.  bits <= 3: entry e (byte of a level word) at byte offset
// e*256 + lane*4 holds half2(cb[lo(e)], cb[hi(e)]); nibble bits above the
// level width are ignored.  bits == 4: key k = m2lo<<7 | byte<<8 | m2hi<<16
// (+ lane*4) holds half2(cb[byte&15 | m2lo<<4], cb[byte>>4 | m2hi<<4]).
// The codebook (<= 32 fp16) sits one entry per lane and is read by shuffle;
// each warp instruction stores four 128-byte table rows.
template <int BITS>
__device__ __forceinline__ void build_lut(unsigned char* lut, uint32_t cbv, int warp, int lane, int nwarps) {
  const int row = lane >> 3, col = lane & 7;
  constexpr int kEntries = BITS <= 3 ? 256 : 1024;
  for (int e0 = warp * 4; e0 < kEntries; e0 += nwarps * 4) {
    const int e = e0 + row;
    uint32_t lo, hi;
    int off;
    if (BITS <= 3) {
      constexpr unsigned lmask = (1u << (BITS + 1)) - 1u;
      lo = __shfl_sync(0xffffffffu, cbv, e & 15 & lmask);
      hi = __shfl_sync(0xffffffffu, cbv, (e >> 4) & lmask);
      off = e * 256;
    } else {
      const int byte = e & 255, m2lo = (e >> 8) & 1, m2hi = e >> 9;
      lo = __shfl_sync(0xffffffffu, cbv, (byte & 15) | (m2lo << 4));
      hi = __shfl_sync(0xffffffffu, cbv, (byte >> 4) | (m2hi << 4));
      off = (m2lo << 7) | (byte << 8) | (m2hi << 16);
    }
    const uint32_t v = lo | (hi << 16);
    *reinterpret_cast<uint4*>(lut + off + col * 16) = make_uint4(v, v, v, v);
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

// pair-table lookup at an absolute shared-window address
__device__ __forceinline__ uint32_t lds_abs(uint32_t addr) {
  uint32_t v;
  asm("ld.shared.b32 %0, [%1];" : "=r"(v) : "r"(addr));
  return v;
}

// ABS (bits <= 3 only): the pair table sits at shared-window address
// 0x10000 and `lanew` carries 0x10000 | lane*4, so one byte permute forms the
// final address (byte 2 from lanew) and no base add is needed.
template <int BITS, int S, int NT, bool ABS = false>
__device__ __forceinline__ void process_chunk(const unsigned char* lut, uint32_t lanew, const uint4* zq,
                                              uint32_t Pg, uint32_t Hg, uint32_t Pq, uint32_t Hq, uint32_t Mg0,
                                              uint32_t Mg1, uint32_t Mg2, uint32_t Mq0, uint32_t Mq1, uint32_t Mq2,
                                              const int* zoff, float (*acc)[NT][4]) {
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
    for (int nt = 0; nt < NT; ++nt) zv[nt] = zq[zoff[nt] + w];
#pragma unroll
    for (int q = 0; q < 2; ++q) {
      uint32_t a0, a1, a2, a3;
      if (BITS <= 3) {
        if (ABS) {
          // [lane*4, level byte, 0x01, 0] = 0x10000 + byte*256 + lane*4
          const uint32_t s0 = 0x7604u | ((2u * q) << 4), s1 = 0x7604u | ((2u * q + 1u) << 4);
          a0 = lds_abs(prmt(Lg[w], lanew, s0));
          a2 = lds_abs(prmt(Lg[w], lanew, s1));
          a1 = lds_abs(prmt(Lq[w], lanew, s0));
          a3 = lds_abs(prmt(Lq[w], lanew, s1));
        } else {
          // [lane*4, level byte, 0, 0] = byte*256 + lane*4
          const uint32_t s0 = 0x5504u | ((2u * q) << 4), s1 = 0x5504u | ((2u * q + 1u) << 4);
          a0 = lds32(lut, prmt(Lg[w], lanew, s0));
          a2 = lds32(lut, prmt(Lg[w], lanew, s1));
          a1 = lds32(lut, prmt(Lq[w], lanew, s0));
          a3 = lds32(lut, prmt(Lq[w], lanew, s1));
        }
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
        mma16816(acc[q][nt], a0, a1, a2, a3, b0, b1);
      }
    }
  }
}

// Warp-local butterflies over index bits [0, lg) of s[0, 2^lg): radix-8
// groups per lane, __syncwarp between groups (compact code; no CTA barrier).
__device__ __forceinline__ void fwht_warp(float* s, int lg, int lane) {
  for (int b0 = 0; b0 < lg; b0 += 3) {
    const int nb = lg - b0 < 3 ? lg - b0 : 3;
    const int G = 1 << nb;
    const int groups = (1 << lg) >> nb;
    for (int grp = lane; grp < groups; grp += 32) {
      const int lo = grp & ((1 << b0) - 1);
      const int base = ((grp >> b0) << (b0 + nb)) | lo;
      float v[8];
#pragma unroll
      for (int e = 0; e < 8; ++e)
        if (e < G) v[e] = s[base + (e << b0)];
#pragma unroll
      for (int h = 1; h < 8; h <<= 1) {
        if (h >= G) break;
#pragma unroll
        for (int e = 0; e < 8; ++e)
          if (e < G && !(e & h)) {
            const float x0 = v[e], x1 = v[e + h];
            v[e] = x0 + x1;
            v[e + h] = x0 - x1;
          }
      }
#pragma unroll
      for (int e = 0; e < 8; ++e)
        if (e < G) s[base + (e << b0)] = v[e];
    }
    __syncwarp();
  }
}

}  // namespace tp

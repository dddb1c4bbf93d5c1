// Stream-K packed-TCQ GEMV for batch 1..8 on sm_100a.
//
// y[b, r] = scale[r] * sum_c codebook[level(r, c)] * z[b, c]  (+ bias[r]),
// z = blockFWHT(x * rot_scale).
//
// Work split.  The weight units (16 rows x 256 columns, tile-major in the
// native stream) of a K-slice form one flat index space; every warp of the
// grid (one CTA of up to 32 warps per SM) takes an equal contiguous run of it,
// so all SMs stream the same number of bytes whatever the shape.  A run may
// start or end inside a row tile: the partial sums of such a tile go to the
// caller's workspace and the last warp to finish it (a per-tile counter) adds
// them in warp order (deterministic) and writes the outputs.
//
// Weight bytes go straight from HBM to registers: L2 bulk prefetches run 8-24
// units ahead of each warp and the next unit's 16-byte loads are in flight
// while the current one is decoded, so shared memory carries only the pair
// table and the rotated activations (its bandwidth is the decode's limit).
//
// Decode (per lane: rows g and g+8 of two 32-column chunks per unit): the
// GF(2) convolution of the path word with the trellis taps gives the two
// subset bit-planes; merged with the member words they form four "level
// words" of eight 4-bit levels; each byte of a level word (two levels) indexes
// a lane-replicated pair table of half2(codebook[lo], codebook[hi]) with one
// byte permute (the table sits at shared-window address 0x10000, so the
// permute forms the whole address); the pairs are the A fragments of
// m16n8k16 MMAs against the activations (batch = the n side), fp32 accumulate.
// For 3-bit payloads a second table (offset 128 bytes, nibble-rotated) lets
// two of the four level words skip their shifts.
#include "tp_gemv_sk.cuh"
#include "tp_rotate.cuh"
#include "tp_sk_core.cuh"

namespace tp {
namespace {

using namespace sk;

constexpr int kSkMaxWarps = 16;
constexpr int kSkThreads = kSkMaxWarps * 32;
#ifdef TP_SK_TRACE
// Development-only phase timeline (built only with -DTP_SK_TRACE, never in the
// shipped library): per CTA and warp 0/last, %globaltimer at each phase.
__device__ unsigned long long g_sk_trace[1024][8];
__device__ __forceinline__ void sk_trace(int k) {
  if ((threadIdx.x & 31) == 0 && (threadIdx.x == 0 || threadIdx.x == blockDim.x - 32) && blockIdx.x < 512) {
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    g_sk_trace[blockIdx.x * 2 + (threadIdx.x != 0)][k] = t;
  }
}
#else
__device__ __forceinline__ void sk_trace(int) {}
#endif

struct SkParams {
  const unsigned char* stream;
  const uint16_t* scales;
  const uint16_t* bias;
  const uint16_t* codebook;
  const void* x;
  const uint16_t* rot_scale;
  const uint4* zperm;  // pre-rotated [B][d_pad] fp16 (workspace) or null: rotate in-CTA
  void* y;
  float* partial;      // [row_tiles][kparts][maxc][16 * B]
  unsigned* counters;  // [row_tiles]
  unsigned* status;
  int x_dtype, y_dtype, B;
  int x_vec;           // x is fp16, 16-byte aligned, d % 8 == 0: 16-byte activation loads
  int rs_vec;          // rot_scale is 16-byte aligned
  int64_t n, d, d_pad;
  int units_k, row_tiles;
  int kparts, us;  // K-slices of `us` units (the last one may be shorter)
  int cps, wpc;    // CTAs per slice, warps per CTA
  int maxc;        // partial-sum slots per row tile and K-slice (warps one tile can span)
  SliceSplit split[2];  // [0]: slices 0..kparts-2, [1]: the last slice
  int block, lg_block;
  float norm;
  int rows_per_pass;  // fused rotation: batch rows per scratch pass
  int abs_layout;     // 1: offsets below are shared-window addresses
  uint32_t lut_off, z_off, scr_off, cb_off;
  uint32_t lo_addr, end_addr;  // abs: window [lo, end) must lie in the allocation; rel: end = bytes used
};

// ---------------------------------------------------------------------------
// in-CTA rotation: zs[b][c] = fp16(blockFWHT(x * rot_scale) / sqrt(block)) in
// the decoder's permuted pair order, columns [d, zcols) zero.
// ---------------------------------------------------------------------------
__device__ __forceinline__ void store_z(__half* zs, int zst, int row, int col, float v) {
  zs[row * zst + sk_zpos(col)] = __float2half_rn(v);
}

// Columns of 2^HB elements at stride 256 (index bits 8..8+HB) from the fp32
// scratch: the last stages of blocks of 2^(8+HB), then the output.
template <int HB>
__device__ __forceinline__ void column_pass(const SkParams& p, __half* zs, const float* scratch, int zcols, int b0,
                                            int rows) {
  const int d = static_cast<int>(p.d), blk = p.block, nb = d / blk;
  const int ncol = rows * nb * 256;
  for (int i = threadIdx.x; i < ncol; i += blockDim.x) {
    const int bi = i >> 8, c = i & 255;
    const float* src = scratch + bi * blk + c;
    float w[1 << HB];
#pragma unroll
    for (int k = 0; k < (1 << HB); ++k) w[k] = src[k * 256];
    fwht_regs<HB>(w);
    const int row = b0 + bi / nb, col0 = (bi - (bi / nb) * nb) * blk + c;
#pragma unroll
    for (int k = 0; k < (1 << HB); ++k) store_z(zs, zcols + kZPad, row, col0 + k * 256, w[k] * p.norm);
  }
}

// Hadamard blocks of 256..8192 columns: a warp transforms 256 consecutive
// columns in registers (8 per lane: bits 0-2 in place, bits 3-7 by shuffles);
// larger blocks finish with one column pass through the fp32 scratch.
__device__ void rotate_blocks(const SkParams& p, __half* zs, float* scratch, int zcols, uint4 rs0) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nwarps = blockDim.x >> 5;
  const int d = static_cast<int>(p.d), lg = p.lg_block, B = p.B;
  const int tpr = d >> 8;  // 256-column tasks per row
  for (int b0 = 0; b0 < B; b0 += p.rows_per_pass) {
    const int rows = min(p.rows_per_pass, B - b0);
    for (int k = warp; k < rows * tpr; k += nwarps) {
      const int rr = k / tpr, c0 = (k - rr * tpr) * 256 + lane * 8;
      const int64_t xo = (int64_t)(b0 + rr) * d + c0;
      float v[8];
      // the warp's first task uses the scales loaded before the dependency wait
      const uint4 rs = (b0 == 0 && k == warp) ? rs0 : *reinterpret_cast<const uint4*>(p.rot_scale + c0);
      const uint32_t rsw[4] = {rs.x, rs.y, rs.z, rs.w};
      if (p.x_vec) {
        const uint4 xv = *reinterpret_cast<const uint4*>(reinterpret_cast<const __half*>(p.x) + xo);
        const uint32_t xw[4] = {xv.x, xv.y, xv.z, xv.w};
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float2 xf = __half22float2(*reinterpret_cast<const __half2*>(&xw[e]));
          const float2 rf = __half22float2(*reinterpret_cast<const __half2*>(&rsw[e]));
          v[2 * e] = xf.x * rf.x;
          v[2 * e + 1] = xf.y * rf.y;
        }
      } else {
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float2 rf = __half22float2(*reinterpret_cast<const __half2*>(&rsw[e]));
          v[2 * e] = load_as_float(p.x, xo + 2 * e, p.x_dtype) * rf.x;
          v[2 * e + 1] = load_as_float(p.x, xo + 2 * e + 1, p.x_dtype) * rf.y;
        }
      }
      fwht_regs<3>(v);
#pragma unroll
      for (int sbit = 0; sbit < 5; ++sbit) {
        const float sg = (lane >> sbit) & 1 ? -1.f : 1.f;
#pragma unroll
        for (int e = 0; e < 8; ++e) v[e] = fmaf(sg, v[e], __shfl_xor_sync(0xffffffffu, v[e], 1 << sbit));
      }
      if (lg == 8) {
#pragma unroll
        for (int e = 0; e < 8; ++e) store_z(zs, zcols + kZPad, b0 + rr, c0 + e, v[e] * p.norm);
      } else {
        float4* dst = reinterpret_cast<float4*>(scratch + rr * d + c0);
        dst[0] = make_float4(v[0], v[1], v[2], v[3]);
        dst[1] = make_float4(v[4], v[5], v[6], v[7]);
      }
    }
    if (lg > 8) {
      __syncthreads();
      switch (lg - 8) {
        case 1: column_pass<1>(p, zs, scratch, zcols, b0, rows); break;
        case 2: column_pass<2>(p, zs, scratch, zcols, b0, rows); break;
        case 3: column_pass<3>(p, zs, scratch, zcols, b0, rows); break;
        case 4: column_pass<4>(p, zs, scratch, zcols, b0, rows); break;
        default: column_pass<5>(p, zs, scratch, zcols, b0, rows); break;
      }
      __syncthreads();
    }
  }
  for (int i = threadIdx.x; i < B * (zcols - d); i += blockDim.x) {
    const int b = i / (zcols - d);
    store_z(zs, zcols + kZPad, b, d + (i - b * (zcols - d)), 0.f);
  }
}

// Any block size (small or odd widths): fp32 staging and the shared-memory
// butterflies.
__device__ void rotate_generic(const SkParams& p, __half* zs, float* scratch, int zcols) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nwarps = blockDim.x >> 5;
  const int tid = threadIdx.x, nthreads = blockDim.x;
  const int d = static_cast<int>(p.d), blk = p.block, B = p.B;
  for (int b0 = 0; b0 < B; b0 += p.rows_per_pass) {
    const int rows = min(p.rows_per_pass, B - b0);
    for (int i = tid; i < rows * d; i += nthreads) {
      const int rr = i / d, c = i - rr * d;
      scratch[i] = load_as_float(p.x, (int64_t)(b0 + rr) * d + c, p.x_dtype) * h2f_bits(p.rot_scale[c]);
    }
    __syncthreads();
    if (blk <= 1024) {
      const int nb = rows * d / blk;
      for (int k = warp; k < nb; k += nwarps) fwht_warp(scratch + (size_t)k * blk, p.lg_block, lane);
      __syncthreads();
    } else {
      fwht_shared(scratch, rows * d, p.lg_block);
    }
    for (int i = tid; i < rows * d; i += nthreads) {
      const int rr = i / d, c = i - rr * d;
      store_z(zs, zcols + kZPad, b0 + rr, c, scratch[i] * p.norm);
    }
    __syncthreads();
  }
  for (int i = tid; i < B * (zcols - d); i += nthreads) {
    const int b = i / (zcols - d);
    store_z(zs, zcols + kZPad, b, d + (i - b * (zcols - d)), 0.f);
  }
}

template <int BITS, int S>
__global__ void __launch_bounds__(kSkThreads, 1) tcq_gemv_sk_kernel(SkParams p) {
  extern __shared__ __align__(128) unsigned char smem[];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int g = lane >> 2, t = lane & 3;
  const int nthreads = blockDim.x, nwarps = nthreads >> 5;

  // ---- shared-memory layout check (uniform across the CTA) ----
  const uint32_t base = smem_u32(smem);
  uint32_t dsz;
  asm volatile("mov.u32 %0, %%dynamic_smem_size;" : "=r"(dsz));
  const bool layout_ok =
      p.abs_layout ? (base <= p.lo_addr && base + dsz >= p.end_addr) : (dsz >= p.end_addr);
  if (!layout_ok) {
    if (tid == 0) atomicOr(p.status, kStatusLayout);
    return;
  }
  auto at = [&](uint32_t off) { return p.abs_layout ? smem + (off - base) : smem + off; };
  unsigned char* lut = at(p.lut_off);
  __half* zs = reinterpret_cast<__half*>(at(p.z_off));
  float* scratch = reinterpret_cast<float*>(at(p.scr_off));
  uint32_t* cbs = reinterpret_cast<uint32_t*>(at(p.cb_off));
  sk_trace(0);
  // one warp fetches the codebook (<= 32 fp16 levels) for the whole CTA
  if (warp == 0) cbs[lane] = lane < (1 << (BITS + 1)) ? p.codebook[lane] : 0u;
  pdl_trigger();

  // ---- this warp's run of the slice's flat unit index space ----
  const int slice = blockIdx.x / p.cps;
  const int wl = (blockIdx.x - slice * p.cps) * p.wpc + warp;
  const int us0 = slice * p.us;
  const SliceSplit& sp = p.split[slice == p.kparts - 1 ? 1 : 0];
  const int Us = sp.us;
  const int j0 = sp.start(wl), j1 = sp.start(wl + 1);
  constexpr unsigned UB = 512u * BITS;  // bytes per unit
  auto unit_ptr = [&](int rt_, int ul_) {
    return p.stream + ((int64_t)rt_ * p.units_k + us0 + ul_) * UB;
  };
  // L2 bulk prefetch of units [x0, x0 + 16) of the run, one per lane
  auto prefetch16 = [&](int x0) {
    const int x = x0 + lane;
    if (lane < 16 && x < j1) {
      const int r = sp.row_tile(x);
      prefetch_l2(unit_ptr(r, x - r * Us), UB);
    }
  };

  // ---- prologue independent of the previous kernel: start the weights ----
  int rt = sp.row_tile(j0), ul = j0 - rt * Us;
  prefetch16(j0);
  uint4 wa[BITS];  // the current unit's words of this lane
  // this lane's chunk-(4+t) path words of the unit before the current one
  // (zero before a row's first column: the trellis starts in state 0)
  uint32_t hg = 0u, hq = 0u, hng = 0u, hnq = 0u;
  if (j0 < j1) {
    const uint4* src = reinterpret_cast<const uint4*>(unit_ptr(rt, ul)) + lane * BITS;
#pragma unroll
    for (int k = 0; k < BITS; ++k) wa[k] = ldg_stream(src + k);
    if (us0 + ul > 0) {
      const uint4 pv = ldg_stream(reinterpret_cast<const uint4*>(unit_ptr(rt, ul - 1)) + lane * BITS);
      hg = pv.z;
      hq = pv.w;
    }
  }
  // rotation scales of this warp's first rotation task (independent of x)
  const bool fast_rot = p.zperm == nullptr && p.lg_block >= 8 && p.lg_block <= 13 && p.rs_vec;
  uint4 rs0 = make_uint4(0u, 0u, 0u, 0u);
  if (fast_rot && warp < p.B * (static_cast<int>(p.d) >> 8))
    rs0 = *reinterpret_cast<const uint4*>(p.rot_scale + (warp % (static_cast<int>(p.d) >> 8)) * 256 + lane * 8);
  __syncthreads();  // codebook in shared memory
  build_tables<BITS>(lut, cbs[lane], warp, lane, nwarps);
  sk_trace(1);

  // ---- activations: wait for x's producer, then rotate (or copy) them ----
  pdl_wait();
  sk_trace(2);
  const int B = p.B;
  const int zcols = Us * kUnitCols;  // activation columns held in shared memory
  const int zst = zcols + kZPad;     // row stride (halves)
  if (p.zperm) {
    const int q = zcols / 8;
    for (int i = tid; i < B * q; i += nthreads) {
      const int b = i / q, r = i - b * q;
      reinterpret_cast<uint4*>(zs + b * zst)[r] = p.zperm[(int64_t)b * (p.d_pad / 8) + (int64_t)us0 * 32 + r];
    }
  } else if (fast_rot) {
    rotate_blocks(p, zs, scratch, zcols, rs0);
  } else {
    rotate_generic(p, zs, scratch, zcols);
  }
  for (int i = tid; i < zcols / 8; i += nthreads) reinterpret_cast<uint4*>(zs + B * zst)[i] = make_uint4(0u, 0u, 0u, 0u);
  __syncthreads();
  sk_trace(3);

  // ---- decode + MMA over the run ----
  float acc[2][4];
#pragma unroll
  for (int q = 0; q < 2; ++q) acc[q][0] = acc[q][1] = acc[q][2] = acc[q][3] = 0.f;
  const uint32_t lwA = BITS <= 3 ? (kLutAbs | (uint32_t)lane * 4u) : (uint32_t)lane * 4u * 0x10001u;
  const uint32_t lwB = lwA | 0x80u;
  // lanes past the batch read row B of zs, which is all zero
  const uint4* zp = reinterpret_cast<const uint4*>(zs + min(g, B) * zst) + t + ul * 32;
  const int src = (lane & ~3) | ((t + 3) & 3);
  // stream bytes skipped at a row-tile change: the other K-slices' units
  const int64_t row_skip = (int64_t)(p.units_k - Us) * UB;
  const unsigned char* wp = unit_ptr(rt, ul) + lane * BITS * 16;  // this lane's words of the current unit

  // Partial sums of row tile `frt`: written out directly when this warp owns
  // the whole tile, otherwise into the tile's slot for this warp in the
  // workspace; the last of the tile's warps adds the slots in order.
  auto flush = [&](int frt) {
    float v[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) v[e] = acc[0][e] + acc[1][e];
#pragma unroll
    for (int q = 0; q < 2; ++q) acc[q][0] = acc[q][1] = acc[q][2] = acc[q][3] = 0.f;
    const bool solo = p.kparts == 1 && j0 <= frt * Us && (frt + 1) * Us <= j1;
    if (!solo) {
      const int k = wl - sp.warp_of(frt * Us);  // this warp's rank among the tile's warps in the slice
      float* pc = p.partial + ((int64_t)(frt * p.kparts + slice) * p.maxc + k) * 16 * B;
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int col = 2 * t + (e & 1), row = g + 8 * (e >> 1);
        if (col < B) __stcg(pc + row * B + col, v[e]);
      }
      __syncwarp();
      const SliceSplit& s0 = p.split[0];
      const SliceSplit& s1 = p.split[1];
      const int c0 = s0.warp_of((frt + 1) * s0.us - 1) - s0.warp_of(frt * s0.us) + 1;
      const int c1 = s1.warp_of((frt + 1) * s1.us - 1) - s1.warp_of(frt * s1.us) + 1;
      // one acq_rel add by lane 0 after the warp barrier: publishes the
      // warp's partials (release, cumulative over the warp's stores) and, for
      // the last warp of the tile, orders its reads of the others' (acquire)
      unsigned last = 0u;
      if (lane == 0) {
        unsigned old;
        asm volatile("atom.acq_rel.gpu.global.add.u32 %0, [%1], 1;" : "=r"(old) : "l"(&p.counters[frt]) : "memory");
        last = old == (unsigned)((p.kparts - 1) * c0 + c1 - 1) ? 1u : 0u;
      }
      last = __shfl_sync(0xffffffffu, last, 0);
      if (!last) return;
      __syncwarp();
#pragma unroll
      for (int e = 0; e < 4; ++e) v[e] = 0.f;
      for (int sl = 0; sl < p.kparts; ++sl) {
        const int cnt = sl == p.kparts - 1 ? c1 : c0;
        const float* pp = p.partial + (int64_t)(frt * p.kparts + sl) * p.maxc * 16 * B;
        for (int kk = 0; kk < cnt; ++kk, pp += 16 * B) {
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const int col = 2 * t + (e & 1), row = g + 8 * (e >> 1);
            if (col < B) v[e] += __ldcg(pp + row * B + col);
          }
        }
      }
      if (lane == 0) p.counters[frt] = 0u;
    }
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const int col = 2 * t + (e & 1);
      const int64_t row = (int64_t)frt * kTileRows + g + 8 * (e >> 1);
      if (col < B && row < p.n) {
        float o = v[e] * h2f_bits(p.scales[row]);
        if (p.bias) o += h2f_bits(p.bias[row]);
        store_from_float(p.y, (int64_t)col * p.n + row, p.y_dtype, o);
      }
    }
  };

  // Per unit: level words of both chunks from `cur`, then the next unit's
  // loads into `cur` (in flight during this unit's lookups), then the
  // lookups and MMAs.
  uint4 zv = make_uint4(0u, 0u, 0u, 0u);
  const bool zon = g < B;
  for (int j = j0; j < j1; ++j) {
    const bool row_end = ul + 1 == Us;
    const bool more = j + 1 < j1;
    const uint32_t P0g = wa[0].x, P0q = wa[0].y, P1g = wa[0].z, P1q = wa[0].w;
    // halos: the neighbour lane's chunk (t-1); lane t=0 takes lane 3's
    const uint32_t H0g = __shfl_sync(0xffffffffu, t == 3 ? hg : P0g, src);
    const uint32_t H0q = __shfl_sync(0xffffffffu, t == 3 ? hq : P0q, src);
    const uint32_t H1g = __shfl_sync(0xffffffffu, t == 3 ? P0g : P1g, src);
    const uint32_t H1q = __shfl_sync(0xffffffffu, t == 3 ? P0q : P1q, src);
    uint32_t m0[4] = {0u, 0u, 0u, 0u}, m1[4] = {0u, 0u, 0u, 0u}, m2[4] = {0u, 0u, 0u, 0u};
    if (BITS >= 2) m0[0] = wa[1].x, m0[1] = wa[1].y, m0[2] = wa[1].z, m0[3] = wa[1].w;
    if (BITS >= 3) m1[0] = wa[2].x, m1[1] = wa[2].y, m1[2] = wa[2].z, m1[3] = wa[2].w;
    if (BITS >= 4) m2[0] = wa[3].x, m2[1] = wa[3].y, m2[2] = wa[3].z, m2[3] = wa[3].w;
    uint32_t L0g[4], L0q[4], L1g[4], L1q[4];
    level_words_sk<BITS, S>(P0g, H0g, m0[0], m1[0], L0g);
    level_words_sk<BITS, S>(P0q, H0q, m0[1], m1[1], L0q);
    level_words_sk<BITS, S>(P1g, H1g, m0[2], m1[2], L1g);
    level_words_sk<BITS, S>(P1q, H1q, m0[3], m1[3], L1q);
    hg = P1g;
    hq = P1q;
    const unsigned char* np = wp + UB + (row_end ? row_skip : 0);
    if (more) {
#pragma unroll
      for (int k = 0; k < BITS; ++k) wa[k] = ldg_stream(reinterpret_cast<const uint4*>(np) + k);
      if (row_end && us0 > 0) {  // a later K-slice: the new row tile's halo is the slice's left neighbour
        const uint4 pv = ldg_stream(reinterpret_cast<const uint4*>(np - UB));
        hng = pv.z;
        hnq = pv.w;
      }
    }
    if (((j - j0) & 15) == 8) prefetch16(j + 8);
    sk_mma_chunk<BITS>(lwA, lwB, lut, zp, zon, zv, L0g, L0q, m2[0], m2[1], acc);
    sk_mma_chunk<BITS>(lwA, lwB, lut, zp + 4, zon, zv, L1g, L1q, m2[2], m2[3], acc);
    zp += 32;
    wp = np;
    if (row_end || !more) flush(rt);
    if (row_end) {
      hg = hng;
      hq = hnq;
      zp -= Us * 32;
      ++rt;
      ul = 0;
    } else {
      ++ul;
    }
  }
  sk_trace(4);
}

// ---------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------
struct SkPlan {
  int kparts = 0, us = 0, cps = 0, wpc = 0, maxc = 0;
  int split_us[2] = {0, 0}, split_r[2] = {0, 0}, split_rem[2] = {0, 0};
  bool fused = false;
  int rows_per_pass = 1;
  int abs_layout = 0;
  uint32_t lut_off = 0, z_off = 0, scr_off = 0, cb_off = 0, lo_addr = 0, end_addr = 0;
  size_t dyn = 0;
  int64_t ws_z = 0, ws_part = 0;
};

int device_smem_info(int* reserved, int* optin) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return -1;
  if (cudaDeviceGetAttribute(reserved, cudaDevAttrReservedSharedMemoryPerBlock, dev) != cudaSuccess) return -1;
  if (cudaDeviceGetAttribute(optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev) != cudaSuccess) return -1;
  return 0;
}

// Returns false when no layout fits (the caller falls back).
bool make_sk_plan(int64_t B, int64_t n, int64_t d, int bits, int64_t block, int sms, int reserved, int optin,
                  SkPlan& pl) {
  if (B < 1 || B > kSkMaxBatch || bits < 1 || bits > 4) return false;
  const int64_t n_pad = pad_to(n, kTileRows), d_pad = pad_to(d, kUnitCols);
  const int64_t row_tiles = n_pad / kTileRows;
  const int U = static_cast<int>(d_pad / kUnitCols);
  if (row_tiles > kMaxRowBlocks || row_tiles * U >= (int64_t(1) << 30)) return false;
  const uint32_t base = static_cast<uint32_t>((reserved + 127) / 128 * 128);  // no static shared memory
  const uint32_t lut_bytes = bits == 4 ? 131072u : 65536u;
  // regions available around the pair table
  int64_t cap_a, cap_b;  // bits <= 3: before / after the table; bits 4: after the table (cap_b unused)
  if (bits <= 3) {
    cap_a = (int64_t)kLutAbs - base;
    cap_b = (int64_t)base + optin - (kLutAbs + lut_bytes);
  } else {
    cap_a = (int64_t)optin - lut_bytes;
    cap_b = 0;
  }
  if (cap_a < 0) cap_a = 0;
  if (cap_b < 0) cap_b = 0;
  const int64_t zmax = std::max(cap_a, cap_b) - 256;
  int kparts = 1;
  // activations of one slice: B rows plus an all-zero row read by the lanes past the batch
  while (kparts <= U && (B + 1) * ((int64_t)((U + kparts - 1) / kparts) * kUnitCols + kZPad) * 2 > zmax) ++kparts;
  if (kparts > U) return false;
  const int us = (U + kparts - 1) / kparts;
  kparts = (U + us - 1) / us;  // no empty slice
  // plus 128 bytes for the codebook
  const int64_t zbytes = ((B + 1) * ((int64_t)us * kUnitCols + kZPad) * 2 + 127) / 128 * 128 + 128;
  // Place z, then (fused rotation) the fp32 scratch.  bits <= 3: region a
  // grows down from the table ([kLutAbs - used_a, kLutAbs)), region b starts
  // after it; bits 4: one region after the table.
  int64_t used_a = 0, used_b = 0, z_at = 0, s_at = 0;
  const bool z_in_a = bits == 4 || zbytes <= cap_a - 256;
  (z_in_a ? used_a : used_b) = zbytes;
  bool s_in_a = true;
  pl.fused = false;
  pl.rows_per_pass = 1;
  if (kparts == 1 && block <= 8192) {
    const int64_t room_a = cap_a - used_a - 256, room_b = bits == 4 ? 0 : cap_b - used_b - 256;
    const int64_t room = std::max(room_a, room_b), per_row = d * 4;
    if (room >= per_row) {
      pl.fused = true;
      pl.rows_per_pass = static_cast<int>(std::min<int64_t>(B, room / per_row));
      const int64_t sb = (pl.rows_per_pass * per_row + 127) / 128 * 128;
      s_in_a = room_a >= room_b;
      s_at = s_in_a ? used_a : used_b;
      (s_in_a ? used_a : used_b) += sb;
    }
  }
  if (bits <= 3) {
    pl.abs_layout = 1;
    pl.lut_off = kLutAbs;
    const uint32_t a0 = kLutAbs - static_cast<uint32_t>(used_a), b0 = kLutAbs + lut_bytes;
    pl.z_off = z_in_a ? a0 + static_cast<uint32_t>(z_at) : b0 + static_cast<uint32_t>(z_at);
    pl.scr_off = s_in_a ? a0 + static_cast<uint32_t>(s_at) : b0 + static_cast<uint32_t>(s_at);
    pl.cb_off = pl.z_off + static_cast<uint32_t>(zbytes - 128);
    pl.lo_addr = a0;
    pl.end_addr = b0 + static_cast<uint32_t>(used_b);
    if (pl.lo_addr < base) return false;
    pl.dyn = pl.end_addr - base;
  } else {
    pl.abs_layout = 0;
    pl.lut_off = 0;
    pl.z_off = lut_bytes + static_cast<uint32_t>(z_at);
    pl.scr_off = lut_bytes + static_cast<uint32_t>(s_at);
    pl.cb_off = pl.z_off + static_cast<uint32_t>(zbytes - 128);
    pl.lo_addr = 0;
    pl.end_addr = lut_bytes + static_cast<uint32_t>(used_a);
    pl.dyn = pl.end_addr;
  }
  if (pl.dyn > static_cast<size_t>(optin)) return false;
  // grid: one CTA per SM, warps split evenly over the flat unit space
  const int64_t T_min = row_tiles * (U - (int64_t)(kparts - 1) * us);
  int cps = std::max(1, sms / kparts);
  int wpc = static_cast<int>(std::min<int64_t>(kSkMaxWarps, T_min / cps));
  if (wpc < 1) {
    wpc = 1;
    cps = static_cast<int>(T_min);
  }
  pl.kparts = kparts;
  pl.us = us;
  pl.cps = cps;
  pl.wpc = wpc;
  pl.ws_z = pl.fused ? 0 : align256(B * d_pad * 2);
  const int64_t W = (int64_t)cps * wpc;
  pl.maxc = 0;
  for (int k = 0; k < 2; ++k) {
    // [0]: the regular slices, [1]: the last one
    const int64_t su = k == 0 ? us : U - (int64_t)(kparts - 1) * us;
    const int64_t T = row_tiles * su;
    pl.split_us[k] = static_cast<int>(su);
    pl.split_r[k] = static_cast<int>(T / W);
    pl.split_rem[k] = static_cast<int>(T % W);
    // warps (runs of >= r units) that one row tile of su units can span
    const int64_t r = T / W;
    pl.maxc = std::max<int>(pl.maxc, static_cast<int>((su + r - 1) / r + 1));
  }
  pl.ws_part = align256(row_tiles * kparts * pl.maxc * 16 * B * 4);
  return true;
}

template <int BITS, int S>
tp_status launch_sk_t(const SkParams& p, const SkPlan& pl, cudaStream_t stream) {
  auto kern = tcq_gemv_sk_kernel<BITS, S>;
  static int smem_set[64] = {0};
  if (tp_status s = ensure_smem(kern, pl.dyn, smem_set, "cudaFuncSetAttribute(gemv_sk)")) return s;
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(static_cast<unsigned>(pl.kparts * pl.cps), 1, 1);
  cfg.blockDim = dim3(static_cast<unsigned>(pl.wpc * 32), 1, 1);
  cfg.dynamicSmemBytes = pl.dyn;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  TP_CUDA_TRY(cudaLaunchKernelEx(&cfg, kern, p), "tcq_gemv_sk_kernel launch");
  return check_launch("tcq_gemv_sk_kernel");
}

template <int BITS>
tp_status launch_sk_s(const SkParams& p, const SkPlan& pl, int n_states, cudaStream_t stream) {
  switch (n_states) {
    case 4: return launch_sk_t<BITS, 4>(p, pl, stream);
    case 8: return launch_sk_t<BITS, 8>(p, pl, stream);
    case 16: return launch_sk_t<BITS, 16>(p, pl, stream);
    default: return launch_sk_t<BITS, 64>(p, pl, stream);
  }
}

bool sk_plan_for(int64_t B, int64_t n, int64_t d, int bits, int64_t block, SkPlan& pl) {
  int reserved = 0, optin = 0;
  if (device_smem_info(&reserved, &optin)) {
    reserved = 1024;
    optin = 227 * 1024;
  }
  return make_sk_plan(B, n, d, bits, block, sm_count(), reserved, optin, pl);
}

}  // namespace

int64_t sk_workspace_extra(int64_t B, int64_t n, int64_t d, int bits, int64_t block) {
  SkPlan pl;
  if (!sk_plan_for(B, n, d, bits, block, pl)) return -1;
  // bound over the rotation choice: the pre-rotated activations are counted
  return align256(B * pad_to(d, kUnitCols) * 2) + pl.ws_part;
}

tp_status sk_gemv(const SkRequest& r, cudaStream_t stream) {
  SkPlan pl;
  if (!sk_plan_for(r.B, r.n, r.d, r.bits, r.block, pl))
    return fail(TP_ERR_UNSUPPORTED, "tp_tcq_gemv: no stream-K layout for B=%d n=%lld d=%lld", r.B, (long long)r.n,
                (long long)r.d);
  const int64_t d_pad = pad_to(r.d, kUnitCols), n_pad = pad_to(r.n, kTileRows);
  unsigned char* ws = r.workspace;
  const int64_t zreg = align256(r.B * d_pad * 2);
  int lg = 0;
  while ((int64_t(1) << lg) < r.block) ++lg;
  SkParams p{};
  if (!pl.fused) {
    RotateArgs ra{};
    ra.x = r.x;
    ra.x_dtype = r.x_dtype;
    ra.scale = r.rot_scale;
    ra.z = ws + kCounterBytes;
    ra.z_dtype = TP_F16;
    ra.d = r.d;
    ra.d_pad = d_pad;
    ra.block = r.block;
    ra.mode = 3;
    if (tp_status s = launch_rotate(ra, r.B, stream)) return s;
    p.zperm = reinterpret_cast<const uint4*>(ws + kCounterBytes);
  }
  p.stream = r.stream;
  p.scales = r.scales;
  p.bias = r.bias;
  p.codebook = r.codebook;
  p.x = r.x;
  p.rot_scale = r.rot_scale;
  p.y = r.y;
  p.partial = reinterpret_cast<float*>(ws + kCounterBytes + zreg);
  p.counters = reinterpret_cast<unsigned*>(ws);
  p.status = reinterpret_cast<unsigned*>(ws + kStatusOff);
  p.x_dtype = r.x_dtype;
  p.y_dtype = r.y_dtype;
  p.B = r.B;
  p.n = r.n;
  p.d = r.d;
  p.d_pad = d_pad;
  p.units_k = static_cast<int>(d_pad / kUnitCols);
  p.row_tiles = static_cast<int>(n_pad / kTileRows);
  p.kparts = pl.kparts;
  p.us = pl.us;
  p.cps = pl.cps;
  p.wpc = pl.wpc;
  p.maxc = pl.maxc;
  p.rs_vec = aligned(r.rot_scale, 16);
  p.cb_off = pl.cb_off;
  for (int k = 0; k < 2; ++k) {
    p.split[k].us = pl.split_us[k];
    p.split[k].r = pl.split_r[k];
    p.split[k].rem = pl.split_rem[k];
    p.split[k].nw = pl.cps * pl.wpc;
    p.split[k].div_us = make_fastdiv(static_cast<uint32_t>(pl.split_us[k]));
    p.split[k].div_r = make_fastdiv(static_cast<uint32_t>(pl.split_r[k]));
    p.split[k].div_r1 = make_fastdiv(static_cast<uint32_t>(pl.split_r[k] + 1));
  }
  p.x_vec = r.x_dtype == TP_F16 && aligned(r.x, 16) && r.d % 8 == 0;
  p.block = static_cast<int>(r.block);
  p.lg_block = lg;
  p.norm = static_cast<float>(1.0 / __builtin_sqrt(static_cast<double>(r.block)));
  p.rows_per_pass = pl.rows_per_pass;
  p.abs_layout = pl.abs_layout;
  p.lut_off = pl.lut_off;
  p.z_off = pl.z_off;
  p.scr_off = pl.scr_off;
  p.lo_addr = pl.lo_addr;
  p.end_addr = pl.end_addr;
  if (getenv("TP_DEBUG_PLAN") && *getenv("TP_DEBUG_PLAN") != '0')
    fprintf(stderr, "tp_tcq_gemv[sk] n=%lld d=%lld B=%d bits=%d: kparts=%d us=%d cps=%d wpc=%d fused=%d rpp=%d "
            "dyn=%zu lut=%#x z=%#x scr=%#x lo=%#x end=%#x\n", (long long)r.n, (long long)r.d, r.B, r.bits,
            pl.kparts, pl.us, pl.cps, pl.wpc, (int)pl.fused, pl.rows_per_pass, pl.dyn, pl.lut_off, pl.z_off,
            pl.scr_off, pl.lo_addr, pl.end_addr);
  switch (r.bits) {
    case 1: return launch_sk_s<1>(p, pl, r.n_states, stream);
    case 2: return launch_sk_s<2>(p, pl, r.n_states, stream);
    case 3: return launch_sk_s<3>(p, pl, r.n_states, stream);
    default: return launch_sk_s<4>(p, pl, r.n_states, stream);
  }
}

}  // namespace tp

#ifdef TP_SK_TRACE
extern "C" TP_API int tp_sk_trace_read(unsigned long long* host) {
  return (int)cudaMemcpyFromSymbol(host, tp::g_sk_trace, sizeof(tp::g_sk_trace));
}
#endif

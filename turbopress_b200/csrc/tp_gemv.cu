// Fused rotate + packed-TCQ GEMV / skinny GEMM for batch 1..32 on sm_100a.
//
// y[b, r] = scale[r] * sum_c codebook[level(r, c)] * z[b, c]  (+ bias[r]),
// z = blockFWHT(x * rot_scale) computed inside the kernel.
//
// One launch per linear.  CTA = 8 warps = RT row tiles (16 rows each) x KW
// warps along K; a cluster of `ksplit` CTAs shares each row block's K range.
// Per CTA:
//   1. programmatic dependent launch: start weight loads (independent of the
//      previous kernel) and build the pair table, then griddepcontrol.wait;
//   2. rotate the CTA's K-slice of x (fp32 block FWHT in shared memory) into
//      fp16 activations in the decoder's permuted pair order;
//   3. per warp: coalesced 16-byte non-allocating loads of the true-rate
//      stream (bits words per row per 32 columns), trellis halo by one warp
//      shuffle, register bit-slicing (GF(2) convolution of the path word ->
//      subset planes -> four "level words" of 8 nibbles), one byte permute
//      per weight pair to address a lane-replicated pair table holding
//      half2(codebook[lo], codebook[hi]) (32 lanes, 32 banks), and the pairs
//      as A fragments of a warp-level m16n8k16 MMA with fp32 accumulation
//      (one MMA per 256 weights);
//   4. reduce KW warps in shared memory, then the cluster's CTAs through
//      distributed shared memory (deterministic order), scale/bias/cast.
//      Above 8 K-splits the partials go through the caller's workspace and
//      the last CTA of a row block reduces them.
//
// 4-bit payloads (5-bit levels) use a 1024-entry pair table: the two fifth
// level bits ride in address bits 7 and 16 via a second permute source.
#include <cooperative_groups.h>

#include <algorithm>
#include <cstdlib>
#include <mutex>

#include "tp_decode.cuh"
#include "tp_gemv_sk.cuh"
#include "tp_rotate.cuh"

namespace cg = cooperative_groups;
using namespace tp;

namespace {

constexpr int kMaxBatchPerLaunch = 32;  // 4 n-tiles of the m16n8k16 MMA
constexpr int kWarps = 8;               // warps per CTA (RT * KW)
constexpr int kThreads = kWarps * 32;
constexpr int kMaxCluster = 8;          // portable cluster size
constexpr int kMaxFusedBlock = 8192;    // Hadamard blocks rotated in-kernel
constexpr int kScratchFloats = 8192;    // fp32 FWHT scratch (32 KB)
constexpr int kMaxSlots = 16;           // weight units in flight per warp
// dynamic shared memory per CTA (227 KB opt-in minus the static part)
constexpr size_t kMaxDynSmem = 227u * 1024u - 2048u;
// The workspace starts with a fixed-size block of split-K counters (and the
// status word, tp_gemv_sk.cuh), so calls of different shapes sharing one
// workspace never overlap each other's counters with their activation or
// partial-sum regions.

template <int BITS>
struct Cfg {
  static constexpr int kLutBytes = BITS == 4 ? 131072 : 65536;
};


struct GemvParams {
  const uint4* stream;
  const uint16_t* scales;
  const uint16_t* bias;
  const uint16_t* codebook;
  const void* x;             // [B][d] activations (x_dtype)
  const uint16_t* rot_scale;
  const uint4* zperm;        // pre-rotated [B][d_pad] fp16 (only when block > kMaxFusedBlock)
  void* y;
  float* partial;            // [ksplit][B][n_pad] (global split-K only)
  unsigned* counters;        // [row_blocks]      (global split-K only)
  unsigned* status;          // workspace status word (kStatus* bits)
  int x_dtype, y_dtype;
  int B;
  int64_t n, n_pad, d, d_pad;
  int units_k;
  int block, lg_block;
  float norm;
  int rt;        // row tiles per CTA
  int kw;        // warps along K per CTA (rt * kw == kWarps)
  int ksplit;    // CTAs along K
  int cluster;   // 1: reduce the ksplit CTAs through DSMEM
  int zrows_per_pass;
  int slots;     // weight units staged per warp (ring depth)
  uint32_t w_off, z_off, scratch_off, red_off;  // shared-memory carve-up (bytes)
};

#ifdef TP_TRACE
// Development-only phase timeline (built only with -DTP_TRACE, never in the
// shipped library): thread 0 of each CTA stamps %globaltimer per phase.
static __device__ unsigned long long g_trace[8192][16];
__device__ __forceinline__ void trace(int k) {
  if (threadIdx.x == 0) {
    const unsigned cta = blockIdx.x * gridDim.y + blockIdx.y;
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    if (cta < 8192) g_trace[cta][k] = t;
  }
}
// record the first layout / bounds violation of a CTA in slots 12..15
__device__ __forceinline__ void trace_bad(unsigned code, unsigned long long a, unsigned long long b) {
  const unsigned cta = blockIdx.x * gridDim.y + blockIdx.y;
  if (cta < 8192 && atomicCAS(&g_trace[cta][12], 0ull, (unsigned long long)code) == 0ull) {
    g_trace[cta][13] = a;
    g_trace[cta][14] = b;
    g_trace[cta][15] = threadIdx.x;
  }
}
__device__ __forceinline__ unsigned dyn_smem_size() {
  unsigned v;
  asm volatile("mov.u32 %0, %%dynamic_smem_size;" : "=r"(v));
  return v;
}
#define TP_CHECKED 1
#else
__device__ __forceinline__ void trace(int) {}
#define TP_CHECKED 0
#endif


// Rotated activations of the CTA's K-slice [c0, c0 + ncols) into zs
// ([B][ncols] fp16, permuted pair order inside each 32-column chunk), with
// columns >= d zeroed.  The covering Hadamard blocks of x * rot_scale are
// staged in fp32 scratch (rows in passes of zrows_per_pass); blocks of up to
// 1024 columns are transformed one per warp, larger ones by the whole CTA.
__device__ void rotate_slice(const GemvParams& p, int64_t c0, int ncols, __half* zs, float* scratch) {
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int64_t c1 = c0 + ncols;
  const int64_t vend = c1 < p.d ? c1 : p.d;  // valid columns end
  const int B = p.B;
  if (p.zperm) {  // pre-rotated by a separate launch (very large Hadamard blocks)
    const int q = ncols / 8;  // uint4 per row
    for (int i = tid; i < B * q; i += kThreads) {
      const int b = i / q, r = i - b * q;
      reinterpret_cast<uint4*>(zs)[i] = p.zperm[(int64_t)b * (p.d_pad / 8) + c0 / 8 + r];
    }
    return;
  }
  if (vend < c1) {  // zero the slice columns past d
    const int lc0 = static_cast<int>((vend > c0 ? vend : c0) - c0);
    for (int b = 0; b < B; ++b)
      for (int lc = lc0 + tid; lc < ncols; lc += kThreads)
        zs[b * ncols + (lc & ~31) + zperm_pos(lc & 31)] = __float2half_rn(0.f);
  }
  if (c0 >= p.d) return;
  const int64_t blk = p.block;
  const int64_t s0 = c0 / blk * blk;
  const int64_t s1 = (vend + blk - 1) / blk * blk;
  const int span = static_cast<int>(s1 - s0);
  for (int b0 = 0; b0 < B; b0 += p.zrows_per_pass) {
    const int rows = B - b0 < p.zrows_per_pass ? B - b0 : p.zrows_per_pass;
    for (int rr = 0; rr < rows; ++rr)
      for (int c = tid; c < span; c += kThreads)
        scratch[rr * span + c] =
            load_as_float(p.x, (int64_t)(b0 + rr) * p.d + s0 + c, p.x_dtype) * h2f_bits(p.rot_scale[s0 + c]);
    __syncthreads();
    trace(8);
    if (blk <= 1024) {
      const int nblocks = rows * span / static_cast<int>(blk);
      for (int k = warp; k < nblocks; k += kWarps) fwht_warp(scratch + (size_t)k * blk, p.lg_block, lane);
      __syncthreads();
    } else {
      fwht_shared(scratch, rows * span, p.lg_block);
    }
    trace(9);
    const int nvalid = static_cast<int>(vend - c0), soff = static_cast<int>(c0 - s0);
    for (int rr = 0; rr < rows; ++rr)
      for (int lc = tid; lc < nvalid; lc += kThreads)
        zs[(b0 + rr) * ncols + (lc & ~31) + zperm_pos(lc & 31)] =
            __float2half_rn(scratch[rr * span + soff + lc] * p.norm);
    __syncthreads();
  }
}

template <int BITS, int S, int NT>
__global__ void __launch_bounds__(kThreads, 2) tcq_gemv_kernel(GemvParams p) {
  extern __shared__ __align__(128) unsigned char smem[];
  unsigned char* lut = smem;
  __half* zs = reinterpret_cast<__half*>(smem + p.z_off);
  float* scratch = reinterpret_cast<float*>(smem + p.scratch_off);
  float* red = reinterpret_cast<float*>(smem + p.red_off);
  __shared__ unsigned s_last;

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int g = lane >> 2, t = lane & 3;
  const int rtl = warp % p.rt, kwi = warp / p.rt;
  const int ks = blockIdx.y;
  const int u0 = static_cast<int>((int64_t)ks * p.units_k / p.ksplit);
  const int u1 = static_cast<int>((int64_t)(ks + 1) * p.units_k / p.ksplit);
  const int U = u1 - u0;
  const int wu0 = u0 + kwi * U / p.kw, wu1 = u0 + (kwi + 1) * U / p.kw;
  const int nunits = wu1 - wu0;
  const int64_t rt = (int64_t)blockIdx.x * p.rt + rtl;
  const bool active = rt * kTileRows < p.n_pad;

  trace(0);
  // codebook entry of this lane (<= 32 levels), fetched before anything else
  const uint32_t cbv = lane < (1 << (BITS + 1)) ? p.codebook[lane] : 0u;
  // the next kernel in the stream may start its own prologue now; it waits
  // for this grid's completion before touching our outputs
  pdl_trigger();

  // ---- prologue independent of the previous kernel ----
  // Each warp's weights (row tile rt, units [wu0, wu1)) are one contiguous
  // run of the stream; lane 0 streams it unit by unit into the warp's ring
  // of `slots` shared-memory units with bulk copies, all in flight now.
  __shared__ __align__(8) uint64_t s_bar[kWarps][kMaxSlots];
  __shared__ int s_fail;
  constexpr unsigned kUnitBytes = 32u * 16u * BITS;
  unsigned char* ring = smem + p.w_off + (size_t)warp * p.slots * kUnitBytes;
  const unsigned char* wsrc =
      reinterpret_cast<const unsigned char*>(p.stream) + ((size_t)(rt * p.units_k + wu0)) * kUnitBytes;
  const bool staged = active && nunits > 0;
  if (tid == 0) s_fail = 0;
  if (staged && lane == 0) {
    const int first = nunits < p.slots ? nunits : p.slots;
    for (int s = 0; s < first; ++s) mbar_init(&s_bar[warp][s], 1);
    fence_mbar_init();
    for (int s = 0; s < first; ++s) bulk_load(ring + (size_t)s * kUnitBytes, wsrc + (size_t)s * kUnitBytes,
                                              kUnitBytes, &s_bar[warp][s]);
  }
  uint32_t prevP1g = 0u, prevP1q = 0u;  // trellis halo: last chunk before wu0
  if (staged && wu0 > 0) {
    const uint4 pv = ldg_stream(reinterpret_cast<const uint4*>(wsrc - kUnitBytes) + lane * BITS);
    prevP1g = pv.z;
    prevP1q = pv.w;
  }
  trace(1);
  build_lut<BITS>(lut, cbv, warp, lane, kWarps);
  trace(2);

  // ---- activations: wait for the producer of x, then rotate our slice ----
  pdl_wait();
  trace(3);
  const int ncols = U * kUnitCols;
  rotate_slice(p, (int64_t)u0 * kUnitCols, ncols, zs, scratch);
  if (tid < 16) reinterpret_cast<uint32_t*>(zs + p.B * ncols)[tid] = 0u;  // zero block (64 B)
  __syncthreads();
  trace(4);

  // two independent accumulator chains (byte pairs q = 0 / 1) keep the
  // dependent MMA sequence short
  float acc[2][NT][4];
#pragma unroll
  for (int q = 0; q < 2; ++q)
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) acc[q][nt][0] = acc[q][nt][1] = acc[q][nt][2] = acc[q][nt][3] = 0.f;

  if (staged) {
    const uint4* zq = reinterpret_cast<const uint4*>(zs);
    const int zchunk = ncols / 8;  // uint4 per batch row
    int zbase[NT], zunit[NT];
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
      const int bn = nt * 8 + g;
      zbase[nt] = bn < p.B ? bn * zchunk + (wu0 - u0) * 32 + t * 4 : p.B * zchunk;
      zunit[nt] = bn < p.B ? 1 : 0;
    }
    const uint32_t lanew = BITS <= 3 ? (uint32_t)lane * 4u : (uint32_t)lane * 4u * 0x10001u;
    const int src = (lane & ~3) | ((t + 3) & 3);
    bool ok = true;
    int s = 0;             // ring slot of unit i
    unsigned parity = 0u;  // mbarrier phase parity of that slot
    for (int i = 0; i < nunits; ++i) {
      if (!mbar_wait(&s_bar[warp][s], parity)) {
        ok = false;
        break;
      }
      uint4 cur[BITS];
      const uint4* su = reinterpret_cast<const uint4*>(ring + (size_t)s * kUnitBytes) + lane * BITS;
#pragma unroll
      for (int k = 0; k < BITS; ++k) cur[k] = su[k];
      __syncwarp();
      if (lane == 0 && i + p.slots < nunits) {  // refill the slot just drained
        fence_proxy_async();
        bulk_load(ring + (size_t)s * kUnitBytes, wsrc + (size_t)(i + p.slots) * kUnitBytes, kUnitBytes,
                  &s_bar[warp][s]);
      }
      const uint32_t P0g = cur[0].x, P0q = cur[0].y, P1g = cur[0].z, P1q = cur[0].w;
      // halos: neighbour lane's chunk (t-1); lane t=0 takes lane 3's
      const uint32_t H0g = __shfl_sync(0xffffffffu, t == 3 ? prevP1g : P0g, src);
      const uint32_t H0q = __shfl_sync(0xffffffffu, t == 3 ? prevP1q : P0q, src);
      const uint32_t H1g = __shfl_sync(0xffffffffu, t == 3 ? P0g : P1g, src);
      const uint32_t H1q = __shfl_sync(0xffffffffu, t == 3 ? P0q : P1q, src);
      prevP1g = P1g;
      prevP1q = P1q;
#pragma unroll
      for (int cgi = 0; cgi < 2; ++cgi) {
        int zoff[NT];
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) zoff[nt] = zbase[nt] + zunit[nt] * (i * 32 + cgi * 16);
        const uint32_t Pg = cgi ? P1g : P0g, Pq = cgi ? P1q : P0q;
        const uint32_t Hg = cgi ? H1g : H0g, Hq = cgi ? H1q : H0q;
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
        process_chunk<BITS, S, NT>(lut, lanew, zq, Pg, Hg, Pq, Hq, Mg0, Mg1, Mg2, Mq0, Mq1, Mq2, zoff, acc);
      }
      if (++s == p.slots) {
        s = 0;
        parity ^= 1u;
      }
    }
    if (!ok) {  // copies never landed: outputs become NaN below
      s_fail = 1;
      if (lane == 0) atomicOr(p.status, kStatusTimeout);
    }
  }

  trace(5);
  // ---- reduction ----
  // red: [kw][rt*16][Bp] fp32; the CTA partial lands in slab 0.
  const int Bp = NT * 8;
  const int crows = p.rt * kTileRows;
#pragma unroll
  for (int nt = 0; nt < NT; ++nt) {
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const int bn = nt * 8 + 2 * t + (e & 1);
      const int r = rtl * kTileRows + g + ((e < 2) ? 0 : 8);
      red[(kwi * crows + r) * Bp + bn] = acc[0][nt][e] + acc[1][nt][e];
    }
  }
  __syncthreads();
  if (p.kw > 1) {
    for (int i = tid; i < crows * Bp; i += kThreads) {
      float v = red[i];
      for (int k = 1; k < p.kw; ++k) v += red[k * crows * Bp + i];
      red[i] = v;
    }
    __syncthreads();
  }
  const int64_t row0 = (int64_t)blockIdx.x * crows;
  trace(6);
  if (s_fail) {
    for (int i = tid; i < crows * Bp; i += kThreads) red[i] = __int_as_float(0x7fc00000);
    __syncthreads();
  }
  if (p.ksplit == 1) {
    for (int i = tid; i < crows * p.B; i += kThreads) {
      const int bn = i / crows, r = i - bn * crows;
      const int64_t row = row0 + r;
      if (row < p.n) {
        float v = red[r * Bp + bn] * h2f_bits(p.scales[row]);
        if (p.bias) v += h2f_bits(p.bias[row]);
        store_from_float(p.y, (int64_t)bn * p.n + row, p.y_dtype, v);
      }
    }
    trace(7);
    return;
  }
  if (p.cluster) {
    cg::cluster_group cl = cg::this_cluster();
    cl.sync();
    const int rank = static_cast<int>(cl.block_rank());
    // rank r finishes rows [r*crows/ks, (r+1)*crows/ks), summing ranks in order
    const int ra = rank * crows / p.ksplit, rb = (rank + 1) * crows / p.ksplit;
    const int nr = rb - ra;
    const float* rp[kMaxCluster];
#pragma unroll
    for (int k = 0; k < kMaxCluster; ++k) rp[k] = cl.map_shared_rank(red, k < p.ksplit ? k : 0);
    for (int i = tid; i < nr * p.B; i += kThreads) {
      const int bn = i / nr, r = ra + (i - bn * nr);
      const int64_t row = row0 + r;
      float part[kMaxCluster];
#pragma unroll
      for (int k = 0; k < kMaxCluster; ++k) part[k] = k < p.ksplit ? rp[k][r * Bp + bn] : 0.f;
      float v = 0.f;
#pragma unroll
      for (int k = 0; k < kMaxCluster; ++k) v += part[k];
      if (row < p.n) {
        v *= h2f_bits(p.scales[row]);
        if (p.bias) v += h2f_bits(p.bias[row]);
        store_from_float(p.y, (int64_t)bn * p.n + row, p.y_dtype, v);
      }
    }
    cl.sync();  // keep every CTA's shared memory alive until all reads are done
    trace(7);
    return;
  }
  // global split-K through the workspace; the last CTA of the row block reduces
  for (int i = tid; i < crows * p.B; i += kThreads) {
    const int bn = i / crows, r = i - bn * crows;
    p.partial[((int64_t)ks * p.B + bn) * p.n_pad + row0 + r] = red[r * Bp + bn];
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
  for (int i = tid; i < crows * p.B; i += kThreads) {
    const int bn = i / crows;
    const int64_t row = row0 + (i - bn * crows);
    if (row >= p.n) continue;
    float v = 0.f;
    for (int k = 0; k < p.ksplit; ++k) v += __ldcg(&p.partial[((int64_t)k * p.B + bn) * p.n_pad + row]);
    v *= h2f_bits(p.scales[row]);
    if (p.bias) v += h2f_bits(p.bias[row]);
    store_from_float(p.y, (int64_t)bn * p.n + row, p.y_dtype, v);
  }
  if (tid == 0) p.counters[blockIdx.x] = 0u;
  trace(7);
}

// ---------------------------------------------------------------------------
// launch configuration
// ---------------------------------------------------------------------------
// TP_DEBUG_PLAN=1 prints every launch configuration to stderr.
bool debug_plans() {
  static const bool on = [] {
    const char* e = getenv("TP_DEBUG_PLAN");
    return e && *e && *e != '0';
  }();
  return on;
}

inline uint32_t align128(uint32_t v) { return (v + 127) / 128 * 128; }

struct Plan {
  int rt, kw, ksplit, cluster;
  int64_t row_blocks;
  int units_k;
  int zrows_per_pass;
  int slots;
  bool fused_rotation;
  uint32_t w_off, z_off, scratch_off, red_off;
  size_t smem;
  int64_t ws_z, ws_partial, ws_total;
};

// Shared-memory carve-up of a configuration: pair table, activation slice,
// fp32 FWHT scratch and the reduction slabs.
void carve(Plan& pl, int bits, int64_t Bc, int slice_units, int64_t block) {
  const int Bp = static_cast<int>((Bc + 7) / 8) * 8;
  pl.w_off = bits == 4 ? Cfg<4>::kLutBytes : Cfg<3>::kLutBytes;
  pl.z_off = pl.w_off + static_cast<uint32_t>(kWarps * pl.slots * 512 * bits);
  const uint32_t zbytes = static_cast<uint32_t>(Bc * slice_units * kUnitCols * 2 + 64);
  pl.scratch_off = align128(pl.z_off + zbytes);
  uint32_t scratch = 0;
  pl.zrows_per_pass = 1;
  if (pl.fused_rotation) {
    // Hadamard blocks overlapping a slice of `cols` columns that starts on a
    // 256-column boundary: exactly the slice when block <= 256, otherwise at
    // most ceil(cols / block) + 1 whole blocks.
    const int64_t cols = (int64_t)slice_units * kUnitCols;
    const int64_t per_row = block <= kUnitCols ? cols : ((cols + block - 1) / block + 1) * block;
    pl.zrows_per_pass = static_cast<int>(std::max<int64_t>(1, std::min<int64_t>(Bc, kScratchFloats / per_row)));
    scratch = static_cast<uint32_t>(pl.zrows_per_pass * per_row * 4);
  }
  pl.red_off = align128(pl.scratch_off + scratch);
  const uint32_t red = static_cast<uint32_t>(pl.kw * pl.rt * kTileRows * Bp * 4);
  pl.smem = align128(pl.red_off + red);
}

Plan make_plan(int64_t B, int64_t n, int64_t d, int bits, int64_t block, int sms) {
  Plan best{};
  const int64_t Bc = std::min<int64_t>(B, kMaxBatchPerLaunch);
  const int64_t n_pad = pad_to(n, kTileRows), d_pad = pad_to(d, kUnitCols);
  const int64_t row_tiles = n_pad / kTileRows;
  const int units_k = static_cast<int>(d_pad / kUnitCols);
  const bool can_fuse = block <= kMaxFusedBlock;
  // Pick the configuration with the lowest modelled time: waves of CTAs
  // times a fixed per-wave latency, plus the bytes over the bandwidth that
  // the SMs in use can pull with the weight bytes they keep in flight.
  const double total_bytes = (double)n_pad * d_pad * bits / 8.0;
  double best_t = 1e30;
  for (int rt : {8, 4, 2, 1}) {
    const int kw = kWarps / rt;
    const int64_t row_blocks = (row_tiles + rt - 1) / rt;
    if (row_blocks > kMaxRowBlocks) continue;
    for (int ks = 1; ks <= std::min(32, units_k); ++ks) {
      const int slice = (units_k + ks - 1) / ks;
      if (slice < kw && !(ks == 1 && rt == 8)) continue;  // every warp gets >= 1 unit
      const int warp_units = (slice + kw - 1) / kw;
      for (int fuse = can_fuse ? 1 : 0; fuse >= 0; --fuse)
      for (int slots : {warp_units, 4, 3, 2}) {
        if (slots > warp_units || slots > kMaxSlots || slots < 1) continue;
        const bool fused = fuse != 0;
        Plan pl{};
        pl.rt = rt;
        pl.kw = kw;
        pl.ksplit = ks;
        pl.cluster = ks > 1 && ks <= kMaxCluster ? 1 : 0;
        pl.row_blocks = row_blocks;
        pl.units_k = units_k;
        pl.fused_rotation = fused;
        pl.slots = slots;
        carve(pl, bits, Bc, slice, block);
        if (pl.smem > kMaxDynSmem) continue;
        // registers (<= 128 per thread, launch bound of 2 CTAs) and shared memory
        const int per_sm = std::max(1, std::min<int>((228 * 1024) / (int)(pl.smem + 3072), 2));
        const int64_t cap = (int64_t)sms * per_sm;
        const int64_t ctas = row_blocks * ks;
        const int64_t waves = (ctas + cap - 1) / cap;
        // CTAs spread over SMs before doubling up
        const double sm_used = (double)std::min<int64_t>(ctas, sms);
        const int64_t per_sm_used = std::min<int64_t>(per_sm, (std::min(ctas, cap) + sms - 1) / sms);
        const double inflight = (double)per_sm_used * kWarps * slots * 512.0 * bits;
        const double t_mem = total_bytes / (6.5e12 * (sm_used / sms) * std::min(1.0, inflight / (72.0 * 1024)));
        // issue-limited decode: ~2.2 lane instructions per weight, half the
        // issue rate at 8 resident warps per SM, full rate from 16
        const double issue = std::min(1.0, per_sm_used * kWarps / 16.0);
        const double t_cmp = total_bytes * 8.0 / bits * 2.2 / (sm_used * 128.0 * issue * 1.9e9);
        double t = waves * 4e-6 + std::max(t_mem, t_cmp);
        // rotation: in every CTA over the Hadamard blocks its slice touches,
        // or once by a separate (PDL-overlapped) launch into the workspace
        const int64_t span = block <= kUnitCols ? (int64_t)slice * kUnitCols
                                                : ((int64_t)slice * kUnitCols + block - 1) / block * block;
        int lgb = 0;
        while ((int64_t(1) << lgb) < block) ++lgb;
        t += fused ? (double)Bc * span * (lgb + 6) / (0.5 * 128.0 * 1.9e9) + 0.5e-6 : 2.5e-6;
        if (ks > kMaxCluster) t += 1.5e-6;  // global reduction through the workspace
        t += ks * 1e-8;                     // prefer fewer splits on ties
        if (t < best_t) {
          best_t = t;
          best = pl;
        }
      }
    }
  }
  best.ws_z = best.fused_rotation ? 0 : align256(Bc * d_pad * 2);
  best.ws_partial = (best.ksplit > 1 && !best.cluster) ? align256((int64_t)best.ksplit * Bc * n_pad * 4) : 0;
  best.ws_total = kCounterBytes + best.ws_z + best.ws_partial;
  return best;
}

template <int BITS, int S, int NT>
tp_status launch_gemv_t(const GemvParams& p, const Plan& pl, cudaStream_t stream) {
  auto kern = tcq_gemv_kernel<BITS, S, NT>;
  static int smem_set[64] = {0};
  if (tp_status s = ensure_smem(kern, pl.smem, smem_set, "cudaFuncSetAttribute(gemv)")) return s;
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(static_cast<unsigned>(pl.row_blocks), static_cast<unsigned>(pl.ksplit), 1);
  cfg.blockDim = dim3(kThreads, 1, 1);
  cfg.dynamicSmemBytes = pl.smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[2];
  int na = 0;
  attr[na].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[na].val.programmaticStreamSerializationAllowed = 1;
  ++na;
  if (pl.cluster) {
    attr[na].id = cudaLaunchAttributeClusterDimension;
    attr[na].val.clusterDim.x = 1;
    attr[na].val.clusterDim.y = static_cast<unsigned>(pl.ksplit);
    attr[na].val.clusterDim.z = 1;
    ++na;
  }
  cfg.attrs = attr;
  cfg.numAttrs = na;
  TP_CUDA_TRY(cudaLaunchKernelEx(&cfg, kern, p), "tcq_gemv_kernel launch");
  return check_launch("tcq_gemv_kernel");
}

template <int BITS, int S>
tp_status launch_gemv_nt(const GemvParams& p, const Plan& pl, cudaStream_t stream) {
  switch ((p.B + 7) / 8) {
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

namespace tp {
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

}  // namespace tp

extern "C" int64_t tp_gemv_workspace_bytes(int64_t B, int64_t n, int64_t d, int bits) {
  if (B < 1 || n < 1 || d < 1 || bits < 1 || bits > 4) return -1;
  // Upper bound over every launch plan: counters, pre-rotated activations and
  // partial sums for the largest split along K (32).
  const int64_t Bc = std::min<int64_t>(B, kMaxBatchPerLaunch);
  int64_t extra = align256(Bc * pad_to(d, kUnitCols) * 2) + align256(32 * Bc * pad_to(n, kTileRows) * 4);
  // the stream-K kernel (batch chunks up to 8) needs its own partial-sum slots
  // (any Hadamard block: block 1 gives the largest plan)
  const int64_t sk = sk_workspace_extra(std::min<int64_t>(B, kSkMaxBatch), n, d, bits, 1);
  if (sk > extra) extra = sk;
  return kCounterBytes + extra;
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
  if (block < 1 || (block & (block - 1)) || d % block)
    return fail(TP_ERR_ARG, "block must be a power of two dividing d (d=%lld, block=%lld)", (long long)d,
                (long long)block);
  if (block > kMaxRotateBlock)
    return fail(TP_ERR_UNSUPPORTED, "Hadamard block %lld exceeds the supported maximum %d", (long long)block,
                kMaxRotateBlock);
  const int sms = sm_count();
  const Plan pl = make_plan(B, n, d, bits, block, sms);
  if (pl.row_blocks == 0 || pl.smem == 0)
    return fail(TP_ERR_UNSUPPORTED, "tp_tcq_gemv: no launch configuration for n=%lld d=%lld", (long long)n,
                (long long)d);
  const int64_t need = tp_gemv_workspace_bytes(B, n, d, bits);
  if (!workspace || workspace_bytes < need)
    return fail(TP_ERR_WORKSPACE, "tp_tcq_gemv: workspace of %lld bytes required (got %lld)", (long long)need,
                (long long)workspace_bytes);
  if (!aligned(workspace, 256)) return fail(TP_ERR_ALIGN, "tp_tcq_gemv: workspace must be 256-byte aligned");
  cudaStream_t st = as_stream(stream);
  unsigned char* ws = static_cast<unsigned char*>(workspace);
  const int64_t d_pad = pad_to(d, kUnitCols), n_pad = pad_to(n, kTileRows);
  const size_t xel = x_dtype == TP_F32 ? 4 : 2, yel = y_dtype == TP_F32 ? 4 : 2;
  int lg = 0;
  while ((int64_t(1) << lg) < block) ++lg;
  for (int64_t b0 = 0; b0 < B; b0 += kMaxBatchPerLaunch) {
    const int64_t Bc = std::min<int64_t>(kMaxBatchPerLaunch, B - b0);
    const Plan pc = make_plan(Bc, n, d, bits, block, sms);
    if (pc.ws_total > need)
      return fail(TP_ERR_WORKSPACE, "tp_tcq_gemv: plan needs %lld workspace bytes (bound %lld)",
                  (long long)pc.ws_total, (long long)need);
    const void* xc = static_cast<const unsigned char*>(x) + b0 * d * xel;
    if (Bc <= kSkMaxBatch && sk_workspace_extra(Bc, n, d, bits, block) >= 0) {
      SkRequest r{};
      r.x = xc;
      r.x_dtype = x_dtype;
      r.rot_scale = rot_scale;
      r.stream = tcq_stream;
      r.scales = scales;
      r.codebook = codebook;
      r.bias = bias;
      r.y = static_cast<unsigned char*>(y) + b0 * n * yel;
      r.y_dtype = y_dtype;
      r.B = static_cast<int>(Bc);
      r.n = n;
      r.d = d;
      r.block = block;
      r.bits = bits;
      r.n_states = n_states;
      r.workspace = ws;
      if (tp_status s = sk_gemv(r, st)) return s;
      continue;
    }
    GemvParams p{};
    if (!pc.fused_rotation) {
      RotateArgs ra{};
      ra.x = xc;
      ra.x_dtype = x_dtype;
      ra.scale = rot_scale;
      ra.z = ws + kCounterBytes;
      ra.z_dtype = TP_F16;
      ra.d = d;
      ra.d_pad = d_pad;
      ra.block = block;
      ra.mode = 2;
      if (tp_status s = launch_rotate(ra, Bc, st)) return s;
      p.zperm = reinterpret_cast<const uint4*>(ws + kCounterBytes);
    }
    p.stream = reinterpret_cast<const uint4*>(tcq_stream);
    p.scales = scales;
    p.bias = bias;
    p.codebook = codebook;
    p.x = xc;
    p.rot_scale = rot_scale;
    p.y = static_cast<unsigned char*>(y) + b0 * n * yel;
    p.partial = reinterpret_cast<float*>(ws + kCounterBytes + pc.ws_z);
    p.counters = reinterpret_cast<unsigned*>(ws);
    p.status = reinterpret_cast<unsigned*>(ws + kStatusOff);
    p.x_dtype = x_dtype;
    p.y_dtype = y_dtype;
    p.B = static_cast<int>(Bc);
    p.n = n;
    p.n_pad = n_pad;
    p.d = d;
    p.d_pad = d_pad;
    p.units_k = pc.units_k;
    p.block = static_cast<int>(block);
    p.lg_block = lg;
    p.norm = static_cast<float>(1.0 / __builtin_sqrt(static_cast<double>(block)));
    p.rt = pc.rt;
    p.kw = pc.kw;
    p.ksplit = pc.ksplit;
    p.cluster = pc.cluster;
    p.zrows_per_pass = pc.zrows_per_pass;
    p.slots = pc.slots;
    p.w_off = pc.w_off;
    p.z_off = pc.z_off;
    p.scratch_off = pc.scratch_off;
    p.red_off = pc.red_off;
    if (debug_plans())
      fprintf(stderr, "tp_tcq_gemv n=%lld d=%lld B=%lld bits=%d: rt=%d kw=%d ksplit=%d cluster=%d slots=%d "
              "smem=%zu grid=%lldx%d fused=%d\n", (long long)n, (long long)d, (long long)Bc, bits, pc.rt, pc.kw,
              pc.ksplit, pc.cluster, pc.slots, pc.smem, (long long)pc.row_blocks, pc.ksplit, (int)pc.fused_rotation);
    if (tp_status s = launch_gemv(p, pc, bits, n_states, st)) return s;
  }
  return clear_ok();
}

// Status word of a GEMV workspace.  A call that completes leaves the
// counter block zero; one whose kernel gave up (a bounded wait ran out, or
// the shared-memory layout check failed) sets a status bit and may leave
// split-K counters part-way, which would make the next call on the same
// workspace combine the wrong partial sums.  So a nonzero status clears the
// whole counter block (counters and status) before it is reported.
namespace tp {
tp_status gemv_status_at(const unsigned char* ws, cudaStream_t st, const char* who) {
  unsigned v = 0;
  TP_CUDA_TRY(cudaMemcpyAsync(&v, ws + kStatusOff, 4, cudaMemcpyDeviceToHost, st), "status copy");
  TP_CUDA_TRY(cudaStreamSynchronize(st), "status sync");
  if (v == 0) return clear_ok();
  TP_CUDA_TRY(cudaMemsetAsync(const_cast<unsigned char*>(ws), 0, kCounterBytes, st), "counter block clear");
  TP_CUDA_TRY(cudaStreamSynchronize(st), "counter block clear sync");
  if (v & kStatusLayout)
    return fail(TP_ERR_DEVICE, "%s: shared-memory layout check failed, outputs not written (status %u)", who, v);
  return fail(TP_ERR_DEVICE, "%s: a bounded device wait ran out, outputs are NaN (status %u)", who, v);
}
}  // namespace tp

extern "C" tp_status tp_gemv_status(const void* workspace, void* stream) {
  if (!workspace) return fail(TP_ERR_ARG, "tp_gemv_status: null workspace");
  return gemv_status_at(static_cast<const unsigned char*>(workspace), as_stream(stream), "tp_tcq_gemv");
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

#ifdef TP_TRACE
extern "C" TP_API int tp_trace_read(unsigned long long* host, int ctas) {
  return (int)cudaMemcpyFromSymbol(host, g_trace, (size_t)ctas * 16 * sizeof(unsigned long long));
}
#endif

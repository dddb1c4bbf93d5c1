// Persistent decoder step on sm_100a: one cooperative launch runs a whole
// batch-B decode step of a Qwen3 / Llama-style decoder whose linears are
// packed-TCQ layers, stage after stage with a grid barrier between stages.
//
// Stages per layer (h = the fp16 residual stream):
//   QKV    x = rmsnorm(h) * ln1; q, k, v = packed linears of x
//   ATTN   q/k head norms (Qwen3), RoPE at position pos, append k/v to the
//          fp16 KV cache, GQA attention over tokens [0, pos] (split over
//          CTAs, combined by the last CTA of each (batch row, kv head))
//   O      h += o_proj(attn)
//   GATEUP x = rmsnorm(h) * ln2; gate, up = packed linears of x
//   DOWN   h += down_proj(silu(gate) * up)
// and a final stage out = rmsnorm(h) * final_norm (the LM head follows as its
// own launch, tp_lm_head_argmax).
//
// A linear stage is the stream-K GEMV of tp_gemv_sk.cu over all of its ops'
// row tiles at once (one flat unit space split evenly over every warp of the
// grid): each CTA builds the input transform (norm or SiLU product, fp16 as
// the reference model rounds it), rotates it with each op's seeded Hadamard
// scales into shared memory, then decodes its warps' runs.  Weight units of
// the next stage are prefetched into L2 before each barrier.  The fp16
// rounding points (norm output, linear outputs, residual adds, SiLU product,
// RoPE) follow the reference model's fp16 forward; attention is computed in
// fp32 (flash-decoding style) and rounded once.
#include <cooperative_groups.h>

#include <algorithm>
#include <cmath>
#include <cstring>
#include <mutex>
#include <vector>

#include "tp_gemv_sk.cuh"
#include "tp_sk_core.cuh"

namespace tp {
namespace {

using namespace sk;

constexpr int kStepWarps = 16;
constexpr int kStepThreads = kStepWarps * 32;
constexpr int kMaxStageOps = 3;
constexpr int kStepMaxBatch = 8;
constexpr int kMaxGroup = 8;        // query heads per kv head
constexpr int kMaxSplits = 32;      // attention splits per (batch row, kv head)
constexpr unsigned long long kBarrierNs = 2000000000ull;  // a grid barrier gives up after 2 s

enum StageType : int { kLinear = 0, kAttention = 1, kFinalNorm = 2 };
enum InKind : int { kInPlain = 0, kInRmsNorm = 1, kInSiluMul = 2 };
enum EpiKind : int { kEpiStore = 0, kEpiResidual = 1 };

// workspace words
constexpr int64_t kWsStatus = 64;      // status bits (kStepStatus*)
constexpr int64_t kWsFlags = 1024;     // grid barrier counter (zeroed before each run)
constexpr int kMaxGrid = 512;
constexpr int64_t kWsCounters = kWsFlags + 4 * kMaxGrid;  // per-row-tile / per-attention-group counters
constexpr unsigned kStepStatusLayout = 1u, kStepStatusBarrier = 2u;

struct alignas(16) StepOp {
  const unsigned char* stream;
  const uint16_t* scales;
  const uint16_t* rot_scale;
  const uint16_t* bias;
  uint16_t* out;  // fp16 [B][n]
  int n, row_tiles, rt_off, pad;
};

struct alignas(16) LinearStage {
  const uint16_t* codebook;
  const uint16_t* in0;    // [B][d] fp16: x (plain / norm) or gate (SiLU product)
  const uint16_t* in1;    // [B][d] fp16: up (SiLU product)
  const uint16_t* gamma;  // [d] fp16 norm weight
  int nops, in_kind, epi, bits;
  int d, d_pad, units_k, lg_block;
  float norm, eps;
  int kparts, us, cps, maxc, rt_total, rpp, rs_smem, pad2[3];
  uint32_t z_off, xin_off, scr_off, rs_off;  // shared-memory offsets from the dynamic base
  SliceSplit split[2];
  StepOp ops[kMaxStageOps];
};

struct alignas(16) AttnStage {
  const uint16_t* q;  // [B][q_heads*hd] fp16 (q_proj output)
  const uint16_t* k;  // [B][kv_heads*hd]
  const uint16_t* v;
  const uint16_t* q_norm;  // [hd] or null
  const uint16_t* k_norm;
  uint16_t* k_cache;  // [B][kv_heads][max_t][hd]
  uint16_t* v_cache;
  uint16_t* out;  // [B][q_heads*hd]
  const float* inv_freq;  // [hd/2]
  int q_heads, kv_heads, hd, max_t;
  int nsplit;
  float eps, scaling;
  uint32_t buf_off;
};

struct alignas(16) NormStage {
  const uint16_t* x;
  const uint16_t* gamma;
  uint16_t* out;
  int d;
  float eps;
};

struct alignas(16) StepStage {
  int type, pad[3];
  union {
    LinearStage lin;
    AttnStage attn;
    NormStage fnorm;
  };
};

struct alignas(16) StepHeader {
  int nstages, B, grid, has4;
  uint32_t base, dyn, lut_off, misc_off;
  int64_t ws_part_off, ws_attn_off, ws_bytes;
  int max_rt, attn_groups;
  // grid-barrier limit in microseconds (0: kBarrierNs), and arrivals a
  // barrier waits for beyond the grid's own (0 in every program that runs a
  // model; tp_step_set_wait raises it to make the waits run out on purpose)
  unsigned barrier_us;
  int extra_arrivals;
};

constexpr int kRecordBytes = (sizeof(StepStage) + 15) / 16 * 16;
constexpr int kMiscRecord = 0;                      // three stage-record slots
constexpr int kMiscCodebook = 3 * kRecordBytes;     // 32 codebook words
constexpr int kMiscRed = kMiscCodebook + 128;       // [B + 1][16] fp32 reduction scratch (576 B)
constexpr int kMiscFlags = kMiscRed + 640;          // barrier / last-CTA flags
constexpr int kMiscBytes = (kMiscFlags + 64 + 127) / 128 * 128;
static_assert(kMiscBytes <= 2304, "stage records");

#ifdef TP_STEP_TRACE
// Development-only stage timeline (built only with -DTP_STEP_TRACE, never in
// the shipped library): %globaltimer per stage, CTA and phase.
__device__ unsigned long long g_step_trace[256][160][8];
__shared__ int s_step_trace_stage;
__device__ __forceinline__ void step_trace(int s, int k) {
  if (threadIdx.x == 0 && blockIdx.x < 160 && s < 256) {
    // SM cycle counter: differences are meaningful within one CTA
    g_step_trace[s][blockIdx.x][k] = static_cast<unsigned long long>(clock64());
    if (k == 0) s_step_trace_stage = s;
  }
}
// a mark inside a stage (thread 0 of the CTA)
__device__ __forceinline__ void step_mark(int k) {
  if (threadIdx.x == 0 && blockIdx.x < 160) step_trace(s_step_trace_stage, k);
}
#else
__device__ __forceinline__ void step_trace(int, int) {}
__device__ __forceinline__ void step_mark(int) {}
#endif

__device__ __forceinline__ float h2f(uint16_t b) { return __half2float(__ushort_as_half(b)); }
__device__ __forceinline__ uint16_t f2h(float v) { return __half_as_ushort(__float2half_rn(v)); }
__device__ __forceinline__ float r16(float v) { return __half2float(__float2half_rn(v)); }

__device__ __forceinline__ unsigned ld_acquire(const unsigned* p) {
  unsigned v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ unsigned long long global_ns() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// Grid barrier on a cumulative arrival counter: one thread per CTA adds one
// (after a release fence) and spins on acquire loads until `target`; bounded
// by kBarrierNs of global time, after which it sets the status and every
// CTA abandons the step.
__device__ bool grid_barrier(unsigned* bar, unsigned* status, unsigned target, unsigned long long limit_ns,
                             int* s_ok) {
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    atomicAdd(bar, 1u);
    int ok = 0;
    const unsigned long long t0 = global_ns();
    for (unsigned i = 0;; ++i) {
      if (ld_acquire(bar) >= target) {
        ok = 1;
        break;
      }
      if ((i & 255u) == 255u && (global_ns() - t0 > limit_ns || (ld_acquire(status) & kStepStatusBarrier))) break;
    }
    if (!ok) atomicOr(status, kStepStatusBarrier);
    *s_ok = ok;
  }
  __syncthreads();
  return *s_ok != 0;
}

// ---------------------------------------------------------------------------
// linear stage
// ---------------------------------------------------------------------------
__device__ __forceinline__ void cp_async16(void* dst, const void* src, bool valid) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(smem_u32(dst)), "l"(src), "r"(valid ? 16 : 0)
               : "memory");
}
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_all;" ::: "memory"); }

__device__ __forceinline__ float sumsq8(uint4 v) {
  const uint32_t w[4] = {v.x, v.y, v.z, v.w};
  float s = 0.f;
#pragma unroll
  for (int e = 0; e < 4; ++e) {
    const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&w[e]));
    s = fmaf(f.x, f.x, fmaf(f.y, f.y, s));
  }
  return s;
}

// Input transform of rows [b0, b0+rows) over slice columns [c0, c0+cols):
// xin (fp16 bits, [rows][cols]) = the stage's input as the reference rounds
// it.  Every thread issues all of its 16-byte loads of a round before using
// them (one memory round trip per round of 512 chunks of 8 columns).
__device__ __forceinline__ uint4 transform8(int kind, uint4 xv, uint4 uv, uint4 gv, float r) {
  const uint32_t xw[4] = {xv.x, xv.y, xv.z, xv.w};
  uint32_t ow[4];
  if (kind == kInRmsNorm) {
    const uint32_t gw[4] = {gv.x, gv.y, gv.z, gv.w};
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const float2 xf = __half22float2(*reinterpret_cast<const __half2*>(&xw[e]));
      const float2 gf = __half22float2(*reinterpret_cast<const __half2*>(&gw[e]));
      const __half2 hv = __floats2half2_rn(gf.x * r16(xf.x * r), gf.y * r16(xf.y * r));
      ow[e] = *reinterpret_cast<const uint32_t*>(&hv);
    }
  } else if (kind == kInSiluMul) {
    const uint32_t uw[4] = {uv.x, uv.y, uv.z, uv.w};
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const float2 gf = __half22float2(*reinterpret_cast<const __half2*>(&xw[e]));
      const float2 uf = __half22float2(*reinterpret_cast<const __half2*>(&uw[e]));
      const float a0 = r16(gf.x / (1.f + __expf(-gf.x))), a1 = r16(gf.y / (1.f + __expf(-gf.y)));
      const __half2 hv = __floats2half2_rn(a0 * uf.x, a1 * uf.y);
      ow[e] = *reinterpret_cast<const uint32_t*>(&hv);
    }
  } else {
#pragma unroll
    for (int e = 0; e < 4; ++e) ow[e] = xw[e];
  }
  return make_uint4(ow[0], ow[1], ow[2], ow[3]);
}

// Input transform of rows [b0, b0+rows) over slice columns [c0, c0+cols):
// xin (fp16 bits, [rows][cols]) = the stage's input as the reference rounds
// it.  Warps split over the rows (fixed order: deterministic sums); every
// lane issues all its 16-byte loads of a round before using them, and when a
// row fits one round the norm's sum of squares comes from the same loads.
__device__ __forceinline__ void stage_input(const LinearStage& L, int b0, int rows, int c0, int cols,
                                            uint16_t* xin, float* red) {
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  float* rinv = red + kStepMaxBatch * kStepWarps;
  const int wpr = kStepWarps / rows, row = warp / wpr, sub = warp - row * wpr;
  const bool act = row < rows;
  const int64_t xrow = (int64_t)(b0 + (act ? row : 0)) * L.d;
  constexpr int U = 4;  // 16-byte loads per lane in flight
  const int stride = wpr * 32;
  const int cpr = cols >> 3;
  const bool norm = L.in_kind == kInRmsNorm;
  // one round covers the whole row: load once, norm from the same registers
  const bool single = cols == L.d && cpr <= stride * U;
  uint4 xv[U], uv[U], gv[U];
  auto load_round = [&](int cb) {
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int ci = cb + u * stride, c = c0 + ci * 8;
      if (act && ci < cpr && c < L.d) {
        xv[u] = *reinterpret_cast<const uint4*>(L.in0 + xrow + c);
        if (L.in_kind == kInSiluMul) uv[u] = *reinterpret_cast<const uint4*>(L.in1 + xrow + c);
        if (norm) gv[u] = *reinterpret_cast<const uint4*>(L.gamma + c);
      }
    }
  };
  if (single) load_round(sub * 32 + lane);
  if (norm) {
    float ssum = 0.f;
    if (single) {
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const int ci = sub * 32 + lane + u * stride;
        if (act && ci < cpr) ssum += sumsq8(xv[u]);
      }
    } else {
      const int dpr = L.d >> 3;
      for (int cb = sub * 32 + lane; act && cb < dpr; cb += stride * U) {
        uint4 v[U];
#pragma unroll
        for (int u = 0; u < U; ++u)
          if (cb + u * stride < dpr) v[u] = *reinterpret_cast<const uint4*>(L.in0 + xrow + (cb + u * stride) * 8);
#pragma unroll
        for (int u = 0; u < U; ++u)
          if (cb + u * stride < dpr) ssum += sumsq8(v[u]);
      }
    }
    for (int o = 16; o; o >>= 1) ssum += __shfl_xor_sync(0xffffffffu, ssum, o);
    if (lane == 0) red[warp] = ssum;
    __syncthreads();
    if (tid < rows) {
      float sv = 0.f;
      for (int w = 0; w < wpr; ++w) sv += red[tid * wpr + w];
      rinv[tid] = rsqrtf(sv / (float)L.d + L.eps);
    }
    __syncthreads();
  }
  const float r = norm && act ? rinv[row] : 1.f;
  for (int cb = sub * 32 + lane; act && cb < cpr; cb += stride * U) {
    if (!single) load_round(cb);
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int ci = cb + u * stride, c = c0 + ci * 8;
      if (ci >= cpr) break;
      const uint4 o = c < L.d ? transform8(L.in_kind, xv[u], uv[u], gv[u], r) : make_uint4(0u, 0u, 0u, 0u);
      *reinterpret_cast<uint4*>(xin + row * cols + ci * 8) = o;
    }
  }
  cp_async_wait_all();  // the rotation scales of the stage (issued before its barrier)
  __syncthreads();
}

template <int HB>
__device__ __forceinline__ void step_column_pass(const float* scr, __half* z, int zst, int rows, int cols, int blk,
                                                 float norm) {
  const int nb = cols / blk;
  for (int i = threadIdx.x; i < rows * nb * 256; i += kStepThreads) {
    const int bi = i >> 8, c = i & 255;
    const float* src = scr + bi * blk + c;
    float w[1 << HB];
#pragma unroll
    for (int k = 0; k < (1 << HB); ++k) w[k] = src[k * 256];
    fwht_regs<HB>(w);
    const int row = bi / nb, col0 = (bi - row * nb) * blk + c;
#pragma unroll
    for (int k = 0; k < (1 << HB); ++k) z[row * zst + sk_zpos(col0 + k * 256)] = __float2half_rn(w[k] * norm);
  }
}

// z rows [b0, b0+rows) of one op: FWHT(xin * rot_scale) per Hadamard block.
__device__ __forceinline__ void stage_rotate(const LinearStage& L, const uint16_t* rs, const uint16_t* xin, int rows, int c0,
                             int cols, float* scr, __half* z, int zst) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int lg = L.lg_block, tpr = cols >> 8;
  for (int k = warp; k < rows * tpr; k += kStepWarps) {
    const int rr = k / tpr, cl = (k - rr * tpr) * 256 + lane * 8;
    float v[8];
    const uint4 xv = *reinterpret_cast<const uint4*>(xin + rr * cols + cl);
    const uint32_t xw[4] = {xv.x, xv.y, xv.z, xv.w};
    // slice-local scales (shared memory: zero past d; global: guarded)
    uint4 rv = make_uint4(0u, 0u, 0u, 0u);
    if (L.rs_smem || c0 + cl < L.d) rv = *reinterpret_cast<const uint4*>(rs + cl);
    const uint32_t rw[4] = {rv.x, rv.y, rv.z, rv.w};
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const float2 xf = __half22float2(*reinterpret_cast<const __half2*>(&xw[e]));
      const float2 rf = __half22float2(*reinterpret_cast<const __half2*>(&rw[e]));
      v[2 * e] = xf.x * rf.x;
      v[2 * e + 1] = xf.y * rf.y;
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
      for (int e = 0; e < 8; ++e) z[rr * zst + sk_zpos(cl + e)] = __float2half_rn(v[e] * L.norm);
    } else {
      float4* dst = reinterpret_cast<float4*>(scr + rr * cols + cl);
      dst[0] = make_float4(v[0], v[1], v[2], v[3]);
      dst[1] = make_float4(v[4], v[5], v[6], v[7]);
    }
  }
  __syncthreads();
  if (lg > 8) {
    const int blk = 1 << lg;
    switch (lg - 8) {
      case 1: step_column_pass<1>(scr, z, zst, rows, cols, blk, L.norm); break;
      case 2: step_column_pass<2>(scr, z, zst, rows, cols, blk, L.norm); break;
      case 3: step_column_pass<3>(scr, z, zst, rows, cols, blk, L.norm); break;
      case 4: step_column_pass<4>(scr, z, zst, rows, cols, blk, L.norm); break;
      default: step_column_pass<5>(scr, z, zst, rows, cols, blk, L.norm); break;
    }
    __syncthreads();
  }
}

// Hadamard blocks of 256 or 512 columns, every op at once: one warp per
// (op, row, block) holds the block in registers (E = 8 or 16 columns per
// lane: the low index bits in place, the five lane bits by shuffles) and
// writes the fp16 activations; no shared-memory staging, one barrier.
template <int E>
__device__ __forceinline__ void rotate_small_blocks(const LinearStage& L, const uint16_t* rs_all, int rs_stride,
                                                    const uint16_t* xin, int rows, int b0, int B, int c0, int cols,
                                                    __half* z, int zst) {
  constexpr int LGE = E == 16 ? 4 : 3;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int blk = 32 * E, nblk = cols / blk, per_op = rows * nblk;
  for (int task = warp; task < L.nops * per_op; task += kStepWarps) {
    const int k = task / per_op, rem = task - k * per_op, rr = rem / nblk, bi = rem - rr * nblk;
    const int cl = bi * blk + lane * E;
    const uint16_t* rs = rs_all + (int64_t)k * rs_stride;
    float v[E];
#pragma unroll
    for (int q = 0; q < E / 8; ++q) {
      const uint4 xv = *reinterpret_cast<const uint4*>(xin + rr * cols + cl + 8 * q);
      uint4 rv = make_uint4(0u, 0u, 0u, 0u);
      if (L.rs_smem || c0 + cl + 8 * q < L.d) rv = *reinterpret_cast<const uint4*>(rs + cl + 8 * q);
      const uint32_t xw[4] = {xv.x, xv.y, xv.z, xv.w}, rw[4] = {rv.x, rv.y, rv.z, rv.w};
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float2 xf = __half22float2(*reinterpret_cast<const __half2*>(&xw[e]));
        const float2 rf = __half22float2(*reinterpret_cast<const __half2*>(&rw[e]));
        v[8 * q + 2 * e] = xf.x * rf.x;
        v[8 * q + 2 * e + 1] = xf.y * rf.y;
      }
    }
    fwht_regs<LGE>(v);
#pragma unroll
    for (int sbit = 0; sbit < 5; ++sbit) {
      const float sg = (lane >> sbit) & 1 ? -1.f : 1.f;
#pragma unroll
      for (int e = 0; e < E; ++e) v[e] = fmaf(sg, v[e], __shfl_xor_sync(0xffffffffu, v[e], 1 << sbit));
    }
    __half* zr = z + (k * (B + 1) + b0 + rr) * zst;
#pragma unroll
    for (int e = 0; e < E; ++e) zr[sk_zpos(cl + e)] = __float2half_rn(v[e] * L.norm);
  }
  __syncthreads();
}

// Rotation scales of a linear stage into shared memory (cp.async, waited for
// in stage_input): issued before the barrier that precedes the stage, they
// depend on nothing the barrier orders.
__device__ void stage_rs_prefetch(const LinearStage& L, unsigned char* smem) {
  const int slice = blockIdx.x / L.cps;
  if (slice >= L.kparts || !L.rs_smem) return;
  const int Us = L.split[slice == L.kparts - 1 ? 1 : 0].us;
  const int cols = Us * kUnitCols, c0 = slice * L.us * kUnitCols;
  uint16_t* rs_s = reinterpret_cast<uint16_t*>(smem + L.rs_off);
  for (int i = threadIdx.x; i < L.nops * (cols / 8); i += kStepThreads) {
    const int k = i / (cols / 8), ci = i - k * (cols / 8);
    const bool valid = c0 + ci * 8 < L.d;
    cp_async16(rs_s + k * cols + ci * 8, L.ops[k].rot_scale + (valid ? c0 + ci * 8 : 0), valid);
  }
}

// Stage prologue: rotation scales to shared memory (async), the input
// transform, every op's rotated activations, and the zero rows (CTAs of a
// K-slice: the slice's columns).
__device__ __forceinline__ void stage_prologue(const LinearStage& L, unsigned char* smem, int B, float* red) {
  const int tid = threadIdx.x;
  const int slice = blockIdx.x / L.cps;
  if (slice >= L.kparts) return;
  const int Us = L.split[slice == L.kparts - 1 ? 1 : 0].us;
  const int cols = Us * kUnitCols, c0 = slice * L.us * kUnitCols;
  const int zst = L.us * kUnitCols + kZPad;
  __half* z = reinterpret_cast<__half*>(smem + L.z_off);
  uint16_t* xin = reinterpret_cast<uint16_t*>(smem + L.xin_off);
  float* scr = reinterpret_cast<float*>(smem + L.scr_off);
  uint16_t* rs_s = reinterpret_cast<uint16_t*>(smem + L.rs_off);
  for (int b0 = 0; b0 < B; b0 += L.rpp) {
    const int rows = min(L.rpp, B - b0);
    stage_input(L, b0, rows, c0, cols, xin, red);
    step_mark(4);
    if (L.lg_block <= 9 && L.rs_smem) {
      if (L.lg_block == 9) rotate_small_blocks<16>(L, rs_s, cols, xin, rows, b0, B, c0, cols, z, zst);
      else rotate_small_blocks<8>(L, rs_s, cols, xin, rows, b0, B, c0, cols, z, zst);
    } else {
      for (int k = 0; k < L.nops; ++k)
        stage_rotate(L, L.rs_smem ? rs_s + k * cols : L.ops[k].rot_scale + c0, xin, rows, c0, cols, scr,
                     z + (k * (B + 1) + b0) * zst, zst);
    }
  }
  step_mark(5);
  for (int i = tid; i < L.nops * (cols / 8); i += kStepThreads) {
    const int k = i / (cols / 8), r = i - k * (cols / 8);
    reinterpret_cast<uint4*>(z + (k * (B + 1) + B) * zst)[r] = make_uint4(0u, 0u, 0u, 0u);
  }
  __syncthreads();
}

template <int BITS>
__device__ __forceinline__ void linear_stage(const LinearStage& L, unsigned char* smem, int B, const unsigned char* lut,
                             unsigned char* ws, const StepHeader& H, int sidx) {
  constexpr int S = 64;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int g = lane >> 2, t = lane & 3;
  const int slice = blockIdx.x / L.cps;
  if (slice >= L.kparts) return;  // CTAs beyond the split idle until the barrier
  // warp-major numbering spreads the working warps of a small stage over
  // every CTA
  const int wl = warp * L.cps + (blockIdx.x - slice * L.cps);
  const int us0 = slice * L.us;
  const SliceSplit& sp = L.split[slice == L.kparts - 1 ? 1 : 0];
  const int Us = sp.us;
  const int j0 = wl < sp.nw ? sp.start(wl) : 0, j1 = wl < sp.nw ? sp.start(wl + 1) : 0;
  constexpr unsigned UB = 512u * BITS;
  // flat row tile -> op
  auto op_of = [&](int rt) {
    int k = 0;
    while (k + 1 < L.nops && rt >= L.ops[k + 1].rt_off) ++k;
    return k;
  };
  auto unit_ptr = [&](int k, int rt, int ul) {
    return L.ops[k].stream + ((int64_t)(rt - L.ops[k].rt_off) * L.units_k + us0 + ul) * UB;
  };

  // the rotated activations were built by stage_prologue (called before)
  const int zst = L.us * kUnitCols + kZPad;
  __half* z = reinterpret_cast<__half*>(smem + L.z_off);

  // ---- first unit of the run and its trellis halo (in L2: prefetched
  // before the barrier) ----
  int rt = sp.row_tile(j0), ul = j0 - rt * Us;
  int opk = op_of(rt);
  uint4 wa[BITS];
  uint32_t hg = 0u, hq = 0u, hng = 0u, hnq = 0u;
  if (j0 < j1) {
    const uint4* src = reinterpret_cast<const uint4*>(unit_ptr(opk, rt, ul)) + lane * BITS;
#pragma unroll
    for (int k = 0; k < BITS; ++k) wa[k] = ldg_stream(src + k);
    if (us0 + ul > 0) {
      const uint4 pv = ldg_stream(reinterpret_cast<const uint4*>(unit_ptr(opk, rt, ul - 1)) + lane * BITS);
      hg = pv.z;
      hq = pv.w;
    }
  }
  step_trace(sidx, 1);

  // ---- decode + MMA over the run ----
  float acc[2][4];
#pragma unroll
  for (int q = 0; q < 2; ++q) acc[q][0] = acc[q][1] = acc[q][2] = acc[q][3] = 0.f;
  const uint32_t lwA = BITS <= 3 ? (kLutAbs | (uint32_t)lane * 4u) : (uint32_t)lane * 4u * 0x10001u;
  const uint32_t lwB = lwA | 0x80u;
  const int zrow = min(g, B);
  auto zbase = [&](int k) { return reinterpret_cast<const uint4*>(z + (k * (B + 1) + zrow) * zst) + t; };
  const uint4* zp = zbase(opk) + ul * 32;
  const int src = (lane & ~3) | ((t + 3) & 3);
  const int64_t row_skip = (int64_t)(L.units_k - Us) * UB;
  const unsigned char* wp = unit_ptr(opk, rt, ul) + lane * BITS * 16;
  unsigned* counters = reinterpret_cast<unsigned*>(ws + kWsCounters);
  float* part = reinterpret_cast<float*>(ws + H.ws_part_off);

  auto flush = [&](int frt, int k) {
    float v[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) v[e] = acc[0][e] + acc[1][e];
#pragma unroll
    for (int q = 0; q < 2; ++q) acc[q][0] = acc[q][1] = acc[q][2] = acc[q][3] = 0.f;
    const bool solo = L.kparts == 1 && j0 <= frt * Us && (frt + 1) * Us <= j1;
    step_mark(6);
    if (!solo) {
      const int rank = wl - sp.warp_of(frt * Us);
      float* pc = part + ((int64_t)(frt * L.kparts + slice) * L.maxc + rank) * 16 * B;
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int col = 2 * t + (e & 1), row = g + 8 * (e >> 1);
        if (col < B) __stcg(pc + row * B + col, v[e]);
      }
      __threadfence();
      __syncwarp();
      const SliceSplit& s0 = L.split[0];
      const SliceSplit& s1 = L.split[1];
      const int c0_ = s0.warp_of((frt + 1) * s0.us - 1) - s0.warp_of(frt * s0.us) + 1;
      const int c1_ = s1.warp_of((frt + 1) * s1.us - 1) - s1.warp_of(frt * s1.us) + 1;
      unsigned last = 0u;
      if (lane == 0)
        last = atomicAdd(&counters[frt], 1u) == (unsigned)((L.kparts - 1) * c0_ + c1_ - 1) ? 1u : 0u;
      last = __shfl_sync(0xffffffffu, last, 0);
      if (!last) return;
      step_mark(7);
      __threadfence();
#pragma unroll
      for (int e = 0; e < 4; ++e) v[e] = 0.f;
      for (int sl = 0; sl < L.kparts; ++sl) {
        const int cnt = sl == L.kparts - 1 ? c1_ : c0_;
        const float* pp = part + (int64_t)(frt * L.kparts + sl) * L.maxc * 16 * B;
        for (int kk = 0; kk < cnt; ++kk, pp += 16 * B) {
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const int col = 2 * t + (e & 1), row = g + 8 * (e >> 1);
            if (col < B) v[e] += __ldcg(pp + row * B + col);
          }
        }
      }
      if (lane == 0) counters[frt] = 0u;
    }
    const StepOp& op = L.ops[k];
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const int col = 2 * t + (e & 1);
      const int row = (frt - op.rt_off) * kTileRows + g + 8 * (e >> 1);
      if (col < B && row < op.n) {
        float o = v[e] * h2f(op.scales[row]);
        if (op.bias) o += h2f(op.bias[row]);
        uint16_t* dst = op.out + (int64_t)col * op.n + row;
        if (L.epi == kEpiResidual) o = h2f(*dst) + r16(o);
        *dst = f2h(o);
      }
    }
  };

  uint4 zv = make_uint4(0u, 0u, 0u, 0u);
  const bool zon = g < B;
  for (int j = j0; j < j1; ++j) {
    const bool row_end = ul + 1 == Us;
    const bool more = j + 1 < j1;
    const uint32_t P0g = wa[0].x, P0q = wa[0].y, P1g = wa[0].z, P1q = wa[0].w;
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
    // next unit: same row tile, or the next row tile (possibly the next op)
    int nrt = rt, nk = opk;
    const unsigned char* np;
    if (row_end) {
      nrt = rt + 1;
      nk = (opk + 1 < L.nops && nrt >= L.ops[opk + 1].rt_off) ? opk + 1 : opk;
      np = (nk == opk ? wp + UB + row_skip : unit_ptr(nk, nrt, 0) + lane * BITS * 16);
    } else {
      np = wp + UB;
    }
    if (more) {
#pragma unroll
      for (int k = 0; k < BITS; ++k) wa[k] = ldg_stream(reinterpret_cast<const uint4*>(np) + k);
      if (row_end && us0 > 0) {
        const uint4 pv = ldg_stream(reinterpret_cast<const uint4*>(np - UB));
        hng = pv.z;
        hnq = pv.w;
      }
    }
    sk_mma_chunk<BITS>(lwA, lwB, lut, zp, zon, zv, L0g, L0q, m2[0], m2[1], acc);
    sk_mma_chunk<BITS>(lwA, lwB, lut, zp + 4, zon, zv, L1g, L1q, m2[2], m2[3], acc);
    zp += 32;
    wp = np;
    if (row_end || !more) flush(rt, opk);
    if (row_end) {
      hg = hng;
      hq = hnq;
      rt = nrt;
      opk = nk;
      ul = 0;
      zp = zbase(opk);
    } else {
      ++ul;
    }
  }
}

// L2 prefetch of this warp's first units of a linear stage (issued before
// the barrier that precedes the stage).
__device__ void prefetch_stage(const LinearStage& L) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int slice = blockIdx.x / L.cps;
  if (slice >= L.kparts || lane >= 8) return;
  const int wl = warp * L.cps + (blockIdx.x - slice * L.cps);
  const SliceSplit& sp = L.split[slice == L.kparts - 1 ? 1 : 0];
  if (wl >= sp.nw) return;
  const int x = sp.start(wl) + lane;
  if (x >= sp.start(wl + 1)) return;
  const int rt = sp.row_tile(x), ul = x - rt * sp.us;
  int k = 0;
  while (k + 1 < L.nops && rt >= L.ops[k + 1].rt_off) ++k;
  const unsigned UB = 512u * L.bits;
  prefetch_l2(L.ops[k].stream + ((int64_t)(rt - L.ops[k].rt_off) * L.units_k + L.us * slice + ul) * UB, UB);
}

// ---------------------------------------------------------------------------
// attention stage
// ---------------------------------------------------------------------------
// RMS norm of one head vector held E values per lane (the whole warp), fp16
// rounding as the reference: fp16(gamma * fp16(x * rsqrt(mean(x^2) + eps))).
template <int E>
__device__ __forceinline__ void head_norm(float* x, const float* gam, int hd, float eps) {
  float s = 0.f;
#pragma unroll
  for (int e = 0; e < E; ++e) s += x[e] * x[e];
  for (int o = 16; o; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
  const float r = rsqrtf(s / (float)hd + eps);
#pragma unroll
  for (int e = 0; e < E; ++e) x[e] = r16(gam[e] * r16(x[e] * r));
}

// RoPE (rotate-half form) on a head vector (E values per lane, lanes 0-15
// hold the first half): fp16(fp16(x*cos) + fp16(rot*sin)), cos / sin of
// pos * inv_freq rounded to fp16.
template <int E>
__device__ __forceinline__ void rope(float* x, const float* freq, int pos, int lane) {
  float partner[E];
#pragma unroll
  for (int e = 0; e < E; ++e) partner[e] = __shfl_xor_sync(0xffffffffu, x[e], 16);
  const bool hi = lane >= 16;
#pragma unroll
  for (int e = 0; e < E; ++e) {
    const float f = (float)pos * freq[e];
    const float c = r16(cosf(f)), s = r16(sinf(f));
    const float rot = hi ? partner[e] : -partner[e];
    x[e] = r16(r16(x[e] * c) + r16(rot * s));
  }
}

template <int E>
__device__ __forceinline__ void load_h(float* v, const uint16_t* p) {
  if constexpr (E == 4) {
    const uint2 w = *reinterpret_cast<const uint2*>(p);
    const float2 a = __half22float2(*reinterpret_cast<const __half2*>(&w.x));
    const float2 b = __half22float2(*reinterpret_cast<const __half2*>(&w.y));
    v[0] = a.x, v[1] = a.y, v[2] = b.x, v[3] = b.y;
  } else {
    const float2 a = __half22float2(*reinterpret_cast<const __half2*>(p));
    v[0] = a.x, v[1] = a.y;
  }
}

template <int E, int G>
__device__ __noinline__ void attn_item(const AttnStage& A, int b, int kvh, int sp, int pos, unsigned char* buf, float* part,
                          unsigned* counters, int cgroup, unsigned* s_last) {
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int hd = A.hd, gs = A.q_heads / A.kv_heads;
  float* sq = reinterpret_cast<float*>(buf);                 // [gs][hd] normed, roped q
  float* knew = sq + kMaxGroup * hd;                         // [hd]
  float* vnew = knew + hd;                                   // [hd]
  float* wst = vnew + hd;                                    // [16 warps][gs][hd + 2]
  const int T = pos + 1, Ls = (T + A.nsplit - 1) / A.nsplit;
  const int t0 = sp * Ls, t1 = min(T, t0 + Ls);
  const int64_t kv0 = ((int64_t)b * A.kv_heads + kvh) * A.max_t;
  // this warp's first cached token, loaded before anything waits
  float kx[E], vx[E];
  int tok = t0 + warp;
  if (tok < t1 && tok != pos) {
    load_h<E>(kx, A.k_cache + (kv0 + tok) * hd + lane * E);
    load_h<E>(vx, A.v_cache + (kv0 + tok) * hd + lane * E);
  }
  // q heads of the group (one warp per head) and the new token's k / v
  const bool newtok = t1 == T && t0 < t1;
  if (warp < gs || (warp == kStepWarps - 1 && newtok)) {
    const bool isq = warp < gs;
    const uint16_t* src = isq ? A.q + (int64_t)b * A.q_heads * hd + (kvh * gs + warp) * hd
                              : A.k + (int64_t)b * A.kv_heads * hd + kvh * hd;
    const uint16_t* gam = isq ? A.q_norm : A.k_norm;
    float x[E], gm[E], fr[E], vv[E];
    load_h<E>(x, src + lane * E);
    if (gam) load_h<E>(gm, gam + lane * E);
#pragma unroll
    for (int e = 0; e < E; ++e) fr[e] = A.inv_freq[(lane & 15) * E + e];
    if (!isq) load_h<E>(vv, A.v + (int64_t)b * A.kv_heads * hd + kvh * hd + lane * E);
    if (gam) head_norm<E>(x, gm, hd, A.eps);
    rope<E>(x, fr, pos, lane);
    if (isq) {
#pragma unroll
      for (int e = 0; e < E; ++e) sq[warp * hd + lane * E + e] = x[e];
    } else {
      const int64_t ci = (kv0 + pos) * hd;
#pragma unroll
      for (int e = 0; e < E; ++e) {
        knew[lane * E + e] = x[e];
        vnew[lane * E + e] = vv[e];
        A.k_cache[ci + lane * E + e] = f2h(x[e]);
        A.v_cache[ci + lane * E + e] = f2h(vv[e]);
      }
    }
  }
  __syncthreads();
  step_mark(4);
  // per-warp online softmax over its tokens
  float qv[G][E], m[G], l[G], acc[G][E];
#pragma unroll
  for (int j = 0; j < G; ++j) {
    m[j] = -INFINITY;
    l[j] = 0.f;
#pragma unroll
    for (int e = 0; e < E; ++e) {
      qv[j][e] = j < gs ? sq[j * hd + lane * E + e] : 0.f;
      acc[j][e] = 0.f;
    }
  }
  for (; tok < t1; tok += kStepWarps) {
    if (tok == pos) {
#pragma unroll
      for (int e = 0; e < E; ++e) kx[e] = knew[lane * E + e], vx[e] = vnew[lane * E + e];
    }
    // next token's k / v in flight while this one is used
    float kn[E], vn[E];
    const int nt = tok + kStepWarps;
    if (nt < t1 && nt != pos) {
      load_h<E>(kn, A.k_cache + (kv0 + nt) * hd + lane * E);
      load_h<E>(vn, A.v_cache + (kv0 + nt) * hd + lane * E);
    }
#pragma unroll
    for (int j = 0; j < G; ++j) {
      if (j >= gs) break;
      float sc = 0.f;
#pragma unroll
      for (int e = 0; e < E; ++e) sc = fmaf(qv[j][e], kx[e], sc);
      for (int o = 16; o; o >>= 1) sc += __shfl_xor_sync(0xffffffffu, sc, o);
      // the reference's fp16 scores: fp16(q.k), then fp16(* scaling)
      sc = r16(r16(sc) * A.scaling);
      const float mn = fmaxf(m[j], sc);
      const float corr = __expf(m[j] - mn), p = __expf(sc - mn);
      l[j] = l[j] * corr + p;
#pragma unroll
      for (int e = 0; e < E; ++e) acc[j][e] = fmaf(acc[j][e], corr, p * vx[e]);
      m[j] = mn;
    }
#pragma unroll
    for (int e = 0; e < E; ++e) kx[e] = kn[e], vx[e] = vn[e];
  }
  step_mark(5);
  // combine the warps
  const int ws_ = hd + 2;
#pragma unroll
  for (int j = 0; j < G; ++j) {
    if (j >= gs) break;
    float* dst = wst + (warp * gs + j) * ws_;
#pragma unroll
    for (int e = 0; e < E; ++e) dst[2 + lane * E + e] = acc[j][e];
    if (lane == 0) dst[0] = m[j], dst[1] = l[j];
  }
  __syncthreads();
  float* mypart = part + ((int64_t)cgroup * A.nsplit + sp) * gs * ws_;
  for (int i = tid; i < gs * hd; i += kStepThreads) {
    const int j = i / hd, dd = i - j * hd;
    float M = -INFINITY;
    for (int w = 0; w < kStepWarps; ++w) M = fmaxf(M, wst[(w * gs + j) * ws_]);
    float Lsum = 0.f, Ad = 0.f;
    for (int w = 0; w < kStepWarps; ++w) {
      const float* src = wst + (w * gs + j) * ws_;
      const float f = src[0] == -INFINITY ? 0.f : __expf(src[0] - M);
      Lsum += src[1] * f;
      Ad += src[2 + dd] * f;
    }
    __stcg(mypart + j * ws_ + 2 + dd, Ad);
    if (dd == 0) {
      __stcg(mypart + j * ws_, M);
      __stcg(mypart + j * ws_ + 1, Lsum);
    }
  }
  // the last CTA of the (b, kvh) group combines the splits
  __threadfence();
  __syncthreads();
  if (tid == 0) *s_last = atomicAdd(&counters[cgroup], 1u) == (unsigned)(A.nsplit - 1) ? 1u : 0u;
  __syncthreads();
  step_mark(6);
  if (!*s_last) return;
  __threadfence();
  const float* gp = part + (int64_t)cgroup * A.nsplit * gs * ws_;
  // split maxima and sums into shared memory first (one pass of loads)
  float* ml = wst;  // [nsplit][gs][2]
  for (int i = tid; i < A.nsplit * gs; i += kStepThreads) {
    ml[2 * i] = __ldcg(gp + i * ws_);
    ml[2 * i + 1] = __ldcg(gp + i * ws_ + 1);
  }
  __syncthreads();
  step_mark(1);
  for (int i = tid; i < gs * hd; i += kStepThreads) {
    const int j = i / hd, dd = i - j * hd;
    float M = -INFINITY;
    for (int s2 = 0; s2 < A.nsplit; ++s2) M = fmaxf(M, ml[2 * (s2 * gs + j)]);
    // every split's partial in flight at once, then the weighted sum
    float av[kMaxSplits];
#pragma unroll
    for (int s2 = 0; s2 < kMaxSplits; ++s2)
      if (s2 < A.nsplit) av[s2] = __ldcg(gp + (s2 * gs + j) * ws_ + 2 + dd);
    float Lsum = 0.f, Ad = 0.f;
#pragma unroll
    for (int s2 = 0; s2 < kMaxSplits; ++s2) {
      if (s2 >= A.nsplit) break;
      const float ms = ml[2 * (s2 * gs + j)];
      const float f = ms == -INFINITY ? 0.f : __expf(ms - M);
      Lsum += ml[2 * (s2 * gs + j) + 1] * f;
      Ad += av[s2] * f;
    }
    A.out[(int64_t)b * A.q_heads * hd + (kvh * gs + j) * hd + dd] = f2h(Ad / Lsum);
  }
  step_mark(7);
  if (tid == 0) counters[cgroup] = 0u;
}

__device__ void attn_stage(const AttnStage& A, int B, int pos, unsigned char* smem, unsigned char* ws,
                           const StepHeader& H) {
  unsigned char* buf = smem + A.buf_off;
  unsigned* s_last = reinterpret_cast<unsigned*>(smem + H.misc_off + kMiscFlags + 4);
  float* part = reinterpret_cast<float*>(ws + H.ws_attn_off);
  unsigned* counters = reinterpret_cast<unsigned*>(ws + kWsCounters);
  const int items = B * A.kv_heads * A.nsplit;
  for (int it = blockIdx.x; it < items; it += gridDim.x) {
    const int grp = it / A.nsplit, sp = it - grp * A.nsplit;
    const int b = grp / A.kv_heads, kvh = grp - b * A.kv_heads;
    const int gs = A.q_heads / A.kv_heads;
    if (A.hd == 128) {
      if (gs <= 4) attn_item<4, 4>(A, b, kvh, sp, pos, buf, part, counters, grp, s_last);
      else attn_item<4, kMaxGroup>(A, b, kvh, sp, pos, buf, part, counters, grp, s_last);
    } else {
      if (gs <= 4) attn_item<2, 4>(A, b, kvh, sp, pos, buf, part, counters, grp, s_last);
      else attn_item<2, kMaxGroup>(A, b, kvh, sp, pos, buf, part, counters, grp, s_last);
    }
    __syncthreads();
  }
}

// L2 bulk prefetch of the cached keys / values this CTA's attention items
// will read (issued a stage ahead: the cache is far larger than L2).
__device__ void prefetch_attention(const AttnStage& A, int B, int pos) {
  if (threadIdx.x >= 32) return;
  const int lane = threadIdx.x;
  const int items = B * A.kv_heads * A.nsplit;
  const int T = pos + 1, Ls = (T + A.nsplit - 1) / A.nsplit;
  int n = 0;
  for (int it = blockIdx.x; it < items; it += gridDim.x, ++n) {
    if (lane != (2 * n) % 32 && lane != (2 * n + 1) % 32) continue;
    const int grp = it / A.nsplit, sp = it - grp * A.nsplit;
    const int t0 = sp * Ls, t1 = min(pos, t0 + Ls);  // the new token is not cached yet
    if (t1 <= t0) continue;
    const int64_t row = (int64_t)grp * A.max_t + t0;
    const uint16_t* src = (lane & 1) ? A.v_cache : A.k_cache;
    const unsigned bytes = (unsigned)(t1 - t0) * A.hd * 2u;
    for (unsigned off = 0; off < bytes; off += 65536u)
      prefetch_l2(src + row * A.hd + off / 2, min(65536u, bytes - off));
  }
}

__device__ void final_norm_stage(const NormStage& N, int B, float* red) {
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  for (int b = blockIdx.x; b < B; b += gridDim.x) {
    const uint16_t* x = N.x + (int64_t)b * N.d;
    float s = 0.f;
    for (int c = tid; c < N.d; c += kStepThreads) {
      const float f = h2f(x[c]);
      s += f * f;
    }
    for (int o = 16; o; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    if (lane == 0) red[warp] = s;
    __syncthreads();
    float tot = 0.f;
    for (int w = 0; w < kStepWarps; ++w) tot += red[w];
    const float r = rsqrtf(tot / (float)N.d + N.eps);
    for (int c = tid; c < N.d; c += kStepThreads) N.out[(int64_t)b * N.d + c] = f2h(h2f(N.gamma[c]) * r16(h2f(x[c]) * r));
    __syncthreads();
  }
}

// ---------------------------------------------------------------------------
// the persistent kernel
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(kStepThreads, 1)
    step_kernel(const StepHeader* __restrict__ img, unsigned char* ws, const int* pos_p) {
  extern __shared__ __align__(128) unsigned char smem[];
  const StepHeader H = *img;
  const StepStage* stages = reinterpret_cast<const StepStage*>(img + 1);
  unsigned* bar = reinterpret_cast<unsigned*>(ws + kWsFlags);
  unsigned* status = reinterpret_cast<unsigned*>(ws + kWsStatus);
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  if (smem_u32(smem) != H.base) {  // the layout was planned for this base
    if (tid == 0) atomicOr(status, kStepStatusLayout);
    return;
  }
  const int pos = *pos_p;
  const unsigned long long limit_ns = H.barrier_us ? 1000ull * H.barrier_us : kBarrierNs;
  // stage records: slot s % 3 is in use, the next one has landed, the one
  // after that is in flight (cp.async), so no stage reads its record from HBM
  StepStage* slots = reinterpret_cast<StepStage*>(smem + H.misc_off + kMiscRecord);
  auto fetch = [&](int idx) {
    if (idx >= H.nstages) return;
    for (int i = tid; i < (int)(sizeof(StepStage) / 16); i += kStepThreads)
      cp_async16(reinterpret_cast<uint4*>(&slots[idx % 3]) + i, reinterpret_cast<const uint4*>(&stages[idx]) + i,
                 true);
  };
  uint32_t* cbs = reinterpret_cast<uint32_t*>(smem + H.misc_off + kMiscCodebook);
  // pair tables: bits <= 3 at shared-window address kLutAbs, 4-bit at the
  // start of the dynamic area (it spans the other one)
  unsigned char* lut3 = smem + (kLutAbs - H.base);
  unsigned char* lut4 = smem;
  int* s_ok = reinterpret_cast<int*>(smem + H.misc_off + kMiscFlags);
  float* red = reinterpret_cast<float*>(smem + H.misc_off + kMiscRed);
  const uint16_t* cur_cb = nullptr;
  int cur_bits = 0;
  fetch(0);
  fetch(1);
  cp_async_wait_all();
  __syncthreads();
  if (H.nstages > 0 && slots[0].type == kLinear) stage_rs_prefetch(slots[0].lin, smem);
  for (int s = 0; s < H.nstages; ++s) {
    const StepStage& st = slots[s % 3];
    fetch(s + 2);
    step_trace(s, 0);
    if (s + 1 < H.nstages && slots[(s + 1) % 3].type == kAttention) prefetch_attention(slots[(s + 1) % 3].attn, H.B, pos);
    if (st.type == kLinear) {
      const LinearStage& L = st.lin;
      if (L.codebook != cur_cb || L.bits != cur_bits) {
        if (warp == 0) cbs[lane] = lane < (1 << (L.bits + 1)) ? L.codebook[lane] : 0u;
        __syncthreads();
        if (L.bits == 2) build_tables<2>(lut3, cbs[lane], warp, lane, kStepWarps);
        else if (L.bits == 3) build_tables<3>(lut3, cbs[lane], warp, lane, kStepWarps);
        else build_tables<4>(lut4, cbs[lane], warp, lane, kStepWarps);
        cur_cb = L.codebook;
        cur_bits = L.bits;
        __syncthreads();
      }
      stage_prologue(L, smem, H.B, red);
      step_trace(s, 1);
      if (L.bits == 2) linear_stage<2>(L, smem, H.B, lut3, ws, H, s);
      else if (L.bits == 3) linear_stage<3>(L, smem, H.B, lut3, ws, H, s);
      else linear_stage<4>(L, smem, H.B, lut4, ws, H, s);
    } else if (st.type == kAttention) {
      attn_stage(st.attn, H.B, pos, smem, ws, H);
    } else {
      final_norm_stage(st.fnorm, H.B, red);
    }
    step_trace(s, 2);
    if (s + 1 == H.nstages) break;
    cp_async_wait_all();  // the next records have landed
    __syncthreads();      // and this stage's shared buffers are free
    const StepStage& nx = slots[(s + 1) % 3];
    if (nx.type == kLinear) {
      prefetch_stage(nx.lin);
      stage_rs_prefetch(nx.lin, smem);
    }
    if (!grid_barrier(bar, status, (unsigned)(s + 1) * gridDim.x + (unsigned)H.extra_arrivals, limit_ns, s_ok)) break;
    step_trace(s, 3);
  }
}

// ---------------------------------------------------------------------------
// host: program builder
// ---------------------------------------------------------------------------
int step_sm_count() {
  int dev = 0, v = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return 148;
  if (cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || v <= 0) return 148;
  return v;
}

struct Regions {
  uint32_t base, dyn_max;
  bool has4;
  // free areas: [a0, a1) before the bits<=3 table (none with 4-bit stages), [b0, b1) after the table
  uint32_t a0, a1, b0, b1;
};

bool valid_linear(const tp_step_linear& l) {
  return l.tcq_stream && l.scales && l.codebook && l.rot_scale && l.n > 0 && l.d > 0 && l.bits >= 2 && l.bits <= 4 &&
         l.n_states == 64 && l.block >= 256 && l.block <= 8192 && (l.block & (l.block - 1)) == 0 &&
         l.d % l.block == 0 && aligned(l.tcq_stream, 16) && aligned(l.rot_scale, 16);
}

// Plan one linear stage (ops share d, block, bits, codebook).
tp_status plan_linear(LinearStage& L, const tp_step_linear* const* ops, uint16_t* const* outs, int nops, int B,
                      int G, const Regions& R, int64_t* rt_max, int64_t* part_floats) {
  const tp_step_linear& f = *ops[0];
  for (int k = 0; k < nops; ++k) {
    const tp_step_linear& o = *ops[k];
    if (!valid_linear(o)) return fail(TP_ERR_UNSUPPORTED, "tp_step: unsupported linear (bits 2-4, 64 states, "
                                                          "Hadamard block 256-8192, 16-byte aligned streams)");
    if (o.d != f.d || o.block != f.block || o.bits != f.bits || o.codebook != f.codebook)
      return fail(TP_ERR_ARG, "tp_step: ops of one stage must share d, block, bits and codebook values");
  }
  L.codebook = f.codebook;
  L.bits = f.bits;
  L.nops = nops;
  L.d = static_cast<int>(f.d);
  L.d_pad = static_cast<int>(pad_to(f.d, kUnitCols));
  L.units_k = L.d_pad / kUnitCols;
  int lg = 0;
  while ((int64_t(1) << lg) < f.block) ++lg;
  L.lg_block = lg;
  L.norm = static_cast<float>(1.0 / std::sqrt(static_cast<double>(f.block)));
  int rt = 0;
  for (int k = 0; k < nops; ++k) {
    StepOp& op = L.ops[k];
    op.stream = ops[k]->tcq_stream;
    op.scales = ops[k]->scales;
    op.rot_scale = ops[k]->rot_scale;
    op.bias = ops[k]->bias;
    op.out = outs[k];
    op.n = static_cast<int>(ops[k]->n);
    op.row_tiles = static_cast<int>(pad_to(ops[k]->n, kTileRows) / kTileRows);
    op.rt_off = rt;
    rt += op.row_tiles;
  }
  L.rt_total = rt;
  const int U = L.units_k;
  const int blk_units = std::max(1, static_cast<int>(f.block / kUnitCols));
  // K-slices: the smallest count whose buffers fit; slices are whole
  // Hadamard blocks.  Buffers go to region a (below the bits <= 3 table)
  // first -- a small shared-memory footprint leaves the SM more L1 -- then
  // to region b (after the table).
  int us = 0, kparts = 0, rpp = 0, rs_smem = 1;
  uint32_t off[4] = {0, 0, 0, 0};  // z, xin, scr, rs
  bool found = false;
  auto place = [&](const uint32_t* sz) {
    uint32_t ua = 0, ub = 0;
    const uint32_t ca = R.has4 ? 0 : R.a1 - R.a0, cb = R.b1 - R.b0;
    for (int i = 0; i < 4; ++i) {
      if (sz[i] == 0) {
        off[i] = R.b0 - R.base;
        continue;
      }
      if (ua + sz[i] <= ca) {
        off[i] = R.a0 - R.base + ua;
        ua += sz[i];
      } else if (ub + sz[i] <= cb) {
        off[i] = R.b0 - R.base + ub;
        ub += sz[i];
      } else {
        return false;
      }
    }
    return true;
  };
  for (int attempt = 0; attempt < 2 && !found; ++attempt) {
    rs_smem = attempt == 0 ? 1 : 0;
    for (kparts = 1; kparts <= U && !found; ++kparts) {
      us = (U + kparts - 1) / kparts;
      us = (us + blk_units - 1) / blk_units * blk_units;
      const int kp = (U + us - 1) / us;
      if (kp != kparts) continue;
      const int cols = us * kUnitCols;
      const bool need_scr = !(rs_smem && L.lg_block <= 9);
      for (rpp = B; rpp >= 1; --rpp) {
        const uint32_t sz[4] = {
            static_cast<uint32_t>(((int64_t)nops * (B + 1) * (cols + kZPad) * 2 + 127) / 128 * 128),
            static_cast<uint32_t>(((int64_t)rpp * cols * 2 + 127) / 128 * 128),
            need_scr ? static_cast<uint32_t>((int64_t)rpp * cols * 4) : 0u,
            static_cast<uint32_t>((int64_t)rs_smem * nops * cols * 2)};
        if (place(sz)) {
          found = true;
          break;
        }
      }
      if (found) break;
    }
  }
  if (!found) return fail(TP_ERR_UNSUPPORTED, "tp_step: activations of d=%d do not fit shared memory", L.d);
  L.rs_smem = rs_smem;
  L.kparts = kparts;
  L.us = us;
  L.rpp = rpp;
  L.z_off = off[0];
  L.xin_off = off[1];
  L.scr_off = off[2];
  L.rs_off = off[3];
  // grid split
  L.cps = std::max(1, G / kparts);
  const int64_t W = (int64_t)L.cps * kStepWarps;
  L.maxc = 0;
  for (int k = 0; k < 2; ++k) {
    const int64_t su = k == 0 ? us : U - (int64_t)(kparts - 1) * us;
    const int64_t T = (int64_t)rt * su;
    const int64_t Wk = std::min<int64_t>(W, T);  // a small stage leaves some warps idle
    L.split[k].us = static_cast<int>(su);
    L.split[k].nw = static_cast<int>(Wk);
    L.split[k].r = static_cast<int>(T / Wk);
    L.split[k].rem = static_cast<int>(T % Wk);
    L.split[k].div_us = make_fastdiv(static_cast<uint32_t>(su));
    L.split[k].div_r = make_fastdiv(static_cast<uint32_t>(T / Wk));
    L.split[k].div_r1 = make_fastdiv(static_cast<uint32_t>(T / Wk + 1));
    const int64_t r = T / Wk;
    L.maxc = std::max<int>(L.maxc, static_cast<int>((su + r - 1) / r + 1));
  }
  *rt_max = std::max<int64_t>(*rt_max, rt);
  *part_floats = std::max<int64_t>(*part_floats, (int64_t)rt * kparts * L.maxc * 16 * B);
  return TP_OK;
}

std::mutex g_step_mu;
int g_step_smem_set[64] = {0};

}  // namespace
}  // namespace tp

using namespace tp;

extern "C" int64_t tp_step_image_bytes(int layers) {
  if (layers < 1) return -1;
  return (int64_t)sizeof(StepHeader) + (int64_t)(5 * layers + 1) * sizeof(StepStage);
}

extern "C" int64_t tp_step_act_bytes(const tp_step_model* m) {
  if (!m || m->B < 1) return -1;
  const int64_t qd = (int64_t)m->q_heads * m->head_dim, kd = (int64_t)m->kv_heads * m->head_dim;
  // q, k, v, attn, gate, up (fp16), each 256-byte aligned
  return 2 * m->B * (align256(qd) + 2 * align256(kd) + align256(qd) + 2 * align256(m->inter)) + 6 * 256;
}

extern "C" tp_status tp_step_build(const tp_step_model* m, const tp_step_layer* layers, void* image_host,
                                   int64_t image_bytes, int64_t* workspace_bytes) {
  if (!m || !layers || !image_host || !workspace_bytes) return fail(TP_ERR_ARG, "tp_step_build: null argument");
  const int B = m->B;
  if (B < 1 || B > kStepMaxBatch) return fail(TP_ERR_UNSUPPORTED, "tp_step: batch must be 1..%d", kStepMaxBatch);
  if (m->layers < 1 || image_bytes < tp_step_image_bytes(m->layers))
    return fail(TP_ERR_ARG, "tp_step_build: image buffer too small");
  if (!(m->head_dim == 128 || m->head_dim == 64) || m->q_heads % m->kv_heads || m->q_heads / m->kv_heads > kMaxGroup)
    return fail(TP_ERR_UNSUPPORTED, "tp_step: head_dim must be 64 or 128 with at most %d query heads per kv head",
                kMaxGroup);
  if (!m->hidden_state || !m->final_out || !m->final_norm || !m->act || !m->inv_freq || m->max_tokens < 1)
    return fail(TP_ERR_ARG, "tp_step_build: missing buffers");
  int dev = 0, reserved = 0, optin = 0;
  TP_CUDA_TRY(cudaGetDevice(&dev), "cudaGetDevice");
  TP_CUDA_TRY(cudaDeviceGetAttribute(&reserved, cudaDevAttrReservedSharedMemoryPerBlock, dev), "attr");
  TP_CUDA_TRY(cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev), "attr");
  cudaFuncAttributes fa{};
  TP_CUDA_TRY(cudaFuncGetAttributes(&fa, step_kernel), "cudaFuncGetAttributes(step)");
  const int G = step_sm_count();
  if (G > kMaxGrid) return fail(TP_ERR_UNSUPPORTED, "tp_step: more than %d SMs", kMaxGrid);
  Regions R{};
  R.base = static_cast<uint32_t>((reserved + fa.sharedSizeBytes + 127) / 128 * 128);
  R.dyn_max = static_cast<uint32_t>(optin) - static_cast<uint32_t>(fa.sharedSizeBytes);
  bool has4 = false;
  for (int i = 0; i < m->layers; ++i) {
    const tp_step_linear* ls[7] = {&layers[i].q, &layers[i].k, &layers[i].v, &layers[i].o,
                                   &layers[i].gate, &layers[i].up, &layers[i].down};
    for (auto* l : ls) has4 |= l->bits == 4;
  }
  R.has4 = has4;
  const uint32_t lut_end = has4 ? R.base + 131072u : kLutAbs + 65536u;
  if (!has4 && R.base > kLutAbs - 4096) return fail(TP_ERR_UNSUPPORTED, "tp_step: shared-memory base too high");
  R.a0 = R.base;
  R.a1 = has4 ? R.base : kLutAbs - kMiscBytes;
  R.b0 = has4 ? lut_end + kMiscBytes : lut_end;
  R.b1 = R.base + R.dyn_max;
  const uint32_t misc_off = (has4 ? lut_end : kLutAbs - kMiscBytes) - R.base;

  // Codebooks are compared by value (read once here): layers whose
  // codebooks hold the same levels share one pointer, so the kernel rebuilds
  // its pair table only where the values change.
  std::vector<tp_step_layer> lys(layers, layers + m->layers);
  {
    std::vector<std::pair<std::vector<uint16_t>, const uint16_t*>> seen;
    for (auto& ly : lys) {
      tp_step_linear* ls[7] = {&ly.q, &ly.k, &ly.v, &ly.o, &ly.gate, &ly.up, &ly.down};
      for (auto* l : ls) {
        if (!l->codebook || l->bits < 1 || l->bits > 4) continue;
        std::vector<uint16_t> v(static_cast<size_t>(2) << l->bits);
        TP_CUDA_TRY(cudaMemcpy(v.data(), l->codebook, v.size() * 2, cudaMemcpyDeviceToHost), "codebook read");
        const uint16_t* canon = nullptr;
        for (auto& e : seen)
          if (e.first == v) canon = e.second;
        if (!canon) {
          seen.emplace_back(v, l->codebook);
          canon = l->codebook;
        }
        l->codebook = canon;
      }
    }
  }
  layers = lys.data();
  StepHeader* H = static_cast<StepHeader*>(image_host);
  memset(image_host, 0, static_cast<size_t>(tp_step_image_bytes(m->layers)));
  StepStage* st = reinterpret_cast<StepStage*>(H + 1);
  const int64_t hd = m->head_dim, qd = m->q_heads * hd, kd = m->kv_heads * hd;
  unsigned char* act = static_cast<unsigned char*>(m->act);
  uint16_t* qb = reinterpret_cast<uint16_t*>(act);
  uint16_t* kb = reinterpret_cast<uint16_t*>(act + B * align256(qd) * 2 + 256);
  uint16_t* vb = reinterpret_cast<uint16_t*>(reinterpret_cast<unsigned char*>(kb) + B * align256(kd) * 2 + 256);
  uint16_t* ab = reinterpret_cast<uint16_t*>(reinterpret_cast<unsigned char*>(vb) + B * align256(kd) * 2 + 256);
  uint16_t* gb = reinterpret_cast<uint16_t*>(reinterpret_cast<unsigned char*>(ab) + B * align256(qd) * 2 + 256);
  uint16_t* ub = reinterpret_cast<uint16_t*>(reinterpret_cast<unsigned char*>(gb) + B * align256(m->inter) * 2 + 256);
  int64_t rt_max = 0, part_floats = 0;
  int ns = 0;
  int nsplit = std::min(kMaxSplits, std::max(1, G / (B * m->kv_heads)));
  const int gs = m->q_heads / m->kv_heads;
  const uint32_t attn_buf = static_cast<uint32_t>(
      (kMaxGroup * hd + 2 * hd + kStepWarps * gs * (hd + 2)) * 4);
  const bool attn_in_a = !has4 && R.a0 + attn_buf <= R.a1;
  const uint32_t attn_at = attn_in_a ? R.a0 : R.b0;
  if (!attn_in_a && R.b0 + attn_buf > R.b1) return fail(TP_ERR_UNSUPPORTED, "tp_step: attention buffers do not fit");
  for (int i = 0; i < m->layers; ++i) {
    const tp_step_layer& ly = layers[i];
    if (!ly.ln1 || !ly.ln2 || !ly.k_cache || !ly.v_cache) return fail(TP_ERR_ARG, "tp_step: layer %d incomplete", i);
    if (ly.q.n != qd || ly.k.n != kd || ly.v.n != kd || ly.o.d != qd || ly.o.n != m->hidden || ly.q.d != m->hidden ||
        ly.gate.n != m->inter || ly.up.n != m->inter || ly.down.d != m->inter || ly.down.n != m->hidden ||
        ly.gate.d != m->hidden)
      return fail(TP_ERR_ARG, "tp_step: layer %d shapes do not match the model", i);
    // QKV
    {
      StepStage& s = st[ns++];
      s.type = kLinear;
      const tp_step_linear* ops[3] = {&ly.q, &ly.k, &ly.v};
      uint16_t* outs[3] = {qb, kb, vb};
      if (tp_status e = plan_linear(s.lin, ops, outs, 3, B, G, R, &rt_max, &part_floats)) return e;
      s.lin.in_kind = kInRmsNorm;
      s.lin.in0 = m->hidden_state;
      s.lin.gamma = ly.ln1;
      s.lin.eps = m->rms_eps;
      s.lin.epi = kEpiStore;
    }
    // ATTN
    {
      StepStage& s = st[ns++];
      s.type = kAttention;
      AttnStage& A = s.attn;
      A.q = qb;
      A.k = kb;
      A.v = vb;
      A.q_norm = ly.q_norm;
      A.k_norm = ly.k_norm;
      A.k_cache = ly.k_cache;
      A.v_cache = ly.v_cache;
      A.out = ab;
      A.inv_freq = m->inv_freq;
      A.q_heads = m->q_heads;
      A.kv_heads = m->kv_heads;
      A.hd = m->head_dim;
      A.max_t = m->max_tokens;
      A.nsplit = nsplit;
      A.eps = m->rms_eps;
      A.scaling = static_cast<float>(1.0 / std::sqrt(static_cast<double>(hd)));
      A.buf_off = attn_at - R.base;
    }
    // O
    {
      StepStage& s = st[ns++];
      s.type = kLinear;
      const tp_step_linear* ops[1] = {&ly.o};
      uint16_t* outs[1] = {m->hidden_state};
      if (tp_status e = plan_linear(s.lin, ops, outs, 1, B, G, R, &rt_max, &part_floats)) return e;
      s.lin.in_kind = kInPlain;
      s.lin.in0 = ab;
      s.lin.epi = kEpiResidual;
    }
    // GATE / UP
    {
      StepStage& s = st[ns++];
      s.type = kLinear;
      const tp_step_linear* ops[2] = {&ly.gate, &ly.up};
      uint16_t* outs[2] = {gb, ub};
      if (tp_status e = plan_linear(s.lin, ops, outs, 2, B, G, R, &rt_max, &part_floats)) return e;
      s.lin.in_kind = kInRmsNorm;
      s.lin.in0 = m->hidden_state;
      s.lin.gamma = ly.ln2;
      s.lin.eps = m->rms_eps;
      s.lin.epi = kEpiStore;
    }
    // DOWN
    {
      StepStage& s = st[ns++];
      s.type = kLinear;
      const tp_step_linear* ops[1] = {&ly.down};
      uint16_t* outs[1] = {m->hidden_state};
      if (tp_status e = plan_linear(s.lin, ops, outs, 1, B, G, R, &rt_max, &part_floats)) return e;
      s.lin.in_kind = kInSiluMul;
      s.lin.in0 = gb;
      s.lin.in1 = ub;
      s.lin.epi = kEpiResidual;
    }
  }
  {
    StepStage& s = st[ns++];
    s.type = kFinalNorm;
    s.fnorm.x = m->hidden_state;
    s.fnorm.gamma = m->final_norm;
    s.fnorm.out = m->final_out;
    s.fnorm.d = m->hidden;
    s.fnorm.eps = m->rms_eps;
  }
  // the largest footprint over the stages sets the dynamic shared memory size
  uint32_t end = std::max<uint32_t>(has4 ? R.b0 : kLutAbs + 65536u, attn_at + attn_buf);
  for (int s = 0; s < ns; ++s) {
    if (st[s].type != kLinear) continue;
    const LinearStage& L = st[s].lin;
    const int cols = L.us * kUnitCols;
    const bool need_scr = !(L.rs_smem && L.lg_block <= 9);
    const uint32_t sz[4] = {
        static_cast<uint32_t>(((int64_t)L.nops * (B + 1) * (cols + kZPad) * 2 + 127) / 128 * 128),
        static_cast<uint32_t>(((int64_t)L.rpp * cols * 2 + 127) / 128 * 128),
        need_scr ? static_cast<uint32_t>((int64_t)L.rpp * cols * 4) : 0u,
        static_cast<uint32_t>((int64_t)L.rs_smem * L.nops * cols * 2)};
    const uint32_t offs[4] = {L.z_off, L.xin_off, L.scr_off, L.rs_off};
    for (int i = 0; i < 4; ++i)
      if (sz[i]) end = std::max(end, R.base + offs[i] + sz[i]);
  }
  H->nstages = ns;
  H->B = B;
  H->grid = G;
  H->has4 = has4 ? 1 : 0;
  H->base = R.base;
  H->dyn = end - R.base;
  H->lut_off = has4 ? 0 : kLutAbs - R.base;
  H->misc_off = misc_off;
  const int attn_groups = B * m->kv_heads;
  const int64_t counters = std::max<int64_t>(rt_max, attn_groups);
  H->ws_part_off = align256(kWsCounters + counters * 4);
  H->ws_attn_off = H->ws_part_off + align256(part_floats * 4);
  H->ws_bytes = H->ws_attn_off + align256((int64_t)attn_groups * nsplit * gs * (hd + 2) * 4);
  H->max_rt = static_cast<int>(rt_max);
  H->barrier_us = 0;
  H->extra_arrivals = 0;
  H->attn_groups = attn_groups;
  *workspace_bytes = H->ws_bytes;
  return clear_ok();
}

extern "C" tp_status tp_step_run(const void* image_dev, const void* image_host, const int* pos_dev, void* workspace,
                                 int64_t workspace_bytes, void* stream) {
  if (!image_dev || !image_host || !pos_dev || !workspace) return fail(TP_ERR_ARG, "tp_step_run: null argument");
  const StepHeader* H = static_cast<const StepHeader*>(image_host);
  if (workspace_bytes < H->ws_bytes)
    return fail(TP_ERR_WORKSPACE, "tp_step_run: workspace of %lld bytes required", (long long)H->ws_bytes);
  if (!aligned(workspace, 256)) return fail(TP_ERR_ALIGN, "tp_step_run: workspace must be 256-byte aligned");
  if (H->grid != step_sm_count()) return fail(TP_ERR_ARG, "tp_step_run: program built for another device");
  int dev = 0;
  TP_CUDA_TRY(cudaGetDevice(&dev), "cudaGetDevice");
  {
    std::lock_guard<std::mutex> lk(g_step_mu);
    if (dev < 0 || dev >= 64) return fail(TP_ERR_UNSUPPORTED, "device index out of range");
    if (g_step_smem_set[dev] != (int)H->dyn) {
      TP_CUDA_TRY(cudaFuncSetAttribute(step_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)H->dyn),
                  "cudaFuncSetAttribute(step)");
      // ask for the smallest shared-memory carve-out that holds the program,
      // so the rest of the SM's on-chip memory serves as L1 (register spills
      // and the noinline calls' saves stay on chip)
      int smem_sm = 0;
      TP_CUDA_TRY(cudaDeviceGetAttribute(&smem_sm, cudaDevAttrMaxSharedMemoryPerMultiprocessor, dev), "attr");
      const int pct = std::min(100, (int)(((int64_t)(H->dyn + H->base) * 100 + smem_sm - 1) / smem_sm));
      TP_CUDA_TRY(cudaFuncSetAttribute(step_kernel, cudaFuncAttributePreferredSharedMemoryCarveout, pct),
                  "cudaFuncSetAttribute(step carveout)");
      g_step_smem_set[dev] = (int)H->dyn;
    }
  }
  cudaStream_t st = as_stream(stream);
  TP_CUDA_TRY(cudaMemsetAsync(static_cast<unsigned char*>(workspace) + kWsFlags, 0, 4 * kMaxGrid, st),
              "memset(barrier words)");
  const StepHeader* img = static_cast<const StepHeader*>(image_dev);
  unsigned char* ws = static_cast<unsigned char*>(workspace);
  void* args[] = {(void*)&img, (void*)&ws, (void*)&pos_dev};
  TP_CUDA_TRY(cudaLaunchCooperativeKernel((const void*)step_kernel, dim3(H->grid), dim3(kStepThreads), args, H->dyn,
                                          st),
              "step_kernel launch");
  return check_launch("step_kernel");
}

extern "C" tp_status tp_step_set_wait(void* image_host, int64_t barrier_us, int extra_arrivals) {
  if (!image_host || barrier_us < 0 || barrier_us > 60000000 || extra_arrivals < 0)
    return fail(TP_ERR_ARG, "tp_step_set_wait: bad argument");
  StepHeader* H = static_cast<StepHeader*>(image_host);
  H->barrier_us = static_cast<unsigned>(barrier_us);
  H->extra_arrivals = extra_arrivals;
  return clear_ok();
}

extern "C" tp_status tp_step_status(const void* workspace, void* stream) {
  if (!workspace) return fail(TP_ERR_ARG, "tp_step_status: null workspace");
  unsigned v = 0;
  cudaStream_t st = as_stream(stream);
  const unsigned char* ws = static_cast<const unsigned char*>(workspace);
  TP_CUDA_TRY(cudaMemcpyAsync(&v, ws + kWsStatus, 4, cudaMemcpyDeviceToHost, st), "status copy");
  TP_CUDA_TRY(cudaStreamSynchronize(st), "status sync");
  if (v == 0) return clear_ok();
  TP_CUDA_TRY(cudaMemsetAsync(const_cast<unsigned char*>(ws) + kWsStatus, 0, 4, st), "status clear");
  if (v & kStepStatusLayout) return fail(TP_ERR_DEVICE, "tp_step: shared-memory layout check failed (status %u)", v);
  return fail(TP_ERR_DEVICE, "tp_step: a grid barrier timed out (status %u)", v);
}

#ifdef TP_STEP_TRACE
extern "C" TP_API int tp_step_trace_read(unsigned long long* host) {
  return (int)cudaMemcpyFromSymbol(host, tp::g_step_trace, sizeof(tp::g_step_trace));
}
#endif

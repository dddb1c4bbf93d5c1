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

// workspace words
constexpr int64_t kWsStatus = 64;      // status bits (kStepStatus*)
constexpr int64_t kWsLayout = 128;     // [acc offset, acc bytes] (int64), written by every run
constexpr int64_t kWsFlags = 1024;     // grid barrier counter (zeroed before each run)
constexpr int kMaxGrid = 512;
constexpr int64_t kWsCounters = kWsFlags + 4 * kMaxGrid;  // per-attention-group counters
constexpr unsigned kStepStatusLayout = 1u, kStepStatusBarrier = 2u;
// pointer fields of a built image that name workspace buffers hold
// kWsTag | offset until tp_step_bind resolves them
constexpr uintptr_t kWsTag = uintptr_t(1) << 62;

// A linear op writes raw fp32 dot products (before its row scale) into an
// accumulator with red.add; the stages that read the op's output apply
// scale / bias and the fp16 rounding of the reference there.
struct alignas(16) StepOp {
  const unsigned char* stream;
  float* acc;  // fp32 [B][n], zero before the stage
  const uint16_t* rot_scale;
  int n, row_tiles, rt_off, pad;
};

// An input vector of a stage: r16(base + r16(acc * scale + bias)) with the
// terms that are present (base alone: a plain fp16 input).
struct alignas(16) InVec {
  const uint16_t* base;   // fp16 [B][d] or null
  const float* acc;       // fp32 [B][d] or null
  const uint16_t* scale;  // fp16 [d] (with acc)
  const uint16_t* bias;   // fp16 [d] or null
};

struct alignas(16) LinearStage {
  const uint16_t* codebook;
  const uint16_t* gamma;  // [d] fp16 norm weight
  uint16_t* hout;         // norm input: the reconstructed residual is written here
  InVec in[2];            // plain / norm: in[0]; SiLU product: gate in[0], up in[1]
  int nops, in_kind, bits, d;
  int d_pad, units_k, lg_block, kparts;
  float norm, eps;
  int us, cps, rt_total, rpp, rs_smem, nin, pad2[2];
  // shared-memory offsets from the dynamic base: activations, input rows,
  // fp32 scratch, rotation scales, norm weight, producer scales
  uint32_t z_off, xin_off, scr_off, rs_off, gam_off, psc_off, stg_off, pad3;
  SliceSplit split[2];
  StepOp ops[kMaxStageOps];
};

struct alignas(16) AttnStage {
  InVec q, k, v;  // q_proj / k_proj / v_proj outputs (accumulators + scales)
  const uint16_t* q_norm;  // [hd] or null
  const uint16_t* k_norm;
  uint16_t* k_cache;  // [B][kv_heads][max_t][hd]
  uint16_t* v_cache;
  uint16_t* out;  // [B][q_heads*hd]
  const float* inv_freq;  // [hd/2]
  const uint16_t* rope_cos;  // [max_t][hd/2] fp16 or null (then computed)
  const uint16_t* rope_sin;
  int q_heads, kv_heads, hd, max_t;
  int nsplit;
  float eps, scaling;
  uint32_t buf_off;
};

struct alignas(16) NormStage {
  InVec x;  // residual base + down_proj accumulator
  const uint16_t* gamma;
  uint16_t* out;
  uint16_t* hout;  // the final residual stream
  int d;
  float eps;
  uint32_t buf_off;  // fp16 [d] row buffer in shared memory
};

struct alignas(16) StepStage {
  int type, nzero, pad[2];
  // buffers every CTA clears (grid-stride) at the start of the stage: the
  // accumulators whose readers finished in an earlier stage
  float* zero_ptr[2];
  int64_t zero_bytes[2];
  union {
    LinearStage lin;
    AttnStage attn;
    NormStage fnorm;
  };
};

struct alignas(16) StepHeader {
  int nstages, B, grid, has4;
  uint32_t base, dyn, lut_off, misc_off;
  int64_t ws_acc_off, ws_acc_bytes, ws_attn_off, ws_h2_off, ws_bytes;
  int attn_groups, pad0;
  uint64_t bound_ws;  // the workspace tp_step_bind resolved the image's workspace pointers against
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
static_assert(kMiscBytes <= 3072, "stage records");

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
// Arrival: after a CTA barrier (every thread's writes of the stage are
// done), thread 0 adds one with release semantics at GPU scope (a reduction:
// it does not wait for the add to complete, so the CTA goes on with work that
// does not depend on the barrier).
__device__ __forceinline__ void grid_arrive(unsigned* bar) {
  __syncthreads();
  if (threadIdx.x == 0) asm volatile("red.release.gpu.global.add.u32 [%0], 1;" ::"l"(bar) : "memory");
}

// Wait: thread 0 spins on acquire loads until the counter reaches `target`.
__device__ bool grid_wait(unsigned* bar, unsigned* status, unsigned target, unsigned long long limit_ns, int* s_ok) {
  if (threadIdx.x == 0) {
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
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
__device__ __forceinline__ void cp_async_wait_group1() { asm volatile("cp.async.wait_group 1;" ::: "memory"); }

__device__ __forceinline__ void unpack8(uint4 v, float* f) {
  const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
  for (int e = 0; e < 4; ++e) {
    const float2 t = __half22float2(*reinterpret_cast<const __half2*>(&w[e]));
    f[2 * e] = t.x;
    f[2 * e + 1] = t.y;
  }
}
__device__ __forceinline__ uint4 pack8(const float* f) {
  uint32_t w[4];
#pragma unroll
  for (int e = 0; e < 4; ++e) {
    const __half2 h = __floats2half2_rn(f[2 * e], f[2 * e + 1]);
    w[e] = *reinterpret_cast<const uint32_t*>(&h);
  }
  return make_uint4(w[0], w[1], w[2], w[3]);
}

// Raw loads of one 8-column chunk of an input vector (row offset `ro`,
// column c): the dynamic parts (base, accumulator) come from L2 (.cg: other
// SMs wrote them during this launch); scales from shared memory (`ssc`,
// staged before the stage's barrier) or global; bias from global.
struct ChunkRaw {
  uint4 base;
  float4 a0, a1;
};
// BASE / ACC: which terms the vector has (fixed per call site, so the
// registers of absent terms are not kept)
template <bool BASE, bool ACC>
__device__ __forceinline__ void load_chunk(const InVec& V, int64_t ro, int c, ChunkRaw& r) {
  if constexpr (BASE) r.base = __ldcg(reinterpret_cast<const uint4*>(V.base + ro + c));
  if constexpr (ACC) {
    r.a0 = __ldcg(reinterpret_cast<const float4*>(V.acc + ro + c));
    r.a1 = __ldcg(reinterpret_cast<const float4*>(V.acc + ro + c + 4));
  }
}
// the vector's 8 values (fp16-exact floats): r16(base + r16(acc * scale + bias));
// scales at ssc[cs..], bias at global column cg
template <bool BASE, bool ACC>
__device__ __forceinline__ void finish_chunk(const InVec& V, const ChunkRaw& r, const uint16_t* ssc, int cs, int cg,
                                             float* f) {
  float b[8];
  if constexpr (BASE) unpack8(r.base, b);
  if constexpr (ACC) {
    float sc[8], bi[8];
    unpack8(*reinterpret_cast<const uint4*>(ssc + cs), sc);
    const bool hb = V.bias != nullptr;
    if (hb) unpack8(*reinterpret_cast<const uint4*>(V.bias + cg), bi);
    const float a[8] = {r.a0.x, r.a0.y, r.a0.z, r.a0.w, r.a1.x, r.a1.y, r.a1.z, r.a1.w};
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      float o = a[e] * sc[e];
      if (hb) o += bi[e];
      f[e] = BASE ? r16(b[e] + r16(o)) : r16(o);
    }
  } else {
#pragma unroll
    for (int e = 0; e < 8; ++e) f[e] = b[e];
  }
}

// Bytes per column and row of a stage's input staging area: fp16 base,
// fp32 accumulator(s); a plain input is copied straight into xin.
__host__ __device__ __forceinline__ int stage_bytes_per_col(int in_kind, int nin) {
  return in_kind == kInSiluMul ? 8 : in_kind == kInRmsNorm ? 2 + 4 * nin : 0;
}

// Input transform of rows [b0, b0+rows) over slice columns [c0, c0+cols):
// xin (fp16 bits, [rows][cols]) holds
//   plain:    the input row;
//   RMS norm: the residual h = r16(base + r16(acc*scale + bias)) (the norm
//             itself, r16(gamma * r16(h * rinv)), is applied by the rotation
//             with rinv[row] from here); h is also written back to L.hout,
//             each CTA of the K-slice writing its share of the chunks;
//   SiLU:     r16(r16(silu(gate)) * up).
// The dynamic inputs (base rows, accumulators: written by other SMs in
// earlier stages) come into a shared-memory staging area with cp.async, all
// copies in flight at once (one memory round trip, no registers held); the
// transform then reads shared memory.  Warps split over the rows (fixed
// order: deterministic sums).
template <int KIND, bool ACC>
__device__ __forceinline__ void stage_input_k(const LinearStage& L, int b0, int rows, int c0, int cols, uint16_t* xin,
                                              float* red, unsigned char* smem) {
  constexpr bool norm = KIND == kInRmsNorm, silu = KIND == kInSiluMul;
  constexpr bool BASE = KIND != kInSiluMul;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  float* rinv = red + kStepMaxBatch * kStepWarps;
  const int n8 = cols >> 3;
  unsigned char* stg = smem + L.stg_off;
  uint16_t* sb = KIND == kInPlain ? xin : reinterpret_cast<uint16_t*>(stg);
  float* sa0 = reinterpret_cast<float*>(stg + (BASE ? rows * cols * 2 : 0));
  float* sa1 = sa0 + rows * cols;
  for (int i = tid; i < rows * n8; i += kStepThreads) {
    const int r = i / n8, ci = i - r * n8, c = c0 + ci * 8;
    const bool v = c < L.d;
    const int64_t g = (int64_t)(b0 + r) * L.d + (v ? c : 0);
    const int o = r * cols + ci * 8;
    if constexpr (BASE) cp_async16(sb + o, L.in[0].base + g, v);
    if constexpr (ACC) {
      cp_async16(sa0 + o, L.in[0].acc + g, v);
      cp_async16(sa0 + o + 4, L.in[0].acc + g + 4, v);
    }
    if constexpr (silu) {
      cp_async16(sa1 + o, L.in[1].acc + g, v);
      cp_async16(sa1 + o + 4, L.in[1].acc + g + 4, v);
    }
  }
  cp_async_commit();
  // the staging copies, the stage's static vectors (issued before its
  // barrier) and the stage record in flight
  cp_async_wait_all();
  __syncthreads();
  if constexpr (KIND == kInPlain) return;
  const int wpr = kStepWarps / rows, row = warp / wpr, sub = warp - row * wpr;
  const bool act = row < rows;
  const int64_t xrow = (int64_t)(b0 + (act ? row : 0)) * L.d;
  const int stride = wpr * 32;
  const uint16_t* psc = reinterpret_cast<const uint16_t*>(smem + L.psc_off);
  // CTAs of this K-slice share the write-back of h
  const int slice = blockIdx.x / L.cps, cta_in = blockIdx.x - slice * L.cps;
  float ssum = 0.f;
  for (int ci = sub * 32 + lane; act && ci < n8; ci += stride) {
    const int c = c0 + ci * 8, o = row * cols + ci * 8;
    ChunkRaw r0, r1;
    if constexpr (BASE) r0.base = *reinterpret_cast<const uint4*>(sb + o);
    if constexpr (ACC) {
      r0.a0 = *reinterpret_cast<const float4*>(sa0 + o);
      r0.a1 = *reinterpret_cast<const float4*>(sa0 + o + 4);
    }
    if constexpr (silu) {
      r1.a0 = *reinterpret_cast<const float4*>(sa1 + o);
      r1.a1 = *reinterpret_cast<const float4*>(sa1 + o + 4);
    }
    uint4 ov = make_uint4(0u, 0u, 0u, 0u);
    if (c < L.d) {
      float f[8];
      finish_chunk<BASE, ACC>(L.in[0], r0, psc, ci * 8, c, f);
      if constexpr (silu) {
        float up[8];
        finish_chunk<false, true>(L.in[1], r1, psc + cols, ci * 8, c, up);
#pragma unroll
        for (int e = 0; e < 8; ++e) f[e] = r16(r16(f[e] / (1.f + __expf(-f[e]))) * up[e]);
      }
      ov = pack8(f);
      if constexpr (norm) {
#pragma unroll
        for (int e = 0; e < 8; ++e) ssum = fmaf(f[e], f[e], ssum);
        if (L.hout && ci % L.cps == cta_in) *reinterpret_cast<uint4*>(L.hout + xrow + c) = ov;
      }
    }
    *reinterpret_cast<uint4*>(xin + row * cols + ci * 8) = ov;
  }
  if constexpr (norm) {
    if (cols != L.d) {
      // K-split: the sum of squares needs the whole row (scales from global)
      ssum = 0.f;
      for (int cb = sub * 32 + lane; act && cb < (L.d >> 3); cb += stride) {
        ChunkRaw r0;
        load_chunk<BASE, ACC>(L.in[0], xrow, cb * 8, r0);
        float f[8];
        finish_chunk<BASE, ACC>(L.in[0], r0, L.in[0].scale, cb * 8, cb * 8, f);
#pragma unroll
        for (int e = 0; e < 8; ++e) ssum = fmaf(f[e], f[e], ssum);
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
  }
  __syncthreads();
}

__device__ __forceinline__ void stage_input(const LinearStage& L, int b0, int rows, int c0, int cols, uint16_t* xin,
                                            float* red, unsigned char* smem) {
  if (L.in_kind == kInRmsNorm) {
    if (L.in[0].acc) stage_input_k<kInRmsNorm, true>(L, b0, rows, c0, cols, xin, red, smem);
    else stage_input_k<kInRmsNorm, false>(L, b0, rows, c0, cols, xin, red, smem);
  } else if (L.in_kind == kInSiluMul) {
    stage_input_k<kInSiluMul, true>(L, b0, rows, c0, cols, xin, red, smem);
  } else {
    stage_input_k<kInPlain, false>(L, b0, rows, c0, cols, xin, red, smem);
  }
}

// x of one rotation input chunk: the staged value, normed for RMS-norm stages
__device__ __forceinline__ void rot_input8(const LinearStage& L, uint4 xv, const uint16_t* gam, float r, float* v) {
  unpack8(xv, v);
  if (L.in_kind == kInRmsNorm) {
    float g[8];
    unpack8(*reinterpret_cast<const uint4*>(gam), g);
#pragma unroll
    for (int e = 0; e < 8; ++e) v[e] = r16(g[e] * r16(v[e] * r));
  }
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
                             int cols, float* scr, __half* z, int zst, const uint16_t* gam, const float* rinv) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int lg = L.lg_block, tpr = cols >> 8;
  for (int k = warp; k < rows * tpr; k += kStepWarps) {
    const int rr = k / tpr, cl = (k - rr * tpr) * 256 + lane * 8;
    float v[8], rf[8];
    rot_input8(L, *reinterpret_cast<const uint4*>(xin + rr * cols + cl), gam + cl, rinv[rr], v);
    // slice-local scales (shared memory: zero past d; global: guarded)
    uint4 rv = make_uint4(0u, 0u, 0u, 0u);
    if (L.rs_smem || c0 + cl < L.d) rv = *reinterpret_cast<const uint4*>(rs + cl);
    unpack8(rv, rf);
#pragma unroll
    for (int e = 0; e < 8; ++e) v[e] *= rf[e];
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
                                                    __half* z, int zst, const uint16_t* gam, const float* rinv) {
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
      float rf[8];
      rot_input8(L, *reinterpret_cast<const uint4*>(xin + rr * cols + cl + 8 * q), gam + cl + 8 * q, rinv[rr],
                 v + 8 * q);
      uint4 rv = make_uint4(0u, 0u, 0u, 0u);
      if (L.rs_smem || c0 + cl + 8 * q < L.d) rv = *reinterpret_cast<const uint4*>(rs + cl + 8 * q);
      unpack8(rv, rf);
#pragma unroll
      for (int e = 0; e < 8; ++e) v[8 * q + e] *= rf[e];
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

// Static vectors of a linear stage into shared memory (cp.async, one commit
// group, waited for in stage_input): every op's rotation scales, the norm
// weight and the producer scales of accumulator inputs.  Issued before the
// barrier that precedes the stage: they depend on nothing it orders.
__device__ void stage_static_prefetch(const LinearStage& L, unsigned char* smem) {
  const int slice = blockIdx.x / L.cps;
  if (slice < L.kparts) {
    const int Us = L.split[slice == L.kparts - 1 ? 1 : 0].us;
    const int cols = Us * kUnitCols, c0 = slice * L.us * kUnitCols, n8 = cols / 8;
    uint16_t* rs_s = reinterpret_cast<uint16_t*>(smem + L.rs_off);
    uint16_t* gam_s = reinterpret_cast<uint16_t*>(smem + L.gam_off);
    uint16_t* psc_s = reinterpret_cast<uint16_t*>(smem + L.psc_off);
    const bool gam = L.in_kind == kInRmsNorm;
    const int nrs = L.rs_smem ? L.nops : 0;
    const int nv = nrs + (gam ? 1 : 0) + L.nin;
    for (int i = threadIdx.x; i < nv * n8; i += kStepThreads) {
      const int k = i / n8, ci = i - k * n8, c = c0 + ci * 8;
      const bool valid = c < L.d;
      const uint16_t* src;
      uint16_t* dst;
      if (k < nrs) {
        src = L.ops[k].rot_scale;
        dst = rs_s + k * cols;
      } else if (gam && k == nrs) {
        src = L.gamma;
        dst = gam_s;
      } else {
        const int j = k - nrs - (gam ? 1 : 0);
        src = L.in[j].scale;
        dst = psc_s + j * cols;
      }
      cp_async16(dst + ci * 8, src + (valid ? c : 0), valid);
    }
  }
  cp_async_commit();
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
  const uint16_t* gam = reinterpret_cast<const uint16_t*>(smem + L.gam_off);
  const float* rinv = red + kStepMaxBatch * kStepWarps;
  for (int b0 = 0; b0 < B; b0 += L.rpp) {
    const int rows = min(L.rpp, B - b0);
    stage_input(L, b0, rows, c0, cols, xin, red, smem);
    step_mark(4);
    if (L.lg_block <= 9 && L.rs_smem) {
      if (L.lg_block == 9) rotate_small_blocks<16>(L, rs_s, cols, xin, rows, b0, B, c0, cols, z, zst, gam, rinv);
      else rotate_small_blocks<8>(L, rs_s, cols, xin, rows, b0, B, c0, cols, z, zst, gam, rinv);
    } else {
      for (int k = 0; k < L.nops; ++k)
        stage_rotate(L, L.rs_smem ? rs_s + k * cols : L.ops[k].rot_scale + c0, xin, rows, c0, cols, scr,
                     z + (k * (B + 1) + b0) * zst, zst, gam, rinv);
    }
  }
  step_mark(5);
  for (int i = tid; i < L.nops * (cols / 8); i += kStepThreads) {
    const int k = i / (cols / 8), r = i - k * (cols / 8);
    reinterpret_cast<uint4*>(z + (k * (B + 1) + B) * zst)[r] = make_uint4(0u, 0u, 0u, 0u);
  }
  __syncthreads();
}

// This warp's first weight unit of a linear stage and the trellis halo
// before it (issued before the stage's barrier: the weights depend on
// nothing it orders).
__device__ __forceinline__ void preload_first(const LinearStage& L, uint4* pre, uint32_t& hg, uint32_t& hq) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  hg = hq = 0u;
  const int slice = blockIdx.x / L.cps;
  if (slice >= L.kparts) return;
  const int wl = warp * L.cps + (blockIdx.x - slice * L.cps);
  const SliceSplit& sp = L.split[slice == L.kparts - 1 ? 1 : 0];
  if (wl >= sp.nw) return;
  const int j0 = sp.start(wl);
  if (j0 >= sp.start(wl + 1)) return;
  const int rt = sp.row_tile(j0), ul = j0 - rt * sp.us;
  int k = 0;
  while (k + 1 < L.nops && rt >= L.ops[k + 1].rt_off) ++k;
  const int64_t UB = 512 * L.bits;
  const int us0 = slice * L.us;
  const unsigned char* u = L.ops[k].stream + ((int64_t)(rt - L.ops[k].rt_off) * L.units_k + us0 + ul) * UB;
  const uint4* src = reinterpret_cast<const uint4*>(u) + lane * L.bits;
#pragma unroll
  for (int q = 0; q < 4; ++q)
    if (q < L.bits) pre[q] = ldg_stream(src + q);
  if (us0 + ul > 0) {
    const uint4 pv = ldg_stream(reinterpret_cast<const uint4*>(u - UB) + lane * L.bits);
    hg = pv.z;
    hq = pv.w;
  }
}

template <int BITS>
__device__ __forceinline__ void linear_stage(const LinearStage& L, unsigned char* smem, int B, const unsigned char* lut,
                                             int sidx, const uint4* pre, uint32_t pre_hg, uint32_t pre_hq) {
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

  // ---- first unit of the run and its trellis halo: loaded by
  // preload_first before the barrier that preceded the stage ----
  int rt = sp.row_tile(j0), ul = j0 - rt * Us;
  int opk = op_of(rt);
  uint4 wa[BITS];
#pragma unroll
  for (int k = 0; k < BITS; ++k) wa[k] = pre[k];
  uint32_t hg = pre_hg, hq = pre_hq, hng = 0u, hnq = 0u;
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
  // a finished (row tile, K range): its raw sums are added to the op's fp32
  // accumulator (red.add, no ordering needed before the stage's barrier)
  auto flush = [&](int frt, int k) {
    step_mark(6);
    const StepOp& op = L.ops[k];
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const float v = acc[0][e] + acc[1][e];
      const int col = 2 * t + (e & 1);
      const int row = (frt - op.rt_off) * kTileRows + g + 8 * (e >> 1);
      if (col < B && row < op.n) atomicAdd(op.acc + (int64_t)col * op.n + row, v);
    }
#pragma unroll
    for (int q = 0; q < 2; ++q) acc[q][0] = acc[q][1] = acc[q][2] = acc[q][3] = 0.f;
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
// hold the first half): fp16(fp16(x*cos) + fp16(rot*sin)) with the fp16 cos /
// sin of the fp32 angle pos * inv_freq (c, s: this lane's E values).
template <int E>
__device__ __forceinline__ void rope(float* x, const float* c, const float* sn, int lane) {
  float partner[E];
#pragma unroll
  for (int e = 0; e < E; ++e) partner[e] = __shfl_xor_sync(0xffffffffu, x[e], 16);
  const bool hi = lane >= 16;
#pragma unroll
  for (int e = 0; e < E; ++e) {
    const float rot = hi ? partner[e] : -partner[e];
    x[e] = r16(r16(x[e] * c[e]) + r16(rot * sn[e]));
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
// E fp16 values as raw bits (one 8- or 4-byte load), converted later
template <int E>
struct HRaw {
  uint32_t w[E / 2];
};
template <int E>
__device__ __forceinline__ HRaw<E> ld_hraw(const uint16_t* p) {
  HRaw<E> r;
  if constexpr (E == 4) {
    const uint2 v = *reinterpret_cast<const uint2*>(p);
    r.w[0] = v.x, r.w[1] = v.y;
  } else {
    r.w[0] = *reinterpret_cast<const uint32_t*>(p);
  }
  return r;
}
template <int E>
__device__ __forceinline__ void cvt_hraw(const HRaw<E>& r, float* v) {
#pragma unroll
  for (int i = 0; i < E / 2; ++i) {
    const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&r.w[i]));
    v[2 * i] = f.x, v[2 * i + 1] = f.y;
  }
}

// One head vector of a projection output from its accumulator: E values of
// r16(acc * scale + bias) at column `col` of batch row b.
template <int E>
struct ProjRaw {
  float a[E];
  HRaw<E> sc, bi;
};
template <int E>
__device__ __forceinline__ void proj_load(const InVec& V, int64_t row_off, int col, ProjRaw<E>& r) {
  if constexpr (E == 4) {
    const float4 v = __ldcg(reinterpret_cast<const float4*>(V.acc + row_off + col));
    r.a[0] = v.x, r.a[1] = v.y, r.a[2] = v.z, r.a[3] = v.w;
  } else {
    const float2 v = __ldcg(reinterpret_cast<const float2*>(V.acc + row_off + col));
    r.a[0] = v.x, r.a[1] = v.y;
  }
  r.sc = ld_hraw<E>(V.scale + col);
  if (V.bias) r.bi = ld_hraw<E>(V.bias + col);
}
template <int E>
__device__ __forceinline__ void proj_finish(const InVec& V, const ProjRaw<E>& r, float* x) {
  float sc[E], bi[E];
  cvt_hraw<E>(r.sc, sc);
  if (V.bias) cvt_hraw<E>(r.bi, bi);
#pragma unroll
  for (int e = 0; e < E; ++e) x[e] = r16(V.bias ? r.a[e] * sc[e] + bi[e] : r.a[e] * sc[e]);
}

constexpr int kTok = 4;  // cached tokens per warp in flight

// One attention item: batch row b, kv head kvh, split sp of the positions
// [0, pos]: the q heads of the group (head norm, RoPE), the new token's k / v
// (appended to the caches by the split that owns position pos), an online
// softmax per warp over its tokens (kTok in flight, the next kTok loading
// while these are used), the warps combined in shared memory, the split's
// (max, sum, weighted values) written to the workspace; the last split of the
// group to finish combines all splits into the fp16 output.
template <int E, int G>
__device__ __noinline__ void attn_item(const AttnStage& A, int b, int kvh, int sp, int pos, unsigned char* buf,
                                          float* part, unsigned* counters, int cgroup, unsigned* s_last) {
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int hd = A.hd, gs = G;  // G: the exact query heads per kv head
  constexpr int kT = G >= 8 ? 2 : kTok;  // cached tokens per warp in flight
  float* sq = reinterpret_cast<float*>(buf);                 // [gs][hd] normed, roped q
  float* knew = sq + kMaxGroup * hd;                         // [hd]
  float* vnew = knew + hd;                                   // [hd]
  float* wst = vnew + hd;                                    // [16 warps][gs][hd + 2]
  const int T = pos + 1, Ls = (T + A.nsplit - 1) / A.nsplit;
  const int t0 = sp * Ls, t1 = min(T, t0 + Ls);
  const int64_t kv0 = ((int64_t)b * A.kv_heads + kvh) * A.max_t;
  // this warp's first cached tokens, loaded before anything waits
  HRaw<E> kr[kT], vr[kT];
#define TP_ATTN_LOAD(K, V, FIRST)                                \
  _Pragma("unroll") for (int i = 0; i < kT; ++i) {             \
    const int tk = (FIRST) + i * kStepWarps;                     \
    if (tk < t1 && tk != pos) {                                  \
      K[i] = ld_hraw<E>(A.k_cache + (kv0 + tk) * hd + lane * E); \
      V[i] = ld_hraw<E>(A.v_cache + (kv0 + tk) * hd + lane * E); \
    }                                                            \
  }
  TP_ATTN_LOAD(kr, vr, t0 + warp)
  // q heads of the group (one warp per head) and the new token's k / v
  const bool newtok = t1 == T && t0 < t1;
  if (warp < gs || (warp == kStepWarps - 1 && newtok)) {
    const bool isq = warp < gs;
    const InVec& P = isq ? A.q : A.k;
    const int col = (isq ? (kvh * gs + warp) * hd : kvh * hd) + lane * E;
    const int64_t ro = (int64_t)b * (isq ? A.q_heads : A.kv_heads) * hd;
    const uint16_t* gam = isq ? A.q_norm : A.k_norm;
    ProjRaw<E> pr, vrw;
    HRaw<E> gr, cr, sr;
    proj_load<E>(P, ro, col, pr);
    if (!isq) proj_load<E>(A.v, ro, col, vrw);
    if (gam) gr = ld_hraw<E>(gam + lane * E);
    const int fo = (lane & 15) * E;
    if (A.rope_cos) {
      cr = ld_hraw<E>(A.rope_cos + (int64_t)pos * (hd / 2) + fo);
      sr = ld_hraw<E>(A.rope_sin + (int64_t)pos * (hd / 2) + fo);
    }
    float x[E], c[E], sn[E];
    proj_finish<E>(P, pr, x);
    if (A.rope_cos) {
      cvt_hraw<E>(cr, c);
      cvt_hraw<E>(sr, sn);
    } else {
#pragma unroll
      for (int e = 0; e < E; ++e) {
        const float f = (float)pos * A.inv_freq[fo + e];
        c[e] = r16(cosf(f));
        sn[e] = r16(sinf(f));
      }
    }
    if (gam) {
      float gm[E];
      cvt_hraw<E>(gr, gm);
      head_norm<E>(x, gm, hd, A.eps);
    }
    rope<E>(x, c, sn, lane);
    if (isq) {
#pragma unroll
      for (int e = 0; e < E; ++e) sq[warp * hd + lane * E + e] = x[e];
    } else {
      float vv[E];
      proj_finish<E>(A.v, vrw, vv);
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
  float m[G], l[G], acc[G][E];
#pragma unroll
  for (int j = 0; j < G; ++j) {
    m[j] = -INFINITY;
    l[j] = 0.f;
#pragma unroll
    for (int e = 0; e < E; ++e) acc[j][e] = 0.f;
  }
  for (int first = t0 + warp; first < t1; first += kT * kStepWarps) {
    // the next tokens load while these are used
    HRaw<E> kn[kT], vn[kT];
    TP_ATTN_LOAD(kn, vn, first + kT * kStepWarps)
    // the chunk's tokens (past t1: masked) -- every (token, head) score
    // reduced together, then one online-softmax rescale per head
    float kx[kT][E], vx[kT][E];
    bool valid[kT];
#pragma unroll
    for (int i = 0; i < kT; ++i) {
      const int tk = first + i * kStepWarps;
      valid[i] = tk < t1;
      if (!valid[i]) {  // masked below; its registers hold no loaded data
#pragma unroll
        for (int e = 0; e < E; ++e) kx[i][e] = vx[i][e] = 0.f;
      } else if (tk == pos) {
#pragma unroll
        for (int e = 0; e < E; ++e) kx[i][e] = knew[lane * E + e], vx[i][e] = vnew[lane * E + e];
      } else {
        cvt_hraw<E>(kr[i], kx[i]);
        cvt_hraw<E>(vr[i], vx[i]);
      }
    }
    float sc[kT][G];
#pragma unroll
    for (int j = 0; j < G; ++j) {
      float qv[E];
      if constexpr (E == 4) {
        const float4 q4 = *reinterpret_cast<const float4*>(sq + j * hd + lane * 4);
        qv[0] = q4.x, qv[1] = q4.y, qv[2] = q4.z, qv[3] = q4.w;
      } else {
        const float2 q2 = *reinterpret_cast<const float2*>(sq + j * hd + lane * 2);
        qv[0] = q2.x, qv[1] = q2.y;
      }
#pragma unroll
      for (int i = 0; i < kT; ++i) {
        float d = 0.f;
#pragma unroll
        for (int e = 0; e < E; ++e) d = fmaf(qv[e], kx[i][e], d);
        sc[i][j] = d;
      }
    }
#pragma unroll
    for (int o = 16; o; o >>= 1)
#pragma unroll
      for (int i = 0; i < kT; ++i)
#pragma unroll
        for (int j = 0; j < G; ++j) sc[i][j] += __shfl_xor_sync(0xffffffffu, sc[i][j], o);
#pragma unroll
    for (int j = 0; j < G; ++j) {
      // the reference's fp16 scores: fp16(q.k), then fp16(* scaling)
      float mx = m[j];
#pragma unroll
      for (int i = 0; i < kT; ++i) {
        sc[i][j] = valid[i] ? r16(r16(sc[i][j]) * A.scaling) : -INFINITY;
        mx = fmaxf(mx, sc[i][j]);
      }
      const float corr = m[j] == -INFINITY ? 0.f : __expf(m[j] - mx);
      float lsum = l[j] * corr;
#pragma unroll
      for (int e = 0; e < E; ++e) acc[j][e] *= corr;
#pragma unroll
      for (int i = 0; i < kT; ++i) {
        const float p = valid[i] ? __expf(sc[i][j] - mx) : 0.f;
        lsum += p;
#pragma unroll
        for (int e = 0; e < E; ++e) acc[j][e] = fmaf(p, vx[i][e], acc[j][e]);
      }
      l[j] = lsum;
      m[j] = mx;
    }
#pragma unroll
    for (int i = 0; i < kT; ++i) kr[i] = kn[i], vr[i] = vn[i];
  }
#undef TP_ATTN_LOAD
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
  // the last CTA of the (b, kvh) group combines the splits: one acq_rel
  // add by thread 0 after the CTA barrier publishes this split's partials
  // (release, cumulative over the CTA's writes) and, for the last split,
  // orders its reads of the others' partials (acquire)
  __syncthreads();
  if (tid == 0) {
    unsigned old;
    asm volatile("atom.acq_rel.gpu.global.add.u32 %0, [%1], 1;" : "=r"(old) : "l"(&counters[cgroup]) : "memory");
    *s_last = old == (unsigned)(A.nsplit - 1) ? 1u : 0u;
  }
  __syncthreads();
  step_mark(6);
  if (!*s_last) return;
  // warp w: head j = w % gs, a 1 / (16 / gs) share of its columns; lane s
  // holds split s's max and sum, every lane its columns of all splits (all
  // loads in flight at once)
  const float* gp = part + (int64_t)cgroup * A.nsplit * gs * ws_;
  const int wph = kStepWarps / gs, j = warp % gs, quarter = warp / gs;
  const int per = hd / wph;  // columns per warp: 8 .. 64
  const int dd0 = quarter * per;
  float ms = -INFINITY, ls = 0.f;
  if (lane < A.nsplit) {
    ms = __ldcg(gp + (lane * gs + j) * ws_);
    ls = __ldcg(gp + (lane * gs + j) * ws_ + 1);
  }
  // every split's value of this lane's column (dd0 + h + lane) in flight
  // together with the split maxima and sums: one memory round trip per 32
  // columns of the warp
  for (int h = 0; h < per; h += 32) {
    const bool on = lane + h < per;
    float av[kMaxSplits];
#pragma unroll
    for (int s2 = 0; s2 < kMaxSplits; ++s2)
      av[s2] = s2 < A.nsplit && on ? __ldcg(gp + (s2 * gs + j) * ws_ + 2 + dd0 + h + lane) : 0.f;
    float M = ms;
    for (int o = 16; o; o >>= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, o));
    const float fs = ms == -INFINITY ? 0.f : __expf(ms - M);
    float Lsum = fs * ls;
    for (int o = 16; o; o >>= 1) Lsum += __shfl_xor_sync(0xffffffffu, Lsum, o);
    float ao = 0.f;
#pragma unroll
    for (int s2 = 0; s2 < kMaxSplits; ++s2) ao = fmaf(__shfl_sync(0xffffffffu, fs, s2), av[s2], ao);
    if (on) A.out[(int64_t)b * A.q_heads * hd + (kvh * gs + j) * hd + dd0 + h + lane] = f2h(ao / Lsum);
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
#define TP_ATTN_CALL(E_)                                                                        \
  switch (gs) {                                                                                 \
    case 1: attn_item<E_, 1>(A, b, kvh, sp, pos, buf, part, counters, grp, s_last); break;       \
    case 2: attn_item<E_, 2>(A, b, kvh, sp, pos, buf, part, counters, grp, s_last); break;       \
    case 4: attn_item<E_, 4>(A, b, kvh, sp, pos, buf, part, counters, grp, s_last); break;       \
    default: attn_item<E_, 8>(A, b, kvh, sp, pos, buf, part, counters, grp, s_last); break;      \
  }
    if (A.hd == 128) {
      TP_ATTN_CALL(4)
    } else {
      TP_ATTN_CALL(2)
    }
#undef TP_ATTN_CALL
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

// Final stage: h = r16(base + r16(acc * scale + bias)) (the last down_proj
// added to the residual), written to hout; out = r16(gamma * r16(h * rinv)).
// One CTA per batch row; it also clears the row of the accumulator it read.
__device__ void final_norm_stage(const NormStage& N, int B, float* red, uint16_t* hbuf) {
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  for (int b = blockIdx.x; b < B; b += gridDim.x) {
    const int64_t ro = (int64_t)b * N.d;
    float s = 0.f;
    for (int c = tid * 8; c < N.d; c += kStepThreads * 8) {
      ChunkRaw r;
      load_chunk<true, true>(N.x, ro, c, r);
      float f[8];
      finish_chunk<true, true>(N.x, r, N.x.scale, c, c, f);
#pragma unroll
      for (int e = 0; e < 8; ++e) s = fmaf(f[e], f[e], s);
      *reinterpret_cast<uint4*>(hbuf + c) = pack8(f);
      if (N.x.acc) {
        __stcg(reinterpret_cast<float4*>(const_cast<float*>(N.x.acc) + ro + c), make_float4(0.f, 0.f, 0.f, 0.f));
        __stcg(reinterpret_cast<float4*>(const_cast<float*>(N.x.acc) + ro + c + 4), make_float4(0.f, 0.f, 0.f, 0.f));
      }
    }
    for (int o = 16; o; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    if (lane == 0) red[warp] = s;
    __syncthreads();
    float tot = 0.f;
    for (int w = 0; w < kStepWarps; ++w) tot += red[w];
    const float r = rsqrtf(tot / (float)N.d + N.eps);
    for (int c = tid * 8; c < N.d; c += kStepThreads * 8) {
      float h[8], g[8], o[8];
      const uint4 hv = *reinterpret_cast<const uint4*>(hbuf + c);
      unpack8(hv, h);
      unpack8(*reinterpret_cast<const uint4*>(N.gamma + c), g);
#pragma unroll
      for (int e = 0; e < 8; ++e) o[e] = r16(g[e] * r16(h[e] * r));
      *reinterpret_cast<uint4*>(N.hout + ro + c) = hv;
      *reinterpret_cast<uint4*>(N.out + ro + c) = pack8(o);
    }
    __syncthreads();
  }
}

// every CTA clears its share (16-byte stores, grid-stride) of the stage's
// zero list
__device__ __forceinline__ void stage_zero(const StepStage& st) {
  for (int z = 0; z < st.nzero; ++z) {
    float4* p = reinterpret_cast<float4*>(st.zero_ptr[z]);
    const int64_t n = st.zero_bytes[z] / 16;
    for (int64_t i = (int64_t)blockIdx.x * kStepThreads + threadIdx.x; i < n; i += (int64_t)gridDim.x * kStepThreads)
      __stcg(p + i, make_float4(0.f, 0.f, 0.f, 0.f));
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
  if (blockIdx.x == 0 && tid == 0) {
    reinterpret_cast<int64_t*>(ws + kWsLayout)[0] = H.ws_acc_off;
    reinterpret_cast<int64_t*>(ws + kWsLayout)[1] = H.ws_acc_bytes;
  }
  fetch(0);
  fetch(1);
  cp_async_wait_all();
  __syncthreads();
  uint4 pre[4];
  uint32_t pre_hg = 0u, pre_hq = 0u;
  if (H.nstages > 0 && slots[0].type == kLinear) {
    stage_static_prefetch(slots[0].lin, smem);
    preload_first(slots[0].lin, pre, pre_hg, pre_hq);
  }
  for (int s = 0; s < H.nstages; ++s) {
    const StepStage& st = slots[s % 3];
    fetch(s + 2);
    cp_async_commit();
    step_trace(s, 0);
    stage_zero(st);
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
      if (L.bits == 2) linear_stage<2>(L, smem, H.B, lut3, s, pre, pre_hg, pre_hq);
      else if (L.bits == 3) linear_stage<3>(L, smem, H.B, lut3, s, pre, pre_hg, pre_hq);
      else linear_stage<4>(L, smem, H.B, lut4, s, pre, pre_hg, pre_hq);
    } else if (st.type == kAttention) {
      attn_stage(st.attn, H.B, pos, smem, ws, H);
    } else {
      final_norm_stage(st.fnorm, H.B, red, reinterpret_cast<uint16_t*>(smem + st.fnorm.buf_off));
    }
    step_trace(s, 2);
    if (s + 1 == H.nstages) break;
    grid_arrive(bar);     // this stage's results are published
    cp_async_wait_all();  // the next records have landed
    __syncthreads();      // and this stage's shared buffers are free
    // work that depends on nothing the barrier orders, while it completes
    const StepStage& nx = slots[(s + 1) % 3];
    if (nx.type == kLinear) {
      prefetch_stage(nx.lin);
      stage_static_prefetch(nx.lin, smem);
      preload_first(nx.lin, pre, pre_hg, pre_hq);
    }
    if (!grid_wait(bar, status, (unsigned)(s + 1) * gridDim.x + (unsigned)H.extra_arrivals, limit_ns, s_ok)) break;
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

// Shared-memory buffer sizes of a linear stage for K-slices of `cols`
// columns and rpp rows per pass: activations z, input rows, fp32 scratch,
// rotation scales, norm weight, producer scales.
void linear_sizes(const LinearStage& L, int B, int cols, int rpp, int rs_smem, uint32_t* sz) {
  const bool need_scr = !(rs_smem && L.lg_block <= 9);
  auto r128 = [](int64_t v) { return static_cast<uint32_t>((v + 127) / 128 * 128); };
  sz[0] = r128((int64_t)L.nops * (B + 1) * (cols + kZPad) * 2);
  sz[1] = r128((int64_t)rpp * cols * 2);
  sz[2] = need_scr ? r128((int64_t)rpp * cols * 4) : 0u;
  sz[3] = r128((int64_t)rs_smem * L.nops * cols * 2);
  sz[4] = L.in_kind == kInRmsNorm ? r128((int64_t)cols * 2) : 0u;
  sz[5] = r128((int64_t)L.nin * cols * 2);
  sz[6] = r128((int64_t)rpp * cols * stage_bytes_per_col(L.in_kind, L.nin));
}
constexpr int kBufs = 7;

// Plan one linear stage (ops share d, block, bits, codebook); the input
// description (in_kind, in[], nin) is set by the caller before.
tp_status plan_linear(LinearStage& L, const tp_step_linear* const* ops, float* const* accs, int nops, int B, int G,
                      const Regions& R) {
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
    op.acc = accs[k];
    op.rot_scale = ops[k]->rot_scale;
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
  bool alias = false;
  uint32_t off[kBufs] = {0, 0, 0, 0, 0, 0, 0};
  bool found = false;
  auto place = [&](const uint32_t* sz) {
    uint32_t ua = 0, ub = 0;
    const uint32_t ca = R.has4 ? 0 : R.a1 - R.a0, cb = R.b1 - R.b0;
    for (int i = 0; i < kBufs; ++i) {
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
  // Stages whose input is not normed split K so that each CTA reads and
  // rotates at most kSliceTarget units of columns: their K-slices add into
  // the same accumulators, so a split costs nothing downstream.  A norm needs
  // the whole row in every CTA, so those start from one slice.
  constexpr int kSliceTarget = 10;
  const int kp0 = L.in_kind == kInRmsNorm
                      ? 1
                      : std::max(1, std::min((U + kSliceTarget - 1) / kSliceTarget, (U + blk_units - 1) / blk_units));
  for (int attempt = 0; attempt < 2 && !found; ++attempt) {
    rs_smem = attempt == 0 ? 1 : 0;
    for (kparts = kp0; kparts <= U && !found; ++kparts) {
      us = (U + kparts - 1) / kparts;
      us = (us + blk_units - 1) / blk_units * blk_units;
      const int kp = (U + us - 1) / us;
      if (kp != kparts) continue;
      const int cols = us * kUnitCols;
      for (rpp = B; rpp >= 1; --rpp) {
        uint32_t sz[kBufs];
        linear_sizes(L, B, cols, rpp, rs_smem, sz);
        // the producer scales and the input staging are dead before the
        // rotation writes the activations: they share the activations'
        // buffer when they fit in it (a smaller footprint leaves more L1)
        // (one pass over the batch rows only: a second pass would stage
        // over the first pass's activations)
        alias = rpp == B && sz[5] + sz[6] <= sz[0];
        if (alias) sz[5] = sz[6] = 0;
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
  L.gam_off = off[4];
  L.psc_off = off[5];
  L.stg_off = off[6];
  if (alias) {
    uint32_t sz[kBufs];
    linear_sizes(L, B, us * kUnitCols, rpp, rs_smem, sz);
    L.psc_off = L.z_off;
    L.stg_off = L.z_off + sz[5];
  }
  // grid split
  L.cps = std::max(1, G / kparts);
  const int64_t W = (int64_t)L.cps * kStepWarps;
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
  }
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
  const int64_t qd = (int64_t)m->q_heads * m->head_dim;
  // the attention output (fp16 [B][q_heads * head_dim]); the linears'
  // outputs live in the workspace as fp32 accumulators
  return 2 * m->B * align256(qd) + 256;
}

extern "C" tp_status tp_step_build(const tp_step_model* m, const tp_step_layer* layers, void* image_host,
                                   int64_t image_bytes, int64_t* workspace_bytes) {
  if (!m || !layers || !image_host || !workspace_bytes) return fail(TP_ERR_ARG, "tp_step_build: null argument");
  const int B = m->B;
  if (B < 1 || B > kStepMaxBatch) return fail(TP_ERR_UNSUPPORTED, "tp_step: batch must be 1..%d", kStepMaxBatch);
  if (m->layers < 1 || image_bytes < tp_step_image_bytes(m->layers))
    return fail(TP_ERR_ARG, "tp_step_build: image buffer too small");
  const int gsz = m->kv_heads > 0 ? m->q_heads / m->kv_heads : 0;
  if (!(m->head_dim == 128 || m->head_dim == 64) || m->kv_heads < 1 || m->q_heads % m->kv_heads || gsz > kMaxGroup ||
      (gsz & (gsz - 1)))
    return fail(TP_ERR_UNSUPPORTED,
                "tp_step: head_dim must be 64 or 128 with 1, 2, 4 or %d query heads per kv head", kMaxGroup);
  if (m->hidden % 8 || m->inter % 8) return fail(TP_ERR_UNSUPPORTED, "tp_step: hidden and inter must be multiples of 8");
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
  const int64_t hd = m->head_dim, qd = m->q_heads * hd, kd = m->kv_heads * hd, hid = m->hidden, inter = m->inter;
  uint16_t* ab = reinterpret_cast<uint16_t*>(m->act);  // attention output
  // workspace: status / barrier / attention counters, attention partials,
  // fp32 accumulators (one set, reused by every layer), the second residual
  // buffer
  const int attn_groups = B * m->kv_heads;
  int nsplit = std::min(kMaxSplits, std::max(1, G / attn_groups));
  H->ws_attn_off = align256(kWsCounters + (int64_t)attn_groups * 4);
  H->ws_acc_off = H->ws_attn_off + align256((int64_t)attn_groups * nsplit * gsz * (hd + 2) * 4);
  int64_t acc_at = H->ws_acc_off;
  auto acc_alloc = [&](int64_t n) {
    const int64_t o = acc_at;
    acc_at += align256(B * n * 4);
    return o;
  };
  const int64_t o_q = acc_alloc(qd), o_k = acc_alloc(kd), o_v = acc_alloc(kd), o_o = acc_alloc(hid),
                o_g = acc_alloc(inter), o_u = acc_alloc(inter), o_d = acc_alloc(hid);
  H->ws_acc_bytes = acc_at - H->ws_acc_off;
  H->ws_h2_off = acc_at;
  H->ws_bytes = H->ws_h2_off + align256(B * hid * 2);
  // device addresses are not known yet: the image holds workspace offsets
  // in these pointer fields (tagged), patched by tp_step_run
  auto wsp = [&](int64_t off) { return reinterpret_cast<float*>(static_cast<uintptr_t>(off) | kWsTag); };
  float *acc_q = wsp(o_q), *acc_k = wsp(o_k), *acc_v = wsp(o_v), *acc_o = wsp(o_o), *acc_g = wsp(o_g),
        *acc_u = wsp(o_u), *acc_d = wsp(o_d);
  uint16_t* h2 = reinterpret_cast<uint16_t*>(wsp(H->ws_h2_off));
  uint16_t* h0 = m->hidden_state;
  const int gs = gsz;
  const uint32_t attn_buf = static_cast<uint32_t>((kMaxGroup * hd + 2 * hd + kStepWarps * gs * (hd + 2)) * 4);
  const bool attn_in_a = !has4 && R.a0 + attn_buf <= R.a1;
  const uint32_t attn_at = attn_in_a ? R.a0 : R.b0;
  if (!attn_in_a && R.b0 + attn_buf > R.b1) return fail(TP_ERR_UNSUPPORTED, "tp_step: attention buffers do not fit");
  int ns = 0;
  // zero list of a stage: adjacent accumulators merge into one region
  bool zero_overflow = false;
  auto zero = [&](StepStage& s, float* p, int64_t n) {
    const int64_t bytes = align256(B * n * 4);
    if (s.nzero > 0 && reinterpret_cast<uintptr_t>(s.zero_ptr[s.nzero - 1]) + s.zero_bytes[s.nzero - 1] ==
                           reinterpret_cast<uintptr_t>(p)) {
      s.zero_bytes[s.nzero - 1] += bytes;
      return;
    }
    if (s.nzero == 2) {
      zero_overflow = true;
      return;
    }
    s.zero_ptr[s.nzero] = p;
    s.zero_bytes[s.nzero] = bytes;
    ++s.nzero;
  };
  const tp_step_linear* prev_down = nullptr;
  for (int i = 0; i < m->layers; ++i) {
    const tp_step_layer& ly = layers[i];
    if (!ly.ln1 || !ly.ln2 || !ly.k_cache || !ly.v_cache) return fail(TP_ERR_ARG, "tp_step: layer %d incomplete", i);
    if (ly.q.n != qd || ly.k.n != kd || ly.v.n != kd || ly.o.d != qd || ly.o.n != hid || ly.q.d != hid ||
        ly.gate.n != inter || ly.up.n != inter || ly.down.d != inter || ly.down.n != hid || ly.gate.d != hid)
      return fail(TP_ERR_ARG, "tp_step: layer %d shapes do not match the model", i);
    // QKV: x = rmsnorm(h), h = h0 (+ the previous layer's down_proj), h written to h2
    {
      StepStage& s = st[ns++];
      s.type = kLinear;
      LinearStage& L = s.lin;
      L.in_kind = kInRmsNorm;
      L.in[0] = InVec{h0, prev_down ? acc_d : nullptr, prev_down ? prev_down->scales : nullptr,
                      prev_down ? prev_down->bias : nullptr};
      L.nin = prev_down ? 1 : 0;
      L.gamma = ly.ln1;
      L.eps = m->rms_eps;
      L.hout = h2;
      const tp_step_linear* ops[3] = {&ly.q, &ly.k, &ly.v};
      float* accs[3] = {acc_q, acc_k, acc_v};
      if (tp_status e = plan_linear(L, ops, accs, 3, B, G, R)) return e;
      if (i > 0) zero(s, acc_g, inter), zero(s, acc_u, inter);  // read by the previous DOWN
    }
    // ATTN
    {
      StepStage& s = st[ns++];
      s.type = kAttention;
      AttnStage& A = s.attn;
      A.q = InVec{nullptr, acc_q, ly.q.scales, ly.q.bias};
      A.k = InVec{nullptr, acc_k, ly.k.scales, ly.k.bias};
      A.v = InVec{nullptr, acc_v, ly.v.scales, ly.v.bias};
      A.q_norm = ly.q_norm;
      A.k_norm = ly.k_norm;
      A.k_cache = ly.k_cache;
      A.v_cache = ly.v_cache;
      A.out = ab;
      A.inv_freq = m->inv_freq;
      A.rope_cos = m->rope_cos;
      A.rope_sin = m->rope_sin;
      A.q_heads = m->q_heads;
      A.kv_heads = m->kv_heads;
      A.hd = m->head_dim;
      A.max_t = m->max_tokens;
      A.nsplit = nsplit;
      A.eps = m->rms_eps;
      A.scaling = static_cast<float>(1.0 / std::sqrt(static_cast<double>(hd)));
      A.buf_off = attn_at - R.base;
      if (i > 0) zero(s, acc_d, hid);  // read by this layer's QKV
    }
    // O: plain input (the attention output)
    {
      StepStage& s = st[ns++];
      s.type = kLinear;
      LinearStage& L = s.lin;
      L.in_kind = kInPlain;
      L.in[0] = InVec{ab, nullptr, nullptr, nullptr};
      L.nin = 0;
      const tp_step_linear* ops[1] = {&ly.o};
      float* accs[1] = {acc_o};
      if (tp_status e = plan_linear(L, ops, accs, 1, B, G, R)) return e;
      zero(s, acc_q, qd), zero(s, acc_k, kd), zero(s, acc_v, kd);  // read by ATTN
    }
    // GATE / UP: x = rmsnorm(h2 + o_proj), written back to h0
    {
      StepStage& s = st[ns++];
      s.type = kLinear;
      LinearStage& L = s.lin;
      L.in_kind = kInRmsNorm;
      L.in[0] = InVec{h2, acc_o, ly.o.scales, ly.o.bias};
      L.nin = 1;
      L.gamma = ly.ln2;
      L.eps = m->rms_eps;
      L.hout = h0;
      const tp_step_linear* ops[2] = {&ly.gate, &ly.up};
      float* accs[2] = {acc_g, acc_u};
      if (tp_status e = plan_linear(L, ops, accs, 2, B, G, R)) return e;
    }
    // DOWN: x = silu(gate) * up
    {
      StepStage& s = st[ns++];
      s.type = kLinear;
      LinearStage& L = s.lin;
      L.in_kind = kInSiluMul;
      L.in[0] = InVec{nullptr, acc_g, ly.gate.scales, ly.gate.bias};
      L.in[1] = InVec{nullptr, acc_u, ly.up.scales, ly.up.bias};
      L.nin = 2;
      const tp_step_linear* ops[1] = {&ly.down};
      float* accs[1] = {acc_d};
      if (tp_status e = plan_linear(L, ops, accs, 1, B, G, R)) return e;
      zero(s, acc_o, hid);  // read by GATE / UP
    }
    prev_down = &ly.down;
  }
  {
    StepStage& s = st[ns++];
    s.type = kFinalNorm;
    s.fnorm.x = InVec{h0, acc_d, prev_down->scales, prev_down->bias};
    s.fnorm.gamma = m->final_norm;
    s.fnorm.out = m->final_out;
    s.fnorm.hout = m->hidden_state;
    s.fnorm.d = m->hidden;
    s.fnorm.eps = m->rms_eps;
    s.fnorm.buf_off = (!has4 && R.a0 + hid * 2 <= R.a1 ? R.a0 : R.b0) - R.base;
    zero(s, acc_g, inter), zero(s, acc_u, inter);  // read by the last DOWN; acc_d: cleared by the stage itself
  }
  if (zero_overflow) return fail(TP_ERR_UNSUPPORTED, "tp_step: internal error (zero list)");
  // the largest footprint over the stages sets the dynamic shared memory size
  uint32_t end = std::max<uint32_t>(has4 ? R.b0 : kLutAbs + 65536u, attn_at + attn_buf);
  end = std::max<uint32_t>(end, R.base + st[ns - 1].fnorm.buf_off + static_cast<uint32_t>(hid * 2));
  if (R.b0 + hid * 2 > R.b1) return fail(TP_ERR_UNSUPPORTED, "tp_step: hidden size too large");
  for (int s = 0; s < ns; ++s) {
    if (st[s].type != kLinear) continue;
    const LinearStage& L = st[s].lin;
    uint32_t sz[kBufs];
    linear_sizes(L, B, L.us * kUnitCols, L.rpp, L.rs_smem, sz);
    const uint32_t offs[kBufs] = {L.z_off, L.xin_off, L.scr_off, L.rs_off, L.gam_off, L.psc_off, L.stg_off};
    for (int i = 0; i < kBufs; ++i)
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
  H->barrier_us = 0;
  H->extra_arrivals = 0;
  H->attn_groups = attn_groups;
  *workspace_bytes = H->ws_bytes;
  return clear_ok();
}

extern "C" tp_status tp_step_bind(void* image_host, void* workspace, int64_t workspace_bytes) {
  if (!image_host || !workspace) return fail(TP_ERR_ARG, "tp_step_bind: null argument");
  StepHeader* H = static_cast<StepHeader*>(image_host);
  if (workspace_bytes < H->ws_bytes)
    return fail(TP_ERR_WORKSPACE, "tp_step_bind: workspace of %lld bytes required", (long long)H->ws_bytes);
  if (!aligned(workspace, 256)) return fail(TP_ERR_ALIGN, "tp_step_bind: workspace must be 256-byte aligned");
  if (H->bound_ws) {
    if (H->bound_ws == reinterpret_cast<uint64_t>(workspace)) return clear_ok();
    return fail(TP_ERR_ARG, "tp_step_bind: image already bound to another workspace");
  }
  unsigned char* ws = static_cast<unsigned char*>(workspace);
  auto fix = [&](auto*& p) {
    const uintptr_t v = reinterpret_cast<uintptr_t>(p);
    if (v & kWsTag) p = reinterpret_cast<std::remove_reference_t<decltype(p)>>(ws + (v & ~kWsTag));
  };
  StepStage* st = reinterpret_cast<StepStage*>(H + 1);
  for (int i = 0; i < H->nstages; ++i) {
    StepStage& S = st[i];
    for (int z = 0; z < S.nzero; ++z) fix(S.zero_ptr[z]);
    if (S.type == kLinear) {
      for (auto& v : S.lin.in) fix(v.base), fix(v.acc);
      fix(S.lin.hout);
      for (int k = 0; k < S.lin.nops; ++k) fix(S.lin.ops[k].acc);
    } else if (S.type == kAttention) {
      fix(S.attn.q.acc), fix(S.attn.k.acc), fix(S.attn.v.acc);
    } else {
      fix(S.fnorm.x.base), fix(S.fnorm.x.acc);
    }
  }
  H->bound_ws = reinterpret_cast<uint64_t>(workspace);
  return clear_ok();
}

extern "C" tp_status tp_step_run(const void* image_dev, const void* image_host, const int* pos_dev, void* workspace,
                                 int64_t workspace_bytes, void* stream) {
  if (!image_dev || !image_host || !pos_dev || !workspace) return fail(TP_ERR_ARG, "tp_step_run: null argument");
  const StepHeader* H = static_cast<const StepHeader*>(image_host);
  if (workspace_bytes < H->ws_bytes)
    return fail(TP_ERR_WORKSPACE, "tp_step_run: workspace of %lld bytes required", (long long)H->ws_bytes);
  if (!aligned(workspace, 256)) return fail(TP_ERR_ALIGN, "tp_step_run: workspace must be 256-byte aligned");
  if (H->bound_ws != reinterpret_cast<uint64_t>(workspace))
    return fail(TP_ERR_ARG, "tp_step_run: the image is not bound to this workspace (tp_step_bind)");
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
  // a step that gave up leaves accumulators and counters part-written: clear
  // them (and the status) so the next step starts from zero
  int64_t lay[2] = {0, 0};
  TP_CUDA_TRY(cudaMemcpyAsync(lay, ws + kWsLayout, sizeof(lay), cudaMemcpyDeviceToHost, st), "layout copy");
  TP_CUDA_TRY(cudaStreamSynchronize(st), "status sync");
  unsigned char* w = const_cast<unsigned char*>(ws);
  TP_CUDA_TRY(cudaMemsetAsync(w + kWsStatus, 0, 4, st), "status clear");
  if (lay[0] > kWsCounters)  // attention counters and partials
    TP_CUDA_TRY(cudaMemsetAsync(w + kWsCounters, 0, static_cast<size_t>(lay[0] - kWsCounters), st), "counter clear");
  if (lay[0] > 0 && lay[1] > 0)
    TP_CUDA_TRY(cudaMemsetAsync(w + lay[0], 0, static_cast<size_t>(lay[1]), st), "accumulator clear");
  TP_CUDA_TRY(cudaStreamSynchronize(st), "status sync");
  if (v & kStepStatusLayout) return fail(TP_ERR_DEVICE, "tp_step: shared-memory layout check failed (status %u)", v);
  return fail(TP_ERR_DEVICE, "tp_step: a grid barrier timed out (status %u)", v);
}

#ifdef TP_STEP_TRACE
extern "C" TP_API int tp_step_trace_read(unsigned long long* host) {
  return (int)cudaMemcpyFromSymbol(host, tp::g_step_trace, sizeof(tp::g_step_trace));
}
#endif

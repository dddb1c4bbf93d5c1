// Persistent decode engine: a whole chain of packed-TCQ linears in one launch.
//
// One CTA per SM stays resident for the program (cooperative launch) and
// builds the pair table once.  Consecutive ops that read the same input
// (same x, dependency, width and Hadamard block: q/k/v, gate/up) form a
// STAGE; a stage is decoded as one matrix whose row tiles are the ops' row
// tiles one after another (all of them have the same units per row tile).
// The stage's weight units (16 rows x 256 columns, tile-major, contiguous
// in each op's native stream) are split into equal contiguous runs, one per
// consumer warp of the grid.
//
// Warp roles inside a CTA: kEWarps consumer warps decode; one producer warp
// keeps, for every consumer, a ring of `slots` units in flight with bulk
// copies (lane w serves consumer w: full barrier per slot completed by the
// copy, empty barrier per slot released by the consumer), walking the
// consumer's runs stage after stage, so weights of later layers stream in
// while a stage waits for its input.  Per stage the consumers (synchronised
// among themselves with a named barrier; the producer never joins it):
//   1. wait (bounded) until every CTA finished the stage producing x;
//   2. stage x * rot_scale of every op (fp32) in shared memory in one round
//      of loads, then transform whole Hadamard blocks (warp registers +
//      shuffles for blocks 32..1024, consumer-wide otherwise) into fp16
//      activations in the decoder's permuted pair order, one row per op and
//      batch row;
//   3. decode units as the per-call GEMV (level words, pair table, m16n8k16
//      MMA), two units per iteration where the run allows, accumulating per
//      row tile in registers, then in shared memory;
//   4. scale (and bias, once per row) the CTA's tile partials and add them
//      to the ops' fp32 outputs with atomics; publish completion.
#include <algorithm>
#include <cstdlib>
#include <vector>

#include "tp_decode.cuh"
#include "tp_rotate.cuh"

using namespace tp;

namespace {

#ifndef TP_EWARPS
#define TP_EWARPS 11
#endif
constexpr int kEWarps = TP_EWARPS;             // consumer warps
constexpr int kECThreads = kEWarps * 32;       // consumer threads
constexpr int kEThreads = kECThreads + 32;     // + the producer warp
constexpr int kEMaxB = 4;
#ifndef TP_EMAXSLOTS
#define TP_EMAXSLOTS 8
#endif
constexpr int kEMaxSlots = TP_EMAXSLOTS;
constexpr int kEMaxStageOps = 8;
constexpr int kEXStageBytes = 48 * 1024;   // staged x rows per pass
constexpr int kEZStageBytes = 48 * 1024;   // activations + rot_scale rows of one stage (grouping cap)
constexpr unsigned kEMaxSpin = 1u << 24;   // dependency polls (~1 s with backoff)
constexpr unsigned kEMaxIdle = 1u << 25;   // producer polls without progress (~4 s)
constexpr int kEMagic = 0x54504533;        // "TPE3"
constexpr unsigned kEStaticSmem = 4096;    // bound on the kernel's static shared memory

struct alignas(16) EOp {
  const uint4* stream;
  const uint16_t* scales;
  const uint16_t* bias;
  const uint16_t* rot_scale;
  uint64_t y;            // fp32 output: address (single GPU) or byte offset into the arena (tensor parallel)
  int32_t n, tile_base;  // rows decoded here; first row tile of this op inside its stage
  int32_t unit_base, r0;  // first unit inside the stage; first output row of this shard
  int32_t n_full, pad0;   // rows of the full output (row stride of y)
};

struct alignas(16) EStage {
  const void* x;
  int32_t x_dtype, dep, first_op, n_ops;  // dep: stage index or -1
  int32_t d, d_pad, units_k, total_tiles;
  int32_t total_units, vec, block, lg;
  int32_t rows_per_pass;       // batch rows of x staged per pass
  float norm;                  // 1/sqrt(block)
  uint32_t rs_off, work_off;   // in the scratch area: staged rot_scale rows, fp32 work row
  int32_t direct;              // 1: blocks above 1024, read straight from global memory (no x / rot_scale staging)
  int32_t work_blocks;         // direct stages: Hadamard blocks per pass through the fp32 work area
};

struct alignas(16) EHeader {
  int32_t magic, n_ops, n_stages, B;
  int32_t bits, n_states, grid, slots;
  const uint16_t* codebook;
  uint32_t ring_off, z_off, scratch_off, red_off;
  uint32_t smem, zero_q, max_tiles, sc_off;  // sc_off: per-CTA row scales, then biases (fp16)
  uint32_t lut_off, lut_abs;  // pair table offset; 1: it sits at shared-window address 0x10000
  uint32_t dyn_base, pad_h;   // expected shared-window address of the dynamic area (lut_abs)
  // tensor parallel (n_ranks > 1): outputs live in a double-buffered arena
  // replicated on every rank; every CTA adds its partials into all ranks'
  // copies and counts completion on all ranks (peer pointers, NVLink).
  int32_t n_ranks, rank;
  uint64_t arena[2];             // this rank's arena buffers (0 on one GPU: op.y is an address)
  uint64_t arena_bytes;          // bytes of one arena buffer
  const uint64_t* peer_arena;    // [n_ranks][2] arena buffer addresses on every rank
  unsigned* const* peer_ctr;     // [n_ranks] counter blocks on every rank
};

static_assert(sizeof(EOp) == 64 && sizeof(EStage) % 16 == 0 && sizeof(EHeader) % 16 == 0, "image layout");

#ifdef TP_TRACE
// development-only timeline: CTA 0 and CTA gridDim/2 stamp each stage's phases
static __device__ unsigned long long g_etrace[2][512][8];
__device__ __forceinline__ void etrace(int o, int k) {
  const int which = blockIdx.x == 0 ? 0 : (blockIdx.x == gridDim.x / 2 ? 1 : -1);
  if (threadIdx.x == 0 && which >= 0 && o < 512) {
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    g_etrace[which][o][k] = t;
  }
}
#else
__device__ __forceinline__ void etrace(int, int) {}
#endif

// barrier of the consumer warps only (the producer warp runs its own loop)
__device__ __forceinline__ void csync() { asm volatile("bar.sync 1, %0;" ::"n"(kECThreads) : "memory"); }

__device__ __forceinline__ float load_x(const EStage& st, int64_t i) {
  if (st.x_dtype == TP_F32) return __ldcg(reinterpret_cast<const float*>(st.x) + i);  // may be produced by this grid
  return load_as_float(st.x, i, st.x_dtype);
}

// completion counters: release increment / acquire read at gpu scope
__device__ __forceinline__ void red_release(unsigned* p) {
  asm volatile("fence.acq_rel.gpu;\n red.relaxed.gpu.global.add.u32 [%0], 1;" ::"l"(p) : "memory");
}
// gpu-scope acq_rel increment returning the old count
__device__ __forceinline__ unsigned atom_add_acq_rel(unsigned* p) {
  unsigned old;
  asm volatile("atom.acq_rel.gpu.global.add.u32 %0, [%1], 1;" : "=r"(old) : "l"(p) : "memory");
  return old;
}
// one system-scope release, then +1 on word idx of every rank's counter block
__device__ __forceinline__ void red_release_sys(unsigned* const* ctrs, int n, int idx) {
  asm volatile("fence.acq_rel.sys;" ::: "memory");
  for (int p = 0; p < n; ++p) asm volatile("red.relaxed.sys.global.add.u32 [%0], 1;" ::"l"(ctrs[p] + idx) : "memory");
}
__device__ __forceinline__ unsigned ld_acquire_sys(const unsigned* p) {
  unsigned v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ unsigned ld_acquire(const unsigned* p) {
  unsigned v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ void cp_async16(void* dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(dst)), "l"(src) : "memory");
}
// copies src_bytes (0..4) and zero-fills the rest of the 4 bytes
__device__ __forceinline__ void cp_async4(void* dst, const void* src, int src_bytes) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4, %2;" ::"r"(smem_u32(dst)), "l"(src), "r"(src_bytes)
               : "memory");
}
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_all;" ::: "memory"); }

// Stage the inputs of a rotation pass in the scratch area: x rows
// [b0, b0 + rows) at offset 0 and, on the first pass, every op's rot_scale
// row at rs_off.  Aligned stages copy raw bytes with cp.async (all copies in
// flight at once: one round trip whatever the size); others convert x to
// fp32 with plain loads.
__device__ void stage_inputs(const EStage& st, const EOp* cops, int b0, int rows, bool first, unsigned char* scr,
                             int ctid) {
  if (st.vec) {
    const int esz = st.x_dtype == TP_F32 ? 4 : 2;
    const int rowc = st.d * esz / 16;
    const char* xsrc = reinterpret_cast<const char*>(st.x) + (size_t)b0 * st.d * esz;
    for (int i = ctid; i < rows * rowc; i += kECThreads) cp_async16(scr + i * 16, xsrc + i * 16);
    if (first) {
      const int rc = st.d * 2 / 16;
      for (int j = 0; j < st.n_ops; ++j)
        for (int i = ctid; i < rc; i += kECThreads)
          cp_async16(scr + st.rs_off + j * st.d * 2 + i * 16, reinterpret_cast<const char*>(cops[j].rot_scale) + i * 16);
    }
    cp_async_wait_all();
  } else {
    float* xs = reinterpret_cast<float*>(scr);
    for (int r = 0; r < rows; ++r)
      for (int c = ctid; c < st.d; c += kECThreads) xs[r * st.d + c] = load_x(st, (int64_t)(b0 + r) * st.d + c);
    if (first) {
      uint16_t* rs = reinterpret_cast<uint16_t*>(scr + st.rs_off);
      for (int j = 0; j < st.n_ops; ++j)
        for (int c = ctid; c < st.d; c += kECThreads) rs[j * st.d + c] = cops[j].rot_scale[c];
    }
  }
}

// element i of the staged x rows
__device__ __forceinline__ float xs_at(const unsigned char* scr, int dt, int i) {
  if (dt == TP_F32) return reinterpret_cast<const float*>(scr)[i];
  if (dt == TP_F16) return __half2float(reinterpret_cast<const __half*>(scr)[i]);
  return __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(scr)[i]);
}

// Warp-level FWHT of R*32 elements held as v[r] = element lane + 32 r.
template <int R>
__device__ __forceinline__ void warp_fwht_regs(float* v, int lane) {
#pragma unroll
  for (int h = 1; h < R; h <<= 1) {
#pragma unroll
    for (int r = 0; r < R; ++r) {
      if (!(r & h)) {
        const float a = v[r], b = v[r + h];
        v[r] = a + b;
        v[r + h] = a - b;
      }
    }
  }
#pragma unroll
  for (int m = 1; m < 32; m <<= 1) {
    const float sgn = (lane & m) ? -1.f : 1.f;  // upper lane: o - v, lower lane: o + v
#pragma unroll
    for (int r = 0; r < R; ++r) {
      const float o = __shfl_xor_sync(0xffffffffu, v[r], m);
      v[r] = fmaf(sgn, v[r], o);
    }
  }
}

// one Hadamard block: x (staged, dtype dt, from element xoff) * rot_scale
// row -> FWHT -> fp16 zs row in the decoder's permuted order
template <int R>
__device__ __forceinline__ void warp_block_rotate(const unsigned char* scr, int dt, int xoff, const uint16_t* rs,
                                                  __half* zrow, float norm, int lane, int zp) {
  float v[R];
#pragma unroll
  for (int r = 0; r < R; ++r) v[r] = xs_at(scr, dt, xoff + lane + 32 * r) * h2f_bits(rs[lane + 32 * r]);
  warp_fwht_regs<R>(v, lane);
#pragma unroll
  for (int r = 0; r < R; ++r) zrow[32 * r + zp] = __float2half_rn(v[r] * norm);
}

// Butterflies over index bits [b_start, lg) of s[0, count) by the consumer
// threads (radix-8 groups, one consumer barrier per group of three bits).
__device__ void fwht_consumers(float* s, int count, int b_start, int lg, int ctid) {
  for (int b0 = b_start; b0 < lg; b0 += 3) {
    const int nb = lg - b0 < 3 ? lg - b0 : 3;
    const int G = 1 << nb;
    const int groups = count >> nb;
    for (int grp = ctid; grp < groups; grp += kECThreads) {
      const int lo = grp & ((1 << b0) - 1);
      const int hi = grp >> b0;
      const int base = (hi << (b0 + nb)) | lo;
      float v[8];
#pragma unroll
      for (int e = 0; e < 8; ++e)
        if (e < G) v[e] = s[base + (e << b0)];
#pragma unroll
      for (int h = 1; h < 8; h <<= 1) {
        if (h >= G) break;
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          if (e < G && !(e & h)) {
            const float a = v[e], b = v[e + h];
            v[e] = a + b;
            v[e + h] = a - b;
          }
        }
      }
#pragma unroll
      for (int e = 0; e < 8; ++e)
        if (e < G) s[base + (e << b0)] = v[e];
    }
    csync();
  }
}

// R-point transform of the values at one position of R consecutive 512-wide
// chunks (stride 512 in the work area; the chunks are already transformed),
// scaled and written as fp16 activations of absolute columns cc0 + 512 e.
template <int R>
__device__ __forceinline__ void chunk_combine(const float* w, __half* zrow, int cc0, float norm) {
  float v[R];
#pragma unroll
  for (int e = 0; e < R; ++e) v[e] = w[e * 512];
#pragma unroll
  for (int h = 1; h < R; h <<= 1) {
#pragma unroll
    for (int e = 0; e < R; ++e) {
      if (!(e & h)) {
        const float a = v[e], b = v[e + h];
        v[e] = a + b;
        v[e + h] = a - b;
      }
    }
  }
#pragma unroll
  for (int e = 0; e < R; ++e) {
    const int cc = cc0 + e * 512;
    zrow[(cc & ~31) + zperm_pos(cc & 31)] = __float2half_rn(v[e] * norm);
  }
}

// x -> fp16 rotated activations of every (op j, batch row b) job of the
// stage; the job's row lives at zs + (j * B + b) * d_pad.  Blocks of
// 32..1024 are one warp job each (registers + shuffles); larger blocks go
// through the fp32 work row as 512-wide warp transforms plus consumer-wide
// passes over the upper index bits, smaller ones consumer-wide.  Ends with a
// consumer barrier.
__device__ void rotate_stage(const EStage& st, const EOp* cops, int B, __half* zs, unsigned char* scr, int warp,
                             int lane, int ctid, int si) {
  const int zp = zperm_pos(lane);
  const int nblk = st.d / st.block;
  const int dt = st.vec ? st.x_dtype : TP_F32;
  const uint16_t* rs = reinterpret_cast<const uint16_t*>(scr + st.rs_off);
  for (int b0 = 0; b0 < B; b0 += st.rows_per_pass) {
    const int rows = B - b0 < st.rows_per_pass ? B - b0 : st.rows_per_pass;
    if (!st.direct) {
      stage_inputs(st, cops, b0, rows, b0 == 0, scr, ctid);
      csync();
    }
    if (b0 == 0) etrace(si, 5);
    if (st.block >= 32 && st.block <= 1024) {
      // warp jobs (op j, row rr, block kb), kb fastest
      const int R = st.block / 32;
      int j = 0, rr = 0, kb = warp;
      while (kb >= nblk) {
        kb -= nblk;
        if (++rr == rows) {
          rr = 0;
          ++j;
        }
      }
      while (j < st.n_ops) {
        const int xoff = rr * st.d + kb * st.block;
        const uint16_t* rsb = rs + j * st.d + kb * st.block;
        __half* zrow = zs + (size_t)(j * B + b0 + rr) * st.d_pad + kb * st.block;
        switch (R) {
          case 1: warp_block_rotate<1>(scr, dt, xoff, rsb, zrow, st.norm, lane, zp); break;
          case 2: warp_block_rotate<2>(scr, dt, xoff, rsb, zrow, st.norm, lane, zp); break;
          case 4: warp_block_rotate<4>(scr, dt, xoff, rsb, zrow, st.norm, lane, zp); break;
          case 8: warp_block_rotate<8>(scr, dt, xoff, rsb, zrow, st.norm, lane, zp); break;
          case 16: warp_block_rotate<16>(scr, dt, xoff, rsb, zrow, st.norm, lane, zp); break;
          default: warp_block_rotate<32>(scr, dt, xoff, rsb, zrow, st.norm, lane, zp); break;
        }
        kb += kEWarps;
        while (kb >= nblk) {
          kb -= nblk;
          if (++rr == rows) {
            rr = 0;
            ++j;
          }
        }
      }
    } else if (st.direct) {
      // blocks of 2048..8192, work_blocks at a time: (A) every warp transforms
      // 512-wide chunks of x * rot_scale, loaded straight from global memory
      // (L2), in registers into the fp32 work area; (B) every consumer thread
      // combines the block/512 chunk values at one position and writes them.
      float* work = reinterpret_cast<float*>(scr + st.work_off);
      const int R = st.block >> 9;
      for (int j = 0; j < st.n_ops; ++j) {
        const uint16_t* rsg = cops[j].rot_scale;
        for (int rr = 0; rr < rows; ++rr) {
          __half* zrow = zs + (size_t)(j * B + b0 + rr) * st.d_pad;
          const int64_t xrow = (int64_t)(b0 + rr) * st.d;
          for (int kb0 = 0; kb0 < nblk; kb0 += st.work_blocks) {
            const int nb = nblk - kb0 < st.work_blocks ? nblk - kb0 : st.work_blocks;
            const int c0 = kb0 * st.block;
            for (int ch = warp; ch < nb * R; ch += kEWarps) {
              const int cb = c0 + ch * 512;
              float v[16];
#pragma unroll
              for (int r = 0; r < 16; ++r) v[r] = load_x(st, xrow + cb + lane + 32 * r);
#pragma unroll
              for (int r = 0; r < 16; ++r) v[r] *= h2f_bits(rsg[cb + lane + 32 * r]);
              warp_fwht_regs<16>(v, lane);
#pragma unroll
              for (int r = 0; r < 16; ++r) work[ch * 512 + lane + 32 * r] = v[r];
            }
            csync();
            for (int g = ctid; g < nb * 512; g += kECThreads) {
              const int b = g >> 9, p = g & 511;
              const float* w = work + b * st.block + p;
              const int cc0 = c0 + b * st.block + p;
              if (R == 4) chunk_combine<4>(w, zrow, cc0, st.norm);
              else if (R == 8) chunk_combine<8>(w, zrow, cc0, st.norm);
              else chunk_combine<16>(w, zrow, cc0, st.norm);
            }
            csync();
          }
        }
      }
    } else {
      // one Hadamard block at a time through the fp32 work row: blocks above
      // 1024 as 512-wide warp transforms plus consumer-wide passes over the
      // upper index bits, blocks below 32 consumer-wide
      float* work = reinterpret_cast<float*>(scr + st.work_off);
      for (int j = 0; j < st.n_ops; ++j)
        for (int rr = 0; rr < rows; ++rr)
          for (int kb = 0; kb < nblk; ++kb) {
            const int c0 = kb * st.block;
            for (int c = ctid; c < st.block; c += kECThreads)
              work[c] = xs_at(scr, dt, rr * st.d + c0 + c) * h2f_bits(rs[j * st.d + c0 + c]);
            csync();
            int b_start = 0;
            if (st.block > 1024) {
              for (int sb = warp; sb < st.block / 512; sb += kEWarps) {
                float v[16];
#pragma unroll
                for (int r = 0; r < 16; ++r) v[r] = work[sb * 512 + lane + 32 * r];
                warp_fwht_regs<16>(v, lane);
#pragma unroll
                for (int r = 0; r < 16; ++r) work[sb * 512 + lane + 32 * r] = v[r];
              }
              csync();
              b_start = 9;
            }
            fwht_consumers(work, st.block, b_start, st.lg, ctid);
            __half* zrow = zs + (size_t)(j * B + b0 + rr) * st.d_pad;
            for (int c = ctid; c < st.block; c += kECThreads) {
              const int cc = c0 + c;  // the permutation works on absolute 32-column chunks
              zrow[(cc & ~31) + zperm_pos(cc & 31)] = __float2half_rn(work[c] * st.norm);
            }
            csync();
          }
    }
    csync();
  }
  // padding columns [d, d_pad) of every job row
  if (st.d_pad > st.d) {
    for (int jr = 0; jr < st.n_ops * B; ++jr)
      for (int c = st.d + ctid; c < st.d_pad; c += kECThreads)
        zs[(size_t)jr * st.d_pad + (c & ~31) + zperm_pos(c & 31)] = __float2half_rn(0.f);
    csync();
  }
}

// L2 prefetch of what stage `nx` reads with plain loads: every op's
// rot_scale, scales and bias (spread over the grid's consumer threads, one
// 128-byte line each), and each warp's trellis-halo unit.  Issued one stage
// ahead so those loads hit L2 instead of queueing behind the streamed weights.
__device__ __forceinline__ void prefetch_l2(const void* p) { asm volatile("prefetch.global.L2 [%0];" ::"l"(p)); }
__device__ void prefetch_stage(const EStage& nx, const EOp* nops, int64_t v, int64_t V, int lane, int ctid,
                               int unit_bytes) {
  const int gt = blockIdx.x * kECThreads + ctid, nt = gridDim.x * kECThreads;
  const int rs_lines = (nx.d * 2 + 127) / 128;
  for (int j = 0; j < nx.n_ops; ++j) {
    const EOp& op = nops[j];
    const int sc_lines = (op.n * 2 + 127) / 128;
    const int lines = rs_lines + sc_lines * (op.bias ? 2 : 1);
    for (int l = gt; l < lines; l += nt) {
      const char* p = l < rs_lines ? reinterpret_cast<const char*>(op.rot_scale) + l * 128
                      : l < rs_lines + sc_lines
                          ? reinterpret_cast<const char*>(op.scales) + (l - rs_lines) * 128
                          : reinterpret_cast<const char*>(op.bias) + (l - rs_lines - sc_lines) * 128;
      prefetch_l2(p);
    }
  }
  // halo: the unit before this warp's first unit, when that starts inside a row tile
  const int wb = static_cast<int>(v * nx.total_units / V), we = static_cast<int>((v + 1) * nx.total_units / V);
  if (wb < we && wb % nx.units_k != 0 && lane * 128 < unit_bytes) {
    int k = 0;
    while (k < nx.n_ops - 1 && wb - 1 >= nops[k + 1].unit_base) ++k;
    prefetch_l2(reinterpret_cast<const char*>(nops[k].stream) + (int64_t)(wb - 1 - nops[k].unit_base) * unit_bytes +
                lane * 128);
  }
}

// One unit (two 32-column chunks per lane) into `acc`; `prevg/prevq` carry
// the trellis halo (last path words of the previous unit of the row tile).
template <int BITS, int S, bool ABS>
__device__ __forceinline__ void decode_unit(const unsigned char* lut, uint32_t lanew, const uint4* zq,
                                            const uint4 (&cur)[BITS], uint32_t& prevg, uint32_t& prevq, int t,
                                            int src, int zoff0, int zstep, float (*acc)[1][4]) {
  const uint32_t P0g = cur[0].x, P0q = cur[0].y, P1g = cur[0].z, P1q = cur[0].w;
  const uint32_t H0g = __shfl_sync(0xffffffffu, t == 3 ? prevg : P0g, src);
  const uint32_t H0q = __shfl_sync(0xffffffffu, t == 3 ? prevq : P0q, src);
  const uint32_t H1g = __shfl_sync(0xffffffffu, t == 3 ? P0g : P1g, src);
  const uint32_t H1q = __shfl_sync(0xffffffffu, t == 3 ? P0q : P1q, src);
  prevg = P1g;
  prevq = P1q;
#pragma unroll
  for (int cgi = 0; cgi < 2; ++cgi) {
    int zoff[1];
    zoff[0] = zoff0 + cgi * zstep;
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
    process_chunk<BITS, S, 1, ABS>(lut, lanew, zq, Pg, Hg, Pq, Hq, Mg0, Mg1, Mg2, Mq0, Mq1, Mq2, zoff, acc);
  }
}

template <int BITS, int S, bool ABS>
__global__ void __launch_bounds__(kEThreads, 1) tcq_engine_kernel(const EHeader* __restrict__ hdr_g,
                                                                  unsigned* __restrict__ counters) {
  extern __shared__ __align__(128) unsigned char smem[];
  __shared__ __align__(8) uint64_t s_full[kEWarps][kEMaxSlots];
  __shared__ __align__(8) uint64_t s_empty[kEWarps][kEMaxSlots];
  __shared__ __align__(16) EOp s_ops[3][kEMaxStageOps];  // descriptors of stages si, si+1, si+2
  __shared__ __align__(16) EStage s_st[3];
  __shared__ int s_abort;
  __shared__ unsigned s_epoch;

  const EHeader hdr = *hdr_g;
  const EOp* ops = reinterpret_cast<const EOp*>(hdr_g + 1);
  const EStage* stages = reinterpret_cast<const EStage*>(ops + hdr.n_ops);
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int g = lane >> 2, t = lane & 3;
  const int G = gridDim.x;
  const int64_t V = (int64_t)G * kEWarps;
  const int B = hdr.B, Bp = 8;
  constexpr unsigned kUnitBytes = 32u * 16u * BITS;
  unsigned char* lut = smem + hdr.lut_off;
  if (ABS) {
    // the absolute pair-table addresses assume this layout: check it before
    // touching any shared memory, and give up (status 3) if it differs
    unsigned dsz;
    asm volatile("mov.u32 %0, %%dynamic_smem_size;" : "=r"(dsz));
    if (smem_u32(smem) != hdr.dyn_base || smem_u32(lut) != 0x10000u || hdr.lut_off + 65536u > dsz) {
      if (threadIdx.x == 0) atomicExch(counters + hdr.n_ops, 3u);
      return;
    }
  }
  __half* zs = reinterpret_cast<__half*>(smem + hdr.z_off);
  unsigned char* scratch = smem + hdr.scratch_off;
  float* red = reinterpret_cast<float*>(smem + hdr.red_off);
  uint16_t* s_sc = reinterpret_cast<uint16_t*>(smem + hdr.sc_off);  // [max_tiles * 16]
  uint16_t* s_bi = s_sc + hdr.max_tiles * kTileRows;
  const int slots = hdr.slots;

  // descriptor cache: stage s (and up to kEMaxStageOps ops from op f) ->
  // buffer s % 3 with async copies by consumer threads; complete at the
  // issuing threads' next cp_async_wait_all
  auto load_desc = [&](int s, int f) {
    constexpr int kStChunks = sizeof(EStage) / 16, kOpChunks = sizeof(EOp) / 16;
    const int cnt = min(kEMaxStageOps, hdr.n_ops - f);
    const int b = s % 3;
    if (tid < kStChunks)
      cp_async16(reinterpret_cast<char*>(&s_st[b]) + tid * 16, reinterpret_cast<const char*>(stages + s) + tid * 16);
    else if (tid < kStChunks + cnt * kOpChunks)
      cp_async16(reinterpret_cast<char*>(&s_ops[b][0]) + (tid - kStChunks) * 16,
                 reinterpret_cast<const char*>(ops + f) + (tid - kStChunks) * 16);
  };

  const uint32_t cbv = lane < (1 << (BITS + 1)) ? hdr.codebook[lane] : 0u;
  if (tid == 0) s_abort = 0;
#ifdef TP_TRACE
  if (tid == 0 && blockIdx.x == 0) {
    unsigned dsz;
    asm volatile("mov.u32 %0, %%dynamic_smem_size;" : "=r"(dsz));
    g_etrace[0][511][0] = smem_u32(smem);
    g_etrace[0][511][1] = dsz;
    g_etrace[0][511][2] = smem_u32(&s_full[0][0]);
  }
#endif
  if (tid < kEWarps * kEMaxSlots) {
    mbar_init(&s_full[0][0] + tid, 1);
    mbar_init(&s_empty[0][0] + tid, 1);
  }
  fence_mbar_init();
  if (tid < kECThreads) load_desc(0, 0);
  build_lut<BITS>(lut, cbv, warp, lane, kEWarps + 1);
  // zero block read by lanes of batch rows >= B; tile partials start at zero
  if (tid < 16) reinterpret_cast<uint32_t*>(zs)[hdr.zero_q * 4 + tid] = 0u;
  for (int i = tid; i < (int)hdr.max_tiles * kTileRows * 8; i += kEThreads) red[i] = 0.f;
  cp_async_wait_all();
  __syncthreads();
  if (tid < kECThreads && hdr.n_stages > 1) load_desc(1, s_st[0].first_op + s_st[0].n_ops);
  cp_async_wait_all();
  __syncthreads();

  // ===================== producer warp =====================
  if (warp == kEWarps) {
    const int w = lane;  // consumer served by this lane
    const int64_t v = (int64_t)blockIdx.x * kEWarps + w;
    unsigned char* ring = smem + hdr.ring_off + (size_t)w * slots * kUnitBytes;
    int is = 0, ik = 0, iu = 0, iend = 0, slot = 0, n_iss = 0;
    unsigned eph = 0;
    auto warp_range = [&](int s) {
      const int64_t T = stages[s].total_units;
      iu = static_cast<int>(v * T / V);
      iend = static_cast<int>((v + 1) * T / V);
      ik = stages[s].first_op;
    };
    auto seek = [&]() {  // next non-empty run, and the op holding unit iu
      while (is < hdr.n_stages && iu >= iend) {
        ++is;
        if (is < hdr.n_stages) warp_range(is);
      }
      if (is < hdr.n_stages) {
        const int last = stages[is].first_op + stages[is].n_ops - 1;
        while (ik < last && iu >= ops[ik + 1].unit_base) ++ik;
      }
    };
    bool active = w < kEWarps;
    if (active) {
      warp_range(0);
      seek();
      active = is < hdr.n_stages;
    }
    unsigned idle = 0;
    while (__any_sync(0xffffffffu, active)) {
      bool did = false;
      if (active && mbar_test(&s_empty[w][slot], eph ^ 1u)) {
        const EOp& op = ops[ik];
        bulk_load(ring + (size_t)slot * kUnitBytes, op.stream + (int64_t)(iu - op.unit_base) * 32 * BITS,
                  kUnitBytes, &s_full[w][slot]);
        ++n_iss;
        if (++slot == slots) {
          slot = 0;
          eph ^= 1u;
        }
        ++iu;
        seek();
        active = is < hdr.n_stages;
        did = true;
      }
      if (__any_sync(0xffffffffu, did)) {
        idle = 0;
      } else {
        if (*reinterpret_cast<volatile int*>(&s_abort) || ++idle > kEMaxIdle) break;
        __nanosleep(128);
      }
    }
    // every issued copy must land before the CTA exits: wait (bounded) for
    // the phase of the last copy issued into each slot
    if (w < kEWarps) {
      const int last = min(n_iss, slots);
      for (int k = 0; k < last; ++k) {
        const int i = n_iss - 1 - k;  // issue index
        const int s = i % slots;
        mbar_wait(&s_full[w][s], (unsigned)((i / slots) & 1));
      }
    }
    return;
  }

  // ===================== consumer warps =====================
  const int ctid = tid;
  const int P = hdr.n_ranks;
  // epoch = runs of this program so far (each CTA counts itself once per run;
  // counters are never cleared between runs on several ranks)
  if (ctid == 0) s_epoch = atomicAdd(counters + hdr.n_ops + 1, 1u) / (unsigned)G;
  csync();
  const unsigned epoch = s_epoch;
  // On one GPU a stage is complete when its counter reaches G (cleared per
  // run).  On several ranks every CTA counts on its own GPU (word si), and the
  // last CTA of each rank to finish a stage counts once on every rank (word
  // n_ops + 2 + si): complete when that reaches P per run so far.
  const unsigned local_target = (unsigned)G * (epoch + 1u);
  const unsigned target = P > 1 ? (unsigned)P * (epoch + 1u) : (unsigned)G;
  unsigned* const gctr = P > 1 ? counters + hdr.n_ops + 2 : counters;
  const int buf_y = P > 1 ? (int)(epoch & 1u) : 0;
  const uint64_t arena_y = buf_y ? hdr.arena[1] : hdr.arena[0];  // (select: no dynamic index into hdr)
  if (P > 1) {
    // clear the arena buffer the NEXT run writes into: every rank finished
    // writing it (the previous run's last stage completed everywhere before
    // this kernel started), and peers write it again only after this run
    uint4* nz = reinterpret_cast<uint4*>(buf_y ? hdr.arena[0] : hdr.arena[1]);
    const uint64_t n16 = hdr.arena_bytes / 16;
    for (uint64_t i = (uint64_t)blockIdx.x * kECThreads + ctid; i < n16; i += (uint64_t)G * kECThreads)
      nz[i] = make_uint4(0u, 0u, 0u, 0u);
    csync();
  }
  const int64_t v = (int64_t)blockIdx.x * kEWarps + warp;
  const unsigned char* ring = smem + hdr.ring_off + (size_t)warp * slots * kUnitBytes;
  int slot = 0;
  unsigned fph = 0u;
  const uint32_t lanew =
      BITS <= 3 ? (uint32_t)lane * 4u | (ABS ? 0x10000u : 0u) : (uint32_t)lane * 4u * 0x10001u;
  const int src = (lane & ~3) | ((t + 3) & 3);

  int done_upto = -1;  // newest stage known complete on every CTA (same in all consumer threads)
  prefetch_stage(s_st[0], s_ops[0], v, V, lane, ctid, kUnitBytes);
  for (int si = 0, buf = 0; si < hdr.n_stages; ++si, buf = buf == 2 ? 0 : buf + 1) {
    bool ok = true;  // this warp's copies landed
    EStage st = s_st[buf];
    if (st.dep >= 0) st.x = reinterpret_cast<const void*>(arena_y + reinterpret_cast<uint64_t>(st.x));
    const EOp* cops = s_ops[buf];
    const int nbuf = buf == 2 ? 0 : buf + 1;
    etrace(si, 0);
    if (si + 2 < hdr.n_stages) load_desc(si + 2, s_st[nbuf].first_op + s_st[nbuf].n_ops);
    if (si + 1 < hdr.n_stages) prefetch_stage(s_st[nbuf], s_ops[nbuf], v, V, lane, ctid, kUnitBytes);
    const int T = st.total_units;
    const int cb = static_cast<int>((int64_t)blockIdx.x * kEWarps * T / V);
    const int ce = static_cast<int>((int64_t)(blockIdx.x + 1) * kEWarps * T / V);
    const int t0 = cb / st.units_k;
    const int ntiles = ce > cb ? (ce - 1) / st.units_k - t0 + 1 : 0;
    // this CTA's row scales and biases (2 rows per 4-byte copy, zero past n)
    for (int i = ctid; i < ntiles * 16; i += kECThreads) {
      const int tl = i >> 4, pr = (i >> 1) & 7, which = i & 1;
      const int tile_i = t0 + tl;
      int j = 0;
      while (j < st.n_ops - 1 && tile_i >= cops[j + 1].tile_base) ++j;
      const int row = (tile_i - cops[j].tile_base) * kTileRows + 2 * pr;
      const int nb = max(0, min(4, (cops[j].n - row) * 2));
      const uint16_t* base = which ? cops[j].bias : cops[j].scales;
      uint16_t* dst = (which ? s_bi : s_sc) + tl * kTileRows + 2 * pr;
      if (base) cp_async4(dst, base + (nb ? row : 0), nb);
      else cp_async4(dst, cops[j].scales, 0);
    }
    // ---- 1. dependency.  Every CTA publishes its stages in order, so once
    // stage X is complete on all CTAs every stage before X is too.
    if (st.dep > done_upto) {
      if (ctid == 0) {
        unsigned spins = 0;
        while ((P > 1 ? ld_acquire_sys(gctr + st.dep) : ld_acquire(counters + st.dep)) < target) {
          if (++spins > kEMaxSpin) {
            s_abort = 1;
            atomicExch(counters + hdr.n_ops, 1u);
            break;
          }
          __nanosleep(64);
        }
      }
      csync();
      if (s_abort) break;  // same value in every consumer thread
      done_upto = st.dep;
    }
    etrace(si, 1);
    // ---- 2. activations ----
    rotate_stage(st, cops, B, zs, scratch, warp, lane, ctid, si);
    etrace(si, 6);
    etrace(si, 2);

    // ---- 3. decode this warp's units, two per iteration where possible ----
    const int wb = static_cast<int>(v * T / V), we = static_cast<int>((v + 1) * T / V);
    if (wb < we) {
      float accA[2][1][4], accB[2][1][4];
      int cur_tile = -1;
      uint32_t prevg = 0u, prevq = 0u;
      const uint4* zq = reinterpret_cast<const uint4*>(zs);
      const int zrow_q = st.d_pad / 8;  // one job row, in uint4
      int k = 0;                        // op (within the stage) of the current tile
      const int last_op = st.n_ops - 1;
      int zb = 0;
      const int zu = g < B ? 1 : 0;
      auto flush = [&](int tile) {
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int bn = 2 * t + (e & 1);
          const int r = (tile - t0) * kTileRows + g + ((e < 2) ? 0 : 8);
          if (bn < B) atomicAdd(&red[r * Bp + bn], accA[0][0][e] + accA[1][0][e] + accB[0][0][e] + accB[1][0][e]);
        }
      };
      int tile = wb / st.units_k;
      int u = wb - tile * st.units_k;
      int idx = wb;
      while (idx < we) {
        if (tile != cur_tile) {
          if (cur_tile >= 0) flush(cur_tile);
          cur_tile = tile;
          while (k < last_op && tile >= cops[k + 1].tile_base) ++k;
          zb = g < B ? (k * B + g) * zrow_q + t * 4 : static_cast<int>(hdr.zero_q);
#pragma unroll
          for (int q = 0; q < 2; ++q)
#pragma unroll
            for (int e = 0; e < 4; ++e) accA[q][0][e] = accB[q][0][e] = 0.f;
          prevg = prevq = 0u;
          if (u > 0) {  // trellis halo: last chunk of the previous unit of this row tile
            const EOp& op = cops[k];
            const uint4 pv = ldg_stream(op.stream + ((int64_t)(idx - 1 - op.unit_base) * 32 + lane) * BITS);
            prevg = pv.z;
            prevq = pv.w;
          }
        }
        const int slot2 = slot + 1 == slots ? 0 : slot + 1;
        const unsigned fph2 = slot + 1 == slots ? fph ^ 1u : fph;
        if (idx + 1 < we && u + 1 < st.units_k) {
          // two units of the same row tile: independent work for the scheduler
          if (!mbar_wait(&s_full[warp][slot], fph) || !mbar_wait(&s_full[warp][slot2], fph2)) {
            ok = false;
            break;
          }
          uint4 ca[BITS], cb2[BITS];
          const uint4* sa = reinterpret_cast<const uint4*>(ring + (size_t)slot * kUnitBytes) + lane * BITS;
          const uint4* sb = reinterpret_cast<const uint4*>(ring + (size_t)slot2 * kUnitBytes) + lane * BITS;
#pragma unroll
          for (int q = 0; q < BITS; ++q) {
            ca[q] = sa[q];
            cb2[q] = sb[q];
          }
          __syncwarp();
          if (lane == 0) {
            mbar_arrive(&s_empty[warp][slot]);
            mbar_arrive(&s_empty[warp][slot2]);
          }
          slot = slot2 + 1 == slots ? 0 : slot2 + 1;
          fph = slot2 + 1 == slots ? fph2 ^ 1u : fph2;
          decode_unit<BITS, S, ABS>(lut, lanew, zq, ca, prevg, prevq, t, src, zb + zu * (u * 32), zu * 16, accA);
          decode_unit<BITS, S, ABS>(lut, lanew, zq, cb2, prevg, prevq, t, src, zb + zu * (u * 32 + 32), zu * 16, accB);
          u += 2;
          idx += 2;
        } else {
          if (!mbar_wait(&s_full[warp][slot], fph)) {
            ok = false;
            break;
          }
          uint4 ca[BITS];
          const uint4* sa = reinterpret_cast<const uint4*>(ring + (size_t)slot * kUnitBytes) + lane * BITS;
#pragma unroll
          for (int q = 0; q < BITS; ++q) ca[q] = sa[q];
          __syncwarp();
          if (lane == 0) mbar_arrive(&s_empty[warp][slot]);
          slot = slot2;
          fph = fph2;
          decode_unit<BITS, S, ABS>(lut, lanew, zq, ca, prevg, prevq, t, src, zb + zu * (u * 32), zu * 16, accA);
          u += 1;
          idx += 1;
        }
        if (u == st.units_k) {
          u = 0;
          ++tile;
        }
      }
      if (ok && cur_tile >= 0) flush(cur_tile);
    }
    if (!ok) {
      s_abort = 1;
      atomicExch(counters + hdr.n_ops, 2u);
    }
    cp_async_wait_all();  // row scales / biases and the descriptors of stage si + 2
    csync();
    etrace(si, 3);

    // ---- 4. publish: scaled tile partials into y, bias once per row ----
    for (int bn = 0; bn < B; ++bn) {
      for (int rr = ctid; rr < ntiles * kTileRows; rr += kECThreads) {
        const int tile_i = t0 + (rr >> 4);
        int kk = 0;
        while (kk < st.n_ops - 1 && tile_i >= cops[kk + 1].tile_base) ++kk;
        const EOp& op = cops[kk];
        const int row = (tile_i - op.tile_base) * kTileRows + (rr & 15);
        const float part = red[rr * Bp + bn];
        red[rr * Bp + bn] = 0.f;  // ready for the next stage
        if (row >= op.n) continue;
        float val = part * h2f_bits(s_sc[rr]);
        const int first = tile_i * st.units_k;  // unit 0 of this row tile: its CTA adds the bias
        if (first >= cb && first < ce) val += h2f_bits(s_bi[rr]);
        const uint64_t off = op.y + 4ull * ((uint64_t)bn * op.n_full + op.r0 + row);
        if (P == 1) {
          atomicAdd(reinterpret_cast<float*>(off), val);
        } else {
          for (int pr = 0; pr < P; ++pr) atomicAdd(reinterpret_cast<float*>(hdr.peer_arena[2 * pr + buf_y] + off), val);
        }
      }
    }
    // consumer barrier, then a release (cumulative over the writes the
    // barrier ordered before it) ahead of the completion count
    csync();
    if (ctid == 0) {
      if (P == 1) {
        red_release(counters + si);
      } else if (atom_add_acq_rel(counters + si) + 1u == local_target) {
        // last CTA of this rank: its acquire saw every local CTA's release
        // (which covered that CTA's adds into the peers' copies), so one
        // system-scope release publishes the whole rank's stage
        red_release_sys(hdr.peer_ctr, P, hdr.n_ops + 2 + si);
      }
    }
    etrace(si, 4);
    if (s_abort) break;  // read after the barrier above: same in every consumer thread
  }
  cp_async_wait_all();
  if (P > 1 && ctid == 0 && !s_abort) {
    // peers may still be adding into this rank's arena: leave only when the
    // last stage is complete everywhere (the next run clears this buffer's twin)
    unsigned spins = 0;
    while (ld_acquire_sys(gctr + hdr.n_stages - 1) < target) {
      if (++spins > kEMaxSpin) {
        atomicExch(counters + hdr.n_ops, 1u);
        break;
      }
      __nanosleep(64);
    }
  }
}

int sm_count_e() {
  int dev = 0, v = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return 148;
  if (cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || v <= 0) return 148;
  return v;
}

inline uint32_t al128(uint64_t v) { return static_cast<uint32_t>((v + 127) / 128 * 128); }

template <int BITS, int S, bool ABS>
tp_status launch_engine_t(const EHeader& h, const void* image_dev, unsigned* counters, cudaStream_t st) {
  auto kern = tcq_engine_kernel<BITS, S, ABS>;
  static int smem_set[64] = {0};
  if (tp_status s = ensure_smem(kern, h.smem, smem_set, "cudaFuncSetAttribute(engine)")) return s;
  cudaFuncAttributes fa{};
  TP_CUDA_TRY(cudaFuncGetAttributes(&fa, kern), "engine attributes");
  if (fa.sharedSizeBytes > kEStaticSmem)
    return fail(TP_ERR_UNSUPPORTED, "engine: static shared memory %zu above the %u reserved", fa.sharedSizeBytes,
                kEStaticSmem);
  int occ = 0;
  TP_CUDA_TRY(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, kern, kEThreads, h.smem), "engine occupancy");
  if (occ < 1) return fail(TP_ERR_UNSUPPORTED, "engine: one CTA per SM does not fit (smem %u)", h.smem);
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(static_cast<unsigned>(h.grid), 1, 1);
  cfg.blockDim = dim3(kEThreads, 1, 1);
  cfg.dynamicSmemBytes = h.smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeCooperative;  // every CTA resident: dependency waits cannot deadlock
  attr[0].val.cooperative = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  TP_CUDA_TRY(cudaLaunchKernelEx(&cfg, kern, reinterpret_cast<const EHeader*>(image_dev), counters),
              "tcq_engine_kernel launch");
  return check_launch("tcq_engine_kernel");
}

template <int BITS, bool ABS>
tp_status launch_engine_a(const EHeader& h, const void* img, unsigned* c, cudaStream_t st) {
  switch (h.n_states) {
    case 4: return launch_engine_t<BITS, 4, ABS>(h, img, c, st);
    case 8: return launch_engine_t<BITS, 8, ABS>(h, img, c, st);
    case 16: return launch_engine_t<BITS, 16, ABS>(h, img, c, st);
    default: return launch_engine_t<BITS, 64, ABS>(h, img, c, st);
  }
}
template <int BITS>
tp_status launch_engine_s(const EHeader& h, const void* img, unsigned* c, cudaStream_t st) {
  if (BITS <= 3 && h.lut_abs) return launch_engine_a<BITS, true>(h, img, c, st);
  return launch_engine_a<BITS, false>(h, img, c, st);
}

// static shared memory of the kernel that will run a program
template <int BITS, bool ABS>
size_t engine_static_smem_t(int n_states) {
  cudaFuncAttributes fa{};
  cudaError_t e;
  switch (n_states) {
    case 4: e = cudaFuncGetAttributes(&fa, tcq_engine_kernel<BITS, 4, ABS>); break;
    case 8: e = cudaFuncGetAttributes(&fa, tcq_engine_kernel<BITS, 8, ABS>); break;
    case 16: e = cudaFuncGetAttributes(&fa, tcq_engine_kernel<BITS, 16, ABS>); break;
    default: e = cudaFuncGetAttributes(&fa, tcq_engine_kernel<BITS, 64, ABS>); break;
  }
  if (e != cudaSuccess) {
    (void)cudaGetLastError();
    return ~size_t(0);
  }
  return fa.sharedSizeBytes;
}
size_t engine_static_smem_abs(int bits, int n_states) {
  switch (bits) {
    case 1: return engine_static_smem_t<1, true>(n_states);
    case 2: return engine_static_smem_t<2, true>(n_states);
    default: return engine_static_smem_t<3, true>(n_states);
  }
}

}  // namespace

extern "C" int64_t tp_engine_image_bytes(int n_ops) {
  if (n_ops < 1) return -1;
  return (int64_t)sizeof(EHeader) + (int64_t)n_ops * (int64_t)(sizeof(EOp) + sizeof(EStage));
}

extern "C" int64_t tp_engine_counter_bytes(int n_ops) {
  if (n_ops < 1) return -1;
  return (int64_t)(2 * n_ops + 2) * 4;
}

namespace {
// row0 / n_full: first output row and full output rows of every op (shards
// of a tensor-parallel program), or null (whole ops).  tp: null on one GPU.
tp_status build_impl(const tp_engine_op* ops, const int64_t* row0, const int64_t* n_full, int n_ops, int B, int bits,
                     int n_states, const uint16_t* codebook, const tp_engine_tp* tp, void* image,
                     int64_t image_bytes) {
  if (!ops || n_ops < 1 || !codebook || !image) return fail(TP_ERR_ARG, "tp_engine_build: bad arguments");
  const int P = tp ? tp->n_ranks : 1;
  if (tp && (P < 2 || P > 64 || tp->rank < 0 || tp->rank >= P || !tp->arena[0] || !tp->arena[1] ||
             !tp->peer_arena || !tp->peer_counters || tp->arena_bytes <= 0 || tp->arena_bytes % 16 ||
             !aligned(tp->arena[0], 16) || !aligned(tp->arena[1], 16)))
    return fail(TP_ERR_ARG, "tp_engine_build_tp: bad tensor-parallel description");
  auto full_rows = [&](int i) { return n_full ? n_full[i] : ops[i].n; };
  auto first_row = [&](int i) { return row0 ? row0[i] : (int64_t)0; };
  if (image_bytes < tp_engine_image_bytes(n_ops)) return fail(TP_ERR_ARG, "tp_engine_build: image too small");
  if (!aligned(image, 16)) return fail(TP_ERR_ALIGN, "tp_engine_build: image must be 16-byte aligned");
  if (B < 1 || B > kEMaxB) return fail(TP_ERR_UNSUPPORTED, "engine: batch must be 1..%d (got %d)", kEMaxB, B);
  if (bits < 1 || bits > 4) return fail(TP_ERR_UNSUPPORTED, "engine: bits must be 1..4 (got %d)", bits);
  if (log2_states(n_states) < 0) return fail(TP_ERR_UNSUPPORTED, "n_states must be 4, 8, 16 or 64");
  const int G = sm_count_e();
  const int64_t V = (int64_t)G * kEWarps;
  for (int i = 0; i < n_ops; ++i) {
    const tp_engine_op& s = ops[i];
    // on several ranks y (and a dependent x) are byte offsets into the arena
    if (!s.tcq_stream || !s.scales || !s.rot_scale || (!tp && (!s.x || !s.y)) || (tp && s.dep < 0 && !s.x) ||
        s.n < 1 || s.d < 1)
      return fail(TP_ERR_ARG, "engine op %d: bad arguments", i);
    if (first_row(i) < 0 || first_row(i) + s.n > full_rows(i) || first_row(i) % kTileRows)
      return fail(TP_ERR_ARG, "engine op %d: shard rows out of range or not 16-row aligned", i);
    if (tp && ((uint64_t)(uintptr_t)s.y % 16 || (uint64_t)(uintptr_t)s.y + full_rows(i) * B * 4 > (uint64_t)tp->arena_bytes))
      return fail(TP_ERR_ARG, "engine op %d: output outside the arena", i);
    if (!aligned(s.tcq_stream, 16)) return fail(TP_ERR_ALIGN, "engine op %d: stream must be 16-byte aligned", i);
    if (!aligned(s.scales, 4) || (s.bias && !aligned(s.bias, 4)))
      return fail(TP_ERR_ALIGN, "engine op %d: scales and bias must be 4-byte aligned", i);
    if (!valid_dtype(s.x_dtype)) return fail(TP_ERR_ARG, "engine op %d: bad x dtype", i);
    if (s.dep >= i || s.dep < -1) return fail(TP_ERR_ARG, "engine op %d: dep must be -1 or an earlier op", i);
    if (s.dep >= 0 && (s.x_dtype != TP_F32 || full_rows(s.dep) != s.d || s.x != ops[s.dep].y))
      return fail(TP_ERR_ARG, "engine op %d: a dependent input must be op %d's fp32 output", i, s.dep);
    if (s.block < 1 || s.block > 8192 || (s.block & (s.block - 1)) || s.d % s.block)
      return fail(TP_ERR_UNSUPPORTED, "engine op %d: Hadamard block %d unsupported (1..8192)", i, s.block);
    if (s.n > (int64_t)1 << 26 || s.d > (int64_t)1 << 20) return fail(TP_ERR_UNSUPPORTED, "engine op %d too big", i);
  }
  // ---- group consecutive ops with the same input into stages ----
  std::vector<EStage> st;
  std::vector<int> stage_of(n_ops);
  for (int i = 0; i < n_ops; ++i) {
    const tp_engine_op& s = ops[i];
    const int64_t d_pad = pad_to(s.d, kUnitCols);
    bool join = false;
    if (!st.empty()) {
      const EStage& c = st.back();
      const tp_engine_op& f = ops[c.first_op];
      // activations (+ staged rot_scale rows, except for direct stages)
      const int64_t row_bytes = B * d_pad * 2 + (c.direct ? 0 : s.d * 2);
      join = f.x == s.x && f.x_dtype == s.x_dtype && f.dep == s.dep && f.d == s.d && f.block == s.block &&
             c.n_ops < kEMaxStageOps && (int64_t)(c.n_ops + 1) * row_bytes <= kEZStageBytes;
    }
    if (!join) {
      EStage e{};
      e.x = s.x;
      e.x_dtype = s.x_dtype;
      e.dep = s.dep < 0 ? -1 : stage_of[s.dep];
      e.first_op = i;
      e.d = static_cast<int32_t>(s.d);
      e.d_pad = static_cast<int32_t>(d_pad);
      e.units_k = e.d_pad / kUnitCols;
      e.block = s.block;
      int lg = 0;
      while ((1 << lg) < s.block) ++lg;
      e.lg = lg;
      e.norm = static_cast<float>(1.0 / __builtin_sqrt(static_cast<double>(s.block)));
      // raw cp.async staging: 16-byte aligned rows of x and of rot_scale
      e.vec = (s.d % 8 == 0 && aligned(s.x, 16)) ? 1 : 0;
      // blocks above 1024 are transformed one at a time through the fp32 work
      // row anyway; reading them straight from global memory keeps wide
      // inputs (d up to 32K) within shared memory
      e.direct = s.block > 1024 ? 1 : 0;
      st.push_back(e);
    }
    stage_of[i] = static_cast<int>(st.size()) - 1;
    EStage& c = st.back();
    c.n_ops += 1;
    if (!aligned(s.rot_scale, 16)) c.vec = 0;
  }
  const int n_stages = static_cast<int>(st.size());
  EHeader* h = static_cast<EHeader*>(image);
  EOp* eo = reinterpret_cast<EOp*>(h + 1);
  EStage* es = reinterpret_cast<EStage*>(eo + n_ops);
  int64_t max_tiles = 1, zrows_q = 0, scratch_bytes = 0;
  for (int si = 0; si < n_stages; ++si) {
    EStage& c = st[si];
    int64_t tiles = 0;
    for (int i = c.first_op; i < c.first_op + c.n_ops; ++i) {
      EOp e{};
      e.stream = reinterpret_cast<const uint4*>(ops[i].tcq_stream);
      e.scales = ops[i].scales;
      e.bias = ops[i].bias;
      e.rot_scale = ops[i].rot_scale;
      e.y = reinterpret_cast<uint64_t>(ops[i].y);
      e.n = static_cast<int32_t>(ops[i].n);
      e.r0 = static_cast<int32_t>(first_row(i));
      e.n_full = static_cast<int32_t>(full_rows(i));
      e.tile_base = static_cast<int32_t>(tiles);
      e.unit_base = static_cast<int32_t>(tiles * c.units_k);
      eo[i] = e;
      tiles += pad_to(ops[i].n, kTileRows) / kTileRows;
    }
    if (tiles * c.units_k > (int64_t)1 << 30) return fail(TP_ERR_UNSUPPORTED, "engine: stage %d too big", si);
    c.total_tiles = static_cast<int32_t>(tiles);
    c.total_units = static_cast<int32_t>(tiles * c.units_k);
    const int64_t jobs = (int64_t)c.n_ops * B;
    // scratch: staged x rows (raw dtype, or fp32), rot_scale rows, fp32 work row
    const int64_t xes = c.vec && c.x_dtype != TP_F32 ? 2 : 4;
    c.rows_per_pass = c.direct ? B
                                : static_cast<int32_t>(std::max<int64_t>(1, std::min<int64_t>(B, kEXStageBytes / (c.d * xes))));
    c.rs_off = c.direct ? 0 : static_cast<uint32_t>(pad_to((int64_t)c.rows_per_pass * c.d * xes, 16));
    const int64_t rs_end = c.direct ? 0 : c.rs_off + pad_to((int64_t)c.n_ops * c.d * 2, 16);
    // fp32 work row for blocks not done as one warp job
    c.work_off = static_cast<uint32_t>(rs_end);
    // direct stages: as many whole blocks per pass as fit 32 KB (8192 floats)
    c.work_blocks = c.direct ? static_cast<int32_t>(std::max(1, std::min(c.d / c.block, 8192 / c.block))) : 0;
    const int64_t work = c.direct ? (int64_t)c.work_blocks * c.block * 4
                                  : (c.block > 1024 || c.block < 32) ? (int64_t)c.block * 4 : 0;
    scratch_bytes = std::max<int64_t>(scratch_bytes, rs_end + work);
    zrows_q = std::max<int64_t>(zrows_q, jobs * c.d_pad / 8);
    const int64_t per_cta = (kEWarps * (int64_t)c.total_units + V - 1) / V;
    max_tiles = std::max<int64_t>(max_tiles, per_cta / c.units_k + 2);
    es[si] = c;
  }
  EHeader hh{};
  hh.magic = kEMagic;
  hh.n_ops = n_ops;
  hh.n_stages = n_stages;
  hh.B = B;
  hh.bits = bits;
  hh.n_states = n_states;
  hh.grid = G;
  hh.n_ranks = P;
  hh.rank = tp ? tp->rank : 0;
  if (tp) {
    hh.arena[0] = reinterpret_cast<uint64_t>(tp->arena[0]);
    hh.arena[1] = reinterpret_cast<uint64_t>(tp->arena[1]);
    hh.arena_bytes = static_cast<uint64_t>(tp->arena_bytes);
    hh.peer_arena = tp->peer_arena;
    hh.peer_ctr = tp->peer_counters;
  }
  hh.codebook = codebook;
  hh.max_tiles = static_cast<uint32_t>(max_tiles);
  hh.zero_q = static_cast<uint32_t>(zrows_q);  // 64 zero bytes after the widest stage's rows
  const uint32_t lut = bits == 4 ? LutCfg<4>::kLutBytes : LutCfg<3>::kLutBytes;
  const uint64_t zbytes = (uint64_t)zrows_q * 16 + 64;
  const uint64_t scratch = (uint64_t)scratch_bytes;
  const uint64_t red = (uint64_t)max_tiles * kTileRows * 8 * 4;
  const uint64_t rowc = (uint64_t)max_tiles * kTileRows * 2 * 2;  // row scales + biases
  const uint64_t unit = 512u * bits;
  bool placed = false;
  // bits <= 3: try the layout with the pair table at shared-window address
  // 0x10000 (the weight ring and the other buffers around it)
  const char* no_abs = getenv("TP_ENGINE_NO_ABS");
  if (bits <= 3 && !(no_abs && no_abs[0] == '1')) {
    int dev = 0, reserved = 0;
    const size_t st_smem = engine_static_smem_abs(bits, n_states);
    if (st_smem != ~size_t(0) && cudaGetDevice(&dev) == cudaSuccess &&
        cudaDeviceGetAttribute(&reserved, cudaDevAttrReservedSharedMemoryPerBlock, dev) == cudaSuccess &&
        st_smem <= kEStaticSmem) {
      const uint64_t base = (reserved + st_smem + 127) / 128 * 128;  // dynamic area, 128-byte aligned
      const uint64_t dyn_max = 227u * 1024u - st_smem;
      if (base < 0x10000u && 0x10000u - base + lut <= dyn_max) {
        const uint64_t front = 0x10000u - base, back0 = front + lut;
        for (int slots = kEMaxSlots; slots >= 2 && !placed; --slots) {
          // first fit, largest first: ring, scratch, zs, red, rowc -> front or back
          struct Item { uint64_t bytes; uint32_t* off; } items[5] = {
              {(uint64_t)kEWarps * slots * unit, &hh.ring_off}, {scratch, &hh.scratch_off}, {zbytes, &hh.z_off},
              {red, &hh.red_off}, {rowc, &hh.sc_off}};
          uint64_t f = 0, b = back0;
          bool ok = true;
          for (auto& it : items) {
            const uint64_t sz = al128(it.bytes);
            if (f + sz <= front) {
              *it.off = static_cast<uint32_t>(f);
              f += sz;
            } else if (b + sz <= dyn_max) {
              *it.off = static_cast<uint32_t>(b);
              b += sz;
            } else {
              ok = false;
              break;
            }
          }
          if (ok) {
            placed = true;
            hh.slots = slots;
            hh.lut_off = static_cast<uint32_t>(front);
            hh.lut_abs = 1;
            hh.dyn_base = static_cast<uint32_t>(base);
            hh.smem = static_cast<uint32_t>(al128(b));
          }
        }
      }
    }
  }
  if (!placed) {
    const uint64_t fixed = lut + al128(zbytes) + al128(scratch) + al128(red) + al128(rowc);
    const uint64_t budget = 227u * 1024u - kEStaticSmem;
    if (fixed + kEWarps * 2 * unit > budget)
      return fail(TP_ERR_UNSUPPORTED, "engine: activations (%lld halves, B=%d) do not fit shared memory",
                  (long long)(zrows_q * 8), B);
    hh.slots = static_cast<int32_t>(std::min<uint64_t>(kEMaxSlots, (budget - fixed) / (kEWarps * unit)));
    hh.lut_off = 0;
    hh.lut_abs = 0;
    hh.ring_off = lut;
    hh.z_off = al128(hh.ring_off + (uint64_t)kEWarps * hh.slots * unit);
    hh.scratch_off = al128(hh.z_off + zbytes);
    hh.red_off = al128(hh.scratch_off + scratch);
    hh.sc_off = al128(hh.red_off + red);
    hh.smem = al128(hh.sc_off + rowc);
  }
  *h = hh;
  return clear_ok();
}
}  // namespace

extern "C" tp_status tp_engine_build(const tp_engine_op* ops, int n_ops, int B, int bits, int n_states,
                                     const uint16_t* codebook, void* image, int64_t image_bytes) {
  return build_impl(ops, nullptr, nullptr, n_ops, B, bits, n_states, codebook, nullptr, image, image_bytes);
}

extern "C" tp_status tp_engine_build_tp(const tp_engine_op* ops, const int64_t* row0, const int64_t* n_full,
                                        int n_ops, int B, int bits, int n_states, const uint16_t* codebook,
                                        const tp_engine_tp* tp, void* image, int64_t image_bytes) {
  if (!tp || !row0 || !n_full) return fail(TP_ERR_ARG, "tp_engine_build_tp: bad arguments");
  return build_impl(ops, row0, n_full, n_ops, B, bits, n_states, codebook, tp, image, image_bytes);
}

extern "C" tp_status tp_engine_run(const void* image_dev, const void* image_host, unsigned* counters, void* stream) {
  if (!image_dev || !image_host || !counters) return fail(TP_ERR_ARG, "tp_engine_run: bad arguments");
  if (!aligned(image_dev, 16)) return fail(TP_ERR_ALIGN, "tp_engine_run: image must be 16-byte aligned");
  const EHeader& h = *static_cast<const EHeader*>(image_host);
  if (h.magic != kEMagic) return fail(TP_ERR_ARG, "tp_engine_run: not an engine image");
  if (h.grid != sm_count_e()) return fail(TP_ERR_ARG, "tp_engine_run: image built for another device");
  cudaStream_t st = as_stream(stream);
  switch (h.bits) {
    case 1: return launch_engine_s<1>(h, image_dev, counters, st);
    case 2: return launch_engine_s<2>(h, image_dev, counters, st);
    case 3: return launch_engine_s<3>(h, image_dev, counters, st);
    default: return launch_engine_s<4>(h, image_dev, counters, st);
  }
}

#ifdef TP_TRACE
extern "C" TP_API int tp_engine_trace_read(unsigned long long* host) {
  return (int)cudaMemcpyFromSymbol(host, g_etrace, sizeof(g_etrace));
}
#endif

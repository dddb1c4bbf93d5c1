// Persistent decode engine: a whole chain of packed-TCQ linears in one launch.
//
// One CTA per SM stays resident for the program (cooperative launch).  It
// builds the pair table once.  Each op's weight units (16 rows x 256
// columns, tile-major, contiguous in the native stream) are split into
// equal contiguous runs, one per warp of the grid; lane 0 of every warp
// keeps a ring of `slots` units in flight with bulk copies, walking its
// runs op after op, so the weights of later layers stream in while an op
// waits for its activations.  Per op and CTA:
//   1. wait (bounded) until every CTA finished the op producing x;
//   2. stage x * rot_scale (fp32) in shared memory in one round of loads,
//      then transform whole Hadamard blocks (warp registers + shuffles for
//      blocks <= 1024, CTA-wide above) into fp16 activations in the
//      decoder's permuted pair order (CTA-wide too for blocks < 32);
//   3. decode units exactly as the per-call GEMV (level words, pair table,
//      m16n8k16 MMA), accumulating per row tile in registers, then in
//      shared memory;
//   4. scale (and bias, once per row) the CTA's tile partials and add them
//      to the op's fp32 output with atomics; publish completion.
#include <algorithm>

#include "tp_decode.cuh"
#include "tp_rotate.cuh"

using namespace tp;

namespace {

constexpr int kEWarps = 8;
constexpr int kEThreads = kEWarps * 32;
constexpr int kEMaxB = 4;
constexpr int kEMaxSlots = 16;
constexpr int kEScratchFloats = 8192;      // largest Hadamard block
constexpr int kEScratchRowFloats = 12288;  // fp32 activation staging target
constexpr unsigned kEMaxSpin = 1u << 24;   // dependency polls (~1 s with backoff)
constexpr int kEMagic = 0x54504531;        // "TPE1"

struct EOp {
  const uint4* stream;
  const uint16_t* scales;
  const uint16_t* bias;
  const uint16_t* rot_scale;
  const void* x;
  float* y;
  int32_t x_dtype, dep, n, d;
  int32_t n_pad, d_pad, units_k, row_tiles;
  int32_t block, lg, total_units, pad0;
  float norm;
  int32_t pad1[3];
};

struct alignas(16) EHeader {
  int32_t magic, n_ops, B, bits;
  int32_t n_states, grid, slots, max_tiles;
  const uint16_t* codebook;
  uint32_t ring_off, z_off, scratch_off, red_off;
  uint32_t smem, d_pad_max, big_blocks, rows_per_pass;
};

#ifdef TP_TRACE
// development-only timeline: CTA 0 and CTA gridDim/2 stamp each op's phases
static __device__ unsigned long long g_etrace[2][512][6];
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

__device__ __forceinline__ float load_x(const EOp& op, int64_t i) {
  if (op.x_dtype == TP_F32) return __ldcg(reinterpret_cast<const float*>(op.x) + i);  // produced by this grid
  return load_as_float(op.x, i, op.x_dtype);
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
    const bool upper = lane & m;
#pragma unroll
    for (int r = 0; r < R; ++r) {
      const float o = __shfl_xor_sync(0xffffffffu, v[r], m);
      v[r] = upper ? o - v[r] : v[r] + o;
    }
  }
}

// one Hadamard block (32R columns of fp32 x*rot_scale at `s`) -> zs row
template <int R>
__device__ __forceinline__ void warp_block_rotate(const float* s, __half* zrow, float norm, int lane, int zp) {
  float v[R];
#pragma unroll
  for (int r = 0; r < R; ++r) v[r] = s[lane + 32 * r];
  warp_fwht_regs<R>(v, lane);
#pragma unroll
  for (int r = 0; r < R; ++r) zrow[32 * r + zp] = __float2half_rn(v[r] * norm);
}

// x (all rows, full width) -> fp16 rotated activations in zs.  All threads
// first stage x * rot_scale for `rows_per_pass` rows in fp32 scratch (one
// round of independent loads), then warps transform whole blocks from shared
// memory (blocks <= 1024) or the CTA does (larger blocks).
__device__ void rotate_op(const EOp& op, int B, int rows_per_pass, __half* zs, float* scratch, int warp, int lane,
                          int tid) {
  const int zp = zperm_pos(lane);
  const int nblk = op.d / op.block;
  for (int b0 = 0; b0 < B; b0 += rows_per_pass) {
    const int rows = B - b0 < rows_per_pass ? B - b0 : rows_per_pass;
    for (int rr = 0; rr < rows; ++rr)
      for (int c = tid; c < op.d; c += kEThreads)
        scratch[rr * op.d + c] = load_x(op, (int64_t)(b0 + rr) * op.d + c) * h2f_bits(op.rot_scale[c]);
    __syncthreads();
    if (op.block >= 32 && op.block <= 1024) {
      const int R = op.block / 32;
      for (int job = warp; job < rows * nblk; job += kEWarps) {
        const int rr = job / nblk, k = job - rr * nblk;
        const float* s = scratch + rr * op.d + k * op.block;
        __half* zrow = zs + (size_t)(b0 + rr) * op.d_pad + k * op.block;
        switch (R) {
          case 1: warp_block_rotate<1>(s, zrow, op.norm, lane, zp); break;
          case 2: warp_block_rotate<2>(s, zrow, op.norm, lane, zp); break;
          case 4: warp_block_rotate<4>(s, zrow, op.norm, lane, zp); break;
          case 8: warp_block_rotate<8>(s, zrow, op.norm, lane, zp); break;
          case 16: warp_block_rotate<16>(s, zrow, op.norm, lane, zp); break;
          default: warp_block_rotate<32>(s, zrow, op.norm, lane, zp); break;
        }
      }
    } else {
      fwht_shared(scratch, rows * op.d, op.lg);
      for (int rr = 0; rr < rows; ++rr)
        for (int c = tid; c < op.d; c += kEThreads)
          zs[(size_t)(b0 + rr) * op.d_pad + (c & ~31) + zperm_pos(c & 31)] =
              __float2half_rn(scratch[rr * op.d + c] * op.norm);
    }
    __syncthreads();
  }
  // padding columns [d, d_pad) of every row
  for (int b = 0; b < B; ++b)
    for (int c = op.d + tid; c < op.d_pad; c += kEThreads)
      zs[(size_t)b * op.d_pad + (c & ~31) + zperm_pos(c & 31)] = __float2half_rn(0.f);
}

template <int BITS, int S>
__global__ void __launch_bounds__(kEThreads, 1) tcq_engine_kernel(const EHeader* __restrict__ hdr_g,
                                                                  unsigned* __restrict__ counters) {
  extern __shared__ __align__(128) unsigned char smem[];
  __shared__ __align__(8) uint64_t s_bar[kEWarps][kEMaxSlots];
  __shared__ int s_abort;

  const EHeader hdr = *hdr_g;
  const EOp* ops = reinterpret_cast<const EOp*>(hdr_g + 1);
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int g = lane >> 2, t = lane & 3;
  const int G = gridDim.x;
  const int64_t V = (int64_t)G * kEWarps, v = (int64_t)blockIdx.x * kEWarps + warp;
  const int B = hdr.B, Bp = 8;
  constexpr unsigned kUnitBytes = 32u * 16u * BITS;
  unsigned char* lut = smem;
  unsigned char* ring = smem + hdr.ring_off + (size_t)warp * hdr.slots * kUnitBytes;
  __half* zs = reinterpret_cast<__half*>(smem + hdr.z_off);
  float* scratch = reinterpret_cast<float*>(smem + hdr.scratch_off);
  float* red = reinterpret_cast<float*>(smem + hdr.red_off);
  const int slots = hdr.slots;

  const uint32_t cbv = lane < (1 << (BITS + 1)) ? hdr.codebook[lane] : 0u;
  if (tid == 0) s_abort = 0;

  // ---- issue cursor (lane 0): this warp's unit runs, op after op ----
  int io = 0;
  int64_t iidx = 0, iend = 0;
  int n_issued = 0;
  auto warp_range = [&](int o, int64_t& b, int64_t& e) {
    const int64_t T = ops[o].total_units;
    b = v * T / V;
    e = (v + 1) * T / V;
  };
  auto skip_empty = [&]() {
    while (io < hdr.n_ops && iidx >= iend) {
      ++io;
      if (io < hdr.n_ops) warp_range(io, iidx, iend);
    }
  };
  if (lane == 0) {
    warp_range(0, iidx, iend);
    skip_empty();
    for (int s = 0; s < slots; ++s) mbar_init(&s_bar[warp][s], 1);
    fence_mbar_init();
    for (int s = 0; s < slots && io < hdr.n_ops; ++s) {
      bulk_load(ring + (size_t)s * kUnitBytes, ops[io].stream + iidx * 32 * BITS, kUnitBytes, &s_bar[warp][s]);
      ++n_issued;
      ++iidx;
      skip_empty();
    }
  }
  build_lut<BITS>(lut, cbv, warp, lane, kEWarps);
  // zero block read by lanes of batch rows >= B
  if (tid < 16) reinterpret_cast<uint32_t*>(zs + (size_t)B * hdr.d_pad_max)[tid] = 0u;
  __syncthreads();

  int slot = 0;
  unsigned parity = 0u;
  int n_consumed = 0;
  const uint32_t lanew = BITS <= 3 ? (uint32_t)lane * 4u : (uint32_t)lane * 4u * 0x10001u;
  const int src = (lane & ~3) | ((t + 3) & 3);

  for (int o = 0; o < hdr.n_ops; ++o) {
    bool ok = true;  // this warp's copies landed
    const EOp op = ops[o];
    etrace(o, 0);
    // ---- 1. dependency ----
    if (op.dep >= 0) {
      if (tid == 0) {
        volatile unsigned* c = counters + op.dep;
        unsigned spins = 0;
        while (*c < (unsigned)G) {
          if (++spins > kEMaxSpin) {
            s_abort = 1;
            atomicExch(counters + hdr.n_ops, 1u);
            break;
          }
          __nanosleep(64);
        }
        __threadfence();
      }
      __syncthreads();
      if (s_abort) break;  // CTA-uniform
    }
    etrace(o, 1);
    // ---- 2. activations ----
    rotate_op(op, B, hdr.rows_per_pass, zs, scratch, warp, lane, tid);
    const int64_t T = op.total_units;
    const int64_t cb = (int64_t)blockIdx.x * kEWarps * T / V, ce = (int64_t)(blockIdx.x + 1) * kEWarps * T / V;
    const int t0 = static_cast<int>(cb / op.units_k);
    const int ntiles = ce > cb ? static_cast<int>((ce - 1) / op.units_k) - t0 + 1 : 0;
    for (int i = tid; i < ntiles * kTileRows * Bp; i += kEThreads) red[i] = 0.f;
    __syncthreads();
    etrace(o, 2);

    // ---- 3. decode this warp's units ----
    int64_t wb, we;
    warp_range(o, wb, we);
    if (wb < we) {
      float acc[2][1][4];
      int cur_tile = -1;
      uint32_t prevP1g = 0u, prevP1q = 0u;
      const uint4* zq = reinterpret_cast<const uint4*>(zs);
      const int zrow_stride = op.d_pad / 8;
      const int zb = g < B ? g * zrow_stride + t * 4 : B * (int)hdr.d_pad_max / 8;
      const int zu = g < B ? 1 : 0;
      auto flush = [&](int tile) {
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int bn = 2 * t + (e & 1);
          const int r = (tile - t0) * kTileRows + g + ((e < 2) ? 0 : 8);
          if (bn < B) atomicAdd(&red[r * Bp + bn], acc[0][0][e] + acc[1][0][e]);
        }
      };
      int tile = static_cast<int>(wb / op.units_k);
      int u = static_cast<int>(wb - (int64_t)tile * op.units_k);
      for (int64_t idx = wb; idx < we; ++idx) {
        if (tile != cur_tile) {
          if (cur_tile >= 0) flush(cur_tile);
          cur_tile = tile;
#pragma unroll
          for (int q = 0; q < 2; ++q) acc[q][0][0] = acc[q][0][1] = acc[q][0][2] = acc[q][0][3] = 0.f;
          prevP1g = prevP1q = 0u;
          if (u > 0) {  // trellis halo: last chunk of the previous unit of this row tile
            const uint4 pv = ldg_stream(op.stream + ((idx - 1) * 32 + lane) * BITS);
            prevP1g = pv.z;
            prevP1q = pv.w;
          }
        }
        if (!mbar_wait(&s_bar[warp][slot], parity)) {
          ok = false;
          break;
        }
        uint4 cur[BITS];
        const uint4* su = reinterpret_cast<const uint4*>(ring + (size_t)slot * kUnitBytes) + lane * BITS;
#pragma unroll
        for (int k = 0; k < BITS; ++k) cur[k] = su[k];
        __syncwarp();
        if (lane == 0 && io < hdr.n_ops) {  // refill with the next unit of this warp's stream
          fence_proxy_async();
          bulk_load(ring + (size_t)slot * kUnitBytes, ops[io].stream + iidx * 32 * BITS, kUnitBytes,
                    &s_bar[warp][slot]);
          ++n_issued;
          ++iidx;
          skip_empty();
        }
        ++n_consumed;
        if (++slot == slots) {
          slot = 0;
          parity ^= 1u;
        }
        const uint32_t P0g = cur[0].x, P0q = cur[0].y, P1g = cur[0].z, P1q = cur[0].w;
        const uint32_t H0g = __shfl_sync(0xffffffffu, t == 3 ? prevP1g : P0g, src);
        const uint32_t H0q = __shfl_sync(0xffffffffu, t == 3 ? prevP1q : P0q, src);
        const uint32_t H1g = __shfl_sync(0xffffffffu, t == 3 ? P0g : P1g, src);
        const uint32_t H1q = __shfl_sync(0xffffffffu, t == 3 ? P0q : P1q, src);
        prevP1g = P1g;
        prevP1q = P1q;
#pragma unroll
        for (int cgi = 0; cgi < 2; ++cgi) {
          int zoff[1];
          zoff[0] = zb + zu * (u * 32 + cgi * 16);
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
          process_chunk<BITS, S, 1>(lut, lanew, zq, Pg, Hg, Pq, Hq, Mg0, Mg1, Mg2, Mq0, Mq1, Mq2, zoff, acc);
        }
        if (++u == op.units_k) {
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
    __syncthreads();
    etrace(o, 3);

    // ---- 4. publish: scaled tile partials into y, bias once per row ----
    for (int i = tid; i < ntiles * kTileRows * B; i += kEThreads) {
      const int bn = i / (ntiles * kTileRows);
      const int rr = i - bn * ntiles * kTileRows;
      const int tile_i = t0 + rr / kTileRows;
      const int row = tile_i * kTileRows + (rr % kTileRows);
      if (row >= op.n) continue;
      float val = red[rr * Bp + bn] * h2f_bits(op.scales[row]);
      const int64_t first = (int64_t)tile_i * op.units_k;  // unit 0 of this row tile
      if (op.bias && first >= cb && first < ce) val += h2f_bits(op.bias[row]);
      atomicAdd(op.y + (int64_t)bn * op.n + row, val);
    }
    __threadfence();
    __syncthreads();
    if (tid == 0) atomicAdd(counters + o, 1u);
    etrace(o, 4);
    if (s_abort) break;  // read after the barrier above: CTA-uniform
  }

  // ---- drain copies still in flight (only after an abort) ----
  if (lane == 0) {
    while (n_consumed < n_issued) {
      if (!mbar_wait(&s_bar[warp][slot], parity)) break;
      ++n_consumed;
      if (++slot == slots) {
        slot = 0;
        parity ^= 1u;
      }
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

template <int BITS, int S>
tp_status launch_engine_t(const EHeader& h, const void* image_dev, unsigned* counters, cudaStream_t st) {
  auto kern = tcq_engine_kernel<BITS, S>;
  static int smem_set[64] = {0};
  if (tp_status s = ensure_smem(kern, h.smem, smem_set, "cudaFuncSetAttribute(engine)")) return s;
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

template <int BITS>
tp_status launch_engine_s(const EHeader& h, const void* img, unsigned* c, cudaStream_t st) {
  switch (h.n_states) {
    case 4: return launch_engine_t<BITS, 4>(h, img, c, st);
    case 8: return launch_engine_t<BITS, 8>(h, img, c, st);
    case 16: return launch_engine_t<BITS, 16>(h, img, c, st);
    default: return launch_engine_t<BITS, 64>(h, img, c, st);
  }
}

}  // namespace

extern "C" int64_t tp_engine_image_bytes(int n_ops) {
  if (n_ops < 1) return -1;
  return (int64_t)sizeof(EHeader) + (int64_t)n_ops * (int64_t)sizeof(EOp);
}

extern "C" int64_t tp_engine_counter_bytes(int n_ops) {
  if (n_ops < 1) return -1;
  return (int64_t)(n_ops + 1) * 4;
}

extern "C" tp_status tp_engine_build(const tp_engine_op* ops, int n_ops, int B, int bits, int n_states,
                                     const uint16_t* codebook, void* image, int64_t image_bytes) {
  if (!ops || n_ops < 1 || !codebook || !image) return fail(TP_ERR_ARG, "tp_engine_build: bad arguments");
  if (image_bytes < tp_engine_image_bytes(n_ops)) return fail(TP_ERR_ARG, "tp_engine_build: image too small");
  if (!aligned(image, 16)) return fail(TP_ERR_ALIGN, "tp_engine_build: image must be 16-byte aligned");
  if (B < 1 || B > kEMaxB) return fail(TP_ERR_UNSUPPORTED, "engine: batch must be 1..%d (got %d)", kEMaxB, B);
  if (bits < 1 || bits > 4) return fail(TP_ERR_UNSUPPORTED, "engine: bits must be 1..4 (got %d)", bits);
  if (log2_states(n_states) < 0) return fail(TP_ERR_UNSUPPORTED, "n_states must be 4, 8, 16 or 64");
  EHeader* h = static_cast<EHeader*>(image);
  EOp* eo = reinterpret_cast<EOp*>(h + 1);
  const int G = sm_count_e();
  const int64_t V = (int64_t)G * kEWarps;
  int64_t d_pad_max = 0, max_tiles = 1;
  bool big = false;
  for (int i = 0; i < n_ops; ++i) {
    const tp_engine_op& s = ops[i];
    if (!s.tcq_stream || !s.scales || !s.rot_scale || !s.x || !s.y || s.n < 1 || s.d < 1)
      return fail(TP_ERR_ARG, "engine op %d: bad arguments", i);
    if (!aligned(s.tcq_stream, 16)) return fail(TP_ERR_ALIGN, "engine op %d: stream must be 16-byte aligned", i);
    if (!valid_dtype(s.x_dtype)) return fail(TP_ERR_ARG, "engine op %d: bad x dtype", i);
    if (s.dep >= i || s.dep < -1) return fail(TP_ERR_ARG, "engine op %d: dep must be -1 or an earlier op", i);
    if (s.dep >= 0 && (s.x_dtype != TP_F32 || ops[s.dep].n != s.d || s.x != ops[s.dep].y))
      return fail(TP_ERR_ARG, "engine op %d: a dependent input must be op %d's fp32 output", i, s.dep);
    if (s.block < 1 || s.block > kEScratchFloats || (s.block & (s.block - 1)) || s.d % s.block)
      return fail(TP_ERR_UNSUPPORTED, "engine op %d: Hadamard block %d unsupported (1..8192)", i, s.block);
    if (s.n > (int64_t)1 << 30 || s.d > (int64_t)1 << 20) return fail(TP_ERR_UNSUPPORTED, "engine op %d too big", i);
    EOp e{};
    e.stream = reinterpret_cast<const uint4*>(s.tcq_stream);
    e.scales = s.scales;
    e.bias = s.bias;
    e.rot_scale = s.rot_scale;
    e.x = s.x;
    e.y = s.y;
    e.x_dtype = s.x_dtype;
    e.dep = s.dep;
    e.n = static_cast<int32_t>(s.n);
    e.d = static_cast<int32_t>(s.d);
    e.n_pad = static_cast<int32_t>(pad_to(s.n, kTileRows));
    e.d_pad = static_cast<int32_t>(pad_to(s.d, kUnitCols));
    e.units_k = e.d_pad / kUnitCols;
    e.row_tiles = e.n_pad / kTileRows;
    e.block = s.block;
    int lg = 0;
    while ((1 << lg) < s.block) ++lg;
    e.lg = lg;
    e.total_units = e.row_tiles * e.units_k;
    e.norm = static_cast<float>(1.0 / __builtin_sqrt(static_cast<double>(s.block)));
    eo[i] = e;
    d_pad_max = std::max<int64_t>(d_pad_max, e.d_pad);
    const int64_t per_cta = (kEWarps * (int64_t)e.total_units + V - 1) / V;
    max_tiles = std::max<int64_t>(max_tiles, per_cta / e.units_k + 2);
    big = big || s.block > 1024;
  }
  EHeader hh{};
  hh.magic = kEMagic;
  hh.n_ops = n_ops;
  hh.B = B;
  hh.bits = bits;
  hh.n_states = n_states;
  hh.grid = G;
  hh.max_tiles = static_cast<int32_t>(max_tiles);
  hh.codebook = codebook;
  hh.d_pad_max = static_cast<uint32_t>(d_pad_max);
  hh.big_blocks = big ? 1u : 0u;
  const uint32_t lut = bits == 4 ? LutCfg<4>::kLutBytes : LutCfg<3>::kLutBytes;
  const uint64_t zbytes = (uint64_t)B * d_pad_max * 2 + 64;
  // fp32 staging of x * rot_scale: whole rows, as many as fit kEScratchRowFloats
  const int64_t rpp = std::max<int64_t>(1, std::min<int64_t>(B, kEScratchRowFloats / d_pad_max));
  hh.rows_per_pass = static_cast<uint32_t>(rpp);
  const uint64_t scratch = (uint64_t)std::max<int64_t>(rpp * d_pad_max, big ? kEScratchFloats : 0) * 4;
  const uint64_t red = (uint64_t)max_tiles * kTileRows * 8 * 4;
  const uint64_t fixed = lut + al128(zbytes) + al128(scratch) + al128(red);
  const uint64_t budget = 227u * 1024u - 2048u;
  const uint64_t unit = 512u * bits;
  if (fixed + kEWarps * 2 * unit > budget)
    return fail(TP_ERR_UNSUPPORTED, "engine: activations (d=%lld, B=%d) do not fit shared memory",
                (long long)d_pad_max, B);
  hh.slots = static_cast<int32_t>(std::min<uint64_t>(kEMaxSlots, (budget - fixed) / (kEWarps * unit)));
  hh.ring_off = lut;
  hh.z_off = al128(hh.ring_off + (uint64_t)kEWarps * hh.slots * unit);
  hh.scratch_off = al128(hh.z_off + zbytes);
  hh.red_off = al128(hh.scratch_off + scratch);
  hh.smem = al128(hh.red_off + red);
  *h = hh;
  return clear_ok();
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

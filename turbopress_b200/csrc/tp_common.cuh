// Shared host/device helpers for the turbopress_b200 kernels (sm_100a).
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <cstdarg>
#include <cstdio>

#include "../../include/turbopress_b200.h"

namespace tp {

// ---------------------------------------------------------------------------
// error reporting (per host thread)
// ---------------------------------------------------------------------------
extern thread_local char g_last_error[512];

inline tp_status fail(tp_status code, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_last_error, sizeof(g_last_error), fmt, ap);
  va_end(ap);
  return code;
}

inline tp_status clear_ok() {
  g_last_error[0] = 0;
  return TP_OK;
}

// Check the last launch (non-sticky errors are cleared by cudaGetLastError).
inline tp_status check_launch(const char* what) {
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return fail(TP_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
  return clear_ok();
}

// On failure the error is also cleared from the runtime's last-error slot so
// it cannot be misattributed to a later launch check.
#define TP_CUDA_TRY(call, what)                                                    \
  do {                                                                             \
    cudaError_t _e = (call);                                                       \
    if (_e != cudaSuccess) {                                                       \
      (void)cudaGetLastError();                                                    \
      return fail(TP_ERR_CUDA, "%s: %s", what, cudaGetErrorString(_e));            \
    }                                                                              \
  } while (0)

// Raise a kernel's dynamic shared memory limit to at least `bytes` (once per
// device and size).  `slot` is a per-kernel array of the sizes already set.
template <class K>
inline tp_status ensure_smem(K kernel, size_t bytes, int* slot, const char* what) {
  int dev = 0;
  TP_CUDA_TRY(cudaGetDevice(&dev), "cudaGetDevice");
  if (dev < 0 || dev >= 64) return fail(TP_ERR_UNSUPPORTED, "device index %d out of range", dev);
  if (bytes <= 48 * 1024 || (size_t)__atomic_load_n(&slot[dev], __ATOMIC_ACQUIRE) >= bytes) return TP_OK;
  TP_CUDA_TRY(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes), what);
  int cur = __atomic_load_n(&slot[dev], __ATOMIC_ACQUIRE);
  while (cur < (int)bytes && !__atomic_compare_exchange_n(&slot[dev], &cur, (int)bytes, false, __ATOMIC_ACQ_REL,
                                                          __ATOMIC_ACQUIRE)) {
  }
  return TP_OK;
}

inline cudaStream_t as_stream(void* s) { return reinterpret_cast<cudaStream_t>(s); }

inline bool aligned(const void* p, uintptr_t a) { return (reinterpret_cast<uintptr_t>(p) & (a - 1)) == 0; }

inline int log2_states(int n_states) {
  switch (n_states) {
    case 4: return 2;
    case 8: return 3;
    case 16: return 4;
    case 64: return 6;
    default: return -1;
  }
}

// ---------------------------------------------------------------------------
// trellis taps
//
// The shift-register trellis (turbopress/trellis.py:55-87) emits, at column
// t, subset = parity(x & g1) << 1 | parity(x & g0) with x = (b_t << m) | state
// and state bit k = b_{t-1-k}.  Writing D_k for the path bit b_{t-k}, the
// generator bit for D_0 is bit m and for D_k (k >= 1) it is bit k-1, so each
// subset bit is an XOR of delayed path bits: a GF(2) convolution.  kmask()
// lists the delays k whose generator bit is set.
// ---------------------------------------------------------------------------
__host__ __device__ constexpr unsigned gen0(int s) { return s == 4 ? 05u : s == 8 ? 015u : s == 16 ? 023u : 0133u; }
__host__ __device__ constexpr unsigned gen1(int s) { return s == 4 ? 07u : s == 8 ? 017u : s == 16 ? 035u : 0171u; }
__host__ __device__ constexpr int mlog(int s) { return s == 4 ? 2 : s == 8 ? 3 : s == 16 ? 4 : 6; }
__host__ __device__ constexpr unsigned kmask(unsigned g, int m) {
  unsigned r = 0;
  for (int k = 0; k <= m; ++k)
    if ((g >> (k == 0 ? m : k - 1)) & 1u) r |= 1u << k;
  return r;
}

// Runtime form (decode kernels that are not templated on S).
__host__ __device__ inline void tap_masks(int n_states, unsigned& k0, unsigned& k1, int& m) {
  m = mlog(n_states);
  k0 = kmask(gen0(n_states), m);
  k1 = kmask(gen1(n_states), m);
}

// subset of one column from the delay window: bit k of `win` = b_{t-k}.
__host__ __device__ inline unsigned subset_of_window(unsigned win, unsigned k0, unsigned k1) {
#ifdef __CUDA_ARCH__
  return ((__popc(win & k1) & 1u) << 1) | (__popc(win & k0) & 1u);
#else
  return ((__builtin_popcount(win & k1) & 1u) << 1) | (__builtin_popcount(win & k0) & 1u);
#endif
}

// ---------------------------------------------------------------------------
// element type helpers
// ---------------------------------------------------------------------------
__device__ __forceinline__ float load_as_float(const void* p, int64_t i, int dtype) {
  if (dtype == TP_F16) return __half2float(reinterpret_cast<const __half*>(p)[i]);
  if (dtype == TP_BF16) return __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(p)[i]);
  return reinterpret_cast<const float*>(p)[i];
}

__device__ __forceinline__ void store_from_float(void* p, int64_t i, int dtype, float v) {
  if (dtype == TP_F16) reinterpret_cast<__half*>(p)[i] = __float2half_rn(v);
  else if (dtype == TP_BF16) reinterpret_cast<__nv_bfloat16*>(p)[i] = __float2bfloat16_rn(v);
  else reinterpret_cast<float*>(p)[i] = v;
}

__device__ __forceinline__ float h2f_bits(uint16_t b) { return __half2float(__ushort_as_half(b)); }

inline bool valid_dtype(int t) { return t == TP_F16 || t == TP_F32 || t == TP_BF16; }

// ---------------------------------------------------------------------------
// native stream geometry
//
// Tile unit = 16 rows x 256 columns.  Lane (g, t) of the warp (g = lane/4,
// t = lane%4) owns rows {g, g+8} and the 32-column chunks {t, 4+t} of the
// unit, 4*bits words = 16*bits bytes:
//   uint4 #0     : path words   {P(g,c0), P(g+8,c0), P(g,c1), P(g+8,c1)}
//   uint4 #1..   : member words in the same order (bit arrangement below)
// Units are stored row-tile major: offset = ((rt * units_k + u) * 32 + lane)
// * 16 * bits.
//
// Inside a 32-column chunk the decoder forms four "level words" L_a..L_d;
// byte j of L_w holds two 4-bit level nibbles (low nibble = column
// 8j+lo[w], high nibble = column 8j+hi[w]) with lo/hi = a:(0,4) b:(2,6)
// c:(1,5) d:(3,7).  Pair p = 4*w + j of the chunk is that byte.
// ---------------------------------------------------------------------------
constexpr int kUnitCols = 256;
constexpr int kTileRows = 16;

__host__ __device__ inline int64_t pad_to(int64_t v, int64_t m) { return (v + m - 1) / m * m; }

__host__ __device__ inline int64_t stream_bytes(int64_t n, int64_t d, int bits) {
  return pad_to(n, kTileRows) * pad_to(d, kUnitCols) * bits / 8;
}

// column (0..7 inside an 8-column group) -> (word w, half h) of the pair byte
// r: 0->a.lo 4->a.hi 2->b.lo 6->b.hi 1->c.lo 5->c.hi 3->d.lo 7->d.hi
__host__ __device__ inline void col_slot(int r, int& w, int& h) {
  w = ((r & 1) << 1) | ((r >> 1) & 1);
  h = r >> 2;
}

// position (0..31, in halves) of local column lc inside a chunk's permuted
// activation block: pair p = 4*w + j, half h -> 2*p + h.
__host__ __device__ inline int zperm_pos(int lc) {
  int w, h;
  col_slot(lc & 7, w, h);
  return 2 * (4 * w + (lc >> 3)) + h;
}

// Shared-memory order of the rotated activations inside a 256-column unit:
// the 8 halves that one level word w of chunk c pairs with (positions
// 8w..8w+7 of the chunk's permuted pair order) form 16-byte piece w*8 + c, so
// the four lanes t that read word w of chunks t (or 4+t) hit 64 contiguous
// bytes.  tp_rotate mode 3 writes the same order.
__host__ __device__ inline int64_t sk_zpos(int64_t col) {
  const int pos = zperm_pos(static_cast<int>(col & 31));
  return (col & ~int64_t(255)) + (((pos >> 3) * 8 + ((col >> 5) & 7)) << 3) + (pos & 7);
}

// Bit position, inside member word `word` (0-based after the path word), of
// member bit `mb` of local column lc (see the GEMV decoder for the use).
//   bits 2: one word; the 1-bit member of column (8j + r) sits at bit
//           8j + {2,0,3,1,6,4,7,5}[r]... (see member_bit_pos)
//   bits 3/4: word 0 holds even columns, word 1 odd columns, 2-bit fields at
//           byte offsets {2,0,6,4} for columns {8j, 8j+2, 8j+4, 8j+6}
//           (resp. 8j+1, 8j+3, 8j+5, 8j+7); bits 4 adds word 2 with the
//           third member bit (level bit 4), see m2_bit_pos.
__host__ __device__ inline int member_bit_pos(int bits, int lc, int mb, int& word) {
  const int j = lc >> 3, r = lc & 7;
  if (bits == 2) {
    // A = M (cols 8j+0 @2, 8j+4 @6), B = M>>1 (8j+2 @3, 8j+6 @7),
    // C = M<<2 (8j+1 @0, 8j+5 @4), D = M<<1 (8j+3 @1, 8j+7 @5)
    const int pos[8] = {2, 0, 3, 1, 6, 4, 7, 5};
    word = 0;
    return 8 * j + pos[r];
  }
  if (mb < 2) {
    // Mlo/Mhi: A = Mlo (8j @2-3, 8j+4 @6-7), B = Mlo<<2 (8j+2 @0-1, 8j+6 @4-5);
    // C = Mhi, D = Mhi<<2 likewise for odd columns.
    const int fld[8] = {2, 2, 0, 0, 6, 6, 4, 4};
    word = r & 1;
    return 8 * j + fld[r] + mb;
  }
  // third member bit (bits == 4): word 2, see m2_bit_pos
  word = 2;
  return -1;
}

// bits == 4: the third member bit of every column lives in word M2.  The
// decoder builds, for each level word w and byte pair (j = 2q, 2q+1), an
// address word X = rotr(M2, 2*(2w+q)) & 0x01800180 | lane*4*(1 + 2^16);
// bit 7 / 8 of X carry the lo / hi column of byte 2q, bits 23 / 24 those of
// byte 2q+1.  Inverse mapping from (lc) to the M2 bit:
__host__ __device__ inline int m2_bit_pos(int lc) {
  const int j = lc >> 3, r = lc & 7;
  int w, h;
  col_slot(r, w, h);
  const int q = j >> 1, jj = j & 1;
  const int xbit = jj == 0 ? (h == 0 ? 7 : 8) : (h == 0 ? 23 : 24);
  const int s = 2 * (2 * w + q);
  return (xbit + s) & 31;
}

}  // namespace tp

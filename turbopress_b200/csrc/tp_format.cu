// Format kernels: bit packing, window decode, bit-exact row decode and the
// load-time re-layout into the native TCQ stream.  None of these is on the
// per-token path; they run at load time (or in the decode_rows API).
#include "tp_common.cuh"

namespace tp {
thread_local char g_last_error[512] = {0};
}

using namespace tp;

extern "C" int tp_abi_version(void) { return 1; }
extern "C" const char* tp_last_error(void) { return g_last_error; }

namespace {

constexpr int kThreads = 256;

inline unsigned grid_for(int64_t work, int threads = kThreads) {
  int64_t g = (work + threads - 1) / threads;
  if (g < 1) g = 1;
  if (g > (1ll << 30)) g = 1ll << 30;
  return static_cast<unsigned>(g);
}

// -- pack_le / unpack_le (turbopress/runtime.py:73-100) ---------------------
// One thread per output byte: stream bit i = element (i / width), bit (i % width).
__global__ void pack_le_kernel(const uint8_t* __restrict__ vals, uint8_t* __restrict__ out,
                               int64_t n, int64_t d, int width, int64_t row_bytes) {
  const int64_t total = n * row_bytes;
  for (int64_t idx = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; idx < total;
       idx += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = idx / row_bytes, byte = idx % row_bytes;
    unsigned v = 0;
    for (int k = 0; k < 8; ++k) {
      const int64_t bit = byte * 8 + k;
      const int64_t c = bit / width;
      if (c < d) v |= ((vals[r * d + c] >> (bit % width)) & 1u) << k;
    }
    out[idx] = static_cast<uint8_t>(v);
  }
}

__global__ void unpack_le_kernel(const uint8_t* __restrict__ packed, uint8_t* __restrict__ out,
                                 int64_t n, int64_t d, int width, int64_t row_bytes) {
  const int64_t total = n * d;
  for (int64_t idx = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; idx < total;
       idx += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = idx / d, c = idx % d;
    const uint8_t* row = packed + r * row_bytes;
    unsigned v = 0;
    for (int j = 0; j < width; ++j) {
      const int64_t bit = c * width + j;
      v |= ((row[bit >> 3] >> (bit & 7)) & 1u) << j;
    }
    out[idx] = static_cast<uint8_t>(v);
  }
}

// -- v1 flat MSB-first -> v2 row-aligned LE (turbopress/runtime.py:428-447) --
__global__ void v1_to_v2_kernel(const uint8_t* __restrict__ v1, uint8_t* __restrict__ out, int64_t n, int64_t d,
                                int width, int64_t row_bytes) {
  const int64_t total = n * row_bytes;
  for (int64_t idx = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; idx < total;
       idx += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = idx / row_bytes, byte = idx % row_bytes;
    unsigned v = 0;
    for (int k = 0; k < 8; ++k) {
      const int64_t bit = byte * 8 + k;  // row stream bit = c*width + j
      if (bit >= d * width) break;
      const int64_t i = r * d * width + bit;  // flat stream bit
      v |= ((v1[i >> 3] >> (7 - (i & 7))) & 1u) << k;
    }
    out[idx] = static_cast<uint8_t>(v);
  }
}

// -- window decode (turbopress/runtime.py:122-139) --------------------------
__global__ void window_decode_kernel(const uint8_t* __restrict__ path, const uint8_t* __restrict__ member,
                                     uint8_t* __restrict__ levels, int64_t n, int64_t d,
                                     unsigned k0, unsigned k1, int m) {
  const int64_t total = n * d;
  for (int64_t idx = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; idx < total;
       idx += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = idx / d, c = idx % d;
    unsigned win = 0;  // bit k = b_{c-k}, zero before column 0
    for (int k = 0; k <= m; ++k)
      if (c - k >= 0) win |= (unsigned)(path[r * d + c - k] & 1u) << k;
    const unsigned mem = member ? member[idx] : 0u;
    levels[idx] = static_cast<uint8_t>(mem * 4u + subset_of_window(win, k0, k1));
  }
}

// Read up to 64 bits of a byte-aligned LE bit stream row starting at bit
// `bit0` (a multiple of 8), zero beyond `row_bytes`.
__device__ __forceinline__ uint64_t read_bits64(const uint8_t* row, int64_t byte0, int64_t row_bytes) {
  uint64_t v = 0;
#pragma unroll
  for (int k = 0; k < 8; ++k) {
    const int64_t b = byte0 + k;
    if (b >= 0 && b < row_bytes) v |= (uint64_t)row[b] << (8 * k);
  }
  return v;
}

// -- bit-exact decode_rows (turbopress/runtime.py:291-301) -----------------
// One thread per (row, 8-column group): the path byte of the group plus the
// previous byte give every window; member bits of the group span
// (bits-1) bytes.
__global__ void decode_rows_kernel(const uint8_t* __restrict__ path, const uint8_t* __restrict__ member,
                                   const uint16_t* __restrict__ scales, const uint16_t* __restrict__ codebook,
                                   uint16_t* __restrict__ out, int64_t r0, int64_t r1, int64_t d, int bits,
                                   unsigned k0, unsigned k1, int m) {
  const int64_t groups = (d + 7) / 8;
  const int64_t path_rb = (d + 7) / 8;
  const int64_t mem_rb = (d * (bits - 1) + 7) / 8;
  const int64_t total = (r1 - r0) * groups;
  for (int64_t idx = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; idx < total;
       idx += (int64_t)gridDim.x * blockDim.x) {
    const int64_t rr = idx / groups, gcol = idx % groups, r = r0 + rr;
    const uint8_t* prow = path + r * path_rb;
    const unsigned cur = prow[gcol];
    const unsigned prev = gcol > 0 ? prow[gcol - 1] : 0u;
    const unsigned hist = (cur << 8) | prev;  // bit 8+i = column 8*gcol+i
    uint64_t mem = 0;
    if (bits > 1) mem = read_bits64(member + r * mem_rb, gcol * (bits - 1), mem_rb);
    const float sc = h2f_bits(scales[r]);
    for (int i = 0; i < 8; ++i) {
      const int64_t c = gcol * 8 + i;
      if (c >= d) break;
      unsigned win = 0;
      for (int k = 0; k <= m; ++k) win |= ((hist >> (8 + i - k)) & 1u) << k;
      const unsigned mb = bits > 1 ? (unsigned)((mem >> (i * (bits - 1))) & ((1u << (bits - 1)) - 1u)) : 0u;
      const unsigned level = mb * 4u + subset_of_window(win, k0, k1);
      const float v = h2f_bits(codebook[level]) * sc;
      out[rr * d + c] = __half_as_ushort(__float2half_rn(v));
    }
  }
}

// -- rot_scale (turbopress/runtime.py:245-249) -------------------------------
__global__ void rot_scale_kernel(const uint8_t* __restrict__ signs, const uint16_t* __restrict__ inv_equil,
                                 uint16_t* __restrict__ rs, int64_t d) {
  for (int64_t c = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; c < d; c += (int64_t)gridDim.x * blockDim.x) {
    const float s = ((signs[c >> 3] >> (c & 7)) & 1u) ? 1.f : -1.f;
    rs[c] = __half_as_ushort(__float2half_rn(s * h2f_bits(inv_equil[c])));
  }
}

// -- native stream re-layout -------------------------------------------------
// Source accessor: fetch path bit / member value of (r, c) from either a
// format-v2 row-aligned LE stream or a format-v1 flat MSB-first stream.
struct SrcV2 {
  const uint8_t* path;
  const uint8_t* member;
  int64_t d;
  int bits;
  __device__ unsigned path_bit(int64_t r, int64_t c) const {
    return (path[r * ((d + 7) / 8) + (c >> 3)] >> (c & 7)) & 1u;
  }
  __device__ unsigned member_val(int64_t r, int64_t c) const {
    if (bits <= 1) return 0u;
    const int w = bits - 1;
    const uint8_t* row = member + r * ((d * w + 7) / 8);
    unsigned v = 0;
    for (int j = 0; j < w; ++j) {
      const int64_t bit = c * w + j;
      v |= ((row[bit >> 3] >> (bit & 7)) & 1u) << j;
    }
    return v;
  }
};

struct SrcV1 {
  // numpy packbits (MSB-first) of the flat LSB-first value bits
  // (turbopress/pipeline.py:106-117): stream bit i lives in byte i>>3 at
  // bit 7 - (i&7).
  const uint8_t* path;
  const uint8_t* member;
  int64_t d;
  int bits;
  __device__ unsigned path_bit(int64_t r, int64_t c) const {
    const int64_t i = r * d + c;
    return (path[i >> 3] >> (7 - (i & 7))) & 1u;
  }
  __device__ unsigned member_val(int64_t r, int64_t c) const {
    if (bits <= 1) return 0u;
    const int w = bits - 1;
    unsigned v = 0;
    for (int j = 0; j < w; ++j) {
      const int64_t i = (r * d + c) * w + j;
      v |= ((member[i >> 3] >> (7 - (i & 7))) & 1u) << j;
    }
    return v;
  }
};

// One thread per (row, 32-column chunk) of the padded matrix: builds the
// chunk's path word and member words and stores them at their native slots.
template <class Src>
__global__ void relayout_kernel(Src src, uint32_t* __restrict__ out, int64_t n, int64_t n_pad,
                                int64_t d, int64_t d_pad) {
  const int bits = src.bits;
  const int64_t chunks = d_pad / 32;
  const int64_t units_k = d_pad / kUnitCols;
  const int64_t total = n_pad * chunks;
  for (int64_t idx = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; idx < total;
       idx += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = idx / chunks, ch = idx % chunks;
    uint32_t P = 0, M[3] = {0, 0, 0};
    if (r < n) {
      for (int lc = 0; lc < 32; ++lc) {
        const int64_t c = ch * 32 + lc;
        if (c >= d) break;
        P |= src.path_bit(r, c) << lc;
        const unsigned mv = src.member_val(r, c);
        for (int mb = 0; mb < bits - 1; ++mb) {
          if (!((mv >> mb) & 1u)) continue;
          int word;
          int pos = member_bit_pos(bits, lc, mb, word);
          if (word == 2) pos = m2_bit_pos(lc);
          M[word] |= 1u << pos;
        }
      }
    }
    const int64_t rt = r / kTileRows;
    const int rr = static_cast<int>(r % kTileRows);
    const int g = rr & 7, half = rr >> 3;
    const int64_t u = ch / 8;
    const int cc = static_cast<int>(ch % 8);
    const int cg = cc >> 2, t = cc & 3;
    const int lane = g * 4 + t;
    const int comp = cg * 2 + half;
    uint32_t* base = out + ((rt * units_k + u) * 32 + lane) * 4 * bits;
    base[comp] = P;
    for (int w = 0; w < bits - 1; ++w) base[4 * (w + 1) + comp] = M[w];
  }
}

// Bit-exact decode straight from the native stream (inverse of the
// re-layout followed by the reference decode).
__global__ void decode_stream_kernel(const uint32_t* __restrict__ st, const uint16_t* __restrict__ scales,
                                     const uint16_t* __restrict__ codebook, uint16_t* __restrict__ out,
                                     int64_t r0, int64_t r1, int64_t d, int64_t d_pad, int bits,
                                     unsigned k0, unsigned k1, int m) {
  const int64_t chunks = d_pad / 32;
  const int64_t units_k = d_pad / kUnitCols;
  const int64_t total = (r1 - r0) * chunks;
  for (int64_t idx = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; idx < total;
       idx += (int64_t)gridDim.x * blockDim.x) {
    const int64_t rr = idx / chunks, ch = idx % chunks, r = r0 + rr;
    auto word_at = [&](int64_t chunk, int w) -> uint32_t {
      const int64_t rt = r / kTileRows;
      const int q = static_cast<int>(r % kTileRows);
      const int g = q & 7, half = q >> 3;
      const int64_t u = chunk / 8;
      const int cc = static_cast<int>(chunk % 8);
      const int lane = g * 4 + (cc & 3);
      const int comp = (cc >> 2) * 2 + half;
      return st[((rt * units_k + u) * 32 + lane) * 4 * bits + 4 * w + comp];
    };
    const uint32_t P = word_at(ch, 0);
    const uint32_t H = ch > 0 ? word_at(ch - 1, 0) : 0u;
    uint32_t M[3] = {0, 0, 0};
    for (int w = 0; w < bits - 1; ++w) M[w] = word_at(ch, w + 1);
    const uint64_t hist = ((uint64_t)P << 32) | H;
    const float sc = h2f_bits(scales[r]);
    for (int lc = 0; lc < 32; ++lc) {
      const int64_t c = ch * 32 + lc;
      if (c >= d) break;
      unsigned win = 0;
      for (int k = 0; k <= m; ++k) win |= (unsigned)((hist >> (32 + lc - k)) & 1u) << k;
      unsigned mv = 0;
      for (int mb = 0; mb < bits - 1; ++mb) {
        int word;
        int pos = member_bit_pos(bits, lc, mb, word);
        if (word == 2) pos = m2_bit_pos(lc);
        mv |= ((M[word] >> pos) & 1u) << mb;
      }
      const unsigned level = mv * 4u + subset_of_window(win, k0, k1);
      out[rr * d + c] = __half_as_ushort(__float2half_rn(h2f_bits(codebook[level]) * sc));
    }
  }
}

tp_status check_states(int n_states, unsigned& k0, unsigned& k1, int& m) {
  if (log2_states(n_states) < 0) return fail(TP_ERR_UNSUPPORTED, "n_states must be 4, 8, 16 or 64 (got %d)", n_states);
  tap_masks(n_states, k0, k1, m);
  return TP_OK;
}

}  // namespace

extern "C" tp_status tp_pack_le(const uint8_t* vals, uint8_t* out, int64_t n, int64_t d, int width, void* stream) {
  if (!vals || !out || n < 0 || d < 0) return fail(TP_ERR_ARG, "tp_pack_le: bad arguments");
  if (width < 1 || width > 8) return fail(TP_ERR_ARG, "width must be in [1, 8], got %d", width);
  if (n == 0 || d == 0) return clear_ok();
  const int64_t rb = (d * width + 7) / 8;
  pack_le_kernel<<<grid_for(n * rb), kThreads, 0, as_stream(stream)>>>(vals, out, n, d, width, rb);
  return check_launch("tp_pack_le");
}

extern "C" tp_status tp_unpack_le(const uint8_t* packed, uint8_t* out, int64_t n, int64_t d, int width, void* stream) {
  if (!packed || !out || n < 0 || d < 0) return fail(TP_ERR_ARG, "tp_unpack_le: bad arguments");
  if (width < 1 || width > 8) return fail(TP_ERR_ARG, "width must be in [1, 8], got %d", width);
  if (n == 0 || d == 0) return clear_ok();
  const int64_t rb = (d * width + 7) / 8;
  unpack_le_kernel<<<grid_for(n * d), kThreads, 0, as_stream(stream)>>>(packed, out, n, d, width, rb);
  return check_launch("tp_unpack_le");
}

extern "C" tp_status tp_window_decode_levels(const uint8_t* path_bits, const uint8_t* member_codes, uint8_t* levels,
                                             int64_t n, int64_t d, int n_states, void* stream) {
  if (!path_bits || !levels || n < 0 || d < 0) return fail(TP_ERR_ARG, "tp_window_decode_levels: bad arguments");
  unsigned k0, k1;
  int m;
  if (tp_status s = check_states(n_states, k0, k1, m)) return s;
  if (n == 0 || d == 0) return clear_ok();
  window_decode_kernel<<<grid_for(n * d), kThreads, 0, as_stream(stream)>>>(path_bits, member_codes, levels, n, d,
                                                                          k0, k1, m);
  return check_launch("tp_window_decode_levels");
}

extern "C" tp_status tp_decode_rows(const uint8_t* path_packed, const uint8_t* member_packed, const uint16_t* scales,
                                    const uint16_t* codebook, uint16_t* out, int64_t r0, int64_t r1, int64_t d,
                                    int bits, int n_states, void* stream) {
  if (!path_packed || !scales || !codebook || !out || r0 < 0 || r1 < r0 || d < 0)
    return fail(TP_ERR_ARG, "tp_decode_rows: bad arguments");
  if (bits < 1 || bits > 7) return fail(TP_ERR_UNSUPPORTED, "bits must be in [1, 7], got %d", bits);
  if (bits > 1 && !member_packed) return fail(TP_ERR_ARG, "tp_decode_rows: member stream required for bits > 1");
  unsigned k0, k1;
  int m;
  if (tp_status s = check_states(n_states, k0, k1, m)) return s;
  if (r1 == r0 || d == 0) return clear_ok();
  decode_rows_kernel<<<grid_for((r1 - r0) * ((d + 7) / 8)), kThreads, 0, as_stream(stream)>>>(
      path_packed, member_packed, scales, codebook, out, r0, r1, d, bits, k0, k1, m);
  return check_launch("tp_decode_rows");
}

extern "C" tp_status tp_rot_scale(const uint8_t* signs_packed, const uint16_t* inv_equil, uint16_t* rot_scale,
                                  int64_t d, void* stream) {
  if (!signs_packed || !inv_equil || !rot_scale || d < 0) return fail(TP_ERR_ARG, "tp_rot_scale: bad arguments");
  if (d == 0) return clear_ok();
  rot_scale_kernel<<<grid_for(d), kThreads, 0, as_stream(stream)>>>(signs_packed, inv_equil, rot_scale, d);
  return check_launch("tp_rot_scale");
}

extern "C" int64_t tp_stream_bytes(int64_t n, int64_t d, int bits) {
  if (n < 0 || d < 0 || bits < 1 || bits > 4) return -1;
  return stream_bytes(n, d, bits);
}

namespace {
tp_status relayout_checks(const void* path, const void* member, const void* out, int64_t n, int64_t d, int bits) {
  if (!path || !out || n < 0 || d < 0) return fail(TP_ERR_ARG, "relayout: bad arguments");
  if (bits < 1 || bits > 4) return fail(TP_ERR_UNSUPPORTED, "native stream supports bits 1..4, got %d", bits);
  if (bits > 1 && !member) return fail(TP_ERR_ARG, "relayout: member stream required for bits > 1");
  if (!aligned(out, 16)) return fail(TP_ERR_ALIGN, "relayout: output must be 16-byte aligned");
  return TP_OK;
}
}  // namespace

extern "C" tp_status tp_relayout_v2(const uint8_t* path_packed, const uint8_t* member_packed, uint8_t* stream_out,
                                    int64_t n, int64_t d, int bits, void* stream) {
  if (tp_status s = relayout_checks(path_packed, member_packed, stream_out, n, d, bits)) return s;
  if (n == 0 || d == 0) return clear_ok();
  const int64_t n_pad = pad_to(n, kTileRows), d_pad = pad_to(d, kUnitCols);
  SrcV2 src{path_packed, member_packed, d, bits};
  relayout_kernel<<<grid_for(n_pad * (d_pad / 32)), kThreads, 0, as_stream(stream)>>>(
      src, reinterpret_cast<uint32_t*>(stream_out), n, n_pad, d, d_pad);
  return check_launch("tp_relayout_v2");
}

extern "C" tp_status tp_relayout_v1(const uint8_t* path_bits, const uint8_t* member_bits, uint8_t* stream_out,
                                    int64_t n, int64_t d, int bits, void* stream) {
  if (tp_status s = relayout_checks(path_bits, member_bits, stream_out, n, d, bits)) return s;
  if (n == 0 || d == 0) return clear_ok();
  const int64_t n_pad = pad_to(n, kTileRows), d_pad = pad_to(d, kUnitCols);
  SrcV1 src{path_bits, member_bits, d, bits};
  relayout_kernel<<<grid_for(n_pad * (d_pad / 32)), kThreads, 0, as_stream(stream)>>>(
      src, reinterpret_cast<uint32_t*>(stream_out), n, n_pad, d, d_pad);
  return check_launch("tp_relayout_v1");
}

extern "C" tp_status tp_decode_stream(const uint8_t* tcq_stream, const uint16_t* scales, const uint16_t* codebook,
                                      uint16_t* out, int64_t r0, int64_t r1, int64_t n, int64_t d, int bits,
                                      int n_states, void* stream) {
  if (!tcq_stream || !scales || !codebook || !out || r0 < 0 || r1 < r0 || r1 > n || d < 0)
    return fail(TP_ERR_ARG, "tp_decode_stream: bad arguments");
  if (bits < 1 || bits > 4) return fail(TP_ERR_UNSUPPORTED, "native stream supports bits 1..4, got %d", bits);
  if (!aligned(tcq_stream, 16)) return fail(TP_ERR_ALIGN, "tp_decode_stream: stream must be 16-byte aligned");
  unsigned k0, k1;
  int m;
  if (tp_status s = check_states(n_states, k0, k1, m)) return s;
  if (r1 == r0 || d == 0) return clear_ok();
  const int64_t d_pad = pad_to(d, kUnitCols);
  decode_stream_kernel<<<grid_for((r1 - r0) * (d_pad / 32)), kThreads, 0, as_stream(stream)>>>(
      reinterpret_cast<const uint32_t*>(tcq_stream), scales, codebook, out, r0, r1, d, d_pad, bits, k0, k1, m);
  return check_launch("tp_decode_stream");
}

extern "C" tp_status tp_v1_to_v2(const uint8_t* v1, uint8_t* out, int64_t n, int64_t d, int width, void* stream) {
  if (!v1 || !out || n < 0 || d < 0) return fail(TP_ERR_ARG, "tp_v1_to_v2: bad arguments");
  if (width < 1 || width > 8) return fail(TP_ERR_ARG, "width must be in [1, 8], got %d", width);
  if (n == 0 || d == 0) return clear_ok();
  const int64_t rb = (d * width + 7) / 8;
  v1_to_v2_kernel<<<grid_for(n * rb), kThreads, 0, as_stream(stream)>>>(v1, out, n, d, width, rb);
  return check_launch("tp_v1_to_v2");
}

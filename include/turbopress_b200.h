/*
 * turbopress_b200 -- C ABI of the B200 (sm_100a) packed-TCQ decode path.
 *
 * The library replaces the GPU side of TurboPress's packed runtime
 * (turbopress/runtime.py + turbopress/triton_kernel.py in
 * godsonj64/turbopress v0.5.2).  Host code in any language binds these
 * entry points with plain pointers and sizes; nothing here mentions torch.
 *
 * Conventions shared by every entry point:
 *   - All pointers are DEVICE pointers unless stated otherwise.  Buffers are
 *     owned and allocated by the caller; no entry point allocates device
 *     memory, synchronizes the device or the stream, or keeps a pointer
 *     after it returns.  Every launch is enqueued on `stream` (a
 *     cudaStream_t passed as void*, NULL = legacy default stream).
 *   - Half-precision values travel as uint16_t bit patterns (IEEE fp16).
 *   - n = out_features, d = in_features, bits = payload bits per weight,
 *     n_states = trellis states S in {4, 8, 16, 64}.
 *   - A status code is returned; on failure tp_last_error() describes it.
 *     No entry point throws across the ABI.
 *   - Thread safety: every entry point is reentrant; the only global state
 *     is a per-thread error string and one-time per-device kernel attribute
 *     setup.
 */
#ifndef TURBOPRESS_B200_H
#define TURBOPRESS_B200_H

#include <stdint.h>

#if defined(__GNUC__)
#define TP_API __attribute__((visibility("default")))
#else
#define TP_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

typedef int tp_status;
#define TP_OK 0
#define TP_ERR_ARG 1          /* bad argument (null pointer, bad size)          */
#define TP_ERR_UNSUPPORTED 2  /* unsupported bits / n_states / block / batch    */
#define TP_ERR_ALIGN 3        /* pointer or stride alignment requirement broken */
#define TP_ERR_CUDA 4         /* a CUDA launch or runtime call failed           */
#define TP_ERR_WORKSPACE 6    /* workspace missing or smaller than required     */
#define TP_ERR_DEVICE 7       /* a kernel reported a device-side failure        */

/* Activation / output element types. */
#define TP_F16 0
#define TP_F32 1
#define TP_BF16 2

/* Version of this ABI (bumped on any signature change). */
TP_API int tp_abi_version(void);

/* Message describing the last failure on the calling thread ("" if none). */
TP_API const char* tp_last_error(void);

/* ------------------------------------------------------------------------
 * Format-v2 bit streams (little-endian within a byte, rows byte-aligned).
 * ---------------------------------------------------------------------- */

/* out[n, ceil(d*width/8)] = pack of vals[n, d] (uint8 values < 2^width).
 * Replaces turbopress/runtime.py:73-90 (pack_le). */
TP_API tp_status tp_pack_le(const uint8_t* vals, uint8_t* out, int64_t n, int64_t d,
                     int width, void* stream);

/* out[n, d] = unpack of packed[n, ceil(d*width/8)].
 * Replaces turbopress/runtime.py:93-100 (unpack_le). */
TP_API tp_status tp_unpack_le(const uint8_t* packed, uint8_t* out, int64_t n, int64_t d,
                       int width, void* stream);

/* levels[n, d] = member*4 + subset(window of path bits), zero-padded start.
 * path_bits / member_codes are unpacked uint8 [n, d]; member may be NULL.
 * Replaces turbopress/runtime.py:122-139 (window_decode_levels). */
TP_API tp_status tp_window_decode_levels(const uint8_t* path_bits, const uint8_t* member_codes,
                                  uint8_t* levels, int64_t n, int64_t d, int n_states,
                                  void* stream);

/* out[r1-r0, d] (fp16) = fp16(codebook[level] * scale[row]) for rows [r0, r1)
 * of the format-v2 streams, bit-exact with the reference decode.
 * path_packed: [n, ceil(d/8)], member_packed: [n, ceil(d*(bits-1)/8)] or NULL
 * when bits == 1.  bits in [1, 7].
 * Replaces turbopress/runtime.py:291-301 (PackedTCQLinear.decode_rows). */
TP_API tp_status tp_decode_rows(const uint8_t* path_packed, const uint8_t* member_packed,
                         const uint16_t* scales, const uint16_t* codebook, uint16_t* out,
                         int64_t r0, int64_t r1, int64_t d, int bits, int n_states,
                         void* stream);

/* rot_scale[d] (fp16) = fp16((2*sign - 1) * inv_equil), signs_packed [1, ceil(d/8)].
 * Replaces turbopress/runtime.py:245-249. */
TP_API tp_status tp_rot_scale(const uint8_t* signs_packed, const uint16_t* inv_equil,
                       uint16_t* rot_scale, int64_t d, void* stream);

/* Format-v1 flat stream (numpy packbits, MSB-first, of LSB-first `width`-bit
 * values over the whole [n, d] matrix, turbopress/pipeline.py:106-117) ->
 * format-v2 row-aligned LE stream out[n, ceil(d*width/8)].
 * Replaces the numpy unpack + pack_le of turbopress/runtime.py:428-447. */
TP_API tp_status tp_v1_to_v2(const uint8_t* v1, uint8_t* out, int64_t n, int64_t d, int width,
                      void* stream);

/* ------------------------------------------------------------------------
 * Seeded randomized Hadamard rotation of activations.
 * ---------------------------------------------------------------------- */

/* z[B, d] = blockFWHT(x[B, d] * rot_scale[d]) over blocks of `block` columns
 * (orthonormal Sylvester order), computed in fp32.  x_dtype / z_dtype are
 * TP_F16, TP_F32 or TP_BF16; rows are contiguous (row stride d).
 * block must be a power of two dividing d, 1 <= block <= 32768.
 * Replaces turbopress/triton_kernel.py:235-260 (fwht_scale) and the torch
 * path turbopress/runtime.py:192-208 + :322-323. */
TP_API tp_status tp_rotate(const void* x, int x_dtype, const uint16_t* rot_scale, void* z,
                    int z_dtype, int64_t B, int64_t d, int64_t block, void* stream);

/* Load-time fold used by the "cached" mode (turbopress/runtime.py:278-286):
 * w_out[n, d] (fp16) = fp16(blockFWHT(w_rot[n, d]) * post_scale[d]), with
 * w_rot fp16 and post_scale = (2*sign-1) * inv_equil (the rot_scale vector). */
TP_API tp_status tp_fold_rows(const uint16_t* w_rot, const uint16_t* post_scale, uint16_t* w_out,
                       int64_t n, int64_t d, int64_t block, void* stream);

/* ------------------------------------------------------------------------
 * Native true-rate tile layout ("TCQ stream") and the fused GEMV.
 *
 * The stream keeps exactly `bits` bits per weight (plus padding of n to a
 * multiple of 16 rows and d to a multiple of 256 columns), re-arranged so a
 * warp reads 16-row x 256-column tiles with coalesced 16-byte loads and
 * decodes them with register bit-slicing.  It is derived data: built on the
 * device from the format-v2 (or v1) streams at load time.
 * ---------------------------------------------------------------------- */

/* Bytes of the native stream for an [n, d] matrix at `bits` (1..4). */
TP_API int64_t tp_stream_bytes(int64_t n, int64_t d, int bits);

/* Build the native stream from format-v2 streams (layout of tp_decode_rows).
 * stream_out must hold tp_stream_bytes(n, d, bits) bytes, 16-byte aligned.
 * Replaces the load-time re-pack of turbopress/runtime.py:253-277. */
TP_API tp_status tp_relayout_v2(const uint8_t* path_packed, const uint8_t* member_packed,
                         uint8_t* stream_out, int64_t n, int64_t d, int bits,
                         void* stream);

/* Build the native stream straight from a format-v1 artifact matrix
 * (flat MSB-first numpy packbits streams, turbopress/pipeline.py:106-117,
 * :445-455).  path_bits: ceil(n*d/8) bytes; member_bits: ceil(n*d*(bits-1)/8)
 * bytes or NULL when bits == 1.
 * Replaces turbopress/runtime.py:417-452 (v1_payload_to_packed) + :253-277. */
TP_API tp_status tp_relayout_v1(const uint8_t* path_bits, const uint8_t* member_bits,
                         uint8_t* stream_out, int64_t n, int64_t d, int bits,
                         void* stream);

/* Bit-exact fp16 decode of rows [r0, r1) from the native stream (same values
 * as tp_decode_rows on the source streams). */
TP_API tp_status tp_decode_stream(const uint8_t* tcq_stream, const uint16_t* scales,
                           const uint16_t* codebook, uint16_t* out, int64_t r0, int64_t r1,
                           int64_t n, int64_t d, int bits, int n_states, void* stream);

/* Device workspace (bytes) that tp_tcq_gemv needs for a given problem.
 * The workspace must be zero-filled once when allocated; every call leaves
 * its counters at zero again, so the same buffer serves any later call of
 * equal or smaller size.  Calls that share a workspace must not overlap on
 * the GPU (use one workspace per stream). */
TP_API int64_t tp_gemv_workspace_bytes(int64_t B, int64_t n, int64_t d, int bits);

/* y[B, n] = blockFWHT(x[B, d] * rot_scale) @ W'^T (+ bias), W' the dequantized
 * rotated weights held in the native stream: the fused decode-in-GEMV.
 * x_dtype / y_dtype in {TP_F16, TP_F32, TP_BF16}; bias fp16 [n] or NULL.
 * bits in 1..4, n_states in {4, 8, 16, 64}, 1 <= B (batches above 32 run in
 * chunks of 32).  Accumulates in fp32.  Deterministic (fixed reduction order).
 * Replaces turbopress/triton_kernel.py:132-157 (packed_gemv) together with
 * fwht_scale, i.e. PackedTCQLinear.forward in mode "triton"
 * (turbopress/runtime.py:312-316, :332-334). */
TP_API tp_status tp_tcq_gemv(const void* x, int x_dtype, const uint16_t* rot_scale,
                      const uint8_t* tcq_stream, const uint16_t* scales,
                      const uint16_t* codebook, const uint16_t* bias, void* y, int y_dtype,
                      int64_t B, int64_t n, int64_t d, int64_t block, int bits, int n_states,
                      void* workspace, int64_t workspace_bytes, void* stream);

/* Allocation-free form of tp_tcq_gemv, for callers that cannot allocate
 * device memory (e.g. plugins whose host engine owns all allocations, or
 * loops where a cudaMalloc is not allowed).  No counterpart in the
 * reference.  Same arguments and result as tp_tcq_gemv without the
 * workspace: the scratch lives in an 8 MiB array inside this library,
 * held on every GPU that loads it until the process exits.  Problems whose
 * tp_gemv_workspace_bytes() exceed 8 MiB are rejected with
 * TP_ERR_UNSUPPORTED.  The first call on a device looks up the array's
 * device address and clears its counters; make that first call before any
 * stream capture.  All calls share the one array: calls that overlap on
 * the GPU (concurrent streams) race and must be serialized by the caller. */
TP_API tp_status tp_tcq_gemv_noalloc(const void* x, int x_dtype, const uint16_t* rot_scale,
                                     const uint8_t* tcq_stream, const uint16_t* scales,
                                     const uint16_t* codebook, const uint16_t* bias, void* y,
                                     int y_dtype, int64_t B, int64_t n, int64_t d, int64_t block,
                                     int bits, int n_states, void* stream);

/* Reads (synchronizing `stream`) the status word that tp_tcq_gemv kernels
 * leave in `workspace`: TP_OK, or TP_ERR_DEVICE when a kernel gave up (a
 * bounded wait ran out: the outputs of that call are NaN; or the
 * shared-memory layout check failed: they were not written).  Every
 * completed call leaves the workspace's counter block zero; a call that gave
 * up may not, so on TP_ERR_DEVICE the whole counter block (split-K counters
 * and status) is cleared and the workspace is fit for the next call.  The
 * reference has no device-side failure to report (its Triton kernel has no
 * waits).  tp_gemv_noalloc_status does the same for the built-in scratch of
 * tp_tcq_gemv_noalloc on the current device. */
TP_API tp_status tp_gemv_status(const void* workspace, void* stream);
TP_API tp_status tp_gemv_noalloc_status(void* stream);

/* Skinny GEMM on the 5th-generation tensor cores (tcgen05, TMEM accumulator)
 * for batches of 16 and more: same arguments and result as tp_tcq_gemv.
 * The weights are decoded into shared memory (fp16, UMMA operand layout) and
 * multiplied with tcgen05.mma against the rotated activations; batches are
 * processed 64 rows per pass.  Needs tp_gemm_tc_workspace_bytes(B, n, d)
 * bytes of workspace (256-byte aligned; no zero-fill needed). */
TP_API int64_t tp_gemm_tc_workspace_bytes(int64_t B, int64_t n, int64_t d);
TP_API tp_status tp_tcq_gemm_tc(const void* x, int x_dtype, const uint16_t* rot_scale, const uint8_t* tcq_stream,
                                const uint16_t* scales, const uint16_t* codebook, const uint16_t* bias, void* y,
                                int y_dtype, int64_t B, int64_t n, int64_t d, int64_t block, int bits,
                                int n_states, void* workspace, int64_t workspace_bytes, void* stream);

/* Greedy LM head: idx[b] = argmax_v (x[b] . w[v]) over a fp16 weight matrix
 * w [V][h] (row-major, 16-byte aligned, h a multiple of 8) and fp16 input
 * x [B][h] (16-byte aligned), 1 <= B <= 8, B*h <= 25600; fp32 accumulation;
 * the first index wins among equal logits (NaN counts as largest).  val[b]
 * (NULL to skip) receives the winning logit; logits (fp32 [B][V], NULL to
 * skip) all of them.  One HBM-bound pass over w; the logits are not needed
 * in memory.  Needs tp_lm_head_workspace_bytes(B) bytes of workspace,
 * zero-filled once (every call leaves it zeroed; one workspace per stream).
 * Replaces the tied fp16 lm_head F.linear + logits[:, -1:].argmax(-1) of
 * the reference's decode loops (scripts/run_packed.py:164,178,190;
 * scripts/graph_decode_bench.py:55-112). */
TP_API int64_t tp_lm_head_workspace_bytes(int64_t B);
TP_API tp_status tp_lm_head_argmax(const uint16_t* x, const uint16_t* w, int64_t B, int64_t V, int64_t h,
                                   float* logits, int64_t* idx, float* val, void* workspace,
                                   int64_t workspace_bytes, void* stream);

/* ------------------------------------------------------------------------
 * Persistent decode engine: a chain of packed linears in ONE launch.
 *
 * Every SM keeps one CTA resident for the whole program, builds the pair
 * table once, and streams each warp's weight units through a bulk-copy ring
 * that runs ahead across op boundaries, so later layers' weights load while
 * earlier ones wait for their activations.  An op waits (bounded) until
 * every CTA has finished the op that produces its input; partial outputs
 * are scaled and accumulated with fp32 atomics (order not fixed, so results
 * may differ from tp_tcq_gemv in the last bits).  All ops share one bit
 * width, state count and codebook; batch <= 4; Hadamard blocks 1..8192.
 * Replaces a sequence of PackedTCQLinear.forward calls in mode "triton"
 * (turbopress/runtime.py:312-334) chained by their activations.
 * ---------------------------------------------------------------------- */
typedef struct tp_engine_op {
  const uint8_t* tcq_stream;  /* native stream of the layer                      */
  const uint16_t* scales;     /* fp16 [n]                                         */
  const uint16_t* bias;       /* fp16 [n] or NULL                                 */
  const uint16_t* rot_scale;  /* fp16 [d]                                         */
  const void* x;              /* input activations [B][d] (x_dtype)               */
  float* y;                   /* fp32 output [B][n]; must be zero before each run */
  int64_t n, d;
  int32_t block;              /* Hadamard block of the layer                      */
  int32_t x_dtype;            /* TP_F16 / TP_BF16 / TP_F32                        */
  int32_t dep;                /* index of the op whose y is this op's x, or -1    */
  int32_t reserved;
} tp_engine_op;

/* Bytes of the program image for n_ops ops. */
TP_API int64_t tp_engine_image_bytes(int n_ops);

/* Build the program image in HOST memory (no device work): validates the
 * ops and derives the launch layout for the current device.  The caller
 * copies the image to a device buffer of the same size (16-byte aligned)
 * and passes both copies to tp_engine_run.  codebook: fp16 device pointer
 * shared by every op. */
TP_API tp_status tp_engine_build(const tp_engine_op* ops, int n_ops, int B, int bits, int n_states,
                                 const uint16_t* codebook, void* image, int64_t image_bytes);

/* Bytes of the counter block (2 * n_ops + 2 words).  On one GPU zero it
 * before each run; after a run, word n_ops is non-zero if a wait timed out. */
TP_API int64_t tp_engine_counter_bytes(int n_ops);

/* Tensor-parallel program over n_ranks GPUs of one node (one process per
 * GPU).  Each rank runs a shard of every op (a 16-row-aligned range of its
 * output rows: ops[i].n rows starting at row0[i] of n_full[i]) and adds its
 * partial outputs into EVERY rank's copy of the output with fp32 atomics over
 * NVLink peer mappings, then counts completion on every rank; a stage waits
 * until every CTA of every rank has published its input.  This is the
 * all-gather / all-reduce of the layer outputs fused into the GEMV epilogue
 * (no separate collective).  Outputs live in a double-buffered arena that
 * every rank maps: ops[i].y and a dependent ops[i].x are BYTE OFFSETS into
 * one arena buffer; run r writes buffer r % 2 and clears the other.  The
 * counter block must be peer-mapped too, zeroed once before the first run and
 * never again (counts are cumulative).  Before the first run every rank must
 * have zeroed both arena buffers (then synchronise the ranks). */
typedef struct tp_engine_tp {
  int32_t n_ranks, rank;
  void* arena[2];                  /* this rank's two arena buffers (16-byte aligned)       */
  int64_t arena_bytes;             /* bytes of one buffer (multiple of 16)                   */
  const uint64_t* peer_arena;      /* device array [n_ranks][2]: every rank's buffers here   */
  unsigned* const* peer_counters;  /* device array [n_ranks]: every rank's counter block     */
} tp_engine_tp;

TP_API tp_status tp_engine_build_tp(const tp_engine_op* ops, const int64_t* row0, const int64_t* n_full,
                                    int n_ops, int B, int bits, int n_states, const uint16_t* codebook,
                                    const tp_engine_tp* tp, void* image, int64_t image_bytes);

/* Peer memory for tensor-parallel programs (CUDA IPC within one node).
 * tp_ipc_alloc: zero-filled device allocation whose IPC handle covers
 * exactly it (the fill completes before the call returns);
 * tp_ipc_get_handle writes TP_IPC_HANDLE_BYTES bytes; tp_ipc_open maps a
 * peer's allocation into this process (the current device). */
#define TP_IPC_HANDLE_BYTES 64
TP_API tp_status tp_ipc_alloc(int64_t bytes, void** ptr);
TP_API tp_status tp_ipc_free(void* ptr);
TP_API tp_status tp_ipc_get_handle(void* ptr, void* handle);
TP_API tp_status tp_ipc_open(const void* handle, void** ptr);
TP_API tp_status tp_ipc_close(void* ptr);

/* Run the program on `stream` (image_dev: device copy; image_host: the
 * host image it was copied from). */
TP_API tp_status tp_engine_run(const void* image_dev, const void* image_host, unsigned* counters,
                               void* stream);

/* ------------------------------------------------------------------------
 * Decoder step: one cooperative launch runs a whole batch-B decode step of
 * a Qwen3 / Llama-style decoder whose seven linears per layer are packed TCQ
 * (bits 2..4, 64 states): per layer RMSNorm -> q/k/v -> (Qwen3 q/k head
 * norms) -> RoPE -> KV-cache append -> GQA attention over positions
 * [0, pos] -> o_proj + residual -> RMSNorm -> gate/up -> SiLU(gate)*up ->
 * down_proj + residual, and the final RMSNorm.  fp16 activations, rounded
 * where the reference model's fp16 forward rounds them (the LM head follows
 * as tp_lm_head_argmax on final_out).  Replaces the decoder forward that the
 * reference runs with PackedTCQLinear layers inside a Hugging Face model
 * (turbopress/runtime.py:455-541 load_packed_model, stepped by
 * scripts/run_packed.py:160-190 and scripts/graph_decode_bench.py:70-118).
 * ---------------------------------------------------------------------- */
typedef struct tp_step_linear {
  const uint8_t* tcq_stream;  /* native stream (tp_relayout_v2 / _v1), 16-byte aligned */
  const uint16_t* scales;     /* fp16 [n]                                             */
  const uint16_t* codebook;   /* fp16 [2^(bits+1)]                                    */
  const uint16_t* rot_scale;  /* fp16 [d], 16-byte aligned                            */
  const uint16_t* bias;       /* fp16 [n] or NULL                                     */
  int64_t n, d, block;        /* block: Hadamard block, 256..8192                     */
  int32_t bits, n_states;
} tp_step_linear;

typedef struct tp_step_layer {
  tp_step_linear q, k, v, o, gate, up, down;
  const uint16_t* ln1;      /* input_layernorm weight, fp16 [hidden]                 */
  const uint16_t* ln2;      /* post_attention_layernorm weight                       */
  const uint16_t* q_norm;   /* fp16 [head_dim] (Qwen3) or NULL                       */
  const uint16_t* k_norm;
  uint16_t* k_cache;        /* fp16 [B][kv_heads][max_tokens][head_dim], post-RoPE   */
  uint16_t* v_cache;
} tp_step_layer;

typedef struct tp_step_model {
  int32_t B, layers, hidden, inter, q_heads, kv_heads, head_dim, max_tokens;
  float rms_eps;
  const float* inv_freq;        /* fp32 [head_dim/2] RoPE inverse frequencies        */
  const uint16_t* final_norm;   /* fp16 [hidden]                                     */
  uint16_t* hidden_state;       /* fp16 [B][hidden]: input embeddings in, residual   */
  uint16_t* final_out;          /* fp16 [B][hidden]: final RMSNorm output            */
  void* act;                    /* tp_step_act_bytes() bytes of activation scratch   */
  /* Optional RoPE tables, fp16 [max_tokens][head_dim/2]: cos / sin of the
   * fp32 angle pos * inv_freq[i], rounded to fp16 (what the reference model's
   * rotary embedding feeds its fp16 forward).  NULL: the kernel evaluates
   * them from inv_freq (slower). */
  const uint16_t* rope_cos;
  const uint16_t* rope_sin;
} tp_step_model;

/* Bytes of the step program image for `layers` layers / of the activation
 * scratch the model needs. */
TP_API int64_t tp_step_image_bytes(int layers);
TP_API int64_t tp_step_act_bytes(const tp_step_model* m);

/* Build the program image in HOST memory for the current device (no device
 * work); *workspace_bytes receives the workspace size tp_step_run needs (zero
 * it once; each run leaves its counters at zero).  Copy the image to a
 * 16-byte aligned device buffer of the same size. */
TP_API tp_status tp_step_build(const tp_step_model* m, const tp_step_layer* layers, void* image_host,
                               int64_t image_bytes, int64_t* workspace_bytes);

/* Resolves the workspace buffers a built image refers to (fp32 projection
 * accumulators, the second residual buffer) against `workspace` (256-byte
 * aligned, *workspace_bytes from tp_step_build, zero-filled once).  Call once
 * per image, before copying it to the device; tp_step_run refuses an image
 * bound to another workspace. */
TP_API tp_status tp_step_bind(void* image_host, void* workspace, int64_t workspace_bytes);

/* One decode step at position *pos_dev (device int: the number of tokens
 * already in the caches; the step writes k/v at that position).  Enqueued on
 * `stream` (graph-capturable: a 2 KB memset of the barrier block and one cooperative launch). */
TP_API tp_status tp_step_run(const void* image_dev, const void* image_host, const int* pos_dev,
                             void* workspace, int64_t workspace_bytes, void* stream);

/* Reads (synchronizing `stream`) and clears the device status word of a
 * step workspace: TP_OK, or TP_ERR_DEVICE when a grid barrier timed out or
 * the shared-memory layout check failed.  After a failed step it also clears
 * the accumulators and attention counters the step left part-written, so the
 * next step starts clean (its outputs are not valid). */
TP_API tp_status tp_step_status(const void* workspace, void* stream);

/* Sets the grid-barrier limit of a built program (`image_host`, in
 * microseconds; 0 = the default of 2 s) and the number of arrivals each
 * barrier waits for beyond the grid's own (0 for every real run).  With
 * extra_arrivals > 0 no barrier can complete: every CTA gives up after the
 * limit, the step returns with incomplete outputs, and tp_step_status
 * reports TP_ERR_DEVICE; the CUDA context stays usable.  This is how the
 * timeout path is tested.  Copy the host image to the device again after
 * the call. */
TP_API tp_status tp_step_set_wait(void* image_host, int64_t barrier_us, int extra_arrivals);

/* Reference-order GEMV straight from the format-v2 streams, any bits in 1..7:
 * y[B, n] = z[B, d] @ decode_rows^T (+ bias), z fp32 rotated activations.
 * Used for payloads the native stream does not cover (bits 5..7) and as an
 * independent GPU cross-check.  Replaces the "tiled" forward loop of
 * turbopress/runtime.py:324-331. */
TP_API tp_status tp_gemv_v2(const float* z, const uint8_t* path_packed, const uint8_t* member_packed,
                     const uint16_t* scales, const uint16_t* codebook, const uint16_t* bias,
                     void* y, int y_dtype, int64_t B, int64_t n, int64_t d, int bits,
                     int n_states, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* TURBOPRESS_B200_H */

"""CPU oracle for the packed-TCQ decode path -- TEST INFRASTRUCTURE ONLY.

This module restates, in numpy, the reference TurboPress (godsonj64/turbopress
v0.5.2) arithmetic for the packed decode path.  It is the checker that the
CUDA kernels in ``turbopress_b200`` are compared against; nothing in the
product imports it.  Only ``tests/``, ``__graft_entry__.smoke()`` and the
``cpu_baseline`` / ``--impl reference`` legs of ``bench.py`` may use it.

Each function cites the reference file:line it follows.  Parity of this
restatement is pinned by golden vectors produced by the reference itself
(``tests/golden/make_golden.py`` imports the reference and records its
outputs; ``tests/test_oracle_golden.py`` checks this module against them).

Conventions (all from the reference):
  * n = out_features, d = in_features, bits = payload bits, S = n_states,
    m = log2(S).
  * Format v2 streams are little-endian within a byte, each row padded to a
    whole byte (turbopress/runtime.py:73-100).
  * Format v1 streams are flat over the whole matrix, numpy ``packbits``
    (MSB-first within a byte) of LSB-first value bits
    (turbopress/pipeline.py:106-117).
"""

from __future__ import annotations

import math

import numpy as np

# Rate-1/2 convolutional generators (octal) per state count.
# turbopress/trellis.py:47-52 (identical table: pipeline.py:183).
GENERATORS: dict[int, tuple[int, int]] = {
    4: (0o5, 0o7),
    8: (0o15, 0o17),
    16: (0o23, 0o35),
    64: (0o133, 0o171),
}


def _log2_states(n_states: int) -> int:
    if n_states not in GENERATORS:
        raise ValueError(f"n_states must be one of {sorted(GENERATORS)}, got {n_states}")
    return n_states.bit_length() - 1


# ---------------------------------------------------------------------------
# bit packing
# ---------------------------------------------------------------------------
def pack_le(vals: np.ndarray, width: int) -> np.ndarray:
    """Format-v2 packing (turbopress/runtime.py:73-90).

    [n, d] uint8 values < 2**width -> [n, ceil(d*width/8)] uint8; bit j of
    element c is stream bit c*width + j, stream bit i is byte i>>3, bit i&7.
    """
    vals = np.asarray(vals)
    if vals.ndim != 2 or vals.dtype != np.uint8:
        raise ValueError("expected a 2D uint8 array")
    if not 1 <= width <= 8:
        raise ValueError(f"width must be in [1, 8], got {width}")
    n, d = vals.shape
    bits = (vals[:, :, None] >> np.arange(width, dtype=np.uint8)) & 1
    stream = bits.reshape(n, d * width)
    return np.packbits(stream, axis=1, bitorder="little")


def unpack_le(packed: np.ndarray, d: int, width: int) -> np.ndarray:
    """Inverse of :func:`pack_le` (turbopress/runtime.py:93-100) -> [n, d] uint8."""
    packed = np.asarray(packed, dtype=np.uint8)
    n = packed.shape[0]
    stream = np.unpackbits(packed, axis=1, bitorder="little")[:, : d * width]
    weights = (1 << np.arange(width)).astype(np.int32)
    return (stream.reshape(n, d, width).astype(np.int32) * weights).sum(-1).astype(np.uint8)


def pack_bits_v1(codes: np.ndarray, width: int) -> np.ndarray:
    """Format-v1 flat packing (turbopress/pipeline.py:106-110)."""
    flat = np.asarray(codes, dtype=np.uint8).reshape(-1)
    bits = (flat[:, None] >> np.arange(width, dtype=np.uint8)) & 1
    return np.packbits(bits.reshape(-1))


def unpack_bits_v1(buf: np.ndarray, count: int, width: int) -> np.ndarray:
    """Format-v1 flat unpacking (turbopress/pipeline.py:113-117)."""
    bits = np.unpackbits(np.asarray(buf, dtype=np.uint8))[: count * width].reshape(count, width)
    return (bits << np.arange(width, dtype=np.uint8)).sum(axis=1).astype(np.uint8)


# ---------------------------------------------------------------------------
# trellis
# ---------------------------------------------------------------------------
def subset_table(n_states: int) -> np.ndarray:
    """[S, 2] subset label per (state, input bit) (turbopress/trellis.py:62-79).

    subset = parity(x & g1) << 1 | parity(x & g0) with x = (b << m) | s.
    """
    m = _log2_states(n_states)
    g0, g1 = GENERATORS[n_states]
    out = np.empty((n_states, 2), dtype=np.int64)
    for s in range(n_states):
        for b in (0, 1):
            x = (b << m) | s
            out[s, b] = ((bin(x & g1).count("1") & 1) << 1) | (bin(x & g0).count("1") & 1)
    return out


def subset_lut(n_states: int) -> np.ndarray:
    """Window-integer -> subset LUT (turbopress/runtime.py:106-119).

    Window x has b_{t-m+j} at bit j; the current bit is bit m, the state is
    the bit-reverse of the low m bits.
    """
    m = _log2_states(n_states)
    xs = np.arange(1 << (m + 1))
    b_cur = (xs >> m) & 1
    state = np.zeros_like(xs)
    for k in range(m):
        state |= ((xs >> (m - 1 - k)) & 1) << k
    return subset_table(n_states)[state, b_cur].astype(np.uint8)


def window_decode_levels(path_bits: np.ndarray, member_codes: np.ndarray, n_states: int) -> np.ndarray:
    """Walk-free level decode (turbopress/runtime.py:122-139).

    level[r, t] = member[r, t] * 4 + LUT[window(r, t)], window zero-padded on
    the left by m bits (the encoder starts in state 0).
    """
    path_bits = np.asarray(path_bits)
    n, d = path_bits.shape
    m = _log2_states(n_states)
    lut = subset_lut(n_states)
    padded = np.pad(path_bits.astype(np.int32), ((0, 0), (m, 0)))
    x = padded[:, m:] << m
    for j in range(m):
        x = x | (padded[:, j : j + d] << j)
    subsets = lut[x]
    return (np.asarray(member_codes).astype(np.int32) * 4 + subsets).astype(np.uint8)


def sequential_decode_levels(path_bits: np.ndarray, member_codes: np.ndarray, n_states: int) -> np.ndarray:
    """Sequential trellis walk from state 0 (turbopress/trellis.py:182-199)."""
    path_bits = np.asarray(path_bits)
    n, d = path_bits.shape
    table = subset_table(n_states)
    mask = n_states - 1
    out = np.empty((n, d), dtype=np.uint8)
    state = np.zeros(n, dtype=np.int64)
    for t in range(d):
        b = path_bits[:, t].astype(np.int64)
        out[:, t] = (np.asarray(member_codes)[:, t].astype(np.int64) * 4 + table[state, b]).astype(np.uint8)
        state = ((state << 1) | b) & mask
    return out


# ---------------------------------------------------------------------------
# payload helpers (format v2 dicts with numpy arrays)
# ---------------------------------------------------------------------------
def levels_from_payload(p: dict, r0: int = 0, r1: int | None = None) -> np.ndarray:
    """Unpack + window-decode rows [r0, r1) (turbopress/runtime.py:291-299)."""
    d, bits = int(p["d"]), int(p["bits"])
    r1 = int(p["n"]) if r1 is None else r1
    pathb = unpack_le(np.asarray(p["path_packed"])[r0:r1], d, 1)
    if p.get("member_packed") is not None:
        memb = unpack_le(np.asarray(p["member_packed"])[r0:r1], d, bits - 1)
    else:
        memb = np.zeros_like(pathb)
    return window_decode_levels(pathb, memb, int(p["n_states"]))


def decode_rows(p: dict, r0: int = 0, r1: int | None = None) -> np.ndarray:
    """Bit-exact dequant of rows [r0, r1) (turbopress/runtime.py:291-301).

    W'[r, c] = fp16(float32(codebook[level]) * float32(scale[r])).
    """
    r1 = int(p["n"]) if r1 is None else r1
    levels = levels_from_payload(p, r0, r1)
    cb = np.asarray(p["codebook"], dtype=np.float16).astype(np.float32)
    sc = np.asarray(p["scales"], dtype=np.float16).astype(np.float32)[r0:r1]
    return (cb[levels] * sc[:, None]).astype(np.float16)


def rot_scale(p: dict) -> np.ndarray:
    """Per-channel activation scale (turbopress/runtime.py:245-249).

    rot_scale = fp16((2 * sign - 1) * float32(inv_equil)).
    """
    d = int(p["d"])
    signs = unpack_le(np.asarray(p["signs_packed"]), d, 1)[0].astype(np.float32)
    ie = np.asarray(p["inv_equil"], dtype=np.float16).astype(np.float32)
    return ((signs * 2 - 1) * ie).astype(np.float16)


def fwht(x: np.ndarray) -> np.ndarray:
    """Orthonormal Sylvester-order FWHT on the last axis, in the input dtype.

    Same butterfly order as turbopress/runtime.py:192-201 (and hadamard.py:37-56):
    stages h = 1, 2, 4, ... then one division by sqrt(d).
    """
    x = np.asarray(x)
    d = x.shape[-1]
    if d & (d - 1):
        raise ValueError(f"fwht requires a power-of-2 last dimension, got {d}")
    y = x.reshape(-1, d)
    h = 1
    while h < d:
        y = y.reshape(-1, d // (2 * h), 2, h)
        even, odd = y[:, :, 0, :], y[:, :, 1, :]
        y = np.stack((even + odd, even - odd), axis=2).reshape(-1, d)
        h *= 2
    return (y / x.dtype.type(math.sqrt(d))).reshape(x.shape)


def block_fwht(x: np.ndarray, block: int) -> np.ndarray:
    """Block-diagonal FWHT (turbopress/runtime.py:204-208)."""
    x = np.asarray(x)
    if block == x.shape[-1]:
        return fwht(x)
    m = x.shape[-1] // block
    return fwht(x.reshape(*x.shape[:-1], m, block)).reshape(x.shape)


def rotate_activations(x: np.ndarray, rs: np.ndarray, block: int) -> np.ndarray:
    """z = blockFWHT(x * rot_scale) in fp32 (turbopress/runtime.py:322-323)."""
    return block_fwht(np.asarray(x, dtype=np.float32) * np.asarray(rs).astype(np.float32), block)


def forward_fp32(p: dict, x: np.ndarray) -> np.ndarray:
    """Reference fp32 dequant-then-matmul of the packed layer.

    z = blockFWHT(x * rot_scale) (turbopress/runtime.py:322-323);
    y = z @ W'^T + bias with W' the fp16 ``decode_rows`` matrix
    (turbopress/runtime.py:324-333), everything else in fp32.  Returns fp32
    [..., n].
    """
    d, n = int(p["d"]), int(p["n"])
    x = np.asarray(x)
    flat = x.reshape(-1, d).astype(np.float32)
    z = rotate_activations(flat, rot_scale(p), int(p["block"]))
    w = decode_rows(p).astype(np.float32)      # fp16-rounded dequant, as decode_rows returns
    y = z @ w.T
    if p.get("bias") is not None:
        y = y + np.asarray(p["bias"], dtype=np.float16).astype(np.float32)
    return y.reshape(*x.shape[:-1], n)


def fold_original_basis(p: dict) -> np.ndarray:
    """Cached-mode weights in the original basis, fp32 before the fp16 cast.

    W = blockFWHT(W'_fp32) * signs * inv_equil (turbopress/runtime.py:278-286).
    """
    d = int(p["d"])
    w_rot = decode_rows(p).astype(np.float32)
    signs = unpack_le(np.asarray(p["signs_packed"]), d, 1)[0].astype(np.float32) * 2 - 1
    w = block_fwht(w_rot, int(p["block"])) * signs[None, :]
    return w * np.asarray(p["inv_equil"], dtype=np.float16).astype(np.float32)[None, :]


def v1_to_v2(payload: dict, bias: np.ndarray | None = None) -> dict:
    """Format-v1 artifact matrix -> format-v2 payload (turbopress/runtime.py:417-452)."""
    n, d, bits = int(payload["n"]), int(payload["d"]), int(payload["bits"])
    path = unpack_bits_v1(payload["path_bits"], n * d, 1).reshape(n, d)
    member = (unpack_bits_v1(payload["member_bits"], n * d, bits - 1).reshape(n, d)
              if bits > 1 else None)
    signs = unpack_bits_v1(payload["signs"], d, 1).reshape(1, d)
    equil = np.maximum(np.asarray(payload["equil"], dtype=np.float16).astype(np.float32), 1e-12)
    return {
        "format": 2, "n": n, "d": d, "bits": bits,
        "n_states": int(payload["n_states"]), "block": int(payload["block"]),
        "path_packed": pack_le(path, 1),
        "member_packed": pack_le(member, bits - 1) if member is not None else None,
        "scales": np.asarray(payload["scales"], dtype=np.float16),
        "signs_packed": pack_le(signs, 1),
        "inv_equil": (np.float32(1.0) / equil).astype(np.float16),
        "codebook": np.asarray(payload["codebook"], dtype=np.float16),
        "bias": None if bias is None else np.asarray(bias).astype(np.float16),
        "seed": 0,
    }


# ---------------------------------------------------------------------------
# synthetic payloads (every path/member bit string is a valid TCQ codeword,
# so uniformly random streams exercise the decoder exactly like encoder output)
# ---------------------------------------------------------------------------
def random_payload(n: int, d: int, bits: int, n_states: int = 64, seed: int = 0,
                   codebook: np.ndarray | None = None, bias: bool = False) -> dict:
    """Seeded random format-v2 payload of the given shape (test input generator)."""
    rng = np.random.default_rng(seed)
    path = rng.integers(0, 2, (n, d), dtype=np.uint8)
    member = rng.integers(0, 1 << (bits - 1), (n, d), dtype=np.uint8) if bits > 1 else None
    if codebook is None:
        codebook = np.sort(rng.standard_normal(1 << (bits + 1)) * 1.2)
    signs = rng.integers(0, 2, (1, d), dtype=np.uint8)
    block = d & -d
    return {
        "format": 2, "n": n, "d": d, "bits": bits, "n_states": n_states, "block": block,
        "path_packed": pack_le(path, 1),
        "member_packed": pack_le(member, bits - 1) if member is not None else None,
        "scales": (np.abs(rng.standard_normal(n)) * 0.01 + 0.015).astype(np.float16),
        "signs_packed": pack_le(signs, 1),
        "inv_equil": (rng.uniform(0.6, 1.6, d)).astype(np.float16),
        "codebook": np.asarray(codebook).astype(np.float16),
        "bias": (rng.standard_normal(n) * 0.1).astype(np.float16) if bias else None,
        "seed": seed,
    }


def lm_head_argmax(x: np.ndarray, w: np.ndarray) -> tuple[np.ndarray, np.ndarray]:
    """Greedy next token of the reference's decode loops: fp16 lm_head
    logits then ``logits[:, -1:].argmax(-1)`` (scripts/run_packed.py:164,178,190;
    scripts/graph_decode_bench.py:55-112).  The logits are computed in
    float64 and rounded to fp16 as the reference's fp16 F.linear returns
    them; the argmax keeps the first index among equal fp16 values (as
    torch.argmax does) and takes a NaN as the maximum.  Returns (token index
    per batch row, float64 logits [B, V])."""
    logits = np.asarray(x, dtype=np.float64) @ np.asarray(w, dtype=np.float64).T
    l16 = logits.astype(np.float16).astype(np.float64)
    nan = np.isnan(l16)
    l16 = np.where(nan, np.inf, l16)
    tok = np.where(nan.any(axis=-1), np.argmax(nan, axis=-1), np.argmax(l16, axis=-1))
    return tok, logits

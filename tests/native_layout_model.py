"""Word-level model of the native TCQ stream and of the GEMV decoder.

TEST INFRASTRUCTURE: a numpy restatement of what the CUDA kernels in
``turbopress_b200/csrc`` do with bits (stream layout, halo exchange,
GF(2) subset convolution, level words, pair table, permuted activations),
so the layout can be checked against the oracle on the CPU.  It mirrors
the kernel code, not the reference; the reference side is the oracle.
"""

from __future__ import annotations

import numpy as np

from oracle import tcq_oracle as O

M32 = 0xFFFFFFFF
WTAB = [0, 2, 1, 3, 0, 2, 1, 3]          # column r (mod 8) -> level word
LO_HI = {0: (0, 4), 1: (2, 6), 2: (1, 5), 3: (3, 7)}


def col_slot(r):
    return WTAB[r], r >> 2


def zperm_pos(lc):
    w, h = col_slot(lc & 7)
    return 2 * (4 * w + (lc >> 3)) + h


def member_bit_pos(bits, lc, mb):
    j, r = lc >> 3, lc & 7
    if bits == 2:
        return 0, 8 * j + [2, 0, 3, 1, 6, 4, 7, 5][r]
    if mb < 2:
        return r & 1, 8 * j + [2, 2, 0, 0, 6, 6, 4, 4][r] + mb
    w, h = col_slot(r)
    q, jj = j >> 1, j & 1
    xbit = (7 if h == 0 else 8) if jj == 0 else (23 if h == 0 else 24)
    return 2, (xbit + 2 * (2 * w + q)) & 31


def kmask(g, m):
    return sum(1 << k for k in range(m + 1) if (g >> (m if k == 0 else k - 1)) & 1)


def relayout(path, member, bits):
    """path/member: unpacked uint8 [n, d] -> dict[(row, chunk)] = [P, M0, M1, M2]."""
    n, d = path.shape
    n_pad = -(-n // 16) * 16
    d_pad = -(-d // 256) * 256
    words = np.zeros((n_pad, d_pad // 32, 4), dtype=np.uint64)
    for r in range(n):
        for c in range(d):
            ch, lc = divmod(c, 32)
            words[r, ch, 0] |= int(path[r, c]) << lc
            for mb in range(bits - 1):
                if (int(member[r, c]) >> mb) & 1:
                    w, pos = member_bit_pos(bits, lc, mb)
                    words[r, ch, 1 + w] |= 1 << pos
    return words, n_pad, d_pad


def funnel_l(lo, hi, k):
    return ((hi << k) | (lo >> (32 - k))) & M32 if k else hi


def level_words(P, H, mw, bits, s):
    m = s.bit_length() - 1
    g0, g1 = O.GENERATORS[s]
    k0, k1 = kmask(g0, m), kmask(g1, m)
    s0 = s1 = 0
    for k in range(m + 1):
        dk = funnel_l(H, P, k)
        if (k0 >> k) & 1:
            s0 ^= dk
        if (k1 >> k) & 1:
            s1 ^= dk
    E = (s0 & 0x55555555) | ((s1 << 1) & 0xAAAAAAAA)
    O_ = ((s0 >> 1) & 0x55555555) | (s1 & 0xAAAAAAAA)
    M0, M1 = mw[0], mw[1]
    if bits == 1:
        A = Bm = Cw = Dm = 0
    elif bits == 2:
        A, Bm, Cw, Dm = M0, M0 >> 1, (M0 << 2) & M32, (M0 << 1) & M32
    else:
        A, Bm, Cw, Dm = M0, (M0 << 2) & M32, M1, (M1 << 2) & M32
    return [(E & 0x33333333) | (A & 0xCCCCCCCC), ((E >> 2) & 0x33333333) | (Bm & 0xCCCCCCCC),
            (O_ & 0x33333333) | (Cw & 0xCCCCCCCC), ((O_ >> 2) & 0x33333333) | (Dm & 0xCCCCCCCC)]


def pair_levels(L, w, j, bits, M2):
    """Levels (lo, hi) looked up by the kernel for byte j of level word w."""
    byte = (L[w] >> (8 * j)) & 0xFF
    lmask = (1 << (bits + 1)) - 1 if bits <= 3 else 15
    lo, hi = byte & 15 & lmask, (byte >> 4) & lmask
    if bits == 4:
        q, jj = j >> 1, j & 1
        s = 2 * (2 * w + q)
        X = ((M2 >> s) | (M2 << (32 - s))) & M32 if s else M2
        X &= 0x01800180
        lo_b, hi_b = (7, 8) if jj == 0 else (23, 24)
        lo |= ((X >> lo_b) & 1) << 4
        hi |= ((X >> hi_b) & 1) << 4
    return lo, hi


def decode_levels_native(path, member, bits, s):
    """Levels [n, d] recovered through the native layout + kernel decode."""
    n, d = path.shape
    words, n_pad, d_pad = relayout(path, member, bits)
    out = np.zeros((n_pad, d_pad), dtype=np.int64)
    for r in range(n_pad):
        for ch in range(d_pad // 32):
            P = int(words[r, ch, 0])
            H = int(words[r, ch - 1, 0]) if ch else 0
            mw = [int(words[r, ch, 1]), int(words[r, ch, 2]), int(words[r, ch, 3])]
            L = level_words(P, H, mw, bits, s)
            for w in range(4):
                for j in range(4):
                    lo, hi = pair_levels(L, w, j, bits, mw[2])
                    clo, chi = 8 * j + LO_HI[w][0], 8 * j + LO_HI[w][1]
                    out[r, ch * 32 + clo] = lo
                    out[r, ch * 32 + chi] = hi
    return out[:n, :d]


def gemv_native(p, x):
    """y = z @ (cb[level] * scale)^T through the native decode model, fp32 z."""
    d, bits, s = int(p["d"]), int(p["bits"]), int(p["n_states"])
    path = O.unpack_le(p["path_packed"], d, 1)
    member = O.unpack_le(p["member_packed"], d, bits - 1) if bits > 1 else np.zeros_like(path)
    lv = decode_levels_native(path, member, bits, s)
    cb = np.asarray(p["codebook"], np.float16).astype(np.float32)
    z = O.rotate_activations(np.asarray(x).reshape(-1, d), O.rot_scale(p), int(p["block"]))
    # permuted activations: the kernel multiplies pair (lo, hi) by z at the
    # permuted positions; reconstruct the column order to check the perm.
    d_pad = -(-d // 256) * 256
    zp = np.zeros((z.shape[0], d_pad), np.float32)
    for c in range(d):
        zp[:, (c // 32) * 32 + zperm_pos(c % 32)] = z[:, c]
    inv = np.zeros(d, np.int64)
    for c in range(d):
        inv[c] = (c // 32) * 32 + zperm_pos(c % 32)
    acc = zp[:, inv] @ cb[lv].T
    y = acc * np.asarray(p["scales"], np.float16).astype(np.float32)[None, :]
    if p.get("bias") is not None:
        y = y + np.asarray(p["bias"], np.float16).astype(np.float32)
    return y

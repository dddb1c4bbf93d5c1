"""Torch restatement of the reference's own CPU forward paths (test and
benchmark infrastructure: the timed CPU baseline of bench.py, checked against
the numpy oracle in tests/test_oracle_golden.py; never on a product path).

The reference runs PackedTCQLinear on the CPU with torch ops in fp32:
``mode="tiled"`` unpacks the bit streams, window-decodes the level codes,
dequantizes one tile of rows at a time and multiplies
(turbopress/runtime.py:291-331), ``mode="cached"`` decodes once, folds the
rotation back into the weights and runs ``F.linear`` (runtime.py:278-288,
:308-310).  The functions below perform the same tensor operations.
"""

from __future__ import annotations

import math

import numpy as np
import torch
import torch.nn.functional as F

from . import tcq_oracle as O


def unpack_le(packed: torch.Tensor, d: int, width: int) -> torch.Tensor:
    """runtime.py:93-100."""
    n = packed.shape[0]
    shifts = torch.arange(8, dtype=torch.uint8)
    bits = (packed[:, :, None] >> shifts) & 1
    stream = bits.reshape(n, -1)[:, : d * width]
    weights = 1 << torch.arange(width, dtype=torch.int32)
    return (stream.reshape(n, d, width).to(torch.int32) * weights).sum(-1).to(torch.uint8)


def window_decode_levels(path_bits: torch.Tensor, member: torch.Tensor, n_states: int) -> torch.Tensor:
    """runtime.py:122-139 (the LUT of runtime.py:106-119 from the oracle)."""
    n, d = path_bits.shape
    m = n_states.bit_length() - 1
    lut = torch.from_numpy(O.subset_lut(n_states).astype(np.uint8))
    padded = F.pad(path_bits.to(torch.int32), (m, 0))
    x = padded[:, m:] << m
    for j in range(m):
        x = x | (padded[:, j: j + d] << j)
    return (member.to(torch.int32) * 4 + lut[x.long()]).to(torch.uint8)


def decode_rows(p: dict, r0: int, r1: int) -> torch.Tensor:
    """runtime.py:291-301: rows [r0, r1) of the rotated weights, fp16."""
    d, bits = int(p["d"]), int(p["bits"])
    path = torch.from_numpy(np.ascontiguousarray(p["path_packed"][r0:r1]))
    pathb = unpack_le(path, d, 1)
    if p.get("member_packed") is not None:
        memb = unpack_le(torch.from_numpy(np.ascontiguousarray(p["member_packed"][r0:r1])), d, bits - 1)
    else:
        memb = torch.zeros_like(pathb)
    levels = window_decode_levels(pathb, memb, int(p["n_states"]))
    cb = torch.from_numpy(p["codebook"]).float()
    sc = torch.from_numpy(p["scales"][r0:r1]).float()
    return (cb[levels.long()] * sc[:, None]).to(torch.float16)


def fwht(x: torch.Tensor) -> torch.Tensor:
    """runtime.py:192-201."""
    d = x.shape[-1]
    y = x.reshape(-1, d)
    h = 1
    while h < d:
        y = y.reshape(-1, d // (2 * h), 2, h)
        even, odd = y[:, :, 0, :], y[:, :, 1, :]
        y = torch.stack((even + odd, even - odd), dim=2).reshape(-1, d)
        h *= 2
    return (y / math.sqrt(d)).reshape(x.shape)


def block_fwht(x: torch.Tensor, block: int) -> torch.Tensor:
    """runtime.py:204-208."""
    if block == x.shape[-1]:
        return fwht(x)
    m = x.shape[-1] // block
    return fwht(x.reshape(*x.shape[:-1], m, block)).reshape(x.shape)


def rot_scale(p: dict) -> torch.Tensor:
    """runtime.py:245-249."""
    return torch.from_numpy(O.rot_scale(p))


def tiled_forward(p: dict, x: torch.Tensor, rs: torch.Tensor, tile_rows: int = 1024) -> torch.Tensor:
    """runtime.py:304-331 (the tiled branch, CPU: fp32 compute)."""
    n, d = int(p["n"]), int(p["d"])
    z = block_fwht(x.to(torch.float32) * rs.to(torch.float32), int(p["block"]))
    flat = z.reshape(-1, d)
    y = torch.empty(flat.shape[0], n, dtype=torch.float32)
    for r0 in range(0, n, tile_rows):
        r1 = min(r0 + tile_rows, n)
        y[:, r0:r1] = flat @ decode_rows(p, r0, r1).to(torch.float32).T
    if p.get("bias") is not None:
        y = y + torch.from_numpy(p["bias"]).float()
    return y.reshape(*z.shape[:-1], n)


def cached_weight(p: dict) -> torch.Tensor:
    """runtime.py:278-288: decode, rotate back to the original basis, fp16."""
    n, d = int(p["n"]), int(p["d"])
    w_rot = decode_rows(p, 0, n).float()
    signs = O.unpack_le(p["signs_packed"], d, 1)[0].astype(np.float32) * 2 - 1
    w = block_fwht(w_rot, int(p["block"])) * torch.from_numpy(signs)[None, :]
    w = w * torch.from_numpy(p["inv_equil"]).float()[None, :]
    return w.to(torch.float16)


def cached_forward(w16: torch.Tensor, x: torch.Tensor) -> torch.Tensor:
    """runtime.py:308-310 on the CPU: F.linear in fp32."""
    return F.linear(x.to(torch.float32), w16.to(torch.float32))

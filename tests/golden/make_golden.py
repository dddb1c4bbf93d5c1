"""Generate the golden fixtures in this folder from the reference itself.

Run in a container where the reference TurboPress sources are importable:

    TURBOPRESS_REF=/path/to/turbopress python tests/golden/make_golden.py

It imports the reference's own functions (runtime.pack_le / window decode /
pack_linear / PackedTCQLinear, trellis encoder, pipeline.quantize_matrix,
hadamard) and records their inputs and outputs as compressed ``.npz`` files.
The fixtures travel with the repository; the GPU box never needs the
reference.  Everything is seeded, so re-running reproduces the same bytes.
"""

from __future__ import annotations

import hashlib
import os
import sys
from pathlib import Path

import numpy as np
import torch
from torch import nn

REF = os.environ.get("TURBOPRESS_REF")
if not REF:
    sys.exit("set TURBOPRESS_REF to the reference TurboPress source tree (the folder holding turbopress/)")
sys.path.insert(0, REF)

from turbopress import pipeline as P  # noqa: E402
from turbopress.runtime import (  # noqa: E402
    PackedTCQLinear,
    _block_fwht,
    pack_le,
    pack_linear,
    subset_lut,
    unpack_le,
    v1_payload_to_packed,
    window_decode_levels,
)
from turbopress.trellis import Trellis, decode_levels, tcq_optimized_codebook, tcq_quantize_rows  # noqa: E402

OUT = Path(__file__).resolve().parent
torch.set_num_threads(os.cpu_count() or 8)


def _np(t):
    return None if t is None else t.detach().cpu().numpy()


def _payload_arrays(prefix: str, p: dict, out: dict) -> None:
    for k in ("n", "d", "bits", "n_states", "block", "seed"):
        out[f"{prefix}{k}"] = np.int64(p[k])
    for k in ("path_packed", "member_packed", "scales", "signs_packed", "inv_equil", "codebook", "bias"):
        if p[k] is not None:
            out[f"{prefix}{k}"] = _np(p[k])


def bitpack_cases() -> None:
    out = {}
    for width in (1, 2, 3, 5, 8):
        gen = torch.Generator().manual_seed(0)
        vals = torch.randint(0, 1 << width, (5, 77), generator=gen, dtype=torch.uint8)
        out[f"w{width}_vals"] = _np(vals)
        out[f"w{width}_packed"] = _np(pack_le(vals, width))
        assert torch.equal(unpack_le(pack_le(vals, width), 77, width), vals)
    for s in (4, 8, 16, 64):
        out[f"lut{s}"] = _np(subset_lut(Trellis(s)))
        out[f"subset_table{s}"] = _np(Trellis(s).subset_table)
    # v1 flat MSB-first packing
    vals = np.array([5, 1], dtype=np.uint8)
    out["v1_pack_51_w3"] = P.pack_bits(vals, 3)
    gen = torch.Generator().manual_seed(3)
    vals = torch.randint(0, 8, (333,), generator=gen, dtype=torch.uint8).numpy()
    out["v1_vals"] = vals
    out["v1_packed_w3"] = P.pack_bits(vals, 3)
    np.savez_compressed(OUT / "bitpack.npz", **out)


def encoder_cases() -> None:
    """Window decode == sequential walk == encoder level codes
    (reference test tests/test_runtime.py:28-42), recorded."""
    out = {}
    for s in (4, 8, 16, 64):
        for bits in (1, 2, 3, 4):
            gen = torch.Generator().manual_seed(0)
            w = torch.randn(6, 96, generator=gen)
            q = tcq_quantize_rows(w, bits=bits, n_states=s)
            tr = Trellis(s)
            assert torch.equal(decode_levels(q.path_bits, q.member_codes, tr), q.level_codes)
            assert torch.equal(window_decode_levels(q.path_bits, q.member_codes, tr), q.level_codes)
            key = f"s{s}_b{bits}"
            out[f"{key}_path"] = _np(q.path_bits)
            out[f"{key}_member"] = _np(q.member_codes)
            out[f"{key}_levels"] = _np(q.level_codes)
    np.savez_compressed(OUT / "encoder.npz", **out)


def codebooks() -> None:
    out = {}
    for s in (16, 64):
        for bits in (1, 2, 3, 4):
            out[f"opt_b{bits}_s{s}"] = _np(tcq_optimized_codebook(bits, s).to(torch.float16))
    for bits in (2, 3, 4):
        out[f"pipe_b{bits}_s64"] = _np(P.tcq_codebook(bits, 64).to(torch.float16))
    np.savez_compressed(OUT / "codebooks.npz", **out)


def _layer_case(name, n, d, bits, s, seed, bias, batch, equil_one, out, full=True):
    gen = torch.Generator().manual_seed(seed)
    lin = nn.Linear(d, n, bias=bias)
    lin.weight.data = torch.randn(n, d, generator=gen) * 0.02
    if bias:
        lin.bias.data = torch.randn(n, generator=gen) * 0.1
    act = lin.weight.data.norm(dim=0) if equil_one else torch.rand(d, generator=gen) + 0.5
    p = pack_linear(lin, act, bits=bits, n_states=s, seed=seed)
    _payload_arrays(f"{name}_", p, out)
    tiled = PackedTCQLinear(p, mode="tiled", tile_rows=256)
    cached = PackedTCQLinear(p, mode="cached")
    w = tiled.decode_rows(0, n)
    gx = torch.Generator().manual_seed(seed + 1)
    x = torch.randn(batch, d, generator=gx).to(torch.float16)
    with torch.no_grad():
        y_tiled = tiled(x.float())          # CPU reference path computes in fp32
        y_cached = cached(x.float())
        z = _block_fwht(x.float() * tiled.rot_scale.float(), tiled.block)
    out[f"{name}_x"] = _np(x)
    out[f"{name}_rot_scale"] = _np(tiled.rot_scale)
    out[f"{name}_z"] = _np(z)
    out[f"{name}_y_tiled"] = _np(y_tiled)
    out[f"{name}_y_cached"] = _np(y_cached)
    out[f"{name}_w_sha256"] = np.frombuffer(hashlib.sha256(_np(w).tobytes()).digest(), dtype=np.uint8)
    out[f"{name}_w_rows0_4"] = _np(w[:4])
    out[f"{name}_cache_sha256"] = np.frombuffer(
        hashlib.sha256(_np(cached._w_cache).tobytes()).digest(), dtype=np.uint8)
    out[f"{name}_packed_bytes_tiled"] = np.int64(tiled.packed_bytes())
    if full:
        out[f"{name}_w"] = _np(w)
        out[f"{name}_cache"] = _np(cached._w_cache)


def layer_cases() -> None:
    out = {}
    # 1024x1024, 2-bit, S=64, seed 0, equilibration 1, batch 1
    _layer_case("c1", 1024, 1024, 2, 64, 0, False, 1, True, out, full=False)
    # the reference Triton test shape (tests/test_runtime.py:164-174)
    _layer_case("t256", 192, 256, 3, 64, 0, False, 2, False, out)
    # bias + S=16 (tests/test_runtime.py:62-92)
    _layer_case("b16", 64, 128, 2, 16, 3, True, 5, False, out)
    _layer_case("b16w3", 64, 128, 3, 16, 3, True, 3, False, out)
    # S=8, ragged n, small block (d=96 -> block 32)
    _layer_case("s8", 200, 96, 2, 8, 0, False, 4, False, out)
    # 4-bit, d=576 (block 64), n=37 ragged
    _layer_case("w4", 37, 576, 4, 64, 5, True, 3, False, out)
    # 1-bit (no member stream), S=4
    _layer_case("w1", 48, 160, 1, 4, 2, False, 2, False, out)
    # 3-bit S=64, d=2560 (block 512), n=40: the Qwen3-4B hidden size
    _layer_case("q4b", 40, 2560, 3, 64, 7, False, 1, False, out)
    np.savez_compressed(OUT / "layers.npz", **out)


def v1_cases() -> None:
    out = {}
    for bits in (2, 3, 4):
        torch.manual_seed(0)
        n, d = 96, 256
        w = torch.randn(n, d) * 0.05
        act = w.abs().mean(0).clamp_min(1e-4)
        payload, w_hat = P.quantize_matrix(w, act, bits, 16, seed=0, device="cpu")
        key = f"v1b{bits}"
        for k in ("n", "d", "block", "bits", "n_states"):
            out[f"{key}_{k}"] = np.int64(payload[k])
        for k in ("path_bits", "member_bits", "scales", "signs", "equil", "codebook"):
            if payload[k] is not None:
                out[f"{key}_{k}"] = _np(payload[k])
        out[f"{key}_w_hat"] = _np(w_hat)
        bias = torch.randn(n) if bits == 3 else None
        if bias is not None:
            out[f"{key}_bias"] = _np(bias)
        v2 = v1_payload_to_packed(payload, bias, "cpu")
        _payload_arrays(f"{key}_v2_", v2, out)
        out[f"{key}_v2_decoded"] = _np(PackedTCQLinear(v2, mode="tiled").decode_rows(0, n))
    np.savez_compressed(OUT / "v1.npz", **out)


def fwht_cases() -> None:
    out = {}
    gen = torch.Generator().manual_seed(7)
    for d, block in ((576, 64), (1536, 512), (1024, 1024), (3072, 1024), (128, 128),
                     (2560, 512), (96, 32), (160, 32), (8192, 8192), (4096, 4096), (48, 16), (6, 2)):
        rs = (torch.randn(d, generator=gen).sign() * (torch.rand(d, generator=gen) + 0.5)).to(torch.float16)
        x = torch.randn(3, d, generator=gen).to(torch.float16)
        z = _block_fwht(x.float() * rs.float(), block)
        key = f"d{d}_b{block}"
        out[f"{key}_x"] = _np(x)
        out[f"{key}_rs"] = _np(rs)
        out[f"{key}_z"] = _np(z)
    np.savez_compressed(OUT / "fwht.npz", **out)


if __name__ == "__main__":
    bitpack_cases()
    encoder_cases()
    codebooks()
    fwht_cases()
    v1_cases()
    layer_cases()
    for f in sorted(OUT.glob("*.npz")):
        print(f.name, f.stat().st_size)

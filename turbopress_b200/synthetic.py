"""Seeded synthetic packed decoders for benchmarks and tests.

The BASELINE decoder configurations (Qwen3-0.6B / Qwen3-4B / Llama-3-70B
shapes) are random-init models: every linear is a packed-TCQ layer whose
trellis path and member streams are uniform random bits (every bit string
is a valid trellis codeword), with the reference encoder's data-free
codebook for its bit width, per-row scales of about 1/sqrt(d) (so the
chained activations stay O(1)) and the per-layer rotation seed convention of
turbopress/runtime.py:393.  The streams are generated on the GPU.
"""

from __future__ import annotations

import math
import zlib

import numpy as np
import torch
from torch import Tensor

from .runtime import PackedTCQLinear
from .step import LayerWeights, StepConfig

QWEN3_0_6B = dict(name="qwen3-0.6b", label="Qwen3-0.6B", layers=28, hidden=1024, inter=3072, q_heads=16,
                  kv_heads=8, head_dim=128, vocab=151936, rope_theta=1_000_000.0, qk_norm=True)
QWEN3_4B = dict(name="qwen3-4b", label="Qwen3-4B", layers=36, hidden=2560, inter=9728, q_heads=32, kv_heads=8,
                head_dim=128, vocab=151936, rope_theta=1_000_000.0, qk_norm=True)
# vocabulary not stated by the benchmark configuration: Llama-3's 128256
LLAMA3_70B = dict(name="llama3-70b", label="Llama-3-70B", layers=80, hidden=8192, inter=28672, q_heads=64,
                  kv_heads=8, head_dim=128, vocab=128256, rope_theta=500_000.0, qk_norm=False)
MODELS = {m["name"]: m for m in (QWEN3_0_6B, QWEN3_4B, LLAMA3_70B)}

LINEAR_NAMES = ("q_proj", "k_proj", "v_proj", "o_proj", "gate_proj", "up_proj", "down_proj")


def layer_seed(seed: int, i: int, name: str) -> int:
    """Per-layer rotation seed convention of turbopress/runtime.py:393."""
    return seed + 7919 * i + zlib.crc32(name.encode()) % 1000


def linear_shapes(cfg: dict) -> list[tuple[str, int, int]]:
    """(name, in_features d, out_features n) of one decoder layer."""
    h, i, hd = cfg["hidden"], cfg["inter"], cfg["head_dim"]
    return [("q_proj", h, cfg["q_heads"] * hd), ("k_proj", h, cfg["kv_heads"] * hd),
            ("v_proj", h, cfg["kv_heads"] * hd), ("o_proj", cfg["q_heads"] * hd, h),
            ("gate_proj", h, i), ("up_proj", h, i), ("down_proj", i, h)]


def random_packed_linear(n: int, d: int, bits: int, codebook: Tensor, device, seed: int,
                         bias: bool = False) -> PackedTCQLinear:
    """A format-v2 payload of uniform random trellis streams, in native mode."""
    g = torch.Generator(device=device).manual_seed(seed)
    payload = {
        "format": 2, "n": n, "d": d, "bits": bits, "n_states": 64, "block": d & -d, "seed": seed,
        "path_packed": torch.randint(0, 256, (n, -(-d // 8)), generator=g, dtype=torch.uint8, device=device),
        "member_packed": torch.randint(0, 256, (n, -(-d * (bits - 1) // 8)), generator=g, dtype=torch.uint8,
                                       device=device) if bits > 1 else None,
        "scales": ((torch.rand(n, generator=g, device=device) * 0.5 + 0.75) / math.sqrt(d)).half(),
        "signs_packed": torch.randint(0, 256, (1, -(-d // 8)), generator=g, dtype=torch.uint8, device=device),
        "inv_equil": (torch.rand(d, generator=g, device=device) * 0.4 + 0.8).half(),
        "codebook": codebook.to(device=device, dtype=torch.float16).clone(),
        "bias": (torch.randn(n, generator=g, device=device) * 0.05).half() if bias else None,
    }
    return PackedTCQLinear(payload, mode="cuda")


def mixed_bits(layers: int, choices=(2, 3, 4), seed: int = 0) -> list[int]:
    """Seeded per-layer bit widths averaging 3.0: a balanced multiset of
    `choices` (2 and 4 paired around 3) shuffled with `seed`."""
    rng = np.random.default_rng(seed)
    base = [choices[i % len(choices)] for i in range(layers)]
    # keep the weighted average at exactly 3.0 when the count is not a multiple of 3
    while sum(base) != 3 * layers:
        i = base.index(4) if sum(base) > 3 * layers else base.index(2)
        base[i] = 3
    rng.shuffle(base)
    return [int(b) for b in base]


def step_config(cfg: dict) -> StepConfig:
    return StepConfig(hidden=cfg["hidden"], inter=cfg["inter"], q_heads=cfg["q_heads"], kv_heads=cfg["kv_heads"],
                      head_dim=cfg["head_dim"], rms_eps=1e-6, rope_theta=cfg["rope_theta"])


def synthetic_decoder(cfg: dict, layer_bits: list[int], codebooks: dict[int, Tensor], device, seed: int = 0,
                      layers: int | None = None) -> tuple[list[LayerWeights], Tensor]:
    """Packed layers + fp16 norm weights (1 + N(0, 0.1^2)) of a random-init
    decoder with one entry of `layer_bits` per layer (`layers` of them, default
    all of layer_bits); returns (layers, final_norm)."""
    nl = len(layer_bits) if layers is None else layers
    g = torch.Generator(device=device).manual_seed(seed + 1)
    out = []
    hd = cfg["head_dim"]

    def norm_w(n):
        return (1.0 + 0.1 * torch.randn(n, generator=g, device=device)).half()

    for i in range(nl):
        bits = layer_bits[i]
        mods = {}
        for name, d, n in linear_shapes(cfg):
            mods[name] = random_packed_linear(n, d, bits, codebooks[bits], device, layer_seed(seed, i, name))
        out.append(LayerWeights(
            q=mods["q_proj"], k=mods["k_proj"], v=mods["v_proj"], o=mods["o_proj"], gate=mods["gate_proj"],
            up=mods["up_proj"], down=mods["down_proj"], ln1=norm_w(cfg["hidden"]), ln2=norm_w(cfg["hidden"]),
            q_norm=norm_w(hd) if cfg.get("qk_norm") else None, k_norm=norm_w(hd) if cfg.get("qk_norm") else None))
    return out, norm_w(cfg["hidden"])

"""Whole-model decode step on one GPU: ``tp_step_run`` behind a small class.

The reference decodes with a Hugging Face model whose linears are
``PackedTCQLinear`` layers (turbopress/runtime.py:455-541 ``load_packed_model``;
the token loops of scripts/run_packed.py:160-190 and
scripts/graph_decode_bench.py:70-118).  ``DecodeStep`` runs the same decoder
step -- RMSNorm, q/k/v, Qwen3 head norms, RoPE, KV-cache append, GQA
attention, o_proj + residual, RMSNorm, gate/up, SiLU product, down_proj +
residual, final RMSNorm -- as one cooperative kernel launch over the packed
layers, followed by the greedy LM head (``GreedyLMHead``).

    step = DecodeStep.from_hf(model, batch=1, max_tokens=2048)
    step.load_cache(past_key_values)            # optional: a prefilled HF cache
    tok = step.greedy(token_ids, pos)           # one token per batch row

Layers are given as ``LayerWeights`` (seven ``PackedTCQLinear`` modules in the
native mode plus the norm weights); ``DecodeStep`` owns the KV caches
([layers][B][kv_heads][max_tokens][head_dim] fp16, post-RoPE keys), the fp16
activations, the position counter on the device and the workspace.
"""

from __future__ import annotations

import ctypes
import math
from dataclasses import dataclass

import torch
from torch import Tensor

from . import _abi
from .lm_head import GreedyLMHead
from .runtime import PackedTCQLinear

LINEARS = ("q", "k", "v", "o", "gate", "up", "down")


class _Linear(ctypes.Structure):
    _fields_ = [("tcq_stream", ctypes.c_void_p), ("scales", ctypes.c_void_p), ("codebook", ctypes.c_void_p),
                ("rot_scale", ctypes.c_void_p), ("bias", ctypes.c_void_p), ("n", ctypes.c_int64),
                ("d", ctypes.c_int64), ("block", ctypes.c_int64), ("bits", ctypes.c_int32),
                ("n_states", ctypes.c_int32)]


class _Layer(ctypes.Structure):
    _fields_ = [(nm, _Linear) for nm in LINEARS] + [
        ("ln1", ctypes.c_void_p), ("ln2", ctypes.c_void_p), ("q_norm", ctypes.c_void_p), ("k_norm", ctypes.c_void_p),
        ("k_cache", ctypes.c_void_p), ("v_cache", ctypes.c_void_p)]


class _Model(ctypes.Structure):
    _fields_ = [("B", ctypes.c_int32), ("layers", ctypes.c_int32), ("hidden", ctypes.c_int32),
                ("inter", ctypes.c_int32), ("q_heads", ctypes.c_int32), ("kv_heads", ctypes.c_int32),
                ("head_dim", ctypes.c_int32), ("max_tokens", ctypes.c_int32), ("rms_eps", ctypes.c_float),
                ("inv_freq", ctypes.c_void_p), ("final_norm", ctypes.c_void_p), ("hidden_state", ctypes.c_void_p),
                ("final_out", ctypes.c_void_p), ("act", ctypes.c_void_p), ("rope_cos", ctypes.c_void_p),
                ("rope_sin", ctypes.c_void_p)]


@dataclass
class LayerWeights:
    """One decoder layer: packed linears and fp16 norm weights (q_norm /
    k_norm: Qwen3's per-head norms, None for Llama)."""

    q: PackedTCQLinear
    k: PackedTCQLinear
    v: PackedTCQLinear
    o: PackedTCQLinear
    gate: PackedTCQLinear
    up: PackedTCQLinear
    down: PackedTCQLinear
    ln1: Tensor
    ln2: Tensor
    q_norm: Tensor | None = None
    k_norm: Tensor | None = None


@dataclass
class StepConfig:
    hidden: int
    inter: int
    q_heads: int
    kv_heads: int
    head_dim: int
    rms_eps: float = 1e-6
    rope_theta: float = 1_000_000.0


def rope_inv_freq(head_dim: int, theta: float) -> Tensor:
    """RoPE inverse frequencies as the reference model computes them (fp32)."""
    return 1.0 / (theta ** (torch.arange(0, head_dim, 2, dtype=torch.int64).to(dtype=torch.float) / head_dim))


def _lin(m: PackedTCQLinear) -> _Linear:
    if getattr(m, "tcq_stream", None) is None:
        raise ValueError("DecodeStep needs PackedTCQLinear layers in the native mode ('cuda' / 'triton' / 'tiled')")
    return _Linear(m.tcq_stream.data_ptr(), m.scales.data_ptr(), m.codebook.data_ptr(), m.rot_scale.data_ptr(),
                   _abi.ptr(m.bias), m.out_features, m.in_features, m.block, m.bits, m.n_states)


class DecodeStep:
    """One batch-B decode step of a packed decoder as a single kernel launch."""

    def __init__(self, layers: list[LayerWeights], cfg: StepConfig, final_norm: Tensor, batch: int = 1,
                 max_tokens: int = 2048, lm_head: Tensor | None = None) -> None:
        if not layers:
            raise ValueError("no layers")
        dev = layers[0].q.tcq_stream.device if layers[0].q.tcq_stream is not None else None
        if dev is None or dev.type != "cuda":
            raise RuntimeError("DecodeStep runs on CUDA devices only; move the layers to a GPU first")
        self.device, self.cfg, self.B, self.max_tokens = dev, cfg, batch, max_tokens
        self.layers = layers
        L, hd = len(layers), cfg.head_dim
        f16 = dict(dtype=torch.float16, device=dev)
        self.k_cache = torch.zeros(L, batch, cfg.kv_heads, max_tokens, hd, **f16)
        self.v_cache = torch.zeros(L, batch, cfg.kv_heads, max_tokens, hd, **f16)
        self.hidden = torch.zeros(batch, cfg.hidden, **f16)
        self.final_out = torch.zeros(batch, cfg.hidden, **f16)
        self.final_norm = final_norm.to(**f16).contiguous()
        self.inv_freq = rope_inv_freq(hd, cfg.rope_theta).to(dev)
        # fp16 cos / sin of the fp32 angles pos * inv_freq, as the reference
        # model's rotary embedding computes them, for every position
        ang = torch.arange(max_tokens, device=dev, dtype=torch.float32)[:, None] * self.inv_freq[None, :]
        self.rope_cos = ang.cos().half().contiguous()
        self.rope_sin = ang.sin().half().contiguous()
        self.pos = torch.zeros(1, dtype=torch.int32, device=dev)
        self._keep = []
        lib = _abi.lib()
        model = _Model(batch, L, cfg.hidden, cfg.inter, cfg.q_heads, cfg.kv_heads, hd, max_tokens, cfg.rms_eps,
                       self.inv_freq.data_ptr(), self.final_norm.data_ptr(), self.hidden.data_ptr(),
                       self.final_out.data_ptr(), 0, self.rope_cos.data_ptr(), self.rope_sin.data_ptr())
        self.act = torch.zeros(lib.tp_step_act_bytes(ctypes.addressof(model)), dtype=torch.uint8, device=dev)
        model.act = self.act.data_ptr()
        arr = (_Layer * L)()
        for i, lw in enumerate(layers):
            norms = []
            for t in (lw.ln1, lw.ln2, lw.q_norm, lw.k_norm):
                norms.append(None if t is None else t.to(**f16).contiguous())
            self._keep += norms
            arr[i] = _Layer(*[_lin(getattr(lw, nm)) for nm in LINEARS], *[_abi.ptr(t) for t in norms],
                            self.k_cache[i].data_ptr(), self.v_cache[i].data_ptr())
        nbytes = lib.tp_step_image_bytes(L)
        self._image_host = (ctypes.c_uint8 * nbytes)()
        ws = ctypes.c_int64(0)
        _abi.check(lib.tp_step_build(ctypes.addressof(model), ctypes.addressof(arr), ctypes.addressof(self._image_host),
                                     nbytes, ctypes.addressof(ws)), "step_build")
        self._model, self._layers_c = model, arr
        self.workspace = torch.zeros(int(ws.value), dtype=torch.uint8, device=dev)
        _abi.check(lib.tp_step_bind(ctypes.addressof(self._image_host), self.workspace.data_ptr(),
                                    self.workspace.numel()), "step_bind")
        host = torch.frombuffer(bytearray(self._image_host), dtype=torch.uint8)
        self.image = host.to(dev)
        self.lm_head = GreedyLMHead(lm_head) if lm_head is not None else None

    # -- state ----------------------------------------------------------------
    def set_position(self, pos: int) -> None:
        """Number of tokens already in the caches (the next step writes at pos)."""
        if not 0 <= pos < self.max_tokens:
            raise ValueError(f"position {pos} outside [0, {self.max_tokens})")
        self.pos.fill_(pos)

    def load_cache(self, keys: list[Tensor], values: list[Tensor]) -> int:
        """Copy per-layer [B, kv_heads, T, head_dim] (post-RoPE) caches in;
        returns T (and sets the position to it)."""
        T = keys[0].shape[2]
        if T > self.max_tokens:
            raise ValueError("cache longer than max_tokens")
        for i, (k, v) in enumerate(zip(keys, values)):
            self.k_cache[i, :, :, :T].copy_(k)
            self.v_cache[i, :, :, :T].copy_(v)
        self.set_position(T)
        return T

    # -- running --------------------------------------------------------------
    def run(self) -> Tensor:
        """One step on the current stream from ``self.hidden`` (the input
        embeddings) at the device position; returns ``final_out`` [B, hidden]."""
        lib = _abi.lib()
        st = torch.cuda.current_stream(self.device).cuda_stream
        _abi.check(lib.tp_step_run(self.image.data_ptr(), ctypes.addressof(self._image_host), self.pos.data_ptr(),
                                   self.workspace.data_ptr(), self.workspace.numel(), st), "step_run")
        return self.final_out

    def status(self) -> None:
        """Raise if a device-side wait of the last step timed out (synchronizes)."""
        st = torch.cuda.current_stream(self.device).cuda_stream
        _abi.check(_abi.lib().tp_step_status(self.workspace.data_ptr(), st), "step")

    def set_wait(self, barrier_us: int = 0, extra_arrivals: int = 0) -> None:
        """Grid-barrier limit (microseconds; 0 restores the 2 s default) and
        extra arrivals each barrier waits for.  ``extra_arrivals > 0`` is a
        wait that nothing satisfies: the step gives up after ``barrier_us``,
        leaves its outputs incomplete and ``status()`` raises.  Used to test
        the timeout path; every model run keeps 0."""
        _abi.check(_abi.lib().tp_step_set_wait(ctypes.addressof(self._image_host), int(barrier_us),
                                               int(extra_arrivals)), "step_set_wait")
        host = torch.frombuffer(bytearray(self._image_host), dtype=torch.uint8)
        self.image.copy_(host)

    def advance(self) -> None:
        """pos += 1 on the device (graph-capturable)."""
        self.pos.add_(1)

    def greedy(self, embeddings: Tensor) -> Tensor:
        """embeddings [B, hidden] fp16 -> next tokens int64 [B]; advances pos."""
        if self.lm_head is None:
            raise RuntimeError("no LM head given")
        self.hidden.copy_(embeddings)
        out = self.run()
        tok, _ = self.lm_head(out)
        self.advance()
        return tok

    # -- construction from a Hugging Face model ---------------------------------
    @classmethod
    def from_hf(cls, model, batch: int = 1, max_tokens: int = 2048) -> "DecodeStep":
        """From a Qwen3 / Llama ``*ForCausalLM`` whose linears are PackedTCQLinear."""
        c = model.config
        hd = getattr(c, "head_dim", None) or c.hidden_size // c.num_attention_heads
        cfg = StepConfig(hidden=c.hidden_size, inter=c.intermediate_size, q_heads=c.num_attention_heads,
                         kv_heads=c.num_key_value_heads, head_dim=hd, rms_eps=c.rms_norm_eps,
                         rope_theta=_rope_theta(c))
        layers = []
        for blk in model.model.layers:
            a, m = blk.self_attn, blk.mlp
            layers.append(LayerWeights(
                q=a.q_proj, k=a.k_proj, v=a.v_proj, o=a.o_proj, gate=m.gate_proj, up=m.up_proj, down=m.down_proj,
                ln1=blk.input_layernorm.weight.detach(), ln2=blk.post_attention_layernorm.weight.detach(),
                q_norm=a.q_norm.weight.detach() if hasattr(a, "q_norm") else None,
                k_norm=a.k_norm.weight.detach() if hasattr(a, "k_norm") else None))
        head = model.lm_head.weight.detach().to(torch.float16)
        return cls(layers, cfg, model.model.norm.weight.detach(), batch=batch, max_tokens=max_tokens, lm_head=head)


def _rope_theta(c) -> float:
    rp = getattr(c, "rope_parameters", None) or {}
    if isinstance(rp, dict) and "rope_theta" in rp:
        return float(rp["rope_theta"])
    return float(getattr(c, "rope_theta", 10000.0))


def packed_bytes(layers: list[LayerWeights]) -> int:
    """Native-stream bytes of the step's packed linears (the bytes it streams)."""
    return sum(getattr(lw, nm).tcq_stream.numel() for lw in layers for nm in LINEARS)


def step_algorithmic_bytes(layers: list[LayerWeights], cfg: StepConfig, B: int, tokens: int) -> int:
    """Algorithmic HBM bytes of one step: true-rate packed weights with their
    scales / codebooks / rotation scales, the KV cache read over `tokens`
    positions plus the appended k/v, and the fp16 activations in and out of
    every linear."""
    total = 0
    for lw in layers:
        for nm in LINEARS:
            m = getattr(lw, nm)
            n, d, b = m.out_features, m.in_features, m.bits
            total += n * math.ceil(d / 8) + n * math.ceil(d * (b - 1) / 8) + 2 * n + 2 * 2 ** (b + 1) + 2 * d
            total += 2 * B * d + 2 * B * n
    kv = 2 * B * cfg.kv_heads * cfg.head_dim * 2  # k and v per position, fp16
    total += len(layers) * kv * (tokens + 1)
    return total

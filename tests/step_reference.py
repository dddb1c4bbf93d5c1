"""Torch restatement of one decoder step for checking ``DecodeStep``.

It follows the Hugging Face Qwen3 / Llama fp16 forward that the reference
runs its packed models in (transformers Qwen3RMSNorm, apply_rotary_pos_emb,
eager_attention_forward, Qwen3MLP, Qwen3DecoderLayer), with the linears
being the same ``PackedTCQLinear`` modules in their per-call path.
"""

from __future__ import annotations

import torch
import torch.nn.functional as F


def rms_norm(x: torch.Tensor, w: torch.Tensor, eps: float) -> torch.Tensor:
    x32 = x.float()
    var = x32.pow(2).mean(-1, keepdim=True)
    return w * (x32 * torch.rsqrt(var + eps)).to(x.dtype)


def rotate_half(x: torch.Tensor) -> torch.Tensor:
    h = x.shape[-1] // 2
    return torch.cat((-x[..., h:], x[..., :h]), dim=-1)


def reference_step(step, hidden: torch.Tensor, pos: int, k_cache: torch.Tensor, v_cache: torch.Tensor):
    """One step of `step`'s model from fp16 `hidden` [B, h] at position `pos`
    over copies of its caches ([L][B][kv][T][hd], written at pos).  Returns
    (final normed output [B, h], residual stream [B, h])."""
    cfg = step.cfg
    B = hidden.shape[0]
    hd, qh, kvh = cfg.head_dim, cfg.q_heads, cfg.kv_heads
    eps = cfg.rms_eps
    inv = step.inv_freq.float()
    freqs = pos * inv
    emb = torch.cat((freqs, freqs))
    cos, sin = emb.cos().half(), emb.sin().half()
    scaling = hd ** -0.5
    h = hidden.clone()
    for i, lw in enumerate(step.layers):
        x = rms_norm(h, lw.ln1.half(), eps)
        q = lw.q(x).view(B, qh, hd)
        k = lw.k(x).view(B, kvh, hd)
        v = lw.v(x).view(B, kvh, hd)
        if lw.q_norm is not None:
            q = rms_norm(q, lw.q_norm.half(), eps)
            k = rms_norm(k, lw.k_norm.half(), eps)
        q = q * cos + rotate_half(q) * sin
        k = k * cos + rotate_half(k) * sin
        k_cache[i, :, :, pos] = k
        v_cache[i, :, :, pos] = v
        K = k_cache[i, :, :, : pos + 1]  # [B, kv, T, hd]
        V = v_cache[i, :, :, : pos + 1]
        g = qh // kvh
        Kr = K.repeat_interleave(g, dim=1)
        Vr = V.repeat_interleave(g, dim=1)
        att = torch.matmul(q.unsqueeze(2), Kr.transpose(2, 3)) * scaling  # [B, qh, 1, T]
        att = F.softmax(att, dim=-1, dtype=torch.float32).to(torch.float16)
        o = torch.matmul(att, Vr).reshape(B, qh * hd)
        h = h + lw.o(o)
        x = rms_norm(h, lw.ln2.half(), eps)
        h = h + lw.down(F.silu(lw.gate(x)) * lw.up(x))
    return rms_norm(h, step.final_norm, eps), h

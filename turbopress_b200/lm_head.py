"""Greedy LM head: the fp16 vocabulary GEMV fused with argmax.

Replaces the last step of the reference's decode loops -- the tied fp16
``lm_head`` ``F.linear`` followed by ``logits[:, -1:].argmax(-1)``
(scripts/run_packed.py:164,178,190; scripts/graph_decode_bench.py:55-112) --
with one HBM-bound kernel (``tp_lm_head_argmax``) that streams the weight
matrix once and keeps the running argmax on chip.

    head = GreedyLMHead(model.lm_head.weight)   # fp16 [V, h] on the GPU
    tokens, best = head(h_last)                 # int64 [B], fp32 [B]
"""

from __future__ import annotations

import torch
from torch import Tensor

from . import _abi

MAX_BATCH = 8


class GreedyLMHead:
    """Greedy token selection over an fp16 [V, h] weight matrix."""

    def __init__(self, weight: Tensor) -> None:
        if weight.dim() != 2 or weight.dtype != torch.float16 or not weight.is_cuda:
            raise ValueError("GreedyLMHead needs a 2-D fp16 CUDA weight [V, h]")
        self.weight = weight.contiguous()
        if self.weight.data_ptr() % 16 or self.weight.shape[1] % 8:
            raise ValueError("weight must be 16-byte aligned with h a multiple of 8")
        self.vocab, self.hidden = self.weight.shape
        lib = _abi.lib()
        # zero-filled once; every call leaves it zeroed (use one head per stream)
        self.workspace = torch.zeros(lib.tp_lm_head_workspace_bytes(MAX_BATCH), dtype=torch.uint8,
                                     device=self.weight.device)

    def __call__(self, x: Tensor, return_logits: bool = False):
        """x [B, h] (or [..., h] with B = prod of the leading dims, <= 8).
        Returns (tokens int64 [B], best logit fp32 [B]) and, when asked, the
        fp32 logits [B, V]."""
        if x.shape[-1] != self.hidden:
            raise ValueError(f"expected last dim {self.hidden}, got {x.shape[-1]}")
        x2 = x.reshape(-1, self.hidden).to(device=self.weight.device, dtype=torch.float16).contiguous()
        B = x2.shape[0]
        if not 1 <= B <= MAX_BATCH:
            raise ValueError(f"batch must be in [1, {MAX_BATCH}], got {B}")
        dev = self.weight.device
        tokens = torch.empty(B, dtype=torch.int64, device=dev)
        best = torch.empty(B, dtype=torch.float32, device=dev)
        logits = torch.empty(B, self.vocab, dtype=torch.float32, device=dev) if return_logits else None
        with torch.cuda.device(dev):
            st = torch.cuda.current_stream(dev).cuda_stream
            _abi.check(_abi.lib().tp_lm_head_argmax(
                x2.data_ptr(), self.weight.data_ptr(), B, self.vocab, self.hidden, _abi.ptr(logits),
                tokens.data_ptr(), best.data_ptr(), self.workspace.data_ptr(), self.workspace.numel(), st),
                "lm_head_argmax")
        return (tokens, best, logits) if return_logits else (tokens, best)

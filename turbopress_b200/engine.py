"""Persistent decode engine: a chain of packed-TCQ linears in one launch.

``DecodeEngine`` compiles a list of native ``PackedTCQLinear`` modules and
their data flow into a program image for ``tp_engine_run``
(``include/turbopress_b200.h``).  One cooperative kernel with one CTA per
SM then runs every op: weights stream through per-warp bulk-copy rings
across op boundaries, and an op waits (bounded, on the device) only for
the op that produces its input.  It replaces a sequence of
``PackedTCQLinear.forward`` calls in mode ``"triton"``
(turbopress/runtime.py:312-334) chained by their activations; outputs are
fp32, accumulated with atomics (order not fixed).

    eng = DecodeEngine([q, k, v, o], inputs=[None, None, None, 0])
    outs = eng.run(x)          # list of fp32 [B, n] views, one per op

``inputs[i]`` is ``None`` (op i reads the external input of its width,
shared by every such op) or the index of an earlier op whose output is op
i's input.
"""

from __future__ import annotations

import ctypes
from typing import Sequence

import numpy as np
import torch
from torch import Tensor

from . import _abi
from .runtime import PackedTCQLinear

MAX_BATCH = 4


class _EngineOp(ctypes.Structure):
    """Mirror of ``tp_engine_op``."""

    _fields_ = [
        ("tcq_stream", ctypes.c_void_p),
        ("scales", ctypes.c_void_p),
        ("bias", ctypes.c_void_p),
        ("rot_scale", ctypes.c_void_p),
        ("x", ctypes.c_void_p),
        ("y", ctypes.c_void_p),
        ("n", ctypes.c_int64),
        ("d", ctypes.c_int64),
        ("block", ctypes.c_int32),
        ("x_dtype", ctypes.c_int32),
        ("dep", ctypes.c_int32),
        ("reserved", ctypes.c_int32),
    ]


class DecodeEngine:
    """Program of packed-TCQ linears run by one persistent kernel."""

    def __init__(self, layers: Sequence[PackedTCQLinear], inputs: Sequence[int | None] | None = None, *,
                 batch: int = 1, input_dtype: torch.dtype = torch.float16) -> None:
        layers = list(layers)
        if not layers:
            raise ValueError("DecodeEngine needs at least one layer")
        inputs = [None] * len(layers) if inputs is None else list(inputs)
        if len(inputs) != len(layers):
            raise ValueError("inputs must have one entry per layer")
        if not 1 <= batch <= MAX_BATCH:
            raise ValueError(f"batch must be in [1, {MAX_BATCH}], got {batch}")
        first = layers[0]
        for i, m in enumerate(layers):
            if not isinstance(m, PackedTCQLinear):
                raise TypeError(f"layer {i} is not a PackedTCQLinear")
            if m._needs_materialize():
                m._materialize()
            if m.tcq_stream is None:
                raise ValueError(f"layer {i} has no native stream (bits 1..4 and a packed mode are required)")
            if (m.bits, m.n_states) != (first.bits, first.n_states) or not torch.equal(m.codebook, first.codebook):
                raise ValueError("all layers of one engine must share bits, n_states and codebook")
            dep = inputs[i]
            if dep is not None:
                if not 0 <= dep < i:
                    raise ValueError(f"layer {i}: input must come from an earlier layer (got {dep})")
                if layers[dep].out_features != m.in_features:
                    raise ValueError(f"layer {i}: width {m.in_features} != layer {dep} output "
                                     f"{layers[dep].out_features}")
        dev = first.tcq_stream.device
        self.device = dev
        self.layers = layers
        self.inputs = inputs
        self.batch = batch
        self.input_dtype = input_dtype
        self.codebook = first.codebook.contiguous()
        # one fp32 arena for every output (zeroed by one memset per run)
        offs, total = [], 0
        for m in layers:
            offs.append(total)
            total += (batch * m.out_features + 63) // 64 * 64
        self.y_arena = torch.zeros(total, dtype=torch.float32, device=dev)
        self.outputs = [self.y_arena[o:o + batch * m.out_features].view(batch, m.out_features)
                        for o, m in zip(offs, layers)]
        self.x_ext: dict[int, Tensor] = {}
        for m, dep in zip(layers, inputs):
            if dep is None and m.in_features not in self.x_ext:
                self.x_ext[m.in_features] = torch.zeros(batch, m.in_features, dtype=input_dtype, device=dev)
        lib = _abi.lib()
        n_ops = len(layers)
        ops = (_EngineOp * n_ops)()
        for i, (m, dep) in enumerate(zip(layers, inputs)):
            x = self.x_ext[m.in_features] if dep is None else self.outputs[dep]
            ops[i] = _EngineOp(m.tcq_stream.data_ptr(), m.scales.data_ptr(), _abi.ptr(m.bias),
                               m.rot_scale.data_ptr(), x.data_ptr(), self.outputs[i].data_ptr(),
                               m.out_features, m.in_features, m.block,
                               _abi.dtype_code(x.dtype), -1 if dep is None else dep, 0)
        self._ops = ops
        self.n_ops = n_ops
        self._build(absolute_table=True)
        self.counters = torch.zeros(lib.tp_engine_counter_bytes(n_ops) // 4, dtype=torch.int32, device=dev)
        self._layout_checked = False

    def _build(self, absolute_table: bool) -> None:
        """Program image for this device.  With `absolute_table` the builder
        may place the bits <= 3 pair table at a fixed shared-window address
        (one permute per lookup); the kernel checks that layout before use."""
        import os

        lib = _abi.lib()
        first = self.layers[0]
        nbytes = lib.tp_engine_image_bytes(self.n_ops)
        self._image_host = np.zeros((nbytes + 15) // 16 * 16, dtype=np.uint8)  # numpy data is 16-aligned
        prev = os.environ.get("TP_ENGINE_NO_ABS")
        if not absolute_table:
            os.environ["TP_ENGINE_NO_ABS"] = "1"
        try:
            with torch.cuda.device(self.device):
                _abi.check(lib.tp_engine_build(self._ops, self.n_ops, self.batch, first.bits, first.n_states,
                                               self.codebook.data_ptr(), self._image_host.ctypes.data, nbytes),
                           "engine_build")
        finally:
            if not absolute_table:
                if prev is None:
                    os.environ.pop("TP_ENGINE_NO_ABS", None)
                else:
                    os.environ["TP_ENGINE_NO_ABS"] = prev
        self.image = torch.from_numpy(self._image_host).to(self.device)

    def set_input(self, x: Tensor) -> None:
        """Copy ``x`` [batch, d] into the external input of width d."""
        d = x.shape[-1]
        if d not in self.x_ext:
            raise ValueError(f"no layer reads an external input of width {d}")
        self.x_ext[d].copy_(x.reshape(self.batch, d))

    def run(self, x: Tensor | Sequence[Tensor] | None = None) -> list[Tensor]:
        """Run the program on the current stream; returns the fp32 outputs."""
        if x is not None:
            for t in ([x] if isinstance(x, Tensor) else x):
                self.set_input(t)
        with torch.cuda.device(self.device):
            self.y_arena.zero_()
            self.counters.zero_()
            self.launch()
            if not self._layout_checked and not torch.cuda.is_current_stream_capturing():
                # first run: if the kernel found the shared-memory layout of
                # the fixed-address pair table different from the planned
                # one (status 3), rebuild with the relative layout and rerun
                self._layout_checked = True
                if int(self.counters[self.n_ops].item()) == 3:
                    self._build(absolute_table=False)
                    self.y_arena.zero_()
                    self.counters.zero_()
                    self.launch()
        return self.outputs

    def launch(self) -> None:
        """The engine kernel alone (outputs and counters must be zero)."""
        st = torch.cuda.current_stream(self.device).cuda_stream
        _abi.check(_abi.lib().tp_engine_run(self.image.data_ptr(), self._image_host.ctypes.data,
                                            self.counters.data_ptr(), st), "engine_run")

    def check(self) -> None:
        """Raise if the last run gave up (a dependency or copy wait timed out)."""
        flag = int(self.counters[self.n_ops].item())
        if flag:
            if flag == 3:
                raise RuntimeError("decode engine aborted: the shared-memory layout differs from the one the "
                                   "program was built for (fixed-address pair table); rebuild it")
            what = {1: "a dependency wait", 2: "a weight copy wait"}.get(flag, f"status {flag}")
            raise RuntimeError(f"decode engine aborted: {what} timed out")

"""Tensor-parallel decode engine over the GPUs of one node.

One process per GPU (``torch.distributed``; NCCL for the plumbing).  Every
packed linear is split across the ranks by output rows in 16-row tiles; each
rank decodes its shard with the persistent engine kernel and adds its
partial outputs into every rank's copy of the output through CUDA-IPC peer
mappings (NVLink), then counts completion on every rank.  The all-gather of
the layer outputs (and the all-reduce of split-K partials) is thereby fused
into the GEMV epilogue; no separate collective runs on the data path.

Why every linear is split by output rows (column-parallel in the usual
naming), o/down included: each linear's input is rotated by a Hadamard
transform over whole blocks (turbopress/runtime.py:192-208, block = largest
power of two dividing in_features), and for o_proj the block is the entire
input vector, so a row-parallel o/down would need the full input on every
rank anyway.  With the input replicated, output-row sharding needs no
trellis halo at shard edges and exchanges exactly one output vector per
stage, the same count as column-parallel + all-gather + row-parallel +
all-reduce.

    eng = TPDecodeEngine(mods, inputs)       # same arguments as DecodeEngine
    outs = eng.run(x)                        # full outputs, on every rank
"""

from __future__ import annotations

import ctypes
from typing import Sequence

import numpy as np
import torch
import torch.distributed as dist
from torch import Tensor

from . import _abi
from .engine import MAX_BATCH, _EngineOp
from .runtime import PackedTCQLinear

TILE_ROWS = 16
UNIT_COLS = 256
HANDLE_BYTES = 64


def shard_rows(n: int, rank: int, world: int) -> tuple[int, int]:
    """Rows [r0, r1) of an n-row output owned by `rank`: a contiguous range of
    16-row tiles, tiles split as evenly as possible."""
    tiles = -(-n // TILE_ROWS)
    t0 = rank * tiles // world
    t1 = (rank + 1) * tiles // world
    return min(n, t0 * TILE_ROWS), min(n, t1 * TILE_ROWS)


def shard_stream_bytes(n: int, d: int, bits: int, r0: int, r1: int) -> tuple[int, int]:
    """Byte range of rows [r0, r1) (tile aligned) in the native stream: tiles
    are stored one after another, each units_k * 512 * bits bytes."""
    units_k = -(-d // UNIT_COLS)
    tile_bytes = units_k * 512 * bits
    return (r0 // TILE_ROWS) * tile_bytes, (-(-r1 // TILE_ROWS)) * tile_bytes


def arena_layout(n_fulls: Sequence[int], batch: int, align: int = 256) -> tuple[list[int], int]:
    """Byte offsets of every op's fp32 [batch, n_full] output in one arena
    buffer, and the buffer size."""
    offs, total = [], 0
    for n in n_fulls:
        offs.append(total)
        total += -(-(batch * n * 4) // align) * align
    return offs, max(total, align)


class _CudaView:
    """Zero-copy tensor view of raw device memory (__cuda_array_interface__)."""

    def __init__(self, ptr: int, shape: tuple[int, ...], typestr: str = "<f4"):
        self.__cuda_array_interface__ = {"shape": shape, "typestr": typestr, "data": (ptr, False), "version": 3}


def _view(ptr: int, shape: tuple[int, ...], device: torch.device, typestr: str = "<f4") -> Tensor:
    with torch.cuda.device(device):
        return torch.as_tensor(_CudaView(ptr, shape, typestr), device=device)


class TPDecodeEngine:
    """Tensor-parallel program of packed linears, one shard per rank.

    `layers` / `inputs` are the FULL modules and data flow (as for
    ``DecodeEngine``), identical on every rank; each rank keeps only its row
    shard of every weight stream.  Outputs are fp32 and complete on every
    rank after ``run``.
    """

    def __init__(self, layers: Sequence[PackedTCQLinear], inputs: Sequence[int | None] | None = None, *,
                 batch: int = 1, input_dtype: torch.dtype = torch.float16, group=None) -> None:
        if not dist.is_initialized():
            raise RuntimeError("TPDecodeEngine needs torch.distributed initialised (one process per GPU)")
        self.group = group
        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)
        if self.world < 2:
            raise ValueError("TPDecodeEngine needs at least 2 ranks; use DecodeEngine on one GPU")
        layers = list(layers)
        if not layers:
            raise ValueError("TPDecodeEngine needs at least one layer")
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
            if dep is not None and (not 0 <= dep < i or layers[dep].out_features != m.in_features):
                raise ValueError(f"layer {i}: input must be an earlier layer's output of width {m.in_features}")
        dev = first.tcq_stream.device
        self.device, self.batch, self.inputs = dev, batch, inputs
        self.n_ops = len(layers)
        lib = _abi.lib()

        # ---- this rank's shards ----
        self._keep: list[Tensor] = []
        self.row0, self.rows, self.n_full = [], [], []
        for m in layers:
            r0, r1 = shard_rows(m.out_features, self.rank, self.world)
            if r1 <= r0:
                raise ValueError(f"layer with {m.out_features} rows is too small for {self.world} ranks")
            b0, b1 = shard_stream_bytes(m.out_features, m.in_features, m.bits, r0, r1)
            self._keep.append(m.tcq_stream[b0:b1].clone())
            self._keep.append(m.scales[r0:r1].clone())
            self._keep.append(None if m.bias is None else m.bias[r0:r1].clone())
            self.row0.append(r0)
            self.rows.append(r1 - r0)
            self.n_full.append(m.out_features)
        self.codebook = first.codebook.contiguous()
        self.rot_scales = [m.rot_scale for m in layers]

        # ---- peer-mapped arena (2 buffers) and counter block ----
        offs, self.arena_bytes = arena_layout(self.n_full, batch)
        self.y_offsets = offs
        ctr_bytes = -(-lib.tp_engine_counter_bytes(self.n_ops) // 256) * 256
        self._own: list[int] = []
        with torch.cuda.device(dev):
            for nbytes in (self.arena_bytes, self.arena_bytes, ctr_bytes):
                p = ctypes.c_void_p()
                _abi.check(lib.tp_ipc_alloc(nbytes, ctypes.byref(p)), "ipc_alloc")
                self._own.append(p.value)
            handles = []
            for p in self._own:
                h = ctypes.create_string_buffer(HANDLE_BYTES)
                _abi.check(lib.tp_ipc_get_handle(p, h), "ipc_get_handle")
                handles.append(h.raw)
        gathered: list = [None] * self.world
        dist.all_gather_object(gathered, (self.rank, handles), group=group)
        self._opened: list[int] = []
        peer = [[0, 0, 0] for _ in range(self.world)]
        with torch.cuda.device(dev):
            for r, hs in gathered:
                if r == self.rank:
                    peer[r] = list(self._own)
                    continue
                for k, h in enumerate(hs):
                    p = ctypes.c_void_p()
                    _abi.check(lib.tp_ipc_open(ctypes.create_string_buffer(h, HANDLE_BYTES), ctypes.byref(p)),
                               "ipc_open")
                    peer[r][k] = p.value
                    self._opened.append(p.value)
        self.peer_arena = torch.tensor([[peer[r][0], peer[r][1]] for r in range(self.world)], dtype=torch.int64,
                                       device=dev)
        self.peer_ctr = torch.tensor([peer[r][2] for r in range(self.world)], dtype=torch.int64, device=dev)
        self.counters_ptr = self._own[2]
        self.outputs_buf = [[_view(self._own[b] + o, (batch, n), dev) for o, n in zip(offs, self.n_full)]
                            for b in range(2)]

        # ---- external inputs (replicated: every rank gets the same x) ----
        self.x_ext: dict[int, Tensor] = {}
        for m, dep in zip(layers, inputs):
            if dep is None and m.in_features not in self.x_ext:
                self.x_ext[m.in_features] = torch.zeros(batch, m.in_features, dtype=input_dtype, device=dev)

        # ---- program image ----
        ops = (_EngineOp * self.n_ops)()
        for i, (m, dep) in enumerate(zip(layers, inputs)):
            stream, scales, bias = self._keep[3 * i: 3 * i + 3]
            if dep is None:
                x_ptr, x_dt = self.x_ext[m.in_features].data_ptr(), _abi.dtype_code(input_dtype)
            else:
                x_ptr, x_dt = offs[dep], _abi.TP_F32
            ops[i] = _EngineOp(stream.data_ptr(), scales.data_ptr(), _abi.ptr(bias), m.rot_scale.data_ptr(),
                               x_ptr, offs[i], self.rows[i], m.in_features, m.block, x_dt,
                               -1 if dep is None else dep, 0)
        row0 = (ctypes.c_int64 * self.n_ops)(*self.row0)
        n_full = (ctypes.c_int64 * self.n_ops)(*self.n_full)
        tpd = _TPDesc(self.world, self.rank, (ctypes.c_void_p * 2)(self._own[0], self._own[1]), self.arena_bytes,
                      self.peer_arena.data_ptr(), self.peer_ctr.data_ptr())
        nbytes = lib.tp_engine_image_bytes(self.n_ops)
        self._image_host = np.zeros((nbytes + 15) // 16 * 16, dtype=np.uint8)
        with torch.cuda.device(dev):
            _abi.check(lib.tp_engine_build_tp(ops, row0, n_full, self.n_ops, batch, first.bits, first.n_states,
                                              self.codebook.data_ptr(), ctypes.byref(tpd),
                                              self._image_host.ctypes.data, nbytes), "engine_build_tp")
        self.image = torch.from_numpy(self._image_host).to(dev)
        self.step = 0
        torch.cuda.synchronize(dev)
        dist.barrier(group=group)  # every rank's arena and counters are zero before anyone runs

    # ------------------------------------------------------------------
    def set_input(self, x: Tensor) -> None:
        d = x.shape[-1]
        if d not in self.x_ext:
            raise ValueError(f"no layer reads an external input of width {d}")
        self.x_ext[d].copy_(x.reshape(self.batch, d))

    def launch(self) -> None:
        """The engine kernel alone (stream-ordered; run k writes buffer k % 2)."""
        st = torch.cuda.current_stream(self.device).cuda_stream
        with torch.cuda.device(self.device):
            _abi.check(_abi.lib().tp_engine_run(self.image.data_ptr(), self._image_host.ctypes.data,
                                                self.counters_ptr, st), "engine_run")
        self.step += 1

    def run(self, x: Tensor | Sequence[Tensor] | None = None) -> list[Tensor]:
        if x is not None:
            for t in ([x] if isinstance(x, Tensor) else x):
                self.set_input(t)
        self.launch()
        return self.outputs

    @property
    def outputs(self) -> list[Tensor]:
        """Full fp32 outputs of the latest launch (valid until the next one)."""
        return self.outputs_buf[(self.step - 1) % 2]

    def check(self) -> None:
        flag = int(_view(self.counters_ptr + 4 * self.n_ops, (1,), self.device, "<u4").item())
        if flag == 3:
            raise RuntimeError(f"tensor-parallel engine aborted on rank {self.rank}: the shared-memory layout "
                               "differs from the one the program was built for (set TP_ENGINE_NO_ABS=1 and rebuild)")
        if flag:
            what = {1: "a dependency wait", 2: "a weight copy wait"}.get(flag, f"status {flag}")
            raise RuntimeError(f"tensor-parallel engine aborted on rank {self.rank}: {what} timed out")

    def close(self) -> None:
        """Unmap peers and free this rank's buffers (collective: every rank calls it)."""
        if not self._own:
            return
        torch.cuda.synchronize(self.device)
        dist.barrier(group=self.group)  # no peer still writes into our buffers
        lib = _abi.lib()
        with torch.cuda.device(self.device):
            for p in self._opened:
                lib.tp_ipc_close(p)
            for p in self._own:
                lib.tp_ipc_free(p)
        self._opened, self._own = [], []


class _TPDesc(ctypes.Structure):
    """Mirror of ``tp_engine_tp``."""

    _fields_ = [
        ("n_ranks", ctypes.c_int32),
        ("rank", ctypes.c_int32),
        ("arena", ctypes.c_void_p * 2),
        ("arena_bytes", ctypes.c_int64),
        ("peer_arena", ctypes.c_void_p),
        ("peer_counters", ctypes.c_void_p),
    ]

"""B200-native packed-TCQ runtime: the drop-in for TurboPress's packed linear.

Mirrors the public surface of ``turbopress/runtime.py`` (godsonj64/turbopress
v0.5.2) for the decode path -- ``PackedTCQLinear``, the format-v2 bit-stream
helpers, ``v1_payload_to_packed`` and ``load_packed_model`` -- with every
numerical step executed by the hand-written sm_100a kernels of the C-ABI
library (``include/turbopress_b200.h``).  There is no CPU or Triton
fallback: tensors must live on a CUDA device when a kernel runs, and a
missing native library raises.

Execution modes (``mode=``):
  * ``"cuda"`` -- weights stay at their true bit rate in a native tile layout
    and every forward runs the fused rotate + decode-in-GEMV kernel.
    ``"triton"`` and ``"tiled"`` are accepted aliases (the reference's packed
    modes), so existing callers run unchanged.
  * ``"cached"`` -- decode once on the GPU at load, fold the rotation back
    into fp16 weights, free the packed streams; forward is ``F.linear``
    (turbopress/runtime.py:278-288).

Payloads may arrive on the CPU (``pack_linear`` output, ``torch.load``):
they are kept as registered buffers and converted on the device when the
module is moved there (``.to("cuda")`` / ``.cuda()``), exactly when the
reference would first run them on the GPU.
"""

from __future__ import annotations

import os

import threading
from typing import Any

import torch
import torch.nn.functional as F
from torch import Tensor, nn

from . import _abi

__all__ = [
    "Trellis",
    "pack_le",
    "unpack_le",
    "subset_lut",
    "window_decode_levels",
    "rotate",
    "PackedTCQLinear",
    "v1_payload_to_packed",
    "load_packed_model",
    "MODES",
]

MODES = ("cached", "tiled", "triton", "cuda")
# batch size from which packed forwards use the tcgen05 skinny GEMM (measured
# crossover on B200: level at 16, 1.8-3x faster from 32)
TC_MIN_BATCH = int(os.environ.get("TP_TC_MIN_BATCH", "32"))
_PACKED_MODES = ("tiled", "triton", "cuda")

# Rate-1/2 convolutional generators (octal) per state count
# (turbopress/trellis.py:47-52, pipeline.py:183).
GENERATORS: dict[int, tuple[int, int]] = {4: (0o5, 0o7), 8: (0o15, 0o17), 16: (0o23, 0o35), 64: (0o133, 0o171)}


class Trellis:
    """Decode-side view of the shift-register trellis (turbopress/trellis.py:55-87).

    ``subset_table[s, b]`` is the 2-bit subset emitted from state ``s`` on
    input bit ``b``; the next state is ``((s << 1) | b) & (S - 1)``.
    """

    def __init__(self, n_states: int) -> None:
        if n_states not in GENERATORS:
            raise ValueError(f"n_states must be one of {sorted(GENERATORS)}, got {n_states}")
        self.n_states = n_states
        m = n_states.bit_length() - 1
        g0, g1 = GENERATORS[n_states]
        table = [[0, 0] for _ in range(n_states)]
        for s in range(n_states):
            for b in (0, 1):
                x = (b << m) | s
                table[s][b] = ((bin(x & g1).count("1") & 1) << 1) | (bin(x & g0).count("1") & 1)
        self.subset_table = torch.tensor(table, dtype=torch.int64)


# ---------------------------------------------------------------------------
# format-v2 helpers on the GPU
# ---------------------------------------------------------------------------
def _stream(t: Tensor) -> int:
    return _abi.stream_of(t)


def pack_le(vals: Tensor, width: int) -> Tensor:
    """[n, d] uint8 -> [n, ceil(d*width/8)] uint8, LE bits, rows byte-aligned
    (turbopress/runtime.py:73-90)."""
    if vals.ndim != 2 or vals.dtype != torch.uint8:
        raise ValueError("expected a 2D uint8 tensor")
    if not 1 <= width <= 8:
        raise ValueError(f"width must be in [1, 8], got {width}")
    _abi.require_cuda(vals)
    vals = vals.contiguous()
    n, d = vals.shape
    out = torch.empty(n, -(-d * width // 8), dtype=torch.uint8, device=vals.device)
    _abi.check(_abi.lib().tp_pack_le(vals.data_ptr(), out.data_ptr(), n, d, width, _stream(vals)), "pack_le")
    return out


def unpack_le(packed: Tensor, d: int, width: int) -> Tensor:
    """Inverse of :func:`pack_le` -> [n, d] uint8 (turbopress/runtime.py:93-100)."""
    _abi.require_cuda(packed)
    packed = packed.contiguous()
    n = packed.shape[0]
    if packed.shape[1] * 8 < d * width:
        raise ValueError("packed stream too short for d * width bits")
    out = torch.empty(n, d, dtype=torch.uint8, device=packed.device)
    _abi.check(_abi.lib().tp_unpack_le(packed.data_ptr(), out.data_ptr(), n, d, width, _stream(packed)), "unpack_le")
    return out


def subset_lut(trellis: Trellis) -> Tensor:
    """Window-integer -> subset LUT with 2^(m+1) entries (turbopress/runtime.py:106-119).

    Window bit j holds b_{t-m+j}; the table is tiny trellis metadata.
    """
    m = trellis.n_states.bit_length() - 1
    xs = torch.arange(1 << (m + 1))
    b_cur = (xs >> m) & 1
    state = torch.zeros_like(xs)
    for k in range(m):
        state |= ((xs >> (m - 1 - k)) & 1) << k
    return trellis.subset_table[state, b_cur].to(torch.uint8)


def window_decode_levels(path_bits: Tensor, member_codes: Tensor | None, trellis: Trellis) -> Tensor:
    """Walk-free level decode on the GPU (turbopress/runtime.py:122-139)."""
    _abi.require_cuda(path_bits, member_codes)
    path_bits = path_bits.contiguous()
    n, d = path_bits.shape
    member = None if member_codes is None else member_codes.to(torch.uint8).contiguous()
    out = torch.empty(n, d, dtype=torch.uint8, device=path_bits.device)
    _abi.check(_abi.lib().tp_window_decode_levels(
        path_bits.data_ptr(), _abi.ptr(member), out.data_ptr(), n, d, trellis.n_states, _stream(path_bits)),
        "window_decode_levels")
    return out


def rotate(x: Tensor, rot_scale: Tensor, block: int, out_dtype: torch.dtype | None = None) -> Tensor:
    """``blockFWHT(x * rot_scale)`` in one launch (turbopress/triton_kernel.py:235-260).

    Computed in fp32; returned in ``out_dtype`` (default ``x.dtype``).
    """
    _abi.require_cuda(x, rot_scale)
    d = x.shape[-1]
    flat = x.reshape(-1, d).contiguous()
    out = torch.empty(flat.shape, dtype=out_dtype or x.dtype, device=x.device)
    rs = rot_scale.to(torch.float16).contiguous()
    _abi.check(_abi.lib().tp_rotate(flat.data_ptr(), _abi.dtype_code(flat.dtype), rs.data_ptr(), out.data_ptr(),
                                    _abi.dtype_code(out.dtype), flat.shape[0], d, block, _stream(x)), "rotate")
    return out.reshape(*x.shape[:-1], d)


# ---------------------------------------------------------------------------
# per-device GEMV workspace
# ---------------------------------------------------------------------------
class _WorkspacePool:
    """One zero-initialized scratch buffer per device for the split-K GEMV.

    The kernel leaves the counters at zero on exit, so the buffer is reused
    by every call.  Calls that overlap on the GPU (different streams at the
    same time) must not share it; the reference API is single-stream.
    """

    def __init__(self) -> None:
        self._bufs: dict[int, Tensor] = {}
        self._lock = threading.Lock()

    def get(self, device: torch.device, nbytes: int) -> Tensor:
        idx = device.index if device.index is not None else torch.cuda.current_device()
        with self._lock:
            buf = self._bufs.get(idx)
            if buf is None or buf.numel() < nbytes:
                if torch.cuda.is_current_stream_capturing():
                    raise RuntimeError("turbopress_b200: GEMV workspace must grow during CUDA graph capture; "
                                       "run the model once (warm-up) before capturing")
                size = max(nbytes, 1 << 20, 0 if buf is None else 2 * buf.numel())
                buf = torch.zeros(size, dtype=torch.uint8, device=torch.device("cuda", idx))
                self._bufs[idx] = buf
            return buf

    def check(self, device: torch.device | None = None) -> None:
        """Raise if a GEMV kernel on `device` gave up since the last check
        (tp_gemv_status; it also clears the counter block so the workspace
        is fit for the next call).  Synchronizes the current stream."""
        idx = (device.index if device is not None and device.index is not None
               else torch.cuda.current_device())
        buf = self._bufs.get(idx)
        if buf is None:
            return
        with torch.cuda.device(idx):
            st = _abi.lib().tp_gemv_status(buf.data_ptr(), torch.cuda.current_stream().cuda_stream)
        _abi.check(st, "tcq_gemv (device status)")


WORKSPACE = _WorkspacePool()


def check_device_status(device: torch.device | None = None) -> None:
    """Raise RuntimeError when a packed GEMV on `device` reported a device-side
    failure (a bounded wait that ran out, or a failed layout check) since the
    last check; the affected outputs are NaN or unwritten."""
    WORKSPACE.check(device)
# the tcgen05 path scribbles over its workspace: it must not share the GEMV's
# (whose split-K counter block has to stay zero between calls)
WORKSPACE_TC = _WorkspacePool()


# ---------------------------------------------------------------------------
# the packed linear module
# ---------------------------------------------------------------------------
class PackedTCQLinear(nn.Module):
    """Linear layer running from packed trellis-coded weights on B200.

    Same constructor, attributes, buffers, ``forward`` / ``decode_rows`` /
    ``packed_bytes`` as ``turbopress.runtime.PackedTCQLinear``
    (turbopress/runtime.py:211-362); see the module docstring for modes.
    """

    def __init__(self, payload: dict[str, Any], mode: str = "cached", tile_rows: int = 1024) -> None:
        super().__init__()
        if payload.get("format") != 2:
            raise ValueError("expected a format-v2 payload from pack_linear()")
        if mode not in MODES:
            raise ValueError(f"mode must be one of {MODES}, got {mode!r}")
        self.out_features: int = int(payload["n"])
        self.in_features: int = int(payload["d"])
        self.bits: int = int(payload["bits"])
        self.n_states: int = int(payload["n_states"])
        self.block: int = int(payload["block"])
        self.mode = mode
        self.tile_rows = tile_rows
        self._trellis = Trellis(self.n_states)
        if not 1 <= self.bits <= 7:
            raise ValueError(f"bits must be in [1, 7], got {self.bits}")
        # the native stream covers bits 1..4; 5..7 run the format-v2 GEMV
        self._native = self.bits <= 4

        def _buf(x):
            return None if x is None else torch.as_tensor(x)

        self.register_buffer("path_packed", _buf(payload["path_packed"]))
        self.register_buffer("member_packed", _buf(payload["member_packed"]))
        self.register_buffer("scales", _buf(payload["scales"]).to(torch.float16))
        self.register_buffer("signs_packed", _buf(payload["signs_packed"]))
        self.register_buffer("inv_equil", _buf(payload["inv_equil"]).to(torch.float16))
        self.register_buffer("codebook", _buf(payload["codebook"]).to(torch.float16))
        self.register_buffer("bias", None if payload.get("bias") is None else _buf(payload["bias"]).to(torch.float16))
        self.register_buffer("lut", subset_lut(self._trellis))
        self.register_buffer("rot_scale", None)
        self.register_buffer("tcq_stream", None)
        self.register_buffer("_w_cache", None)
        if self.path_packed is not None and self.path_packed.is_cuda:
            self._materialize()

    # -- device-side preparation ------------------------------------------
    def _apply(self, fn, *args, **kwargs):
        out = super()._apply(fn, *args, **kwargs)
        if self._needs_materialize():
            self._materialize()
        return out

    def _needs_materialize(self) -> bool:
        ref = self.scales
        if ref is None or not ref.is_cuda:
            return False
        if self.rot_scale is None or not self.rot_scale.is_cuda:
            return True
        if self.mode == "cached":
            return self._w_cache is None
        return self._native and self.tcq_stream is None

    @torch.no_grad()
    def _materialize(self) -> None:
        dev = self.scales.device
        lib = _abi.lib()
        d, n = self.in_features, self.out_features
        for name in ("scales", "inv_equil", "codebook", "bias"):
            t = getattr(self, name)
            if t is not None and (t.dtype != torch.float16 or not t.is_contiguous()):
                setattr(self, name, t.to(torch.float16).contiguous())
        with torch.cuda.device(dev):
            st = torch.cuda.current_stream(dev).cuda_stream
            if self.rot_scale is None or not self.rot_scale.is_cuda:
                if self.signs_packed is None:
                    raise RuntimeError("payload has no rotation signs")
                rs = torch.empty(d, dtype=torch.float16, device=dev)
                signs = self.signs_packed.to(dev).contiguous()
                _abi.check(lib.tp_rot_scale(signs.data_ptr(), self.inv_equil.data_ptr(), rs.data_ptr(), d, st),
                           "rot_scale")
                self.rot_scale = rs
            if self.mode == "cached":
                if self._w_cache is None:
                    w_rot = self.decode_rows(0, n)
                    w = torch.empty_like(w_rot)
                    _abi.check(lib.tp_fold_rows(w_rot.data_ptr(), self.rot_scale.data_ptr(), w.data_ptr(), n, d,
                                                self.block, st), "fold_rows")
                    self._w_cache = w
                    for name in ("path_packed", "member_packed", "signs_packed", "lut", "tcq_stream"):
                        setattr(self, name, None)
            elif self._native and self.tcq_stream is None:
                nbytes = lib.tp_stream_bytes(n, d, self.bits)
                out = torch.empty(nbytes, dtype=torch.uint8, device=dev)
                path = self.path_packed.contiguous()
                mem = None if self.member_packed is None else self.member_packed.contiguous()
                _abi.check(lib.tp_relayout_v2(path.data_ptr(), _abi.ptr(mem), out.data_ptr(), n, d, self.bits, st),
                           "relayout_v2")
                self.tcq_stream = out
                # the native stream replaces the format-v2 streams (like the
                # reference's triton mode frees path/member after re-packing)
                for name in ("path_packed", "member_packed", "lut"):
                    setattr(self, name, None)

    # -- decode -------------------------------------------------------------
    @torch.no_grad()
    def decode_rows(self, r0: int, r1: int) -> Tensor:
        """Decode rows [r0, r1) of the rotated weight matrix to fp16, bit-exact
        with the reference (turbopress/runtime.py:291-301)."""
        if not 0 <= r0 <= r1 <= self.out_features:
            raise ValueError(f"bad row range [{r0}, {r1})")
        d = self.in_features
        if self.tcq_stream is not None:
            _abi.require_cuda(self.tcq_stream)
            out = torch.empty(r1 - r0, d, dtype=torch.float16, device=self.tcq_stream.device)
            _abi.check(_abi.lib().tp_decode_stream(
                self.tcq_stream.data_ptr(), self.scales.data_ptr(), self.codebook.data_ptr(), out.data_ptr(),
                r0, r1, self.out_features, d, self.bits, self.n_states, _stream(out)), "decode_stream")
            return out
        if self.path_packed is None:
            raise RuntimeError("packed streams were freed (mode='cached'); decode_rows is unavailable")
        _abi.require_cuda(self.path_packed, self.scales)
        out = torch.empty(r1 - r0, d, dtype=torch.float16, device=self.path_packed.device)
        path = self.path_packed.contiguous()
        mem = None if self.member_packed is None else self.member_packed.contiguous()
        _abi.check(_abi.lib().tp_decode_rows(
            path.data_ptr(), _abi.ptr(mem), self.scales.data_ptr(), self.codebook.data_ptr(), out.data_ptr(),
            r0, r1, d, self.bits, self.n_states, _stream(out)), "decode_rows")
        return out

    # -- forward --------------------------------------------------------------
    def forward(self, x: Tensor) -> Tensor:
        if x.shape[-1] != self.in_features:
            raise ValueError(f"expected last dim {self.in_features}, got {x.shape[-1]}")
        if not x.is_cuda:
            raise RuntimeError("turbopress_b200 runs on CUDA devices only (no CPU fallback); move the input "
                               "and the module to a GPU")
        if self._needs_materialize():
            self._materialize()
        if self.mode == "cached":
            if self._w_cache is None:
                raise RuntimeError("module is not on a CUDA device; call .cuda() first")
            y = F.linear(x.to(torch.float16), self._w_cache)
            if self.bias is not None:
                y = y + self.bias
            return y.to(x.dtype)
        n, d = self.out_features, self.in_features
        flat = x.reshape(-1, d)
        if flat.dtype not in (torch.float16, torch.float32, torch.bfloat16):
            flat = flat.to(torch.float16)
        flat = flat.contiguous()
        B = flat.shape[0]
        y = torch.empty(B, n, dtype=flat.dtype, device=x.device)
        if B == 0:
            return y.reshape(*x.shape[:-1], n).to(x.dtype)
        lib = _abi.lib()
        st = _stream(flat)
        if self._native:
            _abi.require_cuda(self.tcq_stream)
            # batches of TC_MIN_BATCH and more: tcgen05 skinny GEMM; below: the fused GEMV
            use_tc = B >= TC_MIN_BATCH
            ws_bytes = (lib.tp_gemm_tc_workspace_bytes(B, n, d) if use_tc
                        else lib.tp_gemv_workspace_bytes(B, n, d, self.bits))
            ws = (WORKSPACE_TC if use_tc else WORKSPACE).get(x.device, ws_bytes)
            fn = lib.tp_tcq_gemm_tc if use_tc else lib.tp_tcq_gemv
            _abi.check(fn(
                flat.data_ptr(), _abi.dtype_code(flat.dtype), self.rot_scale.data_ptr(), self.tcq_stream.data_ptr(),
                self.scales.data_ptr(), self.codebook.data_ptr(), _abi.ptr(self.bias), y.data_ptr(),
                _abi.dtype_code(y.dtype), B, n, d, self.block, self.bits, self.n_states, ws.data_ptr(), ws.numel(),
                st), "tcq_gemm_tc" if use_tc else "tcq_gemv")
        else:
            z = rotate(flat, self.rot_scale, self.block, out_dtype=torch.float32)
            mem = None if self.member_packed is None else self.member_packed.contiguous()
            _abi.check(lib.tp_gemv_v2(
                z.data_ptr(), self.path_packed.contiguous().data_ptr(), _abi.ptr(mem), self.scales.data_ptr(),
                self.codebook.data_ptr(), _abi.ptr(self.bias), y.data_ptr(), _abi.dtype_code(y.dtype), B, n, d,
                self.bits, self.n_states, st), "gemv_v2")
        return y.reshape(*x.shape[:-1], n).to(x.dtype)

    # -- accounting -----------------------------------------------------------
    def packed_bytes(self) -> int:
        """Resident weight bytes under the current mode (turbopress/runtime.py:337-356)."""
        if self._w_cache is not None:
            total = self._w_cache.numel() * self._w_cache.element_size()
        else:
            if self.tcq_stream is not None:
                total = self.tcq_stream.numel()
            else:
                total = self.path_packed.numel()
                if self.member_packed is not None:
                    total += self.member_packed.numel()
            total += self.signs_packed.numel()
            total += 2 * self.inv_equil.numel()
            total += 2 * (self.rot_scale.numel() if self.rot_scale is not None else self.in_features)
        total += 2 * (self.scales.numel() + self.codebook.numel())
        if self.bias is not None:
            total += 2 * self.bias.numel()
        return total

    def extra_repr(self) -> str:
        return (f"in_features={self.in_features}, out_features={self.out_features}, "
                f"bits={self.bits}, n_states={self.n_states}, mode={self.mode!r}, "
                f"resident={self.packed_bytes() / 2**20:.1f} MiB "
                f"(fp16 {2 * self.in_features * self.out_features / 2**20:.1f} MiB)")


# ---------------------------------------------------------------------------
# artifact loading (format v1, turbopress/pipeline.py:917-935)
# ---------------------------------------------------------------------------
@torch.no_grad()
def v1_payload_to_packed(payload: dict, bias: Tensor | None = None, device: str = "cuda") -> dict[str, Any]:
    """Convert one format-v1 artifact matrix into a format-v2 payload on the GPU.

    Same contract as turbopress/runtime.py:417-452: the stored trellis codes,
    scales, codebook, signs and equilibration are preserved exactly; the
    flat MSB-first streams are re-packed row-aligned LE by a CUDA kernel.
    """
    dev = torch.device(device)
    if dev.type != "cuda":
        raise RuntimeError("v1_payload_to_packed runs on a CUDA device (no CPU fallback)")
    n, d, bits = int(payload["n"]), int(payload["d"]), int(payload["bits"])
    lib = _abi.lib()

    def _conv(buf, width):
        src = torch.as_tensor(buf).to(dev, torch.uint8).contiguous()
        if src.numel() * 8 < n * d * width:
            raise ValueError("v1 stream too short")
        out = torch.empty(n, -(-d * width // 8), dtype=torch.uint8, device=dev)
        _abi.check(lib.tp_v1_to_v2(src.data_ptr(), out.data_ptr(), n, d, width, _stream(out)), "v1_to_v2")
        return out

    def _conv_signs(buf):
        src = torch.as_tensor(buf).to(dev, torch.uint8).contiguous()
        out = torch.empty(1, -(-d // 8), dtype=torch.uint8, device=dev)
        _abi.check(lib.tp_v1_to_v2(src.data_ptr(), out.data_ptr(), 1, d, 1, _stream(out)), "v1_to_v2")
        return out

    equil = torch.as_tensor(payload["equil"]).to(dev).float().clamp_min(1e-12)
    return {
        "format": 2,
        "n": n,
        "d": d,
        "bits": bits,
        "n_states": int(payload["n_states"]),
        "block": int(payload["block"]),
        "path_packed": _conv(payload["path_bits"], 1),
        "member_packed": _conv(payload["member_bits"], bits - 1) if bits > 1 else None,
        "scales": torch.as_tensor(payload["scales"]).to(device=dev, dtype=torch.float16),
        "signs_packed": _conv_signs(payload["signs"]),
        "inv_equil": (1.0 / equil).to(torch.float16),
        "codebook": torch.as_tensor(payload["codebook"]).to(device=dev, dtype=torch.float16),
        "bias": None if bias is None else bias.detach().to(device=dev, dtype=torch.float16),
        "seed": 0,
    }


def _decoder_layers(model: nn.Module) -> nn.ModuleList:
    """Decoder block list of a Llama-family causal LM (turbopress/real_model.py:156-170)."""
    for path in ("model.layers", "transformer.h", "model.decoder.layers"):
        obj = model
        try:
            for attr in path.split("."):
                obj = getattr(obj, attr)
        except AttributeError:
            continue
        if isinstance(obj, nn.ModuleList) and len(obj) > 0:
            return obj
    raise ValueError(f"could not locate decoder layers on {type(model).__name__}")


# (S, generators) table written into artifacts (turbopress/pipeline.py:183)
_TRELLIS_GENERATORS = GENERATORS


@torch.no_grad()
def load_packed_model(artifact_dir, *, device: str = "cuda", mode: str = "cached"):
    """Load a TurboPress artifact directory into a packed causal LM.

    Same contract and errors as turbopress/runtime.py:455-541: every decoder
    ``nn.Linear`` becomes a :class:`PackedTCQLinear` in ``mode``; returns
    ``(model, meta)``.  Needs a CUDA device.
    """
    from pathlib import Path

    if mode not in MODES:
        raise ValueError(f"mode must be one of {MODES}, got {mode!r}")
    root = Path(artifact_dir)
    weights_path = root / "turbopress_weights.pt"
    if not weights_path.exists():
        raise FileNotFoundError(f"not a TurboPress artifact (missing {weights_path})")
    if not str(device).startswith("cuda"):
        raise RuntimeError("turbopress_b200 needs a CUDA device")
    from transformers import AutoConfig, AutoModelForCausalLM

    blob = torch.load(weights_path, map_location="cpu", weights_only=False)
    meta = dict(blob["meta"])
    quantized = blob.pop("quantized")
    extra = blob.pop("extra_state")
    del blob
    if int(meta.get("format_version", -1)) != 1:
        raise RuntimeError("expected a TurboPress format_version=1 artifact")
    n_states = int(meta["n_states"])
    if n_states not in _TRELLIS_GENERATORS or tuple(meta["generators"]) != tuple(_TRELLIS_GENERATORS[n_states]):
        raise RuntimeError("trellis generator mismatch (artifact/runtime incompatible)")

    config = AutoConfig.from_pretrained(root / "hf_config")
    prev = torch.get_default_dtype()
    torch.set_default_dtype(torch.float16)
    try:
        model = AutoModelForCausalLM.from_config(config)
    finally:
        torch.set_default_dtype(prev)
    model = model.to(dtype=torch.float16)
    _missing, unexpected = model.load_state_dict(extra, strict=False)
    del extra
    unexpected = [k for k in unexpected if not k.endswith(".weight")]
    if unexpected:
        raise RuntimeError(f"unexpected keys in artifact: {unexpected[:8]}")
    model.tie_weights()
    for key in list(quantized):
        payload = quantized.pop(key)
        if not key.endswith(".weight"):
            raise RuntimeError(f"invalid quantized key: {key}")
        module_path = key[: -len(".weight")]
        linear = model.get_submodule(module_path)
        if not isinstance(linear, nn.Linear):
            raise RuntimeError(f"{module_path} is not nn.Linear")
        bias = None if linear.bias is None else linear.bias.detach().clone()
        packed = PackedTCQLinear(v1_payload_to_packed(payload, bias, device), mode=mode)
        parent_path, leaf = module_path.rsplit(".", 1)
        setattr(model.get_submodule(parent_path), leaf, packed)
    model = model.to(device=device, dtype=torch.float16).eval()
    model.config.use_cache = True
    model.tie_weights()
    leftover = [f"layers.{i}.{name}" for i, block in enumerate(_decoder_layers(model))
                for name, mod in block.named_modules() if isinstance(mod, nn.Linear)]
    if leftover:
        raise RuntimeError(f"unconverted decoder linears remain: {leftover[:8]}")
    return model, meta

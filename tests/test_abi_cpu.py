"""CPU checks of the C-ABI boundary: the library loads and exports exactly
what ``include/turbopress_b200.h`` declares (no compute call needs a GPU)."""

import ctypes
import re
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent
HEADER = ROOT / "include" / "turbopress_b200.h"


def declared_functions() -> list[str]:
    text = re.sub(r"/\*.*?\*/", "", HEADER.read_text(), flags=re.S)
    return sorted(set(re.findall(r"\b(tp_[a-z0-9_]+)\s*\(", text)))


@pytest.fixture(scope="module")
def lib():
    from turbopress_b200 import build
    path = build.build()
    return ctypes.CDLL(str(path))


def test_header_declares_the_entry_points():
    names = declared_functions()
    for must in ("tp_tcq_gemv", "tp_decode_rows", "tp_rotate", "tp_relayout_v2", "tp_relayout_v1",
                 "tp_decode_stream", "tp_last_error", "tp_gemv_workspace_bytes", "tp_v1_to_v2"):
        assert must in names


def test_library_exports_every_declared_symbol(lib):
    for name in declared_functions():
        assert hasattr(lib, name), name


def test_binding_signatures_cover_header():
    from turbopress_b200 import _abi
    assert sorted(_abi.SIGNATURES) == declared_functions()


def test_library_exports_nothing_else(lib):
    import subprocess
    out = subprocess.run(["nm", "-D", "--defined-only", str(ROOT / "turbopress_b200" / "_lib" /
                                                             "libturbopress_b200.so")],
                         capture_output=True, text=True).stdout
    exported = sorted({ln.split()[-1] for ln in out.splitlines() if " T " in ln and ln.split()[-1].startswith("tp_")})
    assert exported == declared_functions()


def test_host_only_entry_points(lib):
    from turbopress_b200 import _abi
    L = _abi.lib()
    assert L.tp_abi_version() == 1
    # stream size is true-rate bits over the padded tile grid
    assert L.tp_stream_bytes(4096, 4096, 3) == 4096 * 4096 * 3 // 8
    assert L.tp_stream_bytes(37, 576, 4) == 48 * 768 * 4 // 8
    assert L.tp_stream_bytes(10, 10, 5) == -1
    # argument errors come back as statuses, never exceptions
    assert L.tp_pack_le(None, None, 1, 1, 1, None) == _abi.TP_ERR_ARG
    assert b"bad arguments" in L.tp_last_error()
    assert L.tp_decode_rows(None, None, None, None, None, 0, 1, 8, 9, 64, None) == _abi.TP_ERR_ARG
    assert L.tp_tcq_gemv(1, 0, 1, 1, 1, 1, None, 1, 0, 1, 16, 256, 256, 5, 64, 1, 1 << 20, None) == \
        _abi.TP_ERR_UNSUPPORTED
    assert L.tp_tcq_gemv(1, 0, 1, 16, 1, 1, None, 1, 0, 1, 16, 256, 256, 3, 12, 1, 1 << 20, None) == \
        _abi.TP_ERR_UNSUPPORTED
    # greedy LM head: argument checks happen before any device work
    assert L.tp_lm_head_workspace_bytes(8) >= 8 * 8 + 4
    assert L.tp_lm_head_argmax(None, 16, 1, 10, 8, None, 16, None, 16, 1024, None) == _abi.TP_ERR_ARG
    assert L.tp_lm_head_argmax(16, 16, 9, 10, 8, None, 16, None, 16, 1024, None) == _abi.TP_ERR_UNSUPPORTED
    assert L.tp_lm_head_argmax(16, 16, 1, 10, 12, None, 16, None, 16, 1024, None) == _abi.TP_ERR_ARG
    assert L.tp_lm_head_argmax(16, 16, 4, 10, 8192, None, 16, None, 16, 1024, None) == _abi.TP_ERR_UNSUPPORTED
    assert L.tp_lm_head_argmax(16, 17, 1, 10, 8, None, 16, None, 16, 1024, None) == _abi.TP_ERR_ALIGN
    assert L.tp_lm_head_argmax(16, 16, 1, 10, 8, None, 16, None, 16, 8, None) == _abi.TP_ERR_WORKSPACE


def test_module_rejects_cpu_forward():
    import numpy as np
    import torch

    from oracle import tcq_oracle as O
    from turbopress_b200 import PackedTCQLinear
    p = O.random_payload(32, 64, 3, 64, seed=1)
    p = {k: (torch.from_numpy(v) if isinstance(v, np.ndarray) else v) for k, v in p.items()}
    m = PackedTCQLinear(p, mode="cuda")
    with pytest.raises(ValueError):
        m(torch.randn(2, 63))
    with pytest.raises(RuntimeError):
        m(torch.randn(2, 64))
    with pytest.raises(ValueError):
        PackedTCQLinear(p, mode="warp")
    with pytest.raises(ValueError):
        PackedTCQLinear({"format": 1})

"""The allocation-free GEMV entry point gives the workspace entry point's result.

tp_tcq_gemv_noalloc exists for callers that cannot allocate device memory
(host engines that own every allocation, loops where cudaMalloc is not
allowed); it runs on scratch built into the library.  This file is named to
be collected last, so a run stopping at the first failure has already run
every other test.  It also passes alone in a fresh process.
"""

import numpy as np
import pytest
import torch

from oracle import tcq_oracle as O

pytestmark = pytest.mark.gpu

REL_L2_TOL = 1e-3  # same bound as the other GEMV parity tests


def _rel(a, b):
    return float((a.float() - b.float()).norm() / b.float().norm())


@pytest.mark.parametrize("B,n,d,bits", [(1, 2560, 9728, 3), (4, 1024, 2560, 2), (3, 777, 1000, 4)])
def test_noalloc_matches_workspace_entry_point(B, n, d, bits):
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    from turbopress_b200 import PackedTCQLinear, _abi
    L = _abi.lib()
    dev = "cuda"
    p = O.random_payload(n, d, bits, 64, seed=n + d, bias=True)
    pd = {k: (torch.from_numpy(v).to(dev) if isinstance(v, np.ndarray) else v) for k, v in p.items()}
    m = PackedTCQLinear(pd, mode="cuda")
    st = torch.cuda.current_stream().cuda_stream
    need = L.tp_gemv_workspace_bytes(B, n, d, bits)
    ws = torch.zeros(need, dtype=torch.uint8, device=dev)
    for call in range(2):
        x = torch.randn(B, d, device=dev, dtype=torch.float16)
        args = (x.data_ptr(), _abi.TP_F16, m.rot_scale.data_ptr(), m.tcq_stream.data_ptr(), m.scales.data_ptr(),
                m.codebook.data_ptr(), m.bias.data_ptr())
        y_ws = torch.empty(B, n, device=dev, dtype=torch.float16)
        y_na = torch.empty(B, n, device=dev, dtype=torch.float16)
        tail = (B, n, d, m.block, bits, 64)
        _abi.check(L.tp_tcq_gemv(*args, y_ws.data_ptr(), _abi.TP_F16, *tail, ws.data_ptr(), need, st), "tcq_gemv")
        _abi.check(L.tp_tcq_gemv_noalloc(*args, y_na.data_ptr(), _abi.TP_F16, *tail, st), "tcq_gemv_noalloc")
        torch.cuda.synchronize()
        assert _rel(y_na, y_ws) < REL_L2_TOL, call
        ref = torch.from_numpy(O.forward_fp32(p, x.cpu().numpy())).to(dev)
        assert _rel(y_na, ref) < REL_L2_TOL, call


def test_noalloc_rejects_oversized_problems():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    from turbopress_b200 import _abi
    L = _abi.lib()
    # 32 rows of a layer with d = 262144 need > 8 MiB of scratch; null data
    # pointers make sure nothing could launch even if the size guard failed
    assert L.tp_gemv_workspace_bytes(32, 4096, 262144, 2) > (8 << 20)
    st = L.tp_tcq_gemv_noalloc(None, 0, None, None, None, None, None, None, 0, 32, 4096, 262144, 65536, 2, 64,
                               None)
    assert st == _abi.TP_ERR_UNSUPPORTED
    assert b"built-in maximum" in L.tp_last_error()

"""GPU tests of the persistent decode engine (``tp_engine_run`` via
``turbopress_b200.engine.DecodeEngine``).

Each op's output is checked against the oracle's fp32 dequant-then-matmul
(``oracle.forward_fp32``) applied to the input the engine itself fed that op
(an earlier op's fp32 output for chained ops), so every op is held to the
per-layer bound of relative L2 <= 1e-3.
"""

import numpy as np
import pytest
import torch

from oracle import tcq_oracle as O

pytestmark = pytest.mark.gpu

REL_L2_TOL = 1e-3
DEV = "cuda"


def rel_l2(a, b):
    a = np.asarray(a, dtype=np.float64)
    b = np.asarray(b, dtype=np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


def to_dev(p: dict) -> dict:
    return {k: torch.from_numpy(np.ascontiguousarray(v)).to(DEV) if isinstance(v, np.ndarray) else v
            for k, v in p.items()}


@pytest.fixture(scope="module", autouse=True)
def _cuda():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")


def _module(p):
    from turbopress_b200 import PackedTCQLinear
    return PackedTCQLinear(to_dev(p), mode="cuda")


def _check_ops(eng, payloads, inputs, x_ext, outs):
    for i, (p, dep) in enumerate(zip(payloads, inputs)):
        xin = x_ext[p["d"]] if dep is None else outs[dep].cpu().numpy()
        ref = O.forward_fp32(p, xin)
        err = rel_l2(outs[i].cpu().numpy(), ref)
        assert err < REL_L2_TOL, (i, err)


@pytest.mark.parametrize("bits", [2, 3, 4])
@pytest.mark.parametrize("B", [1, 3])
def test_engine_decoder_chain(bits, B):
    """Two decoder-like layers: qkv + o (chained), gate/up + down (chained)."""
    from turbopress_b200.engine import DecodeEngine
    h, inter, q = 640, 1536, 1024
    cb = np.sort(np.random.default_rng(bits).standard_normal(1 << (bits + 1)) * 1.2)
    payloads, inputs = [], []
    seed = 100 * bits
    for _ in range(2):
        base = len(payloads)
        for n, d, dep in [(q, h, None), (256, h, None), (256, h, None), (h, q, base),
                          (inter, h, None), (inter, h, None), (h, inter, base + 4)]:
            payloads.append(O.random_payload(n, d, bits, 64, seed=seed, codebook=cb, bias=(seed % 3 == 0)))
            inputs.append(dep)
            seed += 1
    mods = [_module(p) for p in payloads]
    eng = DecodeEngine(mods, inputs, batch=B)
    rng = np.random.default_rng(B)
    x = rng.standard_normal((B, h)).astype(np.float16)
    for _ in range(2):
        outs = eng.run(torch.from_numpy(x).to(DEV))
        torch.cuda.synchronize()
        eng.check()
        _check_ops(eng, payloads, inputs, {h: x}, outs)


@pytest.mark.parametrize("n,d", [(4096, 2560), (8192, 512), (2560, 9728), (9728, 2560), (96, 200), (1024, 1),
                                 (256, 28672), (512, 8192), (300, 12288)])
def test_engine_single_op_shapes(n, d):
    from turbopress_b200.engine import DecodeEngine
    p = O.random_payload(n, d, 3, 64, seed=n + d, bias=True)
    m = _module(p)
    eng = DecodeEngine([m], [None], batch=1)
    x = np.random.default_rng(d).standard_normal((1, d)).astype(np.float16)
    xt = torch.from_numpy(x).to(DEV)
    y = eng.run(xt)[0]
    torch.cuda.synchronize()
    eng.check()
    ref = O.forward_fp32(p, x)
    assert rel_l2(y.cpu().numpy(), ref) < REL_L2_TOL
    # and against the per-call fused GEMV
    assert rel_l2(y.cpu().numpy(), m(xt.float()).cpu().numpy()) < REL_L2_TOL


def test_engine_input_dtypes():
    from turbopress_b200.engine import DecodeEngine
    p = O.random_payload(300, 1024, 3, 16, seed=7)
    m = _module(p)
    x = np.random.default_rng(0).standard_normal((2, 1024)).astype(np.float32)
    for dt in (torch.float16, torch.bfloat16, torch.float32):
        eng = DecodeEngine([m], batch=2, input_dtype=dt)
        xt = torch.from_numpy(x).to(DEV).to(dt)
        y = eng.run(xt)[0].cpu().numpy()
        eng.check()
        assert rel_l2(y, O.forward_fp32(p, xt.float().cpu().numpy())) < REL_L2_TOL, dt


def test_engine_graph_capture():
    from turbopress_b200.engine import DecodeEngine
    cb = np.sort(np.random.default_rng(1).standard_normal(16) * 1.2)
    payloads = [O.random_payload(768, 512, 3, 64, seed=s, codebook=cb) for s in range(2)]
    payloads.append(O.random_payload(512, 768, 3, 64, seed=9, codebook=cb))
    inputs = [None, None, 0]
    eng = DecodeEngine([_module(p) for p in payloads], inputs)
    x = np.random.default_rng(3).standard_normal((1, 512)).astype(np.float16)
    eng.set_input(torch.from_numpy(x).to(DEV))
    eng.run()
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    s = torch.cuda.Stream()
    with torch.cuda.stream(s):
        with torch.cuda.graph(g, stream=s):
            eng.run()
    for _ in range(3):
        g.replay()
    torch.cuda.synchronize()
    eng.check()
    _check_ops(eng, payloads, inputs, {512: x}, eng.outputs)


def test_engine_rejects():
    from turbopress_b200.engine import DecodeEngine
    p = O.random_payload(64, 256, 3, 64, seed=1)
    m = _module(p)
    with pytest.raises(ValueError):
        DecodeEngine([m, m], [None, 1])  # forward reference
    with pytest.raises(ValueError):
        DecodeEngine([m], batch=9)
    p4 = O.random_payload(64, 256, 4, 64, seed=1)
    with pytest.raises(ValueError):
        DecodeEngine([m, _module(p4)])  # mixed bit widths


@pytest.mark.parametrize("B", [1, 2])
def test_engine_wide_chain(B):
    """Llama-70B widths (rows scaled down for the oracle): q/k/v and gate/up
    read 8192-wide inputs with Hadamard block 8192, down a 28672-wide one
    (block 4096); these blocks are transformed straight from global memory.
    The 28672-wide activations fit shared memory at batch 1 only."""
    from turbopress_b200.engine import DecodeEngine
    h, inter = 8192, 28672
    cb = np.sort(np.random.default_rng(5).standard_normal(8) * 1.2)
    shapes = [(512, h, None), (128, h, None), (128, h, None), (h, 512, 0), (1024, h, 3), (1024, h, 3),
              (512, inter, None)][:7 if B == 1 else 6]
    payloads = [O.random_payload(n, d, 2, 64, seed=40 + i, codebook=cb) for i, (n, d, _) in enumerate(shapes)]
    inputs = [dep for _, _, dep in shapes]
    eng = DecodeEngine([_module(p) for p in payloads], inputs, batch=B)
    rng = np.random.default_rng(6)
    xs = {w: rng.standard_normal((B, w)).astype(np.float16) for w in ((h, inter) if B == 1 else (h,))}
    outs = eng.run([torch.from_numpy(v).to(DEV) for v in xs.values()])
    torch.cuda.synchronize()
    eng.check()
    _check_ops(eng, payloads, inputs, xs, outs)

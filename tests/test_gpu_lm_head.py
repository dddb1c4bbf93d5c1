"""GPU tests of the greedy LM head (``tp_lm_head_argmax`` via
``turbopress_b200.lm_head.GreedyLMHead``) against the oracle's float64
logits + argmax (``oracle.lm_head_argmax``).

Tolerances: logits within 1e-5 relative (fp32 accumulation of fp16
products, order differs from float64); the token must be the oracle's
argmax, or -- only where two logits are closer than that tolerance -- a
token whose float64 logit is within it of the maximum.
"""

import numpy as np
import pytest
import torch

from oracle import tcq_oracle as O

pytestmark = pytest.mark.gpu
DEV = "cuda"
TOL = 1e-5


@pytest.fixture(scope="module", autouse=True)
def _cuda():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")


def _check(x, w, tokens, best, logits=None):
    ref_tok, ref = O.lm_head_argmax(x, w)
    scale = np.abs(ref).max() + 1e-30
    for b in range(x.shape[0]):
        t = int(tokens[b])
        assert 0 <= t < w.shape[0]
        assert t == ref_tok[b] or ref[b, ref_tok[b]] - ref[b, t] <= TOL * scale, (b, t, ref_tok[b])
        assert abs(float(best[b]) - ref[b, t]) <= TOL * scale
    if logits is not None:
        err = np.abs(logits - ref).max() / scale
        assert err <= TOL, err


@pytest.mark.parametrize("V,h,B", [(5003, 2560, 1), (4096, 1024, 2), (1, 8, 1), (777, 136, 3),
                                   (20000, 2560, 4), (3000, 4096, 5), (1500, 3072, 8), (333, 8192, 3),
                                   (700, 12288, 1), (640, 6144, 4)])  # x staging at exactly 48 KB
def test_lm_head_vs_oracle(V, h, B):
    from turbopress_b200.lm_head import GreedyLMHead
    rng = np.random.default_rng(V + h + B)
    w = (rng.standard_normal((V, h)) * 0.02).astype(np.float16)
    x = rng.standard_normal((B, h)).astype(np.float16)
    head = GreedyLMHead(torch.from_numpy(w).to(DEV))
    tok, best, logits = head(torch.from_numpy(x).to(DEV), return_logits=True)
    _check(x, w, tok.cpu().numpy(), best.cpu().numpy(), logits.cpu().numpy())
    # again without logits (workspace reuse), same answer
    tok2, best2 = head(torch.from_numpy(x).to(DEV))
    assert torch.equal(tok, tok2) and torch.equal(best, best2)


def test_lm_head_ties_pick_first_index():
    from turbopress_b200.lm_head import GreedyLMHead
    rng = np.random.default_rng(0)
    V, h = 4000, 512
    w = (rng.standard_normal((V, h)) * 0.02).astype(np.float16)
    x = np.abs(rng.standard_normal((2, h))).astype(np.float16)
    w[[17, 1234, 3999]] = np.full(h, 0.05, dtype=np.float16)  # three identical winning rows
    tok, _ = GreedyLMHead(torch.from_numpy(w).to(DEV))(torch.from_numpy(x).to(DEV))
    assert tok.cpu().tolist() == [17, 17]


def test_lm_head_full_vocab_matches_torch():
    """Qwen3 vocabulary (151936 x 2560, 0.78 GB): token equal to torch's fp32 argmax."""
    from turbopress_b200.lm_head import GreedyLMHead
    g = torch.Generator(device=DEV).manual_seed(3)
    w = (torch.randn(151936, 2560, generator=g, device=DEV) * 0.02).half()
    x = torch.randn(4, 2560, generator=g, device=DEV).half()
    tok, best = GreedyLMHead(w)(x)
    ref = x.double() @ w.double().T
    mx = ref.max(dim=-1).values
    picked = ref.gather(1, tok[:, None])[:, 0]
    assert torch.all(mx - picked <= TOL * ref.abs().max())
    assert torch.allclose(best.double(), picked, rtol=0, atol=float(TOL * ref.abs().max()))


def test_lm_head_in_cuda_graph():
    from turbopress_b200.lm_head import GreedyLMHead
    rng = np.random.default_rng(9)
    w = (rng.standard_normal((6000, 1024)) * 0.02).astype(np.float16)
    x = torch.from_numpy(rng.standard_normal((1, 1024)).astype(np.float16)).to(DEV)
    head = GreedyLMHead(torch.from_numpy(w).to(DEV))
    head(x)
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    s = torch.cuda.Stream()
    with torch.cuda.stream(s):
        with torch.cuda.graph(g, stream=s):
            tok, best = head(x)
    for _ in range(3):
        g.replay()
    torch.cuda.synchronize()
    _check(x.cpu().numpy(), w, tok.cpu().numpy(), best.cpu().numpy())


def test_lm_head_rejects():
    from turbopress_b200.lm_head import GreedyLMHead
    head = GreedyLMHead(torch.zeros(64, 16, dtype=torch.float16, device=DEV))
    with pytest.raises(ValueError):
        head(torch.zeros(9, 16, dtype=torch.float16, device=DEV))
    with pytest.raises(ValueError):
        head(torch.zeros(1, 24, dtype=torch.float16, device=DEV))
    with pytest.raises(RuntimeError):  # B*h above the shared-memory staging limit
        GreedyLMHead(torch.zeros(64, 25600, dtype=torch.float16, device=DEV))(
            torch.zeros(2, 25600, dtype=torch.float16, device=DEV))

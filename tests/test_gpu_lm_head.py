"""GPU tests of the greedy LM head (``tp_lm_head_argmax`` via
``turbopress_b200.lm_head.GreedyLMHead``) against the oracle's logits and
fp16-rounded argmax (``oracle.lm_head_argmax``; the reference's logits are
fp16 F.linear outputs).

Tolerances: logits within 1e-5 relative (fp32 accumulation of fp16
products, order differs from float64).  The token must be the oracle's
argmax, or -- only where the fp32 and float64 values of a logit round to
neighbouring fp16 values -- a token whose fp16 logit is within one fp16 ulp
of the oracle's maximum; the returned best logit is that token's fp16 value.
"""

import numpy as np
import pytest
import torch

from oracle import tcq_oracle as O

pytestmark = pytest.mark.gpu
DEV = "cuda"
TOL = 1e-5


def _ulp16(v):
    return float(np.spacing(np.float16(abs(v)))) if np.isfinite(v) else 0.0


@pytest.fixture(scope="module", autouse=True)
def _cuda():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")


def _check(x, w, tokens, best, logits=None):
    ref_tok, ref = O.lm_head_argmax(x, w)
    scale = np.abs(ref).max() + 1e-30
    r16 = ref.astype(np.float16).astype(np.float64)
    for b in range(x.shape[0]):
        t = int(tokens[b])
        assert 0 <= t < w.shape[0]
        mx = r16[b, ref_tok[b]]
        assert t == ref_tok[b] or r16[b, t] >= mx - _ulp16(mx), (b, t, ref_tok[b])
        assert abs(float(best[b]) - r16[b, t]) <= _ulp16(r16[b, t]), (float(best[b]), r16[b, t])
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
    """Qwen3 vocabulary (151936 x 2560, 0.78 GB): the token of torch's fp16
    F.linear + argmax (fp32 accumulation), unless the two sides' values round
    to neighbouring fp16 numbers."""
    from turbopress_b200.lm_head import GreedyLMHead
    g = torch.Generator(device=DEV).manual_seed(3)
    w = (torch.randn(151936, 2560, generator=g, device=DEV) * 0.02).half()
    x = torch.randn(4, 2560, generator=g, device=DEV).half()
    tok, best = GreedyLMHead(w)(x)
    prev = torch.backends.cuda.matmul.allow_fp16_reduced_precision_reduction
    torch.backends.cuda.matmul.allow_fp16_reduced_precision_reduction = False
    try:
        ref16 = torch.nn.functional.linear(x, w)  # fp16 logits, as the reference's model returns them
    finally:
        torch.backends.cuda.matmul.allow_fp16_reduced_precision_reduction = prev
    ref_tok = ref16.argmax(-1)
    mx = ref16.gather(1, ref_tok[:, None])[:, 0].float()
    picked = ref16.gather(1, tok[:, None])[:, 0].float()
    ulp = torch.tensor([_ulp16(float(v)) for v in mx], device=DEV)
    assert torch.all((tok == ref_tok) | (picked >= mx - ulp))
    assert torch.all((best - picked).abs() <= ulp)


def test_lm_head_ties_after_fp16_rounding_pick_first_index():
    """Logits that differ in fp32 but round to the same fp16 value tie, and
    the first index wins (torch.argmax over the reference's fp16 logits)."""
    from turbopress_b200.lm_head import GreedyLMHead
    V, h = 2048, 64
    rng = np.random.default_rng(5)
    w = (rng.standard_normal((V, h)) * 0.02).astype(np.float16)
    x = np.zeros((2, h), dtype=np.float16)
    x[:, 0] = 1.0
    x[:, 1] = 2.0 ** -14  # below half an fp16 ulp of 1.0
    w[:, :2] = 0
    w[300, 0] = 1.0  # logit 1.0
    w[900, 0] = 1.0
    w[900, 1] = 1.0  # logit 1 + 2^-14 in fp32, 1.0 in fp16
    tok, best = GreedyLMHead(torch.from_numpy(w).to(DEV))(torch.from_numpy(x).to(DEV))
    assert tok.cpu().tolist() == [300, 300]
    assert best.cpu().tolist() == [1.0, 1.0]
    ref16 = torch.nn.functional.linear(torch.from_numpy(x).to(DEV), torch.from_numpy(w).to(DEV))
    assert ref16.argmax(-1).cpu().tolist() == [300, 300]


def test_lm_head_nan_logit_wins():
    """torch.argmax takes a NaN as the maximum (first NaN index)."""
    from turbopress_b200.lm_head import GreedyLMHead
    rng = np.random.default_rng(6)
    w = (rng.standard_normal((1000, 128)) * 0.02).astype(np.float16)
    x = rng.standard_normal((1, 128)).astype(np.float16)
    w[700, 3] = np.nan
    w[40, 9] = np.nan
    tok, _ = GreedyLMHead(torch.from_numpy(w).to(DEV))(torch.from_numpy(x).to(DEV))
    assert tok.cpu().tolist() == [40]
    assert O.lm_head_argmax(x, w)[0].tolist() == [40]


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

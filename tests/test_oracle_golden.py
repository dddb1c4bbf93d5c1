"""Pin the CPU oracle to the reference's own outputs (golden fixtures).

CPU-only.  Every check here compares ``oracle/tcq_oracle.py`` with values the
reference produced (``tests/golden/make_golden.py``).
"""

import hashlib

import numpy as np
import pytest

from oracle import tcq_oracle as O
from tests.conftest import load_golden, payload_from

LAYERS = ("c1", "t256", "b16", "b16w3", "s8", "w4", "w1", "q4b")


def rel_l2(a, b):
    a = np.asarray(a, dtype=np.float64)
    b = np.asarray(b, dtype=np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


@pytest.mark.parametrize("width", [1, 2, 3, 5, 8])
def test_pack_le_matches_reference(width):
    g = load_golden("bitpack")
    vals = g[f"w{width}_vals"]
    packed = O.pack_le(vals, width)
    assert packed.shape == (5, -(-77 * width // 8))
    assert np.array_equal(packed, g[f"w{width}_packed"])
    assert np.array_equal(O.unpack_le(packed, 77, width), vals)


def test_v1_flat_packing_matches_reference():
    g = load_golden("bitpack")
    assert np.array_equal(O.pack_bits_v1(np.array([5, 1], np.uint8), 3), g["v1_pack_51_w3"])
    assert int(g["v1_pack_51_w3"][0]) == 176
    assert np.array_equal(O.pack_bits_v1(g["v1_vals"], 3), g["v1_packed_w3"])
    assert np.array_equal(O.unpack_bits_v1(g["v1_packed_w3"], 333, 3), g["v1_vals"])


@pytest.mark.parametrize("s", [4, 8, 16, 64])
def test_trellis_tables_match_reference(s):
    g = load_golden("bitpack")
    assert np.array_equal(O.subset_table(s), g[f"subset_table{s}"])
    assert np.array_equal(O.subset_lut(s), g[f"lut{s}"])


@pytest.mark.parametrize("s", [4, 8, 16, 64])
@pytest.mark.parametrize("bits", [1, 2, 3, 4])
def test_window_and_sequential_decode_match_encoder(s, bits):
    g = load_golden("encoder")
    key = f"s{s}_b{bits}"
    path, member, levels = g[f"{key}_path"], g[f"{key}_member"], g[f"{key}_levels"]
    assert np.array_equal(O.window_decode_levels(path, member, s), levels)
    assert np.array_equal(O.sequential_decode_levels(path, member, s), levels)


@pytest.mark.parametrize("name", LAYERS)
def test_decode_rows_bit_exact(name):
    g = load_golden("layers")
    p = payload_from(g, f"{name}_")
    w = O.decode_rows(p)
    assert w.dtype == np.float16
    assert hashlib.sha256(w.tobytes()).digest() == g[f"{name}_w_sha256"].tobytes()
    assert np.array_equal(w[:4].view(np.uint16), g[f"{name}_w_rows0_4"].view(np.uint16))
    if f"{name}_w" in g:
        assert np.array_equal(w.view(np.uint16), g[f"{name}_w"].view(np.uint16))


@pytest.mark.parametrize("name", LAYERS)
def test_rot_scale_and_rotation_match_reference(name):
    g = load_golden("layers")
    p = payload_from(g, f"{name}_")
    rs = O.rot_scale(p)
    assert np.array_equal(rs.view(np.uint16), g[f"{name}_rot_scale"].view(np.uint16))
    z = O.rotate_activations(g[f"{name}_x"], rs, p["block"])
    assert np.array_equal(z, g[f"{name}_z"])


@pytest.mark.parametrize("name", LAYERS)
def test_forward_fp32_matches_reference_tiled(name):
    g = load_golden("layers")
    p = payload_from(g, f"{name}_")
    y = O.forward_fp32(p, g[f"{name}_x"])
    ref = g[f"{name}_y_tiled"]
    assert y.shape == ref.shape
    assert rel_l2(y, ref) < 1e-6


@pytest.mark.parametrize("name", LAYERS)
def test_cached_fold_matches_reference(name):
    g = load_golden("layers")
    p = payload_from(g, f"{name}_")
    w16 = O.fold_original_basis(p).astype(np.float16)
    if f"{name}_cache" in g:
        ref = g[f"{name}_cache"].astype(np.float32)
        assert rel_l2(w16.astype(np.float32), ref) < 1e-3
    y = g[f"{name}_x"].astype(np.float32) @ w16.astype(np.float32).T
    if p["bias"] is not None:
        y = y + p["bias"].astype(np.float32)
    assert rel_l2(y, g[f"{name}_y_cached"]) < 1e-3


def test_fwht_matches_reference():
    g = load_golden("fwht")
    keys = sorted({k.rsplit("_", 1)[0] for k in g})
    assert len(keys) >= 10
    for key in keys:
        block = int(key.split("_b")[1])
        z = O.rotate_activations(g[f"{key}_x"], g[f"{key}_rs"], block)
        assert np.array_equal(z, g[f"{key}_z"]), key


def test_fwht_equals_dense_sylvester():
    # hadamard.py:18-26 in the reference tests: FWHT == H_d / sqrt(d)
    for d in (2, 8, 64):
        h = np.array([[1.0]])
        while h.shape[0] < d:
            h = np.block([[h, h], [h, -h]])
        x = np.random.default_rng(d).standard_normal((3, d))
        assert np.allclose(O.fwht(x), x @ h.T / np.sqrt(d))


@pytest.mark.parametrize("bits", [2, 3, 4])
def test_v1_conversion_matches_reference(bits):
    g = load_golden("v1")
    key = f"v1b{bits}"
    pl = {k: int(g[f"{key}_{k}"]) for k in ("n", "d", "block", "bits", "n_states")}
    for k in ("path_bits", "member_bits", "scales", "signs", "equil", "codebook"):
        pl[k] = g.get(f"{key}_{k}")
    v2 = O.v1_to_v2(pl, g.get(f"{key}_bias"))
    ref = payload_from(g, f"{key}_v2_")
    for k in ("path_packed", "member_packed", "scales", "signs_packed", "inv_equil", "codebook", "bias"):
        if ref[k] is None:
            assert v2[k] is None
        else:
            assert np.array_equal(np.asarray(v2[k]).view(np.uint8), np.asarray(ref[k]).view(np.uint8)), k
    w = O.decode_rows(v2)
    assert np.array_equal(w.view(np.uint16), g[f"{key}_v2_decoded"].view(np.uint16))
    # the artifact contract: decoded + rotated back equals w_hat (test_tcq_ldlq.py:98-126)
    w_orig = O.fold_original_basis(v2)
    assert np.allclose(w_orig, g[f"{key}_w_hat"], atol=2e-3)


def test_bit_sliced_taps_equal_window_decode():
    """The kernel's GF(2) convolution form of the subset decode (taps from
    the generator polynomials) equals the reference window decode."""
    g = load_golden("encoder")
    for s in (4, 8, 16, 64):
        m = s.bit_length() - 1
        g0, g1 = O.GENERATORS[s]
        taps = []
        for gen in (g0, g1):
            # window bit j holds b_{t-m+j}; the generator bit for b_t is bit m,
            # for b_{t-1-k} bit k, so window bit j<m maps to generator bit m-1-j.
            taps.append([j for j in range(m + 1) if (gen >> (m if j == m else m - 1 - j)) & 1])
        for bits in (1, 2, 3, 4):
            key = f"s{s}_b{bits}"
            path = g[f"{key}_path"].astype(np.int64)
            pad = np.pad(path, ((0, 0), (m, 0)))
            d = path.shape[1]
            sub = []
            for t in taps:
                acc = np.zeros_like(path)
                for j in t:
                    acc ^= pad[:, j:j + d]
                sub.append(acc)
            lv = g[f"{key}_member"].astype(np.int64) * 4 + (sub[1] << 1 | sub[0])
            assert np.array_equal(lv.astype(np.uint8), g[f"{key}_levels"])


def test_oracle_lm_head_argmax_first_index_on_ties():
    w = np.zeros((5, 8), dtype=np.float16)
    w[1] = w[3] = 1.0
    x = np.ones((2, 8), dtype=np.float16)
    tok, logits = O.lm_head_argmax(x, w)
    assert tok.tolist() == [1, 1] and logits.shape == (2, 5) and logits[0, 3] == 8.0


@pytest.mark.parametrize("name", LAYERS)
def test_torch_cpu_restatement_matches_reference(name):
    """The timed CPU baseline (oracle/torch_cpu.py): bit-exact dequant and the
    reference's tiled / cached outputs."""
    import torch

    from oracle import torch_cpu as T

    g = load_golden("layers")
    p = payload_from(g, f"{name}_")
    w = T.decode_rows(p, 0, int(p["n"])).numpy()
    assert hashlib.sha256(w.tobytes()).digest() == g[f"{name}_w_sha256"].tobytes()
    x = torch.from_numpy(g[f"{name}_x"])
    y = T.tiled_forward(p, x, T.rot_scale(p), tile_rows=256).numpy()
    assert rel_l2(y, g[f"{name}_y_tiled"]) < 1e-5
    yc = T.cached_forward(T.cached_weight(p), x).numpy()
    if p["bias"] is not None:
        yc = yc + p["bias"].astype(np.float32)
    assert rel_l2(yc, g[f"{name}_y_cached"]) < 1e-3

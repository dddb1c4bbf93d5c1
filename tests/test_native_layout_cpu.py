"""CPU check of the native stream layout and the kernel's decode algorithm.

The word-level model in ``tests/native_layout_model.py`` restates the
bit manipulations of the CUDA decoder; these tests pin it to the oracle
(and therefore to the reference) without a GPU.
"""

import numpy as np
import pytest

from oracle import tcq_oracle as O
from tests import native_layout_model as NL
from tests.conftest import load_golden


def test_zperm_is_a_permutation():
    pos = sorted(NL.zperm_pos(c) for c in range(32))
    assert pos == list(range(32))


@pytest.mark.parametrize("bits", [2, 3, 4])
def test_member_bit_positions_are_distinct(bits):
    seen = set()
    for lc in range(32):
        for mb in range(bits - 1):
            key = NL.member_bit_pos(bits, lc, mb)
            assert key not in seen
            seen.add(key)
    assert len(seen) == 32 * (bits - 1)


@pytest.mark.parametrize("s", [4, 8, 16, 64])
@pytest.mark.parametrize("bits", [1, 2, 3, 4])
def test_native_decode_matches_encoder_levels(s, bits):
    g = load_golden("encoder")
    key = f"s{s}_b{bits}"
    lv = NL.decode_levels_native(g[f"{key}_path"], g[f"{key}_member"], bits, s)
    assert np.array_equal(lv, g[f"{key}_levels"].astype(np.int64))


@pytest.mark.parametrize("bits,s,n,d", [(3, 64, 19, 300), (2, 16, 17, 257), (4, 64, 5, 520), (1, 8, 3, 64)])
def test_native_decode_random_ragged(bits, s, n, d):
    p = O.random_payload(n, d, bits, s, seed=bits * 100 + d)
    path = O.unpack_le(p["path_packed"], d, 1)
    member = O.unpack_le(p["member_packed"], d, bits - 1) if bits > 1 else np.zeros_like(path)
    lv = NL.decode_levels_native(path, member, bits, s)
    assert np.array_equal(lv, O.window_decode_levels(path, member, s).astype(np.int64))


@pytest.mark.parametrize("name", ["t256", "b16", "w4", "w1"])
def test_native_gemv_model_matches_oracle(name):
    from tests.conftest import payload_from
    g = load_golden("layers")
    p = payload_from(g, f"{name}_")
    x = g[f"{name}_x"]
    y = NL.gemv_native(p, x)
    ref = O.forward_fp32(p, x)
    rel = np.linalg.norm(y - ref) / np.linalg.norm(ref)
    assert rel < 1e-3

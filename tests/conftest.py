import sys
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parent.parent
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))

GOLDEN = Path(__file__).resolve().parent / "golden"


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")


def load_golden(name: str) -> dict:
    with np.load(GOLDEN / f"{name}.npz") as f:
        return {k: f[k] for k in f.files}


def payload_from(g: dict, prefix: str) -> dict:
    """Rebuild a format-v2 payload dict (numpy arrays) from a golden file."""
    p = {"format": 2}
    for k in ("n", "d", "bits", "n_states", "block", "seed"):
        p[k] = int(g[f"{prefix}{k}"])
    for k in ("path_packed", "member_packed", "scales", "signs_packed", "inv_equil", "codebook", "bias"):
        p[k] = g.get(f"{prefix}{k}")
    return p


@pytest.fixture(scope="session")
def golden():
    return load_golden

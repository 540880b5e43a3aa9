import json
import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
GOLDEN = os.path.join(ROOT, "tests", "golden")
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200, sm_100a)")


@pytest.fixture(scope="session")
def golden_dir():
    return GOLDEN


@pytest.fixture(scope="session")
def pattern_small():
    return dict(np.load(os.path.join(GOLDEN, "pattern_small.npz")))


@pytest.fixture(scope="session")
def pattern_digests():
    with open(os.path.join(GOLDEN, "pattern_digests.json")) as f:
        return json.load(f)


@pytest.fixture(scope="session")
def naive_small():
    with open(os.path.join(GOLDEN, "naive_small.json")) as f:
        meta = json.load(f)
    return meta, dict(np.load(os.path.join(GOLDEN, "naive_small.npz")))


@pytest.fixture(scope="session")
def holes_cases():
    with open(os.path.join(GOLDEN, "holes.json")) as f:
        return json.load(f)


@pytest.fixture(scope="session")
def c1_rows():
    return dict(np.load(os.path.join(GOLDEN, "c1_rows.npz")))


def parse_key(key: str):
    """'L256_H4_w16_nl4_l3' -> (256, 4, 16, 4, 3)."""
    parts = key.split("_")
    return tuple(int(p.lstrip("LHwnl")) for p in parts)


@pytest.fixture(scope="session")
def esa():
    import elastic_sparse_attention_b200 as mod
    return mod

import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (runs the CUDA library)")
    config.addinivalue_line("markers", "slow: takes more than a few seconds")


@pytest.fixture(scope="session")
def golden_ops():
    import numpy as np

    return dict(np.load(os.path.join(ROOT, "tests", "golden", "ops.npz")))


@pytest.fixture(scope="session")
def tiny_model_dir():
    """The seeded two-layer checkpoint behind tests/golden/tiny_model.npz,
    regenerated and checked against the committed sha256."""
    import json

    from titania_b200 import synth

    with open(os.path.join(ROOT, "tests", "golden", "tiny_model.json")) as fh:
        meta = json.load(fh)
    d = os.path.join(ROOT, "_build", "golden-tiny")
    sha_file = os.path.join(d, "SHA256")
    if not os.path.exists(sha_file) or open(sha_file).read().strip() != meta["sha256"]:
        sha = synth.write_model(d, synth.TINY, seed=meta["seed"])
        assert sha == meta["sha256"], "the seeded generator no longer reproduces the golden checkpoint"
    return d


def close(actual, expected, rel, abs_):
    """Asserts |actual - expected| <= abs_ + rel * |expected| elementwise."""
    import numpy as np

    actual = np.asarray(actual, dtype=np.float64)
    expected = np.asarray(expected, dtype=np.float64)
    assert actual.shape == expected.shape, (actual.shape, expected.shape)
    err = np.abs(actual - expected)
    tol = abs_ + rel * np.abs(expected)
    bad = np.flatnonzero(err > tol)
    assert bad.size == 0, (f"{bad.size}/{actual.size} elements out of tolerance; first at {bad[0]}: "
                           f"got {actual.flat[bad[0]]}, expected {expected.flat[bad[0]]}; "
                           f"max err {err.max():.3g}")


@pytest.fixture(scope="session")
def b200():
    """The B200 device; the CUDA library must be built (no fallback)."""
    import titania_b200 as tb

    return tb.B200(0)

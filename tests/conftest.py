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

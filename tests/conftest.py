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
    config.addinivalue_line("markers", "slow: takes more than a few seconds on CPU")


def golden(name):
    return np.load(os.path.join(GOLDEN, name))


@pytest.fixture(scope="session")
def golden_models():
    import json
    with open(os.path.join(GOLDEN, "models.json")) as f:
        return json.load(f)


@pytest.fixture(scope="session")
def model_dirs(tmp_path_factory, golden_models):
    """Shard directories of the golden models, written by this repo's writer
    from the same seeded tensors the fixtures were generated from."""
    from androidllm_b200 import shard, synth
    root = tmp_path_factory.mktemp("models")
    dirs = {}
    for name, rec in golden_models.items():
        d = str(root / name)
        shard.shard_from_tensors(synth.synth_tensors(rec["canon"], seed=rec["seed"]),
                                 rec["canon"], d, **rec["shard"])
        dirs[name] = d
        if name in ("toy", "toyu"):
            shard.prefix_draft(d, str(root / (name + "_draft")), 2)
            dirs[name + "_draft"] = str(root / (name + "_draft"))
    return dirs

import glob
import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
GOLDEN = os.path.join(ROOT, "tests", "golden")
sys.path.insert(0, ROOT)
sys.path.insert(0, os.path.join(ROOT, "oracle"))
sys.path.insert(0, GOLDEN)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100a) GPU")


def golden_names():
    return sorted(os.path.basename(p)[:-4] for p in glob.glob(os.path.join(GOLDEN, "*.npz")))


def load_golden(name):
    """Fixture outputs plus its regenerated inputs (X, label CSR), digest-checked."""
    from filtervectorcode_refactor_b200 import datasets
    from make_golden import digest

    g = dict(np.load(os.path.join(GOLDEN, name + ".npz")))
    if "X" not in g:
        c = datasets.make_config(int(g["cfg"]), seed=int(g["seed"]), n=int(g["n"]))
        g["X"], g["label_offsets"], g["labels"] = c["X"], c["label_offsets"], c["labels"]
    assert digest(g["X"], g["label_offsets"], g["labels"]) == str(g["input_digest"]), \
        f"{name}: regenerated inputs differ from the ones the fixture was made from"
    g["k"] = int(g["k"])
    G = g["group_first"].shape[0] - 2
    ranges = np.zeros(2 * (G + 1), dtype=np.uint32)
    ranges[2::2] = g["group_first"][1:G + 1]
    ranges[3::2] = g["group_first"][2:G + 2]
    g["group_ranges"] = ranges
    g["num_groups"] = G
    g["Xr"] = np.ascontiguousarray(g["X"][g["new_to_old"]])
    return g


@pytest.fixture(params=golden_names())
def golden(request):
    return load_golden(request.param)


def have_gpu():
    try:
        import torch
        return torch.cuda.is_available()
    except Exception:
        return False

import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)
GOLDEN = os.path.join(ROOT, "tests", "golden")


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200)")


def pytest_collection_modifyitems(config, items):
    try:
        import torch
        has_gpu = torch.cuda.is_available()
    except Exception:  # pragma: no cover
        has_gpu = False
    if has_gpu:
        return
    skip = pytest.mark.skip(reason="no CUDA device in this container")
    for it in items:
        if "gpu" in it.keywords:
            it.add_marker(skip)


@pytest.fixture(scope="session")
def golden():
    def load(name):
        return np.load(os.path.join(GOLDEN, name))
    return load


@pytest.fixture(scope="session")
def k3():
    import __graft_entry__ as ge
    return ge.load_package()


@pytest.fixture(scope="session")
def ora():
    from oracle import oracle
    return oracle


def maxrel(got, want):
    """The reference's own agreement metric, max|got-want| / max|want|
    (tests/unit/test_expert.c:214-220 of the reference)."""
    got = np.asarray(got, np.float64)
    want = np.asarray(want, np.float64)
    den = np.abs(want).max()
    return float(np.abs(got - want).max() / den) if den > 0 else float(np.abs(got).max())


@pytest.fixture(scope="session")
def golden_gen():
    """tests/golden/make_golden.py as a module: the seeded cases its fixtures were made from
    (it reads the reference tree only when run as a script)."""
    import importlib.util
    spec = importlib.util.spec_from_file_location("make_golden", os.path.join(GOLDEN, "make_golden.py"))
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def latent_layer_from_npz(f):
    """A latent layer dict (oracle.moe_latent form) from moe_latent_fixture.npz."""
    skip = ("x", "want", "ref_out", "ref_idx", "ref_wt")
    return {k: (f[k] if f[k].ndim else f[k].item()) for k in f.files if k not in skip}

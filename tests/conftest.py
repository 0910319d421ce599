import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)
sys.path.insert(0, os.path.join(ROOT, "tests", "golden"))

GOLDEN = os.path.join(ROOT, "tests", "golden", "golden.npz")


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200); runs the sm_100a kernels")


@pytest.fixture(scope="session")
def golden():
    return np.load(GOLDEN)


@pytest.fixture(scope="session")
def mk():
    import malkin_b200
    return malkin_b200


@pytest.fixture(scope="session")
def oracle():
    from oracle import Oracle
    return Oracle()


@pytest.fixture(scope="session")
def ref():
    from oracle import Ref
    why = Ref.available()
    if why:
        pytest.skip(f"reference CPU path unavailable here: {why}")
    return Ref()


@pytest.fixture(scope="session")
def model_paths(tmp_path_factory, mk):
    """The golden model specs, written by the product's synthetic GGUF writer."""
    from make_golden import SPECS
    d = tmp_path_factory.mktemp("models")
    out = {}
    for name, spec in SPECS.items():
        out[name] = mk.synth_gguf(str(d / f"{name}.gguf"), **spec)
    return out


@pytest.fixture(scope="session")
def torch_cuda():
    import torch
    if not torch.cuda.is_available():
        pytest.fail("GPU test on a machine without CUDA")
    torch.cuda.init()
    return torch

import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (runs the CUDA library)")
    # GB_REQUIRE_REF=1: the reference checker (oracle/_ref/libref.so, built
    # from the reference sources) must be present, so the cases that compare
    # against it fail loudly instead of skipping on a machine without it
    if os.environ.get("GB_REQUIRE_REF") == "1":
        from oracle import oracle as O
        if not O.ref_available():
            raise pytest.UsageError("GB_REQUIRE_REF=1 but oracle/_ref/libref.so is absent "
                                    "(build it with make -C oracle REF=<reference checkout>)")


@pytest.fixture(scope="session")
def golden():
    import numpy as np
    return np.load(os.path.join(ROOT, "tests", "golden", "golden.npz"))


@pytest.fixture(scope="session")
def oracle():
    from oracle import oracle as O
    O.lib()
    return O


@pytest.fixture(scope="session")
def gb():
    import guanaco_b200 as G
    G.lib()
    return G


@pytest.fixture(scope="session")
def cuda():
    import torch
    assert torch.cuda.is_available(), "GPU tests need a CUDA device"
    torch.cuda.init()
    return torch

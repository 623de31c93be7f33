import os
import sys

import numpy as np
import pytest

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
for p in (REPO, os.path.join(REPO, "oracle"), os.path.join(REPO, "infer-llm_b200"), os.path.join(REPO, "tests", "golden")):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100a) GPU")


@pytest.fixture(scope="session")
def port():
    import oracle
    return oracle.Port()


@pytest.fixture(scope="session")
def ref():
    import oracle
    if not oracle.Ref.available():
        pytest.skip("reference engine not built here (make -C oracle ref REF=...)")
    return oracle.Ref()


@pytest.fixture(scope="session")
def golden():
    return np.load(os.path.join(REPO, "tests", "golden", "reference_cpu.npz"))


@pytest.fixture(scope="session")
def inputs():
    from make_golden import op_inputs
    return op_inputs()


def rel_err(got, want, exact=None):
    """max_i |got - want| / (|want_i| + s), s = RMS of the exact result.

    The floor s makes the bound meaningful for outputs near zero, where a plain
    relative error of two correctly rounded F32 dot products is unbounded.
    """
    got = np.asarray(got, np.float64)
    want = np.asarray(want, np.float64)
    ex = want if exact is None else np.asarray(exact, np.float64)
    s = np.sqrt(np.mean(ex * ex)) + 1e-30
    return float(np.max(np.abs(got - want) / (np.abs(want) + s)))


@pytest.fixture(scope="session")
def cuda():
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    import b200infer
    b200infer.lib()  # loads the in-tree .so or raises
    return torch.device("cuda:0")

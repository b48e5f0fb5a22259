import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")
    config.addinivalue_line("markers", "slow: takes more than a few seconds on CPU")


GOLDEN = os.path.join(ROOT, "tests", "golden", "pager_golden.npz")


@pytest.fixture(scope="session")
def golden():
    import numpy as np
    z = np.load(GOLDEN)
    names = [str(n) for n in z["names"]]
    cases = {}
    for n in names:
        cases[n] = {k.split("/", 1)[1]: z[k] for k in z.files if k.startswith(n + "/")}
    return cases


def split_forwards(case):
    """Per-forward [T,k] id arrays of a golden case."""
    import numpy as np
    ids = case["ids"]
    offs = np.concatenate([[0], np.cumsum(case["T"])])
    return [ids[offs[i]:offs[i + 1]] for i in range(len(case["T"]))], offs

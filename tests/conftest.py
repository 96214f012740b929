"""pytest configuration: the `gpu` marker, import paths, and built artefacts.

`-m "not gpu"` runs on a CPU-only machine (oracle, host logic, C-ABI symbol
checks, gloo multi-process tests); `-m gpu` runs the CUDA parity tests on a B200.
"""
import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200, sm_100a)")


@pytest.fixture(scope="session")
def oracle():
    from oracle import oracle as O
    O.lib()  # builds oracle/libkt_oracle.so with gcc if it is missing
    return O


@pytest.fixture(scope="session")
def golden():
    import numpy as np
    path = os.path.join(ROOT, "tests", "golden", "quantized_path.npz")
    with np.load(path) as z:
        return {k: z[k] for k in z.files}


@pytest.fixture(scope="session")
def kt():
    """The product package with its CUDA library (built in-tree if missing)."""
    from kotensor_b200 import build_ext
    if not os.path.exists(build_ext.LIB):
        build_ext.build()
    import kotensor_b200
    kotensor_b200.load_library()
    return kotensor_b200

import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs an sm_100 GPU (runs the CUDA kernels)")
    config.addinivalue_line("markers", "slow: long-running CPU check")


@pytest.fixture(scope="session")
def oracle():
    from oracle.oracle import Oracle
    return Oracle()


@pytest.fixture(scope="session")
def reference():
    from oracle.oracle import Reference, build_reference, reference_path
    if not os.path.exists(reference_path()):
        build_reference()
    if not os.path.exists(reference_path()):
        pytest.skip("reference CPU engine not built (oracle/_ref); golden fixtures cover this case")
    return Reference()


@pytest.fixture(scope="session")
def q3():
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no GPU")
    from metalqwen3_b200.build import build_library, library_path
    if not os.path.exists(library_path()):
        build_library()
    from metalqwen3_b200.q3cu import Q3CU
    ctx = Q3CU(0)
    yield ctx
    ctx.close()

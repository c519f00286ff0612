import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
for p in (ROOT, os.path.join(ROOT, "oracle")):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200); run with -m gpu")
    config.addinivalue_line("markers", "slow: long-running parity case")


@pytest.fixture(scope="session")
def oracle():
    import py_oracle
    py_oracle.build()
    return py_oracle


@pytest.fixture(scope="session")
def gpu_ctx():
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from qx_b200 import Context
    ctx = Context(0)
    # run on torch's stream so torch-made inputs/outputs are ordered with our kernels
    ctx.set_stream(torch.cuda.current_stream())
    yield ctx
    ctx.close()

import os
import sys

import pytest
import torch

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = os.path.join(REPO, "vit-engine-cuda_b200")
for p in (PKG, REPO):
    if p not in sys.path:
        sys.path.insert(0, p)

# Parity is measured against FP32 with TF32 disabled everywhere (the reference's
# tests do the same, e.g. tests/test_qkv.py:6-7 of the reference project).
torch.backends.cuda.matmul.allow_tf32 = False
torch.backends.cudnn.allow_tf32 = False


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA sm_100a device (B200)")


@pytest.fixture(scope="session")
def cuda():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    torch.cuda.init()
    return torch.device("cuda", torch.cuda.current_device())


@pytest.fixture(scope="session")
def vlib(cuda):
    from vit_cuda import _lib
    _lib.check(_lib.lib.vitb200_init(), "vitb200_init")
    return _lib


@pytest.fixture(autouse=True)
def _no_device_errors(request):
    """Every GPU test ends with the device error word clear: no kernel gave up
    on a bounded wait."""
    yield
    if request.node.get_closest_marker("gpu") and torch.cuda.is_available():
        from vit_cuda import _lib
        code = _lib.device_error(clear=True)
        assert code == 0, f"a kernel reported device error code {code}"

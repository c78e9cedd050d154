import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent
for p in (ROOT, ROOT / "python-gen-worker_b200"):
    if str(p) not in sys.path:
        sys.path.insert(0, str(p))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100) GPU and the built libgwb200.so")


@pytest.fixture(scope="session")
def cuda_ready():
    import torch
    from gen_worker_b200 import native

    if not torch.cuda.is_available():
        pytest.fail("gpu test selected on a machine without CUDA")
    reason = native.extension_reason()
    assert reason is None, f"native path unavailable: {reason}"
    return True

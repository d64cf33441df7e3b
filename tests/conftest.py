import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent
sys.path.insert(0, str(ROOT))
sys.path.insert(0, str(Path(__file__).resolve().parent))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")
    # Build missing native libraries (no-op when they exist and are fresh).
    from knng_gpu_b200 import _native

    if not (_native.GPU_LIB_PATH.exists() and _native.SYNTH_LIB_PATH.exists()):
        from knng_gpu_b200 import build

        build.build_all()


@pytest.fixture(scope="session")
def cuda_ok():
    import torch

    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return True

import os
import sys

import pytest

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, REPO)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200, sm_100a)")
    config.addinivalue_line("markers", "multigpu: needs two or more GPUs in one process")


def gpu_count() -> int:
    try:
        import torch
        return torch.cuda.device_count() if torch.cuda.is_available() else 0
    except Exception:
        return 0


@pytest.fixture(scope="session")
def ngpu():
    return gpu_count()


@pytest.fixture(scope="session")
def core():
    from scc26_nccl_shim_b200 import _core
    return _core


def need_gpus(n: int):
    if gpu_count() < n:
        pytest.skip(f"needs {n} GPUs, {gpu_count()} visible")

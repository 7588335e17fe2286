"""Shared test plumbing: the `gpu` marker, the path-loaded ctypes binding and
the oracle import.  GPU tests run only with a CUDA device (`-m gpu`)."""
import importlib.util
import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA B200 (sm_100a) device")


def load_binding():
    """Import llm.cu_b200/llmcu.py (the directory name is not a package name)."""
    if "llmcu" in sys.modules:
        return sys.modules["llmcu"]
    path = os.path.join(ROOT, "llm.cu_b200", "llmcu.py")
    spec = importlib.util.spec_from_file_location("llmcu", path)
    mod = importlib.util.module_from_spec(spec)
    sys.modules["llmcu"] = mod
    spec.loader.exec_module(mod)
    return mod


@pytest.fixture(scope="session")
def llmcu():
    return load_binding()


@pytest.fixture(scope="session")
def cuda_device():
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return torch.device("cuda:0")

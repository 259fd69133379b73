"""Shared fixtures.  GPU tests are marked `gpu`; everything else runs on CPU."""

from __future__ import annotations

import importlib.util
import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs an sm_100 (B200) GPU and the built CUDA library")


def _load(name, path):
    if name in sys.modules:
        return sys.modules[name]
    spec = importlib.util.spec_from_file_location(name, path)
    mod = importlib.util.module_from_spec(spec)
    sys.modules[name] = mod
    spec.loader.exec_module(mod)
    return mod


@pytest.fixture(scope="session")
def synth():
    return _load("mrml_moe_b200_synth", os.path.join(ROOT, "qt_llama.cpp_b200", "synth.py"))


@pytest.fixture(scope="session")
def moe():
    return _load("mrml_moe_b200", os.path.join(ROOT, "qt_llama.cpp_b200", "mrml_moe.py"))


@pytest.fixture(scope="session")
def oracle():
    mod = _load("mrml_oracle", os.path.join(ROOT, "oracle", "oracle.py"))
    mod.lib()
    return mod


@pytest.fixture(scope="session")
def cuda(moe):
    """The CUDA device; on a GPU run a missing GPU or library is a failure."""
    import torch

    assert torch.cuda.is_available(), "GPU test run without a visible GPU"
    major, _ = torch.cuda.get_device_capability(0)
    assert major == 10, "the library targets sm_100 (B200)"
    moe.load_library()
    return torch.device("cuda", 0)

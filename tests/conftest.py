"""Shared pytest setup: the `gpu` marker and access to the package.

The package directory is named `qwen3-aligner-wgpu_b200`, which is not a Python
identifier, so it is imported through importlib under its own name.
"""
import importlib
import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

PKG_NAME = "qwen3-aligner-wgpu_b200"


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (run on the B200 box)")


def pkg():
    return importlib.import_module(PKG_NAME)


@pytest.fixture(scope="session")
def qa():
    return pkg()


def cuda_ok():
    try:
        import torch
        return torch.cuda.is_available()
    except Exception:
        return False

"""Test configuration.

Markers:
  gpu   needs a CUDA device (B200); run with ``-m gpu`` on the GPU box.
Everything else runs on the CPU: the oracle against the golden fixtures, the
host-side logic, and that the native library loads and exports its C ABI.

The native library and the C oracle are (re)built here if missing, so a fresh
checkout tests the code it contains.
"""
import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)
ORACLE_DIR = os.path.join(ROOT, "oracle")
if ORACLE_DIR not in sys.path:
    sys.path.insert(0, ORACLE_DIR)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: test needs a CUDA GPU")
    import oracle as _oracle

    _oracle.build_oracle_lib()
    from metagross_b200 import build as _build

    _build.build()


def cuda_available():
    import torch

    return torch.cuda.is_available()


def pytest_collection_modifyitems(config, items):
    if cuda_available():
        return
    skip = pytest.mark.skip(reason="needs a CUDA GPU")
    for item in items:
        if "gpu" in item.keywords:
            item.add_marker(skip)

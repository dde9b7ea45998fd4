"""Test configuration.

Seeding follows the reference's conftest (tests/conftest.py:17-49 in the ntops project): every
module and every test case seeds ``random`` and ``torch`` from the sha256 of its path, so a case
sees the same inputs on every run.  GPU tests carry the ``gpu`` marker and are skipped when no
CUDA device is present.
"""

import hashlib
import os
import random
import sys

import pytest
import torch

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if REPO not in sys.path:
    sys.path.insert(0, REPO)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200); runs the sm_100a kernels")
    torch.backends.cuda.matmul.allow_fp16_reduced_precision_reduction = False
    torch.backends.cuda.matmul.allow_bf16_reduced_precision_reduction = False


def pytest_collection_modifyitems(config, items):
    if torch.cuda.is_available():
        return
    skip = pytest.mark.skip(reason="needs a CUDA device")
    for item in items:
        if "gpu" in item.keywords:
            item.add_marker(skip)


def _hash(s):
    return int(hashlib.sha256(s.encode("utf-8")).hexdigest(), 16) % 2**32


def _seed(s):
    random.seed(s)
    torch.manual_seed(s)


@pytest.fixture(autouse=True)
def set_seed_per_test(request):
    module = request.module.__name__.replace(".", "/") + ".py"
    _seed(_hash(f"{module}::{request.node.name}"))

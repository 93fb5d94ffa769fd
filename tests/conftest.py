"""pytest configuration: the ``gpu`` marker and shared fixture loaders.

Tests marked ``gpu`` need a CUDA device (B200, sm_100a) and the in-tree CUDA
library; everything else runs on the CPU.
"""
import importlib
import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

PKG_NAME = "910b_e2e_accleration_by_codex_b200"
GOLDEN = os.path.join(ROOT, "tests", "golden")


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200) and the built CUDA library")


def pkg(sub=None):
    """Import the package (its directory name is not a Python identifier) or a submodule."""
    name = PKG_NAME if sub is None else f"{PKG_NAME}.{sub}"
    return importlib.import_module(name)


def load_golden(name):
    """Load tests/golden/<name>; keys stored as bf16 bits ('<key>__bf16') come back as float32."""
    from oracle.gdn_oracle import from_bf16_bits
    raw = np.load(os.path.join(GOLDEN, name))
    out = {}
    for k in raw.files:
        if k.endswith("__bf16"):
            out[k[:-6]] = from_bf16_bits(raw[k])
            out.setdefault("_bf16_keys", set()).add(k[:-6])
        else:
            out[k] = raw[k]
    return out


@pytest.fixture
def golden():
    return load_golden

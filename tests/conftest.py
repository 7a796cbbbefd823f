"""Shared fixtures.  GPU tests carry @pytest.mark.gpu; everything else runs on
CPU.  The oracle (oracle/) is the checker here and nowhere in the product."""

from __future__ import annotations

import os
import sys
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parent.parent
sys.path.insert(0, str(ROOT))

from motoria_b200 import synth  # noqa: E402
from oracle import oracle as oracle_mod  # noqa: E402

GOLDEN = ROOT / "tests" / "golden"
SEED = 1234  # weights
XSEED = 99   # activations


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs an sm_100a GPU (run with -m gpu)")


@pytest.fixture(scope="session")
def orc():
    oracle_mod.build()
    return oracle_mod.oracle()


@pytest.fixture(scope="session")
def ref():
    """The reference engine built from source, or None (e.g. on the GPU box)."""
    return oracle_mod.ref()


_layers: dict = {}


def get_layer(shape, zipf=False, seed=SEED):
    k = (shape, zipf, seed)
    if k not in _layers:
        _layers[k] = synth.layer(shape, seed, zipf=zipf)
    return _layers[k]


@pytest.fixture(scope="session")
def golden():
    return dict(np.load(GOLDEN / "moe_golden.npz"))


def rel_l2(a, b):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


def n_threads():
    return max(1, min(os.cpu_count() or 1, 32))


@pytest.fixture(scope="session")
def torch_cuda():
    import torch

    if not torch.cuda.is_available():
        pytest.fail("GPU test on a machine without CUDA")
    return torch

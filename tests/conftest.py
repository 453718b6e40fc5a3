"""Shared test fixtures.  GPU tests carry ``@pytest.mark.gpu``; everything else
runs on the CPU (the oracle, the host logic, the C-ABI symbol table)."""
from __future__ import annotations

import functools
import json
import os
import sys

import numpy as np
import pytest
import torch

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)
GOLDEN = os.path.join(ROOT, "tests", "golden")


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100a) GPU")
    config.addinivalue_line("markers", "slow: long CPU oracle run")


@functools.lru_cache(maxsize=1)
def _weights():
    from nanovllm_dots_b200 import synthetic as syn
    return syn.make_weights(syn.BASE, seed=0)


@pytest.fixture(scope="session")
def weights():
    return _weights()


@pytest.fixture(scope="session")
def golden():
    with open(os.path.join(GOLDEN, "manifest.json")) as f:
        man = json.load(f)
    arrays = dict(np.load(os.path.join(GOLDEN, "fm_golden.npz")))
    return man, {k: torch.from_numpy(v) for k, v in arrays.items()}


def cos_min(a: torch.Tensor, b: torch.Tensor, dim: int = 64) -> float:
    """Per-latent-frame cosine similarity, minimum over frames (the reference
    tests' idiom, ``tests/conftest.py:63-71`` of the reference)."""
    a = a.float().reshape(-1, dim)
    b = b.float().reshape(-1, dim)
    return torch.nn.functional.cosine_similarity(a, b, dim=-1).min().item()

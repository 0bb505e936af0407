"""Shared fixtures: the CUDA library binding (mx-kmeans_b200/mxk.py), the CPU
oracle (oracle/oracle.py) and helpers.  Tests that need a GPU are marked `gpu`."""
import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
for sub in ("mx-kmeans_b200", "oracle"):
    p = os.path.join(ROOT, sub)
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200, sm_100a)")


@pytest.fixture(scope="session")
def orc():
    import oracle
    oracle.lib()
    return oracle


@pytest.fixture(scope="session")
def mxk():
    import mxk as m
    m.load()
    return m


@pytest.fixture(scope="session")
def torch_cuda():
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return torch


def rng(seed=0):
    return np.random.default_rng(seed)


def reference_fixture_a(m=131, d=256):
    """tests/cuda_checks.cu:37-41: sin(row*17+j) * 2^((row + j/32) % 9 - 4)"""
    row = np.arange(m, dtype=np.float32)[:, None]
    j = np.arange(d)[None, :]
    return (np.sin((row * 17 + j).astype(np.float32)) *
            np.ldexp(np.float32(1.0), ((np.arange(m)[:, None] + j // 32) % 9 - 4))).astype(np.float32)


def reference_fixture_b(n=132, d=256):
    """tests/cuda_checks.cu:42-44: cos(row*7+j) * 2^((row*2 + j/32) % 7 - 3)"""
    row = np.arange(n, dtype=np.float32)[:, None]
    j = np.arange(d)[None, :]
    return (np.cos((row * 7 + j).astype(np.float32)) *
            np.ldexp(np.float32(1.0), ((np.arange(n)[:, None] * 2 + j // 32) % 7 - 3))).astype(np.float32)


def blobs(n, d, k, seed, spread=10.0, sigma=1.0, pad_to=128):
    """Seeded Gaussian blobs, zero-padded to a multiple of pad_to features."""
    g = np.random.default_rng(seed)
    centers = g.uniform(-spread, spread, size=(k, d)).astype(np.float32)
    lab = g.integers(0, k, size=n)
    x = centers[lab] + g.normal(0, sigma, size=(n, d)).astype(np.float32)
    dp = (d + pad_to - 1) // pad_to * pad_to
    out = np.zeros((n, dp), np.float32)
    out[:, :d] = x
    return out

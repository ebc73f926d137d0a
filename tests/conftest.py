"""Shared test setup: import paths, the `gpu` marker, parity metrics."""

from __future__ import annotations

import os
import sys

import numpy as np
import pytest

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG_ROOT = os.path.join(REPO, "vllm-sparse-mla-blackwell_b200")
for p in (REPO, PKG_ROOT, os.path.join(REPO, "tests")):
    if p not in sys.path:
        sys.path.insert(0, p)

# Parity bar for the kernel against the fp32 oracle (the north star's): max
# relative error over the whole output <= 5e-3 and per-(token, head) cosine
# >= 0.99999 over rows whose reference is non-zero.
REL_TOL = 5e-3
COS_TOL = 0.99999
# log2-space LSE, absolute
LSE_TOL = 1e-3


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100a) GPU")


def parity_metrics(got: np.ndarray, ref: np.ndarray):
    """(rel, min_cos, finite) as the reference's gates define them
    (tests/run_installed.py:46-54 of the reference)."""
    got = np.asarray(got, np.float64)
    ref = np.asarray(ref, np.float64)
    finite = bool(np.isfinite(got).all())
    rel = float(np.abs(got - ref).max() / max(np.abs(ref).max(), 1e-6)) if ref.size else 0.0
    g = got.reshape(-1, got.shape[-1])
    r = ref.reshape(-1, ref.shape[-1])
    nz = np.abs(r).sum(-1) > 0
    if nz.any():
        num = (g[nz] * r[nz]).sum(-1)
        den = np.linalg.norm(g[nz], axis=-1) * np.linalg.norm(r[nz], axis=-1)
        cmin = float((num / np.maximum(den, 1e-30)).min())
    else:
        cmin = 1.0
    return rel, cmin, finite


@pytest.fixture(scope="session")
def golden():
    path = os.path.join(REPO, "tests", "golden", "sparse_mla_golden.npz")
    return np.load(path)

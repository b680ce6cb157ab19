"""Shared fixtures. ``-m gpu`` tests need a B200 and the in-tree library; everything else runs on CPU.

The oracle (oracle/) is test infrastructure: tests import it as the checker only.
"""
from __future__ import annotations

import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)
sys.path.insert(0, os.path.join(ROOT, "oracle"))
GOLDEN = os.path.join(ROOT, "tests", "golden")


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA B200 (sm_100a) and libmuyo_cuda.so")


@pytest.fixture(scope="session")
def oracle_mod():
    import oracle

    oracle.build()
    return oracle


@pytest.fixture(scope="session")
def cuda():
    """The CUDA device for -m gpu tests. Fails (does not skip) without a GPU, so a GPU run can
    never pass on a silent fallback."""
    import torch

    from muyo_llm_b200 import _abi, build

    assert torch.cuda.is_available(), "-m gpu tests need a CUDA device"
    build()
    _abi.call("muyo_cuda_init", 0)
    torch.cuda.set_device(0)
    return torch.device("cuda", 0)


def rel_close(actual, expected, tol: float) -> np.ndarray:
    """The reference's float comparison |a - e| <= tol * (1 + |e|) (src/TransformerLayer.cpp:602)."""
    a = np.asarray(actual, np.float64)
    e = np.asarray(expected, np.float64)
    return np.abs(a - e) <= tol * (1.0 + np.abs(e))


def assert_rel_close(actual, expected, tol: float, what: str = "") -> None:
    ok = rel_close(actual, expected, tol)
    if not ok.all():
        a = np.asarray(actual, np.float64).reshape(-1)
        e = np.asarray(expected, np.float64).reshape(-1)
        bad = np.flatnonzero(~ok.reshape(-1))
        i = bad[0]
        raise AssertionError(f"{what}: {bad.size} of {a.size} outside {tol}*(1+|e|); first at {i}: {a[i]} vs {e[i]}"
                             f" (max err {np.max(np.abs(a - e) / (1 + np.abs(e))):.3g})")


def assert_gemv_accurate(actual, w, x, bias=None, what: str = "") -> None:
    """A rigorous accuracy bound for an FP32-accumulated dot product of K terms: |y - exact| <=
    gamma_K * sum_k |w_k x_k| with gamma_K = K * 2^-24 / (1 - K * 2^-24) (recursive summation, any
    order), plus one rounding of the bias add. The exact value is computed in float64."""
    w64 = np.asarray(w, np.float64)
    x64 = np.asarray(x, np.float64)
    exact = w64 @ x64
    mag = np.abs(w64) @ np.abs(x64)
    K = w64.shape[1]
    u = 2.0 ** -24
    bound = (K * u / (1 - K * u)) * mag
    if bias is not None:
        exact = exact + np.asarray(bias, np.float64)
        bound = bound + 2 * u * (np.abs(exact) + mag)
    err = np.abs(np.asarray(actual, np.float64) - exact)
    bad = np.flatnonzero(err > bound + 1e-30)
    assert bad.size == 0, f"{what}: {bad.size} rows exceed the FP32 summation bound; first {bad[0]}: err {err[bad[0]]} > {bound[bad[0]]}"

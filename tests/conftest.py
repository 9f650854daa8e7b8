"""Shared test setup.

Markers: ``gpu`` tests need a B200 and call the CUDA library through its C ABI;
everything else runs on CPU (oracle, golden vectors, host logic, ABI symbols).
"""
from __future__ import annotations

import os
import sys
from pathlib import Path

import pytest

REPO = Path(__file__).resolve().parents[1]
PKG = REPO / "qwen3.8_27b_in_rust_b200"
for p in (REPO, PKG, REPO / "oracle", REPO / "tests" / "golden"):
    if str(p) not in sys.path:
        sys.path.insert(0, str(p))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 GPU and the built CUDA library")


@pytest.fixture(scope="session")
def oracle_lib():
    import oracle
    oracle.build()
    oracle.load()
    return oracle


@pytest.fixture(scope="session")
def cuda_ctx():
    """One q38attn context on cuda:0 for the whole GPU session."""
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    import q38attn
    ctx = q38attn.Context(0)
    yield ctx
    torch.cuda.synchronize()
    ctx.close()


def relative_error(a, b):
    """The reference's metric |a-b| / max(|b|, 1) (src/kernel/x86/tensor.rs:411-413),
    maximised over elements."""
    import numpy as np
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.max(np.abs(a - b) / np.maximum(np.abs(b), 1.0))) if a.size else 0.0

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


def scaled_error(a, b):
    """max|a-b| / max|b|: the error relative to the expected tensor's own scale.
    Unlike the reference's metric it does not turn into an absolute error when
    the values are below 1 (attention outputs at long context are ~0.01)."""
    import numpy as np
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    if not a.size:
        return 0.0
    diff = float(np.max(np.abs(a - b)))
    scale = float(np.max(np.abs(b)))
    return diff / scale if scale > 0 else diff


# Every check_parity result of the session: (test, what, reference metric,
# scaled error, tolerance). Written as JSON to $Q38_PARITY_LOG at the end.
PARITY_LOG: list = []


def check_parity(a, b, tol, what=""):
    """Asserts that both the reference's metric and the scale-aware error are
    below `tol`; records and returns them."""
    r, s = relative_error(a, b), scaled_error(a, b)
    test = os.environ.get("PYTEST_CURRENT_TEST", "").split(" ")[0]
    PARITY_LOG.append({"test": test, "what": what, "ref_metric": r, "scaled": s, "tol": tol})
    print(f"[parity] {test} {what}: ref metric {r:.3e}, scaled {s:.3e} (tol {tol:g})")
    assert r < tol and s < tol, (what, r, s, tol)
    return r, s


def pytest_sessionfinish(session, exitstatus):
    path = os.environ.get("Q38_PARITY_LOG")
    if path and PARITY_LOG:
        import json
        Path(path).parent.mkdir(parents=True, exist_ok=True)
        Path(path).write_text(json.dumps(PARITY_LOG, indent=1))

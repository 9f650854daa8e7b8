"""CPU tests of the C ABI: the library loads without a GPU, exports every
function include/q38attn.h declares, and rejects bad arguments before any
device work (the reference's Err(-1) paths)."""
from __future__ import annotations

import ctypes
import re
import subprocess

import pytest

from conftest import REPO

HEADER = REPO / "include" / "q38attn.h"


def declared_functions() -> set[str]:
    text = HEADER.read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return set(re.findall(r"\b(q38_[a-z0-9_]+)\s*\(", text))


@pytest.fixture(scope="module")
def lib():
    import q38attn
    return q38attn.load()


def test_header_declares_the_boundary():
    names = declared_functions()
    for must in ("q38_ctx_create", "q38_state_create", "q38_full_decode", "q38_linear_decode",
                 "q38_full_core", "q38_linear_core", "q38_full_decode_host",
                 "q38_linear_decode_host"):
        assert must in names


def test_library_exports_every_declared_symbol(lib):
    out = subprocess.run(["nm", "-D", "--defined-only", str(REPO / "qwen3.8_27b_in_rust_b200" /
                                                           "libq38attn.so")],
                         capture_output=True, text=True, check=True).stdout
    exported = set(re.findall(r"\bT (q38_[a-z0-9_]+)", out))
    missing = declared_functions() - exported
    assert not missing, f"declared but not exported: {sorted(missing)}"


def test_binding_covers_every_declared_symbol():
    from q38attn._lib import SIGNATURES
    assert declared_functions() == set(SIGNATURES)


def test_geometry_defaults_match_reference(lib):
    import q38attn
    g = q38attn.geometry()
    assert (g.attn_heads, g.attn_kv_heads, g.attn_head_dim, g.rope_dims) == (24, 4, 256, 64)
    assert (g.linear_qk_heads, g.linear_v_heads, g.linear_head_dim, g.conv_kernel) == (16, 48,
                                                                                      128, 4)
    assert g.rope_theta == 1e7
    assert g.rms_eps == pytest.approx(1e-6)
    assert lib.q38_version().decode().startswith("q38attn")


def test_bad_geometry_is_an_argument_error(lib):
    import q38attn
    g = q38attn.geometry()
    g.attn_head_dim = 128
    h = ctypes.c_void_p()
    assert lib.q38_ctx_create(ctypes.byref(g), 0, ctypes.byref(h)) == q38attn.Q38_ERR_ARG
    assert "256" in q38attn.last_error()
    g = q38attn.geometry()
    g.attn_heads = 25
    assert lib.q38_ctx_create(ctypes.byref(g), 0, ctypes.byref(h)) == q38attn.Q38_ERR_ARG
    g = q38attn.geometry()
    g.linear_v_heads = 50
    assert lib.q38_ctx_create(ctypes.byref(g), 0, ctypes.byref(h)) == q38attn.Q38_ERR_ARG
    assert not h.value


def test_null_handles_are_argument_errors(lib):
    import q38attn
    E = q38attn.Q38_ERR_ARG
    assert lib.q38_ctx_create(None, 0, None) == E
    h = ctypes.c_void_p()
    assert lib.q38_state_create(None, 1, 16, 1, 1, 0, ctypes.byref(h)) == E
    assert lib.q38_full_decode(None, None, 3, 1, None, None, None, None, -1, None, None) == E
    assert lib.q38_linear_decode(None, None, 0, 1, None, None, None, None, None, None) == E
    assert lib.q38_full_core(None, None, 3, *([None] * 9), 0, 0, 0) == E
    assert lib.q38_linear_core(None, None, 0, *([None] * 7)) == E
    assert lib.q38_state_errors(None, None) == E
    assert lib.q38_ctx_destroy(None) == 0
    assert lib.q38_state_destroy(None) == 0


def test_layer_kind_helpers_match_reference():
    import q38attn
    full = [l for l in range(65) if q38attn.is_full_attention(l)]
    assert full == [3, 7, 11, 15, 19, 23, 27, 31, 35, 39, 43, 47, 51, 55, 59, 63, 64]
    assert [q38attn.full_index(l) for l in full] == list(range(16)) + [16]
    lin = [l for l in range(64) if not q38attn.is_full_attention(l)]
    assert [q38attn.recurrent_index(l) for l in lin] == list(range(48))


def test_product_path_does_not_reference_the_oracle():
    """The shipped library and its Python binding never load the checker."""
    pkg = REPO / "qwen3.8_27b_in_rust_b200"
    for p in list(pkg.rglob("*.py")) + list(pkg.rglob("*.cu")) + list(pkg.rglob("*.cuh")) + \
            list(pkg.rglob("*.h")):
        text = p.read_text()
        assert "q38_oracle" not in text and "libq38oracle" not in text, p
        assert "import oracle" not in text, p

"""CPU tests of the projection oracle (oracle/q38_oracle_proj.cpp), pinned by
an independent numpy restatement (quant_ref.py) and by the reference's own
checks of this code (src/kernel/tensor.rs:604-925):

* Q8_K quantization (quant.rs:56-124) bit for bit, including the first
  largest magnitude winning a tie, all-zero blocks and the reference's
  deterministic test activation ((i*7919) % 101) / 50 - 1;
* f16_to_f32 (quant.rs:21-45) over all 65536 half values;
* every K-quant and IQ4 integer dot bit for bit against the numpy
  restatement, and within the reference's 0.05 of a plain dot over the
  dequantized row (kernel_consistency, tensor.rs:604-700); the f32-input dots
  (the IQ4 types' f32 path, iq.rs:311-335, included) within 1e-3;
* token-major batched output equal to the per-row dots
  (gemv_and_gemm_match_serial_row_dot, tensor.rs:792-925).
"""
from __future__ import annotations

import numpy as np
import pytest

import oracle
import quant_ref
from q38attn import synth

K_TYPES = [oracle.GGML_Q2_K, oracle.GGML_Q3_K, oracle.GGML_Q4_K, oracle.GGML_Q5_K,
           oracle.GGML_Q6_K]
F_TYPES = [oracle.GGML_F32, oracle.GGML_F16, oracle.GGML_BF16, oracle.GGML_Q8_0]
IQ_TYPES = [oracle.GGML_IQ4_NL, oracle.GGML_IQ4_XS]


def reference_activation(width: int) -> np.ndarray:
    """tensor.rs:582-586."""
    return np.array([((i * 7919) % 101) / 50.0 - 1.0 for i in range(width)], np.float32)


def relative(a, b) -> float:
    return float(np.max(np.abs(np.float64(a) - np.float64(b)) / np.maximum(np.abs(np.float64(b)), 1.0)))


def test_f16_to_f32_all_halves():
    lib = oracle.load()
    bits = np.arange(65536, dtype=np.uint16)
    want = bits.view(np.float16).astype(np.float32)
    got = np.array([lib.q38o_f16_to_f32(int(h)) for h in bits], np.float32)
    finite = np.isfinite(want) | np.isinf(want)
    np.testing.assert_array_equal(got[finite].view(np.uint32), want[finite].view(np.uint32))
    assert np.all(np.isnan(got[~finite]))
    assert oracle.f16_to_f32(0x0001) == 2.0 ** -24 and oracle.f16_to_f32(0x7BFF) == 65504.0


def _quantize_cases():
    g = np.random.default_rng(3)
    tie = np.zeros(256, np.float32)
    tie[5], tie[9] = -3.0, 3.0  # equal magnitudes: the first (negative) one is the maximum
    tie2 = g.standard_normal(256).astype(np.float32)
    tie2[200], tie2[17] = 7.5, 7.5
    small = (g.standard_normal(256) * 1e-30).astype(np.float32)
    half = np.full(256, 0.5, np.float32)  # inverse * v lands on .5 ties: round half to even
    half[0] = -254.0
    return np.concatenate([reference_activation(512), g.standard_normal(1024).astype(np.float32) * 3,
                           np.zeros(256, np.float32), tie, tie2, small, half])


def test_quantize_q8_k_matches_numpy_restatement():
    x = _quantize_cases()
    blocks = oracle.quantize_q8_k(x)
    scale, quants, sums = quant_ref.quantize_q8_k(x)
    np.testing.assert_array_equal(blocks["scale"].view(np.uint32), scale.view(np.uint32))
    np.testing.assert_array_equal(blocks["quants"], quants)
    np.testing.assert_array_equal(blocks["sums"], sums)
    # The tie block: the maximum is -3 (index 5), so inverse = 127/3 > 0.
    tie = blocks[7]
    assert tie["quants"][5] == -127 and tie["quants"][9] == 127
    assert np.all(blocks[6]["quants"] == 0) and blocks[6]["scale"] == 0.0
    # The reference activation's first block: max |x| is 1.0 at index 0 (x = -1).
    assert blocks[0]["quants"][0] == -127
    assert blocks[0]["scale"] == np.float32(1.0) / np.float32(127.0)


def test_quantize_q8_k_rejects_ragged_length():
    with pytest.raises(ValueError):
        oracle.quantize_q8_k(np.zeros(300, np.float32))


@pytest.mark.parametrize("ggml_type", K_TYPES + IQ_TYPES)
def test_integer_dot_matches_numpy_restatement(ggml_type):
    g = synth.rng(10 + ggml_type)
    rows, width = 6, 1024
    w = synth.quant_weight(g, ggml_type, rows, width)
    rb = oracle.row_bytes(ggml_type, width)
    for x in (reference_activation(width), synth.normal(g, width)):
        blocks = oracle.quantize_q8_k(x)
        scale, quants, sums = quant_ref.quantize_q8_k(x)
        for r in range(rows):
            row = w[r * rb:(r + 1) * rb]
            got = oracle.dot_row_q8_k(ggml_type, row, blocks)
            want = quant_ref.dot_q8_k(ggml_type, row, scale, quants, sums)
            assert np.float32(got).view(np.uint32) == np.float32(want).view(np.uint32), (r, got, want)


@pytest.mark.parametrize("ggml_type", K_TYPES + F_TYPES + IQ_TYPES)
def test_kernel_consistency_against_dequantized_dot(ggml_type):
    """The reference's kernel_consistency bars (tensor.rs:604-700): the
    f32-input dot within 1e-3 and the integer dot within 0.05 of a plain dot
    over the dequantized row, on rows 0 and last."""
    g = synth.rng(30 + ggml_type)
    rows, width = 5, 2048
    w = synth.quant_weight(g, ggml_type, rows, width)
    dq = quant_ref.dequantize(ggml_type, w, rows, width)
    x = reference_activation(width)
    rb = oracle.row_bytes(ggml_type, width)
    for r in (0, rows - 1):
        want = float(np.dot(dq[r], x.astype(np.float64)))
        row = w[r * rb:(r + 1) * rb]
        if oracle.is_q8k_type(ggml_type):
            got = oracle.dot_row_q8_k(ggml_type, row, oracle.quantize_q8_k(x))
            assert relative(got, want) < 0.05
        if not oracle.is_q8k_type(ggml_type) or ggml_type in IQ_TYPES:
            got = oracle.dot_row_f32(ggml_type, row, x)
            assert relative(got, want) < 1e-3


@pytest.mark.parametrize("ggml_type", [oracle.GGML_Q4_K, oracle.GGML_Q6_K, oracle.GGML_Q8_0,
                                       oracle.GGML_BF16, oracle.GGML_IQ4_NL, oracle.GGML_IQ4_XS])
def test_batched_project_is_token_major_row_dots(ggml_type):
    """gemv_and_gemm_match_serial_row_dot (tensor.rs:792-925): every output
    [token * rows + row] is the single-row dot, bitwise; tokens are
    x + token * 0.125."""
    g = synth.rng(50 + ggml_type)
    rows, width, batch = 37, 512, 3
    w = synth.quant_weight(g, ggml_type, rows, width)
    x = reference_activation(width)
    tokens = np.stack([x + np.float32(t * 0.125) for t in range(batch)]).astype(np.float32)
    out = oracle.project(ggml_type, w, rows, width, tokens)
    assert out.shape == (batch, rows)
    rb = oracle.row_bytes(ggml_type, width)
    for r in (0, 1, rows // 2, rows - 2, rows - 1):
        row = w[r * rb:(r + 1) * rb]
        for t in range(batch):
            if oracle.is_q8k_type(ggml_type):
                want = oracle.dot_row_q8_k(ggml_type, row, oracle.quantize_q8_k(tokens[t]))
            else:
                want = oracle.dot_row_f32(ggml_type, row, tokens[t])
            assert np.float32(out[t, r]).view(np.uint32) == np.float32(want).view(np.uint32)


def test_row_bytes_and_shape_errors():
    assert oracle.row_bytes(oracle.GGML_Q4_K, 5120) == 2880
    assert oracle.row_bytes(oracle.GGML_Q6_K, 5120) == 4200
    assert oracle.row_bytes(oracle.GGML_Q8_0, 5120) == 5440
    assert oracle.row_bytes(oracle.GGML_IQ4_NL, 5120) == 2880
    assert oracle.row_bytes(oracle.GGML_IQ4_XS, 5120) == 2720
    assert oracle.is_q8k_type(oracle.GGML_IQ4_NL) and oracle.is_q8k_type(oracle.GGML_IQ4_XS)
    with pytest.raises(ValueError):
        oracle.row_bytes(oracle.GGML_Q4_K, 300)
    with pytest.raises(ValueError):
        oracle.row_bytes(2, 256)  # Q4_0 is not a projection type here
    w = synth.quant_weight(synth.rng(0), oracle.GGML_Q8_0, 4, 96)
    with pytest.raises(ValueError):  # the integer path needs whole 256-blocks
        oracle.gemm_q8_k(oracle.GGML_Q8_0, w, 4, 96, oracle.quantize_q8_k(np.zeros(256, np.float32)), 1)


def test_package_row_bytes_match_the_oracle():
    """The Python package's row sizes (what a caller sizes host buffers with)
    agree with the oracle's row_bytes (src/kernel/tensor.rs:46-53) for every
    projection type, IQ4_NL / IQ4_XS included."""
    import q38attn
    for ggml_type in K_TYPES + F_TYPES + IQ_TYPES:
        for width in (256, 5120, 6144):
            assert q38attn.row_bytes(ggml_type, width) == oracle.row_bytes(ggml_type, width)

"""Seeded synthetic weights and inputs with the distributions of the five
benchmark configurations (no checkpoint or dataset is available, so these
stand in for them):

1. full-attention decode, batch 1, 256 cached positions, fp32 KV ~ N(0,1);
2. Gated DeltaNet decode, batch 1, state S ~ N(0, 0.02^2) of shape 48x128x128;
3. batched long-context decode, bf16 KV ~ N(0,1);
4. causal prefill attention, bf16 Q/K/V ~ N(0,1);
5. Gated DeltaNet chunked prefill with the config-2 distributions per token.

Weights not fixed by the configurations: attn_q_norm / attn_k_norm / ssm_norm
~ 1 + 0.1 N(0,1), ssm_conv1d ~ N(0, 0.5^2), dt_bias ~ N(0,1),
ssm_a = -exp(U(0, 2.7)) (A_log ~ U(0, 2.7)). All arrays are float32 numpy.
"""
from __future__ import annotations

import numpy as np

from . import (ATTN_HEAD_DIM, ATTN_KV_DIM, ATTN_QG_DIM, LINEAR_HEAD_DIM, LINEAR_QKV_DIM,
               LINEAR_V_DIM, LINEAR_V_HEADS)


def rng(seed: int = 0) -> np.random.Generator:
    return np.random.default_rng(seed)


def normal(g: np.random.Generator, shape, std: float = 1.0, mean: float = 0.0) -> np.ndarray:
    x = g.standard_normal(shape, dtype=np.float32)
    if std != 1.0:
        x *= np.float32(std)
    if mean != 0.0:
        x += np.float32(mean)
    return np.ascontiguousarray(x, dtype=np.float32)


def full_weights(g: np.random.Generator) -> dict:
    return {
        "q_norm": normal(g, ATTN_HEAD_DIM, 0.1, 1.0),
        "k_norm": normal(g, ATTN_HEAD_DIM, 0.1, 1.0),
    }


def linear_weights(g: np.random.Generator) -> dict:
    a_log = g.uniform(0.0, 2.7, LINEAR_V_HEADS).astype(np.float32)
    return {
        "conv1d": normal(g, (LINEAR_QKV_DIM, 4), 0.5),
        "dt_bias": normal(g, LINEAR_V_HEADS),
        "ssm_a": np.ascontiguousarray(-np.exp(a_log), dtype=np.float32),
        "ssm_norm": normal(g, LINEAR_HEAD_DIM, 0.1, 1.0),
    }


def full_step(g: np.random.Generator, batch: int = 1) -> dict:
    """Per-token inputs of full_core: q_and_gate, key, value."""
    return {
        "q_and_gate": normal(g, (batch, ATTN_QG_DIM)),
        "key": normal(g, (batch, ATTN_KV_DIM)),
        "value": normal(g, (batch, ATTN_KV_DIM)),
    }


def linear_step(g: np.random.Generator, batch: int = 1) -> dict:
    """Per-token inputs of linear_core: qkv, z, beta and alpha logits."""
    return {
        "qkv": normal(g, (batch, LINEAR_QKV_DIM)),
        "z": normal(g, (batch, LINEAR_V_DIM)),
        "beta": normal(g, (batch, LINEAR_V_HEADS)),
        "alpha": normal(g, (batch, LINEAR_V_HEADS)),
    }


def linear_state(g: np.random.Generator) -> dict:
    return {
        "conv_state": normal(g, (LINEAR_QKV_DIM, 3)),
        "delta_state": normal(g, (LINEAR_V_HEADS, LINEAR_HEAD_DIM, LINEAR_HEAD_DIM), 0.02),
    }


def kv_rows(g: np.random.Generator, count: int, bf16: bool = False) -> tuple:
    """Cached K/V rows (as stored: post-norm, post-RoPE) ~ N(0,1)."""
    k = normal(g, (count, ATTN_KV_DIM))
    v = normal(g, (count, ATTN_KV_DIM))
    if bf16:
        k, v = round_bf16(k), round_bf16(v)
    return k, v


def round_bf16(x: np.ndarray) -> np.ndarray:
    """Round-to-nearest-even to bf16, returned as float32."""
    u = np.ascontiguousarray(x, np.float32).view(np.uint32).astype(np.uint64)
    u = (u + 0x7FFF + ((u >> 16) & 1)) & 0xFFFF0000
    return u.astype(np.uint32).view(np.float32)


# ---------------------------------------------------------------------------
# Projection weights in the ggml block formats (no checkpoint is available).
# Quant bits and packed scales are uniform random bytes; the f16 super-block
# scales d / dmin are drawn so that a dequantized weight is of order 0.02
# (d ~ U(0.5, 1.5) * 1e-4, dmin ~ U(0, 1) * 1e-4 for the K-quants, 3e-4 for
# Q8_0 and IQ4_NL, 1e-5 for IQ4_XS, whose values are table entries up to 127
# times a group scale up to 32; the last is an f16 subnormal), as in a
# trained checkpoint. F32 / F16 / BF16 weights are N(0, 0.02^2).
# ---------------------------------------------------------------------------
_BLOCK_LAYOUT = {
    # type: (elements, bytes, [(offset of an f16 scale, kind)])  kind: "d" or "dmin"
    8: (32, 34, [(0, "d")]),                    # Q8_0
    10: (256, 84, [(80, "d"), (82, "dmin")]),   # Q2_K
    11: (256, 110, [(108, "d")]),               # Q3_K
    12: (256, 144, [(0, "d"), (2, "dmin")]),    # Q4_K
    13: (256, 176, [(0, "d"), (2, "dmin")]),    # Q5_K
    14: (256, 210, [(208, "d")]),               # Q6_K
    20: (32, 18, [(0, "d")]),                   # IQ4_NL
    23: (256, 136, [(0, "d")]),                 # IQ4_XS
}
_D_SCALE = {8: 3e-4, 20: 3e-4, 23: 1e-5}


def quant_weight(g: np.random.Generator, ggml_type: int, rows: int, width: int) -> np.ndarray:
    """Bytes of a [width, rows] GGUF tensor of `ggml_type` (rows * row_bytes uint8)."""
    if ggml_type == 0:
        return normal(g, (rows, width), 0.02).view(np.uint8).reshape(-1)
    if ggml_type in (1, 30):
        w = normal(g, (rows, width), 0.02)
        if ggml_type == 1:
            bits = w.astype(np.float16).view(np.uint16)
        else:
            bits = round_bf16(w).view(np.uint32) >> np.uint32(16)
        return np.ascontiguousarray(bits.astype(np.uint16)).view(np.uint8).reshape(-1)
    el, by, scales = _BLOCK_LAYOUT[ggml_type]
    nblk = rows * (width // el)
    raw = g.integers(0, 256, size=(nblk, by), dtype=np.uint8)
    for off, kind in scales:
        lo, hi = (0.5, 1.5) if kind == "d" else (0.0, 1.0)
        scale = _D_SCALE.get(ggml_type, 1e-4)
        v = (g.uniform(lo, hi, nblk) * scale).astype(np.float16).view(np.uint16)
        raw[:, off] = (v & 0xff).astype(np.uint8)
        raw[:, off + 1] = (v >> 8).astype(np.uint8)
    return np.ascontiguousarray(raw).reshape(-1)

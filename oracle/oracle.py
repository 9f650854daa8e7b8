"""ctypes binding of the CPU oracle (libq38oracle.so).

TEST INFRASTRUCTURE ONLY: the parity checker for tests/, __graft_entry__.smoke()
and the CPU legs of bench.py. The product library never imports this module.

The oracle restates the reference's linear_core (src/model/ops.rs:647-742),
full_core (ops.rs:812-940) and their per-token prefill loops (ops.rs:1088-1099,
1156-1172) in C++ (q38_oracle.cpp). Parity with the Rust is unpinned by the
reference itself (no Rust toolchain here, no golden vectors upstream); see
q38_oracle.h for how it is pinned instead.
"""
from __future__ import annotations

import ctypes
import subprocess
from ctypes import c_float, c_int, c_int64, c_size_t, c_uint32, c_void_p
from pathlib import Path

import numpy as np

ORACLE_DIR = Path(__file__).resolve().parent
LIB_PATH = ORACLE_DIR / "libq38oracle.so"

QKV = 10240
V_DIM = 6144
V_HEADS = 48
QK_HEADS = 16
HD = 128
QG = 12288
KV = 1024
Q_DIM = 6144

_lib = None


def build(force: bool = False) -> Path:
    src = [ORACLE_DIR / "q38_oracle.cpp", ORACLE_DIR / "q38_oracle_proj.cpp",
           ORACLE_DIR / "q38_oracle.h", ORACLE_DIR / "Makefile"]
    if force or not LIB_PATH.exists() or any(p.stat().st_mtime > LIB_PATH.stat().st_mtime
                                               for p in src):
        subprocess.run(["make", "-C", str(ORACLE_DIR), "-B" if force else "all"], check=True)
    return LIB_PATH


def load() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            build()
        lib = ctypes.CDLL(str(LIB_PATH))
        P = c_void_p
        lib.q38o_set_threads.argtypes = [c_int]
        lib.q38o_get_threads.restype = c_int
        lib.q38o_linear_core.argtypes = [P] * 11
        lib.q38o_linear_core.restype = c_int
        lib.q38o_full_core.argtypes = [P] * 11 + [c_size_t, c_size_t, c_uint32, c_size_t, c_int]
        lib.q38o_full_core.restype = c_int
        lib.q38o_linear_prefill.argtypes = [P] * 11 + [c_size_t]
        lib.q38o_linear_prefill.restype = c_int
        lib.q38o_full_prefill.argtypes = [P] * 8 + [c_size_t, c_size_t, c_uint32, c_size_t,
                                                    c_size_t, c_int]
        lib.q38o_full_prefill.restype = c_int
        lib.q38o_full_prefill_rows.argtypes = [P] * 8 + [c_size_t, c_size_t, c_uint32, c_size_t,
                                                         c_size_t, P, c_size_t, c_int]
        lib.q38o_full_prefill_rows.restype = c_int
        lib.q38o_rms_scale.argtypes = [P, c_size_t]
        lib.q38o_rms_scale.restype = c_float
        lib.q38o_l2norm.argtypes = [P, c_size_t]
        lib.q38o_rope.argtypes = [P, c_size_t, c_uint32]
        lib.q38o_f16_to_f32.argtypes = [ctypes.c_uint16]
        lib.q38o_f16_to_f32.restype = c_float
        lib.q38o_is_q8k_type.argtypes = [c_int]
        lib.q38o_is_q8k_type.restype = c_int
        lib.q38o_row_bytes.argtypes = [c_int, c_size_t, P]
        lib.q38o_row_bytes.restype = c_int
        lib.q38o_quantize_q8_k.argtypes = [P, c_size_t, P]
        lib.q38o_quantize_q8_k.restype = c_int
        lib.q38o_dot_row_f32.argtypes = [c_int, P, P, c_size_t]
        lib.q38o_dot_row_f32.restype = c_float
        lib.q38o_dot_row_q8_k.argtypes = [c_int, P, P, c_size_t]
        lib.q38o_dot_row_q8_k.restype = c_float
        for name in ("q38o_gemm_f32", "q38o_gemm_q8_k", "q38o_project"):
            getattr(lib, name).argtypes = [c_int, P, c_size_t, c_size_t, P, c_size_t, P]
            getattr(lib, name).restype = c_int
        for name in ("q38o_sigmoid", "q38o_silu", "q38o_softplus", "q38o_round_bf16"):
            getattr(lib, name).argtypes = [c_float]
            getattr(lib, name).restype = c_float
        _lib = lib
    return _lib


def _p(a, dtype=np.float32):
    if a is None:
        return None
    assert isinstance(a, np.ndarray) and a.dtype == dtype and a.flags.c_contiguous, a.dtype
    return c_void_p(a.ctypes.data)


def set_threads(n: int) -> None:
    load().q38o_set_threads(n)


def get_threads() -> int:
    return load().q38o_get_threads()


def linear_core(w: dict, conv_state, delta_state, qkv, z, beta, alpha, attention) -> int:
    """linear_core (ops.rs:647-742); every array is updated in place."""
    return load().q38o_linear_core(_p(w["conv1d"]), _p(w["dt_bias"]), _p(w["ssm_a"]),
                                   _p(w["ssm_norm"]), _p(conv_state), _p(delta_state), _p(qkv),
                                   _p(z), _p(beta), _p(alpha), _p(attention))


def linear_prefill(w: dict, conv_state, delta_state, qkv, z, beta, alpha, attention) -> int:
    count = qkv.size // QKV
    return load().q38o_linear_prefill(_p(w["conv1d"]), _p(w["dt_bias"]), _p(w["ssm_a"]),
                                      _p(w["ssm_norm"]), _p(conv_state), _p(delta_state),
                                      _p(qkv), _p(z), _p(beta), _p(alpha), _p(attention), count)


def full_core(w: dict, q_and_gate, key, value, q, gate, scores, attention, key_cache,
              value_cache, context_length: int, position: int, layer: int,
              kv_round_bf16: bool = False) -> int:
    """full_core (ops.rs:812-940); cache arrays are [rows][1024]."""
    rows = min(key_cache.size, value_cache.size) // KV
    return load().q38o_full_core(_p(w["q_norm"]), _p(w["k_norm"]), _p(q_and_gate), _p(key),
                                 _p(value), _p(q), _p(gate), _p(scores), _p(attention),
                                 _p(key_cache), _p(value_cache), rows, context_length, position,
                                 layer, int(kv_round_bf16))


def full_prefill(w: dict, q_and_gate, key, value, attention, key_cache, value_cache,
                 context_length: int, base_position: int, layer: int,
                 kv_round_bf16: int = 0, rows_wanted=None) -> int:
    """Per-token loop of batch_full_attention (ops.rs:1156-1172). kv_round_bf16:
    bit 0 rounds the stored K/V rows to bf16, bit 1 also rounds the query."""
    rows = min(key_cache.size, value_cache.size) // KV
    count = q_and_gate.size // QG
    lib = load()
    if rows_wanted is None:
        return lib.q38o_full_prefill(_p(w["q_norm"]), _p(w["k_norm"]), _p(q_and_gate), _p(key),
                                     _p(value), _p(attention), _p(key_cache), _p(value_cache),
                                     rows, context_length, base_position, layer, count,
                                     int(kv_round_bf16))
    r = np.ascontiguousarray(np.sort(np.asarray(rows_wanted, dtype=np.int64)))
    return lib.q38o_full_prefill_rows(_p(w["q_norm"]), _p(w["k_norm"]), _p(q_and_gate),
                                      _p(key), _p(value), _p(attention), _p(key_cache),
                                      _p(value_cache), rows, context_length, base_position,
                                      layer, count, _p(r, np.int64), r.size, int(kv_round_bf16))


def rms_scale(x: np.ndarray) -> float:
    x = np.ascontiguousarray(x, np.float32)
    return float(load().q38o_rms_scale(_p(x), x.size))


def l2norm(x: np.ndarray) -> None:
    load().q38o_l2norm(_p(x), x.size)


def rope(x: np.ndarray, heads: int, position: int) -> None:
    load().q38o_rope(_p(x), heads, position)


def sigmoid(x: float) -> float:
    return float(load().q38o_sigmoid(x))


def silu(x: float) -> float:
    return float(load().q38o_silu(x))


def softplus(x: float) -> float:
    return float(load().q38o_softplus(x))


def round_bf16(x: float) -> float:
    return float(load().q38o_round_bf16(x))


# ---------------------------------------------------------------------------
# Projections (q38_oracle_proj.cpp): Q8_K quantizer, K-quant integer dots,
# f32-input dots, project / batch_project.
# ---------------------------------------------------------------------------
GGML_F32, GGML_F16, GGML_Q8_0, GGML_BF16 = 0, 1, 8, 30
GGML_Q2_K, GGML_Q3_K, GGML_Q4_K, GGML_Q5_K, GGML_Q6_K = 10, 11, 12, 13, 14
GGML_IQ4_NL, GGML_IQ4_XS = 20, 23

# Q38Q8KBlock (src/kernel/mod.rs:20-27), 292 bytes.
Q8K_BLOCK = np.dtype([("scale", "<f4"), ("quants", "i1", (256,)), ("sums", "<i2", (16,))])
assert Q8K_BLOCK.itemsize == 292


def f16_to_f32(h: int) -> float:
    return float(load().q38o_f16_to_f32(h))


def is_q8k_type(ggml_type: int) -> bool:
    return bool(load().q38o_is_q8k_type(ggml_type))


def row_bytes(ggml_type: int, width: int) -> int:
    out = ctypes.c_size_t(0)
    if load().q38o_row_bytes(ggml_type, width, ctypes.byref(out)) != 0:
        raise ValueError(f"type {ggml_type} cannot hold rows of {width}")
    return out.value


def quantize_q8_k(x: np.ndarray) -> np.ndarray:
    """quantize_q8_k (src/kernel/quant.rs:98-124) of a [..., width] array: one
    Q8K_BLOCK per 256 values, token-major."""
    x = np.ascontiguousarray(x, np.float32)
    out = np.zeros(x.size // 256, Q8K_BLOCK)
    if load().q38o_quantize_q8_k(_p(x), x.size, c_void_p(out.ctypes.data)) != 0:
        raise ValueError("length is not a multiple of 256")
    return out


def _w(weights: np.ndarray) -> c_void_p:
    assert weights.dtype == np.uint8 and weights.flags.c_contiguous
    return c_void_p(weights.ctypes.data)


def gemm_q8_k(ggml_type: int, weights: np.ndarray, rows: int, width: int,
              blocks: np.ndarray, batch: int) -> np.ndarray:
    out = np.zeros((batch, rows), np.float32)
    rc = load().q38o_gemm_q8_k(ggml_type, _w(weights), rows, width,
                               c_void_p(blocks.ctypes.data), batch, _p(out))
    if rc != 0:
        raise ValueError("gemm_q8_k: unsupported type or shape")
    return out


def gemm_f32(ggml_type: int, weights: np.ndarray, rows: int, width: int, x: np.ndarray,
             batch: int) -> np.ndarray:
    x = np.ascontiguousarray(x, np.float32)
    out = np.zeros((batch, rows), np.float32)
    if load().q38o_gemm_f32(ggml_type, _w(weights), rows, width, _p(x), batch, _p(out)) != 0:
        raise ValueError("gemm_f32: unsupported type or shape")
    return out


def project(ggml_type: int, weights: np.ndarray, rows: int, width: int,
            x: np.ndarray) -> np.ndarray:
    """project / batch_project (src/model/ops.rs:623-640, 1016-1031): x is
    [batch][width] f32; returns [batch][rows]."""
    x = np.ascontiguousarray(x, np.float32).reshape(-1, width)
    out = np.zeros((x.shape[0], rows), np.float32)
    rc = load().q38o_project(ggml_type, _w(weights), rows, width, _p(x), x.shape[0], _p(out))
    if rc != 0:
        raise ValueError("project: unsupported type or shape")
    return out


def dot_row_f32(ggml_type: int, row: np.ndarray, x: np.ndarray) -> float:
    x = np.ascontiguousarray(x, np.float32)
    return float(load().q38o_dot_row_f32(ggml_type, _w(row), _p(x), x.size))


def dot_row_q8_k(ggml_type: int, row: np.ndarray, blocks: np.ndarray) -> float:
    return float(load().q38o_dot_row_q8_k(ggml_type, _w(row), c_void_p(blocks.ctypes.data),
                                          blocks.size))

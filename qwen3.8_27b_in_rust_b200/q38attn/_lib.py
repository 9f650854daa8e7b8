"""ctypes binding of libq38attn.so (include/q38attn.h).

The library is loaded from the package directory; there is no fallback: if it
is missing, loading raises and nothing computes.
"""
from __future__ import annotations

import ctypes
import threading
from ctypes import POINTER, c_char_p, c_float, c_int, c_int32, c_size_t, c_uint32, c_void_p
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent.parent / "libq38attn.so"
HEADER_PATH = Path(__file__).resolve().parents[2] / "include" / "q38attn.h"

Q38_OK = 0
Q38_ERR_ARG = -1
Q38_ERR_CUDA = -2
Q38_ERR_TIMEOUT = -3
Q38_KV_F32 = 0
Q38_KV_BF16 = 1
Q38_DEVERR_POSITION = 1
Q38_DEVERR_TIMEOUT = 2
Q38_DEVERR_SHAPE = 4
Q38_DEVERR_RANGE = 8
Q38_DEBUG_SKIP_KV_LOADS = 1
Q38_NCCL_ID_BYTES = 128
Q38_IPC_HANDLE_BYTES = 64
Q38_GGML_F32, Q38_GGML_F16, Q38_GGML_Q8_0, Q38_GGML_BF16 = 0, 1, 8, 30
Q38_GGML_Q2_K, Q38_GGML_Q3_K, Q38_GGML_Q4_K, Q38_GGML_Q5_K, Q38_GGML_Q6_K = 10, 11, 12, 13, 14
Q38_GGML_IQ4_NL, Q38_GGML_IQ4_XS = 20, 23
Q38_Q8K_BLOCK_BYTES = 292


class Q38Geom(ctypes.Structure):
    _fields_ = [
        ("attn_heads", c_int32),
        ("attn_kv_heads", c_int32),
        ("attn_head_dim", c_int32),
        ("rope_dims", c_int32),
        ("rope_theta", c_float),
        ("linear_qk_heads", c_int32),
        ("linear_v_heads", c_int32),
        ("linear_head_dim", c_int32),
        ("conv_kernel", c_int32),
        ("rms_eps", c_float),
    ]


class Q38Error(RuntimeError):
    """A non-zero status from the C ABI (code -1 argument, -2 CUDA, -3 timeout)."""

    def __init__(self, code: int, message: str):
        super().__init__(f"q38attn error {code}: {message}")
        self.code = code


_FP = POINTER(c_float)
_IP = POINTER(c_int32)
_VP = c_void_p

# name -> (restype, argtypes); every function in include/q38attn.h.
SIGNATURES = {
    "q38_geom_default": (None, [POINTER(Q38Geom)]),
    "q38_last_error": (c_char_p, []),
    "q38_version": (c_char_p, []),
    "q38_ctx_create": (c_int, [POINTER(Q38Geom), c_int, POINTER(c_void_p)]),
    "q38_ctx_destroy": (c_int, [_VP]),
    "q38_bind_full_layer": (c_int, [_VP, c_int, _VP, _VP]),
    "q38_bind_linear_layer": (c_int, [_VP, c_int, _VP, _VP, _VP, _VP]),
    "q38_gguf_read_f32": (c_int, [c_char_p, c_char_p, _VP, ctypes.c_int64]),
    "q38_bind_gguf": (c_int, [_VP, c_char_p, c_int, c_int]),
    "q38_state_create": (c_int, [_VP, c_int, c_int, c_int, c_int, c_int, POINTER(c_void_p)]),
    "q38_state_destroy": (c_int, [_VP]),
    "q38_state_reset": (c_int, [_VP, _VP]),
    "q38_state_errors": (c_int, [_VP, POINTER(c_int)]),
    "q38_state_set_debug": (c_int, [_VP, c_int, ctypes.c_uint64]),
    "q38_state_reserve_split": (c_int, [_VP, c_int]),
    "q38_full_decode_split": (c_int, [_VP, _VP, c_int, c_int, _VP, _VP, _VP, _VP, c_int, c_int,
                                      _VP, _VP, _VP]),
    "q38_state_split_p2p_handle": (c_int, [_VP, c_int, _VP]),
    "q38_state_split_p2p_open": (c_int, [_VP, c_int, _VP]),
    "q38_full_decode_split_p2p": (c_int, [_VP, _VP, c_int, c_int, _VP, _VP, _VP, _VP, c_int,
                                          c_int, _VP, _VP]),
    "q38_nccl_unique_id": (c_int, [_VP]),
    "q38_nccl_comm_create": (c_int, [_VP, c_int, c_int, c_int, POINTER(c_void_p)]),
    "q38_nccl_comm_destroy": (c_int, [_VP]),
    "q38_full_prefill_heads": (c_int, [_VP, _VP, c_int, c_int, c_int, c_int, c_int, c_int, c_int,
                                       _VP, _VP, _VP, _VP, _VP]),
    "q38_linear_prefill_heads": (c_int, [_VP, _VP, c_int, c_int, c_int, c_int, c_int, c_int, _VP,
                                         _VP, _VP, _VP, _VP, _VP]),
    "q38_state_full_slot": (c_int, [_VP, c_int, POINTER(c_void_p), POINTER(c_void_p),
                                    POINTER(c_size_t)]),
    "q38_state_linear_slot": (c_int, [_VP, c_int, POINTER(c_void_p), POINTER(c_void_p)]),
    "q38_state_upload_kv": (c_int, [_VP, c_int, c_int, c_int, c_int, _VP, _VP]),
    "q38_state_download_kv": (c_int, [_VP, c_int, c_int, c_int, c_int, _VP, _VP]),
    "q38_state_upload_linear": (c_int, [_VP, c_int, c_int, _VP, _VP]),
    "q38_state_download_linear": (c_int, [_VP, c_int, c_int, _VP, _VP]),
    "q38_full_decode": (c_int, [_VP, _VP, c_int, c_int, _VP, _VP, _VP, _VP, c_int, _VP, _VP]),
    "q38_full_decode_shard": (c_int, [_VP, _VP, c_int, c_int, _VP, _VP, _VP, _VP, c_int, c_int,
                                      _VP, _VP]),
    "q38_attn_merge_shards": (c_int, [_VP, c_int, c_int, _VP, _VP, _VP, _VP]),
    "q38_linear_decode": (c_int, [_VP, _VP, c_int, c_int, _VP, _VP, _VP, _VP, _VP, _VP]),
    "q38_full_decode_noalloc": (c_int, [_VP, _VP, _VP, _VP, c_int, c_int, c_int, _VP, _VP, _VP,
                                        _VP, c_int, _VP, _VP, _VP]),
    "q38_state_reserve_prefill": (c_int, [_VP, c_int]),
    "q38_state_checkpoint": (c_int, [_VP, c_int, c_int, _VP]),
    "q38_state_restore": (c_int, [_VP, c_int, c_int, _VP]),
    "q38_full_prefill": (c_int, [_VP, _VP, c_int, c_int, c_int, c_int, c_int, _VP, _VP, _VP, _VP,
                                 _VP]),
    "q38_linear_prefill": (c_int, [_VP, _VP, c_int, c_int, c_int, c_int, _VP, _VP, _VP, _VP,
                                   _VP, _VP]),
    "q38_full_prefill_host": (c_int, [_VP, _VP, c_int, c_int, c_int, c_int, c_int, _VP, _VP,
                                      _VP, _VP, _VP]),
    "q38_linear_prefill_host": (c_int, [_VP, _VP, c_int, c_int, c_int, c_int, _VP, _VP, _VP,
                                        _VP, _VP, _VP]),
    "q38_full_decode_host": (c_int, [_VP, _VP, c_int, c_int, _VP, _VP, _VP, _VP, _VP, _VP]),
    "q38_linear_decode_host": (c_int, [_VP, _VP, c_int, c_int, _VP, _VP, _VP, _VP, _VP, _VP]),
    "q38_linear_core": (c_int, [_VP, _VP, c_int, _VP, _VP, _VP, _VP, _VP, _VP, _VP]),
    "q38_full_core": (c_int, [_VP, _VP, c_int, _VP, _VP, _VP, _VP, _VP, _VP, _VP, _VP, _VP,
                              c_size_t, c_size_t, c_uint32]),
    "q38_weight_create": (c_int, [_VP, c_int, ctypes.c_int64, ctypes.c_int64, _VP, c_size_t,
                                  POINTER(c_void_p)]),
    "q38_weight_destroy": (c_int, [_VP]),
    "q38_weight_build_planes": (c_int, [_VP]),
    "q38_weight_info": (c_int, [_VP, POINTER(c_int), POINTER(ctypes.c_int64),
                                POINTER(ctypes.c_int64)]),
    "q38_weight_from_gguf": (c_int, [_VP, c_char_p, c_char_p, POINTER(c_void_p)]),
    "q38_quantize_q8_k": (c_int, [_VP, c_int, ctypes.c_int64, _VP, _VP, _VP]),
    "q38_project": (c_int, [_VP, _VP, c_int, _VP, _VP, _VP]),
    "q38_project_host": (c_int, [_VP, _VP, c_int, _VP, _VP]),
    "q38_ctx_reserve_projection": (c_int, [_VP, c_int, ctypes.c_int64]),
    "q38_linear_attention_decode": (c_int, [_VP, _VP, c_int, c_int, _VP, _VP, _VP, _VP]),
    "q38_full_attention_decode": (c_int, [_VP, _VP, c_int, c_int, _VP, _VP, _VP, c_int, _VP,
                                          _VP]),
    "q38_state_reserve_attention_prefill": (c_int, [_VP, c_int]),
    "q38_linear_attention_prefill": (c_int, [_VP, _VP, c_int, c_int, c_int, c_int, _VP, _VP, _VP,
                                             _VP]),
    "q38_full_attention_prefill": (c_int, [_VP, _VP, c_int, c_int, c_int, c_int, c_int, _VP, _VP,
                                           _VP, _VP]),
}

_lock = threading.Lock()
_lib = None


def load() -> ctypes.CDLL:
    """Loads libq38attn.so once and declares every exported signature."""
    global _lib
    with _lock:
        if _lib is None:
            if not LIB_PATH.exists():
                raise FileNotFoundError(
                    f"{LIB_PATH} is missing; build it with `python qwen3.8_27b_in_rust_b200/build.py`")
            lib = ctypes.CDLL(str(LIB_PATH))
            for name, (res, args) in SIGNATURES.items():
                fn = getattr(lib, name)
                fn.restype = res
                fn.argtypes = args
            _lib = lib
        return _lib


def last_error() -> str:
    return load().q38_last_error().decode()


def check(rc: int) -> None:
    if rc != Q38_OK:
        raise Q38Error(rc, last_error())

"""q38attn -- host-side mirror of the reference's attention hot path over the
B200 C ABI (include/q38attn.h, libq38attn.so).

The reference (StepfenShawn/qwen3.8_27b_in_rust) calls two crate-private
functions per layer:

* ``linear_core`` (src/model/ops.rs:647-742), the Gated DeltaNet step, and
* ``full_core`` (src/model/ops.rs:812-940), the gated full-attention step,

once per token, including inside the prefill loops (ops.rs:1088-1099,
1156-1172). :class:`Context` exposes the same operations with the same names
and argument meaning, backed only by the sm_100a kernels:

* :meth:`Context.linear_core` / :meth:`Context.full_core` take host (numpy)
  slices exactly like the Rust signatures and write every ``&mut`` argument
  back; they are the parity surface.
* :meth:`Context.linear_decode` / :meth:`Context.full_decode` take device
  tensors for a batch of sequences whose state stays resident in a
  :class:`State`; they are the serving surface.

Errors follow the reference's convention: an argument error (the Rust
``Err(-1)``) raises :class:`Q38Error` with ``code == -1``. There is no CPU
fallback: without the built library or a B200 nothing runs.
"""
from __future__ import annotations

import ctypes
from typing import Optional

import numpy as np

from ._lib import (Q38_DEBUG_SKIP_KV_LOADS, Q38_DEVERR_RANGE, Q38_IPC_HANDLE_BYTES,
                   Q38_NCCL_ID_BYTES,
                   Q38_DEVERR_POSITION, Q38_DEVERR_SHAPE, Q38_DEVERR_TIMEOUT, Q38_ERR_ARG,
                   Q38_ERR_CUDA, Q38_ERR_TIMEOUT, Q38_GGML_BF16, Q38_GGML_F16, Q38_GGML_F32,
                   Q38_GGML_IQ4_NL, Q38_GGML_IQ4_XS, Q38_GGML_Q2_K, Q38_GGML_Q3_K,
                   Q38_GGML_Q4_K, Q38_GGML_Q5_K, Q38_GGML_Q6_K, Q38_GGML_Q8_0, Q38_KV_BF16, Q38_KV_F32, Q38_OK, Q38_Q8K_BLOCK_BYTES, Q38Error,
                   Q38Geom, check, last_error, load)

__all__ = [
    "Context", "State", "Q38Error", "Q38Geom", "geometry", "load", "last_error",
    "Q38_OK", "Q38_ERR_ARG", "Q38_ERR_CUDA", "Q38_ERR_TIMEOUT", "Q38_KV_F32", "Q38_KV_BF16",
    "Q38_DEVERR_POSITION", "Q38_DEVERR_TIMEOUT", "Q38_DEVERR_SHAPE", "Q38_DEVERR_RANGE",
    "Q38_DEBUG_SKIP_KV_LOADS", "Q38_NCCL_ID_BYTES", "nccl_unique_id", "NcclComm",
    "Q38_IPC_HANDLE_BYTES",
    "is_full_attention", "full_index", "recurrent_index", "gguf_read_f32", "Weight",
    "Q38_GGML_F32", "Q38_GGML_F16", "Q38_GGML_BF16", "Q38_GGML_Q8_0", "Q38_GGML_Q2_K",
    "Q38_GGML_Q3_K", "Q38_GGML_Q4_K", "Q38_GGML_Q5_K", "Q38_GGML_Q6_K", "Q38_GGML_IQ4_NL",
    "Q38_GGML_IQ4_XS", "Q38_Q8K_BLOCK_BYTES",
    "row_bytes",
]

# ggml (elements, bytes) per block of the projection types (src/gguf/mod.rs:136-178).
_GGML_BLOCK = {Q38_GGML_F32: (1, 4), Q38_GGML_F16: (1, 2), Q38_GGML_BF16: (1, 2),
               Q38_GGML_Q8_0: (32, 34), Q38_GGML_Q2_K: (256, 84), Q38_GGML_Q3_K: (256, 110),
               Q38_GGML_Q4_K: (256, 144), Q38_GGML_Q5_K: (256, 176), Q38_GGML_Q6_K: (256, 210),
               Q38_GGML_IQ4_NL: (32, 18), Q38_GGML_IQ4_XS: (256, 136)}


def row_bytes(ggml_type: int, width: int) -> int:
    """row_bytes (src/kernel/tensor.rs:46-53) of the projection types."""
    el, by = _GGML_BLOCK[ggml_type]
    if width % el:
        raise ValueError(f"width {width} is not a whole number of {el}-element blocks")
    return width // el * by

# Geometry of src/model/mod.rs:13-26.
ATTN_HEADS = 24
ATTN_KV_HEADS = 4
ATTN_HEAD_DIM = 256
ATTN_Q_DIM = 6144
ATTN_QG_DIM = 12288
ATTN_KV_DIM = 1024
LINEAR_QK_HEADS = 16
LINEAR_V_HEADS = 48
LINEAR_HEAD_DIM = 128
LINEAR_QK_DIM = 2048
LINEAR_V_DIM = 6144
LINEAR_QKV_DIM = 10240
RMS_EPS = 1e-6
FULL_SLOTS = 17     # Q38_TOTAL_FULL_LAYERS
LINEAR_SLOTS = 48   # Q38_RECURRENT_LAYERS


def is_full_attention(layer: int) -> bool:
    """src/model/ops.rs:39-41."""
    return (layer + 1) % 4 == 0 or layer == 64


def full_index(layer: int) -> int:
    return layer // 4


def recurrent_index(layer: int) -> int:
    """src/model/ops.rs:45-47."""
    return layer - (layer + 1) // 4


def geometry() -> Q38Geom:
    g = Q38Geom()
    load().q38_geom_default(ctypes.byref(g))
    return g


def _host_ptr(a, name: str, writable: bool = False, dtype=np.float32):
    if a is None:
        return None
    if not isinstance(a, np.ndarray):
        raise TypeError(f"{name} must be a numpy array")
    if a.dtype != dtype or not a.flags.c_contiguous:
        raise TypeError(f"{name} must be a C-contiguous {np.dtype(dtype).name} array")
    if writable and not a.flags.writeable:
        raise TypeError(f"{name} must be writable")
    return ctypes.c_void_p(a.ctypes.data)


def _host_len(a, n: int, name: str):
    if a is not None and a.size < n:
        raise Q38Error(Q38_ERR_ARG, f"{name} holds {a.size} values, needs {n}")


def _dev_ptr(t, name: str, dtype_name: str = "float32"):
    import torch
    if not isinstance(t, torch.Tensor) or not t.is_cuda:
        raise TypeError(f"{name} must be a CUDA tensor")
    if str(t.dtype) != f"torch.{dtype_name}" or not t.is_contiguous():
        raise TypeError(f"{name} must be a contiguous {dtype_name} CUDA tensor")
    return ctypes.c_void_p(t.data_ptr())


class _CudaArray:
    """Minimal __cuda_array_interface__ holder for wrapping library memory."""

    def __init__(self, ptr: int, shape: tuple, typestr: str):
        self.__cuda_array_interface__ = {
            "data": (int(ptr), False), "shape": tuple(shape), "typestr": typestr,
            "strides": None, "version": 2,
        }


def _cai_tensor(ptr: int, shape: tuple, typestr: str):
    import torch
    return torch.as_tensor(_CudaArray(ptr, shape, typestr), device="cuda")


def _stream_ptr(stream):
    if stream is None:
        import torch
        return ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    if isinstance(stream, int):
        return ctypes.c_void_p(stream)
    return ctypes.c_void_p(stream.cuda_stream)


class State:
    """Device-resident per-sequence state: KV caches, conv and delta states
    (the Q38Model fields of src/model/mod.rs:155-158)."""

    def __init__(self, ctx: "Context", batch: int, context_length: int,
                 full_slots: int = FULL_SLOTS, linear_slots: int = LINEAR_SLOTS,
                 kv_dtype: int = Q38_KV_F32):
        self._lib = load()
        self.ctx = ctx
        self.batch = batch
        self.context_length = context_length
        self.full_slots = full_slots
        self.linear_slots = linear_slots
        self.kv_dtype = kv_dtype
        h = ctypes.c_void_p()
        check(self._lib.q38_state_create(ctx.handle, batch, context_length, full_slots,
                                         linear_slots, kv_dtype, ctypes.byref(h)))
        self.handle = h

    def close(self) -> None:
        if self.handle:
            check(self._lib.q38_state_destroy(self.handle))
            self.handle = ctypes.c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def reset(self, stream=None) -> None:
        check(self._lib.q38_state_reset(self.handle, _stream_ptr(stream)))

    def errors(self) -> int:
        bits = ctypes.c_int(0)
        check(self._lib.q38_state_errors(self.handle, ctypes.byref(bits)))
        return bits.value

    def full_slot_ptrs(self, layer: int):
        k, v, n = ctypes.c_void_p(), ctypes.c_void_p(), ctypes.c_size_t()
        check(self._lib.q38_state_full_slot(self.handle, layer, ctypes.byref(k),
                                            ctypes.byref(v), ctypes.byref(n)))
        return k.value, v.value, n.value

    def linear_slot_ptrs(self, layer: int):
        c, d = ctypes.c_void_p(), ctypes.c_void_p()
        check(self._lib.q38_state_linear_slot(self.handle, layer, ctypes.byref(c),
                                              ctypes.byref(d)))
        return c.value, d.value

    def reserve_prefill(self, max_tokens: int) -> None:
        check(self._lib.q38_state_reserve_prefill(self.handle, max_tokens))

    def reserve_split(self, nranks: int) -> None:
        """Sizes the buffers of split-sequence decode over `nranks` ranks."""
        check(self._lib.q38_state_reserve_split(self.handle, nranks))

    def split_p2p_handle(self, nranks: int) -> bytes:
        """Allocates this rank's split-sequence exchange buffer for `nranks`
        ranks and returns its CUDA IPC handle (q38_state_split_p2p_handle)."""
        buf = ctypes.create_string_buffer(Q38_IPC_HANDLE_BYTES)
        check(self._lib.q38_state_split_p2p_handle(self.handle, nranks, buf))
        return buf.raw

    def split_p2p_open(self, rank: int, handles: list) -> None:
        """Maps every peer's exchange buffer (handles: every rank's, in rank order)."""
        blob = b"".join(handles)
        buf = ctypes.create_string_buffer(blob, len(blob))
        check(self._lib.q38_state_split_p2p_open(self.handle, rank, buf))

    def set_debug(self, flags: int = 0, wait_ns: int = 0) -> None:
        """Error-path testing (q38_state_set_debug): Q38_DEBUG_SKIP_KV_LOADS
        makes the decode's split kernel load nothing, so its waits run out
        after wait_ns; set_debug() restores normal operation."""
        check(self._lib.q38_state_set_debug(self.handle, flags, wait_ns))

    def reserve_attention_prefill(self, max_tokens: int) -> None:
        check(self._lib.q38_state_reserve_attention_prefill(self.handle, max_tokens))

    def checkpoint(self, seq0: int = 0, nseq: Optional[int] = None, stream=None) -> None:
        """Keep the recurrent (conv + delta) state of sequences [seq0, seq0+nseq)
        for a later restore (checkpoint_state, src/model/ops.rs:1627-1640)."""
        nseq = self.batch - seq0 if nseq is None else nseq
        check(self._lib.q38_state_checkpoint(self.handle, seq0, nseq, _stream_ptr(stream)))

    def restore(self, seq0: int = 0, nseq: Optional[int] = None, stream=None) -> None:
        """Roll the recurrent state of sequences [seq0, seq0+nseq) back to their
        checkpoint (restore_target_state, src/model/ops.rs:1642-1647)."""
        nseq = self.batch - seq0 if nseq is None else nseq
        check(self._lib.q38_state_restore(self.handle, seq0, nseq, _stream_ptr(stream)))

    def kv_views(self, layer: int):
        """Zero-copy torch views of one KV slot, [batch][kv_heads][context][256]
        (bf16 or f32), for bulk device-side initialisation."""
        import torch
        k, v, _ = self.full_slot_ptrs(layer)
        shape = (self.batch, ATTN_KV_HEADS, self.context_length, ATTN_HEAD_DIM)
        if self.kv_dtype == Q38_KV_BF16:
            return (_cai_tensor(k, shape, "<i2").view(torch.bfloat16),
                    _cai_tensor(v, shape, "<i2").view(torch.bfloat16))
        return _cai_tensor(k, shape, "<f4"), _cai_tensor(v, shape, "<f4")

    def linear_views(self, layer: int):
        """Zero-copy torch views of one recurrent slot: conv state
        [batch][qkv_dim][3] and delta state [batch][v_heads][128][128], f32."""
        c, d = self.linear_slot_ptrs(layer)
        return (_cai_tensor(c, (self.batch, LINEAR_QKV_DIM, 3), "<f4"),
                _cai_tensor(d, (self.batch, LINEAR_V_HEADS, LINEAR_HEAD_DIM, LINEAR_HEAD_DIM),
                            "<f4"))

    def upload_kv(self, layer: int, seq: int, first: int, key_rows: np.ndarray,
                  value_rows: np.ndarray) -> None:
        count = key_rows.shape[0] if key_rows.ndim > 1 else key_rows.size // ATTN_KV_DIM
        check(self._lib.q38_state_upload_kv(self.handle, layer, seq, first, count,
                                            _host_ptr(key_rows, "key_rows"),
                                            _host_ptr(value_rows, "value_rows")))

    def download_kv(self, layer: int, seq: int, first: int, count: int):
        k = np.empty((count, ATTN_KV_DIM), np.float32)
        v = np.empty((count, ATTN_KV_DIM), np.float32)
        check(self._lib.q38_state_download_kv(self.handle, layer, seq, first, count,
                                              _host_ptr(k, "k", True), _host_ptr(v, "v", True)))
        return k, v

    def upload_linear(self, layer: int, seq: int, conv_state: Optional[np.ndarray],
                      delta_state: Optional[np.ndarray]) -> None:
        check(self._lib.q38_state_upload_linear(self.handle, layer, seq,
                                                _host_ptr(conv_state, "conv_state"),
                                                _host_ptr(delta_state, "delta_state")))

    def download_linear(self, layer: int, seq: int):
        c = np.empty((LINEAR_QKV_DIM, 3), np.float32)
        d = np.empty((LINEAR_V_HEADS, LINEAR_HEAD_DIM, LINEAR_HEAD_DIM), np.float32)
        check(self._lib.q38_state_download_linear(self.handle, layer, seq,
                                                  _host_ptr(c, "c", True),
                                                  _host_ptr(d, "d", True)))
        return c, d


def gguf_read_f32(path, name: str, count: int) -> np.ndarray:
    """The F32 tensor `name` of a GGUF checkpoint (count elements), read by
    the library's parser (the checks of Gguf::open, src/gguf/mod.rs:459-533).
    Host only; raises Q38Error(-1) on a malformed file or a missing, non-F32
    or differently sized tensor."""
    out = np.empty(count, np.float32)
    check(load().q38_gguf_read_f32(str(path).encode(), name.encode(),
                                   out.ctypes.data_as(ctypes.c_void_p), count))
    return out


def nccl_unique_id() -> bytes:
    """A fresh NCCL unique id (Q38_NCCL_ID_BYTES bytes) for q38_nccl_comm_create,
    made on one rank and sent to the others by the host."""
    buf = ctypes.create_string_buffer(Q38_NCCL_ID_BYTES)
    check(load().q38_nccl_unique_id(buf))
    return buf.raw


class NcclComm:
    """An NCCL communicator made by the library (q38_nccl_comm_create); every
    rank of the group must construct it with the same id."""

    def __init__(self, unique_id: bytes, nranks: int, rank: int, device: int):
        if len(unique_id) != Q38_NCCL_ID_BYTES:
            raise ValueError("an NCCL unique id has 128 bytes")
        self._lib = load()
        h = ctypes.c_void_p()
        buf = ctypes.create_string_buffer(unique_id, Q38_NCCL_ID_BYTES)
        check(self._lib.q38_nccl_comm_create(buf, nranks, rank, device, ctypes.byref(h)))
        self.handle = h
        self.nranks, self.rank = nranks, rank

    def close(self) -> None:
        if self.handle:
            check(self._lib.q38_nccl_comm_destroy(self.handle))
            self.handle = ctypes.c_void_p()


class Weight:
    """A projection matrix on the device: ``rows`` outputs over ``width``
    inputs, the GGUF tensor of shape [width, rows] (q38_weight_create)."""

    def __init__(self, ctx: "Context", handle: ctypes.c_void_p):
        self._lib = ctx._lib
        self.ctx = ctx
        self.handle = handle
        t, w, r = ctypes.c_int(), ctypes.c_int64(), ctypes.c_int64()
        check(self._lib.q38_weight_info(handle, ctypes.byref(t), ctypes.byref(w), ctypes.byref(r)))
        self.ggml_type, self.width, self.rows = t.value, w.value, r.value

    def build_planes(self) -> "Weight":
        """Builds the weight's integer planes (q38_weight_build_planes): later
        projections of 9+ tokens stream them on the tensor cores."""
        check(self._lib.q38_weight_build_planes(self.handle))
        return self

    def close(self) -> None:
        if self.handle:
            check(self._lib.q38_weight_destroy(self.handle))
            self.handle = ctypes.c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class _LinearProjections(ctypes.Structure):
    _fields_ = [("qkv", ctypes.c_void_p), ("z", ctypes.c_void_p), ("beta", ctypes.c_void_p),
                ("alpha", ctypes.c_void_p), ("out", ctypes.c_void_p)]


class _FullProjections(ctypes.Structure):
    _fields_ = [("q", ctypes.c_void_p), ("k", ctypes.c_void_p), ("v", ctypes.c_void_p),
                ("out", ctypes.c_void_p)]


class Context:
    """A device, the model geometry and the bound per-layer weights
    (the weight half of Q38Model::bind, src/model/ops.rs:1450-1459)."""

    def __init__(self, device: int = 0, geom: Optional[Q38Geom] = None):
        self._lib = load()
        h = ctypes.c_void_p()
        check(self._lib.q38_ctx_create(ctypes.byref(geom) if geom is not None else None,
                                       device, ctypes.byref(h)))
        self.handle = h
        self.device = device
        self._states = []

    def close(self) -> None:
        if self.handle:
            check(self._lib.q38_ctx_destroy(self.handle))
            self.handle = ctypes.c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    # weights -------------------------------------------------------------
    def bind_full_layer(self, layer: int, q_norm: np.ndarray, k_norm: np.ndarray) -> None:
        _host_len(q_norm, ATTN_HEAD_DIM, "q_norm")
        _host_len(k_norm, ATTN_HEAD_DIM, "k_norm")
        check(self._lib.q38_bind_full_layer(self.handle, layer, _host_ptr(q_norm, "q_norm"),
                                            _host_ptr(k_norm, "k_norm")))

    def bind_linear_layer(self, layer: int, conv1d: np.ndarray, dt_bias: np.ndarray,
                          ssm_a: np.ndarray, ssm_norm: np.ndarray) -> None:
        _host_len(conv1d, LINEAR_QKV_DIM * 4, "conv1d")
        _host_len(dt_bias, LINEAR_V_HEADS, "dt_bias")
        _host_len(ssm_a, LINEAR_V_HEADS, "ssm_a")
        _host_len(ssm_norm, LINEAR_HEAD_DIM, "ssm_norm")
        check(self._lib.q38_bind_linear_layer(self.handle, layer, _host_ptr(conv1d, "conv1d"),
                                              _host_ptr(dt_bias, "dt_bias"),
                                              _host_ptr(ssm_a, "ssm_a"),
                                              _host_ptr(ssm_norm, "ssm_norm")))

    def bind_gguf(self, path, first_layer: int, last_layer: int) -> None:
        """Binds layers first_layer..last_layer (64 = MTP) from a GGUF
        checkpoint by the reference's tensor names (ops.rs:53-100)."""
        check(self._lib.q38_bind_gguf(self.handle, str(path).encode(), first_layer, last_layer))

    # projections ----------------------------------------------------------
    def weight(self, ggml_type: int, width: int, rows: int, data: np.ndarray) -> Weight:
        """Uploads a projection matrix: data holds the GGUF tensor's bytes
        (rows * row_bytes(ggml_type, width) uint8)."""
        data = np.ascontiguousarray(data).view(np.uint8).reshape(-1)
        h = ctypes.c_void_p()
        check(self._lib.q38_weight_create(self.handle, ggml_type, width, rows,
                                          ctypes.c_void_p(data.ctypes.data), data.size,
                                          ctypes.byref(h)))
        return Weight(self, h)

    def weight_from_gguf(self, path, name: str) -> Weight:
        h = ctypes.c_void_p()
        check(self._lib.q38_weight_from_gguf(self.handle, str(path).encode(), name.encode(),
                                             ctypes.byref(h)))
        return Weight(self, h)

    def reserve_projection(self, batch: int, width: int) -> None:
        check(self._lib.q38_ctx_reserve_projection(self.handle, batch, width))

    def quantize_q8_k(self, x, blocks, stream=None) -> None:
        """quantize_q8_k of x [batch][width] (CUDA f32) into blocks (CUDA
        uint8, batch*width/256*292 bytes, the reference's block layout)."""
        b, width = x.shape
        check(self._lib.q38_quantize_q8_k(self.handle, b, width, _dev_ptr(x, "x"),
                                          _dev_ptr(blocks, "blocks", "uint8"),
                                          _stream_ptr(stream)))

    def project(self, w: Weight, x, out, stream=None) -> None:
        """project / batch_project: out [batch][rows] = W x [batch][width] (CUDA f32)."""
        check(self._lib.q38_project(self.handle, w.handle, x.shape[0], _dev_ptr(x, "x"),
                                    _dev_ptr(out, "out"), _stream_ptr(stream)))

    def project_host(self, w: Weight, x: np.ndarray) -> np.ndarray:
        x = np.ascontiguousarray(x, np.float32).reshape(-1, w.width)
        out = np.zeros((x.shape[0], w.rows), np.float32)
        check(self._lib.q38_project_host(self.handle, w.handle, x.shape[0], _host_ptr(x, "x"),
                                         _host_ptr(out, "out", True)))
        return out

    def linear_attention_decode(self, state: "State", layer: int, weights: dict, norm, branch,
                                stream=None) -> None:
        """linear_attention (ops.rs:744-803): weights has Weight values for
        qkv, z, beta, alpha, out; norm and branch are [batch][hidden] CUDA f32."""
        p = _LinearProjections(*(weights[k].handle for k in ("qkv", "z", "beta", "alpha", "out")))
        check(self._lib.q38_linear_attention_decode(
            self.handle, state.handle, layer, norm.shape[0], ctypes.byref(p),
            _dev_ptr(norm, "norm"), _dev_ptr(branch, "branch"), _stream_ptr(stream)))

    def full_attention_decode(self, state: "State", layer: int, weights: dict, norm, positions,
                              branch, max_position: int = -1, stream=None) -> None:
        """full_attention (ops.rs:941-981): weights has Weight values for q,
        k, v, out."""
        p = _FullProjections(*(weights[k].handle for k in ("q", "k", "v", "out")))
        check(self._lib.q38_full_attention_decode(
            self.handle, state.handle, layer, norm.shape[0], ctypes.byref(p),
            _dev_ptr(norm, "norm"), _dev_ptr(positions, "positions", "int32"), max_position,
            _dev_ptr(branch, "branch"), _stream_ptr(stream)))

    def linear_attention_prefill(self, state: "State", layer: int, seq0: int, weights: dict, norm,
                                 branch, stream=None) -> None:
        """batch_linear_attention (ops.rs:1032-1114): norm and branch are
        [nseq][count][hidden] CUDA f32; needs State.reserve_attention_prefill."""
        p = _LinearProjections(*(weights[k].handle for k in ("qkv", "z", "beta", "alpha", "out")))
        nseq, count = norm.shape[0], norm.shape[1]
        check(self._lib.q38_linear_attention_prefill(
            self.handle, state.handle, layer, seq0, nseq, count, ctypes.byref(p),
            _dev_ptr(norm, "norm"), _dev_ptr(branch, "branch"), _stream_ptr(stream)))

    def full_attention_prefill(self, state: "State", layer: int, seq0: int, base_position: int,
                               weights: dict, norm, branch, stream=None) -> None:
        """batch_full_attention (ops.rs:1116-1185) at positions base_position.."""
        p = _FullProjections(*(weights[k].handle for k in ("q", "k", "v", "out")))
        nseq, count = norm.shape[0], norm.shape[1]
        check(self._lib.q38_full_attention_prefill(
            self.handle, state.handle, layer, seq0, nseq, count, base_position, ctypes.byref(p),
            _dev_ptr(norm, "norm"), _dev_ptr(branch, "branch"), _stream_ptr(stream)))

    def state(self, batch: int, context_length: int, full_slots: int = FULL_SLOTS,
              linear_slots: int = LINEAR_SLOTS, kv_dtype: int = Q38_KV_F32) -> State:
        return State(self, batch, context_length, full_slots, linear_slots, kv_dtype)

    # device, batched, stream-ordered --------------------------------------
    def full_decode(self, state: State, layer: int, q_and_gate, key, value, positions,
                    attention, max_position: int = -1, stream=None) -> None:
        b = q_and_gate.shape[0]
        check(self._lib.q38_full_decode(self.handle, state.handle, layer, b,
                                        _dev_ptr(q_and_gate, "q_and_gate"),
                                        _dev_ptr(key, "key"), _dev_ptr(value, "value"),
                                        _dev_ptr(positions, "positions", "int32"),
                                        max_position, _dev_ptr(attention, "attention"),
                                        _stream_ptr(stream)))

    def full_decode_shard(self, state: State, layer: int, q_and_gate, key, value, positions,
                          partials, max_position: int, pos_offset: int, stream=None) -> None:
        """Split-sequence decode, shard side: writes this shard's (o, m, l)
        partials [batch][24][258] over its positions pos_offset.. (see
        q38_full_decode_shard)."""
        b = q_and_gate.shape[0]
        check(self._lib.q38_full_decode_shard(
            self.handle, state.handle, layer, b, _dev_ptr(q_and_gate, "q_and_gate"),
            _dev_ptr(key, "key"), _dev_ptr(value, "value"),
            _dev_ptr(positions, "positions", "int32"), max_position, pos_offset,
            _dev_ptr(partials, "partials"), _stream_ptr(stream)))

    def full_decode_split(self, state: State, layer: int, q_and_gate, key, value, positions,
                          attention, max_position: int, pos_offset: int, comm, stream=None) -> None:
        """Split-sequence decode in one call: shard partials, NCCL all-gather
        over `comm` (an NcclComm or a raw ncclComm_t address), merge."""
        b = q_and_gate.shape[0]
        handle = comm.handle if isinstance(comm, NcclComm) else ctypes.c_void_p(comm)
        check(self._lib.q38_full_decode_split(
            self.handle, state.handle, layer, b, _dev_ptr(q_and_gate, "q_and_gate"),
            _dev_ptr(key, "key"), _dev_ptr(value, "value"),
            _dev_ptr(positions, "positions", "int32"), max_position, pos_offset, handle,
            _dev_ptr(attention, "attention"), _stream_ptr(stream)))

    def full_decode_split_p2p(self, state: State, layer: int, q_and_gate, key, value, positions,
                              attention, max_position: int, pos_offset: int, stream=None) -> None:
        """Split-sequence decode with the exchange fused into the merge kernel
        (peer-memory stores and flags; State.split_p2p_open first)."""
        b = q_and_gate.shape[0]
        check(self._lib.q38_full_decode_split_p2p(
            self.handle, state.handle, layer, b, _dev_ptr(q_and_gate, "q_and_gate"),
            _dev_ptr(key, "key"), _dev_ptr(value, "value"),
            _dev_ptr(positions, "positions", "int32"), max_position, pos_offset,
            _dev_ptr(attention, "attention"), _stream_ptr(stream)))

    def merge_shards(self, partials, q_and_gate, attention, stream=None) -> None:
        """Split-sequence decode, merge side: partials [nparts][batch][24][258]."""
        nparts, b = partials.shape[0], partials.shape[1]
        check(self._lib.q38_attn_merge_shards(self.handle, nparts, b,
                                              _dev_ptr(partials, "partials"),
                                              _dev_ptr(q_and_gate, "q_and_gate"),
                                              _dev_ptr(attention, "attention"),
                                              _stream_ptr(stream)))

    def linear_decode(self, state: State, layer: int, qkv, z, beta, alpha, attention,
                      stream=None) -> None:
        b = qkv.shape[0]
        check(self._lib.q38_linear_decode(self.handle, state.handle, layer, b,
                                          _dev_ptr(qkv, "qkv"), _dev_ptr(z, "z"),
                                          _dev_ptr(beta, "beta"), _dev_ptr(alpha, "alpha"),
                                          _dev_ptr(attention, "attention"),
                                          _stream_ptr(stream)))

    def full_prefill(self, state: State, layer: int, seq0: int, q_and_gate, key, value,
                     attention, base_position: int, stream=None) -> None:
        """Causal prefill of q_and_gate.shape[1] tokens for q_and_gate.shape[0]
        sequences starting at seq0 (the per-token full_core loop of
        batch_full_attention, src/model/ops.rs:1156-1172), on tensor cores."""
        nseq, count = q_and_gate.shape[0], q_and_gate.shape[1]
        check(self._lib.q38_full_prefill(self.handle, state.handle, layer, seq0, nseq, count,
                                         base_position, _dev_ptr(q_and_gate, "q_and_gate"),
                                         _dev_ptr(key, "key"), _dev_ptr(value, "value"),
                                         _dev_ptr(attention, "attention"), _stream_ptr(stream)))

    def full_prefill_heads(self, state: State, layer: int, seq0: int, q_and_gate, key, value,
                           attention, base_position: int, kv_head0: int, kv_head_count: int,
                           stream=None) -> None:
        """full_prefill for KV heads [kv_head0, kv_head0 + kv_head_count) only
        (full-width tensors; only the range's columns are touched)."""
        nseq, count = q_and_gate.shape[0], q_and_gate.shape[1]
        check(self._lib.q38_full_prefill_heads(
            self.handle, state.handle, layer, seq0, nseq, count, base_position, kv_head0,
            kv_head_count, _dev_ptr(q_and_gate, "q_and_gate"), _dev_ptr(key, "key"),
            _dev_ptr(value, "value"), _dev_ptr(attention, "attention"), _stream_ptr(stream)))

    def linear_prefill_heads(self, state: State, layer: int, seq0: int, qkv, z, beta, alpha,
                             attention, v_head0: int, v_head_count: int, stream=None) -> None:
        """linear_prefill for value heads [v_head0, v_head0 + v_head_count) only."""
        nseq, count = qkv.shape[0], qkv.shape[1]
        check(self._lib.q38_linear_prefill_heads(
            self.handle, state.handle, layer, seq0, nseq, count, v_head0, v_head_count,
            _dev_ptr(qkv, "qkv"), _dev_ptr(z, "z"), _dev_ptr(beta, "beta"),
            _dev_ptr(alpha, "alpha"), _dev_ptr(attention, "attention"), _stream_ptr(stream)))

    def linear_prefill(self, state: State, layer: int, seq0: int, qkv, z, beta, alpha,
                       attention, stream=None) -> None:
        """Chunked DeltaNet prefill of qkv.shape[1] tokens for qkv.shape[0]
        sequences starting at seq0 (the per-token linear_core loop of
        batch_linear_attention, src/model/ops.rs:1088-1099)."""
        nseq, count = qkv.shape[0], qkv.shape[1]
        check(self._lib.q38_linear_prefill(self.handle, state.handle, layer, seq0, nseq, count,
                                           _dev_ptr(qkv, "qkv"), _dev_ptr(z, "z"),
                                           _dev_ptr(beta, "beta"), _dev_ptr(alpha, "alpha"),
                                           _dev_ptr(attention, "attention"),
                                           _stream_ptr(stream)))

    # host pointers, batched, synchronous -----------------------------------
    def full_decode_host(self, state: State, layer: int, q_and_gate: np.ndarray,
                         key: np.ndarray, value: np.ndarray, positions: np.ndarray,
                         attention: np.ndarray, stream=0) -> None:
        b = q_and_gate.shape[0]
        check(self._lib.q38_full_decode_host(
            self.handle, state.handle, layer, b, _host_ptr(q_and_gate, "q_and_gate"),
            _host_ptr(key, "key", True), _host_ptr(value, "value"),
            _host_ptr(positions, "positions", dtype=np.int32),
            _host_ptr(attention, "attention", True), _stream_ptr(stream)))

    def linear_decode_host(self, state: State, layer: int, qkv: np.ndarray, z: np.ndarray,
                           beta: np.ndarray, alpha: np.ndarray, attention: np.ndarray,
                           stream=0) -> None:
        b = qkv.shape[0]
        check(self._lib.q38_linear_decode_host(
            self.handle, state.handle, layer, b, _host_ptr(qkv, "qkv", True),
            _host_ptr(z, "z"), _host_ptr(beta, "beta", True), _host_ptr(alpha, "alpha", True),
            _host_ptr(attention, "attention", True), _stream_ptr(stream)))

    def full_prefill_host(self, state: State, layer: int, seq0: int, q_and_gate: np.ndarray,
                          key: np.ndarray, value: np.ndarray, attention: np.ndarray,
                          base_position: int, stream=0) -> None:
        """Host-pointer form of full_prefill ([nseq][count][...] numpy arrays):
        the prompt is streamed through the state's staging buffer in pieces
        and the call returns when attention and key are written back."""
        nseq, count = q_and_gate.shape[0], q_and_gate.shape[1]
        check(self._lib.q38_full_prefill_host(
            self.handle, state.handle, layer, seq0, nseq, count, base_position,
            _host_ptr(q_and_gate, "q_and_gate"), _host_ptr(key, "key", True),
            _host_ptr(value, "value"), _host_ptr(attention, "attention", True),
            _stream_ptr(stream)))

    def linear_prefill_host(self, state: State, layer: int, seq0: int, qkv: np.ndarray,
                            z: np.ndarray, beta: np.ndarray, alpha: np.ndarray,
                            attention: np.ndarray, stream=0) -> None:
        """Host-pointer form of linear_prefill; qkv, beta and alpha are
        rewritten in place as the reference's loop leaves them."""
        nseq, count = qkv.shape[0], qkv.shape[1]
        check(self._lib.q38_linear_prefill_host(
            self.handle, state.handle, layer, seq0, nseq, count, _host_ptr(qkv, "qkv", True),
            _host_ptr(z, "z"), _host_ptr(beta, "beta", True), _host_ptr(alpha, "alpha", True),
            _host_ptr(attention, "attention", True), _stream_ptr(stream)))

    # reference-signature mirrors (host slices) ------------------------------
    def linear_core(self, state: State, layer: int, conv_state: np.ndarray,
                    delta_state: np.ndarray, qkv: np.ndarray, z: np.ndarray, beta: np.ndarray,
                    alpha: np.ndarray, attention: np.ndarray) -> None:
        """linear_core(weights, conv_state, delta_state, qkv, z, beta, alpha,
        attention), src/model/ops.rs:647-657: every &mut slice is updated."""
        _host_len(conv_state, LINEAR_QKV_DIM * 3, "conv_state")
        _host_len(delta_state, LINEAR_V_HEADS * LINEAR_HEAD_DIM ** 2, "delta_state")
        _host_len(qkv, LINEAR_QKV_DIM, "qkv")
        _host_len(z, LINEAR_V_DIM, "z")
        _host_len(beta, LINEAR_V_HEADS, "beta")
        _host_len(alpha, LINEAR_V_HEADS, "alpha")
        _host_len(attention, LINEAR_V_DIM, "attention")
        check(self._lib.q38_linear_core(
            self.handle, state.handle, layer, _host_ptr(conv_state, "conv_state", True),
            _host_ptr(delta_state, "delta_state", True), _host_ptr(qkv, "qkv", True),
            _host_ptr(z, "z"), _host_ptr(beta, "beta", True), _host_ptr(alpha, "alpha", True),
            _host_ptr(attention, "attention", True)))

    def full_core(self, state: State, layer: int, q_and_gate: np.ndarray, key: np.ndarray,
                  value: np.ndarray, q: Optional[np.ndarray], gate: Optional[np.ndarray],
                  scores: Optional[np.ndarray], attention: np.ndarray, key_cache: np.ndarray,
                  value_cache: np.ndarray, context_length: int, current_position: int) -> None:
        """full_core(weights, q_and_gate, key, value, q, gate, scores, attention,
        key_cache, value_cache, context_length, current_position, layer),
        src/model/ops.rs:812-827. Raises Q38Error(-1) where the reference
        returns Err(-1). ``scores`` is scratch and is left untouched."""
        _host_len(q_and_gate, ATTN_QG_DIM, "q_and_gate")
        _host_len(key, ATTN_KV_DIM, "key")
        _host_len(value, ATTN_KV_DIM, "value")
        _host_len(attention, ATTN_Q_DIM, "attention")
        _host_len(q, ATTN_Q_DIM, "q")
        _host_len(gate, ATTN_Q_DIM, "gate")
        rows = min(key_cache.size, value_cache.size) // ATTN_KV_DIM
        check(self._lib.q38_full_core(
            self.handle, state.handle, layer, _host_ptr(q_and_gate, "q_and_gate"),
            _host_ptr(key, "key", True), _host_ptr(value, "value"), _host_ptr(q, "q", True),
            _host_ptr(gate, "gate", True), _host_ptr(scores, "scores", True),
            _host_ptr(attention, "attention", True), _host_ptr(key_cache, "key_cache", True),
            _host_ptr(value_cache, "value_cache", True), rows, context_length,
            current_position))

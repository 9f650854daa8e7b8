"""A small GGUF (v2/v3) writer for the tests: the container layout the
reference's loader parses (src/gguf/mod.rs:459-533) -- header, metadata
key/value entries, tensor descriptors, then the tensor data at
`general.alignment` (default 32) -- so that the library's parser can be
checked without a real checkpoint.

Tensor shapes are given in GGUF order (innermost dimension first), and the
data of a non-F32 tensor is written as opaque bytes of the size its ggml type
implies."""
from __future__ import annotations

import struct

import numpy as np

# metadata value types
U8, I8, U16, I16, U32, I32, F32, BOOL, STRING, ARRAY, U64, I64, F64 = range(13)
_SCALAR = {U8: "<B", I8: "<b", U16: "<H", I16: "<h", U32: "<I", I32: "<i", F32: "<f",
           BOOL: "<?", U64: "<Q", I64: "<q", F64: "<d"}

# ggml tensor types used here: (type id, elements per block, bytes per block)
GGML_F32 = (0, 1, 4)
GGML_F16 = (1, 1, 2)
GGML_Q8_0 = (8, 32, 34)
GGML_Q4_K = (12, 256, 144)
GGML_Q6_K = (14, 256, 210)
GGML_IQ4_NL = (20, 32, 18)
GGML_IQ4_XS = (23, 256, 136)


def _string(s: str | bytes) -> bytes:
    b = s.encode() if isinstance(s, str) else s
    return struct.pack("<Q", len(b)) + b


def _value(ty: int, v) -> bytes:
    if ty == STRING:
        return _string(v)
    if ty == ARRAY:
        elem, items = v
        out = struct.pack("<IQ", elem, len(items))
        return out + b"".join(_value(elem, x) for x in items)
    return struct.pack(_SCALAR[ty], v)


def write_gguf(path, tensors, metadata=(), version: int = 3, alignment: int | None = None,
               magic: bytes = b"GGUF", truncate: int | None = None) -> None:
    """tensors: list of (name, shape (GGUF order), ggml type tuple, data) where
    data is a float32 array for F32 tensors and bytes (or None = zeros) for
    the others. metadata: list of (key, type, value). alignment: written as
    general.alignment (u32) when given."""
    meta = list(metadata)
    if alignment is not None:
        meta.append(("general.alignment", U32, alignment))
    align = alignment or 32
    head = magic + struct.pack("<IQQ", version, len(tensors), len(meta))
    for key, ty, v in meta:
        head += _string(key) + struct.pack("<I", ty) + _value(ty, v)
    blobs, offset = [], 0
    descs = b""
    for name, shape, (tid, bel, bby), data in tensors:
        n = int(np.prod(shape))
        if tid == GGML_F32[0]:
            blob = np.asarray(data, np.float32).reshape(-1).tobytes()
            assert len(blob) == 4 * n
        else:
            size = n // bel * bby  # (a ragged tensor is written short; the parser must reject it)
            blob = bytes(size) if data is None else bytes(data)
        descs += _string(name) + struct.pack("<I", len(shape))
        descs += b"".join(struct.pack("<Q", d) for d in shape)
        descs += struct.pack("<IQ", tid, offset)
        blobs.append((offset, blob))
        offset += len(blob)
        offset = (offset + align - 1) // align * align
    body = head + descs
    data_start = (len(body) + align - 1) // align * align
    out = bytearray(body + bytes(data_start - len(body)))
    for off, blob in blobs:
        need = data_start + off - len(out)
        out += bytes(need) + blob if need >= 0 else b""
    if truncate is not None:
        out = out[:truncate]
    with open(path, "wb") as f:
        f.write(out)


def layer_tensors(layer: int, full: bool, weights: dict) -> list:
    """The F32 tensors of one layer under the reference's names (ops.rs:53-100),
    plus a quantized projection of that layer that the parser must size and
    skip."""
    pre = f"blk.{layer}."
    if full:
        out = [(pre + "attn_q_norm.weight", [256], GGML_F32, weights["q_norm"]),
               (pre + "attn_k_norm.weight", [256], GGML_F32, weights["k_norm"]),
               (pre + "attn_q.weight", [512, 24], GGML_Q4_K, None)]
    else:
        out = [(pre + "ssm_conv1d.weight", [4, 10240], GGML_F32, weights["conv1d"]),
               (pre + "ssm_dt.bias", [48], GGML_F32, weights["dt_bias"]),
               (pre + "ssm_a", [48], GGML_F32, weights["ssm_a"]),
               (pre + "ssm_norm.weight", [128], GGML_F32, weights["ssm_norm"]),
               (pre + "attn_qkv.weight", [256, 40], GGML_Q8_0, None)]
    return out

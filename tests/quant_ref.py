"""An independent numpy restatement of the reference's projection arithmetic,
written from the ggml block formats rather than from the C++ oracle, to pin
the oracle (oracle/q38_oracle_proj.cpp):

* quantize_q8_k (src/kernel/quant.rs:56-124), vectorised over blocks;
* per-element integer weights and per-element integer scales of each K-quant
  type, from which the integer dot of dot_q*_k_q8_k_scalar
  (src/kernel/tensor.rs:301-460) is an exact int64 sum, and the f32 running
  total over blocks is replayed in float32;
* the same for IQ4_XS and IQ4_NL (src/kernel/iq.rs:355-405): 4-bit indices
  into the 16-value IQ4 table, a 6-bit group scale minus 32 (IQ4_XS, one term
  per block) or an f16 scale per 32-value group (IQ4_NL, one term per group);
* dequantized weights (d * scale * q - dmin * min), for the reference's own
  consistency bar between the integer path and a plain f32 dot
  (tensor.rs:604-700).
"""
from __future__ import annotations

import numpy as np

F32 = np.float32


def f16(lo: np.ndarray, hi: np.ndarray) -> np.ndarray:
    return (lo.astype(np.uint16) | (hi.astype(np.uint16) << 8)).view(np.float16).astype(F32)


def quantize_q8_k(x: np.ndarray):
    """Returns (scale [nb] f32, quants [nb][256] int8, sums [nb][16] int16)."""
    b = np.ascontiguousarray(x, F32).reshape(-1, 256)
    a = np.abs(b)
    amax = a.max(axis=1)
    first = np.argmax(a == amax[:, None], axis=1)  # first index of the largest magnitude
    mx = b[np.arange(b.shape[0]), first]
    zero = amax == 0
    with np.errstate(divide="ignore", invalid="ignore"):
        inv = np.where(zero, F32(0), F32(-127.0) / np.where(zero, F32(1), mx)).astype(F32)
        prod = (inv[:, None] * b).astype(F32)
        shifted = (prod + F32(12582912.0)).astype(F32)
    q = (shifted.view(np.uint32) & np.uint32(0x7FFFFF)).astype(np.int64) - 0x400000
    q = np.minimum(q, 127)
    q[zero] = 0
    sums = q.reshape(-1, 16, 16).sum(axis=2)
    with np.errstate(divide="ignore"):
        scale = np.where(zero, F32(0), F32(1.0) / np.where(zero, F32(1), inv)).astype(F32)
    return scale, q.astype(np.int8), sums.astype(np.int16)


def _scale_min_k4(s: np.ndarray):
    """s: [nb][12] packed bytes -> (scales [nb][8], mins [nb][8])."""
    s = s.astype(np.int64)
    sc = np.zeros((s.shape[0], 8), np.int64)
    mn = np.zeros_like(sc)
    sc[:, :4] = s[:, 0:4] & 63
    mn[:, :4] = s[:, 4:8] & 63
    sc[:, 4:] = (s[:, 8:12] & 15) | ((s[:, 0:4] >> 6) << 4)
    mn[:, 4:] = (s[:, 8:12] >> 4) | ((s[:, 4:8] >> 6) << 4)
    return sc, mn


# The IQ4 format's 16 values (kvalues_iq4nl).
IQ4_VALUES = np.array([-127, -104, -83, -65, -49, -35, -22, -10, 1, 13, 25, 38, 53, 69, 89, 113], np.int64)


def _iq4_nibbles(qs: np.ndarray) -> np.ndarray:
    """[n][16] group bytes -> [n][32] table values: byte i gives value i (low
    nibble) and value i + 16 (high nibble)."""
    return np.concatenate([IQ4_VALUES[qs & 15], IQ4_VALUES[qs >> 4]], axis=1)


def decode_iq4_nl(raw: np.ndarray, nblk: int):
    """Per 256 values: (q [nb][256], d [nb][8] f32 group scales)."""
    g = raw.reshape(nblk * 8, 18).astype(np.int64)
    d = f16(g[:, 0], g[:, 1]).reshape(nblk, 8)
    return _iq4_nibbles(g[:, 2:]).reshape(nblk, 256), d


def decode(ggml_type: int, raw: np.ndarray, nblk: int):
    """Per 256-block: (q [nb][256] int, scale per element [nb][256] int,
    min per 16-group [nb][16] int, d [nb] f32, dmin [nb] f32) such that
    value = d*scale*q - dmin*min(group)."""
    b = raw.reshape(nblk, -1).astype(np.int64)
    nb = nblk
    q = np.zeros((nb, 256), np.int64)
    se = np.zeros((nb, 256), np.int64)
    mg = np.zeros((nb, 16), np.int64)
    if ggml_type in (12, 13):  # Q4_K, Q5_K
        d, dmin = f16(b[:, 0], b[:, 1]), f16(b[:, 2], b[:, 3])
        sc, mn = _scale_min_k4(b[:, 4:16])
        qs = b[:, 16:144] if ggml_type == 12 else b[:, 48:176]
        for c in range(4):
            lo, hi = qs[:, 32 * c:32 * c + 32] & 15, qs[:, 32 * c:32 * c + 32] >> 4
            if ggml_type == 13:
                h = b[:, 16:48]
                lo = lo + ((h >> (2 * c)) & 1) * 16
                hi = hi + ((h >> (2 * c + 1)) & 1) * 16
            q[:, 64 * c:64 * c + 32], q[:, 64 * c + 32:64 * c + 64] = lo, hi
            se[:, 64 * c:64 * c + 32] = sc[:, 2 * c:2 * c + 1]
            se[:, 64 * c + 32:64 * c + 64] = sc[:, 2 * c + 1:2 * c + 2]
            mg[:, 4 * c:4 * c + 2] = mn[:, 2 * c:2 * c + 1]
            mg[:, 4 * c + 2:4 * c + 4] = mn[:, 2 * c + 1:2 * c + 2]
        return q, se, mg, d, dmin
    if ggml_type == 14:  # Q6_K
        d = f16(b[:, 208], b[:, 209])
        scales = b[:, 192:208].astype(np.int8).astype(np.int64)
        for h in range(2):
            ql, qh = b[:, 64 * h:64 * h + 64], b[:, 128 + 32 * h:160 + 32 * h]
            base = 128 * h
            q[:, base:base + 32] = (ql[:, :32] & 15) | ((qh & 3) << 4)
            q[:, base + 32:base + 64] = (ql[:, 32:] & 15) | (((qh >> 2) & 3) << 4)
            q[:, base + 64:base + 96] = (ql[:, :32] >> 4) | (((qh >> 4) & 3) << 4)
            q[:, base + 96:base + 128] = (ql[:, 32:] >> 4) | (((qh >> 6) & 3) << 4)
            for g in range(8):  # 16-element groups within this half
                se[:, base + 16 * g:base + 16 * g + 16] = scales[:, 8 * h + (g % 2) + 2 * (g // 2):
                                                                 8 * h + (g % 2) + 2 * (g // 2) + 1]
        return q - 32, se, mg, d, np.zeros_like(d)
    if ggml_type == 11:  # Q3_K
        hm, qs, p = b[:, 0:32], b[:, 32:96], b[:, 96:108]
        d = f16(b[:, 108], b[:, 109])
        sc = np.zeros((nb, 16), np.int64)
        for i in range(16):
            low = (p[:, i] & 15) if i < 8 else (p[:, i - 8] >> 4)
            high = (p[:, 8 + i % 4] >> (2 * (i // 4))) & 3
            sc[:, i] = (low | (high << 4)) - 32
        for half in range(2):
            for field in range(4):
                group = 4 * half + field
                seg = slice(128 * half + 32 * field, 128 * half + 32 * field + 32)
                two = (qs[:, 32 * half:32 * half + 32] >> (2 * field)) & 3
                q[:, seg] = two - np.where((hm >> group) & 1, 0, 4)
                se[:, seg.start:seg.start + 16] = sc[:, 2 * group:2 * group + 1]
                se[:, seg.start + 16:seg.stop] = sc[:, 2 * group + 1:2 * group + 2]
        return q, se, mg, d, np.zeros_like(d)
    if ggml_type == 23:  # IQ4_XS
        d = f16(b[:, 0], b[:, 1])
        high = b[:, 2] | (b[:, 3] << 8)
        for grp in range(8):
            low = (b[:, 4 + grp // 2] >> (4 * (grp % 2))) & 15
            se[:, 32 * grp:32 * grp + 32] = (low | (((high >> (2 * grp)) & 3) << 4))[:, None] - 32
            q[:, 32 * grp:32 * grp + 32] = _iq4_nibbles(b[:, 8 + 16 * grp:24 + 16 * grp])
        return q, se, mg, d, np.zeros_like(d)
    if ggml_type == 10:  # Q2_K
        scales, qs = b[:, 0:16], b[:, 16:80]
        d, dmin = f16(b[:, 80], b[:, 81]), f16(b[:, 82], b[:, 83])
        for half in range(2):
            for field in range(4):
                si = 8 * half + 2 * field
                seg = 128 * half + 32 * field
                q[:, seg:seg + 16] = (qs[:, 32 * half:32 * half + 16] >> (2 * field)) & 3
                q[:, seg + 16:seg + 32] = (qs[:, 32 * half + 16:32 * half + 32] >> (2 * field)) & 3
                se[:, seg:seg + 16] = scales[:, si:si + 1] & 15
                se[:, seg + 16:seg + 32] = scales[:, si + 1:si + 2] & 15
                mg[:, si] = scales[:, si] >> 4
                mg[:, si + 1] = scales[:, si + 1] >> 4
        return q, se, mg, d, dmin
    raise ValueError(ggml_type)


def dot_q8_k(ggml_type: int, row: np.ndarray, scale, quants, sums) -> np.float32:
    """The reference's integer dot of one weight row with Q8_K blocks."""
    nblk = quants.shape[0]
    if ggml_type == 20:  # IQ4_NL: a term per 32-value group
        q, d = decode_iq4_nl(row, nblk)
        weighted = (q * quants.astype(np.int64)).reshape(nblk, 8, 32).sum(axis=2)
        total = F32(0)
        for blk in range(nblk):
            for grp in range(8):
                total = F32(total + F32(F32(d[blk, grp] * scale[blk]) * F32(weighted[blk, grp])))
        return total
    q, se, mg, d, dmin = decode(ggml_type, row, nblk)
    weighted = (se * q * quants.astype(np.int64)).sum(axis=1)
    minimum = (mg * sums.astype(np.int64)).sum(axis=1)
    total = F32(0)
    for blk in range(nblk):
        dd = F32(d[blk] * scale[blk])
        dm = F32(dmin[blk] * scale[blk])
        term = F32(F32(dd * F32(weighted[blk])) - F32(dm * F32(minimum[blk])))
        total = F32(total + term)
    return total


def dequantize(ggml_type: int, raw: np.ndarray, rows: int, width: int) -> np.ndarray:
    """f64 dequantized matrix [rows][width]."""
    if ggml_type == 0:
        return raw.view(np.float32).reshape(rows, width).astype(np.float64)
    if ggml_type == 1:
        return raw.view(np.float16).reshape(rows, width).astype(np.float64)
    if ggml_type == 30:
        return (raw.view(np.uint16).astype(np.uint32) << 16).view(np.float32).reshape(rows, width).astype(np.float64)
    if ggml_type == 8:
        b = raw.reshape(-1, 34)
        d = f16(b[:, 0], b[:, 1]).astype(np.float64)
        return (d[:, None] * b[:, 2:].view(np.int8)).reshape(rows, width)
    nblk = rows * width // 256
    if ggml_type == 20:
        q, d = decode_iq4_nl(raw, nblk)
        return (np.repeat(d.astype(np.float64), 32, axis=1) * q).reshape(rows, width)
    q, se, mg, d, dmin = decode(ggml_type, raw, nblk)
    mins = np.repeat(mg, 16, axis=1)
    v = d.astype(np.float64)[:, None] * se * q - dmin.astype(np.float64)[:, None] * mins
    return v.reshape(rows, width)

"""CPU tests of the GGUF reader (q38_gguf_read_f32): the container checks of
the reference's loader (src/gguf/mod.rs:459-533, Gguf::open) and the F32
read-out that weight binding uses. No GPU needed."""
from __future__ import annotations

import numpy as np
import pytest

import q38attn
from gguf_writer import (ARRAY, BOOL, F32, F64, GGML_F16, GGML_F32, GGML_Q4_K, GGML_Q8_0, I32,
                         STRING, U8, U32, U64, layer_tensors, write_gguf)


def _rich_metadata():
    return [("general.architecture", STRING, "qwen38"),
            ("qwen38.block_count", U32, 64),
            ("qwen38.rope.freq_base", F32, 1e7),
            ("general.flag", BOOL, True),
            ("general.small", U8, 7),
            ("general.big", U64, 1 << 40),
            ("general.neg", I32, -3),
            ("general.ratio", F64, 0.25),
            ("tokenizer.ggml.tokens", ARRAY, (STRING, ["a", "bc", "def"])),
            ("tokenizer.ggml.scores", ARRAY, (F32, [0.5, 1.5])),
            ("general.empty", ARRAY, (U32, []))]


@pytest.mark.parametrize("version,alignment", [(3, None), (3, 64), (2, 128)])
def test_read_f32_roundtrip(tmp_path, version, alignment):
    g = np.random.default_rng(5)
    a = g.standard_normal(256).astype(np.float32)
    b = g.standard_normal((10240, 4)).astype(np.float32)
    path = tmp_path / "m.gguf"
    write_gguf(path, [("blk.3.attn_q_norm.weight", [256], GGML_F32, a),
                      ("blk.0.attn_qkv.weight", [256, 40], GGML_Q8_0, None),
                      ("blk.0.ssm_conv1d.weight", [4, 10240], GGML_F32, b),
                      ("blk.0.attn_gate.weight", [512, 2], GGML_Q4_K, None),
                      ("token_embd.weight", [64, 3], GGML_F16, None)],
               metadata=_rich_metadata(), version=version, alignment=alignment)
    np.testing.assert_array_equal(q38attn.gguf_read_f32(path, "blk.3.attn_q_norm.weight", 256), a)
    np.testing.assert_array_equal(
        q38attn.gguf_read_f32(path, "blk.0.ssm_conv1d.weight", 4 * 10240), b.reshape(-1))


def test_layer_tensor_names(tmp_path):
    """The tensor names bind_layer looks up (ops.rs:53-100) for both layer kinds."""
    from q38attn import synth
    g = synth.rng(3)
    fw, lw = synth.full_weights(g), synth.linear_weights(g)
    path = tmp_path / "layers.gguf"
    write_gguf(path, layer_tensors(0, False, lw) + layer_tensors(3, True, fw) +
               layer_tensors(64, True, fw))
    np.testing.assert_array_equal(q38attn.gguf_read_f32(path, "blk.64.attn_k_norm.weight", 256),
                                  fw["k_norm"])
    np.testing.assert_array_equal(q38attn.gguf_read_f32(path, "blk.0.ssm_dt.bias", 48),
                                  lw["dt_bias"])
    np.testing.assert_array_equal(q38attn.gguf_read_f32(path, "blk.0.ssm_a", 48), lw["ssm_a"])


def _err(fn):
    with pytest.raises(q38attn.Q38Error) as e:
        fn()
    assert e.value.code == q38attn.Q38_ERR_ARG
    return str(e.value)


def test_read_f32_errors(tmp_path):
    a = np.arange(256, dtype=np.float32)
    ok = tmp_path / "ok.gguf"
    tensors = [("blk.3.attn_q_norm.weight", [256], GGML_F32, a),
               ("blk.3.attn_q.weight", [256, 2], GGML_Q4_K, None)]
    write_gguf(ok, tensors)
    assert "not found" in _err(lambda: q38attn.gguf_read_f32(ok, "blk.3.missing", 256))
    assert "not F32" in _err(lambda: q38attn.gguf_read_f32(ok, "blk.3.attn_q.weight", 512))
    assert "elements" in _err(lambda: q38attn.gguf_read_f32(ok, "blk.3.attn_q_norm.weight", 255))
    _err(lambda: q38attn.gguf_read_f32(tmp_path / "absent.gguf", "x", 1))

    def bad(name, **kw):
        p = tmp_path / name
        write_gguf(p, kw.pop("tensors", tensors), **kw)
        return _err(lambda: q38attn.gguf_read_f32(p, "blk.3.attn_q_norm.weight", 256))

    assert "header" in bad("magic.gguf", magic=b"GGUE")
    assert "header" in bad("v1.gguf", version=1)
    assert "header" in bad("v4.gguf", version=4)
    assert "header" in bad("none.gguf", tensors=[])
    assert "alignment" in bad("align3.gguf", alignment=3)
    assert "outside" in bad("trunc.gguf", truncate=-100)
    bad("short.gguf", truncate=60)
    # nested arrays are rejected
    assert "nested" in bad("nested.gguf", metadata=[("x", ARRAY, (ARRAY, []))])
    # a quantized tensor whose first dimension is not a whole number of blocks
    assert "bytes" in bad("blocks.gguf", tensors=tensors + [("q", [100], GGML_Q8_0, None)])


def test_truncated_files_fail_cleanly(tmp_path):
    """Every prefix of a valid file is rejected (never a crash or a read past the end)."""
    a = np.ones(256, np.float32)
    full = tmp_path / "full.gguf"
    write_gguf(full, [("blk.3.attn_q_norm.weight", [256], GGML_F32, a)],
               metadata=_rich_metadata())
    data = full.read_bytes()
    for cut in list(range(0, 200, 7)) + [len(data) - 1]:
        p = tmp_path / f"cut{cut}.gguf"
        p.write_bytes(data[:cut])
        _err(lambda: q38attn.gguf_read_f32(p, "blk.3.attn_q_norm.weight", 256))

"""GPU tests of weight binding from a GGUF checkpoint (q38_bind_gguf) and of
the MTP block's attention: mtp_layer_forward (src/model/ops.rs:1249-1307)
calls full_attention -> full_core with layer 64, whose cache rows are KV
slot 16 (ops.rs:858).

Weights bound from a GGUF file must give bitwise the results of the same
values bound from arrays (same kernels, same device copies); the layer-64
path is checked against the CPU oracle at the reference's tolerance
(|a-b|/max(|b|,1) < 1e-4, src/kernel/x86/tensor.rs:411-413)."""
from __future__ import annotations

import numpy as np
import pytest

from conftest import check_parity, relative_error
from gguf_writer import STRING, U32, layer_tensors, write_gguf

pytestmark = pytest.mark.gpu

F = np.float32
TOL = 1e-4


def _checkpoint(tmp_path, g):
    from q38attn import synth
    w = {"lin": synth.linear_weights(g), "full": synth.full_weights(g), "mtp": synth.full_weights(g)}
    path = tmp_path / "q38.gguf"
    write_gguf(path, layer_tensors(0, False, w["lin"]) + layer_tensors(3, True, w["full"]) +
               layer_tensors(64, True, w["mtp"]),
               metadata=[("general.architecture", STRING, "qwen38"),
                         ("qwen38.block_count", U32, 64)], alignment=64)
    return path, w


def _full_core(ctx, st, layer, x, kc, vc, ctx_len, pos):
    key = x["key"].copy()
    q, gate, att = np.zeros(6144, F), np.zeros(6144, F), np.zeros(6144, F)
    ctx.full_core(st, layer, x["q_and_gate"], key, x["value"], q, gate, None, att, kc, vc,
                  ctx_len, pos)
    return att, key


def test_bind_gguf_equals_array_binding(cuda_ctx, tmp_path):
    import q38attn
    from q38attn import synth
    g = synth.rng(81)
    path, w = _checkpoint(tmp_path, g)
    ref = cuda_ctx
    ref.bind_linear_layer(0, w["lin"]["conv1d"], w["lin"]["dt_bias"], w["lin"]["ssm_a"],
                          w["lin"]["ssm_norm"])
    ref.bind_full_layer(3, w["full"]["q_norm"], w["full"]["k_norm"])
    ref.bind_full_layer(64, w["mtp"]["q_norm"], w["mtp"]["k_norm"])
    gg = q38attn.Context(0)
    gg.bind_gguf(path, 0, 0)
    gg.bind_gguf(path, 3, 3)
    gg.bind_gguf(path, 64, 64)

    ctx_len, pos = 48, 20
    init = synth.linear_state(g)
    lin_x = {k: v.copy() for k, v in synth.linear_step(g, 1).items()}
    full_x = {k: v[0].copy() for k, v in synth.full_step(g).items()}
    kc = np.zeros((17 * ctx_len, 1024), F)
    vc = np.zeros((17 * ctx_len, 1024), F)
    for slot in (0, 16):
        kc[slot * ctx_len:slot * ctx_len + pos], vc[slot * ctx_len:slot * ctx_len + pos] = \
            synth.kv_rows(g, pos)
    outs = []
    for ctx in (ref, gg):
        st = ctx.state(1, ctx_len, full_slots=17, linear_slots=1)
        st.upload_linear(0, 0, init["conv_state"], init["delta_state"])
        x = {k: v.copy() for k, v in lin_x.items()}
        att = np.zeros((1, 6144), F)
        ctx.linear_decode_host(st, 0, x["qkv"], x["z"], x["beta"], x["alpha"], att)
        res = [att, x["qkv"], x["alpha"], st.download_linear(0, 0)[1]]
        for layer in (3, 64):
            res += list(_full_core(ctx, st, layer, full_x, kc.copy(), vc.copy(), ctx_len, pos))
        assert st.errors() == 0
        st.close()
        outs.append(res)
    for a, b in zip(*outs):
        np.testing.assert_array_equal(a, b)
    gg.close()


def test_mtp_layer_matches_oracle(cuda_ctx, oracle_lib, tmp_path):
    """full_core at layer 64 (the MTP block) reads and writes KV slot 16."""
    from q38attn import synth
    g = synth.rng(82)
    path, w = _checkpoint(tmp_path, g)
    cuda_ctx.bind_gguf(path, 64, 64)
    ctx_len, pos = 96, 70
    kc = np.zeros((17 * ctx_len, 1024), F)
    vc = np.zeros((17 * ctx_len, 1024), F)
    kc[16 * ctx_len:16 * ctx_len + pos], vc[16 * ctx_len:16 * ctx_len + pos] = synth.kv_rows(g, pos)
    x = {k: v[0].copy() for k, v in synth.full_step(g).items()}

    okc, ovc = kc.copy(), vc.copy()
    q, gate, scores = np.zeros(6144, F), np.zeros(6144, F), np.zeros(24 * ctx_len, F)
    oatt, okey = np.zeros(6144, F), x["key"].copy()
    assert oracle_lib.full_core(w["mtp"], x["q_and_gate"], okey, x["value"], q, gate, scores, oatt,
                                okc, ovc, ctx_len, pos, 64, False) == 0

    st = cuda_ctx.state(1, ctx_len, full_slots=17, linear_slots=0)
    gkc, gvc = kc.copy(), vc.copy()
    att, key = _full_core(cuda_ctx, st, 64, x, gkc, gvc, ctx_len, pos)
    check_parity(att, oatt, TOL, "")
    assert relative_error(key, okey) < 1e-5
    row = 16 * ctx_len + pos
    assert relative_error(gkc[row], okc[row]) < 1e-5
    np.testing.assert_array_equal(gvc[row], x["value"])
    # The device cache holds the new row in slot 16.
    dk, dv = st.download_kv(64, 0, pos, 1)
    assert relative_error(dk[0], okc[row]) < 1e-5
    assert st.errors() == 0
    st.close()


def test_bind_gguf_errors(cuda_ctx, tmp_path):
    import q38attn
    from q38attn import synth
    path, _ = _checkpoint(tmp_path, synth.rng(83))
    for first, last in [(0, 3), (4, 4), (60, 64)]:  # layers 1, 2, 4, 60-63 are absent
        with pytest.raises(q38attn.Q38Error) as e:
            cuda_ctx.bind_gguf(path, first, last)
        assert e.value.code == q38attn.Q38_ERR_ARG
        assert "not found" in str(e.value)
    with pytest.raises(q38attn.Q38Error):
        cuda_ctx.bind_gguf(path, 0, 65)
    with pytest.raises(q38attn.Q38Error):
        cuda_ctx.bind_gguf(tmp_path / "missing.gguf", 0, 0)

"""CPU tests of the oracle (the C++ restatement of the reference's cores).

Pins, since the reference ships no golden vectors or known-answer tests for
this path and no Rust toolchain exists here:
  * stored golden outputs (tests/golden/golden.npz) reproduced bit-exactly;
  * known-answer tests derived from the algorithm;
  * agreement with an independent numpy restatement written from the same
    reference lines (src/model/ops.rs:476-610, 648-742, 813-940).
"""
from __future__ import annotations

import math

import numpy as np
import pytest

import vectors as V
from conftest import REPO, relative_error

GOLDEN = np.load(REPO / "tests" / "golden" / "golden.npz")
F = np.float32


# --------------------------------------------------------------------------
# Independent numpy restatement (float64 accumulation, f32 storage).
# --------------------------------------------------------------------------
def np_silu(x):
    x = x.astype(F)
    return (x / (F(1) + np.exp(-x))).astype(F)


def np_sigmoid(x):
    x = x.astype(F)
    return (F(1) / (F(1) + np.exp(-x))).astype(F)


def np_softplus(x):
    x = x.astype(F)
    return np.where(x > F(20), x, np.log(F(1) + np.exp(x))).astype(F)


def np_rms_scale(x):
    s = np.sum(x.astype(np.float64) ** 2, axis=-1, keepdims=True)
    mean = (s / x.shape[-1]).astype(F)
    return (F(1) / np.sqrt(mean + F(1e-6))).astype(F)


def np_l2norm(x):
    s = np.sum(x.astype(np.float64) ** 2, axis=-1, keepdims=True).astype(F)
    return (x * (F(1) / np.maximum(np.sqrt(s), F(1e-6)))).astype(F)


def np_rope(x, position):
    """x: [heads, 256]."""
    scale = F(10000000.0) ** F(-2.0 / 64.0)
    theta = np.empty(32, F)
    t = F(position)
    for i in range(32):
        theta[i] = t
        t = F(t * scale)
    c, s = np.cos(theta.astype(np.float64)).astype(F), np.sin(theta.astype(np.float64)).astype(F)
    y = x.copy()
    x0, x1 = x[:, :32], x[:, 32:64]
    y[:, :32] = x0 * c - x1 * s
    y[:, 32:64] = x0 * s + x1 * c
    return y


def np_linear_core(w, conv, delta, qkv, z, beta, alpha):
    cw = w["conv1d"]
    v = conv[:, 0] * cw[:, 0]
    v = v + conv[:, 1] * cw[:, 1]
    v = v + conv[:, 2] * cw[:, 2]
    v = v + qkv * cw[:, 3]
    new_conv = np.stack([conv[:, 1], conv[:, 2], qkv], axis=1).astype(F)
    y = np_silu(v.astype(F))
    q = np_l2norm(y[:2048].reshape(16, 128))
    k = np_l2norm(y[2048:4096].reshape(16, 128))
    vv = y[4096:].reshape(48, 128)
    b = np_sigmoid(beta)
    a = (w["ssm_a"] * np_softplus(alpha + w["dt_bias"])).astype(F)
    out = np.zeros((48, 128), F)
    new_delta = np.empty_like(delta)
    for h in range(48):
        kh = h % 16
        S = (delta[h] * np.exp(a[h]).astype(F)).astype(np.float64)
        pred = S @ k[kh].astype(np.float64)
        d = ((vv[h].astype(np.float64) - pred) * b[h])
        S = S + np.outer(d, k[kh])
        out[h] = (S @ q[kh].astype(np.float64) / math.sqrt(128)).astype(F)
        new_delta[h] = S.astype(F)
    out = (out * np_rms_scale(out) * w["ssm_norm"]).astype(F)
    out = (out * np_silu(z.reshape(48, 128))).astype(F)
    qkv_out = np.concatenate([q.ravel(), k.ravel(), vv.ravel()]).astype(F)
    return new_conv, new_delta, qkv_out, b, a, out.ravel()


def np_full_core(w, q_and_gate, key, value, kc, vc, context, pos, layer):
    qg = q_and_gate.reshape(24, 512)
    q = qg[:, :256].copy()
    gate = qg[:, 256:].copy()
    q = (q * np_rms_scale(q) * w["q_norm"]).astype(F)
    k = key.reshape(4, 256)
    k = (k * np_rms_scale(k) * w["k_norm"]).astype(F)
    q, k = np_rope(q, pos), np_rope(k, pos)
    row = (layer // 4) * context + pos
    kc[row] = k.ravel()
    vc[row] = value
    base = (layer // 4) * context
    K = kc[base:base + pos + 1].reshape(pos + 1, 4, 256).astype(np.float64)
    Vv = vc[base:base + pos + 1].reshape(pos + 1, 4, 256).astype(np.float64)
    out = np.zeros((24, 256), F)
    for h in range(24):
        g = h // 6
        s = (K[:, g, :] @ q[h].astype(np.float64)) / 16.0
        e = np.exp(s - s.max())
        p = e / e.sum()
        out[h] = (p @ Vv[:, g, :]).astype(F) * np_sigmoid(gate[h])
    return k.ravel(), q.ravel(), out.ravel()


# --------------------------------------------------------------------------
# Golden vectors: the oracle reproduces its stored outputs bit-exactly.
# --------------------------------------------------------------------------
def test_golden_linear_bit_exact(oracle_lib):
    w = V.linear_weights()
    s = V.linear_state()
    conv, delta = s["conv_state"].copy(), s["delta_state"].copy()
    for t in range(3):
        x = V.linear_token(t)
        att = np.zeros(V.V_DIM, F)
        assert oracle_lib.linear_core(w, conv, delta, x["qkv"], x["z"], x["beta"], x["alpha"],
                                      att) == 0
        np.testing.assert_array_equal(att, GOLDEN[f"lin_attention_{t}"])
        np.testing.assert_array_equal(x["beta"], GOLDEN[f"lin_beta_{t}"])
        np.testing.assert_array_equal(x["alpha"], GOLDEN[f"lin_alpha_{t}"])
        if t == 0:
            np.testing.assert_array_equal(x["qkv"], GOLDEN["lin_qkv_0"])
    np.testing.assert_array_equal(delta[0], GOLDEN["lin_delta_head0"])
    np.testing.assert_array_equal(delta[47], GOLDEN["lin_delta_head47"])
    np.testing.assert_array_equal(conv[::16], GOLDEN["lin_conv_final"])


@pytest.mark.parametrize("bf16", [False, True])
def test_golden_full_bit_exact(oracle_lib, bf16):
    tag = "fullbf16" if bf16 else "full"
    w = V.full_weights()
    kc, vc = V.full_cache(64, 37, 7, full_slots=2)
    if bf16:
        from q38attn.synth import round_bf16
        kc, vc = round_bf16(kc).reshape(kc.shape), round_bf16(vc).reshape(vc.shape)
    q = np.zeros(6144, F)
    gate = np.zeros(6144, F)
    scores = np.zeros(24 * 64, F)
    for t in range(3):
        x = V.full_token(t)
        att = np.zeros(6144, F)
        assert oracle_lib.full_core(w, x["q_and_gate"], x["key"], x["value"], q, gate, scores,
                                    att, kc, vc, 64, 37 + t, 7, bf16) == 0
        np.testing.assert_array_equal(att, GOLDEN[f"{tag}_attention_{t}"])
        np.testing.assert_array_equal(x["key"], GOLDEN[f"{tag}_key_{t}"])
        np.testing.assert_array_equal(q, GOLDEN[f"{tag}_q_{t}"])
        row = 64 + 37 + t
        np.testing.assert_array_equal(kc[row], GOLDEN[f"{tag}_krow_{t}"])


def test_golden_scalars(oracle_lib):
    xs = GOLDEN["sc_x"]
    np.testing.assert_array_equal(
        np.array([oracle_lib.sigmoid(float(x)) for x in xs], F), GOLDEN["sc_sigmoid"])
    np.testing.assert_array_equal(
        np.array([oracle_lib.softplus(float(x)) for x in xs], F), GOLDEN["sc_softplus"])
    np.testing.assert_array_equal(
        np.array([oracle_lib.rms_scale(V.activation(256, k)) for k in range(8)], F),
        GOLDEN["sc_rms_scale"])


# --------------------------------------------------------------------------
# Independent restatement agrees.
# --------------------------------------------------------------------------
def test_linear_core_matches_numpy_restatement(oracle_lib):
    from q38attn import synth
    g = synth.rng(0)
    w = synth.linear_weights(g)
    s = synth.linear_state(g)
    x = {k: v[0].copy() for k, v in synth.linear_step(g).items()}
    ref = np_linear_core(w, s["conv_state"], s["delta_state"], x["qkv"], x["z"], x["beta"],
                         x["alpha"])
    conv, delta = s["conv_state"].copy(), s["delta_state"].copy()
    att = np.zeros(6144, F)
    assert oracle_lib.linear_core(w, conv, delta, x["qkv"], x["z"], x["beta"], x["alpha"],
                                  att) == 0
    np.testing.assert_array_equal(conv, ref[0])
    assert relative_error(delta, ref[1]) < 1e-5
    assert relative_error(x["qkv"], ref[2]) < 1e-6
    assert relative_error(x["beta"], ref[3]) < 1e-6
    assert relative_error(x["alpha"], ref[4]) < 1e-6
    assert relative_error(att, ref[5]) < 1e-4


@pytest.mark.parametrize("pos", [0, 1, 100, 255])
def test_full_core_matches_numpy_restatement(oracle_lib, pos):
    from q38attn import synth
    g = synth.rng(pos)
    w = synth.full_weights(g)
    ctx = 256
    kc, vc = synth.kv_rows(g, 2 * ctx)
    kc[ctx + pos:] = 0
    vc[ctx + pos:] = 0
    x = {k: v[0].copy() for k, v in synth.full_step(g).items()}
    kc2, vc2 = kc.copy(), vc.copy()
    ref_k, ref_q, ref_out = np_full_core(w, x["q_and_gate"], x["key"].copy(), x["value"], kc2,
                                         vc2, ctx, pos, 7)
    q = np.zeros(6144, F)
    gate = np.zeros(6144, F)
    scores = np.zeros(24 * ctx, F)
    att = np.zeros(6144, F)
    assert oracle_lib.full_core(w, x["q_and_gate"], x["key"], x["value"], q, gate, scores, att,
                                kc, vc, ctx, pos, 7) == 0
    assert relative_error(x["key"], ref_k) < 1e-5
    assert relative_error(q, ref_q) < 1e-5
    assert relative_error(att, ref_out) < 1e-5
    np.testing.assert_array_equal(gate.reshape(24, 256), x["q_and_gate"].reshape(24, 512)[:, 256:])


# --------------------------------------------------------------------------
# Known-answer tests.
# --------------------------------------------------------------------------
def test_kat_rope_position_zero_is_identity(oracle_lib):
    x = V.activation(24 * 256, 5)
    y = x.copy()
    oracle_lib.rope(y, 24, 0)
    np.testing.assert_array_equal(x, y)


def test_kat_rope_rotation_preserves_pair_norms(oracle_lib):
    x = V.activation(4 * 256, 7)
    y = x.copy()
    oracle_lib.rope(y, 4, 12345)
    a = x.reshape(4, 256)
    b = y.reshape(4, 256)
    na = a[:, :32] ** 2 + a[:, 32:64] ** 2
    nb = b[:, :32] ** 2 + b[:, 32:64] ** 2
    np.testing.assert_allclose(na, nb, rtol=1e-5, atol=1e-6)
    np.testing.assert_array_equal(a[:, 64:], b[:, 64:])


def test_kat_scalars(oracle_lib):
    assert oracle_lib.softplus(21.0) == 21.0
    assert oracle_lib.softplus(0.0) == pytest.approx(math.log(2.0), rel=1e-7)
    assert oracle_lib.sigmoid(0.0) == 0.5
    assert oracle_lib.silu(0.0) == 0.0
    c = np.full(256, 3.0, F)
    assert oracle_lib.rms_scale(c) == pytest.approx(1.0 / math.sqrt(9.0 + 1e-6), rel=1e-7)
    zero = np.zeros(128, F)
    oracle_lib.l2norm(zero)
    assert not zero.any()
    assert oracle_lib.round_bf16(1.0 + 2 ** -9) == 1.0          # tie to even
    assert oracle_lib.round_bf16(1.0 + 3 * 2 ** -9) == 1.0 + 2 ** -7


def test_kat_deltanet_beta_zero_only_decays(oracle_lib):
    """beta = sigmoid(-inf) = 0: the delta term vanishes, S becomes S*exp(g)."""
    w = V.linear_weights()
    s = V.linear_state()
    x = V.linear_token(0)
    x["beta"][:] = -np.inf
    conv, delta = s["conv_state"].copy(), s["delta_state"].copy()
    alpha_in = x["alpha"].copy()
    att = np.zeros(6144, F)
    assert oracle_lib.linear_core(w, conv, delta, x["qkv"], x["z"], x["beta"], x["alpha"], att) == 0
    assert not x["beta"].any()
    g = (w["ssm_a"] * np.array([oracle_lib.softplus(float(a + b))
                                for a, b in zip(alpha_in, w["dt_bias"])], F)).astype(F)
    np.testing.assert_array_equal(x["alpha"], g)
    decay = np.exp(g.astype(np.float64)).astype(F)
    np.testing.assert_allclose(delta, s["delta_state"] * decay[:, None, None], rtol=2e-7, atol=0)


def test_kat_deltanet_unit_key_predicts_value(oracle_lib):
    """decay 1 (ssm_a = 0) and beta = 1: after the update every column of the
    state predicts v exactly along the (unit) key: S_new[j] . k = v[j]."""
    w = V.linear_weights()
    w["ssm_a"][:] = 0.0
    s = V.linear_state()
    x = V.linear_token(1)
    x["beta"][:] = 40.0  # sigmoid(40) == 1.0f
    conv, delta = s["conv_state"].copy(), s["delta_state"].copy()
    att = np.zeros(6144, F)
    assert oracle_lib.linear_core(w, conv, delta, x["qkv"], x["z"], x["beta"], x["alpha"], att) == 0
    assert np.all(x["beta"] == 1.0) and np.all(x["alpha"] == 0.0)
    k = x["qkv"][2048:4096].reshape(16, 128).astype(np.float64)
    v = x["qkv"][4096:].reshape(48, 128).astype(np.float64)
    assert np.allclose(np.linalg.norm(k, axis=1), 1.0, atol=1e-6)
    for h in range(48):
        pred = delta[h].astype(np.float64) @ k[h % 16]
        np.testing.assert_allclose(pred, v[h], rtol=0, atol=2e-5)


def test_kat_attention_single_position_returns_gated_value(oracle_lib):
    """At position 0 the softmax has one entry (p = 1): out = v * sigmoid(gate)."""
    w = V.full_weights()
    kc, vc = V.full_cache(8, 0, 3)
    x = V.full_token(0)
    q = np.zeros(6144, F)
    gate = np.zeros(6144, F)
    scores = np.zeros(24 * 8, F)
    att = np.zeros(6144, F)
    assert oracle_lib.full_core(w, x["q_and_gate"], x["key"], x["value"], q, gate, scores, att,
                                kc, vc, 8, 0, 3) == 0
    g = x["q_and_gate"].reshape(24, 512)[:, 256:]
    sig = np.array([[oracle_lib.sigmoid(float(t)) for t in row] for row in g], F)
    expect = (x["value"].reshape(4, 256)[np.arange(24) // 6] * sig).astype(F)
    np.testing.assert_array_equal(att.reshape(24, 256), expect)


def test_full_core_rejects_row_outside_cache(oracle_lib):
    """ops.rs:860-864: Err(-1) when the cache row does not fit."""
    w = V.full_weights()
    kc, vc = V.full_cache(8, 0, 3)  # 8 rows: layers 3 (slot 0) only
    x = V.full_token(0)
    scratch = [np.zeros(6144, F), np.zeros(6144, F), np.zeros(24 * 8, F), np.zeros(6144, F)]
    assert oracle_lib.full_core(w, x["q_and_gate"], x["key"], x["value"], *scratch, kc, vc, 8, 8,
                                3) == -1
    assert oracle_lib.full_core(w, x["q_and_gate"], x["key"], x["value"], *scratch, kc, vc, 8, 0,
                                7) == -1


def test_prefill_rows_match_full_prefill(oracle_lib):
    """The sampled-row prefill computes the listed rows exactly as the full loop."""
    from q38attn import synth
    g = synth.rng(3)
    w = synth.full_weights(g)
    T, ctx = 40, 64
    x = synth.full_step(g, T)
    kc1 = np.zeros((ctx, 1024), F)
    vc1 = np.zeros((ctx, 1024), F)
    kc2, vc2 = kc1.copy(), vc1.copy()
    a1 = np.zeros((T, 6144), F)
    a2 = np.zeros((T, 6144), F)
    k1, k2 = x["key"].copy(), x["key"].copy()
    assert oracle_lib.full_prefill(w, x["q_and_gate"], k1, x["value"], a1, kc1, vc1, ctx, 0, 3) == 0
    rows = [0, 5, 17, 39]
    assert oracle_lib.full_prefill(w, x["q_and_gate"], k2, x["value"], a2, kc2, vc2, ctx, 0, 3,
                                   rows_wanted=rows) == 0
    np.testing.assert_array_equal(a1[rows], a2[rows])
    np.testing.assert_array_equal(kc1, kc2)
    np.testing.assert_array_equal(k1, k2)

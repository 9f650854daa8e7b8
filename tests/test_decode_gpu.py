"""GPU parity tests of the decode kernels against the CPU oracle, through the
C ABI. Tolerance: the reference's metric |a-b|/max(|b|,1)
(src/kernel/x86/tensor.rs:411-413) below 1e-4 for these fp32 paths."""
from __future__ import annotations

import numpy as np
import pytest

import vectors as V
from conftest import REPO, check_parity, relative_error

pytestmark = pytest.mark.gpu

TOL = 1e-4
F = np.float32
GOLDEN = np.load(REPO / "tests" / "golden" / "golden.npz")


def _torch():
    import torch
    return torch


# ---------------------------------------------------------------------------
# Gated DeltaNet
# ---------------------------------------------------------------------------
def test_linear_core_mirror_matches_oracle_config2(cuda_ctx, oracle_lib):
    """Config 2 (batch 1) through the reference-signature mirror."""
    import q38attn
    from q38attn import synth
    g = synth.rng(0)
    w = synth.linear_weights(g)
    s = synth.linear_state(g)
    x = {k: v[0].copy() for k, v in synth.linear_step(g).items()}
    layer = 0
    cuda_ctx.bind_linear_layer(layer, w["conv1d"], w["dt_bias"], w["ssm_a"], w["ssm_norm"])
    st = cuda_ctx.state(1, 16, full_slots=0, linear_slots=1)

    oc, od = s["conv_state"].copy(), s["delta_state"].copy()
    ox = {k: v.copy() for k, v in x.items()}
    oatt = np.zeros(6144, F)
    assert oracle_lib.linear_core(w, oc, od, ox["qkv"], ox["z"], ox["beta"], ox["alpha"], oatt) == 0

    gc, gd = s["conv_state"].copy(), s["delta_state"].copy()
    gx = {k: v.copy() for k, v in x.items()}
    gatt = np.zeros(6144, F)
    cuda_ctx.linear_core(st, layer, gc, gd, gx["qkv"], gx["z"], gx["beta"], gx["alpha"], gatt)

    np.testing.assert_array_equal(gc, oc)  # conv state: exact (same mul/add sequence)
    assert relative_error(gx["qkv"], ox["qkv"]) < 1e-5
    assert relative_error(gx["beta"], ox["beta"]) < 1e-6
    assert relative_error(gx["alpha"], ox["alpha"]) < 1e-6
    check_parity(gd, od, TOL, "")
    check_parity(gatt, oatt, TOL, "")
    assert st.errors() == 0
    st.close()


def test_linear_golden_vectors_on_gpu(cuda_ctx):
    """The three-token golden sequence, resident state, batch 1."""
    w = V.linear_weights()
    s = V.linear_state()
    layer = 1
    cuda_ctx.bind_linear_layer(layer, w["conv1d"], w["dt_bias"], w["ssm_a"], w["ssm_norm"])
    st = cuda_ctx.state(1, 16, full_slots=0, linear_slots=2)
    st.upload_linear(layer, 0, s["conv_state"], s["delta_state"])
    for t in range(3):
        x = V.linear_token(t)
        att = np.zeros((1, 6144), F)
        qkv, beta, alpha = x["qkv"][None].copy(), x["beta"][None].copy(), x["alpha"][None].copy()
        cuda_ctx.linear_decode_host(st, layer, qkv, x["z"][None].copy(), beta, alpha, att)
        check_parity(att[0], GOLDEN[f"lin_attention_{t}"], TOL, "")
        assert relative_error(beta[0], GOLDEN[f"lin_beta_{t}"]) < 1e-6
        assert relative_error(alpha[0], GOLDEN[f"lin_alpha_{t}"]) < 1e-6
        if t == 0:
            assert relative_error(qkv[0], GOLDEN["lin_qkv_0"]) < 1e-5
    conv, delta = st.download_linear(layer, 0)
    check_parity(delta[0], GOLDEN["lin_delta_head0"], TOL, "")
    check_parity(delta[47], GOLDEN["lin_delta_head47"], TOL, "")
    np.testing.assert_array_equal(conv[::16], GOLDEN["lin_conv_final"])
    st.close()


def test_linear_decode_batched_multi_token(cuda_ctx, oracle_lib):
    """Four sequences with their own states, four tokens in a row, device API."""
    torch = _torch()
    from q38attn import synth
    g = synth.rng(11)
    w = synth.linear_weights(g)
    layer = 2
    cuda_ctx.bind_linear_layer(layer, w["conv1d"], w["dt_bias"], w["ssm_a"], w["ssm_norm"])
    B = 4
    st = cuda_ctx.state(B, 16, full_slots=0, linear_slots=3)
    states = [synth.linear_state(g) for _ in range(B)]
    for b in range(B):
        st.upload_linear(layer, b, states[b]["conv_state"], states[b]["delta_state"])
    for t in range(4):
        x = synth.linear_step(g, B)
        d = {k: torch.from_numpy(v.copy()).cuda() for k, v in x.items()}
        att = torch.zeros(B, 6144, device="cuda")
        cuda_ctx.linear_decode(st, layer, d["qkv"], d["z"], d["beta"], d["alpha"], att)
        torch.cuda.synchronize()
        for b in range(B):
            ox = {k: v[b].copy() for k, v in x.items()}
            oatt = np.zeros(6144, F)
            oracle_lib.linear_core(w, states[b]["conv_state"], states[b]["delta_state"],
                                   ox["qkv"], ox["z"], ox["beta"], ox["alpha"], oatt)
            check_parity(att[b].cpu().numpy(), oatt, TOL, str((t, b)))
            assert relative_error(d["qkv"][b].cpu().numpy(), ox["qkv"]) < 1e-5
    for b in range(B):
        conv, delta = st.download_linear(layer, b)
        np.testing.assert_array_equal(conv, states[b]["conv_state"])
        check_parity(delta, states[b]["delta_state"], TOL, "")
    assert st.errors() == 0
    st.close()


@pytest.mark.parametrize("pinned_host", [True, False])
@pytest.mark.parametrize("batch", [1, 32])
def test_linear_decode_host_equals_device_call(cuda_ctx, batch, pinned_host):
    """The host-pointer decode over pinned buffers lets the kernels read and
    write them in place (mapped host memory); over pageable buffers it stages
    copies. Either way its outputs, its in-place inputs and the state it
    leaves equal the device-pointer call bit for bit, two tokens in a row."""
    torch = _torch()
    from q38attn import synth
    g = synth.rng(12 + batch)
    w = synth.linear_weights(g)
    layer = 0
    cuda_ctx.bind_linear_layer(layer, w["conv1d"], w["dt_bias"], w["ssm_a"], w["ssm_norm"])
    sts = [cuda_ctx.state(batch, 16, full_slots=0, linear_slots=1) for _ in range(2)]
    for b in range(batch):
        s0 = synth.linear_state(g)
        for st in sts:
            st.upload_linear(layer, b, s0["conv_state"], s0["delta_state"])
    keep = []

    def pinned(a):
        if not pinned_host:
            return np.ascontiguousarray(a).copy()
        t = torch.from_numpy(np.ascontiguousarray(a)).pin_memory()
        keep.append(t)
        return t.numpy()

    for _ in range(2):
        x = synth.linear_step(g, batch)
        h = {k: pinned(v) for k, v in x.items()}
        att_h = pinned(np.zeros((batch, 6144), F))
        cuda_ctx.linear_decode_host(sts[0], layer, h["qkv"], h["z"], h["beta"], h["alpha"], att_h)
        d = {k: torch.from_numpy(v.copy()).cuda() for k, v in x.items()}
        att = torch.zeros(batch, 6144, device="cuda")
        cuda_ctx.linear_decode(sts[1], layer, d["qkv"], d["z"], d["beta"], d["alpha"], att)
        torch.cuda.synchronize()
        np.testing.assert_array_equal(att_h.view(np.uint32), att.cpu().numpy().view(np.uint32))
        for k in ("qkv", "beta", "alpha"):
            np.testing.assert_array_equal(h[k].view(np.uint32), d[k].cpu().numpy().view(np.uint32))
    for b in range(batch):
        for a, c in zip(sts[0].download_linear(layer, b), sts[1].download_linear(layer, b)):
            np.testing.assert_array_equal(a, c)
    assert sts[0].errors() == 0 and sts[1].errors() == 0
    for st in sts:
        st.close()


def test_linear_decode_rejects_full_layer(cuda_ctx):
    import q38attn
    st = cuda_ctx.state(1, 16, full_slots=1, linear_slots=1)
    z = np.zeros((1, 6144), F)
    with pytest.raises(q38attn.Q38Error) as e:
        cuda_ctx.linear_decode_host(st, 3, np.zeros((1, 10240), F), z, np.zeros((1, 48), F),
                                    np.zeros((1, 48), F), z.copy())
    assert e.value.code == q38attn.Q38_ERR_ARG
    st.close()


# ---------------------------------------------------------------------------
# Gated full attention
# ---------------------------------------------------------------------------
def _oracle_full(oracle_lib, w, x, kc, vc, ctx_len, pos, layer, bf16):
    q = np.zeros(6144, F)
    gate = np.zeros(6144, F)
    scores = np.zeros(24 * ctx_len, F)
    att = np.zeros(6144, F)
    key = x["key"].copy()
    rc = oracle_lib.full_core(w, x["q_and_gate"], key, x["value"], q, gate, scores, att, kc, vc,
                              ctx_len, pos, layer, bf16)
    assert rc == 0
    return att, key, q


def test_full_core_mirror_matches_oracle_config1(cuda_ctx, oracle_lib):
    """Config 1: batch 1, 256 cached fp32 positions, the new token at 256."""
    from q38attn import synth
    g = synth.rng(0)
    w = synth.full_weights(g)
    layer, ctx_len, pos = 3, 320, 256
    cuda_ctx.bind_full_layer(layer, w["q_norm"], w["k_norm"])
    st = cuda_ctx.state(1, ctx_len, full_slots=1, linear_slots=0)
    kc = np.zeros((ctx_len, 1024), F)
    vc = np.zeros((ctx_len, 1024), F)
    kc[:pos], vc[:pos] = synth.kv_rows(g, pos)
    x = {k: v[0].copy() for k, v in synth.full_step(g).items()}
    oatt, okey, oq = _oracle_full(oracle_lib, w, x, kc.copy(), vc.copy(), ctx_len, pos, layer,
                                  False)
    key = x["key"].copy()
    q = np.zeros(6144, F)
    gate = np.zeros(6144, F)
    att = np.zeros(6144, F)
    kc2, vc2 = kc.copy(), vc.copy()
    cuda_ctx.full_core(st, layer, x["q_and_gate"], key, x["value"], q, gate, None, att, kc2, vc2,
                       ctx_len, pos)
    check_parity(att, oatt, TOL, "")
    assert relative_error(key, okey) < 1e-5
    assert relative_error(q, oq) < 1e-5
    np.testing.assert_array_equal(gate.reshape(24, 256), x["q_and_gate"].reshape(24, 512)[:, 256:])
    assert relative_error(kc2[pos], okey) < 1e-5
    np.testing.assert_array_equal(vc2[pos], x["value"])
    st.close()


@pytest.mark.parametrize("bf16", [False, True])
def test_full_golden_vectors_on_gpu(cuda_ctx, bf16):
    import q38attn
    from q38attn.synth import round_bf16
    tag = "fullbf16" if bf16 else "full"
    w = V.full_weights()
    layer, ctx_len, pre = 7, 64, 37
    cuda_ctx.bind_full_layer(layer, w["q_norm"], w["k_norm"])
    st = cuda_ctx.state(1, ctx_len, full_slots=2, linear_slots=0,
                        kv_dtype=q38attn.Q38_KV_BF16 if bf16 else q38attn.Q38_KV_F32)
    kc, vc = V.full_cache(ctx_len, pre, layer, full_slots=2)
    base = (layer // 4) * ctx_len
    st.upload_kv(layer, 0, 0, np.ascontiguousarray(kc[base:base + pre]),
                 np.ascontiguousarray(vc[base:base + pre]))
    for t in range(3):
        x = V.full_token(t)
        att = np.zeros((1, 6144), F)
        key = x["key"][None].copy()
        cuda_ctx.full_decode_host(st, layer, x["q_and_gate"][None].copy(), key,
                                  x["value"][None].copy(), np.array([pre + t], np.int32), att)
        check_parity(att[0], GOLDEN[f"{tag}_attention_{t}"], TOL, str(t))
        assert relative_error(key[0], GOLDEN[f"{tag}_key_{t}"]) < 1e-5
    k, v = st.download_kv(layer, 0, pre, 3)
    for t in range(3):
        exp_k = GOLDEN[f"{tag}_krow_{t}"]
        assert relative_error(k[t], exp_k) < (1e-2 if bf16 else 1e-5)
        np.testing.assert_array_equal(v[t], GOLDEN[f"{tag}_vrow_{t}"])
    st.close()


@pytest.mark.parametrize("bf16", [False, True])
def test_full_decode_batch_mixed_positions(cuda_ctx, oracle_lib, bf16):
    """Five sequences at positions 0, 1, 63, 64 and 300 in one launch; the
    cache holds f32 or bf16 (the oracle then stores bf16-rounded rows)."""
    import q38attn
    from q38attn import synth
    torch = _torch()
    g = synth.rng(5 + bf16)
    w = synth.full_weights(g)
    layer, ctx_len = 11, 384
    positions = [0, 1, 63, 64, 300]
    B = len(positions)
    cuda_ctx.bind_full_layer(layer, w["q_norm"], w["k_norm"])
    st = cuda_ctx.state(B, ctx_len, full_slots=3, linear_slots=0,
                        kv_dtype=q38attn.Q38_KV_BF16 if bf16 else q38attn.Q38_KV_F32)
    caches = []
    for b, pos in enumerate(positions):
        kc = np.zeros((3 * ctx_len, 1024), F)
        vc = np.zeros((3 * ctx_len, 1024), F)
        base = (layer // 4) * ctx_len
        k, v = synth.kv_rows(g, max(pos, 1), bf16=bf16)
        kc[base:base + pos], vc[base:base + pos] = k[:pos], v[:pos]
        if pos:
            st.upload_kv(layer, b, 0, np.ascontiguousarray(k[:pos]), np.ascontiguousarray(v[:pos]))
        caches.append((kc, vc))
    x = synth.full_step(g, B)
    d = {k: torch.from_numpy(v.copy()).cuda() for k, v in x.items()}
    att = torch.zeros(B, 6144, device="cuda")
    cuda_ctx.full_decode(st, layer, d["q_and_gate"], d["key"], d["value"],
                         torch.tensor(positions, dtype=torch.int32, device="cuda"), att)
    torch.cuda.synchronize()
    for b, pos in enumerate(positions):
        ox = {k: v[b].copy() for k, v in x.items()}
        oatt, okey, _ = _oracle_full(oracle_lib, w, ox, caches[b][0], caches[b][1], ctx_len, pos,
                                     layer, bf16)
        check_parity(att[b].cpu().numpy(), oatt, TOL, str((b, pos)))
        assert relative_error(d["key"][b].cpu().numpy(), okey) < 1e-5
    assert st.errors() == 0
    st.close()


@pytest.mark.parametrize("pinned_host", [True, False])
def test_full_decode_host_equals_device_call(cuda_ctx, pinned_host):
    """The host-pointer decode over pinned buffers (the merge kernel writes
    `attention` into mapped host memory) and over pageable ones (staged
    copies) equals the device-pointer call on an identical state bit for bit:
    attention, the in-place key and the appended cache rows."""
    import q38attn
    from q38attn import synth
    torch = _torch()
    g = synth.rng(21)
    w = synth.full_weights(g)
    layer, ctx_len = 3, 320
    positions = np.array([0, 5, 64, 300], np.int32)
    B = len(positions)
    cuda_ctx.bind_full_layer(layer, w["q_norm"], w["k_norm"])
    sts = [cuda_ctx.state(B, ctx_len, full_slots=1, linear_slots=0, kv_dtype=q38attn.Q38_KV_BF16)
           for _ in range(2)]
    for b, pos in enumerate(positions):
        if pos:
            k, v = synth.kv_rows(g, int(pos), bf16=True)
            for st in sts:
                st.upload_kv(layer, b, 0, k, v)
    keep = []

    def host(a):
        if not pinned_host:
            return np.ascontiguousarray(a).copy()
        t = torch.from_numpy(np.ascontiguousarray(a)).pin_memory()
        keep.append(t)
        return t.numpy()

    x = synth.full_step(g, B)
    h = {k: host(v) for k, v in x.items()}
    att_h = host(np.zeros((B, 6144), F))
    cuda_ctx.full_decode_host(sts[0], layer, h["q_and_gate"], h["key"], h["value"], positions, att_h)
    d = {k: torch.from_numpy(v.copy()).cuda() for k, v in x.items()}
    att = torch.zeros(B, 6144, device="cuda")
    cuda_ctx.full_decode(sts[1], layer, d["q_and_gate"], d["key"], d["value"],
                         torch.from_numpy(positions).cuda(), att)
    torch.cuda.synchronize()
    np.testing.assert_array_equal(att_h.view(np.uint32), att.cpu().numpy().view(np.uint32))
    np.testing.assert_array_equal(h["key"].view(np.uint32), d["key"].cpu().numpy().view(np.uint32))
    for b, pos in enumerate(positions):
        for a, c in zip(sts[0].download_kv(layer, b, int(pos), 1), sts[1].download_kv(layer, b, int(pos), 1)):
            np.testing.assert_array_equal(a, c)
    assert sts[0].errors() == 0 and sts[1].errors() == 0
    for st in sts:
        st.close()


def test_split_count_does_not_change_the_result(cuda_ctx):
    """The LSE merge is invariant to how positions are split across CTAs. The
    split plan depends on the batch (it fills the SMs in whole waves), so the
    same sequence decoded alone (64-position splits) and as one of 8 identical
    sequences (384-position splits) must agree to rounding."""
    import q38attn
    from q38attn import synth
    torch = _torch()
    g = synth.rng(9)
    w = synth.full_weights(g)
    layer, ctx_len, pos = 15, 4096, 3000
    cuda_ctx.bind_full_layer(layer, w["q_norm"], w["k_norm"])
    k, v = synth.kv_rows(g, pos, bf16=True)
    x = synth.full_step(g, 1)
    outs = []
    for batch in (1, 8):
        st = cuda_ctx.state(batch, ctx_len, full_slots=4, linear_slots=0,
                            kv_dtype=q38attn.Q38_KV_BF16)
        for b in range(batch):
            st.upload_kv(layer, b, 0, k, v)
        d = {kk: torch.from_numpy(np.repeat(vv, batch, axis=0)).cuda() for kk, vv in x.items()}
        att = torch.zeros(batch, 6144, device="cuda")
        cuda_ctx.full_decode(st, layer, d["q_and_gate"], d["key"], d["value"],
                             torch.full((batch,), pos, dtype=torch.int32, device="cuda"), att,
                             max_position=pos)
        torch.cuda.synchronize()
        outs.append(att.cpu().numpy())
        st.close()
    assert relative_error(outs[1], np.repeat(outs[0], 8, axis=0)) < 1e-6
    assert relative_error(outs[0], outs[1][:1]) < 1e-6


def test_full_decode_long_context_large_splits(cuda_ctx, oracle_lib):
    """One sequence at position 69999 of a 70000-position bf16 cache: 137
    splits of 512 positions (eight 64-key tiles, every TMEM score column in
    use), the last split ending inside a tile."""
    import q38attn
    from q38attn import synth
    torch = _torch()
    g = synth.rng(13)
    w = synth.full_weights(g)
    layer, ctx_len, pos = 3, 70000, 69999
    cuda_ctx.bind_full_layer(layer, w["q_norm"], w["k_norm"])
    st = cuda_ctx.state(1, ctx_len, full_slots=1, linear_slots=0, kv_dtype=q38attn.Q38_KV_BF16)
    k, v = synth.kv_rows(g, pos, bf16=True)
    st.upload_kv(layer, 0, 0, k, v)
    kc = np.zeros((ctx_len, 1024), F)
    vc = np.zeros((ctx_len, 1024), F)
    kc[:pos], vc[:pos] = k, v
    del k, v
    x = synth.full_step(g, 1)
    d = {kk: torch.from_numpy(vv.copy()).cuda() for kk, vv in x.items()}
    att = torch.zeros(1, 6144, device="cuda")
    cuda_ctx.full_decode(st, layer, d["q_and_gate"], d["key"], d["value"],
                         torch.tensor([pos], dtype=torch.int32, device="cuda"), att)
    torch.cuda.synchronize()
    ox = {kk: vv[0].copy() for kk, vv in x.items()}
    oatt, okey, _ = _oracle_full(oracle_lib, w, ox, kc, vc, ctx_len, pos, layer, True)
    check_parity(att[0].cpu().numpy(), oatt, TOL, "")
    assert relative_error(d["key"][0].cpu().numpy(), okey) < 1e-5
    assert st.errors() == 0
    st.close()


def test_full_core_position_errors(cuda_ctx):
    """Err(-1) paths of full_core (ops.rs:860-864) and device-side position checks."""
    import q38attn
    torch = _torch()
    w = V.full_weights()
    layer, ctx_len = 3, 32
    cuda_ctx.bind_full_layer(layer, w["q_norm"], w["k_norm"])
    st = cuda_ctx.state(2, ctx_len, full_slots=1, linear_slots=0)
    x = V.full_token(0)
    kc = np.zeros((ctx_len, 1024), F)
    vc = np.zeros((ctx_len, 1024), F)
    att = np.zeros(6144, F)
    with pytest.raises(q38attn.Q38Error) as e:  # row past the host cache
        cuda_ctx.full_core(st, layer, x["q_and_gate"], x["key"].copy(), x["value"], None, None,
                           None, att, kc, vc, ctx_len, ctx_len)
    assert e.value.code == q38attn.Q38_ERR_ARG
    with pytest.raises(q38attn.Q38Error) as e:  # not a full-attention layer
        cuda_ctx.full_core(st, 2, x["q_and_gate"], x["key"].copy(), x["value"], None, None,
                           None, att, kc, vc, ctx_len, 0)
    assert e.value.code == q38attn.Q38_ERR_ARG
    with pytest.raises(q38attn.Q38Error):  # host form validates positions first
        cuda_ctx.full_decode_host(st, layer, x["q_and_gate"][None].copy(), x["key"][None].copy(),
                                  x["value"][None].copy(), np.array([ctx_len], np.int32),
                                  np.zeros((1, 6144), F))
    # Device form: sequence 1 is out of range -> flagged and skipped; sequence 0 runs.
    qg = torch.from_numpy(np.stack([x["q_and_gate"]] * 2)).cuda()
    key = torch.from_numpy(np.stack([x["key"]] * 2)).cuda()
    val = torch.from_numpy(np.stack([x["value"]] * 2)).cuda()
    out = torch.full((2, 6144), 7.0, device="cuda")
    cuda_ctx.full_decode(st, layer, qg, key, val,
                         torch.tensor([0, ctx_len + 5], dtype=torch.int32, device="cuda"), out)
    torch.cuda.synchronize()
    assert st.errors() & q38attn.Q38_DEVERR_POSITION
    assert torch.all(out[1] == 7.0)
    assert torch.isfinite(out[0]).all() and not torch.all(out[0] == 7.0)
    assert st.errors() == 0  # cleared by the read
    st.close()


# ---------------------------------------------------------------------------
# The bench's shapes
# ---------------------------------------------------------------------------
def _kv_host_rows(view, b, n):
    """Rows 0..n-1 of sequence b of a device KV view [batch][4][ctx][256] in
    the reference's host layout [n][1024] (f32)."""
    return np.ascontiguousarray(view[b, :, :n].permute(1, 0, 2).reshape(n, 1024).float().cpu()
                                .numpy())


def test_full_decode_headline_shape(cuda_ctx, oracle_lib):
    """The headline workload's attention layer: 32 sequences at 32778 cached
    bf16 positions (the bench's first timed step: 32768 + 10 warm-up steps),
    one new token each, with the split plan the planner picks for that batch
    (512-position splits, 65 per kv head). Four sampled sequences against the
    oracle (bf16 cache rows, new row rounded as the cache stores it)."""
    torch = _torch()
    import q38attn
    from q38attn import synth
    g = synth.rng(40)
    w = synth.full_weights(g)
    layer, B, pos = 3, 32, 32768 + 10
    cap = pos + 8
    cuda_ctx.bind_full_layer(layer, w["q_norm"], w["k_norm"])
    st = cuda_ctx.state(B, cap, full_slots=1, linear_slots=0, kv_dtype=q38attn.Q38_KV_BF16)
    kview, vview = st.kv_views(layer)
    tg = torch.Generator(device="cuda")
    tg.manual_seed(40)
    kview[:, :, :pos].normal_(generator=tg)
    vview[:, :, :pos].normal_(generator=tg)
    sample = [0, 9, 22, 31]
    caches = {b: (_kv_host_rows(kview, b, cap), _kv_host_rows(vview, b, cap)) for b in sample}
    x = synth.full_step(g, B)
    d = {k: torch.from_numpy(v.copy()).cuda() for k, v in x.items()}
    att = torch.zeros(B, 6144, device="cuda")
    positions = torch.full((B,), pos, dtype=torch.int32, device="cuda")
    cuda_ctx.full_decode(st, layer, d["q_and_gate"], d["key"], d["value"], positions, att,
                         max_position=pos)
    torch.cuda.synchronize()
    assert st.errors() == 0
    for b in sample:
        kc, vc = caches[b]
        okey = x["key"][b].copy()
        q = np.zeros(6144, F)
        gate = np.zeros(6144, F)
        scores = np.zeros(24 * cap, F)
        oatt = np.zeros(6144, F)
        assert oracle_lib.full_core(w, x["q_and_gate"][b], okey, x["value"][b], q, gate, scores,
                                    oatt, kc, vc, cap, pos, layer, 1) == 0
        check_parity(att[b].cpu().numpy(), oatt, TOL, f"seq {b}")
        assert relative_error(d["key"][b].cpu().numpy(), okey) < 1e-5
    del kview, vview
    st.close()


def test_full_decode_split_sequence_length_one_gpu(cuda_ctx, oracle_lib):
    """Config 3's split-sequence length on one GPU: one sequence at 131072
    cached bf16 positions (the planner's many-split plan for a batch of one)."""
    torch = _torch()
    import q38attn
    from q38attn import synth
    g = synth.rng(41)
    w = synth.full_weights(g)
    layer, pos = 3, 131072
    cap = pos + 4
    cuda_ctx.bind_full_layer(layer, w["q_norm"], w["k_norm"])
    st = cuda_ctx.state(1, cap, full_slots=1, linear_slots=0, kv_dtype=q38attn.Q38_KV_BF16)
    kview, vview = st.kv_views(layer)
    tg = torch.Generator(device="cuda")
    tg.manual_seed(41)
    kview[:, :, :pos].normal_(generator=tg)
    vview[:, :, :pos].normal_(generator=tg)
    kc, vc = _kv_host_rows(kview, 0, cap), _kv_host_rows(vview, 0, cap)
    x = synth.full_step(g, 1)
    d = {k: torch.from_numpy(v.copy()).cuda() for k, v in x.items()}
    att = torch.zeros(1, 6144, device="cuda")
    cuda_ctx.full_decode(st, layer, d["q_and_gate"], d["key"], d["value"],
                         torch.tensor([pos], dtype=torch.int32, device="cuda"), att,
                         max_position=pos)
    torch.cuda.synchronize()
    assert st.errors() == 0
    okey = x["key"][0].copy()
    q = np.zeros(6144, F)
    gate = np.zeros(6144, F)
    scores = np.zeros(24 * cap, F)
    oatt = np.zeros(6144, F)
    assert oracle_lib.full_core(w, x["q_and_gate"][0], okey, x["value"][0], q, gate, scores, oatt,
                                kc, vc, cap, pos, layer, 1) == 0
    check_parity(att[0].cpu().numpy(), oatt, TOL, "131072 positions")
    del kview, vview
    st.close()


def test_linear_decode_headline_batch(cuda_ctx, oracle_lib):
    """The headline workload's DeltaNet layer: 32 sequences, two tokens, every
    sequence's output and final state against the oracle."""
    torch = _torch()
    from q38attn import synth
    g = synth.rng(42)
    w = synth.linear_weights(g)
    layer, B = 0, 32
    cuda_ctx.bind_linear_layer(layer, w["conv1d"], w["dt_bias"], w["ssm_a"], w["ssm_norm"])
    st = cuda_ctx.state(B, 16, full_slots=0, linear_slots=1)
    states = [synth.linear_state(g) for _ in range(B)]
    for b in range(B):
        st.upload_linear(layer, b, states[b]["conv_state"], states[b]["delta_state"])
    for t in range(2):
        x = synth.linear_step(g, B)
        d = {k: torch.from_numpy(v.copy()).cuda() for k, v in x.items()}
        att = torch.zeros(B, 6144, device="cuda")
        cuda_ctx.linear_decode(st, layer, d["qkv"], d["z"], d["beta"], d["alpha"], att)
        torch.cuda.synchronize()
        got = att.cpu().numpy()
        want = np.zeros((B, 6144), F)
        for b in range(B):
            ox = {k: v[b].copy() for k, v in x.items()}
            oracle_lib.linear_core(w, states[b]["conv_state"], states[b]["delta_state"],
                                   ox["qkv"], ox["z"], ox["beta"], ox["alpha"], want[b])
        check_parity(got, want, TOL, f"token {t}, 32 sequences")
    for b in range(B):
        conv, delta = st.download_linear(layer, b)
        np.testing.assert_array_equal(conv, states[b]["conv_state"])
        check_parity(delta, states[b]["delta_state"], TOL, f"state seq {b}")
    assert st.errors() == 0
    st.close()

"""GPU tests of the layer-level prefill calls, the bodies of
batch_linear_attention (src/model/ops.rs:1032-1114) and batch_full_attention
(ops.rs:1116-1185): projections of every prompt token, the prefill core, the
output projection.

Each call must equal, bit for bit, the same steps taken one by one through the
public API -- q38_project (itself bit-identical to the reference's integer
path, tests/test_proj_gpu.py) and q38_linear_prefill / q38_full_prefill
(checked against the per-token oracle loop in tests/test_deltanet_prefill_gpu.py
and tests/test_prefill_gpu.py) -- including the state they leave (conv and
delta state, appended KV rows). Prompts of 100 tokens per sequence take the
tensor-core projections (9+ tokens) and a ragged last DeltaNet chunk; each
test runs with and without the weights' integer planes.
"""
from __future__ import annotations

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

HIDDEN = 5120


def _weights(ctx, g, spec, planes=False):
    """The layer's weights; with `planes`, the K-quant ones (Q4_K, Q5_K,
    Q6_K) also get integer planes (q38_weight_build_planes)."""
    from q38attn import synth
    out = {k: ctx.weight(t, w, r, synth.quant_weight(g, t, r, w)) for k, (t, w, r) in spec.items()}
    if planes:
        for k, (t, _, _) in spec.items():
            if t in (12, 13, 14):
                out[k].build_planes()
    return out


def _project(ctx, w, x):
    import torch
    out = torch.zeros(x.shape[0], w.rows, device="cuda")
    ctx.project(w, x, out)
    return out


@pytest.mark.parametrize("planes", [False, True])
def test_linear_attention_prefill_equals_its_steps(cuda_ctx, planes):
    import torch
    from q38attn import synth
    g = synth.rng(500)
    layer, nseq, count = 0, 2, 100
    lw = synth.linear_weights(g)
    cuda_ctx.bind_linear_layer(layer, lw["conv1d"], lw["dt_bias"], lw["ssm_a"], lw["ssm_norm"])
    w = _weights(cuda_ctx, g, {"qkv": (12, HIDDEN, 10240), "z": (13, HIDDEN, 6144),
                               "beta": (8, HIDDEN, 48), "alpha": (0, HIDDEN, 48),
                               "out": (14, 6144, HIDDEN)}, planes)
    init = [synth.linear_state(g) for _ in range(nseq)]
    norm = torch.from_numpy(synth.normal(g, (nseq, count, HIDDEN))).cuda()
    states = []
    for _ in range(2):
        st = cuda_ctx.state(nseq, 16, full_slots=0, linear_slots=1)
        st.reserve_attention_prefill(nseq * count)
        for b, s0 in enumerate(init):
            st.upload_linear(layer, b, s0["conv_state"], s0["delta_state"])
        states.append(st)

    branch = torch.zeros(nseq, count, HIDDEN, device="cuda")
    cuda_ctx.linear_attention_prefill(states[0], layer, 0, w, norm, branch)

    flat = norm.reshape(nseq * count, HIDDEN)
    qkv = _project(cuda_ctx, w["qkv"], flat).reshape(nseq, count, 10240)
    z = _project(cuda_ctx, w["z"], flat).reshape(nseq, count, 6144)
    beta = _project(cuda_ctx, w["beta"], flat).reshape(nseq, count, 48)
    alpha = _project(cuda_ctx, w["alpha"], flat).reshape(nseq, count, 48)
    att = torch.zeros(nseq, count, 6144, device="cuda")
    cuda_ctx.linear_prefill(states[1], layer, 0, qkv, z, beta, alpha, att)
    want = _project(cuda_ctx, w["out"], att.reshape(nseq * count, 6144))
    torch.cuda.synchronize()

    np.testing.assert_array_equal(branch.reshape(nseq * count, HIDDEN).cpu().numpy().view(np.uint32),
                                  want.cpu().numpy().view(np.uint32))
    for b in range(nseq):
        for a, c in zip(states[0].download_linear(layer, b), states[1].download_linear(layer, b)):
            np.testing.assert_array_equal(a, c)
    assert states[0].errors() == 0 and states[1].errors() == 0
    for st in states:
        st.close()
    for x in w.values():
        x.close()


@pytest.mark.parametrize("planes", [False, True])
def test_full_attention_prefill_equals_its_steps(cuda_ctx, planes):
    """Two calls in a row: a 100-token prompt at position 0, then 100 more
    tokens at position 100 over the cached rows."""
    import q38attn
    import torch
    from q38attn import synth
    g = synth.rng(501)
    layer, nseq, count, ctx_len = 3, 2, 100, 256
    fw = synth.full_weights(g)
    cuda_ctx.bind_full_layer(layer, fw["q_norm"], fw["k_norm"])
    w = _weights(cuda_ctx, g, {"q": (12, HIDDEN, 12288), "k": (14, HIDDEN, 1024),
                               "v": (8, HIDDEN, 1024), "out": (12, 6144, HIDDEN)}, planes)
    states = []
    for _ in range(2):
        st = cuda_ctx.state(nseq, ctx_len, full_slots=1, linear_slots=0, kv_dtype=q38attn.Q38_KV_BF16)
        st.reserve_attention_prefill(nseq * count)
        states.append(st)
    for base in (0, count):
        norm = torch.from_numpy(synth.normal(g, (nseq, count, HIDDEN))).cuda()
        branch = torch.zeros(nseq, count, HIDDEN, device="cuda")
        cuda_ctx.full_attention_prefill(states[0], layer, 0, base, w, norm, branch)

        flat = norm.reshape(nseq * count, HIDDEN)
        qg = _project(cuda_ctx, w["q"], flat).reshape(nseq, count, 12288)
        key = _project(cuda_ctx, w["k"], flat).reshape(nseq, count, 1024)
        value = _project(cuda_ctx, w["v"], flat).reshape(nseq, count, 1024)
        att = torch.zeros(nseq, count, 6144, device="cuda")
        cuda_ctx.full_prefill(states[1], layer, 0, qg, key, value, att, base)
        want = _project(cuda_ctx, w["out"], att.reshape(nseq * count, 6144))
        torch.cuda.synchronize()
        np.testing.assert_array_equal(
            branch.reshape(nseq * count, HIDDEN).cpu().numpy().view(np.uint32),
            want.cpu().numpy().view(np.uint32), err_msg=f"base {base}")
    for b in range(nseq):
        for a, c in zip(states[0].download_kv(layer, b, 0, 2 * count),
                        states[1].download_kv(layer, b, 0, 2 * count)):
            np.testing.assert_array_equal(a, c)
    assert states[0].errors() == 0 and states[1].errors() == 0
    for st in states:
        st.close()
    for x in w.values():
        x.close()


def test_attention_prefill_needs_its_reservation(cuda_ctx):
    import q38attn
    import torch
    from q38attn import synth
    g = synth.rng(502)
    w = _weights(cuda_ctx, g, {"qkv": (12, HIDDEN, 10240), "z": (12, HIDDEN, 6144),
                               "beta": (8, HIDDEN, 48), "alpha": (8, HIDDEN, 48),
                               "out": (14, 6144, HIDDEN)})
    st = cuda_ctx.state(1, 16, full_slots=0, linear_slots=1)
    norm = torch.zeros(1, 32, HIDDEN, device="cuda")
    branch = torch.zeros(1, 32, HIDDEN, device="cuda")
    with pytest.raises(q38attn.Q38Error) as e:
        cuda_ctx.linear_attention_prefill(st, 0, 0, w, norm, branch)
    assert e.value.code == q38attn.Q38_ERR_ARG
    st.reserve_attention_prefill(16)
    with pytest.raises(q38attn.Q38Error):  # 32 tokens > the 16 reserved
        cuda_ctx.linear_attention_prefill(st, 0, 0, w, norm, branch)
    st.close()
    for x in w.values():
        x.close()

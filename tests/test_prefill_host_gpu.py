"""GPU tests of the host-pointer prefill entry points (q38_full_prefill_host,
q38_linear_prefill_host): the form the reference's host loops
(batch_full_attention, src/model/ops.rs:1156-1172; batch_linear_attention,
ops.rs:1088-1099) would call with their host slices.

The host forms stream the prompt through a staging buffer of at most 4096
tokens, so prompts longer than that run as several pieces, each continuing
from the cache rows and recurrent state the previous one left. Each case here
takes more than one piece and is compared with the device-pointer form on the
same inputs from the same starting state; the device-pointer forms are checked
against the CPU oracle in test_prefill_gpu.py and test_deltanet_prefill_gpu.py.
Pieces start on 128-token (attention) and 64-token (DeltaNet chunk) boundaries,
so the two forms do the same arithmetic; tolerance 1e-6 on the reference's
metric |a-b|/max(|b|,1)."""
from __future__ import annotations

import numpy as np
import pytest

from conftest import relative_error

pytestmark = pytest.mark.gpu

F = np.float32


def _pinned(a: np.ndarray) -> np.ndarray:
    import torch
    t = torch.from_numpy(np.ascontiguousarray(a)).pin_memory()
    return t.numpy()


@pytest.mark.parametrize("nseq,count,base", [(1, 4396, 0), (2, 2500, 64)])
def test_full_prefill_host_matches_device_form(cuda_ctx, nseq, count, base):
    import torch

    import q38attn
    from q38attn import synth
    g = synth.rng(40 + nseq)
    w = synth.full_weights(g)
    layer, ctx_len = 3, base + count
    cuda_ctx.bind_full_layer(layer, w["q_norm"], w["k_norm"])
    sts = []
    for _ in range(2):
        st = cuda_ctx.state(nseq, ctx_len, full_slots=1, linear_slots=0,
                            kv_dtype=q38attn.Q38_KV_BF16)
        st.reserve_prefill(nseq * count)
        sts.append(st)
    if base:
        for s in range(nseq):
            k, v = synth.kv_rows(g, base, bf16=True)
            for st in sts:
                st.upload_kv(layer, s, 0, np.ascontiguousarray(k), np.ascontiguousarray(v))
    x = {k: v.reshape(nseq, count, -1) for k, v in synth.full_step(g, nseq * count).items()}

    d = {k: torch.from_numpy(v.copy()).cuda() for k, v in x.items()}
    att_d = torch.empty(nseq, count, 6144, device="cuda")
    cuda_ctx.full_prefill(sts[0], layer, 0, d["q_and_gate"], d["key"], d["value"], att_d, base)
    torch.cuda.synchronize()

    h = {k: _pinned(v) for k, v in x.items()}
    att_h = _pinned(np.full((nseq, count, 6144), np.nan, F))
    cuda_ctx.full_prefill_host(sts[1], layer, 0, h["q_and_gate"], h["key"], h["value"], att_h,
                               base)
    assert np.isfinite(att_h).all()
    assert relative_error(att_h, att_d.cpu().numpy()) < 1e-6
    assert relative_error(h["key"], d["key"].cpu().numpy()) < 1e-6
    for s in range(nseq):
        ka, va = sts[0].download_kv(layer, s, base, count)
        kb, vb = sts[1].download_kv(layer, s, base, count)
        np.testing.assert_array_equal(kb, ka)
        np.testing.assert_array_equal(vb, va)
    for st in sts:
        assert st.errors() == 0
        st.close()


@pytest.mark.parametrize("nseq,count", [(1, 4396), (2, 2500)])
def test_linear_prefill_host_matches_device_form(cuda_ctx, nseq, count):
    import torch

    from q38attn import synth
    g = synth.rng(50 + nseq)
    w = synth.linear_weights(g)
    layer = 0
    cuda_ctx.bind_linear_layer(layer, w["conv1d"], w["dt_bias"], w["ssm_a"], w["ssm_norm"])
    sts = []
    for _ in range(2):
        st = cuda_ctx.state(nseq, 16, full_slots=0, linear_slots=1)
        st.reserve_prefill(nseq * count)
        sts.append(st)
    for s in range(nseq):
        init = synth.linear_state(g)
        for st in sts:
            st.upload_linear(layer, s, init["conv_state"], init["delta_state"])
    x = {k: v.reshape(nseq, count, -1) for k, v in synth.linear_step(g, nseq * count).items()}

    d = {k: torch.from_numpy(v.copy()).cuda() for k, v in x.items()}
    att_d = torch.empty(nseq, count, 6144, device="cuda")
    cuda_ctx.linear_prefill(sts[0], layer, 0, d["qkv"], d["z"], d["beta"], d["alpha"], att_d)
    torch.cuda.synchronize()

    h = {k: _pinned(v) for k, v in x.items()}
    att_h = _pinned(np.full((nseq, count, 6144), np.nan, F))
    cuda_ctx.linear_prefill_host(sts[1], layer, 0, h["qkv"], h["z"], h["beta"], h["alpha"],
                                 att_h)
    assert np.isfinite(att_h).all()
    assert relative_error(att_h, att_d.cpu().numpy()) < 1e-6
    for name in ("qkv", "beta", "alpha"):
        assert relative_error(h[name], d[name].cpu().numpy()) < 1e-6, name
    for s in range(nseq):
        ca, da = sts[0].download_linear(layer, s)
        cb, db = sts[1].download_linear(layer, s)
        assert relative_error(cb, ca) < 1e-6
        assert relative_error(db, da) < 1e-6
    for st in sts:
        assert st.errors() == 0
        st.close()


def test_prefill_host_argument_errors(cuda_ctx):
    import q38attn
    from q38attn import synth
    g = synth.rng(60)
    w = synth.full_weights(g)
    cuda_ctx.bind_full_layer(3, w["q_norm"], w["k_norm"])
    st = cuda_ctx.state(1, 64, full_slots=1, linear_slots=0, kv_dtype=q38attn.Q38_KV_BF16)
    qg = np.zeros((1, 8, 12288), F)
    k = np.zeros((1, 8, 1024), F)
    a = np.zeros((1, 8, 6144), F)
    with pytest.raises(q38attn.Q38Error) as e:  # no staging reserved
        cuda_ctx.full_prefill_host(st, 3, 0, qg, k, k.copy(), a, 0)
    assert e.value.code == q38attn.Q38_ERR_ARG
    st.reserve_prefill(8)
    with pytest.raises(q38attn.Q38Error) as e:  # positions past the cache
        cuda_ctx.full_prefill_host(st, 3, 0, qg, k, k.copy(), a, 60)
    assert e.value.code == q38attn.Q38_ERR_ARG
    st.close()

"""GPU parity tests of the chunked Gated DeltaNet prefill against the CPU
oracle's per-token linear_core loop (batch_linear_attention,
src/model/ops.rs:1088-1099), on the same seeded inputs: outputs, the final
delta and conv states, and the in-place qkv/beta/alpha results.

The chunked form is f32 throughout; tolerance |a-b|/max(|b|,1) < 1e-3 for the
outputs and state (the prefill contract allows 2e-3)."""
from __future__ import annotations

import numpy as np
import pytest

from conftest import relative_error

pytestmark = pytest.mark.gpu

TOL = 1e-3
F = np.float32


def _case(cuda_ctx, oracle_lib, *, nseq, count, layer, seed, fresh, batch=None):
    import torch

    from q38attn import synth
    g = synth.rng(seed)
    w = synth.linear_weights(g)
    cuda_ctx.bind_linear_layer(layer, w["conv1d"], w["dt_bias"], w["ssm_a"], w["ssm_norm"])
    batch = batch or nseq
    seq0 = batch - nseq
    import q38attn
    slots = q38attn.recurrent_index(layer) + 1
    st = cuda_ctx.state(batch, 16, full_slots=0, linear_slots=slots)
    st.reserve_prefill(nseq * count)
    states = []
    for s in range(nseq):
        if fresh:
            stt = {"conv_state": np.zeros((10240, 3), F),
                   "delta_state": np.zeros((48, 128, 128), F)}
        else:
            stt = synth.linear_state(g)
        st.upload_linear(layer, seq0 + s, stt["conv_state"], stt["delta_state"])
        states.append(stt)
    x = {k: v.reshape(nseq, count, -1) for k, v in synth.linear_step(g, nseq * count).items()}
    d = {k: torch.from_numpy(v.copy()).cuda() for k, v in x.items()}
    att = torch.full((nseq, count, 6144), float("nan"), device="cuda")
    cuda_ctx.linear_prefill(st, layer, seq0, d["qkv"], d["z"], d["beta"], d["alpha"], att)
    torch.cuda.synchronize()
    assert st.errors() == 0
    att = att.cpu().numpy()
    out = {k: v.cpu().numpy() for k, v in d.items()}
    worst = 0.0
    for s in range(nseq):
        ox = {k: np.ascontiguousarray(v[s]) for k, v in x.items()}
        oatt = np.zeros((count, 6144), F)
        conv, delta = states[s]["conv_state"].copy(), states[s]["delta_state"].copy()
        assert oracle_lib.linear_prefill(w, conv, delta, ox["qkv"], ox["z"], ox["beta"],
                                         ox["alpha"], oatt) == 0
        assert np.isfinite(att[s]).all()
        e = relative_error(att[s], oatt)
        worst = max(worst, e)
        assert e < TOL, (s, e)
        assert relative_error(out["qkv"][s], ox["qkv"]) < 1e-5
        # The gates go through expf/logf: CUDA's and the host libm's differ by an ulp.
        assert relative_error(out["beta"][s], ox["beta"]) < 1e-5
        assert relative_error(out["alpha"][s], ox["alpha"]) < 1e-5
        gconv, gdelta = st.download_linear(layer, seq0 + s)
        np.testing.assert_array_equal(gconv, conv)
        es = relative_error(gdelta, delta)
        print(f"linear prefill count={count} seq={s}: output err {e:.2e}, state err {es:.2e}")
        assert es < TOL
    st.close()
    return worst


def test_linear_prefill_partial_chunk_carried_state(cuda_ctx, oracle_lib):
    """100 tokens (one full chunk of 64 and a partial one) after the config-2 state."""
    _case(cuda_ctx, oracle_lib, nseq=1, count=100, layer=0, seed=1, fresh=False)


def test_linear_prefill_two_sequences_fresh_state(cuda_ctx, oracle_lib):
    """Two of three sequences, 256 tokens each, from a zero state (a new prompt)."""
    _case(cuda_ctx, oracle_lib, nseq=2, count=256, layer=5, seed=2, fresh=True, batch=3)


def test_linear_prefill_short_prompts(cuda_ctx, oracle_lib):
    for count in (1, 3, 63, 64, 65):
        _case(cuda_ctx, oracle_lib, nseq=1, count=count, layer=1, seed=10 + count, fresh=False)


def test_linear_prefill_config5_length(cuda_ctx, oracle_lib):
    """Config 5 length for one sequence: 8192 tokens, every output and the final
    state against the token-by-token recurrence."""
    _case(cuda_ctx, oracle_lib, nseq=1, count=8192, layer=2, seed=5, fresh=True)


def test_linear_prefill_then_decode_continues(cuda_ctx, oracle_lib):
    import torch

    from q38attn import synth
    g = synth.rng(7)
    w = synth.linear_weights(g)
    layer, count = 0, 200
    cuda_ctx.bind_linear_layer(layer, w["conv1d"], w["dt_bias"], w["ssm_a"], w["ssm_norm"])
    st = cuda_ctx.state(1, 16, full_slots=0, linear_slots=1)
    st.reserve_prefill(count)
    stt = synth.linear_state(g)
    st.upload_linear(layer, 0, stt["conv_state"], stt["delta_state"])
    x = {k: v.reshape(1, count, -1) for k, v in synth.linear_step(g, count).items()}
    d = {k: torch.from_numpy(v.copy()).cuda() for k, v in x.items()}
    att = torch.empty(1, count, 6144, device="cuda")
    cuda_ctx.linear_prefill(st, layer, 0, d["qkv"], d["z"], d["beta"], d["alpha"], att)
    conv, delta = stt["conv_state"].copy(), stt["delta_state"].copy()
    oatt = np.zeros((count, 6144), F)
    ox = {k: np.ascontiguousarray(v[0]) for k, v in x.items()}
    oracle_lib.linear_prefill(w, conv, delta, ox["qkv"], ox["z"], ox["beta"], ox["alpha"], oatt)
    for step in range(2):
        y = synth.linear_step(g, 1)
        dy = {k: torch.from_numpy(v.copy()).cuda() for k, v in y.items()}
        out = torch.empty(1, 6144, device="cuda")
        cuda_ctx.linear_decode(st, layer, dy["qkv"], dy["z"], dy["beta"], dy["alpha"], out)
        torch.cuda.synchronize()
        oy = {k: v[0].copy() for k, v in y.items()}
        oo = np.zeros(6144, F)
        oracle_lib.linear_core(w, conv, delta, oy["qkv"], oy["z"], oy["beta"], oy["alpha"], oo)
        assert relative_error(out[0].cpu().numpy(), oo) < TOL, step
    assert st.errors() == 0
    st.close()


def test_linear_prefill_argument_errors(cuda_ctx):
    import torch

    import q38attn
    w = {"conv1d": np.zeros((10240, 4), F), "dt_bias": np.zeros(48, F),
         "ssm_a": np.zeros(48, F), "ssm_norm": np.ones(128, F)}
    cuda_ctx.bind_linear_layer(0, w["conv1d"], w["dt_bias"], w["ssm_a"], w["ssm_norm"])
    st = cuda_ctx.state(1, 16, full_slots=1, linear_slots=1)
    qkv = torch.zeros(1, 4, 10240, device="cuda")
    z = torch.zeros(1, 4, 6144, device="cuda")
    b = torch.zeros(1, 4, 48, device="cuda")
    with pytest.raises(q38attn.Q38Error):  # no scratch reserved
        cuda_ctx.linear_prefill(st, 0, 0, qkv, z, b, b.clone(), z.clone())
    st.reserve_prefill(4)
    with pytest.raises(q38attn.Q38Error) as e:  # a full-attention layer
        cuda_ctx.linear_prefill(st, 3, 0, qkv, z, b, b.clone(), z.clone())
    assert e.value.code == q38attn.Q38_ERR_ARG
    st.close()

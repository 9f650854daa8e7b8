"""GPU parity tests of the chunked Gated DeltaNet prefill against the CPU
oracle's per-token linear_core loop (batch_linear_attention,
src/model/ops.rs:1088-1099), on the same seeded inputs: outputs, the final
delta and conv states, and the in-place qkv/beta/alpha results.

The chunk products run on the tcgen05 tensor cores with every operand split
into a bf16 (hi, lo) pair and f32 accumulation (~1e-5 of the per-token
recurrence); tolerance 1e-3 on both the reference's metric |a-b|/max(|b|,1)
and the scale-aware max|a-b|/max|b|, for the outputs and the final state (the
prefill contract allows 2e-3)."""
from __future__ import annotations

import numpy as np
import pytest

from conftest import check_parity, relative_error

pytestmark = pytest.mark.gpu

TOL = 1e-3
F = np.float32


def _case(cuda_ctx, oracle_lib, *, nseq, count, layer, seed, fresh, batch=None, v_range=None):
    """v_range=(h0, n): only value heads h0..h0+n-1 (q38_linear_prefill_heads);
    the q/k channels are processed in full, everything else of the other value
    heads (outputs, gates, v channels, conv and delta state) stays untouched."""
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
    x0 = {k: v.copy() for k, v in x.items()}  # the oracle below rewrites x in place
    d = {k: torch.from_numpy(v.copy()).cuda() for k, v in x.items()}
    att = torch.full((nseq, count, 6144), float("nan"), device="cuda")
    if v_range is None:
        cuda_ctx.linear_prefill(st, layer, seq0, d["qkv"], d["z"], d["beta"], d["alpha"], att)
        heads = np.arange(48)
    else:
        cuda_ctx.linear_prefill_heads(st, layer, seq0, d["qkv"], d["z"], d["beta"], d["alpha"],
                                      att, v_range[0], v_range[1])
        heads = np.arange(v_range[0], v_range[0] + v_range[1])
    torch.cuda.synchronize()
    assert st.errors() == 0
    att = att.cpu().numpy()
    out = {k: v.cpu().numpy() for k, v in d.items()}
    others = np.setdiff1d(np.arange(48), heads)
    vcols = (heads[:, None] * 128 + np.arange(128)).reshape(-1)
    ocols = (others[:, None] * 128 + np.arange(128)).reshape(-1)
    chans = np.concatenate([np.arange(4096), 4096 + vcols])  # q, k and the range's v channels
    other_chans = 4096 + ocols
    worst = 0.0
    for s in range(nseq):
        ox = {k: np.ascontiguousarray(v[s]) for k, v in x.items()}
        oatt = np.zeros((count, 6144), F)
        conv, delta = states[s]["conv_state"].copy(), states[s]["delta_state"].copy()
        assert oracle_lib.linear_prefill(w, conv, delta, ox["qkv"], ox["z"], ox["beta"],
                                         ox["alpha"], oatt) == 0
        assert np.isfinite(att[s][:, vcols]).all()
        _, e = check_parity(att[s][:, vcols], oatt[:, vcols], TOL, f"output seq {s}")
        worst = max(worst, e)
        assert np.isnan(att[s][:, ocols]).all()
        assert relative_error(out["qkv"][s][:, chans], ox["qkv"][:, chans]) < 1e-5
        np.testing.assert_array_equal(out["qkv"][s][:, other_chans], x0["qkv"][s][:, other_chans])
        # The gates go through expf/logf: CUDA's and the host libm's differ by an ulp.
        assert relative_error(out["beta"][s][:, heads], ox["beta"][:, heads]) < 1e-5
        assert relative_error(out["alpha"][s][:, heads], ox["alpha"][:, heads]) < 1e-5
        np.testing.assert_array_equal(out["beta"][s][:, others], x0["beta"][s][:, others])
        np.testing.assert_array_equal(out["alpha"][s][:, others], x0["alpha"][s][:, others])
        gconv, gdelta = st.download_linear(layer, seq0 + s)
        np.testing.assert_array_equal(gconv[chans], conv[chans])
        np.testing.assert_array_equal(gconv[other_chans], states[s]["conv_state"][other_chans])
        check_parity(gdelta[heads], delta[heads], TOL, f"state seq {s}")
        np.testing.assert_array_equal(gdelta[others], states[s]["delta_state"][others])
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


@pytest.mark.parametrize("v_range", [(0, 6), (42, 6), (5, 24), (17, 1)])
def test_linear_prefill_value_head_range(cuda_ctx, oracle_lib, v_range):
    """One call per value-head range (the unit DeltaNet prefill shards across
    GPUs: 6 heads per GPU at 8 GPUs); (5, 24) covers key heads with one and
    with two of their value heads in the range."""
    _case(cuda_ctx, oracle_lib, nseq=2, count=300, layer=0, seed=20 + v_range[0], fresh=False,
          v_range=v_range)


def test_linear_prefill_head_ranges_compose(cuda_ctx):
    """Calls over disjoint value-head ranges, each on its own copy of the state
    (as 8 GPUs run them: every rank convolves the shared q/k channels itself),
    give exactly the result of one call over all heads: outputs, v channels,
    gates and the range's delta-state heads, bitwise."""
    import torch

    from q38attn import synth
    g = synth.rng(31)
    w = synth.linear_weights(g)
    layer, count = 1, 400
    cuda_ctx.bind_linear_layer(layer, w["conv1d"], w["dt_bias"], w["ssm_a"], w["ssm_norm"])
    stt = [synth.linear_state(g) for _ in range(2)]
    x = {k: v.reshape(2, count, -1) for k, v in synth.linear_step(g, 2 * count).items()}

    def run(h0, n):
        st = cuda_ctx.state(2, 16, full_slots=0, linear_slots=2)
        st.reserve_prefill(2 * count)
        for s in range(2):
            st.upload_linear(layer, s, stt[s]["conv_state"], stt[s]["delta_state"])
        d = {k: torch.from_numpy(v.copy()).cuda() for k, v in x.items()}
        att = torch.zeros(2, count, 6144, device="cuda")
        cuda_ctx.linear_prefill_heads(st, layer, 0, d["qkv"], d["z"], d["beta"], d["alpha"], att,
                                      h0, n)
        torch.cuda.synchronize()
        assert st.errors() == 0
        out = ({k: v.cpu().numpy() for k, v in d.items()}, att.cpu().numpy(),
               [st.download_linear(layer, s) for s in range(2)])
        st.close()
        return out

    full_d, full_att, full_states = run(0, 48)
    for r in range(8):
        h0 = 6 * r
        d, att, states = run(h0, 6)
        cols = slice(128 * h0, 128 * (h0 + 6))
        np.testing.assert_array_equal(att[:, :, cols], full_att[:, :, cols])
        np.testing.assert_array_equal(d["qkv"][:, :, :4096], full_d["qkv"][:, :, :4096])
        np.testing.assert_array_equal(d["qkv"][:, :, 4096:][:, :, cols],
                                      full_d["qkv"][:, :, 4096:][:, :, cols])
        np.testing.assert_array_equal(d["beta"][:, :, h0:h0 + 6], full_d["beta"][:, :, h0:h0 + 6])
        np.testing.assert_array_equal(d["alpha"][:, :, h0:h0 + 6],
                                      full_d["alpha"][:, :, h0:h0 + 6])
        for s in range(2):
            np.testing.assert_array_equal(states[s][1][h0:h0 + 6], full_states[s][1][h0:h0 + 6])
            np.testing.assert_array_equal(states[s][0][:4096], full_states[s][0][:4096])


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
        check_parity(out[0].cpu().numpy(), oo, TOL, str(step))
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
    for h0, n in ((48, 1), (-1, 2), (40, 9), (0, 0)):  # value-head ranges outside 0..48
        with pytest.raises(q38attn.Q38Error) as e:
            cuda_ctx.linear_prefill_heads(st, 0, 0, qkv, z, b, b.clone(), z.clone(), h0, n)
        assert e.value.code == q38attn.Q38_ERR_ARG
    st.close()

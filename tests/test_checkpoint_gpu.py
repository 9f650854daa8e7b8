"""GPU tests of the recurrent-state checkpoint / restore used for speculative
decoding rollback (checkpoint_state / restore_target_state,
src/model/ops.rs:1627-1647): the conv and delta state of every DeltaNet slot
is copied aside and copied back, per sequence range.

A restored state must be bitwise the checkpointed one, and re-running the
same inputs from it must reproduce the first run exactly (same kernels, same
data), which is what the reference's rollback-then-re-run relies on."""
from __future__ import annotations

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

F = np.float32


def _bind_two_linear_layers(cuda_ctx, g):
    from q38attn import synth
    ws = []
    for layer in (0, 1):
        w = synth.linear_weights(g)
        cuda_ctx.bind_linear_layer(layer, w["conv1d"], w["dt_bias"], w["ssm_a"], w["ssm_norm"])
        ws.append(w)
    return ws


def test_checkpoint_restore_decode_is_bitwise(cuda_ctx):
    import torch

    from q38attn import synth
    g = synth.rng(70)
    _bind_two_linear_layers(cuda_ctx, g)
    B = 3
    st = cuda_ctx.state(B, 16, full_slots=0, linear_slots=2)
    for layer in (0, 1):
        for b in range(B):
            init = synth.linear_state(g)
            st.upload_linear(layer, b, init["conv_state"], init["delta_state"])
    before = {(l, b): st.download_linear(l, b) for l in (0, 1) for b in range(B)}
    st.checkpoint()  # all sequences
    steps = [synth.linear_step(g, B) for _ in range(2)]

    def run(step):
        outs = []
        for layer in (0, 1):
            d = {k: torch.from_numpy(v.copy()).cuda() for k, v in step.items()}
            out = torch.empty(B, 6144, device="cuda")
            cuda_ctx.linear_decode(st, layer, d["qkv"], d["z"], d["beta"], d["alpha"], out)
            outs.append(out.cpu().numpy())
        torch.cuda.synchronize()
        return outs

    first = [run(x) for x in steps]
    advanced = {(l, b): st.download_linear(l, b) for l in (0, 1) for b in range(B)}
    # Roll back sequences 1 and 2 only.
    st.restore(1, 2)
    torch.cuda.synchronize()
    for l in (0, 1):
        for b in range(B):
            conv, delta = st.download_linear(l, b)
            ref = advanced[(l, b)] if b == 0 else before[(l, b)]
            np.testing.assert_array_equal(conv, ref[0])
            np.testing.assert_array_equal(delta, ref[1])
    # Re-running the same first step from the restored state reproduces it.
    again = run(steps[0])
    for l in (0, 1):
        np.testing.assert_array_equal(again[l][1:], first[0][l][1:])
    assert st.errors() == 0
    st.close()


def test_checkpoint_restore_around_a_verify_prefill(cuda_ctx):
    """Speculative verify: checkpoint, prefill 100 draft tokens, restore, then
    prefill only the 60 accepted ones; the state equals prefilling those 60
    from the checkpoint directly."""
    import torch

    from q38attn import synth
    g = synth.rng(71)
    w = synth.linear_weights(g)
    cuda_ctx.bind_linear_layer(0, w["conv1d"], w["dt_bias"], w["ssm_a"], w["ssm_norm"])
    sts = []
    init = synth.linear_state(g)
    for _ in range(2):
        st = cuda_ctx.state(1, 16, full_slots=0, linear_slots=1)
        st.reserve_prefill(128)
        st.upload_linear(0, 0, init["conv_state"], init["delta_state"])
        sts.append(st)
    x = {k: v.reshape(1, 100, -1) for k, v in synth.linear_step(g, 100).items()}

    def prefill(st, n):
        d = {k: torch.from_numpy(np.ascontiguousarray(v[:, :n])).cuda() for k, v in x.items()}
        out = torch.empty(1, n, 6144, device="cuda")
        cuda_ctx.linear_prefill(st, 0, 0, d["qkv"], d["z"], d["beta"], d["alpha"], out)
        torch.cuda.synchronize()
        return out.cpu().numpy()

    a, b = sts
    a.checkpoint()
    prefill(a, 100)          # the verify pass over all draft tokens
    a.restore()              # roll back
    out_a = prefill(a, 60)   # re-run the committed prefix
    out_b = prefill(b, 60)   # the same prefix on an untouched copy
    np.testing.assert_array_equal(out_a, out_b)
    for s_a, s_b in zip(a.download_linear(0, 0), b.download_linear(0, 0)):
        np.testing.assert_array_equal(s_a, s_b)
    for st in sts:
        assert st.errors() == 0
        st.close()


def test_restore_without_checkpoint_is_an_argument_error(cuda_ctx):
    import q38attn
    from q38attn import synth
    _bind_two_linear_layers(cuda_ctx, synth.rng(72))
    st = cuda_ctx.state(2, 16, full_slots=0, linear_slots=2)
    with pytest.raises(q38attn.Q38Error) as e:
        st.restore()
    assert e.value.code == q38attn.Q38_ERR_ARG
    st.checkpoint(0, 1)
    st.restore(0, 1)
    with pytest.raises(q38attn.Q38Error):  # sequence 1 was never checkpointed
        st.restore(1, 1)
    with pytest.raises(q38attn.Q38Error):  # range outside the batch
        st.checkpoint(1, 2)
    st.close()

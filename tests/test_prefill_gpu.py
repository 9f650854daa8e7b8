"""GPU parity tests of the tcgen05 causal prefill attention against the CPU
oracle's per-token full_core loop (batch_full_attention, src/model/ops.rs:1156-1172).

The prefill computes S = Q K^T from bf16 Q and K and O = P V in f16, with f32
accumulation; the oracle consumes the same bf16-rounded query and K/V values as
f32 (kv_round_bf16 = 3).
Tolerance: |a-b|/max(|b|,1) < 2e-3 (the reference's metric,
src/kernel/x86/tensor.rs:411-413)."""
from __future__ import annotations

import numpy as np
import pytest

from conftest import relative_error

pytestmark = pytest.mark.gpu

TOL = 2e-3
F = np.float32


def _run_case(cuda_ctx, oracle_lib, *, nseq, count, base, ctx_len, layer, seed, rows=None,
              batch=None):
    import torch

    import q38attn
    from q38attn import synth
    g = synth.rng(seed)
    w = synth.full_weights(g)
    cuda_ctx.bind_full_layer(layer, w["q_norm"], w["k_norm"])
    batch = batch or nseq
    slots = layer // 4 + 1
    st = cuda_ctx.state(batch, ctx_len, full_slots=slots, linear_slots=0,
                        kv_dtype=q38attn.Q38_KV_BF16)
    st.reserve_prefill(nseq * count)
    seq0 = batch - nseq
    prior = []
    for s in range(nseq):
        k, v = synth.kv_rows(g, max(base, 1), bf16=True)
        if base:
            st.upload_kv(layer, seq0 + s, 0, np.ascontiguousarray(k[:base]),
                         np.ascontiguousarray(v[:base]))
        prior.append((k[:base], v[:base]))
    x = {kk: vv.reshape(nseq, count, -1) for kk, vv in synth.full_step(g, nseq * count).items()}
    d = {kk: torch.from_numpy(vv.copy()).cuda() for kk, vv in x.items()}
    att = torch.full((nseq, count, 6144), float("nan"), device="cuda")
    cuda_ctx.full_prefill(st, layer, seq0, d["q_and_gate"], d["key"], d["value"], att, base)
    torch.cuda.synchronize()
    assert st.errors() == 0
    att = att.cpu().numpy()
    keys = d["key"].cpu().numpy()
    worst = 0.0
    for s in range(nseq):
        kc = np.zeros((slots * ctx_len, 1024), F)
        vc = np.zeros((slots * ctx_len, 1024), F)
        r0 = (layer // 4) * ctx_len
        kc[r0:r0 + base], vc[r0:r0 + base] = prior[s]
        oatt = np.zeros((count, 6144), F)
        okey = x["key"][s].copy()
        assert oracle_lib.full_prefill(w, np.ascontiguousarray(x["q_and_gate"][s]), okey,
                                       np.ascontiguousarray(x["value"][s]), oatt, kc, vc,
                                       ctx_len, base, layer, 3, rows_wanted=rows) == 0
        sel = slice(None) if rows is None else np.asarray(rows)
        assert np.isfinite(att[s][sel]).all()
        err = relative_error(att[s][sel], oatt[sel])
        worst = max(worst, err)
        assert err < TOL, (s, err)
        assert relative_error(keys[s], okey) < 1e-5
        # The appended cache rows equal the oracle's bf16-rounded rows: V
        # exactly; K (RMSNorm + RoPE in f32, then rounded) up to an occasional
        # one-ulp bf16 rounding flip where GPU and host cosf/sinf differ by an ulp.
        gk, gv = st.download_kv(layer, seq0 + s, base, count)
        ok_k = kc[r0 + base:r0 + base + count]
        assert np.mean(gk != ok_k) < 1e-4
        assert relative_error(gk, ok_k) < 1e-2
        np.testing.assert_array_equal(gv, vc[r0 + base:r0 + base + count])
    st.close()
    return worst


def test_prefill_partial_tile(cuda_ctx, oracle_lib):
    """200 tokens: one full 128-row tile and one partial tile, from position 0."""
    _run_case(cuda_ctx, oracle_lib, nseq=1, count=200, base=0, ctx_len=256, layer=3, seed=1)


def test_prefill_after_cached_prefix_two_sequences(cuda_ctx, oracle_lib):
    """Two sequences of a three-sequence state, 150 new tokens after 100 cached
    positions (key tiles straddle the prefix/prompt boundary)."""
    _run_case(cuda_ctx, oracle_lib, nseq=2, count=150, base=100, ctx_len=512, layer=7, seed=2,
              batch=3)


def test_prefill_single_token(cuda_ctx, oracle_lib):
    """count=1 reduces to one decode step at base_position."""
    _run_case(cuda_ctx, oracle_lib, nseq=1, count=1, base=77, ctx_len=128, layer=3, seed=3)


def test_prefill_1024_tokens(cuda_ctx, oracle_lib):
    _run_case(cuda_ctx, oracle_lib, nseq=2, count=1024, base=0, ctx_len=1024, layer=3, seed=4,
              rows=list(range(0, 1024, 37)) + [1022, 1023])


def test_prefill_config4_size_sampled_rows(cuda_ctx, oracle_lib):
    """Config 4 shape for one sequence: 8192 tokens; every 512th row plus the
    last 4 rows are checked against the oracle."""
    rows = list(range(0, 8192, 512)) + [8188, 8189, 8190, 8191]
    _run_case(cuda_ctx, oracle_lib, nseq=1, count=8192, base=0, ctx_len=8192, layer=3, seed=5,
              rows=rows)


def test_prefill_then_decode_continues(cuda_ctx, oracle_lib):
    """Prefill 300 tokens, then decode two tokens; the decode sees the
    prefilled cache exactly as the oracle's per-token loop leaves it."""
    import torch

    import q38attn
    from q38attn import synth
    g = synth.rng(6)
    w = synth.full_weights(g)
    layer, ctx_len, count = 3, 512, 300
    cuda_ctx.bind_full_layer(layer, w["q_norm"], w["k_norm"])
    st = cuda_ctx.state(1, ctx_len, full_slots=1, linear_slots=0, kv_dtype=q38attn.Q38_KV_BF16)
    st.reserve_prefill(count)
    x = {kk: vv.reshape(1, count, -1) for kk, vv in synth.full_step(g, count).items()}
    d = {kk: torch.from_numpy(vv.copy()).cuda() for kk, vv in x.items()}
    att = torch.empty(1, count, 6144, device="cuda")
    cuda_ctx.full_prefill(st, layer, 0, d["q_and_gate"], d["key"], d["value"], att, 0)
    kc = np.zeros((ctx_len, 1024), F)
    vc = np.zeros((ctx_len, 1024), F)
    oatt = np.zeros((count, 6144), F)
    okey = x["key"][0].copy()
    oracle_lib.full_prefill(w, np.ascontiguousarray(x["q_and_gate"][0]), okey,
                            np.ascontiguousarray(x["value"][0]), oatt, kc, vc, ctx_len, 0, layer,
                            3, rows_wanted=[count - 1])
    for step in range(2):
        y = synth.full_step(g, 1)
        dy = {kk: torch.from_numpy(vv.copy()).cuda() for kk, vv in y.items()}
        out = torch.empty(1, 6144, device="cuda")
        pos = count + step
        cuda_ctx.full_decode(st, layer, dy["q_and_gate"], dy["key"], dy["value"],
                             torch.tensor([pos], dtype=torch.int32, device="cuda"), out)
        torch.cuda.synchronize()
        q = np.zeros(6144, F)
        gate = np.zeros(6144, F)
        scores = np.zeros(24 * ctx_len, F)
        oout = np.zeros(6144, F)
        okey1 = y["key"][0].copy()
        assert oracle_lib.full_core(w, y["q_and_gate"][0], okey1, y["value"][0], q, gate, scores,
                                    oout, kc, vc, ctx_len, pos, layer, 1) == 0
        assert relative_error(out[0].cpu().numpy(), oout) < 1e-4, step
    assert st.errors() == 0
    st.close()


def test_prefill_argument_errors(cuda_ctx):
    import torch

    import q38attn
    w = {"q_norm": np.ones(256, F), "k_norm": np.ones(256, F)}
    cuda_ctx.bind_full_layer(3, w["q_norm"], w["k_norm"])
    z = torch.zeros(1, 4, 12288, device="cuda")
    k = torch.zeros(1, 4, 1024, device="cuda")
    a = torch.zeros(1, 4, 6144, device="cuda")
    st32 = cuda_ctx.state(1, 64, full_slots=1, linear_slots=0, kv_dtype=q38attn.Q38_KV_F32)
    st32.reserve_prefill(4)
    with pytest.raises(q38attn.Q38Error) as e:  # needs a bf16 cache
        cuda_ctx.full_prefill(st32, 3, 0, z, k, k.clone(), a, 0)
    assert e.value.code == q38attn.Q38_ERR_ARG
    st = cuda_ctx.state(1, 64, full_slots=1, linear_slots=0, kv_dtype=q38attn.Q38_KV_BF16)
    with pytest.raises(q38attn.Q38Error):  # no scratch reserved
        cuda_ctx.full_prefill(st, 3, 0, z, k, k.clone(), a, 0)
    st.reserve_prefill(4)
    with pytest.raises(q38attn.Q38Error):  # positions past the cache
        cuda_ctx.full_prefill(st, 3, 0, z, k, k.clone(), a, 61)
    with pytest.raises(q38attn.Q38Error):  # not a full-attention layer
        cuda_ctx.full_prefill(st, 2, 0, z, k, k.clone(), a, 0)
    st.close()
    st32.close()

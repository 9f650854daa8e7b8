"""GPU parity tests of the tcgen05 causal prefill attention against the CPU
oracle's per-token full_core loop (batch_full_attention, src/model/ops.rs:1156-1172).

The prefill computes S = Q K^T from bf16 Q and K and O = P V in f16, with f32
accumulation. With a bf16 cache the oracle consumes the same bf16-rounded
query and K/V values as f32 (kv_round_bf16 = 3); with an f32 cache (the
reference's Vec<f32>) the oracle is the plain f32 reference (kv_round_bf16 =
0) and the cache rows must equal the reference's f32 rows.
Tolerance 2e-3 on both the reference's metric |a-b|/max(|b|,1)
(src/kernel/x86/tensor.rs:411-413) and the scale-aware max|a-b|/max|b|."""
from __future__ import annotations

import numpy as np
import pytest

from conftest import check_parity, relative_error

pytestmark = pytest.mark.gpu

TOL = 2e-3
F = np.float32


def _run_case(cuda_ctx, oracle_lib, *, nseq, count, base, ctx_len, layer, seed, rows=None,
              batch=None, kv_f32=False, kv_range=None):
    """kv_range=(h0, n): prefill only KV heads h0..h0+n-1 (q38_full_prefill_heads);
    the other heads' outputs and cache rows must stay untouched."""
    import torch

    import q38attn
    from q38attn import synth
    g = synth.rng(seed)
    w = synth.full_weights(g)
    cuda_ctx.bind_full_layer(layer, w["q_norm"], w["k_norm"])
    batch = batch or nseq
    slots = layer // 4 + 1
    st = cuda_ctx.state(batch, ctx_len, full_slots=slots, linear_slots=0,
                        kv_dtype=q38attn.Q38_KV_F32 if kv_f32 else q38attn.Q38_KV_BF16)
    st.reserve_prefill(nseq * count)
    seq0 = batch - nseq
    prior = []
    for s in range(nseq):
        k, v = synth.kv_rows(g, max(base, 1), bf16=not kv_f32)
        if base:
            st.upload_kv(layer, seq0 + s, 0, np.ascontiguousarray(k[:base]),
                         np.ascontiguousarray(v[:base]))
        prior.append((k[:base], v[:base]))
    x = {kk: vv.reshape(nseq, count, -1) for kk, vv in synth.full_step(g, nseq * count).items()}
    d = {kk: torch.from_numpy(vv.copy()).cuda() for kk, vv in x.items()}
    att = torch.full((nseq, count, 6144), float("nan"), device="cuda")
    if kv_range is None:
        cuda_ctx.full_prefill(st, layer, seq0, d["q_and_gate"], d["key"], d["value"], att, base)
        heads = range(4)
    else:
        cuda_ctx.full_prefill_heads(st, layer, seq0, d["q_and_gate"], d["key"], d["value"], att,
                                    base, kv_range[0], kv_range[1])
        heads = range(kv_range[0], kv_range[0] + kv_range[1])
    torch.cuda.synchronize()
    assert st.errors() == 0
    att = att.cpu().numpy()
    keys = d["key"].cpu().numpy()
    qcols = np.concatenate([np.arange(256 * q, 256 * q + 256) for h in heads
                            for q in range(6 * h, 6 * h + 6)])
    kcols = np.concatenate([np.arange(256 * h, 256 * h + 256) for h in heads])
    other_q = np.setdiff1d(np.arange(6144), qcols)
    other_k = np.setdiff1d(np.arange(1024), kcols)
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
                                       ctx_len, base, layer, 0 if kv_f32 else 3,
                                       rows_wanted=rows) == 0
        sel = np.arange(count) if rows is None else np.asarray(rows)
        got, want = att[s][sel][:, qcols], oatt[sel][:, qcols]
        assert np.isfinite(got).all()
        _, e = check_parity(got, want, TOL, f"seq {s}")
        worst = max(worst, e)
        assert np.isnan(att[s][:, other_q]).all()  # other heads' outputs untouched
        assert relative_error(keys[s][:, kcols], okey[:, kcols]) < 1e-5
        np.testing.assert_array_equal(keys[s][:, other_k], x["key"][s][:, other_k])
        gk, gv = st.download_kv(layer, seq0 + s, base, count)
        ok_k = kc[r0 + base:r0 + base + count]
        if kv_f32:
            # The reference's f32 rows, as the per-token loop stores them.
            assert relative_error(gk[:, kcols], ok_k[:, kcols]) < 1e-5
            np.testing.assert_array_equal(gv[:, kcols], vc[r0 + base:r0 + base + count][:, kcols])
        else:
            # The appended cache rows equal the oracle's bf16-rounded rows: V
            # exactly; K (RMSNorm + RoPE in f32, then rounded) up to an
            # occasional one-ulp bf16 rounding flip where GPU and host
            # cosf/sinf differ by an ulp.
            assert np.mean(gk[:, kcols] != ok_k[:, kcols]) < 1e-4
            assert relative_error(gk[:, kcols], ok_k[:, kcols]) < 1e-2
            np.testing.assert_array_equal(gv[:, kcols],
                                          vc[r0 + base:r0 + base + count][:, kcols])
        if kv_range is not None:
            assert not gk[:, other_k].any() and not gv[:, other_k].any()
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


def test_prefill_config4_all_sequences(cuda_ctx, oracle_lib):
    """Config 4 in full: 4 sequences x 8192 tokens. In every sequence the first
    64 rows (few keys: the most sensitive to P's rounding), every 128th row and
    the last 4 rows (132 rows) are checked against the oracle."""
    rows = sorted(set(range(64)) | set(range(0, 8192, 128)) | {8188, 8189, 8190, 8191})
    _run_case(cuda_ctx, oracle_lib, nseq=4, count=8192, base=0, ctx_len=8192, layer=3, seed=5,
              rows=rows)


@pytest.mark.parametrize("kv_range", [(0, 1), (3, 1), (1, 2), (0, 3)])
def test_prefill_kv_head_range(cuda_ctx, oracle_lib, kv_range):
    """One call per KV-head group range (the unit prefill shards across GPUs):
    the range's heads match the oracle, the others are left untouched."""
    _run_case(cuda_ctx, oracle_lib, nseq=2, count=300, base=40, ctx_len=512, layer=3, seed=8,
              batch=3, kv_range=kv_range)


def test_prefill_kv_head_ranges_compose(cuda_ctx):
    """Calls over disjoint KV-head ranges leave exactly the result of one call
    over all heads (outputs, keys and cache rows bitwise)."""
    import torch

    import q38attn
    from q38attn import synth
    g = synth.rng(12)
    w = synth.full_weights(g)
    layer, count, base = 3, 700, 0
    cuda_ctx.bind_full_layer(layer, w["q_norm"], w["k_norm"])
    x = {kk: vv.reshape(2, count, -1) for kk, vv in synth.full_step(g, 2 * count).items()}
    outs = []
    for split in ([(0, 4)], [(0, 1), (1, 2), (3, 1)]):
        st = cuda_ctx.state(2, 1024, full_slots=1, linear_slots=0, kv_dtype=q38attn.Q38_KV_BF16)
        st.reserve_prefill(2 * count)
        d = {kk: torch.from_numpy(vv.copy()).cuda() for kk, vv in x.items()}
        att = torch.zeros(2, count, 6144, device="cuda")
        for h0, n in split:
            cuda_ctx.full_prefill_heads(st, layer, 0, d["q_and_gate"], d["key"], d["value"], att,
                                        base, h0, n)
        torch.cuda.synchronize()
        kv = [st.download_kv(layer, s, 0, count) for s in range(2)]
        outs.append((att.cpu().numpy(), d["key"].cpu().numpy(), kv))
        assert st.errors() == 0
        st.close()
    np.testing.assert_array_equal(outs[0][0], outs[1][0])
    np.testing.assert_array_equal(outs[0][1], outs[1][1])
    for s in range(2):
        np.testing.assert_array_equal(outs[0][2][s][0], outs[1][2][s][0])
        np.testing.assert_array_equal(outs[0][2][s][1], outs[1][2][s][1])


def test_prefill_f32_cache(cuda_ctx, oracle_lib):
    """A Q38_KV_F32 state (the reference's cache precision): 2 sequences, 600
    tokens after a 200-position f32 prefix, against the plain f32 oracle; the
    appended cache rows are the reference's f32 rows."""
    _run_case(cuda_ctx, oracle_lib, nseq=2, count=600, base=200, ctx_len=1024, layer=3, seed=9,
              kv_f32=True)


LONG_PREFIX_ROWS = list(range(0, 512, 37)) + [63, 64, 511]


def test_prefill_long_prefix(cuda_ctx, oracle_lib):
    """A continuation after a 4096-position bf16 prefix (the prefix copied to
    f16 V operands in whole 64-row tiles, every query tile's prefix part
    unmasked): 2 sequences x 512 tokens, sampled rows against the oracle."""
    _run_case(cuda_ctx, oracle_lib, nseq=2, count=512, base=4096, ctx_len=4608, layer=3, seed=11,
              rows=LONG_PREFIX_ROWS)


def test_prefill_f32_cache_long_prefix(cuda_ctx, oracle_lib):
    """The same over the reference's f32 cache (K and V of the prefix copied
    to f16 operands): 1 sequence x 512 tokens after 4096 f32 positions."""
    _run_case(cuda_ctx, oracle_lib, nseq=1, count=512, base=4096, ctx_len=4608, layer=3, seed=12,
              kv_f32=True, rows=LONG_PREFIX_ROWS)


def test_prefill_f32_cache_head_range(cuda_ctx, oracle_lib):
    _run_case(cuda_ctx, oracle_lib, nseq=1, count=260, base=0, ctx_len=512, layer=3, seed=10,
              kv_f32=True, kv_range=(2, 2))


def test_prefill_f32_cache_then_decode_reads_f32_rows(cuda_ctx, oracle_lib):
    """After an f32-cache prefill the decode step reads the reference's f32
    rows: its output matches the f32 oracle to the fp32 decode tolerance."""
    import torch

    import q38attn
    from q38attn import synth
    g = synth.rng(13)
    w = synth.full_weights(g)
    layer, ctx_len, count = 3, 512, 300
    cuda_ctx.bind_full_layer(layer, w["q_norm"], w["k_norm"])
    st = cuda_ctx.state(1, ctx_len, full_slots=1, linear_slots=0, kv_dtype=q38attn.Q38_KV_F32)
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
                            0, rows_wanted=[count - 1])
    y = synth.full_step(g, 1)
    dy = {kk: torch.from_numpy(vv.copy()).cuda() for kk, vv in y.items()}
    out = torch.empty(1, 6144, device="cuda")
    cuda_ctx.full_decode(st, layer, dy["q_and_gate"], dy["key"], dy["value"],
                         torch.tensor([count], dtype=torch.int32, device="cuda"), out)
    torch.cuda.synchronize()
    q = np.zeros(6144, F)
    gate = np.zeros(6144, F)
    scores = np.zeros(24 * ctx_len, F)
    oout = np.zeros(6144, F)
    okey1 = y["key"][0].copy()
    assert oracle_lib.full_core(w, y["q_and_gate"][0], okey1, y["value"][0], q, gate, scores,
                                oout, kc, vc, ctx_len, count, layer, 0) == 0
    check_parity(out[0].cpu().numpy(), oout, 1e-4, "decode after f32 prefill")
    assert st.errors() == 0
    st.close()


def test_prefill_v_beyond_f16_range_is_flagged(cuda_ctx):
    """A V value beyond 65504 cannot be held by the f16 P V operand: the call
    records Q38_DEVERR_RANGE (for both cache types) instead of passing silently."""
    import torch

    import q38attn
    from q38attn import synth
    g = synth.rng(14)
    w = synth.full_weights(g)
    cuda_ctx.bind_full_layer(3, w["q_norm"], w["k_norm"])
    for kvd in (q38attn.Q38_KV_BF16, q38attn.Q38_KV_F32):
        st = cuda_ctx.state(1, 128, full_slots=1, linear_slots=0, kv_dtype=kvd)
        st.reserve_prefill(64)
        x = {kk: vv.reshape(1, 64, -1) for kk, vv in synth.full_step(g, 64).items()}
        d = {kk: torch.from_numpy(vv.copy()).cuda() for kk, vv in x.items()}
        d["value"][0, 10, 5] = 1.0e5
        att = torch.empty(1, 64, 6144, device="cuda")
        cuda_ctx.full_prefill(st, 3, 0, d["q_and_gate"], d["key"], d["value"], att, 0)
        torch.cuda.synchronize()
        assert st.errors() & q38attn.Q38_DEVERR_RANGE
        # In range again: no flag.
        d["value"][0, 10, 5] = 1.0
        cuda_ctx.full_prefill(st, 3, 0, d["q_and_gate"], d["key"], d["value"], att, 0)
        assert st.errors() == 0
        st.close()


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
    for h0, n in ((4, 1), (-1, 2), (2, 3), (0, 0)):  # KV-head ranges outside 0..4
        with pytest.raises(q38attn.Q38Error) as e:
            cuda_ctx.full_prefill_heads(st32, 3, 0, z, k, k.clone(), a, 0, h0, n)
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

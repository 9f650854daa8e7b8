"""GPU tests of the projections on either side of the cores, through the C
ABI, against the CPU oracle:

* q38_quantize_q8_k is bit-identical to quantize_q8_k (src/kernel/quant.rs:
  56-124), block layout included;
* q38_project over K-quant and IQ4_NL / IQ4_XS weights is bit-identical to
  the reference's integer path (project -> tensor_gemv_q8_k /
  tensor_gemm_q8_k, ops.rs:623-640, 1016-1031; dot_iq4_*_q8_k,
  src/kernel/iq.rs:355-405), at the model's shapes (5120 -> 10240,
  6144 -> 5120, 48-row gates), over a batch that spans several 8-token
  launches, through both GEMV forms and the tensor-core kernel;
* weights uploaded from a GGUF file equal the same bytes uploaded as arrays;
* F32 / F16 / BF16 / Q8_0 weights agree with the reference's f32 dot within
  its tolerance |a-b|/max(|b|,1) < 1e-4 (src/kernel/x86/tensor.rs:411-413);
* the layer-level calls (linear_attention, ops.rs:744-803; full_attention,
  ops.rs:941-981) equal the oracle's chain project -> core -> quantize ->
  project. The core output is quantized to 8 bits before the output
  projection, so a core difference at the 1e-6 level can move a quant by one
  step near a rounding boundary; the bar there is 2e-3.
"""
from __future__ import annotations

import numpy as np
import pytest

from conftest import relative_error

pytestmark = pytest.mark.gpu

F = np.float32
HIDDEN = 5120


def _torch():
    import torch
    return torch


def _gpu_project(ctx, w, x):
    torch = _torch()
    dx = torch.from_numpy(np.ascontiguousarray(x, F)).cuda()
    out = torch.zeros(x.shape[0], w.rows, device="cuda")
    ctx.project(w, dx, out)
    torch.cuda.synchronize()
    return out.cpu().numpy()


def test_quantize_q8_k_bitwise(cuda_ctx, oracle_lib):
    torch = _torch()
    g = np.random.default_rng(7)
    x = (g.standard_normal((3, HIDDEN)) * 2).astype(F)
    x[0, 256:512] = 0.0                      # an all-zero block
    x[1, 5], x[1, 9] = -40.0, 40.0           # a magnitude tie: the first wins
    x[2, :256] = np.array([((i * 7919) % 101) / 50.0 - 1.0 for i in range(256)], F)
    blocks = torch.zeros(3 * HIDDEN // 256 * 292, dtype=torch.uint8, device="cuda")
    cuda_ctx.quantize_q8_k(torch.from_numpy(x).cuda(), blocks)
    torch.cuda.synchronize()
    got = blocks.cpu().numpy().view(oracle_lib.Q8K_BLOCK)
    want = oracle_lib.quantize_q8_k(x)
    np.testing.assert_array_equal(got.view(np.uint8), want.view(np.uint8))


K_CASES = [(12, 10240, HIDDEN), (13, 6144, HIDDEN), (14, 1000, HIDDEN), (12, 48, HIDDEN),
           (14, HIDDEN, 6144), (11, 300, HIDDEN), (10, 300, HIDDEN), (13, 37, 6144),
           # one and two 256-blocks per row: the pipelines' first / last stages coincide
           (12, 130, 256), (14, 200, 512), (13, 129, 768),
           # more than 32 blocks per row: one token takes the general (8-warp) form
           (12, 64, 9216), (14, 40, 8448),
           # IQ4_NL (a term per 32-value group) and IQ4_XS; odd block counts give
           # IQ4_XS rows 8-byte aligned only
           (20, 300, HIDDEN), (23, 300, HIDDEN), (23, 77, 2304), (23, 130, 256), (20, 64, 9216)]


@pytest.mark.parametrize("ggml_type,rows,width", K_CASES)
def test_project_k_quants_bitwise(cuda_ctx, oracle_lib, ggml_type, rows, width):
    from q38attn import synth
    g = synth.rng(100 + ggml_type + rows)
    data = synth.quant_weight(g, ggml_type, rows, width)
    w = cuda_ctx.weight(ggml_type, width, rows, data)
    # 9 or more tokens over Q4_K / Q5_K take the tensor-core path (one or
    # two 32-token tiles here); fewer, or other types, the integer GEMV.
    for batch in (1, 3, 11, 40):
        x = synth.normal(g, (batch, width))
        got = _gpu_project(cuda_ctx, w, x)
        want = oracle_lib.project(ggml_type, data, rows, width, x)
        np.testing.assert_array_equal(got.view(np.uint32), want.view(np.uint32), err_msg=f"batch {batch}")
    w.close()


PLANE_CASES = [(12, 10240, HIDDEN), (13, 6144, HIDDEN), (14, HIDDEN, 6144), (12, 300, HIDDEN),
               (14, 130, 256), (13, 129, 768), (12, 64, 9216), (14, 40, 8448)]


@pytest.mark.parametrize("ggml_type,rows,width", PLANE_CASES)
def test_project_planes_bitwise(cuda_ctx, oracle_lib, ggml_type, rows, width):
    """Projections of 9+ tokens from the weight's integer planes
    (q38_weight_build_planes) equal the reference's integer dot bit for bit:
    full and ragged 16-, 32- and 64-token tiles, ragged 128-row tiles, one to
    36 blocks."""
    from q38attn import synth
    g = synth.rng(300 + ggml_type + rows)
    data = synth.quant_weight(g, ggml_type, rows, width)
    w = cuda_ctx.weight(ggml_type, width, rows, data).build_planes()
    w.build_planes()  # a second call keeps the planes it has
    for batch in (9, 32, 40, 71, 300):  # 16-, 32- and (from 128 tokens) 64-token tiles
        x = synth.normal(g, (batch, width))
        x[0, :256] = 0.0  # an all-zero activation block (scale 0)
        got = _gpu_project(cuda_ctx, w, x)
        want = oracle_lib.project(ggml_type, data, rows, width, x)
        np.testing.assert_array_equal(got.view(np.uint32), want.view(np.uint32), err_msg=f"batch {batch}")
    w.close()


def test_planes_refuse_other_types(cuda_ctx):
    import q38attn
    from q38attn import synth
    g = synth.rng(5)
    w = cuda_ctx.weight(8, HIDDEN, 16, synth.quant_weight(g, 8, 16, HIDDEN))
    with pytest.raises(q38attn.Q38Error):
        w.build_planes()
    w.close()


@pytest.mark.parametrize("ggml_type", [0, 1, 30, 8])
def test_project_f32_input_types(cuda_ctx, oracle_lib, ggml_type):
    from q38attn import synth
    g = synth.rng(200 + ggml_type)
    rows, width = 300, HIDDEN
    data = synth.quant_weight(g, ggml_type, rows, width)
    w = cuda_ctx.weight(ggml_type, width, rows, data)
    for batch in (1, 9):
        x = synth.normal(g, (batch, width))
        got = _gpu_project(cuda_ctx, w, x)
        want = oracle_lib.project(ggml_type, data, rows, width, x)
        assert relative_error(got, want) < 1e-4
    w.close()


@pytest.mark.parametrize("ggml_type", [0, 1, 30, 8])
def test_project_f32_input_many_tokens(cuda_ctx, oracle_lib, ggml_type):
    """9+ tokens over up to 128 rows (the DeltaNet gates' shape) take the
    chunked form: 128-value chunks of 64 rows x 32 tokens, partial sums added
    in chunk order. Ragged row and token blocks, two of each."""
    from q38attn import synth
    g = synth.rng(210 + ggml_type)
    for rows, width in ((48, HIDDEN), (100, 1024)):
        data = synth.quant_weight(g, ggml_type, rows, width)
        w = cuda_ctx.weight(ggml_type, width, rows, data)
        for batch in (9, 32, 40):
            x = synth.normal(g, (batch, width))
            got = _gpu_project(cuda_ctx, w, x)
            want = oracle_lib.project(ggml_type, data, rows, width, x)
            assert relative_error(got, want) < 1e-4
        w.close()


def test_project_host_matches_device(cuda_ctx):
    from q38attn import synth
    g = synth.rng(301)
    data = synth.quant_weight(g, 12, 200, HIDDEN)
    w = cuda_ctx.weight(12, HIDDEN, 200, data)
    x = synth.normal(g, (4, HIDDEN))
    np.testing.assert_array_equal(cuda_ctx.project_host(w, x), _gpu_project(cuda_ctx, w, x))
    w.close()


def test_weight_from_gguf_equals_array_upload(cuda_ctx, tmp_path):
    from gguf_writer import GGML_IQ4_NL, GGML_IQ4_XS, GGML_Q4_K, GGML_Q6_K, write_gguf
    from q38attn import synth
    g = synth.rng(302)
    q4 = synth.quant_weight(g, 12, 64, HIDDEN)
    q6 = synth.quant_weight(g, 14, 32, 6144)
    nl = synth.quant_weight(g, 20, 48, HIDDEN)
    xs = synth.quant_weight(g, 23, 40, 6144)
    path = tmp_path / "proj.gguf"
    write_gguf(path, [("blk.0.attn_qkv.weight", [HIDDEN, 64], GGML_Q4_K, q4.tobytes()),
                      ("blk.0.ssm_out.weight", [6144, 32], GGML_Q6_K, q6.tobytes()),
                      ("blk.1.attn_gate.weight", [HIDDEN, 48], GGML_IQ4_NL, nl.tobytes()),
                      ("blk.1.ssm_out.weight", [6144, 40], GGML_IQ4_XS, xs.tobytes())])
    for name, ty, width, rows, data in (("blk.0.attn_qkv.weight", 12, HIDDEN, 64, q4),
                                        ("blk.0.ssm_out.weight", 14, 6144, 32, q6),
                                        ("blk.1.attn_gate.weight", 20, HIDDEN, 48, nl),
                                        ("blk.1.ssm_out.weight", 23, 6144, 40, xs)):
        a = cuda_ctx.weight_from_gguf(path, name)
        assert (a.ggml_type, a.width, a.rows) == (ty, width, rows)
        b = cuda_ctx.weight(ty, width, rows, data)
        x = synth.normal(g, (2, width))
        np.testing.assert_array_equal(_gpu_project(cuda_ctx, a, x), _gpu_project(cuda_ctx, b, x))
        a.close()
        b.close()


def test_projection_argument_errors(cuda_ctx):
    import q38attn
    from q38attn import synth
    g = synth.rng(303)
    with pytest.raises(q38attn.Q38Error) as e:  # Q4_0 is not a projection type here
        cuda_ctx.weight(2, 256, 4, np.zeros(4 * 144, np.uint8))
    assert e.value.code == q38attn.Q38_ERR_ARG
    with pytest.raises(q38attn.Q38Error):  # wrong byte count
        cuda_ctx.weight(12, 512, 4, np.zeros(100, np.uint8))
    cuda_ctx.weight(8, 96, 4, synth.quant_weight(g, 8, 4, 96)).close()  # Q8_0: 32-blocks suffice
    with pytest.raises(q38attn.Q38Error):  # K-quant rows must be whole 256-blocks
        cuda_ctx.weight(12, 300, 4, np.zeros(4 * 2 * 144, np.uint8))


def _layer_weights(ctx, g, spec):
    from q38attn import synth
    host, dev = {}, {}
    for name, (ty, width, rows) in spec.items():
        host[name] = (ty, width, rows, synth.quant_weight(g, ty, rows, width))
        dev[name] = ctx.weight(ty, width, rows, host[name][3])
    return host, dev


def _oracle_project(oracle_lib, spec, x):
    ty, width, rows, data = spec
    return oracle_lib.project(ty, data, rows, width, x)


@pytest.mark.parametrize("batch,planes", [(2, False), (12, False), (12, True)])
def test_linear_attention_decode_matches_oracle(cuda_ctx, oracle_lib, batch, planes):
    """linear_attention (ops.rs:744-803) for sequences of DeltaNet layer 0; 12
    sequences take the tensor-core projections (from the integer planes with
    `planes`)."""
    from q38attn import synth
    torch = _torch()
    g = synth.rng(400 + batch)
    layer = 0
    lw = synth.linear_weights(g)
    cuda_ctx.bind_linear_layer(layer, lw["conv1d"], lw["dt_bias"], lw["ssm_a"], lw["ssm_norm"])
    host, dev = _layer_weights(cuda_ctx, g, {
        "qkv": (12, HIDDEN, 10240), "z": (13, HIDDEN, 6144), "beta": (8, HIDDEN, 48),
        "alpha": (0, HIDDEN, 48), "out": (14, 6144, HIDDEN)})
    if planes:
        for name in ("qkv", "z", "out"):
            dev[name].build_planes()
    st = cuda_ctx.state(batch, 16, full_slots=0, linear_slots=1)
    states = [synth.linear_state(g) for _ in range(batch)]
    for b, s0 in enumerate(states):
        st.upload_linear(layer, b, s0["conv_state"], s0["delta_state"])
    norm = synth.normal(g, (batch, HIDDEN))
    branch = torch.zeros(batch, HIDDEN, device="cuda")
    cuda_ctx.linear_attention_decode(st, layer, dev, torch.from_numpy(norm).cuda(), branch)
    torch.cuda.synchronize()
    assert st.errors() == 0

    qkv = _oracle_project(oracle_lib, host["qkv"], norm)
    z = _oracle_project(oracle_lib, host["z"], norm)
    beta = _oracle_project(oracle_lib, host["beta"], norm)
    alpha = _oracle_project(oracle_lib, host["alpha"], norm)
    att = np.zeros((batch, 6144), F)
    for b in range(batch):
        cs, ds = states[b]["conv_state"].copy(), states[b]["delta_state"].copy()
        row = [np.ascontiguousarray(a[b]) for a in (qkv, z, beta, alpha)]
        out = np.zeros(6144, F)
        assert oracle_lib.linear_core(lw, cs, ds, row[0], row[1], row[2], row[3], out) == 0
        att[b] = out
        gcs, gds = st.download_linear(layer, b)
        # The conv state is advanced by the qkv projection's epilogue: exactly
        # the reference's shift.
        np.testing.assert_array_equal(gcs, cs)
        assert relative_error(gds, ds) < 1e-4
    want = _oracle_project(oracle_lib, host["out"], att)
    assert relative_error(branch.cpu().numpy(), want) < 2e-3
    for w in dev.values():
        w.close()
    st.close()


@pytest.mark.parametrize("batch,planes", [(2, False), (12, False), (12, True)])
def test_full_attention_decode_matches_oracle(cuda_ctx, oracle_lib, batch, planes):
    """full_attention (ops.rs:941-981) for sequences of full layer 3 at
    positions 5, 40, ... over an f32 cache; 12 sequences take the tensor-core
    projections."""
    from q38attn import synth
    torch = _torch()
    g = synth.rng(401 + batch)
    layer, ctx_len = 3, 64
    positions = [5, 40, 0, 1, 63, 17, 30, 2, 50, 9, 33, 60][:batch]
    fw = synth.full_weights(g)
    cuda_ctx.bind_full_layer(layer, fw["q_norm"], fw["k_norm"])
    host, dev = _layer_weights(cuda_ctx, g, {
        "q": (12, HIDDEN, 12288), "k": (14, HIDDEN, 1024), "v": (8, HIDDEN, 1024),
        "out": (12, 6144, HIDDEN)})
    if planes:
        for name in ("q", "k", "out"):
            dev[name].build_planes()
    st = cuda_ctx.state(batch, ctx_len, full_slots=1, linear_slots=0)
    caches = []
    for b, pos in enumerate(positions):
        kc = np.zeros((ctx_len, 1024), F)
        vc = np.zeros((ctx_len, 1024), F)
        if pos:
            k, v = synth.kv_rows(g, pos)
            st.upload_kv(layer, b, 0, k, v)
            kc[:pos], vc[:pos] = k, v
        caches.append((kc, vc))
    norm = synth.normal(g, (batch, HIDDEN))
    branch = torch.zeros(batch, HIDDEN, device="cuda")
    cuda_ctx.full_attention_decode(st, layer, dev, torch.from_numpy(norm).cuda(),
                                   torch.tensor(positions, dtype=torch.int32, device="cuda"), branch)
    torch.cuda.synchronize()
    assert st.errors() == 0

    qg = _oracle_project(oracle_lib, host["q"], norm)
    key = _oracle_project(oracle_lib, host["k"], norm)
    value = _oracle_project(oracle_lib, host["v"], norm)
    att = np.zeros((batch, 6144), F)
    for b, pos in enumerate(positions):
        q, gate, scores = np.zeros(6144, F), np.zeros(6144, F), np.zeros(24 * ctx_len, F)
        kb = np.ascontiguousarray(key[b])
        out = np.zeros(6144, F)
        kc, vc = caches[b]
        assert oracle_lib.full_core(fw, np.ascontiguousarray(qg[b]), kb, np.ascontiguousarray(value[b]),
                                    q, gate, scores, out, kc, vc, ctx_len, pos, layer, False) == 0
        att[b] = out
        dk, dv = st.download_kv(layer, b, pos, 1)
        assert relative_error(dk[0], kc[pos]) < 1e-5
    want = _oracle_project(oracle_lib, host["out"], att)
    assert relative_error(branch.cpu().numpy(), want) < 2e-3
    for w in dev.values():
        w.close()
    st.close()


def test_layer_decode_rejects_mismatched_weights(cuda_ctx):
    import q38attn
    from q38attn import synth
    torch = _torch()
    g = synth.rng(402)
    _, dev = _layer_weights(cuda_ctx, g, {
        "q": (12, HIDDEN, 12288), "k": (14, HIDDEN, 1024), "v": (8, HIDDEN, 1024),
        "out": (12, 6144, HIDDEN)})
    st = cuda_ctx.state(1, 16, full_slots=1, linear_slots=1)
    norm = torch.zeros(1, HIDDEN, device="cuda")
    branch = torch.zeros(1, HIDDEN, device="cuda")
    pos = torch.zeros(1, dtype=torch.int32, device="cuda")
    swapped = dict(dev, k=dev["q"])
    with pytest.raises(q38attn.Q38Error) as e:
        cuda_ctx.full_attention_decode(st, 3, swapped, norm, pos, branch)
    assert e.value.code == q38attn.Q38_ERR_ARG
    with pytest.raises(q38attn.Q38Error):  # full projections on a DeltaNet layer's shapes
        cuda_ctx.linear_attention_decode(st, 0, {"qkv": dev["q"], "z": dev["k"], "beta": dev["v"],
                                                 "alpha": dev["v"], "out": dev["out"]}, norm, branch)
    for w in dev.values():
        w.close()
    st.close()

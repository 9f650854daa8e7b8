"""GPU test of q38_full_decode_noalloc, the full-attention decode entry point
that allocates no device memory.

Some GPU callers cannot let a library call cudaMalloc: a serving host that has
reserved all of HBM for its own memory pool or KV-block arena (a library
allocation would fail there, or synchronise the device and stall its other
streams, or create memory it cannot account for). For them the library keeps
the decode scratch in a fixed 16 MiB device array of its own, and the caller
passes every input and output, its KV cache included.

This test calls that entry point through the C ABI and checks it against the
regular entry point (q38_full_decode with a q38_state) on the same inputs, for
two calls in a row (each appends one position per sequence), within the 1e-4
tolerance of the other decode tests; checks that later calls leave the
device's free memory unchanged; and checks that a size beyond the scratch's
maximum, or a misaligned pointer, is refused with an argument error before any
device work. The test's own buffers come from torch; the entry point under
test allocates nothing. The file name makes pytest collect it last.
"""
from __future__ import annotations

import ctypes

import numpy as np
import pytest

from conftest import relative_error

pytestmark = pytest.mark.gpu


def _p(t):
    return ctypes.c_void_p(t.data_ptr())


@pytest.mark.parametrize("bf16", [False, True])
def test_noalloc_decode_matches_regular_entry_point(bf16):
    import torch

    import q38attn
    from q38attn import synth
    lib = q38attn.load()
    torch.cuda.set_device(0)
    kv_dtype = q38attn.Q38_KV_BF16 if bf16 else q38attn.Q38_KV_F32
    tdtype = torch.bfloat16 if bf16 else torch.float32
    ctx = q38attn.Context(0)
    g = synth.rng(21 + int(bf16))
    w = synth.full_weights(g)
    layer, ctx_len, B = 3, 512, 3
    start = [100, 311, 7]
    ctx.bind_full_layer(layer, w["q_norm"], w["k_norm"])
    st = ctx.state(B, ctx_len, full_slots=1, linear_slots=0, kv_dtype=kv_dtype)

    # The caller's own KV cache for the no-allocation path, and the same
    # contents in the regular entry point's state.
    tg = torch.Generator(device="cuda")
    tg.manual_seed(5)
    kc = torch.randn(B, 4, ctx_len, 256, generator=tg, device="cuda").to(tdtype)
    vc = torch.randn(B, 4, ctx_len, 256, generator=tg, device="cuda").to(tdtype)
    kview, vview = st.kv_views(layer)
    kview.copy_(kc)
    vview.copy_(vc)
    qn = torch.from_numpy(w["q_norm"]).cuda()
    kn = torch.from_numpy(w["k_norm"]).cuda()
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)

    for call in range(2):
        pos = torch.tensor([p + call for p in start], dtype=torch.int32, device="cuda")
        x = synth.full_step(g, B)
        a = {k: torch.from_numpy(v.copy()).cuda() for k, v in x.items()}
        b = {k: torch.from_numpy(v.copy()).cuda() for k, v in x.items()}
        out_a = torch.zeros(B, 6144, device="cuda")
        out_b = torch.zeros(B, 6144, device="cuda")
        ctx.full_decode(st, layer, a["q_and_gate"], a["key"], a["value"], pos, out_a)
        rc = lib.q38_full_decode_noalloc(_p(qn), _p(kn), _p(kc), _p(vc), B, ctx_len, kv_dtype,
                                         _p(b["q_and_gate"]), _p(b["key"]), _p(b["value"]),
                                         _p(pos), -1, _p(out_b), _p(err), stream)
        assert rc == q38attn.Q38_OK, q38attn.last_error()
        torch.cuda.synchronize()
        assert torch.isfinite(out_b).all()
        assert relative_error(out_b.cpu().numpy(), out_a.cpu().numpy()) < 1e-4, call
        assert relative_error(b["key"].cpu().numpy(), a["key"].cpu().numpy()) < 1e-5, call

    # Both caches received the same appended rows.
    for s, p0 in enumerate(start):
        rows = slice(p0, p0 + 2)
        assert relative_error(kc[s, :, rows].float().cpu().numpy(),
                              kview[s, :, rows].float().cpu().numpy()) < 1e-5
        assert torch.equal(vc[s, :, rows], vview[s, :, rows])
    assert err.item() == 0
    assert st.errors() == 0
    del kview, vview
    st.close()
    ctx.close()


def test_noalloc_decode_allocates_nothing_on_later_calls():
    """Once the first call has loaded the library's device code (and with it
    the fixed scratch array), further calls leave the device's free memory
    unchanged: the entry point itself allocates nothing."""
    import torch

    import q38attn
    from q38attn import synth
    lib = q38attn.load()
    torch.cuda.set_device(0)
    g = synth.rng(23)
    w = synth.full_weights(g)
    B, ctx_len = 2, 256
    kc = torch.randn(B, 4, ctx_len, 256, device="cuda").to(torch.bfloat16)
    vc = torch.randn(B, 4, ctx_len, 256, device="cuda").to(torch.bfloat16)
    qn = torch.from_numpy(w["q_norm"]).cuda()
    kn = torch.from_numpy(w["k_norm"]).cuda()
    x = {k: torch.from_numpy(v.copy()).cuda() for k, v in synth.full_step(g, B).items()}
    pos = torch.tensor([100, 200], dtype=torch.int32, device="cuda")
    out = torch.zeros(B, 6144, device="cuda")
    args = (_p(qn), _p(kn), _p(kc), _p(vc), B, ctx_len, q38attn.Q38_KV_BF16, _p(x["q_and_gate"]),
            _p(x["key"]), _p(x["value"]), _p(pos), -1, _p(out), None, None)
    assert lib.q38_full_decode_noalloc(*args) == q38attn.Q38_OK, q38attn.last_error()
    torch.cuda.synchronize()
    free0, _ = torch.cuda.mem_get_info()
    for _ in range(3):
        assert lib.q38_full_decode_noalloc(*args) == q38attn.Q38_OK, q38attn.last_error()
    torch.cuda.synchronize()
    free1, _ = torch.cuda.mem_get_info()
    assert free1 == free0
    assert torch.isfinite(out).all()


def test_noalloc_decode_rejects_misaligned_pointers():
    """The KV cache is streamed by the bulk-copy engine or by TMA, which need
    16-byte aligned rows: a cache pointer off by 4 bytes (and any tensor off by
    2) is refused on the host before any device work."""
    import torch

    import q38attn
    lib = q38attn.load()
    torch.cuda.set_device(0)
    buf = torch.zeros(1 << 20, device="cuda")
    pos = torch.zeros(1, dtype=torch.int32, device="cuda")
    base = buf.data_ptr()
    ok = ctypes.c_void_p(base)
    off4 = ctypes.c_void_p(base + 4)
    off2 = ctypes.c_void_p(base + 2)
    for kv_dtype in (q38attn.Q38_KV_F32, q38attn.Q38_KV_BF16):
        rc = lib.q38_full_decode_noalloc(ok, ok, off4, ok, 1, 64, kv_dtype, ok, ok, ok, _p(pos),
                                         -1, ok, None, None)
        assert rc == q38attn.Q38_ERR_ARG
        assert "16-byte" in q38attn.last_error()
        rc = lib.q38_full_decode_noalloc(ok, ok, ok, off4, 1, 64, kv_dtype, ok, ok, ok, _p(pos),
                                         -1, ok, None, None)
        assert rc == q38attn.Q38_ERR_ARG
        rc = lib.q38_full_decode_noalloc(ok, ok, ok, ok, 1, 64, kv_dtype, off2, ok, ok, _p(pos),
                                         -1, ok, None, None)
        assert rc == q38attn.Q38_ERR_ARG
        assert "4-byte" in q38attn.last_error()
    torch.cuda.synchronize()


def test_noalloc_decode_rejects_sizes_beyond_its_scratch():
    """64 sequences at 262144 positions need far more than the fixed 16 MiB:
    the call is refused on the host, before any device work."""
    import torch

    import q38attn
    lib = q38attn.load()
    torch.cuda.set_device(0)
    dummy = torch.zeros(16, device="cuda")
    pos = torch.zeros(64, dtype=torch.int32, device="cuda")
    d = _p(dummy)
    rc = lib.q38_full_decode_noalloc(d, d, d, d, 64, 262144, q38attn.Q38_KV_BF16, d, d, d,
                                     _p(pos), -1, d, None, None)
    assert rc == q38attn.Q38_ERR_ARG
    msg = q38attn.last_error()
    assert "16777216" in msg and "scratch" in msg
    torch.cuda.synchronize()

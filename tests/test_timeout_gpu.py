"""GPU test of the bounded-wait error path, in the form this pool allows: no
fault, trap or hang. With Q38_DEBUG_SKIP_KV_LOADS the decode's split-KV
kernel issues none of its KV tile loads, so the waits on those tiles are
waits on barriers that nothing will complete; each gives up after a short
limit (q38_state_set_debug's wait_ns), the kernel records
Q38_DEVERR_TIMEOUT and returns with no copy or MMA in flight, and the
host-pointer call reports Q38_ERR_TIMEOUT. The context stays usable: the next
step, with the flag cleared, matches the oracle.

Reference error convention: Err(-1) at src/model/ops.rs:59, :863; the
timeout status has no counterpart in the reference (its CPU loops cannot
stall)."""
from __future__ import annotations

import numpy as np
import pytest

from conftest import check_parity

pytestmark = pytest.mark.gpu
F = np.float32


@pytest.mark.parametrize("bf16", [False, True])
def test_decode_wait_timeout_is_reported_and_recovers(cuda_ctx, oracle_lib, bf16):
    import q38attn
    from q38attn import synth
    g = synth.rng(50 + int(bf16))
    w = synth.full_weights(g)
    layer, ctx_len, B, pre = 3, 1024, 2, 700
    cuda_ctx.bind_full_layer(layer, w["q_norm"], w["k_norm"])
    kvd = q38attn.Q38_KV_BF16 if bf16 else q38attn.Q38_KV_F32
    st = cuda_ctx.state(B, ctx_len, full_slots=1, linear_slots=0, kv_dtype=kvd)
    rows = []
    for b in range(B):
        k, v = synth.kv_rows(g, pre, bf16=bf16)
        st.upload_kv(layer, b, 0, k, v)
        kc = np.zeros((ctx_len, 1024), F)
        vc = np.zeros((ctx_len, 1024), F)
        kc[:pre], vc[:pre] = k, v
        rows.append((kc, vc))
    positions = np.full(B, pre, np.int32)

    st.set_debug(q38attn.Q38_DEBUG_SKIP_KV_LOADS, 2_000_000)  # 2 ms waits
    x = synth.full_step(g, B)
    att = np.zeros((B, 6144), F)
    with pytest.raises(q38attn.Q38Error) as e:
        cuda_ctx.full_decode_host(st, layer, x["q_and_gate"], x["key"].copy(), x["value"],
                                  positions, att)
    assert e.value.code == q38attn.Q38_ERR_TIMEOUT
    assert st.errors() & q38attn.Q38_DEVERR_TIMEOUT  # read and cleared

    st.set_debug()
    key = x["key"].copy()
    cuda_ctx.full_decode_host(st, layer, x["q_and_gate"], key, x["value"], positions, att)
    assert st.errors() == 0
    for b in range(B):
        kc, vc = rows[b]
        okey = x["key"][b].copy()
        oatt = np.zeros(6144, F)
        assert oracle_lib.full_core(w, x["q_and_gate"][b], okey, x["value"][b],
                                    np.zeros(6144, F), np.zeros(6144, F),
                                    np.zeros(24 * ctx_len, F), oatt, kc, vc, ctx_len, pre, layer,
                                    int(bf16)) == 0
        check_parity(att[b], oatt, 1e-4, f"recovered step, seq {b}")
    st.close()


def test_debug_flags_are_checked(cuda_ctx):
    import q38attn
    st = cuda_ctx.state(1, 16, full_slots=1, linear_slots=0)
    with pytest.raises(q38attn.Q38Error) as e:
        st.set_debug(0x40, 0)
    assert e.value.code == q38attn.Q38_ERR_ARG
    st.close()

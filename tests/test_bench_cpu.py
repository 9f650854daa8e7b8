"""CPU checks of bench.py's accounting: the default arguments are the
headline configuration, and the FLOP and byte counts behind the roofline
fractions follow their definitions."""
from __future__ import annotations

import sys
from pathlib import Path

import pytest

REPO = Path(__file__).resolve().parent.parent


@pytest.fixture(scope="module")
def bench():
    sys.path.insert(0, str(REPO))
    import bench as b
    return b


def test_defaults_are_the_headline_configuration(bench, monkeypatch):
    monkeypatch.setattr(sys, "argv", ["bench.py"])
    a = bench.parse_args()
    assert (a.gpus, a.batch, a.context, a.impl) == (1, 32, 32768, "ours")
    assert a.warmup >= 3
    # Config 4 from position 0 over a bf16 cache; the continuation and
    # f32-cache forms only when asked for.
    assert (a.prefill_batch, a.prefill_len, a.prefill_base, a.prefill_kv) == (4, 8192, 0, "bf16")
    assert a.split_context == 131072


def test_prefill_flops(bench):
    # Config 4: 4 prompts x 24 heads x (QK^T + PV at 2 x 256 each) per
    # visible (query, key) pair, 8192 * 8193 / 2 pairs a prompt.
    assert bench.prefill_flops(4, 8192) == 3_298_937_536_512.0
    # A continuation of S tokens after B cached ones adds what prefilling the
    # B + S tokens from position 0 adds over prefilling the B alone.
    for b, s in ((8192, 4096), (100, 1), (0, 512)):
        assert bench.prefill_flops(1, s, b) == bench.prefill_flops(1, b + s) - bench.prefill_flops(1, b)


def test_decode_bytes(bench):
    # One more cached position costs its K and V rows: 4 KV heads x 256 x 2 B x 2.
    assert bench.attn_bytes_per_seq(32779) - bench.attn_bytes_per_seq(32778) == 4 * 256 * 2 * 2
    # The DeltaNet step reads and writes every value head's 128 x 128 f32 state.
    assert bench.deltanet_bytes_per_seq() > 2 * 48 * 128 * 128 * 4

"""Writes tests/golden/golden.npz: outputs of the CPU oracle (a restatement of
the reference's linear_core / full_core, src/model/ops.rs:647-742, 812-940) on
the formula-generated inputs of vectors.py.

These fixtures pin the oracle against regressions (tests/test_oracle.py checks
them bit-exactly) and give the GPU tests a second, stored target. Regenerate
with:  python tests/golden/make_golden.py
"""
from __future__ import annotations

import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE))
sys.path.insert(0, str(HERE.parents[1] / "oracle"))

import oracle  # noqa: E402
import vectors as V  # noqa: E402

LIN_TOKENS = 3
FULL_CONTEXT, FULL_PREFILLED, FULL_LAYER, FULL_TOKENS = 64, 37, 7, 3


def linear_case() -> dict:
    w = V.linear_weights()
    s = V.linear_state()
    conv, delta = s["conv_state"].copy(), s["delta_state"].copy()
    out = {}
    for t in range(LIN_TOKENS):
        x = V.linear_token(t)
        att = np.zeros(V.V_DIM, np.float32)
        rc = oracle.linear_core(w, conv, delta, x["qkv"], x["z"], x["beta"], x["alpha"], att)
        assert rc == 0
        out[f"lin_attention_{t}"] = att
        out[f"lin_beta_{t}"] = x["beta"]
        out[f"lin_alpha_{t}"] = x["alpha"]
        if t == 0:
            out["lin_qkv_0"] = x["qkv"]
    out["lin_delta_head0"] = delta[0].copy()
    out["lin_delta_head47"] = delta[47].copy()
    out["lin_delta_sums"] = delta.astype(np.float64).sum(axis=(1, 2))
    out["lin_conv_final"] = conv[::16].copy()
    return out


def full_case(bf16: bool) -> dict:
    tag = "fullbf16" if bf16 else "full"
    w = V.full_weights()
    kc, vc = V.full_cache(FULL_CONTEXT, FULL_PREFILLED, FULL_LAYER, full_slots=2)
    if bf16:
        kc, vc = oracle_round(kc), oracle_round(vc)
    out = {}
    q = np.zeros(V.Q_DIM, np.float32)
    gate = np.zeros(V.Q_DIM, np.float32)
    scores = np.zeros(24 * FULL_CONTEXT, np.float32)
    for t in range(FULL_TOKENS):
        x = V.full_token(t)
        att = np.zeros(V.Q_DIM, np.float32)
        pos = FULL_PREFILLED + t
        rc = oracle.full_core(w, x["q_and_gate"], x["key"], x["value"], q, gate, scores, att,
                              kc, vc, FULL_CONTEXT, pos, FULL_LAYER, bf16)
        assert rc == 0
        out[f"{tag}_attention_{t}"] = att
        out[f"{tag}_key_{t}"] = x["key"]
        out[f"{tag}_q_{t}"] = q.copy()
        row = (FULL_LAYER // 4) * FULL_CONTEXT + pos
        out[f"{tag}_krow_{t}"] = kc[row].copy()
        out[f"{tag}_vrow_{t}"] = vc[row].copy()
    return out


def oracle_round(a: np.ndarray) -> np.ndarray:
    flat = a.reshape(-1)
    return np.array([oracle.round_bf16(float(x)) for x in flat], np.float32).reshape(a.shape)


def scalar_case() -> dict:
    xs = V.activation(257, 3, 25.0)  # [-25, 25]
    return {
        "sc_x": xs,
        "sc_sigmoid": np.array([oracle.sigmoid(float(x)) for x in xs], np.float32),
        "sc_silu": np.array([oracle.silu(float(x)) for x in xs], np.float32),
        "sc_softplus": np.array([oracle.softplus(float(x)) for x in xs], np.float32),
        "sc_rms_scale": np.array([oracle.rms_scale(V.activation(256, k)) for k in range(8)],
                                 np.float32),
    }


def main() -> None:
    oracle.build()
    out = {}
    out.update(linear_case())
    out.update(full_case(False))
    out.update(full_case(True))
    out.update(scalar_case())
    np.savez_compressed(HERE / "golden.npz", **out)
    print(f"wrote {HERE / 'golden.npz'} ({(HERE / 'golden.npz').stat().st_size} bytes, "
          f"{len(out)} arrays)")


if __name__ == "__main__":
    main()

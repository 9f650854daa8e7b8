#!/usr/bin/env python
"""Benchmark of the attention hot path on B200 (one JSON line on rank 0).

Workload (BASELINE.json metric "attn+DeltaNet decode tok/s & % HBM roofline
@32K ctx"; config 3 with the config-2 DeltaNet layers): one decode step of a
32-sequence batch per GPU through one model layer group -- three Gated
DeltaNet layers (linear_core, src/model/ops.rs:647-742) and one gated
full-attention layer (full_core, ops.rs:812-940) over a bf16 KV cache holding
32768 positions per sequence. Every step appends one position per sequence.
Inputs are seeded synthetic data with the configs' distributions (no
checkpoint is available); the KV cache (4.3 GB) is larger than L2, so no L2
flush is needed between steps.

  value  tokens/s over all ranks, device-timed (CUDA events), inputs resident
         in HBM; max over ranks.
  e2e    the same metric through the host-pointer C-ABI calls
         (q38_linear_decode_host / q38_full_decode_host): pinned host inputs
         copied in and outputs copied back every step, host wall clock.
  roofline  the full-attention decode operation (prep + split-KV + merge
         kernels, the dominant cost) against the measured HBM copy bandwidth.
  cpu_baseline  the CPU oracle (a restatement of the reference's Rust cores,
         threaded over heads like its rayon regions) on a bounded sample of the
         same workload, rank 0 at N=1 only.
  projection  the quantized projections around a DeltaNet core (12 layers'
         weights, one CUDA graph) at batch 1 and the decode batch, with the
         oracle's projection path timed beside them (projection.cpu_baseline).

--impl reference runs only the CPU oracle (the reference's algorithm; the
Rust crate itself cannot be built here), rank 0 only.

Multi-GPU: one process per GPU (torchrun). The headline decode shards by
sequence: every rank owns its own 32 sequences (weak scaling, no data-path
collective). The prefill legs keep the global config-4 / config-5 workload
fixed and split its units across the ranks (strong scaling): (sequence,
KV-head group) units for the attention prefill, value heads for the DeltaNet
prefill (--prefill-base N runs the attention prefill as a continuation after N
cached positions, --prefill-kv f32 over the reference's f32 cache). The
split-sequence leg spreads one sequence's positions over the ranks; the merge
kernel exchanges the softmax partials over peer memory (the timed tokens
replayed as one CUDA graph), and the same step with the library's NCCL
all-gather is reported beside it.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import sys
import threading
import time
from pathlib import Path

REPO = Path(__file__).resolve().parent
sys.path.insert(0, str(REPO / "qwen3.8_27b_in_rust_b200"))

METRIC = "attn+DeltaNet decode tok/s & % HBM roofline @32K ctx; prefill TFLOP/s; 1-8 GPU"
FULL_LAYER = 3
LINEAR_LAYERS = (0, 1, 2)


def parse_args():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=400)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--batch", type=int, default=32)
    ap.add_argument("--context", type=int, default=32768)
    ap.add_argument("--seed", type=int, default=0)
    ap.add_argument("--cpu-seconds", type=float, default=10.0,
                    help="CPU work budget of the cpu_baseline sample")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-prefill", action="store_true")
    ap.add_argument("--prefill-batch", type=int, default=4)
    ap.add_argument("--prefill-len", type=int, default=8192)
    ap.add_argument("--prefill-iters", type=int, default=5)
    ap.add_argument("--prefill-base", type=int, default=0,
                    help="config-4 leg: cached positions before each prompt (a continuation)")
    ap.add_argument("--prefill-kv", choices=["bf16", "f32"], default="bf16",
                    help="config-4 leg: KV cache type (f32: the reference's cache)")
    ap.add_argument("--no-cpu", action="store_true")
    ap.add_argument("--no-split", action="store_true")
    ap.add_argument("--split-context", type=int, default=131072)
    ap.add_argument("--split-steps", type=int, default=50)
    ap.add_argument("--no-proj", action="store_true")
    ap.add_argument("--proj-layers", type=int, default=12)
    return ap.parse_args()


# ---------------------------------------------------------------------------
# Byte accounting (algorithmic bytes, fp32 I/O, bf16 KV)
# ---------------------------------------------------------------------------
def attn_bytes_per_seq(positions: int) -> int:
    """Full-attention decode of one sequence at `positions` cached rows
    (including the new one): K and V rows read (bf16), q/gate/key/value in,
    key and attention out, the appended K/V row."""
    kv = positions * 4 * 256 * 2 * 2
    io = (12288 + 1024 + 1024) * 4 + (1024 + 6144) * 4 + 2 * 1024 * 2
    return kv + io


def deltanet_bytes_per_seq() -> int:
    """One DeltaNet decode step of one sequence: the 48x128x128 f32 state read
    and written, the conv state read and written, conv weights, qkv/z/beta/alpha
    in, qkv/beta/alpha/attention out."""
    state = 2 * 48 * 128 * 128 * 4
    conv = 2 * 10240 * 3 * 4 + 10240 * 4 * 4
    io = (10240 + 6144 + 96) * 4 + (10240 + 96 + 6144) * 4
    return state + conv + io


def load_peaks() -> tuple[float, str]:
    p = REPO / "MEASURED_PEAKS.json"
    if p.exists():
        try:
            return float(json.loads(p.read_text())["hbm_gbs"]), "measured"
        except Exception:
            pass
    return 6650.0, "fallback"


def load_tensor_peak() -> tuple[float, str]:
    p = REPO / "MEASURED_PEAKS.json"
    if p.exists():
        try:
            return float(json.loads(p.read_text())["bf16_tflops"]), "measured"
        except Exception:
            pass
    return 1590.0, "fallback"


def prefill_flops(batch: int, seq: int, base: int = 0) -> float:
    """Causal attention FLOPs (config 4): batch * 24 heads * (2*256 for QK^T +
    2*256 for PV) per visible (query, key) pair: seq*(seq+1)/2 pairs, plus
    seq*base with `base` cached positions before the prompt."""
    return float(batch) * 24 * 4 * 256 * (seq * (seq + 1) / 2 + float(seq) * base)


def run_prefill(args, ctx, q38attn, synth, torch, rank: int, world: int, dist) -> dict:
    """Config 4: causal prefill of `prefill_batch` prompts of `prefill_len`
    tokens through one full-attention layer, on the tensor cores. The global
    workload is fixed; its (sequence, KV-head group) units are split across
    the ranks (strong scaling), each rank running q38_full_prefill_heads over
    its share on the same global inputs."""
    from q38attn.parallel import prefill_segments
    B, S, base = args.prefill_batch, args.prefill_len, args.prefill_base
    layer = FULL_LAYER
    segs = prefill_segments(B, 4, world, rank)
    kv = q38attn.Q38_KV_F32 if args.prefill_kv == "f32" else q38attn.Q38_KV_BF16
    st = ctx.state(B, base + S, full_slots=1, linear_slots=0, kv_dtype=kv)
    st.reserve_prefill(max(n for _, n, _, _ in segs) * S)
    tg = torch.Generator(device="cuda")
    tg.manual_seed(args.seed + 77)  # the same global prompts on every rank
    if base:
        # The cached prefix (a continuation prompt), filled on the device.
        kview, vview = st.kv_views(layer)
        kview[:, :, :base].normal_(generator=tg)
        vview[:, :, :base].normal_(generator=tg)
        del kview, vview
    qg = torch.randn(B, S, 12288, device="cuda", generator=tg)
    key0 = torch.randn(B, S, 1024, device="cuda", generator=tg)
    val = torch.randn(B, S, 1024, device="cuda", generator=tg)
    key = torch.empty_like(key0)
    att = torch.empty(B, S, 6144, device="cuda")
    stream = torch.cuda.current_stream()
    evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
           for _ in range(args.prefill_iters)]

    def one():
        for s0, n, h0, nh in segs:
            ctx.full_prefill_heads(st, layer, s0, qg[s0:s0 + n], key[s0:s0 + n], val[s0:s0 + n],
                                   att[s0:s0 + n], base, h0, nh, stream=stream)

    for it in range(2):
        key.copy_(key0)  # key is rewritten in place (RMSNorm + RoPE)
        one()
    torch.cuda.synchronize()
    if dist is not None:
        dist.barrier()
    with ClockSampler(torch.cuda.current_device(), period_s=0.002) as clocks:
        for it in range(args.prefill_iters):
            key.copy_(key0)
            evs[it][0].record(stream)
            one()
            evs[it][1].record(stream)
        torch.cuda.synchronize()
    if st.errors():
        raise RuntimeError("device error bits set during prefill")
    ms = statistics.median(a.elapsed_time(b) for a, b in evs)
    st.close()
    del qg, key0, val, key, att
    torch.cuda.empty_cache()
    return {"ms": ms, "clocks": clocks.summary(),
            "units": sum(n * nh for _, n, _, nh in segs)}


def linear_prefill_flops(batch: int, seq: int) -> float:
    """Chunked DeltaNet prefill FLOPs (config 5, C=64, dk=dv=128, 48 value heads):
    per chunk and head 2*(C*C*dk [KK^T] + C*C*dk [W] + C*C*dv [Ut] + C*dk*dv [WS]
    + C*C*dk [QK^T] + C*dk*dv [QS] + C*C*dv [PU] + C*dk*dv [state])."""
    C, dk = 64, 128
    per_chunk = 2 * (5 * C * C * dk + 3 * C * dk * dk)
    return float(batch) * 48 * (seq // C) * per_chunk


def run_linear_prefill(args, ctx, q38attn, torch, rank: int, world: int, dist) -> dict:
    """Config 5: chunked DeltaNet prefill of `prefill_batch` prompts of
    `prefill_len` tokens through one DeltaNet layer from a zero state. The
    global workload is fixed; its 48 value heads are split across the ranks
    (strong scaling; every rank convolves the shared q/k channels itself)."""
    from q38attn.parallel import shard_range
    B, S = args.prefill_batch, args.prefill_len
    layer = LINEAR_LAYERS[0]
    h0, h1 = shard_range(48, world, rank)
    st = ctx.state(B, 16, full_slots=0, linear_slots=1)
    st.reserve_prefill(B * S)
    tg = torch.Generator(device="cuda")
    tg.manual_seed(args.seed + 99)  # the same global prompts on every rank
    qkv0 = torch.randn(B, S, 10240, device="cuda", generator=tg)
    z = torch.randn(B, S, 6144, device="cuda", generator=tg)
    b0 = torch.randn(B, S, 48, device="cuda", generator=tg)
    a0 = torch.randn(B, S, 48, device="cuda", generator=tg)
    qkv, beta, alpha = torch.empty_like(qkv0), torch.empty_like(b0), torch.empty_like(a0)
    att = torch.empty(B, S, 6144, device="cuda")
    stream = torch.cuda.current_stream()
    evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
           for _ in range(args.prefill_iters)]
    def one(it):
        st.reset(stream)  # a fresh prompt each time (zero conv and delta state)
        qkv.copy_(qkv0)   # qkv/beta/alpha are rewritten in place
        beta.copy_(b0)
        alpha.copy_(a0)
        if it >= 0:
            evs[it][0].record(stream)
        ctx.linear_prefill_heads(st, layer, 0, qkv, z, beta, alpha, att, h0, h1 - h0,
                                 stream=stream)
        if it >= 0:
            evs[it][1].record(stream)

    one(-1)
    one(-1)
    torch.cuda.synchronize()
    if dist is not None:
        dist.barrier()
    with ClockSampler(torch.cuda.current_device(), period_s=0.002) as clocks:
        for it in range(args.prefill_iters):
            one(it)
        torch.cuda.synchronize()
    if st.errors():
        raise RuntimeError("device error bits set during DeltaNet prefill")
    ms = statistics.median(a.elapsed_time(b) for a, b in evs)
    st.close()
    del qkv0, z, b0, a0, qkv, beta, alpha, att
    torch.cuda.empty_cache()
    return {"ms": ms, "clocks": clocks.summary(), "heads": h1 - h0}


# Projection weights of one DeltaNet layer, Q4_K_M-like (ggml type, width, rows):
# attn_qkv and attn_gate Q4_K, the 48-row ssm_beta / ssm_alpha gates Q8_0,
# ssm_out Q6_K (src/model/mod.rs:28-48 names; no checkpoint is available).
PROJ_SPEC = {"qkv": (12, 5120, 10240), "z": (12, 5120, 6144), "beta": (8, 5120, 48),
             "alpha": (8, 5120, 48), "out": (14, 6144, 5120)}


def run_projection(args, ctx, q38attn, synth, torch, rank: int) -> dict:
    """The projections around a DeltaNet core (linear_attention, ops.rs:761-803
    minus the core): quantize the 5120-wide input once, qkv / z / beta /
    alpha, quantize the 6144-wide core output, ssm_out -- for `proj_layers`
    distinct layers' weights (more bytes than L2 holds), replayed as one CUDA
    graph; at batch 1 (the reference's decode) and at the decode batch."""
    g = synth.rng(args.seed + 7 + rank)
    layers, nbytes = [], 0
    for _ in range(args.proj_layers):
        d = {}
        for k, (t, w, r) in PROJ_SPEC.items():
            data = synth.quant_weight(g, t, r, w)
            nbytes += data.size
            d[k] = ctx.weight(t, w, r, data)
        layers.append(d)
    per_layer = nbytes / args.proj_layers
    plane_bytes = None
    out = {}
    legs = [(1, False)] + ([(args.batch, False), (args.batch, True)] if args.batch >= 9 else
                           [(args.batch, False)] if args.batch != 1 else [])
    for B, planes in legs:
        if planes and plane_bytes is None:
            # Integer planes for the K-quant weights (q38_weight_build_planes).
            plane_bytes = 0
            for d in layers:
                for k in ("qkv", "z", "out"):
                    d[k].build_planes()
                    t, w, r = PROJ_SPEC[k]
                    rp = (r + 127) // 128 * 128  # rows padded to the 128-row tile
                    # quant planes (Q4_K / Q5_K) 1 byte per weight, product planes
                    # (Q6_K) 2, plus a 16-byte record per (row, 256-block)
                    plane_bytes += (2 if t == 14 else 1) * rp * w + (w // 256) * rp * 16
            plane_bytes /= args.proj_layers
        ctx.reserve_projection(B, 6144)
        x = torch.randn(B, 5120, device="cuda")
        a = torch.randn(B, 6144, device="cuda")
        outs = {k: torch.zeros(B, r, device="cuda") for k, (t, w, r) in PROJ_SPEC.items()}

        def step():
            for d in layers:
                for k in ("qkv", "z", "beta", "alpha"):
                    ctx.project(d[k], x, outs[k])
                ctx.project(d["out"], a, outs["out"])

        step()
        torch.cuda.synchronize()
        graph = torch.cuda.CUDAGraph()
        side = torch.cuda.Stream()
        side.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(side), torch.cuda.graph(graph, stream=side):
            step()
        torch.cuda.current_stream().wait_stream(side)
        for _ in range(3):
            graph.replay()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        iters = 10
        e0.record()
        for _ in range(iters):
            graph.replay()
        e1.record()
        torch.cuda.synchronize()
        ms = e0.elapsed_time(e1) / iters / args.proj_layers
        peak, _ = load_peaks()
        gbs = per_layer / (ms * 1e-3) / 1e9
        leg = {"ms_per_layer": ms, "weight_gbs": gbs, "frac": gbs / peak,
               "path": ("tcgen05 kind::i8 from integer planes (K-quants), f32 GEMV (Q8_0 gates)" if planes
                        else "tcgen05 kind::i8, operands built per call (K-quants), f32 GEMV (Q8_0 gates)"
                        if B >= 9 else "dp4a integer GEMV (K-quants), f32 GEMV (Q8_0 gates)")}
        if planes:
            # Bytes the kernels stream: the planes of the K-quant matrices plus
            # the gates' Q8_0 bytes.
            streamed = plane_bytes + sum(r * w * 34 / 32 for k, (t, w, r) in PROJ_SPEC.items()
                                         if k in ("beta", "alpha"))
            leg["streamed_bytes_per_layer"] = streamed
            leg["streamed_gbs"] = streamed / (ms * 1e-3) / 1e9
            leg["streamed_frac"] = leg["streamed_gbs"] / peak
        out[f"batch{B}" + ("" if planes or B < 9 or args.batch < 9 else "_operands_per_call")] = leg
        del graph
    out["weight_bytes_per_layer"] = per_layer
    out["layer_decode"] = run_layer_decode(args, ctx, synth, torch, layers, rank)
    for d in layers:
        for w in d.values():
            w.close()
    return out


def run_layer_decode(args, ctx, synth, torch, layers, rank: int) -> dict:
    """linear_attention (src/model/ops.rs:744-803) through the layer-level call
    q38_linear_attention_decode -- the four input projections, the DeltaNet
    core on the resident state, the output projection -- for the projection
    leg's distinct layers (DeltaNet layers 0, 1, 2, 4, 5, ...), one CUDA graph,
    at batch 1 and at the decode batch: ms per layer."""
    import q38attn
    g = synth.rng(args.seed + 11 + rank)
    idx = [l for l in range(64) if not q38attn.is_full_attention(l)][:len(layers)]
    for l in idx:
        wl = synth.linear_weights(g)
        ctx.bind_linear_layer(l, wl["conv1d"], wl["dt_bias"], wl["ssm_a"], wl["ssm_norm"])
    res = {}
    for B in sorted({1, args.batch}):
        st = ctx.state(B, 16, full_slots=0, linear_slots=q38attn.recurrent_index(idx[-1]) + 1)
        for l in idx:
            cview, dview = st.linear_views(l)
            cview.normal_()
            dview.normal_(0.0, 0.02)
        del cview, dview
        ctx.reserve_projection(B, 6144)
        norm = torch.randn(B, 5120, device="cuda")
        branch = torch.empty(B, 5120, device="cuda")

        def step():
            for l, d in zip(idx, layers):
                ctx.linear_attention_decode(st, l, d, norm, branch)

        step()
        torch.cuda.synchronize()
        graph = torch.cuda.CUDAGraph()
        side = torch.cuda.Stream()
        side.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(side), torch.cuda.graph(graph, stream=side):
            step()
        torch.cuda.current_stream().wait_stream(side)
        for _ in range(3):
            graph.replay()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        iters = 10
        e0.record()
        for _ in range(iters):
            graph.replay()
        e1.record()
        torch.cuda.synchronize()
        if st.errors():
            raise RuntimeError("device error bits set during the layer-decode leg")
        res[f"batch{B}"] = {"ms_per_layer": e0.elapsed_time(e1) / iters / len(idx)}
        del graph
        st.close()
    return res


def run_split_sequence(args, ctx, q38attn, torch, dist, rank: int, world: int,
                       transport: str = "p2p") -> dict:
    """Config 3, split-sequence variant: one sequence with `split_context`
    cached bf16 positions, sharded into contiguous ranges across the ranks;
    each decode step computes per-shard softmax partials, exchanges them and
    merges (q38attn.parallel.SplitSequenceDecoder): over peer memory inside
    the merge kernel ("p2p") or with an NCCL all-gather ("nccl"). At one GPU
    the plain decode runs over the whole range."""
    from q38attn.parallel import SplitSequenceDecoder, position_ranges
    P = args.split_context
    cap = P + args.split_steps + 8
    p0, p1 = position_ranges(cap, world)[rank]
    st = ctx.state(1, p1 - p0, full_slots=1, linear_slots=0, kv_dtype=q38attn.Q38_KV_BF16)
    kview, vview = st.kv_views(FULL_LAYER)
    tg = torch.Generator(device="cuda")
    tg.manual_seed(args.seed + 555 + rank)
    n = max(0, min(p1, P) - p0)
    if n:
        kview[0, :, :n].normal_(generator=tg)
        vview[0, :, :n].normal_(generator=tg)
    del kview, vview
    qg = torch.randn(1, 12288, device="cuda", generator=tg)
    # One key row per step: the call normalises and rotates its key in place.
    keys = torch.randn(args.split_steps + 3, 1024, device="cuda", generator=tg)
    val = torch.randn(1, 1024, device="cuda", generator=tg)
    out = torch.empty(1, 6144, device="cuda")
    pos = torch.arange(P, P + args.split_steps + 3, device="cuda", dtype=torch.int32)
    dec = SplitSequenceDecoder(ctx, st, FULL_LAYER, p0, transport=transport) if world > 1 else None
    if dist is not None:
        dist.barrier()
    stream = torch.cuda.current_stream()

    def one(i, s):
        key = keys[i:i + 1]
        if dec is not None:
            dec.step(qg, key, val, pos[i:i + 1], out, cap - 1, stream=s)
        else:
            ctx.full_decode(st, FULL_LAYER, qg, key, val, pos[i:i + 1], out,
                            max_position=P + i, stream=s)

    for i in range(3):
        one(i, stream)
    torch.cuda.synchronize()
    # The timed tokens as one CUDA graph (one GPU, or the peer-memory exchange,
    # whose epoch counter lives on the device): a token's three launches take
    # the host ~24 us to issue, more than a small shard's kernels run. The NCCL
    # transport stays eager.
    graph = None
    if dec is None or transport == "p2p":
        graph = torch.cuda.CUDAGraph()
        side = torch.cuda.Stream()
        side.wait_stream(stream)
        with torch.cuda.stream(side), torch.cuda.graph(graph, stream=side):
            for i in range(args.split_steps):
                one(3 + i, side)
        stream.wait_stream(side)
        graph.replay()  # warm
        torch.cuda.synchronize()
    if dist is not None:
        dist.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    if graph is not None:
        graph.replay()
    else:
        for i in range(args.split_steps):
            one(3 + i, stream)
    e1.record(stream)
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / args.split_steps
    del graph
    if st.errors():
        raise RuntimeError("device error bits set during split-sequence decode")
    if dec is not None:
        dec.close()
    st.close()
    return {"ms": ms}


def load_traffic_profile() -> dict | None:
    p = REPO / "profiles" / "attn_decode_traffic.json"
    if p.exists():
        try:
            return json.loads(p.read_text())
        except Exception:
            return None
    return None


# ---------------------------------------------------------------------------
# Clock sampling during the timed region (NVML, read-only)
# ---------------------------------------------------------------------------
class ClockSampler:
    def __init__(self, device_index: int, period_s: float = 0.02):
        self.samples = []
        self.reasons = set()
        self.max_mhz = None
        self._stop = threading.Event()
        self._thread = None
        try:
            import pynvml
            pynvml.nvmlInit()
            self._nvml = pynvml
            self._h = pynvml.nvmlDeviceGetHandleByIndex(device_index)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self._h, pynvml.NVML_CLOCK_SM)
        except Exception:
            self._nvml = None
        self.period = period_s

    def _reason_names(self, bits: int) -> list[str]:
        names = {
            0x0000000000000004: "sw_power_cap",
            0x0000000000000008: "hw_slowdown",
            0x0000000000000020: "sw_thermal_slowdown",
            0x0000000000000040: "hw_thermal_slowdown",
            0x0000000000000080: "hw_power_brake_slowdown",
        }
        return [n for b, n in names.items() if bits & b]

    def _run(self):
        nv = self._nvml
        while not self._stop.is_set():
            try:
                mhz = nv.nvmlDeviceGetClockInfo(self._h, nv.NVML_CLOCK_SM)
                bits = nv.nvmlDeviceGetCurrentClocksEventReasons(self._h)
                self.samples.append(mhz)
                self.reasons.update(self._reason_names(bits))
            except Exception:
                pass
            self._stop.wait(self.period)

    def __enter__(self):
        if self._nvml is not None:
            self._thread = threading.Thread(target=self._run, daemon=True)
            self._thread.start()
        return self

    def __exit__(self, *exc):
        self._stop.set()
        if self._thread is not None:
            self._thread.join()

    def summary(self) -> dict:
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": self.max_mhz, "reasons": [], "samples": 0}
        return {"sm_mhz": statistics.median(self.samples), "sm_max_mhz": self.max_mhz,
                "reasons": sorted(self.reasons), "samples": len(self.samples)}


# ---------------------------------------------------------------------------
# CPU legs (the oracle restates the reference's algorithm; checker only)
# ---------------------------------------------------------------------------
class CpuWorkload:
    """One sequence of the bench workload on the CPU oracle: a 32768-position
    f32 cache holding bf16-rounded values (what the GPU's bf16 cache holds),
    three DeltaNet layers and one full-attention layer."""

    def __init__(self, context: int, seed: int):
        sys.path.insert(0, str(REPO / "oracle"))
        import numpy as np

        import oracle
        from q38attn import synth
        oracle.build()
        oracle.set_threads(os.cpu_count() or 1)
        self.np, self.oracle = np, oracle
        g = synth.rng(seed + 1000)
        self.context = context
        self.cap = context + 4096
        self.kc = np.zeros((self.cap, 1024), np.float32)
        self.vc = np.zeros((self.cap, 1024), np.float32)
        for i in range(0, context, 4096):
            n = min(4096, context - i)
            k, v = synth.kv_rows(g, n, bf16=True)
            self.kc[i:i + n], self.vc[i:i + n] = k, v
        self.wf = synth.full_weights(g)
        self.wl = [synth.linear_weights(g) for _ in LINEAR_LAYERS]
        self.sl = [synth.linear_state(g) for _ in LINEAR_LAYERS]
        self.full_in = {k: v[0] for k, v in synth.full_step(g).items()}
        self.lin_in = {k: v[0] for k, v in synth.linear_step(g).items()}
        self.pos = context
        self.q = np.zeros(6144, np.float32)
        self.gate = np.zeros(6144, np.float32)
        self.scores = np.zeros(24 * self.cap, np.float32)
        self.att = np.zeros(6144, np.float32)

    def token(self) -> None:
        np, o = self.np, self.oracle
        for i, _ in enumerate(LINEAR_LAYERS):
            x = {k: v.copy() for k, v in self.lin_in.items()}
            o.linear_core(self.wl[i], self.sl[i]["conv_state"], self.sl[i]["delta_state"],
                          x["qkv"], x["z"], x["beta"], x["alpha"], self.att)
        if self.pos >= self.cap:
            self.pos = self.context
        key = self.full_in["key"].copy()
        rc = o.full_core(self.wf, self.full_in["q_and_gate"], key, self.full_in["value"],
                         self.q, self.gate, self.scores, self.att, self.kc, self.vc, self.cap,
                         self.pos, FULL_LAYER % 4, True)
        assert rc == 0
        self.pos += 1


def cpu_projection_baseline(args, batches) -> dict:
    """The projection leg's CPU side: the oracle's quantize_q8_k + integer dots
    (the reference's project / batch_project path, threaded over rows like its
    row-parallel gemm) for one DeltaNet layer's five projections, repeated for
    about `cpu_seconds` / 4 per batch size."""
    sys.path.insert(0, str(REPO / "oracle"))
    import oracle
    from q38attn import synth
    oracle.build()
    oracle.set_threads(os.cpu_count() or 1)
    g = synth.rng(args.seed + 2000)
    ws = {k: (t, w, r, synth.quant_weight(g, t, r, w)) for k, (t, w, r) in PROJ_SPEC.items()}
    out = {}
    for B in batches:
        x, a = synth.normal(g, (B, 5120)), synth.normal(g, (B, 6144))

        def layer():
            for k, (t, w, r, d) in ws.items():
                oracle.project(t, d, r, w, a if k == "out" else x)

        layer()  # warm
        t0, n = time.perf_counter(), 0
        while True:
            layer()
            n += 1
            if time.perf_counter() - t0 >= args.cpu_seconds / 4:
                break
        dt = time.perf_counter() - t0
        out[f"batch{B}"] = {"ms_per_layer": dt / n * 1e3, "sample": f"{n} layers, {dt:.1f} s"}
    out.update({"unit": "ms per layer", "cores": oracle.get_threads(), "kind": "port",
                "what": "C++ restatement of quantize_q8_k and the dot_q*_k_q8_k / f32 dots "
                        "(bit-identical outputs), OpenMP over rows"})
    return out


def cpu_baseline(args) -> dict:
    w = CpuWorkload(args.context, args.seed)
    w.token()  # warm
    t0 = time.perf_counter()
    n = 0
    while True:
        w.token()
        n += 1
        if time.perf_counter() - t0 >= args.cpu_seconds:
            break
    dt = time.perf_counter() - t0
    return {"value": n / dt, "unit": "tok/s", "cores": w.oracle.get_threads(), "kind": "port",
            "sample": f"{n} sequence-tokens of the workload (3 DeltaNet layers + 1 full-attention "
                      f"layer at {args.context} cached positions each), {dt:.1f} s, C++ "
                      f"restatement of the reference cores, OpenMP over heads"}


def run_reference(args) -> None:
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    w = CpuWorkload(args.context, args.seed)
    for _ in range(args.warmup):
        w.token()
    times = []
    for _ in range(args.steps):
        t0 = time.perf_counter()
        w.token()
        times.append(time.perf_counter() - t0)
    total = sum(times)
    value = args.steps / total
    line = {
        "metric": METRIC, "value": value, "unit": "tok/s", "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1e3 * total / args.steps,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic (seeded; config distributions)", "impl": "reference",
        "config": workload_config(args),
        "cpu_baseline": {"value": value, "unit": "tok/s", "cores": w.oracle.get_threads(),
                         "kind": "port",
                         "sample": "1 sequence-token per step (3 DeltaNet layers + 1 "
                                   f"full-attention layer at {args.context} cached positions)"},
        "e2e": {"value": value, "unit": "tok/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def workload_config(args) -> dict:
    return {
        "workload": ("config3+config2: per GPU, 32-sequence decode step through 3 Gated "
                     "DeltaNet layers + 1 gated full-attention layer, bf16 KV cache at "
                     f"{args.context} cached positions per sequence"),
        "global_batch": args.batch * args.gpus, "batch_per_gpu": args.batch,
        "seq_len": args.context, "kv_dtype": "bf16", "state_dtype": "f32",
        "geometry": "24Q/4KV x 256 (RoPE 64, theta 1e7); DeltaNet 16K/48V x 128, conv 4",
        "parallelism": f"sequences sharded, {args.gpus} rank(s), no collective",
        "l2": "inputs > L2 (4.3 GB KV per GPU); no flush",
    }


# ---------------------------------------------------------------------------
# GPU arm
# ---------------------------------------------------------------------------
def run_ours(args) -> None:
    import numpy as np
    import torch

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dist = None
    if world > 1:
        import datetime

        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                device_id=torch.device("cuda", local))

    import q38attn
    from q38attn import synth

    B, ctx_pos = args.batch, args.context
    total_steps = args.warmup + args.steps
    e2e_steps = 0 if args.no_e2e else min(args.steps, 50)
    cap = ctx_pos + total_steps + e2e_steps + 8
    ctx = q38attn.Context(local)
    g = synth.rng(args.seed + 7919 * rank)
    wf = synth.full_weights(g)
    ctx.bind_full_layer(FULL_LAYER, wf["q_norm"], wf["k_norm"])
    for l in LINEAR_LAYERS:
        wl = synth.linear_weights(g)
        ctx.bind_linear_layer(l, wl["conv1d"], wl["dt_bias"], wl["ssm_a"], wl["ssm_norm"])
    st = ctx.state(B, cap, full_slots=1, linear_slots=len(LINEAR_LAYERS),
                   kv_dtype=q38attn.Q38_KV_BF16)

    # Device-side init of the resident state (seeded).
    tg = torch.Generator(device="cuda")
    tg.manual_seed(args.seed + 1000003 * rank)
    kview, vview = st.kv_views(FULL_LAYER)
    for b in range(B):
        kview[b, :, :ctx_pos].normal_(generator=tg)
        vview[b, :, :ctx_pos].normal_(generator=tg)
    for l in LINEAR_LAYERS:
        cview, dview = st.linear_views(l)
        cview.normal_(generator=tg)
        dview.normal_(0.0, 0.02, generator=tg)
    del kview, vview

    # Per-step inputs, generated ahead: the calls rewrite qkv, beta, alpha and
    # key in place, so each step reads a slice of its own (a pool of up to 512
    # slices, reused cyclically by longer runs) and no copy kernel runs inside
    # the timed region.
    n_lin = len(LINEAR_LAYERS)
    sizes = [("qg", (B, 12288)), ("key", (B, 1024)), ("value", (B, 1024))]
    for i in range(n_lin):
        sizes += [(f"qkv{i}", (B, 10240)), (f"z{i}", (B, 6144)), (f"beta{i}", (B, 48)),
                  (f"alpha{i}", (B, 48))]
    total = sum(int(np.prod(s)) for _, s in sizes)

    def views(flat):
        out, off = {}, 0
        for name, shape in sizes:
            n = int(np.prod(shape))
            out[name] = flat[off:off + n].view(*shape)
            off += n
        return out

    pool = min(total_steps, 512)
    inputs = torch.randn(pool, total, device="cuda", generator=tg)
    pristine = [inputs[0].clone(), inputs[min(1, pool - 1)].clone()]  # the e2e leg's host inputs
    step_views = [views(inputs[i]) for i in range(pool)]
    out_full = torch.empty(B, 6144, device="cuda")
    out_lin = [torch.empty(B, 6144, device="cuda") for _ in range(n_lin)]
    positions = (torch.arange(total_steps, device="cuda", dtype=torch.int32)[:, None] + ctx_pos
                 ).expand(total_steps, B).contiguous()
    stream = torch.cuda.current_stream()

    ev_attn = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
               for _ in range(args.steps)]
    ev_lin = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
              for _ in range(args.steps)]

    def step(s: int, timed_index: int = -1):
        wv = step_views[s % pool]
        if timed_index >= 0:
            ev_lin[timed_index][0].record(stream)
        for i, l in enumerate(LINEAR_LAYERS):
            ctx.linear_decode(st, l, wv[f"qkv{i}"], wv[f"z{i}"], wv[f"beta{i}"], wv[f"alpha{i}"],
                              out_lin[i], stream=stream)
        if timed_index >= 0:
            ev_lin[timed_index][1].record(stream)
            ev_attn[timed_index][0].record(stream)
        ctx.full_decode(st, FULL_LAYER, wv["qg"], wv["key"], wv["value"], positions[s],
                        out_full, max_position=ctx_pos + s, stream=stream)
        if timed_index >= 0:
            ev_attn[timed_index][1].record(stream)

    for s in range(args.warmup):
        step(s)
    torch.cuda.synchronize()
    if st.errors():
        raise RuntimeError("device error bits set during warm-up")

    def barrier():
        if dist is not None:
            dist.barrier()
        torch.cuda.synchronize()

    t_start = torch.cuda.Event(enable_timing=True)
    t_end = torch.cuda.Event(enable_timing=True)
    barrier()
    with ClockSampler(local) as clocks:
        t_start.record(stream)
        for k in range(args.steps):
            step(args.warmup + k, k)
        t_end.record(stream)
        torch.cuda.synchronize()
    barrier()
    ms = t_start.elapsed_time(t_end)
    attn_ms = statistics.mean(a.elapsed_time(b) for a, b in ev_attn)
    lin_ms = statistics.mean(a.elapsed_time(b) for a, b in ev_lin)
    if st.errors():
        raise RuntimeError("device error bits set during the timed region")

    split = split_nccl = None
    if not args.no_split:
        split = run_split_sequence(args, ctx, q38attn, torch, dist, rank, world, "p2p")
        if world > 1:
            split_nccl = run_split_sequence(args, ctx, q38attn, torch, dist, rank, world, "nccl")

    prefill = lin_prefill = None
    if not args.no_prefill:
        prefill = run_prefill(args, ctx, q38attn, synth, torch, rank, world, dist)
        lin_prefill = run_linear_prefill(args, ctx, q38attn, torch, rank, world, dist)

    proj = None
    if not args.no_proj:
        proj = run_projection(args, ctx, q38attn, synth, torch, rank)

    # End-to-end through the host-pointer C-ABI calls.
    e2e = None
    if e2e_steps:
        host = []
        for p in pristine:
            h = torch.empty(total, dtype=torch.float32, pin_memory=True)
            h.copy_(p)
            host.append({k: v.numpy() for k, v in views(h).items()})
        outs_full = torch.empty(B, 6144, pin_memory=True).numpy()
        outs_lin = torch.empty(B, 6144, pin_memory=True).numpy()
        pos_host = torch.empty(B, dtype=torch.int32, pin_memory=True).numpy()
        base = ctx_pos + total_steps
        h2d = B * (12288 + 2048) * 4 + B * 4 + n_lin * B * (10240 + 6144 + 96) * 4
        d2h = B * (6144 + 1024) * 4 + n_lin * B * (6144 + 10240 + 96) * 4
        barrier()
        t0 = time.perf_counter()
        for s in range(e2e_steps):
            hv = host[s % 2]
            for i, l in enumerate(LINEAR_LAYERS):
                ctx.linear_decode_host(st, l, hv[f"qkv{i}"], hv[f"z{i}"], hv[f"beta{i}"],
                                       hv[f"alpha{i}"], outs_lin, stream=stream)
            pos_host[:] = base + s
            ctx.full_decode_host(st, FULL_LAYER, hv["qg"], hv["key"], hv["value"], pos_host,
                                 outs_full, stream=stream)
        e2e_s = time.perf_counter() - t0
        barrier()
        e2e = [e2e_s, h2d, d2h]

    # Max over ranks.
    vals = torch.tensor([ms, attn_ms, lin_ms, e2e[0] if e2e else 0.0,
                         prefill["ms"] if prefill else 0.0,
                         lin_prefill["ms"] if lin_prefill else 0.0,
                         split["ms"] if split else 0.0,
                         split_nccl["ms"] if split_nccl else 0.0],
                        device="cuda", dtype=torch.float64)
    if dist is not None:
        dist.all_reduce(vals, op=dist.ReduceOp.MAX)
    ms, attn_ms, lin_ms, e2e_s, prefill_ms, lin_prefill_ms, split_ms, split_nccl_ms = vals.tolist()

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu:
        cpu = cpu_baseline(args)
        if proj:
            proj["cpu_baseline"] = cpu_projection_baseline(args, sorted({1, args.batch}))

    if rank == 0:
        step_ms = ms / args.steps
        tokens = B * world
        mean_pos = ctx_pos + args.warmup + (args.steps - 1) / 2.0 + 1
        attn_bytes = B * attn_bytes_per_seq(int(round(mean_pos)))
        lin_bytes = n_lin * B * deltanet_bytes_per_seq()
        peak, peak_kind = load_peaks()
        achieved = attn_bytes / (attn_ms * 1e-3) / 1e9
        traffic = None
        prof = load_traffic_profile()
        if prof and prof.get("dram_bytes_per_kv_byte"):
            traffic = prof["dram_bytes_per_kv_byte"] * B * int(round(mean_pos)) * 4 * 256 * 2 * 2
        line = {
            "metric": METRIC, "value": tokens / (step_ms * 1e-3), "unit": "tok/s",
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": step_ms, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "f32 (bf16 KV cache)",
            "data": "synthetic (seeded; config distributions)",
            "config": workload_config(args),
            "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                         "frac": achieved / peak, "traffic": traffic,
                         "kernel": "full-attention decode op (prep + split-KV + merge)",
                         "algorithmic_bytes": attn_bytes, "launch_ms": attn_ms,
                         "peak_source": f"{peak_kind} hbm_gbs"},
            "deltanet": {"layers": n_lin, "ms_per_step": lin_ms,
                         "achieved_gbs": lin_bytes / (lin_ms * 1e-3) / 1e9,
                         "frac": lin_bytes / (lin_ms * 1e-3) / 1e9 / peak},
            "step_gbs": (attn_bytes + lin_bytes) / (step_ms * 1e-3) / 1e9,
            "gpu_launches": 9 * args.steps,  # decode timed region (prefill timed separately)
            "clocks": clocks.summary(),
        }
        tpeak, tpeak_kind = load_tensor_peak()
        if prefill:
            flops = prefill_flops(args.prefill_batch, args.prefill_len, args.prefill_base)
            tflops = flops / (prefill_ms * 1e-3) / 1e12
            line["prefill"] = {
                "workload": (f"config4: {args.prefill_batch} x {args.prefill_len}-token causal "
                             "prefill (the whole job)"
                             + (f" after {args.prefill_base} cached positions each"
                                if args.prefill_base else "")
                             + f", {args.prefill_kv} KV cache, 24Q/4KV x 256, RoPE 64, sigmoid gate; "
                             "QK^T bf16, PV f16, f32 accumulate (tcgen05); its "
                             f"{args.prefill_batch * 4} (sequence, KV-head group) units split "
                             f"over {world} GPU(s)"),
                "scaling": "strong", "ms": prefill_ms, "flops": flops, "tflops": tflops,
                "units_per_gpu": prefill["units"],
                # Per GPU: the whole job's rate over the ranks (slowest rank's time).
                "roofline": {"bound": "tensor", "achieved": tflops / world, "peak": tpeak,
                             "unit": "TFLOP/s", "frac": tflops / world / tpeak,
                             "peak_source": f"{tpeak_kind} bf16_tflops (burst)",
                             "kernel": "prep + attn_prefill_pair (one op), per GPU"},
                "clocks": prefill["clocks"],
            }
        if split:
            kv_bytes = args.split_context * 4 * 256 * 2 * 2
            line["split_sequence"] = {
                "workload": (f"config3 split-sequence: 1 sequence, {args.split_context} cached "
                             f"bf16 positions sharded over {world} GPU(s); per-shard partials "
                             "exchanged over peer memory inside the merge kernel "
                             "(q38_full_decode_split_p2p), LSE merge; the timed tokens "
                             "replayed as one CUDA graph"),
                "scaling": "strong", "ms_per_token": split_ms, "tok_s": 1e3 / split_ms,
                "kv_gbs": kv_bytes / (split_ms * 1e-3) / 1e9,
                "hbm_frac_per_gpu": kv_bytes / world / (split_ms * 1e-3) / 1e9 / peak,
            }
            if split_nccl:
                line["split_sequence"]["nccl_transport"] = {
                    "what": "the same step with an ncclAllGather between the shard kernels and "
                            "the merge (q38_full_decode_split), issued token by token",
                    "ms_per_token": split_nccl_ms, "tok_s": 1e3 / split_nccl_ms}
        if lin_prefill:
            flops = linear_prefill_flops(args.prefill_batch, args.prefill_len)
            toks = args.prefill_batch * args.prefill_len
            # Config 5's stated per-token traffic (~45 KB: q/k/v/z/gates in, output
            # out, f32) and the WY-form FLOPs; the path is mixed-bound, so both
            # fractions are reported.
            lp_bytes = toks * 45 * 1024
            line["deltanet_prefill"] = {
                "workload": (f"config5: {args.prefill_batch} x {args.prefill_len}-token chunked "
                             "Gated DeltaNet prefill (the whole job; C=64, 16K/48V x 128) from a "
                             "zero state, outputs + final f32 state; chunk-local WY products and "
                             "state pass on tcgen05 with bf16 hi/lo operand pairs (3 products, "
                             "~1e-5 of the per-token recurrence), TMA-tiled conv; the 48 value "
                             f"heads split over {world} GPU(s), q/k convolved on every GPU"),
                "scaling": "strong", "heads_per_gpu": lin_prefill["heads"],
                "ms": lin_prefill_ms, "tok_s": toks / (lin_prefill_ms * 1e-3),
                "flops": flops, "tflops": flops / (lin_prefill_ms * 1e-3) / 1e12,
                "roofline": {
                    "bound": "mixed",
                    "tensor_frac": flops / world / (lin_prefill_ms * 1e-3) / 1e12 / tpeak,
                    "hbm_frac": lp_bytes / world / (lin_prefill_ms * 1e-3) / 1e9 / peak,
                    "peak_tflops": tpeak, "peak_gbs": peak,
                },
                "clocks": lin_prefill["clocks"],
            }
        if proj:
            line["projection"] = {
                "workload": ("linear_attention projections per DeltaNet layer (quantize_q8_k, "
                             "attn_qkv 5120->10240 Q4_K, attn_gate 5120->6144 Q4_K, ssm_beta / "
                             "ssm_alpha 5120->48 Q8_0, quantize, ssm_out 6144->5120 Q6_K), "
                             f"{args.proj_layers} layers' weights, one CUDA graph"),
                **proj,
            }
        if e2e:
            line["e2e"] = {"value": tokens * e2e_steps / e2e_s, "unit": "tok/s",
                           "h2d_bytes_per_step": e2e[1], "d2h_bytes_per_step": e2e[2],
                           "steps": e2e_steps}
        if cpu:
            line["cpu_baseline"] = cpu
        print(json.dumps(line), flush=True)

    st.close()
    ctx.close()
    if dist is not None:
        dist.barrier()
        dist.destroy_process_group()


def main() -> None:
    args = parse_args()
    if args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()

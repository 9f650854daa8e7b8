"""GPU tests of split-sequence decode: one sequence's cached positions split
into contiguous shards, each shard's softmax partial computed by
q38_full_decode_shard, and the shards merged with q38_attn_merge_shards. On one
GPU the shards are separate states; with two or more GPUs the real NCCL path
runs: q38_full_decode_split (shard kernels, ncclAllGather inside the library on
a communicator from q38_nccl_comm_create, merge), driven by
q38attn.parallel.SplitSequenceDecoder with torch.distributed only exchanging
the NCCL id."""
from __future__ import annotations

import os
import subprocess
import sys

import numpy as np
import pytest

from conftest import REPO, check_parity, relative_error

pytestmark = pytest.mark.gpu
F = np.float32


@pytest.mark.parametrize("nshards,bf16", [(2, True), (3, False), (4, True)])
def test_shards_on_one_gpu_match_unsharded(cuda_ctx, oracle_lib, nshards, bf16):
    import torch

    import q38attn
    from q38attn import synth
    from q38attn.parallel import PARTIAL_FLOATS, position_ranges
    g = synth.rng(30 + nshards)
    w = synth.full_weights(g)
    layer, cap = 3, 3000
    cuda_ctx.bind_full_layer(layer, w["q_norm"], w["k_norm"])
    kvd = q38attn.Q38_KV_BF16 if bf16 else q38attn.Q38_KV_F32
    pre = 2500  # cached positions before the step
    k, v = synth.kv_rows(g, pre, bf16=bf16)
    ranges = position_ranges(cap, nshards)
    shards = []
    for p0, p1 in ranges:
        st = cuda_ctx.state(1, p1 - p0, full_slots=1, linear_slots=0, kv_dtype=kvd)
        n = max(0, min(p1, pre) - p0)
        if n:
            st.upload_kv(layer, 0, 0, np.ascontiguousarray(k[p0:p0 + n]),
                         np.ascontiguousarray(v[p0:p0 + n]))
        shards.append(st)
    full = cuda_ctx.state(1, cap, full_slots=1, linear_slots=0, kv_dtype=kvd)
    full.upload_kv(layer, 0, 0, k, v)
    kc = np.zeros((cap, 1024), F)
    vc = np.zeros((cap, 1024), F)
    kc[:pre], vc[:pre] = k, v
    for step in range(2):
        pos = pre + step
        x = synth.full_step(g, 1)
        qg = torch.from_numpy(x["q_and_gate"]).cuda()
        posd = torch.tensor([pos], dtype=torch.int32, device="cuda")
        parts = torch.empty(nshards, 1, 24, PARTIAL_FLOATS, device="cuda")
        for i, ((p0, p1), st) in enumerate(zip(ranges, shards)):
            key = torch.from_numpy(x["key"].copy()).cuda()
            val = torch.from_numpy(x["value"]).cuda()
            cuda_ctx.full_decode_shard(st, layer, qg, key, val, posd, parts[i],
                                       max_position=cap - 1, pos_offset=p0)
        merged = torch.empty(1, 6144, device="cuda")
        cuda_ctx.merge_shards(parts, qg, merged)
        ref = torch.empty(1, 6144, device="cuda")
        cuda_ctx.full_decode(full, layer, qg, torch.from_numpy(x["key"].copy()).cuda(),
                             torch.from_numpy(x["value"]).cuda(), posd, ref)
        torch.cuda.synchronize()
        assert relative_error(merged.cpu().numpy(), ref.cpu().numpy()) < 1e-5, step
        q = np.zeros(6144, F)
        gt = np.zeros(6144, F)
        sc = np.zeros(24 * cap, F)
        oo = np.zeros(6144, F)
        okey = x["key"][0].copy()
        assert oracle_lib.full_core(w, x["q_and_gate"][0], okey, x["value"][0], q, gt, sc, oo,
                                    kc, vc, cap, pos, layer, int(bf16)) == 0
        check_parity(merged[0].cpu().numpy(), oo, 1e-4, str(step))
    for st in shards:
        assert st.errors() == 0
        st.close()
    full.close()


@pytest.mark.parametrize("bf16", [True, False])
def test_split_p2p_single_rank_equals_decode(cuda_ctx, bf16):
    """The peer-memory exchange path with one rank (the kernel stores its own
    partial into its own buffer, raises its own flag and merges): bitwise the
    regular decode, over three calls (both epoch parities of the buffer). A
    single GPU never runs ranks that wait on one another; the multi-rank path
    is the two-GPU test below."""
    import torch

    import q38attn
    from q38attn import synth
    g = synth.rng(60 + int(bf16))
    w = synth.full_weights(g)
    layer, cap, pre, B = 3, 2048, 1500, 2
    cuda_ctx.bind_full_layer(layer, w["q_norm"], w["k_norm"])
    kvd = q38attn.Q38_KV_BF16 if bf16 else q38attn.Q38_KV_F32
    sts = [cuda_ctx.state(B, cap, full_slots=1, linear_slots=0, kv_dtype=kvd) for _ in range(2)]
    for b in range(B):
        k, v = synth.kv_rows(g, pre, bf16=bf16)
        for st in sts:
            st.upload_kv(layer, b, 0, k, v)
    handle = sts[1].split_p2p_handle(1)
    assert len(handle) == q38attn.Q38_IPC_HANDLE_BYTES
    sts[1].split_p2p_open(0, [handle])
    for step in range(3):
        x = synth.full_step(g, B)
        d = [{kk: torch.from_numpy(vv.copy()).cuda() for kk, vv in x.items()} for _ in range(2)]
        pos = torch.full((B,), pre + step, dtype=torch.int32, device="cuda")
        outs = [torch.empty(B, 6144, device="cuda") for _ in range(2)]
        cuda_ctx.full_decode(sts[0], layer, d[0]["q_and_gate"], d[0]["key"], d[0]["value"], pos,
                             outs[0], max_position=cap - 1)
        cuda_ctx.full_decode_split_p2p(sts[1], layer, d[1]["q_and_gate"], d[1]["key"],
                                       d[1]["value"], pos, outs[1], cap - 1, 0)
        torch.cuda.synchronize()
        assert torch.equal(outs[0], outs[1]), step
        assert torch.equal(d[0]["key"], d[1]["key"])
    for st in sts:
        assert st.errors() == 0
        st.close()


MGPU_SCRIPT = r'''
import os, sys, json, numpy as np, torch, torch.distributed as dist
sys.path.insert(0, os.path.join(os.environ["Q38_REPO"], "qwen3.8_27b_in_rust_b200"))
import q38attn
from q38attn import synth
from q38attn.parallel import SplitSequenceDecoder, position_ranges
rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
torch.cuda.set_device(rank)
import datetime
dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=60), device_id=torch.device("cuda", rank))
ctx = q38attn.Context(rank)
g = synth.rng(77); w = synth.full_weights(g)
layer, cap, pre = 3, 4096, 4000
ctx.bind_full_layer(layer, w["q_norm"], w["k_norm"])
k, v = synth.kv_rows(g, pre, bf16=True)
p0, p1 = position_ranges(cap, world)[rank]
decs = {}
for transport in ("nccl", "p2p"):
    st = ctx.state(1, p1 - p0, full_slots=1, linear_slots=0, kv_dtype=q38attn.Q38_KV_BF16)
    n = max(0, min(p1, pre) - p0)
    if n: st.upload_kv(layer, 0, 0, np.ascontiguousarray(k[p0:p0 + n]), np.ascontiguousarray(v[p0:p0 + n]))
    decs[transport] = (st, SplitSequenceDecoder(ctx, st, layer, p0, transport=transport))
full = ctx.state(1, cap, full_slots=1, linear_slots=0, kv_dtype=q38attn.Q38_KV_BF16)
full.upload_kv(layer, 0, 0, k, v)
err = {"nccl": 0.0, "p2p": 0.0}
for step in range(4):
    x = synth.full_step(g, 1)
    qg = torch.from_numpy(x["q_and_gate"]).cuda(); posd = torch.tensor([pre + step], dtype=torch.int32, device="cuda")
    ref = torch.empty(1, 6144, device="cuda")
    ctx.full_decode(full, layer, qg, torch.from_numpy(x["key"].copy()).cuda(), torch.from_numpy(x["value"]).cuda(), posd, ref)
    for transport, (st, dec) in decs.items():
        out = torch.empty(1, 6144, device="cuda")
        dec.step(qg, torch.from_numpy(x["key"].copy()).cuda(), torch.from_numpy(x["value"]).cuda(), posd, out, cap - 1)
        torch.cuda.synchronize()
        a, b = out.cpu().numpy(), ref.cpu().numpy()
        err[transport] = max(err[transport], float(np.max(np.abs(a - b) / np.maximum(np.abs(b), 1))))
for transport, (st, dec) in decs.items():
    assert st.errors() == 0, transport
errs = [None] * world
dist.all_gather_object(errs, err)
if rank == 0:
    print(json.dumps({"world": world, "max_err_nccl": max(e["nccl"] for e in errs),
                      "max_err_p2p": max(e["p2p"] for e in errs)}))
dist.barrier()
for transport, (st, dec) in decs.items():
    dec.close(); st.close()
full.close()
dist.barrier(); dist.destroy_process_group()
'''


def test_split_sequence_two_gpus(tmp_path):
    """Both transports of split-sequence decode on two GPUs, against the
    one-GPU decode of the whole sequence."""
    import torch
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    script = tmp_path / "split_seq.py"
    script.write_text(MGPU_SCRIPT)
    env = dict(os.environ, Q38_REPO=str(REPO), NCCL_NVLS_ENABLE="0")
    out = subprocess.run(
        ["timeout", "-k", "30", "240", sys.executable, "-m", "torch.distributed.run",
         "--nnodes=1", "--nproc-per-node=2", "--master-addr", "127.0.0.1",
         "--master-port", "29611", str(script)],
        capture_output=True, text=True, env=env)
    assert out.returncode == 0, out.stderr[-3000:]
    import json
    line = [l for l in out.stdout.splitlines() if l.startswith("{")][-1]
    res = json.loads(line)
    print(f"[split-sequence, 2 GPUs] {line}")
    from conftest import PARITY_LOG
    for t in ("nccl", "p2p"):
        PARITY_LOG.append({"test": "test_split_sequence_two_gpus", "what": f"world 2, {t} vs 1-GPU decode",
                           "ref_metric": res[f"max_err_{t}"], "scaled": None, "tol": 1e-5})
    assert res["world"] == 2
    assert res["max_err_nccl"] < 1e-5 and res["max_err_p2p"] < 1e-5

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
st = ctx.state(1, p1 - p0, full_slots=1, linear_slots=0, kv_dtype=q38attn.Q38_KV_BF16)
n = max(0, min(p1, pre) - p0)
if n: st.upload_kv(layer, 0, 0, np.ascontiguousarray(k[p0:p0 + n]), np.ascontiguousarray(v[p0:p0 + n]))
dec = SplitSequenceDecoder(ctx, st, layer, p0)
full = ctx.state(1, cap, full_slots=1, linear_slots=0, kv_dtype=q38attn.Q38_KV_BF16)
full.upload_kv(layer, 0, 0, k, v)
err = 0.0
for step in range(3):
    x = synth.full_step(g, 1)
    qg = torch.from_numpy(x["q_and_gate"]).cuda(); posd = torch.tensor([pre + step], dtype=torch.int32, device="cuda")
    out = torch.empty(1, 6144, device="cuda")
    dec.step(qg, torch.from_numpy(x["key"].copy()).cuda(), torch.from_numpy(x["value"]).cuda(), posd, out, cap - 1)
    ref = torch.empty(1, 6144, device="cuda")
    ctx.full_decode(full, layer, qg, torch.from_numpy(x["key"].copy()).cuda(), torch.from_numpy(x["value"]).cuda(), posd, ref)
    torch.cuda.synchronize()
    a, b = out.cpu().numpy(), ref.cpu().numpy()
    err = max(err, float(np.max(np.abs(a - b) / np.maximum(np.abs(b), 1))))
assert st.errors() == 0
errs = [None] * world
dist.all_gather_object(errs, err)
if rank == 0:
    print(json.dumps({"world": world, "max_err": max(errs), "path": "q38_full_decode_split (NCCL in the library)"}))
dec.close(); st.close(); full.close()
dist.barrier(); dist.destroy_process_group()
'''


def test_split_sequence_nccl_two_gpus(tmp_path):
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
    print(f"[nccl] {line}")
    from conftest import PARITY_LOG
    PARITY_LOG.append({"test": "test_split_sequence_nccl_two_gpus", "what": "world 2 vs 1-GPU decode",
                       "ref_metric": res["max_err"], "scaled": None, "tol": 1e-5})
    assert res["world"] == 2 and res["max_err"] < 1e-5

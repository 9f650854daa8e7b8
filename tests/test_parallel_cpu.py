"""CPU tests (gloo, world size 2) of the multi-GPU host logic: sequence and
position sharding and the split-sequence exchange + log-sum-exp merge, with the
per-shard softmax partials computed in numpy from the reference's attention
(src/model/ops.rs:884-919)."""
from __future__ import annotations

import os
import socket

import numpy as np
import pytest


def test_shard_ranges_cover_exactly():
    from q38attn.parallel import position_ranges, shard_range
    for total in (0, 1, 7, 32, 131072, 131073):
        for world in (1, 2, 3, 4, 8):
            rs = [shard_range(total, world, r) for r in range(world)]
            assert rs[0][0] == 0 and rs[-1][1] == total
            for (a, b), (c, d) in zip(rs, rs[1:]):
                assert b == c and b - a >= d - c >= b - a - 1
            assert position_ranges(total, world) == rs
    with pytest.raises(ValueError):
        shard_range(10, 2, 2)


def test_prefill_segments_cover_units_once():
    """Each rank's calls cover its contiguous range of (sequence, KV head)
    units exactly once; 16 units (config 4) over 1/2/4/8 GPUs give whole
    sequences or whole-sequence halves and quarters."""
    from q38attn.parallel import prefill_segments
    for nseq, kvh in ((4, 4), (3, 4), (1, 4), (5, 2)):
        for world in (1, 2, 3, 4, 5, 8):
            seen = []
            for rank in range(world):
                for s0, n, h0, nh in prefill_segments(nseq, kvh, world, rank):
                    assert n >= 1 and nh >= 1 and 0 <= h0 and h0 + nh <= kvh
                    assert n == 1 or (h0, nh) == (0, kvh)
                    seen += [(s, h) for s in range(s0, s0 + n) for h in range(h0, h0 + nh)]
            assert sorted(seen) == [(s, h) for s in range(nseq) for h in range(kvh)]
    assert prefill_segments(4, 4, 8, 3) == [(1, 1, 2, 2)]
    assert prefill_segments(4, 4, 2, 1) == [(2, 2, 0, 4)]


def _partial(q, K, V):
    """(o, m, l) of one head over rows K/V: the shard's softmax partial."""
    if K.shape[0] == 0:
        return np.zeros(256), -np.inf, 0.0
    s = (K.astype(np.float64) @ q.astype(np.float64)) / 16.0
    m = s.max()
    e = np.exp(s - m)
    return e @ V.astype(np.float64), m, e.sum()


def _merge(parts, gate):
    m = max(p[1] for p in parts)
    l = sum(np.exp(p[1] - m) * p[2] for p in parts if p[1] != -np.inf)
    o = sum(np.exp(p[1] - m) * p[0] for p in parts if p[1] != -np.inf)
    return o / l / (1 + np.exp(-gate))


def _worker(rank, world, port, result):
    import torch
    import torch.distributed as dist

    from q38attn.parallel import PARTIAL_FLOATS, position_ranges
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        g = np.random.default_rng(0)  # same data on every rank
        P, heads = 1000, 3
        K = g.standard_normal((P, 256)).astype(np.float32)
        V = g.standard_normal((P, 256)).astype(np.float32)
        q = g.standard_normal((heads, 256)).astype(np.float32)
        gate = g.standard_normal((heads, 256)).astype(np.float32)
        pos = 900  # attends to rows 0..900
        p0, p1 = position_ranges(P, world)[rank]
        hi = min(p1, pos + 1)
        local = np.zeros((heads, PARTIAL_FLOATS), np.float32)
        for h in range(heads):
            o, m, l = _partial(q[h], K[p0:hi], V[p0:hi])
            local[h, :256], local[h, 256], local[h, 257] = o, m, l
        gathered = torch.empty(world * heads, PARTIAL_FLOATS)  # concatenated along dim 0
        dist.all_gather_into_tensor(gathered, torch.from_numpy(local))
        parts = gathered.view(world, heads, PARTIAL_FLOATS).numpy()
        err = 0.0
        for h in range(heads):
            merged = _merge([(parts[r, h, :256], parts[r, h, 256], parts[r, h, 257])
                             for r in range(world)], gate[h])
            o, m, l = _partial(q[h], K[:pos + 1], V[:pos + 1])
            full = o / l / (1 + np.exp(-gate[h]))
            err = max(err, float(np.max(np.abs(merged - full))))
        result[rank] = err
    finally:
        dist.destroy_process_group()


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _id_worker(rank, world, port, result):
    import torch.distributed as dist

    from q38attn.parallel import exchange_unique_id
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        made = []

        def make():
            made.append(rank)
            return bytes(range(128))
        result[rank] = (exchange_unique_id(dist, make), made)
    finally:
        dist.destroy_process_group()


def _handle_worker(rank, world, port, result):
    import torch.distributed as dist

    from q38attn.parallel import exchange_handles
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        result[rank] = exchange_handles(dist, bytes([rank]) * 64)
    finally:
        dist.destroy_process_group()


def test_ipc_handle_exchange_gloo():
    """The peer-memory transport's set-up: every rank receives every rank's
    64-byte handle in rank order."""
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    manager = ctx.Manager()
    result = manager.dict()
    port = _free_port()
    procs = [ctx.Process(target=_handle_worker, args=(r, 2, port, result)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(120)
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    want = [bytes([0]) * 64, bytes([1]) * 64]
    assert result[0] == want and result[1] == want


def test_nccl_id_exchange_gloo():
    """The split-sequence decoder's set-up: rank 0 alone makes the NCCL id and
    every rank receives the same 128 bytes over the host's process group."""
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    manager = ctx.Manager()
    result = manager.dict()
    port = _free_port()
    procs = [ctx.Process(target=_id_worker, args=(r, 2, port, result)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(120)
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    assert result[0][0] == result[1][0] == bytes(range(128))
    assert result[0][1] == [0] and result[1][1] == []


@pytest.mark.parametrize("world", [2])
def test_split_sequence_exchange_gloo(world):
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    manager = ctx.Manager()
    result = manager.dict()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, result)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(120)
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    assert len(result) == world
    assert max(result.values()) < 1e-6

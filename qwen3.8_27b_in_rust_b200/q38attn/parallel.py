"""Multi-GPU partitioning of the hot path (one process per GPU).

Work is split only where it shards naturally:

* Sequence sharding (batched decode): every rank owns whole sequences; no
  data-path collective. `shard_range` gives a rank's share.
* Prefill attention: the unit is one (sequence, KV-head group) -- a KV head
  and its 6 query heads, the reference's per-head tasks grouped by
  kv_head = head / 6 (src/model/ops.rs:922-938, :877). `prefill_segments`
  turns a rank's contiguous range of units into q38_full_prefill_heads calls.
  No collective.
* DeltaNet prefill: the unit is one value head (ops.rs:717-733); q/k are
  replicated because value head h reads key head h % 16 (ops.rs:699).
  `shard_range(48, world, rank)` is a rank's head range for
  q38_linear_prefill_heads. No collective.
* Split-sequence decode (one long sequence): the sequence's cached positions
  are split into contiguous ranges, one per rank (`position_ranges`). Each
  rank computes softmax partials (o, m, l) over its range, the partials of
  all ranks are exchanged (24 x 258 floats per rank and sequence) and merged
  by log-sum-exp, inside one library call, so a host needs no framework for
  it. Two transports: "p2p" (q38_full_decode_split_p2p: the merge kernel
  stores its partial into every peer's buffer over NVLink and waits for
  theirs -- the exchange fused into the kernel), and "nccl"
  (q38_full_decode_split: one ncclAllGather between the shard kernels and the
  merge). This replaces the single position loop of full_core
  (src/model/ops.rs:884-913) across GPUs.
"""
from __future__ import annotations

PARTIAL_FLOATS = 256 + 2  # o[256], m, l


def shard_range(total: int, world: int, rank: int) -> tuple[int, int]:
    """Contiguous share [begin, end) of `total` units for `rank` of `world`
    (the first total % world ranks take one extra unit)."""
    if world <= 0 or not 0 <= rank < world or total < 0:
        raise ValueError("bad shard arguments")
    base, extra = divmod(total, world)
    begin = rank * base + min(rank, extra)
    return begin, begin + base + (1 if rank < extra else 0)


def position_ranges(capacity: int, world: int) -> list[tuple[int, int]]:
    """Per-rank global position ranges [p0, p1) of a sequence whose cache holds
    `capacity` positions: contiguous, equal up to one position."""
    return [shard_range(capacity, world, r) for r in range(world)]


def prefill_segments(nseq: int, kv_heads: int, world: int,
                     rank: int) -> list[tuple[int, int, int, int]]:
    """A rank's share of the nseq * kv_heads prefill units (sequence-major: unit
    u is sequence u // kv_heads, KV head u % kv_heads) as calls
    (seq0, nseq, kv_head0, kv_head_count): whole sequences in one call, a
    partial sequence at either end of the range in a call of its own."""
    u0, u1 = shard_range(nseq * kv_heads, world, rank)
    out: list[tuple[int, int, int, int]] = []
    u = u0
    while u < u1:
        s, h = divmod(u, kv_heads)
        if h == 0 and u1 - u >= kv_heads:
            n = (u1 - u) // kv_heads  # whole sequences
            out.append((s, n, 0, kv_heads))
            u += n * kv_heads
        else:
            n = min(kv_heads - h, u1 - u)
            out.append((s, 1, h, n))
            u += n
    return out


def exchange_unique_id(dist, make_id, group=None) -> bytes:
    """Rank 0's NCCL unique id on every rank of `group`, sent over the host's
    own process group (any backend)."""
    obj = [make_id() if dist.get_rank(group) == 0 else None]
    src = dist.get_global_rank(group, 0) if group is not None else 0
    dist.broadcast_object_list(obj, src=src, group=group)
    return obj[0]


def exchange_handles(dist, handle: bytes, group=None) -> list:
    """Every rank's IPC handle, in rank order, on every rank of `group`."""
    out = [None] * dist.get_world_size(group)
    dist.all_gather_object(out, handle, group=group)
    return out


class SplitSequenceDecoder:
    """Runs one full-attention decode step of sequences whose KV positions are
    sharded across the ranks of `group`. torch.distributed only carries the
    set-up bytes (the NCCL id or the IPC handles); the step's exchange is the
    library's.

    `state` on each rank holds positions [pos_offset, pos_offset + its
    context_length) of every sequence. transport: "p2p" (the exchange fused
    into the merge kernel over peer memory) or "nccl"."""

    def __init__(self, ctx, state, layer: int, pos_offset: int, group=None,
                 transport: str = "p2p"):
        import torch.distributed as dist

        import q38attn
        if transport not in ("p2p", "nccl"):
            raise ValueError("transport is 'p2p' or 'nccl'")
        self.ctx, self.state, self.layer = ctx, state, layer
        self.pos_offset = pos_offset
        self.transport = transport
        world = dist.get_world_size(group)
        rank = dist.get_rank(group)
        self.comm = None
        if transport == "nccl":
            uid = exchange_unique_id(dist, q38attn.nccl_unique_id, group)
            self.comm = q38attn.NcclComm(uid, world, rank, ctx.device)
            state.reserve_split(world)
        else:
            handles = exchange_handles(dist, state.split_p2p_handle(world), group)
            state.split_p2p_open(rank, handles)
            dist.barrier(group)  # every rank has mapped every buffer before the first step

    def step(self, q_and_gate, key, value, positions, attention, max_position: int,
             stream=None) -> None:
        """Every rank passes the same q_and_gate/key/value/positions (the
        token's projections); every rank receives the merged attention."""
        if self.transport == "nccl":
            self.ctx.full_decode_split(self.state, self.layer, q_and_gate, key, value,
                                       positions, attention, max_position, self.pos_offset,
                                       self.comm, stream=stream)
        else:
            self.ctx.full_decode_split_p2p(self.state, self.layer, q_and_gate, key, value,
                                           positions, attention, max_position, self.pos_offset,
                                           stream=stream)

    def close(self) -> None:
        if self.comm is not None:
            self.comm.close()
            self.comm = None

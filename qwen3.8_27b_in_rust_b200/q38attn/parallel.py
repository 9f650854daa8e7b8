"""Multi-GPU partitioning of the hot path (one process per GPU).

Two schemes, following where the work shards naturally:

* Sequence sharding (batched decode, prefill): every rank owns whole
  sequences; no data-path collective. `shard_range` gives a rank's share.
* Split-sequence decode (one long sequence): the sequence's cached positions
  are split into contiguous ranges, one per rank (`position_ranges`). Each
  rank computes softmax partials (o, m, l) over its range with
  q38_full_decode_shard, the partials of all ranks are exchanged with one
  all-gather over NCCL (24 x 258 floats per rank and sequence), and every rank
  merges them with q38_attn_merge_shards. This replaces the single position
  loop of full_core (src/model/ops.rs:884-913) across GPUs.
"""
from __future__ import annotations

from typing import Optional

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


class SplitSequenceDecoder:
    """Runs one full-attention decode step of sequences whose KV positions are
    sharded across the ranks of `group` (torch.distributed, NCCL backend).

    `state` on each rank holds positions [pos_offset, pos_offset + its
    context_length) of every sequence."""

    def __init__(self, ctx, state, layer: int, pos_offset: int, group=None,
                 batch: Optional[int] = None):
        import torch
        import torch.distributed as dist
        self.ctx, self.state, self.layer = ctx, state, layer
        self.pos_offset = pos_offset
        self.group = group
        self.dist = dist
        self.world = dist.get_world_size(group)
        b = batch or state.batch
        heads = 24
        self.local = torch.empty(b, heads, PARTIAL_FLOATS, device="cuda")
        # Concatenated along dim 0 ([world*b][heads][258]), viewed per rank.
        self.flat = torch.empty(self.world * b, heads, PARTIAL_FLOATS, device="cuda")
        self.gathered = self.flat.view(self.world, b, heads, PARTIAL_FLOATS)

    def step(self, q_and_gate, key, value, positions, attention, max_position: int,
             stream=None) -> None:
        """Every rank passes the same q_and_gate/key/value/positions (the
        token's projections); every rank receives the merged attention."""
        self.ctx.full_decode_shard(self.state, self.layer, q_and_gate, key, value, positions,
                                   self.local, max_position, self.pos_offset, stream=stream)
        self.dist.all_gather_into_tensor(self.flat, self.local, group=self.group)
        self.ctx.merge_shards(self.gathered, q_and_gate, attention, stream=stream)

"""Head sharding of the decode step across the GPUs of one node.

Attention heads are independent given the replicated hidden state, so rank g
owns a contiguous range of whole V blocks (and therefore of KV and query heads),
runs the decode kernels on its own latent cache, and one all-gather per layer
collects the per-head outputs (B, Hq/G, 128) into (G, B, Hq/G, 128) — the input
of ``o_proj`` after a reshape.  There is no other data exchange.

Failure handling is on the host: process groups are created with a timeout, a
partition check makes every rank agree on the head split before the first step
(a mismatch raises on every rank), and a rank that leaves or never joins turns
the next collective into an error within that timeout.
"""

from __future__ import annotations

import copy
import hashlib
import json
from datetime import timedelta
from typing import Optional

import torch
import torch.distributed as dist


def shard_range(spec, rank: int, world: int):
    """(first V block, end V block, first KV head, end KV head) of ``rank``: a
    contiguous range of whole V blocks.  Every rank must get the same number of
    query heads (the per-head outputs are gathered with one equal-sized
    all-gather), so V blocks covering different KV-head counts per rank are
    rejected."""
    nb = spec.num_v_blocks
    if world <= 0 or nb % world:
        raise ValueError(f"{nb} V blocks do not split evenly over {world} ranks")
    per = nb // world
    counts = {sum(spec.v_block_kv[r * per:(r + 1) * per]) for r in range(world)}
    if len(counts) != 1:
        raise ValueError(f"V blocks give the {world} ranks different KV-head counts {sorted(counts)}: "
                         "the equal-sized head all-gather needs equal shards")
    b0, b1 = rank * per, (rank + 1) * per
    return b0, b1, sum(spec.v_block_kv[:b0]), sum(spec.v_block_kv[:b1])


def shard_spec(spec, rank: int, world: int):
    """LayerSpec of the heads rank `rank` owns: a contiguous range of whole V blocks."""
    b0, b1, kv0, kv1 = shard_range(spec, rank, world)
    qpk = spec.num_q_heads // spec.num_kv_heads
    sub = copy.deepcopy(spec)
    sub.k_ranks = list(spec.k_ranks[kv0:kv1])
    sub.v_ranks = list(spec.v_ranks[b0:b1])
    sub.v_block_kv = list(spec.v_block_kv[b0:b1])
    sub.num_kv_heads = kv1 - kv0
    sub.num_q_heads = (kv1 - kv0) * qpk
    return sub


def head_range(spec, rank: int, world: int):
    """[first, last) query heads of `rank`."""
    sub = shard_spec(spec, rank, world)
    first = sum(shard_spec(spec, r, world).num_q_heads for r in range(rank))
    return first, first + sub.num_q_heads


def init(backend: str, timeout_s: float = 60.0, device_id: Optional[torch.device] = None):
    """torch.distributed process group from the torchrun environment, with a timeout."""
    kw = dict(backend=backend, timeout=timedelta(seconds=timeout_s))
    if device_id is not None:
        kw["device_id"] = device_id
    dist.init_process_group(**kw)


def _partition_digest(spec, world: int) -> int:
    d = json.dumps(dict(k=spec.k_ranks, v=spec.v_ranks, blocks=spec.v_block_kv, hq=spec.num_q_heads,
                        hkv=spec.num_kv_heads, world=world), sort_keys=True)
    return int(hashlib.sha256(d.encode()).hexdigest()[:12], 16)


def check_partition(spec, group=None, device=None):
    """Every rank must shard the same layer the same way; raises on all ranks otherwise."""
    world = dist.get_world_size(group)
    mine = torch.tensor([_partition_digest(spec, world)], dtype=torch.int64, device=device)
    alld = [torch.zeros_like(mine) for _ in range(world)]
    dist.all_gather(alld, mine, group=group)
    vals = {int(t.item()) for t in alld}
    if len(vals) != 1:
        raise RuntimeError(f"head partition mismatch across ranks ({len(vals)} different layer layouts)")


def gather_heads(out: torch.Tensor, group=None, buffer: Optional[torch.Tensor] = None) -> torch.Tensor:
    """All-gather the per-rank (B, Hq/G, 128) outputs into (B, Hq, 128), head order = rank order."""
    world = dist.get_world_size(group)
    if buffer is None:
        buffer = torch.empty((world * out.shape[0],) + tuple(out.shape[1:]), dtype=out.dtype, device=out.device)
    dist.all_gather_into_tensor(buffer, out.contiguous(), group=group)   # rank-major concatenation
    return buffer.view(world, *out.shape).permute(1, 0, 2, 3).reshape(out.shape[0], world * out.shape[1],
                                                                       out.shape[2])

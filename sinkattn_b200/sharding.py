"""Multi-GPU partitioning of the sink-attention path.

Every (batch, head) pair ("unit") of an attention call is independent: a
rank can run any subset of units with no communication. Two layouts use this:

* unit sharding (`partition_units`): ranks take disjoint sets of units of a
  job whose inputs they already hold; no data-path collective.
* Ulysses exchange (`sequence_to_units` / `units_to_sequence`): in a
  sequence-parallel DiT the activations arrive sharded by sequence
  ([B, S/P, H, D] per rank). One all-to-all turns them into full-sequence
  units ([U/P, S, D] per rank), the local kernel runs, and the inverse
  all-to-all restores the sequence layout. 12 heads do not divide over 8
  ranks, so (batch, head) units are the sharded dimension (2*12 = 24 units,
  3 per rank at P = 8); a unit count that does not divide is padded.

The reference is single-GPU (wanx/runtime/inference.py:65-69); this module is
the multi-GPU plumbing around its unchanged per-call semantics.
"""
from __future__ import annotations

import math
from typing import Callable, Optional, Sequence

import torch


def partition_units(n_units: int, world: int, rank: int,
                    weights: Optional[Sequence[float]] = None) -> list[int]:
    """Units of `rank` out of `n_units` split over `world` ranks.

    Without weights: contiguous, sizes differ by at most one (30 units on 8
    ranks -> 4,4,4,4,4,4,3,3). With weights (e.g. kept-block counts): longest
    processing time first, each unit to the currently lightest rank; ties go
    to the lower rank, so every rank computes the same assignment.
    """
    if world < 1 or not (0 <= rank < world):
        raise ValueError(f"bad rank {rank} for world {world}")
    if weights is None:
        base, extra = divmod(n_units, world)
        start = rank * base + min(rank, extra)
        return list(range(start, start + base + (1 if rank < extra else 0)))
    if len(weights) != n_units:
        raise ValueError("weights must have one entry per unit")
    loads = [0.0] * world
    owner = [0] * n_units
    for u in sorted(range(n_units), key=lambda i: (-float(weights[i]), i)):
        r = min(range(world), key=lambda i: (loads[i], i))
        owner[u] = r
        loads[r] += float(weights[u])
    return [u for u in range(n_units) if owner[u] == rank]


def units_per_rank(n_units: int, world: int) -> int:
    return math.ceil(n_units / world)


def sequence_to_units(x: torch.Tensor, group=None) -> torch.Tensor:
    """[B, S_r, H, D] sequence shard on every rank -> [n_per, S, D] units.

    Rank p receives units p*n_per .. (p+1)*n_per - 1 of the flattened (b, h)
    order (padded units are zero). All ranks must hold equal-length shards.
    """
    import torch.distributed as dist

    world = dist.get_world_size(group)
    B, Sr, H, D = x.shape
    U = B * H
    n_per = units_per_rank(U, world)
    # [B, S_r, H, D] -> [U, S_r, D] (unit-major), padded to world * n_per
    xu = x.permute(0, 2, 1, 3).reshape(U, Sr, D)
    if n_per * world != U:
        xu = torch.cat([xu, xu.new_zeros(n_per * world - U, Sr, D)], dim=0)
    send = xu.contiguous()  # chunk p = units of rank p
    recv = torch.empty_like(send)
    dist.all_to_all_single(recv, send, group=group)
    # recv chunk q = my units' sequence shard q -> concatenate along sequence
    return recv.view(world, n_per, Sr, D).permute(1, 0, 2, 3).reshape(n_per, world * Sr, D)


def units_to_sequence(y: torch.Tensor, B: int, H: int, group=None) -> torch.Tensor:
    """Inverse of sequence_to_units: [n_per, S, D] -> [B, S/P, H, D]."""
    import torch.distributed as dist

    world = dist.get_world_size(group)
    n_per, S, D = y.shape
    Sr = S // world
    send = y.view(n_per, world, Sr, D).permute(1, 0, 2, 3).contiguous()  # chunk q -> rank q
    recv = torch.empty_like(send)
    dist.all_to_all_single(recv, send, group=group)
    U = B * H
    xu = recv.reshape(world * n_per, Sr, D)[:U]
    return xu.view(B, H, Sr, D).permute(0, 2, 1, 3).contiguous()


def _local_units_attention(qu, ku, vu, mask_units, attn_fn):
    # qu/ku/vu: [n, S, D]; mask_units: [n, nq, nk] -> per unit a [1,1,S,D] call
    # batched as B=1, H=n so one kernel launch covers all local units.
    q = qu.unsqueeze(0)
    k = ku.unsqueeze(0)
    v = vu.unsqueeze(0)
    out, lse = attn_fn(q, k, v, mask_units.unsqueeze(0))
    return out[0], lse[0]


def ulysses_sink_attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor,
                           block_mask: torch.Tensor, group=None,
                           attn_fn: Optional[Callable] = None):
    """Sink attention on sequence-sharded inputs.

    q, k, v: [B, S/P, H, D] (this rank's sequence shard, the DiT layout);
    block_mask: bool [B or 1, H, nq, nk] over the full sequence (identical on
    every rank). Returns (out [B, S/P, H, D], lse [B, H, S/P] fp32).
    attn_fn(q, k, v, mask) -> (out, lse) on [1, n, S, D] tensors; defaults to
    the CUDA kernel (sinkattn_b200.ops.bsattn_fwd).
    """
    import torch.distributed as dist

    if attn_fn is None:
        from . import ops

        def attn_fn(qq, kk, vv, mm):
            return ops.bsattn_fwd(qq, kk, vv, mm)

    world = dist.get_world_size(group)
    rank = dist.get_rank(group)
    B, Sr, H, D = q.shape
    U = B * H
    n_per = units_per_rank(U, world)
    qu = sequence_to_units(q, group)
    ku = sequence_to_units(k, group)
    vu = sequence_to_units(v, group)
    # mask rows of my units (padded units get an all-true mask: their zero
    # inputs give finite, discarded results)
    m = block_mask.expand(B, H, *block_mask.shape[-2:]).reshape(U, *block_mask.shape[-2:])
    ids = [rank * n_per + i for i in range(n_per)]
    mu = torch.stack([m[i] if i < U else torch.ones_like(m[0]) for i in ids]).contiguous()
    ou, lu = _local_units_attention(qu, ku, vu, mu, attn_fn)
    out = units_to_sequence(ou.to(q.dtype), B, H, group)
    # LSE: [n_per, S] -> [B, H, S/P] through the same exchange (as a D=1 tensor)
    lse = units_to_sequence(lu.float().unsqueeze(-1), B, H, group)[..., 0].permute(0, 2, 1)
    return out, lse.contiguous()

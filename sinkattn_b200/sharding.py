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


def _unit_range(units, n_per):
    c0, c1 = (0, n_per) if units is None else units
    if not (0 <= c0 < c1 <= n_per):
        raise ValueError(f"unit range {units} outside 0..{n_per}")
    return c0, c1


def sequence_to_units(x: torch.Tensor, group=None, units=None) -> torch.Tensor:
    """[B, S_r, H, D] sequence shard on every rank -> [n, S, D] units.

    Rank p receives its units p*n_per + c0 .. p*n_per + c1 - 1 of the
    flattened (b, h) order, (c0, c1) = `units` (default: all n_per; padded
    units are zero). All ranks must hold equal-length shards and pass the
    same range.
    """
    import torch.distributed as dist

    world = dist.get_world_size(group)
    B, Sr, H, D = x.shape
    U = B * H
    n_per = units_per_rank(U, world)
    c0, c1 = _unit_range(units, n_per)
    # [B, S_r, H, D] -> [U, S_r, D] (unit-major), padded to world * n_per
    xu = x.permute(0, 2, 1, 3).reshape(U, Sr, D)
    if n_per * world != U:
        xu = torch.cat([xu, xu.new_zeros(n_per * world - U, Sr, D)], dim=0)
    send = xu.view(world, n_per, Sr, D)[:, c0:c1].contiguous()  # chunk p -> rank p
    recv = torch.empty_like(send)
    dist.all_to_all_single(recv, send, group=group)
    # recv chunk q = my units' sequence shard q -> concatenate along sequence
    n = c1 - c0
    return recv.permute(1, 0, 2, 3).reshape(n, world * Sr, D)


def units_to_sequence(y: torch.Tensor, B: int, H: int, group=None, units=None,
                      out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """Inverse of sequence_to_units: [n, S, D] units (c0, c1) of every rank ->
    their rows of the [B, S/P, H, D] sequence shard, written into `out` (made
    if None) and returned; rows of other units are left as they are."""
    import torch.distributed as dist

    world = dist.get_world_size(group)
    n, S, D = y.shape
    Sr = S // world
    U = B * H
    n_per = units_per_rank(U, world)
    c0, c1 = _unit_range(units, n_per)
    if c1 - c0 != n:
        raise ValueError(f"{n} units given for the range {units}")
    send = y.reshape(n, world, Sr, D).permute(1, 0, 2, 3).contiguous()  # chunk q -> rank q
    recv = torch.empty_like(send)
    dist.all_to_all_single(recv, send, group=group)
    if out is None:
        out = y.new_empty(B, Sr, H, D)
    outv = out.permute(0, 2, 1, 3)  # [B, H, S_r, D] view
    for p in range(world):
        u0, u1 = p * n_per + c0, min(p * n_per + c1, U)
        u = u0
        while u < u1:  # the range spans at most a few batch elements
            b, h = divmod(u, H)
            h1 = min(H, h + (u1 - u))
            outv[b, h:h1] = recv[p, u - u0:u - u0 + (h1 - h)]
            u += h1 - h
    return out


def _local_units_attention(qu, ku, vu, mask_units, attn_fn):
    # qu/ku/vu: [n, S, D]; mask_units: [n, nq, nk] -> per unit a [1,1,S,D] call
    # batched as B=1, H=n so one kernel launch covers all local units.
    q = qu.unsqueeze(0)
    k = ku.unsqueeze(0)
    v = vu.unsqueeze(0)
    out, lse = attn_fn(q, k, v, mask_units.unsqueeze(0))
    return out[0], lse[0]


_COMM_STREAMS: dict = {}


def _comm_stream(device) -> "torch.cuda.Stream":
    """One communication stream per device, kept for the process: the caching
    allocator keeps its blocks per stream, so a fresh stream per call would
    make every exchange buffer a new device allocation."""
    idx = torch.device(device).index
    if idx is None:
        idx = torch.cuda.current_device()
    if idx not in _COMM_STREAMS:
        _COMM_STREAMS[idx] = torch.cuda.Stream(idx)
    return _COMM_STREAMS[idx]


def ulysses_sink_attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor,
                           block_mask: torch.Tensor, group=None,
                           attn_fn: Optional[Callable] = None, chunks: int = 1):
    """Sink attention on sequence-sharded inputs.

    q, k, v: [B, S/P, H, D] (this rank's sequence shard, the DiT layout);
    block_mask: bool [B or 1, H, nq, nk] over the full sequence (identical on
    every rank). Returns (out [B, S/P, H, D], lse [B, H, S/P] fp32).
    attn_fn(q, k, v, mask) -> (out, lse) on [1, n, S, D] tensors; defaults to
    the CUDA kernel (sinkattn_b200.ops.bsattn_fwd).

    chunks > 1 splits each rank's units into that many groups. On CUDA
    tensors the input exchange of every group is issued first on a
    communication stream, the attention of group c runs on the current stream
    as soon as its inputs have arrived, and the output exchange of group c
    runs on the communication stream while group c+1 computes: the
    all-to-all traffic overlaps the kernel. Every rank must pass the same
    `chunks`.
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
    C = max(1, min(int(chunks), n_per))
    bounds = [(n_per * c // C, n_per * (c + 1) // C) for c in range(C)]
    # mask rows of my units (padded units get an all-true mask: their zero
    # inputs give finite, discarded results)
    m = block_mask.expand(B, H, *block_mask.shape[-2:]).reshape(U, *block_mask.shape[-2:])
    ids = [rank * n_per + i for i in range(n_per)]
    mu = torch.stack([m[i] if i < U else torch.ones_like(m[0]) for i in ids]).contiguous()
    out = q.new_empty(B, Sr, H, D)
    lse_seq = torch.empty(B, Sr, H, 1, dtype=torch.float32, device=q.device)
    overlap = q.is_cuda and C > 1
    if overlap:
        compute = torch.cuda.current_stream(q.device)
        comm = _comm_stream(q.device)
        comm.wait_stream(compute)
    inputs = []
    for c0, c1 in bounds:
        if overlap:
            with torch.cuda.stream(comm):
                t = [sequence_to_units(x, group, units=(c0, c1)) for x in (q, k, v)]
                ev = torch.cuda.Event()
                ev.record(comm)
            for x in t:
                x.record_stream(compute)
            inputs.append((t, ev))
        else:
            inputs.append(([sequence_to_units(x, group, units=(c0, c1)) for x in (q, k, v)], None))
    for (c0, c1), (t, ev) in zip(bounds, inputs):
        if overlap:
            compute.wait_event(ev)
        ou, lu = _local_units_attention(*t, mu[c0:c1], attn_fn)
        ou = ou.to(q.dtype)
        lu = lu.float().unsqueeze(-1)
        if overlap:
            done = torch.cuda.Event()
            done.record(compute)
            ou.record_stream(comm)
            lu.record_stream(comm)
            with torch.cuda.stream(comm):
                comm.wait_event(done)
                units_to_sequence(ou, B, H, group, units=(c0, c1), out=out)
                # LSE through the same exchange (as a D = 1 tensor)
                units_to_sequence(lu, B, H, group, units=(c0, c1), out=lse_seq)
        else:
            units_to_sequence(ou, B, H, group, units=(c0, c1), out=out)
            units_to_sequence(lu, B, H, group, units=(c0, c1), out=lse_seq)
    if overlap:
        compute.wait_stream(comm)
        out.record_stream(comm)
        lse_seq.record_stream(comm)
    return out, lse_seq[..., 0].permute(0, 2, 1).contiguous()

"""Multi-GPU partitioning of the sink-attention path.

Every (batch, head) pair ("unit") of an attention call is independent: a
rank can run any subset of units with no communication. Two layouts use this:

* unit sharding (`partition_units`): ranks take disjoint sets of units of a
  job whose inputs they already hold; no data-path collective.
* Ulysses exchange: in a sequence-parallel DiT the activations arrive
  sharded by sequence ([B, S/P, H, D] per rank). The exchange turns them
  into full-sequence units ([U/P, S, D] per rank), the local kernel runs,
  and the inverse exchange restores the sequence layout. 12 heads do not
  divide over 8 ranks, so (batch, head) units are the sharded dimension
  (2*12 = 24 units, 3 per rank at P = 8); a unit count that does not divide
  is padded. Two implementations:
  - UlyssesPeerExchange (CUDA): the dispatch and combine kernels
    (csrc/exchange.cu) write every row straight into the owner's buffer
    over NVLink peer memory, mapped once with CUDA IPC; no pack or unpack
    copies and no NCCL data traffic, three 4-byte all-reduces per call to
    order the ranks.
  - ulysses_sink_attention (`sequence_to_units` / `units_to_sequence`): the
    same exchange as torch.distributed all-to-alls, for any backend (the
    CPU tests run it over gloo).

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


def _device_view(ptr: int, nbytes: int, device) -> torch.Tensor:
    """A uint8 tensor over `nbytes` of device memory at `ptr` (memory this
    module allocated with sa_ipc_alloc; the tensor does not own it)."""

    class _Mem:
        pass

    m = _Mem()
    m.__cuda_array_interface__ = {"shape": (nbytes,), "typestr": "|u1", "data": (ptr, False),
                                  "version": 3, "strides": None}
    return torch.as_tensor(m, device=device)


class UlyssesPeerExchange:
    """Sink attention on sequence-sharded inputs with the exchange over NVLink
    peer memory.

    Made once per (B, S, H) on every rank of `group` (a collective call):
    each rank allocates two receive buffers [3, n_per, S, 128] (Q, K, V of its
    units; calls alternate between them), its output [B, S/P, H, 128] and
    LSE [B, H, S/P], and maps the peers' buffers with CUDA IPC. The n_per
    unit slots are split into `chunks` groups g (one by default). A call runs

        exchange stream:  dispatch(g) (Q, K, V rows -> owners); fence(g)
                          for every group in turn; then, as each group's
                          attention ends, combine(g) (output rows and LSE ->
                          sequence owners); a last fence
        attention stream: after fence(g), attention on group g's units (the
                          receive buffer as it lies)

    so the dispatch of group g+1 overlaps the attention of group g and the
    combine of group g the attention of group g+1. (At the Wan layer on two
    B200s, 12 units per rank, one group measured 1.63 ms and two 1.65 ms: the
    attention kernel's fixed cost per launch, ~0.05 ms, outweighs the hidden
    half-dispatch. Groups pay where a group's attention is long.) A fence is a 4-byte
    all-reduce: every rank is past the previous step, so a buffer is read only
    when every writer is done. The attention stream has the higher priority,
    and the exchange kernels run one 128-thread block beside an attention
    block on an SM. Both streams start after the caller's current stream, and
    the current stream waits for the last fence, so the call is ordered on
    the current stream like one kernel.
    A receive buffer is written again two calls later, after its owner's
    attention on it has passed the previous call's fences; an output is
    written after its owner has passed the first fence of the same call. The
    returned output and LSE are this object's buffers: valid until the next
    call, which overwrites them, so read them on the same stream before
    calling again.
    At most 8 ranks; D = 128; S divisible by the world size.
    """

    def __init__(self, B: int, S: int, H: int, D: int = 128, group=None, device=None,
                 chunks: int = 1):
        import ctypes

        import torch.distributed as dist

        from . import _lib

        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        if not 1 <= self.world <= 8:
            raise ValueError(f"UlyssesPeerExchange supports 1 to 8 ranks, got {self.world}")
        if D != 128 or S % self.world:
            raise ValueError(f"need D = 128 and S divisible by {self.world}; got D={D}, S={S}")
        self.B, self.S, self.H, self.D = B, S, H, D
        self.Sr = S // self.world
        self.n_per = units_per_rank(B * H, self.world)
        self.device = torch.device("cuda", torch.cuda.current_device()) if device is None \
            else torch.device(device)
        lib = _lib.load()
        self._lib = lib
        slot = 3 * self.n_per * S * D * 2
        sizes = {"recv": 2 * slot, "out": B * self.Sr * H * D * 2, "lse": B * H * self.Sr * 4}
        self._own: dict[str, int] = {}
        self._opened: list[int] = []
        handles = {}
        with torch.cuda.device(self.device):
            for name, nbytes in sizes.items():
                ptr = ctypes.c_void_p()
                _lib.check(lib.sa_ipc_alloc(nbytes, ctypes.byref(ptr)), "sa_ipc_alloc")
                self._own[name] = int(ptr.value)
                h = (ctypes.c_uint8 * 64)()
                _lib.check(lib.sa_ipc_get_handle(ptr, h), "sa_ipc_get_handle")
                handles[name] = bytes(h)
            views = {n: _device_view(p, sizes[n], self.device) for n, p in self._own.items()}
            for v in views.values():
                v.zero_()  # padding units read zeros
            self._recv2 = views["recv"].view(torch.bfloat16).view(2, 3, self.n_per, S, D)
            self._slot = 0
            self.out = views["out"].view(torch.bfloat16).view(B, self.Sr, H, D)
            self.lse = views["lse"].view(torch.float32).view(B, H, self.Sr)
            everyone = [None] * self.world
            dist.all_gather_object(everyone, handles, group=group)
            ptrs = {n: [0] * self.world for n in sizes}
            for r in range(self.world):
                for n in sizes:
                    if r == self.rank:
                        ptrs[n][r] = self._own[n]
                        continue
                    p = ctypes.c_void_p()
                    h = (ctypes.c_uint8 * 64).from_buffer_copy(everyone[r][n])
                    _lib.check(lib.sa_ipc_open_handle(h, ctypes.byref(p)), "sa_ipc_open_handle")
                    ptrs[n][r] = int(p.value)
                    self._opened.append(int(p.value))
            VP = ctypes.c_void_p * self.world
            self._recv_ptrs = [VP(*[q + k * slot for q in ptrs["recv"]]) for k in range(2)]
            self._out_ptrs = VP(*ptrs["out"])
            self._lse_ptrs = VP(*ptrs["lse"])
            self._attn_out = torch.empty(1, self.n_per, S, D, dtype=torch.bfloat16,
                                         device=self.device)
            self._attn_lse = torch.empty(1, self.n_per, S, dtype=torch.float32, device=self.device)
            self._flag = torch.zeros(1, device=self.device)
            self._masks: Optional[tuple] = None
            # exchange kernels and fences on one stream, attention on a
            # high-priority one: its blocks are placed first when both are ready
            self._xs = torch.cuda.Stream(device=self.device)
            self._as = torch.cuda.Stream(device=self.device, priority=-1)
            torch.cuda.synchronize(self.device)
        n = max(1, min(int(chunks), self.n_per))
        edges = [self.n_per * c // n for c in range(n + 1)]
        self._chunks = [(edges[c], edges[c + 1]) for c in range(n)]
        dist.barrier(group=group)

    def _fence(self):
        import torch.distributed as dist

        dist.all_reduce(self._flag, group=self.group)

    def unit_masks(self, block_mask: torch.Tensor) -> torch.Tensor:
        """This rank's units' rows of a [B or 1, H, nq, nk] mask, as the
        [1, n_per, nq, nk] mask its attention call takes (padding units all
        true)."""
        B, H, U = self.B, self.H, self.B * self.H
        m = block_mask.expand(B, H, *block_mask.shape[-2:]).reshape(U, *block_mask.shape[-2:])
        ids = [self.rank * self.n_per + i for i in range(self.n_per)]
        mu = torch.stack([m[i] if i < U else torch.ones_like(m[0]) for i in ids])
        return mu.unsqueeze(0).contiguous()

    def _unit_masks(self, block_mask: torch.Tensor) -> torch.Tensor:
        # cached for the last mask seen
        key = (block_mask.data_ptr(), tuple(block_mask.shape), block_mask._version)
        if self._masks is None or self._masks[0] != key:
            self._masks = (key, self.unit_masks(block_mask))
        return self._masks[1]

    def __call__(self, q: torch.Tensor, k: torch.Tensor, v: torch.Tensor,
                 block_mask: Optional[torch.Tensor] = None, unit_masks=None,
                 attn_fn: Optional[Callable] = None):
        """q, k, v: [B, S/P, H, 128] bf16 (this rank's shard, any strides with
        stride(-1) == 1); block_mask: bool [B or 1, H, nq, nk] over the full
        sequence, the same on every rank, or unit_masks (from unit_masks()).
        attn_fn(q, k, v, mask, out) runs the attention of one group of the
        rank's units ([1, n, S, 128] views, mask [1, n, nq, nk]) into `out`
        and returns the LSE [1, n, S] fp32 or None, on the current stream
        (the exchange's attention stream while it runs); by default the sink
        attention kernel. Returns (out [B, S/P, H, 128] bf16, lse [B, H, S/P]
        fp32 or None), this object's buffers."""
        import ctypes

        from . import _lib, ops

        shape = (self.B, self.Sr, self.H, self.D)
        for x in (q, k, v):
            if tuple(x.shape) != shape or x.dtype != torch.bfloat16 or x.device != self.device:
                raise ValueError(f"expected bf16 {shape} on {self.device}, got "
                                 f"{x.dtype} {tuple(x.shape)} on {x.device}")
        mu = unit_masks if unit_masks is not None else self._unit_masks(block_mask)
        cur = torch.cuda.current_stream(self.device)
        xs, ast = self._xs, self._as
        xs.wait_stream(cur)
        ast.wait_stream(cur)
        src = (ctypes.c_void_p * 3)(q.data_ptr(), k.data_ptr(), v.data_ptr())
        st = (ctypes.c_int64 * 12)(*q.stride(), *k.stride(), *v.stride())
        k_ = self._slot
        self._slot ^= 1
        r = self._recv2[k_]
        S = self.S
        done = []
        lses = []
        for j0, j1 in self._chunks:
            with torch.cuda.stream(xs):
                _lib.check(self._lib.sa_ulysses_dispatch_units(
                    3, src, st, self.B, self.Sr, self.H, self.D, self.world, self.rank,
                    self.n_per, j0, j1, self._recv_ptrs[k_], ctypes.c_void_p(xs.cuda_stream)),
                    "sa_ulysses_dispatch_units")
                self._fence()
                arrived = torch.cuda.Event()
                arrived.record(xs)
            with torch.cuda.stream(ast):
                ast.wait_event(arrived)
                qc, kc, vc = (r[t, j0:j1].unsqueeze(0) for t in range(3))
                out_c = self._attn_out[:, j0:j1]
                if attn_fn is None:
                    ops.bsattn_fwd(qc, kc, vc, mu[:, j0:j1], out=out_c,
                                   lse=self._attn_lse[:, j0:j1])
                    lse_c = self._attn_lse[:, j0:j1]
                else:
                    lse_c = attn_fn(qc, kc, vc, mu[:, j0:j1], out_c)
                    if lse_c is not None:
                        if (tuple(lse_c.shape) != (1, j1 - j0, S) or
                                lse_c.dtype != torch.float32):
                            raise ValueError(
                                f"attn_fn must return an fp32 [1, {j1 - j0}, {S}] LSE or None")
                        if lse_c.data_ptr() != self._attn_lse[:, j0:j1].data_ptr():
                            self._attn_lse[:, j0:j1].copy_(lse_c)
                finished = torch.cuda.Event()
                finished.record(ast)
            done.append(finished)
            lses.append(lse_c is not None)
        if any(lses) and not all(lses):
            raise ValueError("attn_fn returned an LSE for some unit groups and None for others")
        has_lse = all(lses)
        with torch.cuda.stream(xs):
            for (j0, j1), finished in zip(self._chunks, done):
                xs.wait_event(finished)
                _lib.check(self._lib.sa_ulysses_combine_units(
                    self._attn_out.data_ptr(), self._attn_lse.data_ptr() if has_lse else None,
                    self.B, self.Sr, self.H, self.D, self.world, self.rank, self.n_per, j0, j1,
                    self._out_ptrs, self._lse_ptrs if has_lse else None,
                    ctypes.c_void_p(xs.cuda_stream)), "sa_ulysses_combine_units")
            self._fence()
        cur.wait_stream(xs)
        lse = self.lse if has_lse else None
        return self.out, lse

    def close(self):
        """Unmaps the peers' buffers and frees this rank's (a collective call:
        every rank must be done with every buffer first)."""
        import torch.distributed as dist

        if not self._own:
            return
        torch.cuda.synchronize(self.device)
        dist.barrier(group=self.group)
        with torch.cuda.device(self.device):
            for p in self._opened:
                self._lib.sa_ipc_close(p)
            self._opened = []
            torch.cuda.synchronize(self.device)
        dist.barrier(group=self.group)
        with torch.cuda.device(self.device):
            self._recv2 = self.out = self.lse = None
            for p in self._own.values():
                self._lib.sa_ipc_free(p)
        self._own = {}

"""The Ulysses dispatch and combine kernels (csrc/exchange.cu) on one GPU.

The kernels write into whatever device addresses they are given: for a
real exchange those are the peers' buffers mapped with CUDA IPC; here every
simulated rank's buffers are ordinary allocations on the one GPU, and the
kernel is called once per simulated rank, one after the other. That checks
every index the kernels compute against the layout written out with torch:
  dispatch: rank p's shard row (b, s, h) -> owner of unit u = b*H + h, at
            [t, u % n_per, p*Sr + s];
  combine:  owner r's unit row (j, s) -> rank s // Sr, at [b, s % Sr, h]
            (output) and [b, h, s % Sr] (LSE); padding units are skipped.
Shard lengths that are not a multiple of 4 (63, 21) take the combine's
one-value-per-store LSE path; the others move the LSE four rows per store.
The exchange across real GPUs is in test_gpu_multi.py.
"""
from __future__ import annotations

import ctypes

import pytest
import torch

pytestmark = pytest.mark.gpu


def _stream():
    return ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)


@pytest.mark.parametrize("B,H,P,Sr", [(2, 3, 3, 64), (1, 5, 2, 100), (2, 12, 8, 32),
                                      (2, 12, 8, 63)])
@pytest.mark.parametrize("narrow", [False, True])
def test_dispatch_and_combine_layouts(B, H, P, Sr, narrow):
    """narrow: V rows 272 bytes apart and the unit outputs 16 bytes off a
    32-byte boundary, so that the kernels take their 16-byte path; otherwise
    every address allows 32-byte pieces."""
    from sinkattn_b200 import _lib

    lib = _lib.load()
    D = 128
    U = B * H
    n_per = -(-U // P)
    S = P * Sr
    g = torch.Generator(device="cuda").manual_seed(B * 100 + H * 10 + P)
    # each rank's Q, K, V shards; K as a strided view (H padded to H + 1)
    shards = []
    for p in range(P):
        q = torch.randn(B, Sr, H, D, device="cuda", generator=g).bfloat16()
        k = torch.randn(B, Sr, H + 1, D, device="cuda", generator=g).bfloat16()[:, :, :H]
        pad = 8 if narrow else 0
        v = torch.randn(B, Sr, H, D + pad, device="cuda", generator=g).bfloat16()[..., :D]
        shards.append((q, k, v))
    recv = [torch.zeros(3, n_per, S, D, dtype=torch.bfloat16, device="cuda") for _ in range(P)]
    dst = (ctypes.c_void_p * P)(*[r.data_ptr() for r in recv])
    for p, (q, k, v) in enumerate(shards):
        src = (ctypes.c_void_p * 3)(q.data_ptr(), k.data_ptr(), v.data_ptr())
        st = (ctypes.c_int64 * 12)(*q.stride(), *k.stride(), *v.stride())
        _lib.check(lib.sa_ulysses_dispatch(3, src, st, B, Sr, H, D, P, p, n_per, dst, _stream()),
                   "sa_ulysses_dispatch")
    torch.cuda.synchronize()
    for t in range(3):
        full = torch.cat([shards[p][t] for p in range(P)], dim=1)  # [B, S, H, D]
        for u in range(U):
            b, h = divmod(u, H)
            r, j = divmod(u, n_per)
            assert torch.equal(recv[r][t, j], full[b, :, h]), (t, u)
    # padding units were not written
    for r in range(P):
        for j in range(n_per):
            if r * n_per + j >= U:
                assert not recv[r][:, j].any()

    off = 8 if narrow else 0  # bf16 elements: 16 bytes
    outs = [torch.randn(n_per * S * D + off, device="cuda", generator=g).bfloat16()[off:]
            .view(n_per, S, D) for _ in range(P)]
    lses = [torch.randn(n_per, S, device="cuda", generator=g) for _ in range(P)]
    out_dst = [torch.zeros(B, Sr, H, D, dtype=torch.bfloat16, device="cuda") for _ in range(P)]
    lse_dst = [torch.zeros(B, H, Sr, device="cuda") for _ in range(P)]
    od = (ctypes.c_void_p * P)(*[o.data_ptr() for o in out_dst])
    ld = (ctypes.c_void_p * P)(*[o.data_ptr() for o in lse_dst])
    for r in range(P):
        _lib.check(lib.sa_ulysses_combine(outs[r].data_ptr(), lses[r].data_ptr(), B, Sr, H, D, P,
                                          r, n_per, od, ld, _stream()), "sa_ulysses_combine")
    torch.cuda.synchronize()
    for u in range(U):
        b, h = divmod(u, H)
        r, j = divmod(u, n_per)
        for p in range(P):
            assert torch.equal(out_dst[p][b, :, h], outs[r][j, p * Sr:(p + 1) * Sr]), (u, p)
            assert torch.equal(lse_dst[p][b, h], lses[r][j, p * Sr:(p + 1) * Sr]), (u, p)


@pytest.mark.parametrize("B,H,P,Sr,groups", [(2, 3, 3, 64, 2), (2, 12, 2, 48, 3),
                                             (1, 5, 2, 100, 2), (2, 3, 3, 21, 2)])
def test_unit_groups_cover_the_whole_exchange(B, H, P, Sr, groups):
    """Dispatch and combine run group by group over the unit slots (the
    pipelined exchange) write exactly what the whole-range calls write."""
    from sinkattn_b200 import _lib

    lib = _lib.load()
    D = 128
    n_per = -(-(B * H) // P)
    S = P * Sr
    edges = [n_per * c // groups for c in range(groups + 1)]
    g = torch.Generator(device="cuda").manual_seed(7 * B + H + P)
    shards = [tuple(torch.randn(B, Sr, H, D, device="cuda", generator=g).bfloat16()
                    for _ in range(3)) for _ in range(P)]

    def run(ranges):
        recv = [torch.zeros(3, n_per, S, D, dtype=torch.bfloat16, device="cuda")
                for _ in range(P)]
        dst = (ctypes.c_void_p * P)(*[r.data_ptr() for r in recv])
        for p, (q, k, v) in enumerate(shards):
            src = (ctypes.c_void_p * 3)(q.data_ptr(), k.data_ptr(), v.data_ptr())
            st = (ctypes.c_int64 * 12)(*q.stride(), *k.stride(), *v.stride())
            for j0, j1 in ranges:
                _lib.check(lib.sa_ulysses_dispatch_units(3, src, st, B, Sr, H, D, P, p, n_per,
                                                         j0, j1, dst, _stream()),
                           "sa_ulysses_dispatch_units")
        out_dst = [torch.zeros(B, Sr, H, D, dtype=torch.bfloat16, device="cuda")
                   for _ in range(P)]
        lse_dst = [torch.zeros(B, H, Sr, device="cuda") for _ in range(P)]
        od = (ctypes.c_void_p * P)(*[o.data_ptr() for o in out_dst])
        ld = (ctypes.c_void_p * P)(*[o.data_ptr() for o in lse_dst])
        for r in range(P):
            out = recv[r][0].contiguous()  # any [n_per, S, D] data will do
            lse = recv[r][1, :, :, 0].float().contiguous()
            for j0, j1 in ranges:
                _lib.check(lib.sa_ulysses_combine_units(out.data_ptr(), lse.data_ptr(), B, Sr, H,
                                                        D, P, r, n_per, j0, j1, od, ld,
                                                        _stream()),
                           "sa_ulysses_combine_units")
        torch.cuda.synchronize()
        return recv, out_dst, lse_dst

    whole = run([(0, n_per)])
    parts = run([(edges[c], edges[c + 1]) for c in range(groups)])
    for a, b in zip(whole, parts):
        for x, y in zip(a, b):
            assert torch.equal(x, y)

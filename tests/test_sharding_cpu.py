"""Multi-rank logic on CPU: unit partitioning and the Ulysses exchange, run
as gloo ranks (world sizes 2, 4 and 8; at 8 the 6 units are padded to 8, so
two ranks hold only padding). The local attention of each rank is the CPU
oracle here (the product path runs the CUDA kernel). A rank that leaves
between steps makes the other rank's next exchange raise."""
from __future__ import annotations

import datetime
import os
import socket
import sys
import time
from pathlib import Path

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

ROOT = Path(__file__).resolve().parent.parent


def test_partition_units_contiguous_and_balanced():
    from sinkattn_b200.sharding import partition_units

    for n, world in [(24, 8), (30, 8), (24, 1), (5, 8), (30, 4)]:
        parts = [partition_units(n, world, r) for r in range(world)]
        flat = [u for p in parts for u in p]
        assert flat == list(range(n))
        sizes = [len(p) for p in parts]
        assert max(sizes) - min(sizes) <= 1
    assert [len(partition_units(30, 8, r)) for r in range(8)] == [4, 4, 4, 4, 4, 4, 3, 3]


def test_partition_units_weighted_lpt():
    from sinkattn_b200.sharding import partition_units

    w = [10, 1, 1, 1, 9, 2, 2, 8]
    parts = [partition_units(len(w), 3, r, weights=w) for r in range(3)]
    assert sorted(u for p in parts for u in p) == list(range(len(w)))
    loads = [sum(w[u] for u in p) for p in parts]
    assert max(loads) - min(loads) <= max(w)
    with pytest.raises(ValueError):
        partition_units(4, 2, 2)


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _oracle_attn(q, k, v, m):
    sys.path.insert(0, str(ROOT))
    from oracle import sinkattn_oracle as orc

    out, lse = orc.dense_masked_attention(q.float().numpy(), k.float().numpy(),
                                          v.float().numpy(), m.numpy())
    return torch.from_numpy(out), torch.from_numpy(lse)


def _worker(rank, world, port, result_dir):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    sys.path.insert(0, str(ROOT))
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60))
    try:
        from sinkattn_b200.sharding import sequence_to_units, ulysses_sink_attention, units_to_sequence

        g = torch.Generator().manual_seed(7)
        B, S, H, D = 2, 512, 3, 16
        q = torch.randn(B, S, H, D, generator=g)
        k = torch.randn(B, S, H, D, generator=g)
        v = torch.randn(B, S, H, D, generator=g)
        mask = torch.rand(B, H, 4, 4, generator=g) < 0.6
        mask[..., 0] = True
        Sr = S // world
        sl = slice(rank * Sr, (rank + 1) * Sr)
        # the exchange round-trips
        u = sequence_to_units(q[:, sl].contiguous())
        back = units_to_sequence(u, B, H)
        assert torch.equal(back, q[:, sl])
        # sub-ranges of each rank's units round-trip into a shared output
        n_per = -(-(B * H) // world)
        part = torch.zeros_like(q[:, sl])
        for c0, c1 in ((0, 1), (1, n_per)) if n_per > 1 else ((0, 1),):
            units_to_sequence(sequence_to_units(q[:, sl].contiguous(), units=(c0, c1)), B, H,
                              units=(c0, c1), out=part)
        assert torch.equal(part, q[:, sl])
        out, lse = ulysses_sink_attention(q[:, sl].contiguous(), k[:, sl].contiguous(),
                                          v[:, sl].contiguous(), mask, attn_fn=_oracle_attn)
        # grouped exchange (the overlapped form on GPUs) gives the same result
        for chunks in (2, 3):
            o2, l2 = ulysses_sink_attention(q[:, sl].contiguous(), k[:, sl].contiguous(),
                                            v[:, sl].contiguous(), mask, attn_fn=_oracle_attn,
                                            chunks=chunks)
            assert torch.equal(o2, out) and torch.equal(l2, lse), chunks
        np.save(os.path.join(result_dir, f"out{rank}.npy"), out.numpy())
        np.save(os.path.join(result_dir, f"lse{rank}.npy"), lse.numpy())
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 4, 8])
def test_ulysses_exchange_matches_full_attention(tmp_path, world, oracle):
    port = _free_port()
    mp.start_processes(_worker, args=(world, port, str(tmp_path)), nprocs=world, join=True,
                       start_method="spawn")
    g = torch.Generator().manual_seed(7)
    B, S, H, D = 2, 512, 3, 16
    q = torch.randn(B, S, H, D, generator=g)
    k = torch.randn(B, S, H, D, generator=g)
    v = torch.randn(B, S, H, D, generator=g)
    mask = torch.rand(B, H, 4, 4, generator=g) < 0.6
    mask[..., 0] = True
    ref, ref_lse = oracle.dense_masked_attention(q.permute(0, 2, 1, 3).numpy(),
                                                 k.permute(0, 2, 1, 3).numpy(),
                                                 v.permute(0, 2, 1, 3).numpy(), mask.numpy())
    Sr = S // world
    for r in range(world):
        out = np.load(tmp_path / f"out{r}.npy")
        lse = np.load(tmp_path / f"lse{r}.npy")
        np.testing.assert_allclose(out, ref.transpose(0, 2, 1, 3)[:, r * Sr:(r + 1) * Sr],
                                   atol=1e-5, rtol=1e-5)
        np.testing.assert_allclose(lse, ref_lse[:, :, r * Sr:(r + 1) * Sr], atol=1e-5)


def test_unit_range_checks():
    """Unit sub-ranges of the Ulysses exchange must lie inside 0..n_per and the
    output exchange must be given as many units as the range holds."""
    from sinkattn_b200.sharding import _unit_range

    assert _unit_range(None, 3) == (0, 3)
    assert _unit_range((1, 3), 3) == (1, 3)
    for bad in ((0, 0), (2, 1), (-1, 2), (0, 4)):
        with pytest.raises(ValueError):
            _unit_range(bad, 3)


def _leaving_worker(rank, world, port, result_dir):
    """Rank 1 leaves between steps (after the first exchange, before the
    second); rank 0 must see its next exchange end with an error, not hang."""
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    sys.path.insert(0, str(ROOT))
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=10))
    from sinkattn_b200.sharding import sequence_to_units

    x = torch.randn(2, 64, 3, 16)
    sequence_to_units(x)  # one full step together
    if rank == 1:
        os._exit(0)  # leaves without joining the next exchange
    t0 = time.monotonic()
    try:
        sequence_to_units(x)
        outcome = "no error"
    except Exception as exc:  # the backend's own error type
        outcome = f"error: {type(exc).__name__}"
    with open(os.path.join(result_dir, "rank0.txt"), "w") as f:
        f.write(f"{outcome}\n{time.monotonic() - t0:.1f}\n")
    os._exit(0)  # the group is broken; skip its teardown


@pytest.mark.timeout(120)
def test_exchange_errors_when_a_rank_leaves(tmp_path):
    """Failure detection on the host: a rank that leaves between steps makes
    the other rank's next all-to-all raise (peer closed or the group's 10 s
    timeout) instead of waiting forever."""
    port = _free_port()
    mp.start_processes(_leaving_worker, args=(2, port, str(tmp_path)), nprocs=2, join=True,
                       start_method="spawn")
    outcome, seconds = (tmp_path / "rank0.txt").read_text().split("\n")[:2]
    assert outcome.startswith("error"), outcome
    assert float(seconds) < 60


def test_bench_unit_segments_cover_each_unit_once():
    """bench.py's strong-scaling split: for every world size the rank's units
    become (b0, b1, h0, h1) rectangles that cover each of its units once,
    span whole batch elements or lie inside one, and give views whose LSE
    slice stays contiguous (the kernel's LSE has no strides)."""
    import bench
    from sinkattn_b200.sharding import partition_units

    B, H, S = 2, 12, 256
    lse = torch.empty(B, H, S)
    out = torch.empty(B, S, H, 128).permute(0, 2, 1, 3)
    for world in (1, 2, 3, 4, 5, 8):
        seen = []
        for rank in range(world):
            units = partition_units(B * H, world, rank)
            segs = bench.unit_segments(units, H)
            got = []
            for b0, b1, h0, h1 in segs:
                assert b1 - b0 == 1 or (h0, h1) == (0, H)
                got += [b * H + h for b in range(b0, b1) for h in range(h0, h1)]
                sl = (slice(b0, b1), slice(h0, h1))
                assert lse[sl].is_contiguous()
                o = out[sl]
                assert o.stride() == out.stride()
                assert o.data_ptr() == out[b0, h0].data_ptr()
            assert got == units
            seen += got
        assert sorted(seen) == list(range(B * H))
    assert bench.unit_segments(list(range(24)), 12) == [(0, 2, 0, 12)]
    assert bench.unit_segments(list(range(9, 15)), 12) == [(0, 1, 9, 12), (1, 2, 0, 3)]

"""Two-GPU checks (skipped with fewer than 2 GPUs): the Ulysses exchange
around the CUDA kernel, over NCCL all-to-alls and over NVLink peer memory,
equals the single-GPU result, and unit sharding covers a job exactly."""
from __future__ import annotations

import datetime
import os
import socket
import sys
from pathlib import Path

import pytest
import torch

ROOT = Path(__file__).resolve().parent.parent

pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")]


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, result_dir):
    import torch.distributed as dist

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    sys.path.insert(0, str(ROOT))
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=120),
                            device_id=torch.device("cuda", rank))
    try:
        from sinkattn_b200.sharding import ulysses_sink_attention

        g = torch.Generator().manual_seed(11)
        B, S, H, D = 2, 1024, 3, 128
        q = torch.randn(B, S, H, D, generator=g).bfloat16()
        k = torch.randn(B, S, H, D, generator=g).bfloat16()
        v = torch.randn(B, S, H, D, generator=g).bfloat16()
        mask = torch.rand(B, H, 8, 8, generator=g) < 0.4
        mask[..., 0] = True
        Sr = S // world
        sl = slice(rank * Sr, (rank + 1) * Sr)
        dev = torch.device("cuda", rank)
        qs, ks, vs = (x[:, sl].to(dev).contiguous() for x in (q, k, v))
        out, lse = ulysses_sink_attention(qs, ks, vs, mask.to(dev))
        # grouped exchange overlapped with the kernel on a second stream
        out3, lse3 = ulysses_sink_attention(qs, ks, vs, mask.to(dev), chunks=3)
        torch.cuda.synchronize()
        assert torch.equal(out3, out) and torch.equal(lse3, lse)
        # the same exchange over NVLink peer memory (dispatch / combine
        # kernels into CUDA-IPC-mapped buffers), twice on the same buffers
        from sinkattn_b200.sharding import UlyssesPeerExchange

        # one unit group, then two and three groups (each group's exchange
        # overlapped with another group's attention on a second stream)
        for chunks in (1, 2, 3):
            ex = UlyssesPeerExchange(B, S, H, device=dev, chunks=chunks)
            for _ in range(2):
                out_p, lse_p = ex(qs, ks, vs, mask.to(dev))
                torch.cuda.synchronize()
                assert torch.equal(out_p, out) and torch.equal(lse_p, lse), chunks
            ex.close()
        torch.save({"out": out.cpu(), "lse": lse.cpu()}, os.path.join(result_dir, f"r{rank}.pt"))
        dist.barrier()
    finally:
        dist.destroy_process_group()


def test_ulysses_two_gpus_matches_single_gpu(tmp_path):
    import torch.multiprocessing as mp

    from sinkattn_b200 import ops

    world = 2
    mp.start_processes(_worker, args=(world, _free_port(), str(tmp_path)), nprocs=world,
                       join=True, start_method="spawn")
    g = torch.Generator().manual_seed(11)
    B, S, H, D = 2, 1024, 3, 128
    q = torch.randn(B, S, H, D, generator=g).bfloat16().cuda()
    k = torch.randn(B, S, H, D, generator=g).bfloat16().cuda()
    v = torch.randn(B, S, H, D, generator=g).bfloat16().cuda()
    mask = (torch.rand(B, H, 8, 8, generator=g) < 0.4)
    mask[..., 0] = True
    ref, ref_lse = ops.bsattn_fwd(q.permute(0, 2, 1, 3), k.permute(0, 2, 1, 3),
                                  v.permute(0, 2, 1, 3), mask.cuda())
    torch.cuda.synchronize()
    Sr = S // world
    for r in range(world):
        got = torch.load(tmp_path / f"r{r}.pt")
        # same kernel on the same unit data: bitwise equal
        assert torch.equal(got["out"], ref.permute(0, 2, 1, 3)[:, r * Sr:(r + 1) * Sr].cpu())
        assert torch.equal(got["lse"], ref_lse[:, :, r * Sr:(r + 1) * Sr].cpu())


_DIT_LATENT = (2, 16, 4, 32, 32)  # 1024 tokens: 512 per rank


def _dit_masks():
    g = torch.Generator().manual_seed(3)
    masks = torch.rand(2, 12, 8, 8, generator=g) < 0.5
    masks[..., 0] = True
    return masks


def _install_reference():
    """install() in a process of its own (the reference's packages on
    sys.path, as the `reference` fixture does for a test)."""
    from tests.conftest import REFERENCE_DIR

    sys.path.insert(0, str(REFERENCE_DIR))
    from sinkattn_b200 import reference_api as ra

    ra.install()


def _dit_worker(rank, world, port, result_dir):
    import torch.distributed as dist

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    sys.path.insert(0, str(ROOT))
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=120), device_id=dev)
    try:
        _install_reference()
        from tests import wan_dit

        model, ex = wan_dit.build(_dit_masks(), dev, layers=2, world=world, rank=rank,
                                  latent=_DIT_LATENT)
        x, t, text, rot = wan_dit.inputs(dev, latent=_DIT_LATENT)
        with torch.no_grad():
            out = model(x, t, text, rot, shard=(rank, world))
            out2 = model(x, t, text, rot, shard=(rank, world))  # buffers reused
        torch.cuda.synchronize()
        assert torch.equal(out, out2)
        torch.save(out.float().cpu(), os.path.join(result_dir, f"dit{rank}.pt"))
        ex.close()
        dist.barrier()
    finally:
        dist.destroy_process_group()


def test_ulysses_dit_matches_single_gpu(tmp_path):
    """Two sequence-parallel ranks (peer exchange around the reference's Wan
    processor) give the single-GPU DiT output to within 1e-2 mean-relative
    (the projections run on different row counts)."""
    import torch.multiprocessing as mp

    from tests.conftest import REFERENCE_DIR

    if not (REFERENCE_DIR / "sinkattention").exists():
        pytest.skip("reference packages not installed")
    world = 2
    mp.start_processes(_dit_worker, args=(world, _free_port(), str(tmp_path)), nprocs=world,
                       join=True, start_method="spawn")
    import importlib

    from sinkattn_b200 import reference_api as ra

    path = list(sys.path)
    sys.path.insert(0, str(REFERENCE_DIR))
    saved = []
    for name, attrs in ra._PATCHES.items():
        mod = importlib.import_module(name)
        saved += [(mod, a, getattr(mod, a)) for a in attrs if hasattr(mod, a)]
    wan = importlib.import_module("wanx.runtime.sink_sparse_wan")
    saved += [(wan, "_prepare_attention_tensors", wan._prepare_attention_tensors),
              (wan.WanSinkSparseInnerAttention, "forward", wan.WanSinkSparseInnerAttention.forward)]
    try:
        ra.install()
        from tests import wan_dit

        dev = torch.device("cuda", 0)
        model, _ = wan_dit.build(_dit_masks(), dev, layers=2, latent=_DIT_LATENT)
        x, t, text, rot = wan_dit.inputs(dev, latent=_DIT_LATENT)
        with torch.no_grad():
            full = model(x, t, text, rot).float().cpu()
    finally:
        for mod, a, val in saved:
            setattr(mod, a, val)
        sys.path[:] = path
    Sr = full.shape[1] // world
    for r in range(world):
        got = torch.load(tmp_path / f"dit{r}.pt")
        ref = full[:, r * Sr:(r + 1) * Sr]
        rel = float((got - ref).abs().mean() / ref.abs().mean())
        assert rel <= 1e-2, (r, rel)

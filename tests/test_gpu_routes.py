"""GPU tests of the two routes around the kernels: the device-resident
calibrator (package format v3) and the Z-Image cfg4 attention shape."""
from __future__ import annotations

import math

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


class _Cfg:
    """The fields of SinkSparseConfig the calibrator and mask builder read."""

    block_size = 128
    pooling_mode = "mean"
    offline_direct_coverage = 0.85
    offline_text_video_coverage_mode = "joint"
    force_text_global_attention = False
    text_length = 0
    keep_diagonal = True


def _asdict_cfg(monkeypatch):
    import sinkattn_b200.calibrator as cal

    monkeypatch.setattr(cal, "asdict", lambda c: {k: getattr(c, k) for k in dir(c)
                                                   if not k.startswith("_")})


def test_device_calibrator_statistics_and_package(monkeypatch, tmp_path, oracle):
    from sinkattn_b200 import ops
    from sinkattn_b200.calibrator import DeviceSinkMaskCalibrator

    _asdict_cfg(monkeypatch)
    g = torch.Generator().manual_seed(31)
    B, H, S = 2, 2, 640
    cal = DeviceSinkMaskCalibrator(_Cfg())
    expected_bm = {0: [], 1: []}
    for step in range(3):
        cal.reset_generation() if step == 0 else None
        for layer in (0, 1):
            q = torch.randn(B, H, S, 128, generator=g).bfloat16().cuda()
            k = torch.randn(B, H, S, 128, generator=g).bfloat16().cuda()
            cal.record(layer, q, k, k)
            _, bm = ops.pool_scores(q, k, want_scores=False, want_batch_mean=True)
            expected_bm[layer].append(bm)
    assert cal.current_step == 2 and cal.score_counts == {0: 3, 1: 3}
    pkg = cal.save(str(tmp_path / "pkg.pt"))
    loaded = torch.load(tmp_path / "pkg.pt", map_location="cpu", weights_only=True)
    assert loaded["version"] == 3 and set(loaded["sink_masks"]) == {"0", "1"}
    assert loaded["counts"] == {"0": 3, "1": 3}
    for layer in (0, 1):
        bms = expected_bm[layer]
        # the reference accumulates and divides on the CPU: fp32 adds, then an
        # IEEE fp32 division (CUDA torch would multiply by the reciprocal)
        ssum = ((bms[0] + bms[1]) + bms[2]).cpu()
        mean = ssum / 3
        got_mean = pkg["mean_scores"][str(layer)]
        assert torch.equal(got_mean, mean)
        b = [x.cpu() for x in bms]
        sq = (b[0].square() + b[1].square()) + b[2].square()
        std = torch.sqrt((sq / 3 - mean.square()).clamp_min(0))
        assert torch.equal(pkg["std_scores"][str(layer)], std)
        res = oracle.coverage_mask(mean.numpy(), row_total=mean.sum(-1).numpy())
        np.testing.assert_array_equal(loaded["sink_masks"][str(layer)].numpy(), res.mask)


def test_zimage_cfg4_attention_rows_vs_oracle(oracle):
    """cfg4: B=1, H=30, 16384 image + 512 text tokens (132 blocks). Mask from
    the coverage rule with key block 0 forced, then text rows/columns forced
    dense as the Z-Image runtime does (zimg/runtime/sink_sparse_zimage.py:
    218-230). Sampled rows match the oracle; every row is finite."""
    from sinkattn_b200 import ops
    from tests.gen import zimg_qkv

    q, k, v = zimg_qkv(seed=0, device="cuda")
    _, bm = ops.pool_scores(q, k, want_scores=False, want_batch_mean=True)
    mask, _ = ops.coverage_mask(bm, force_sink_col=True)
    nb = mask.shape[-1]
    assert nb == 132
    text0 = nb - 4
    mask[:, :, text0:] = True
    mask[:, text0:, :] = True
    out, lse = ops.bsattn_fwd(q, k, v, mask.unsqueeze(0))
    torch.cuda.synchronize()
    assert torch.isfinite(out).all() and torch.isfinite(lse).all()
    for h, qb in [(0, 0), (13, 77), (29, 131)]:
        rows = slice(qb * 128, min(qb * 128 + 128, q.shape[2]))
        ref, ref_lse = oracle.dense_masked_attention(
            q[:, h:h + 1, rows].float().cpu().numpy(), k[:, h:h + 1].float().cpu().numpy(),
            v[:, h:h + 1].float().cpu().numpy(), mask[h:h + 1, qb:qb + 1].unsqueeze(0).cpu().numpy())
        err = np.abs(out[:, h:h + 1, rows].float().cpu().numpy() - ref)
        assert err.max() <= 2e-2 and err.mean() / np.abs(ref).mean() <= 1e-2
        np.testing.assert_allclose(lse[0, h, rows].cpu().numpy(), ref_lse[0, 0], atol=2e-3)


@pytest.mark.parametrize("pooling_mode", ["mean", "triton"])
def test_device_zimage_calibrator_alignment(tmp_path, oracle, pooling_mode):
    """Z-Image calibration with samples of different text lengths: the device
    alignment, presence-weighted statistics and masks equal the reference's
    CPU arithmetic (zimg/runtime/sink_sparse_zimage.py:140-186, 262-354),
    restated here on the scores the device computed."""
    from dataclasses import dataclass

    from sinkattn_b200 import reference_api as ra
    from sinkattn_b200.calibrator import DeviceZImageSinkMaskCalibrator

    @dataclass
    class ZCfg:
        block_size: int = 128
        pooling_mode: str = "mean"
        offline_direct_coverage: float = 0.85
        offline_text_video_coverage_mode: str = "joint"
        force_text_global_attention: bool = True
        text_length: int = 300
        keep_diagonal: bool = True
        token_width: int = 32
        token_height: int = 32
        token_depth: int = 1

    cfg = ZCfg(pooling_mode=pooling_mode)
    cal = DeviceZImageSinkMaskCalibrator(cfg)
    assert (cal.image_blocks, cal.total_blocks, cal.max_text_tokens) == (8, 11, 320)
    g = torch.Generator().manual_seed(5)
    H, T, IB = 3, 11, 8
    ref = {}
    for step, text in enumerate([300, 100, 0, 250]):
        for layer in (0, 1):
            S = 1024 + text
            q = torch.randn(1, H, S, 128, generator=g).bfloat16().cuda()
            k = torch.randn(1, H, S, 128, generator=g).bfloat16().cuda()
            cal.record(layer, q, k, k, text_token_count=text)
            # the reference's record on the same device scores
            sc = ra._compute_block_scores(q, k, k, cfg).float().mean(dim=0).cpu()
            tb = -(-text // 128)
            aligned = torch.zeros(H, T, T)
            aligned[:, :IB, :IB] = sc[:, :IB, :IB]
            pres = torch.zeros(H, T, T)
            pres[:, :IB, :IB] = 1.0
            if tb > 0:
                t0 = T - tb
                aligned[:, :IB, t0:] = sc[:, :IB, IB:]
                aligned[:, t0:, :IB] = sc[:, IB:, :IB]
                aligned[:, t0:, t0:] = sc[:, IB:, IB:]
                pres[:, :IB, t0:] = 1.0
                pres[:, t0:, :IB] = 1.0
                pres[:, t0:, t0:] = 1.0
            if layer not in ref:
                ref[layer] = [aligned, aligned.square(), pres]
            else:
                ref[layer][0] += aligned
                ref[layer][1] += aligned.square()
                ref[layer][2] += pres
    assert cal.current_step == 3 and cal.score_counts == {0: 4, 1: 4}
    pkg = cal.save(str(tmp_path / "z.pt"))
    loaded = torch.load(tmp_path / "z.pt", map_location="cpu", weights_only=True)
    assert loaded["meta"]["route"] == "zimg_static_only" and loaded["meta"]["total_blocks"] == 11
    for layer in (0, 1):
        s, sq, pres = ref[layer]
        pres = pres.clamp_min_(1.0)
        mean = s / pres
        std = torch.sqrt((sq / pres - mean.square()).clamp_min_(0.0))
        assert torch.equal(pkg["mean_scores"][str(layer)], mean)
        assert torch.equal(pkg["std_scores"][str(layer)], std)
        assert torch.equal(cal.score_presence_sums[layer].cpu(), pres)
        # the reference's required text blocks are the first ceil(text_length / 128)
        # rows and columns (sparse_attention.py:250-261); fp32 sums as it takes them
        req = torch.zeros(T, T)
        req[:, :3] = 1.0
        req[:3, :] = 1.0
        res = oracle.coverage_mask(mean.numpy(), row_total=mean.sum(-1).numpy(),
                                   row_selected=(mean * req).sum(-1).numpy(),
                                   text_blocks=3, mode="joint", keep_diagonal=True)
        np.testing.assert_array_equal(loaded["sink_masks"][str(layer)].numpy(), res.mask)
    with pytest.raises(ValueError):
        cal.record(0, q, k, k, text_token_count=400)
    with pytest.raises(ValueError):
        cal.record(0, q.expand(2, -1, -1, -1), k.expand(2, -1, -1, -1), k, text_token_count=250)

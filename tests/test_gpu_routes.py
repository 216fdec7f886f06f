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

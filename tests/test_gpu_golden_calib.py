"""The kernels either side of the attention and pooling paths against golden
vectors made by running the reference (tests/golden/make_golden_calib.py):
sa_mean_pool_seq and sa_mix_outputs through the reference-facing drop-ins,
and the device calibrators (sa_score_accumulate(_aligned),
sa_score_finalize(_presence)) fed the reference's own block scores."""
from __future__ import annotations

import json

import numpy as np
import pytest
import torch

from tests.conftest import from_bits, regen_input
from tests.gen import config_from_json
from tests.test_oracle_golden_calib import MIX_ATOL, MIX_RTOL

pytestmark = pytest.mark.gpu

MPOOL_CASES = ["mpool_a", "mpool_b", "mpool_c", "mpool_d"]


@pytest.mark.parametrize("layout", ["bhsd", "bshd"])
@pytest.mark.parametrize("case", MPOOL_CASES)
def test_mean_pool_seq_kernel_matches_reference(calib_golden, oracle, case, layout):
    from sinkattn_b200 import reference_api as ra

    g = calib_golden
    x = regen_input(g, case, "x")
    pool, prefix = int(g[f"{case}/pool"]), int(g[f"{case}/prefix"])
    xd = x.cuda()
    if layout == "bshd":  # the processors' storage, read in place
        xd = xd.permute(0, 2, 1, 3).contiguous().permute(0, 2, 1, 3)
    out = ra._mean_pool_sequence_preserve_prefix(xd, pool, prefix_tokens=prefix)
    torch.cuda.synchronize()
    got = out.float().cpu().numpy()
    want = from_bits(g[f"{case}/out"])
    assert got.shape == want.shape
    ulp = oracle.bf16_ulp_distance(got, want)
    assert ulp.max() <= 1 and (ulp == 0).mean() >= 0.99
    n = min(prefix, x.shape[2])
    assert np.array_equal(got[:, :, :n], want[:, :, :n])


def test_mix_kernel_matches_reference(calib_golden):
    from sinkattn_b200 import reference_api as ra

    class Cfg:
        mixing_mode = "adaptive"
        sample_gap = int(calib_golden["mix/sample_gap"])

    g = calib_golden
    o_s = regen_input(g, "mix", "o_s")
    o_d = regen_input(g, "mix", "o_d")
    # the reference's LSE arguments: bf16 [B,H,S,1]
    ls = torch.from_numpy(g["mix/lse_s"].view(np.int16)).view(torch.bfloat16)
    ld = torch.from_numpy(g["mix/lse_d"].view(np.int16)).view(torch.bfloat16)
    out = ra._mix_attention_outputs(o_s.cuda(), ls.cuda(), o_d.cuda(), ld.cuda(), Cfg,
                                    Cfg.sample_gap)
    torch.cuda.synchronize()
    got = out.float().cpu().numpy()
    want = from_bits(g["mix/out"])
    assert got.shape == want.shape
    # the reference's bf16 rounding, plus one more rounding of the kernel's output
    err = np.abs(got - want)
    bound = MIX_ATOL + (MIX_RTOL + 2.0 ** -8) * (np.abs(o_s.float().numpy())
                                                 + np.abs(o_d.float().numpy()))
    assert (err <= bound).all(), float((err - bound).max())


def _check_package(pkg_path, g, prefix):
    loaded = torch.load(pkg_path, map_location="cpu", weights_only=True)
    assert loaded["version"] == 3
    assert loaded["meta"] == json.loads(str(g[f"{prefix}/meta"]))
    assert loaded["config"] == json.loads(str(g[f"{prefix}/config"]))
    for layer in ("0", "1"):
        assert loaded["counts"][layer] == int(g[f"{prefix}/count/{layer}"])
        # the mean and std carry the reference's bits; the mask is the reference's
        assert np.array_equal(loaded["mean_scores"][layer].numpy(), g[f"{prefix}/mean/{layer}"])
        assert np.array_equal(loaded["std_scores"][layer].numpy(), g[f"{prefix}/std/{layer}"])
        assert np.array_equal(loaded["sink_masks"][layer].numpy(), g[f"{prefix}/mask/{layer}"])


def test_device_calibrator_fed_reference_scores(calib_golden, tmp_path):
    from sinkattn_b200.calibrator import DeviceSinkMaskCalibrator

    g = calib_golden
    cal = DeviceSinkMaskCalibrator(config_from_json(g["wan_cal/config"]))
    for layer, scores in zip(g["wan_cal/layers"], g["wan_cal/scores"]):
        cal._accumulate_score(int(layer), torch.from_numpy(scores).cuda())
    cal.save(str(tmp_path / "wan.pt"))
    _check_package(tmp_path / "wan.pt", g, "wan_cal")


def test_device_zimage_calibrator_fed_reference_scores(calib_golden, tmp_path, monkeypatch):
    import sinkattn_b200.calibrator as calmod

    g = calib_golden
    cal = calmod.DeviceZImageSinkMaskCalibrator(config_from_json(g["z_cal/config"]))
    image_tokens, image_blocks, total_blocks, max_text = (int(v) for v in g["z_cal/layout"])
    assert (cal.image_token_count, cal.image_blocks, cal.total_blocks, cal.max_text_tokens) == \
        (image_tokens, image_blocks, total_blocks, max_text)
    feed = []
    monkeypatch.setattr(calmod, "_compute_block_scores", lambda q, k, v, config: feed.pop(0))
    i = 0
    for text in g["z_cal/texts"]:
        for layer in (0, 1):
            feed.append(torch.from_numpy(g[f"z_cal/scores/{i}"]).unsqueeze(0).cuda())
            i += 1
            cal.record(layer, torch.zeros(1, device="cuda"), None, None,
                       text_token_count=int(text))
    assert not feed
    cal.save(str(tmp_path / "z.pt"))
    _check_package(tmp_path / "z.pt", g, "z_cal")
    for layer in (0, 1):
        assert np.array_equal(cal.score_presence_sums[layer].cpu().numpy(),
                              g[f"z_cal/presence/{layer}"])

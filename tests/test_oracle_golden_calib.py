"""The oracle's restatements of the steps either side of the kernels against
golden vectors made by running the reference (tests/golden/make_golden_calib.py):
sequence mean pooling with a kept prefix, the adaptive LSE mix, the mask
adaptation to 128-token tiles, and both calibrators' statistics and masks.

These pin the oracle functions that the GPU tests of sa_mean_pool_seq,
sa_mix_outputs and the calibrator kernels check against.
"""
from __future__ import annotations

import math

import numpy as np
import pytest
import torch

from tests.conftest import from_bits, regen_input
from tests.gen import config_from_json

MPOOL_CASES = ["mpool_a", "mpool_b", "mpool_c", "mpool_d"]
# The reference mixes in bf16 arithmetic (ln(gap), alpha, 1 - alpha, both
# products and their sum each rounded to bf16, sparse_attention.py:910-919);
# the restatement is fp32. Bound: three bf16 roundings (2^-8 relative each) of
# the operands' magnitude, plus a small absolute floor.
MIX_RTOL = 3 * 2.0 ** -8
MIX_ATOL = 1e-3


def mix_within_reference_rounding(got, want, o_s, o_d) -> None:
    err = np.abs(got - want)
    bound = MIX_ATOL + MIX_RTOL * (np.abs(o_s) + np.abs(o_d))
    worst = np.unravel_index(np.argmax(err - bound), err.shape)
    assert (err <= bound).all(), f"mix error {err[worst]} > {bound[worst]} at {worst}"


@pytest.mark.parametrize("case", MPOOL_CASES)
def test_mean_pool_sequence_preserve_prefix_matches_reference(calib_golden, oracle, case):
    g = calib_golden
    x = regen_input(g, case, "x").float().numpy()
    pool, prefix = int(g[f"{case}/pool"]), int(g[f"{case}/prefix"])
    got = oracle.bf16_round(oracle.mean_pool_sequence_preserve_prefix(x, pool, prefix))
    want = from_bits(g[f"{case}/out"])
    assert got.shape == want.shape
    # the reference averages bf16 in torch's own order; one bf16 step at most
    ulp = oracle.bf16_ulp_distance(got, want)
    assert ulp.max() <= 1 and (ulp == 0).mean() >= 0.99
    if prefix > 0:
        n = min(prefix, x.shape[2])
        assert np.array_equal(got[:, :, :n], want[:, :, :n])  # kept rows are copied


def test_mix_outputs_matches_reference(calib_golden, oracle):
    g = calib_golden
    o_s = regen_input(g, "mix", "o_s").float().numpy()
    o_d = regen_input(g, "mix", "o_d").float().numpy()
    ls = from_bits(g["mix/lse_s"])[..., 0]
    ld = from_bits(g["mix/lse_d"])[..., 0]
    got = oracle.mix_outputs(o_s, ls, o_d, ld, int(g["mix/sample_gap"]))
    want = from_bits(g["mix/out"])
    assert got.shape == want.shape
    mix_within_reference_rounding(got, want, o_s, o_d)


def _mask_via_oracle(oracle, mean: np.ndarray, cfg) -> np.ndarray:
    """The oracle's coverage rule on a calibrated mean, with the fp32 row
    totals and required-block sums taken by torch as the reference takes them
    (sparse_attention.py:334, 339)."""
    H, nq, nk = mean.shape
    T = 0
    if cfg.force_text_global_attention and int(cfg.text_length) > 0:
        T = min(math.ceil(int(cfg.text_length) / int(cfg.block_size)), nq, nk)
    t = torch.from_numpy(mean)
    req = torch.from_numpy(oracle.required_mask(nq, nk, T))
    res = oracle.coverage_mask(mean, coverage=float(cfg.offline_direct_coverage),
                               keep_diagonal=bool(cfg.keep_diagonal), text_blocks=T,
                               mode=str(cfg.offline_text_video_coverage_mode),
                               row_total=t.sum(-1).numpy(),
                               row_selected=(t * req.float()).sum(-1).numpy())
    assert not res.tie_rows.any()
    return res.mask


def test_wan_calibrator_statistics_match_reference(calib_golden, oracle):
    g = calib_golden
    cfg = config_from_json(g["wan_cal/config"])
    sums: dict[int, tuple] = {}
    for layer, scores in zip(g["wan_cal/layers"], g["wan_cal/scores"]):
        prev = sums.get(int(layer), (None, None))
        sums[int(layer)] = oracle.accumulate(prev[0], prev[1], scores)
    for layer in (0, 1):
        count = int(g[f"wan_cal/count/{layer}"])
        assert count == int((g["wan_cal/layers"] == layer).sum())
        mean, std = oracle.finalize(*sums[layer], count)
        assert np.array_equal(mean, g[f"wan_cal/mean/{layer}"])
        # numpy's square root is correctly rounded; torch's CPU one may be a step off
        assert np.abs(std.view(np.int32) - g[f"wan_cal/std/{layer}"].view(np.int32)).max() <= 1
        assert np.array_equal(_mask_via_oracle(oracle, mean, cfg), g[f"wan_cal/mask/{layer}"])


def test_zimage_calibrator_statistics_match_reference(calib_golden, oracle):
    g = calib_golden
    cfg = config_from_json(g["z_cal/config"])
    _, image_blocks, total_blocks, _ = (int(v) for v in g["z_cal/layout"])
    bs = int(cfg.block_size)
    acc: dict[int, list] = {}
    i = 0
    for text in g["z_cal/texts"]:
        for layer in (0, 1):
            scores = g[f"z_cal/scores/{i}"]
            i += 1
            aligned, pres = oracle.zimage_align(scores, image_blocks, -(-int(text) // bs),
                                                total_blocks)
            if layer not in acc:
                s, sq = oracle.accumulate(None, None, aligned)
                acc[layer] = [s, sq, pres]
            else:
                s, sq = oracle.accumulate(acc[layer][0], acc[layer][1], aligned)
                acc[layer] = [s, sq, (acc[layer][2] + pres).astype(np.float32)]
    for layer in (0, 1):
        mean, std, pres = oracle.finalize_presence(*acc[layer])
        assert np.array_equal(pres, g[f"z_cal/presence/{layer}"])
        assert np.array_equal(mean, g[f"z_cal/mean/{layer}"])
        assert np.abs(std.view(np.int32) - g[f"z_cal/std/{layer}"].view(np.int32)).max() <= 1
        assert np.array_equal(_mask_via_oracle(oracle, mean, cfg), g[f"z_cal/mask/{layer}"])


def test_zimage_align_rejects_a_mismatched_shape(oracle):
    with pytest.raises(ValueError, match="Unexpected Z-Image block score shape"):
        oracle.zimage_align(np.zeros((2, 9, 9), np.float32), 8, 2, 11)


@pytest.mark.parametrize("case", ["adapt_coarse", "adapt_fine", "adapt_same"])
def test_adapt_block_mask_matches_reference(calib_golden, oracle, case):
    g = calib_golden
    seq_q, seq_k = (int(v) for v in g[f"{case}/seq"])
    got = oracle.adapt_block_mask(g[f"{case}/mask"], int(g[f"{case}/source"]), seq_q, seq_k)
    want = g[f"{case}/out"]
    assert got.shape == want.shape and got.dtype == want.dtype
    assert np.array_equal(got, want)


def test_adapt_block_mask_rejects_what_the_reference_rejects(oracle):
    m = np.ones((1, 2, 8, 6), dtype=bool)
    with pytest.raises(ValueError, match="wrong shape"):
        oracle.adapt_block_mask(m, 128, 1000, 1000)
    with pytest.raises(ValueError, match="coarse"):
        oracle.adapt_block_mask(m, 192, 1000, 700)
    with pytest.raises(ValueError, match="fine"):
        oracle.adapt_block_mask(m, 48, 1000, 700)

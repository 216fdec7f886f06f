"""The device Wan calibrator in each calibration score mode.

SinkMaskCalibrator.record (sinkattention/sparse_attention.py:575-582) takes
_compute_block_scores (lines 230-238) of every self-attention call:
  "triton" (the SinkSparseConfig default; compared case-sensitively at
           line 124)  -> the Triton kernel's block maxima (pooling_kernel.py)
  "exact"             -> block masses of the full softmax (lines 145-227)
  "mean" or another spelling of "triton" -> softmax of mean-pooled Q/K (138-142)
then the batch mean on the device (line 580) and the running sums on the host.

Each test records through DeviceSinkMaskCalibrator with the reference's
default configuration (or one field changed), and checks
  * that every record's batch mean is the block scores of the mode the
    reference dispatches to, bit for bit, and that those scores match the
    reference's own outputs (golden vectors made by running the reference:
    its Triton kernel on a B200 for "triton", its exact path for "exact");
  * that the package's mean and std equal the reference calibrator's
    arithmetic (fp32 sums on the host, then sum / count) on those records,
    bit for bit;
  * that the package's masks equal the reference coverage rule on that mean
    with its own fp32 row totals, bit for bit (the oracle, pinned to the
    reference's masks);
  * for "triton", that on every row whose scores equal the reference kernel's
    bit for bit, the mask also equals the mask the reference calibrator
    builds from the reference kernel's own scores.
"""
from __future__ import annotations

from pathlib import Path

import numpy as np
import pytest
import torch

from tests.conftest import regen_input
from tests.gen import default_config

pytestmark = pytest.mark.gpu

TRITON_GOLDEN = Path(__file__).resolve().parent / "golden" / "triton_max.npz"


def _reference_package_arithmetic(records):
    """SinkMaskCalibrator._accumulate_score and _build_mean_and_masks
    (sparse_attention.py:537-573) on CPU fp32 tensors: running sum and sum of
    squares in record order, then mean = sum / n, var = sq / n - mean^2
    clamped at 0, std = sqrt(var)."""
    s = records[0].clone()
    sq = records[0].square()
    for r in records[1:]:
        s += r
        sq += r.square()
    n = len(records)
    mean = s / n
    std = torch.sqrt((sq / n - mean.square()).clamp_min_(0.0))
    return mean, std


def _oracle_mask(oracle, mean: torch.Tensor, cfg) -> np.ndarray:
    return oracle.coverage_mask(mean.numpy(), row_total=mean.sum(-1).numpy(),
                                coverage=float(cfg.offline_direct_coverage),
                                keep_diagonal=bool(cfg.keep_diagonal)).mask


def _run(cfg, inputs_per_step, tmp_path):
    """Records [(layer, q, k)] per step through the device calibrator and,
    alongside, the block scores of the mode the reference would call."""
    from sinkattn_b200 import ops
    from sinkattn_b200.calibrator import DeviceSinkMaskCalibrator

    mode = str(cfg.pooling_mode).strip().lower()
    cal = DeviceSinkMaskCalibrator(cfg)
    recs: dict[int, list] = {}
    per_batch: dict[int, list] = {}
    for step in inputs_per_step:
        for layer, q, k in step:
            cal.record(layer, q, k, k)
            if mode == "exact":
                sc = ops.block_stats(q, k, mode="exact")
            elif cfg.pooling_mode == "triton":
                sc = ops.block_stats(q, k, mode="max")
            else:
                sc, _ = ops.pool_scores(q, k)
            per_batch.setdefault(layer, []).append(sc)
            recs.setdefault(layer, []).append(sc.float().mean(dim=0).cpu())
    pkg = cal.save(str(tmp_path / f"{mode}.pt"))
    loaded = torch.load(tmp_path / f"{mode}.pt", map_location="cpu", weights_only=True)
    return cal, pkg, loaded, recs, per_batch


def _check_package(oracle, cfg, cal, pkg, loaded, recs):
    assert loaded["version"] == 3
    assert loaded["config"]["pooling_mode"] == cfg.pooling_mode
    for layer, rs in recs.items():
        key = str(layer)
        assert cal.score_counts[layer] == len(rs) == loaded["counts"][key]
        mean, std = _reference_package_arithmetic(rs)
        assert torch.equal(pkg["mean_scores"][key], mean), layer
        assert torch.equal(pkg["std_scores"][key], std), layer
        assert torch.equal(loaded["mean_scores"][key], mean)
        np.testing.assert_array_equal(loaded["sink_masks"][key].numpy(),
                                      _oracle_mask(oracle, mean, cfg))


def _golden_qk(g, case):
    return regen_input(g, case, "q").cuda(), regen_input(g, case, "k").cuda()


@pytest.mark.skipif(not TRITON_GOLDEN.exists(), reason="triton_max.npz not generated")
def test_default_config_records_triton_block_maxima(oracle, tmp_path):
    """pooling_mode "triton", the reference default: the reference kernel's
    block maxima, not the mean-pooled rule."""
    from sinkattn_b200 import ops

    cfg = default_config()
    assert cfg.pooling_mode == "triton"
    g = dict(np.load(TRITON_GOLDEN))
    qb, kb = _golden_qk(g, "tri_b")  # [2,3,1024,128]: two batch elements
    qc, kc = _golden_qk(g, "tri_c")  # [1,2,2048,128]
    steps = [[(0, qb, kb), (1, qc, kc)],
             [(0, kb, qb), (1, kc, qc)],
             [(0, qb * 0.5, kb), (1, qc, kc * 2.0)]]
    cal, pkg, loaded, recs, per_batch = _run(cfg, steps, tmp_path)
    _check_package(oracle, cfg, cal, pkg, loaded, recs)
    # the first record of each layer is the reference kernel's own output
    for layer, case in ((0, "tri_b"), (1, "tri_c")):
        got = per_batch[layer][0].cpu().numpy()
        want = g[f"{case}/scores"]
        assert (got == want).mean() >= 0.97
        np.testing.assert_allclose(got, want, rtol=2 ** -6, atol=1e-6)
        # not the mean rule
        mean_rule, _ = ops.pool_scores(*(_golden_qk(g, case)))
        assert not torch.allclose(per_batch[layer][0], mean_rule, rtol=1e-2, atol=1e-3)
        # the reference calibrator's mask on the reference kernel's scores,
        # compared where the scores agree bit for bit
        ref_mean = torch.from_numpy(want).float().mean(dim=0)
        ours = recs[layer][0]
        ref_mask = _oracle_mask(oracle, ref_mean, cfg)
        our_mask = _oracle_mask(oracle, ours, cfg)
        same_rows = (ours == ref_mean).all(dim=-1).numpy()
        assert same_rows.mean() >= 0.5
        np.testing.assert_array_equal(our_mask[same_rows], ref_mask[same_rows])


@pytest.mark.parametrize("case", ["exact_a", "exact_b"])
def test_exact_mode_records_block_masses(oracle, golden, tmp_path, case):
    """pooling_mode "exact", the calibration CLIs' default
    (wanx/offline/calibrate_sink_sparse.py:99-107)."""
    cfg = default_config(pooling_mode="exact")
    q, k = _golden_qk(golden, case)
    g2 = torch.Generator().manual_seed(7)
    noise = torch.randn(q.shape, generator=g2).bfloat16().cuda()
    steps = [[(0, q, k)], [(0, noise, k)], [(0, q, noise)]]
    cal, pkg, loaded, recs, per_batch = _run(cfg, steps, tmp_path)
    _check_package(oracle, cfg, cal, pkg, loaded, recs)
    np.testing.assert_allclose(per_batch[0][0].cpu().numpy(), golden[f"{case}/scores"],
                               rtol=2e-3, atol=1e-6)


@pytest.mark.parametrize("mode", ["mean", "Triton"])
def test_mean_rule_modes(oracle, golden, tmp_path, mode):
    """pooling_mode "mean", and "Triton": _compute_block_scores lower-cases it
    to reach _compute_pooled_qk_block_scores, whose own test is
    case-sensitive (line 124), so the reference runs the mean rule."""
    cfg = default_config(pooling_mode=mode)
    q, k = _golden_qk(golden, "pool_a")
    steps = [[(0, q, k), (1, k, q)], [(0, q, q), (1, k, k)]]
    cal, pkg, loaded, recs, per_batch = _run(cfg, steps, tmp_path)
    _check_package(oracle, cfg, cal, pkg, loaded, recs)
    np.testing.assert_allclose(per_batch[0][0].cpu().numpy(), golden["pool_a/scores"],
                               rtol=2e-5, atol=1e-7)

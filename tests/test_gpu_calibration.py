"""GPU parity of the calibration chain: pooled scores, coverage masks, the
calibrator statistics and the dynamic-branch helpers."""
from __future__ import annotations

import math

import numpy as np
import pytest
import torch

from tests.conftest import regen_input

pytestmark = pytest.mark.gpu

POOL_CASES = ["pool_a", "pool_b", "pool_c"]
COV_CASES = ["cov_joint", "cov_peaky", "cov_text", "cov_video", "cov_ties", "cov_zero",
             "cov_nonsq", "cov_wide", "cov_sink"]


def _cov_kw(golden, case):
    return dict(coverage=float(golden[f"{case}/coverage"]),
                keep_diagonal=bool(int(golden[f"{case}/keep_diagonal"])),
                text_blocks=int(golden[f"{case}/text_blocks"]),
                mode=str(golden[f"{case}/mode"]),
                force_sink_col=bool(int(golden[f"{case}/force_sink"])))


@pytest.mark.parametrize("case", POOL_CASES)
def test_pooled_scores_vs_reference(golden, case):
    from sinkattn_b200 import ops

    q = regen_input(golden, case, "q").cuda()
    k = regen_input(golden, case, "k").cuda()
    block = int(golden[f"{case}/block"])
    scores, bmean = ops.pool_scores(q, k, block=block, want_batch_mean=True)
    torch.cuda.synchronize()
    want = golden[f"{case}/scores"]
    np.testing.assert_allclose(scores.cpu().numpy(), want, rtol=2e-5, atol=2e-7)
    np.testing.assert_allclose(bmean.cpu().numpy(), want.mean(0), rtol=2e-5, atol=2e-7)


def test_pooled_scores_strided_input(golden):
    from sinkattn_b200 import ops

    q = regen_input(golden, "pool_a", "q")
    k = regen_input(golden, "pool_a", "k")
    qs = q.permute(0, 2, 1, 3).contiguous().cuda().permute(0, 2, 1, 3)  # BSHD memory
    ks = k.permute(0, 2, 1, 3).contiguous().cuda().permute(0, 2, 1, 3)
    a, _ = ops.pool_scores(qs, ks)
    b, _ = ops.pool_scores(q.cuda(), k.cuda())
    torch.cuda.synchronize()
    assert torch.equal(a, b)


@pytest.mark.parametrize("case", COV_CASES)
def test_coverage_mask_bit_exact(golden, case):
    """Given the reference's fp32 row totals, the mask equals the reference's
    bit for bit; rows that differ must be flagged as ties at the cut."""
    from sinkattn_b200 import _lib, ops

    scores = torch.from_numpy(golden[f"{case}/scores"]).cuda()
    total = torch.from_numpy(golden[f"{case}/total"]).cuda()
    sel = torch.from_numpy(golden[f"{case}/selected"]).cuda()
    mask, flags = ops.coverage_mask(scores, row_total=total, row_selected=sel, want_flags=True,
                                    **_cov_kw(golden, case))
    torch.cuda.synchronize()
    want = golden[f"{case}/mask"]
    got = mask.cpu().numpy()
    fl = flags.cpu().numpy()
    diff = np.argwhere((got != want).any(-1))
    for h, i in diff:
        assert fl[h, i] & _lib.SA_ROW_TIE_AT_CUT, f"{case}: row ({h},{i}) differs unflagged"
    if case != "cov_ties":
        assert diff.size == 0
    else:
        np.testing.assert_array_equal(got.sum(-1), want.sum(-1))


@pytest.mark.parametrize("case", COV_CASES)
def test_coverage_mask_matches_oracle_stable_order(golden, oracle, case):
    """Against the oracle (same stable tie order) the mask is bit-exact everywhere."""
    from sinkattn_b200 import ops

    s = golden[f"{case}/scores"]
    kw = _cov_kw(golden, case)
    res = oracle.coverage_mask(s, row_total=golden[f"{case}/total"],
                               row_selected=golden[f"{case}/selected"], **kw)
    mask, _ = ops.coverage_mask(torch.from_numpy(s).cuda(),
                                row_total=torch.from_numpy(golden[f"{case}/total"]).cuda(),
                                row_selected=torch.from_numpy(golden[f"{case}/selected"]).cuda(),
                                **kw)
    torch.cuda.synchronize()
    np.testing.assert_array_equal(mask.cpu().numpy(), res.mask)


@pytest.mark.parametrize("case", ["cov_joint", "cov_peaky", "cov_text", "cov_nonsq", "cov_wide"])
def test_coverage_mask_device_totals_flag_near_target(golden, case):
    from sinkattn_b200 import _lib, ops

    s = torch.from_numpy(golden[f"{case}/scores"]).cuda()
    mask, flags = ops.coverage_mask(s, want_flags=True, **_cov_kw(golden, case))
    torch.cuda.synchronize()
    diff = np.argwhere((mask.cpu().numpy() != golden[f"{case}/mask"]).any(-1))
    fl = flags.cpu().numpy()
    for h, i in diff:
        assert fl[h, i] & (_lib.SA_ROW_NEAR_TARGET | _lib.SA_ROW_TIE_AT_CUT)


def test_dropin_mask_builder_on_cpu_scores(golden):
    """The drop-in _build_direct_mean_coverage_mask, given CPU scores (the
    calibrator's case), returns a CPU mask identical to the reference's."""
    from sinkattn_b200.reference_api import _build_direct_mean_coverage_mask

    class Cfg:
        offline_direct_coverage = 0.85
        offline_text_video_coverage_mode = "joint"
        force_text_global_attention = True
        text_length = 512
        block_size = 128
        keep_diagonal = True

    s = torch.from_numpy(golden["cov_text/scores"])
    m = _build_direct_mean_coverage_mask(s, Cfg)
    assert m.device.type == "cpu" and m.dtype == torch.bool
    np.testing.assert_array_equal(m.numpy(), golden["cov_text/mask"])


def test_wan_layer_pool_and_mask_vs_oracle(oracle):
    """cfg3 layer 0 at full size: pooled batch-mean scores vs the oracle, then
    the mask from those scores vs the oracle mask on the same scores."""
    from sinkattn_b200 import _lib, ops
    from tests.gen import wan_qk

    q, k, _ = wan_qk(seed=0, device="cuda")
    scores, bmean = ops.pool_scores(q, k, want_batch_mean=True)
    torch.cuda.synchronize()
    ref = oracle.pooled_block_scores(q[:, :2].float().cpu().numpy(), k[:, :2].float().cpu().numpy())
    np.testing.assert_allclose(scores[:, :2].cpu().numpy(), ref, rtol=1e-4, atol=1e-7)
    bm = bmean.cpu().numpy()
    total = torch.from_numpy(bm).sum(-1)
    mask, flags = ops.coverage_mask(bmean, row_total=total.cuda(), force_sink_col=True,
                                    want_flags=True)
    torch.cuda.synchronize()
    res = oracle.coverage_mask(bm, row_total=total.numpy(), force_sink_col=True)
    np.testing.assert_array_equal(mask.cpu().numpy(), res.mask)
    density = mask.float().mean().item()
    assert 0.5 < density < 0.95  # the stated generator gives ~0.83 (flat pooled logits)
    assert not (flags.cpu().numpy() & _lib.SA_ROW_EMPTY_FALLBACK).any()


def test_accumulate_finalize(oracle):
    from sinkattn_b200 import ops

    g = torch.Generator().manual_seed(2)
    xs = [torch.rand(3, 17, 19, generator=g) for _ in range(3)]
    s = torch.empty(3, 17, 19, device="cuda")
    sq = torch.empty_like(s)
    for i, x in enumerate(xs):
        ops.score_accumulate(x.cuda(), s, sq, first=(i == 0))
    mean, std = ops.score_finalize(s, sq, 3)
    torch.cuda.synchronize()
    rs, rsq = None, None
    for x in xs:
        rs, rsq = oracle.accumulate(rs, rsq, x.numpy())
    rm, rstd = oracle.finalize(rs, rsq, 3)
    np.testing.assert_allclose(mean.cpu().numpy(), rm, rtol=1e-6, atol=1e-7)
    np.testing.assert_allclose(std.cpu().numpy(), rstd, rtol=1e-4, atol=1e-6)


@pytest.mark.parametrize("S,pool,prefix,H", [(32760, 30, 0, 3), (1000, 30, 0, 3), (1000, 30, 77, 3),
                                             (500, 7, 600, 3), (1000, 40, 3, 3), (4100, 128, 0, 3),
                                             (1000, 200, 5, 3), (31, 30, 0, 3), (64, 30, 40, 3),
                                             (2000, 30, 0, 30), (1000, 64, 10, 13),
                                             (20, 30, 0, 3), (20, 30, 5, 3)])
def test_mean_pool_seq(oracle, S, pool, prefix, H):
    """Gap pooling with a kept prefix; head counts that split into uneven
    groups of heads per load (30 = 12 + 12 + 6, 13 at pool 64 = 6 + 6 + 1)."""
    from sinkattn_b200 import ops

    g = torch.Generator().manual_seed(S + pool)
    x = torch.randn(2, S, H, 128, generator=g).bfloat16().cuda().permute(0, 2, 1, 3)
    out = ops.mean_pool_seq(x, pool, prefix)
    torch.cuda.synchronize()
    ref = oracle.bf16_round(oracle.mean_pool_sequence_preserve_prefix(
        x.float().cpu().numpy(), pool, prefix))
    assert out.shape == ref.shape
    np.testing.assert_allclose(out.float().cpu().numpy(), ref, atol=1e-2, rtol=1e-2)


def test_mix_outputs(oracle):
    from sinkattn_b200 import ops

    g = torch.Generator().manual_seed(4)
    B, H, S = 2, 3, 257
    os_ = torch.randn(B, H, S, 128, generator=g).bfloat16()
    od = torch.randn(B, H, S, 128, generator=g).bfloat16()
    ls = torch.randn(B, H, S, generator=g) * 3
    ld = torch.randn(B, H, S, generator=g) * 3
    out = ops.mix_outputs(os_.cuda(), ls.cuda(), od.cuda(), ld.cuda(), 30)
    torch.cuda.synchronize()
    ref = oracle.mix_outputs(os_.float().numpy(), ls.numpy(), od.float().numpy(), ld.numpy(), 30)
    np.testing.assert_allclose(out.float().cpu().numpy(), ref, atol=2e-2, rtol=1e-2)


@pytest.mark.parametrize("fused,chunk,head_groups", [(True, 3, 1), (False, 1, 1), (False, 2, 1),
                                                     (False, 10, 1), (False, 2, 3),
                                                     (False, 4, 3)])
def test_calibration_pass_matches_serial_chain(fused, chunk, head_groups):
    """The pass over layers, as one fused launch per layer or as the chunked,
    two-stream pipeline (stacked pooled softmax and one mask launch per
    chunk, also with layers split into head groups): the batch means agree
    with the per-layer serial chain within one ulp (bit for bit for the
    pipeline), and the masks and flags equal the serial mask kernel's on the
    pass's own batch means."""
    from sinkattn_b200 import ops

    g = torch.Generator().manual_seed(8)
    layers = []
    for _ in range(5):
        q = torch.randn(2, 3, 1000, 128, generator=g).bfloat16().cuda()
        k = torch.randn(2, 3, 1000, 128, generator=g).bfloat16().cuda()
        layers.append((q, k))
    masks, bms, flags = ops.calibration_pass(layers, force_sink_col=True, want_batch_mean=True,
                                             chunk=chunk, head_groups=head_groups,
                                             want_flags=True, fused=fused)
    torch.cuda.synchronize()
    for l, (q, k) in enumerate(layers):
        qp, kp = ops.pool_means(q, k)
        _, bm = ops.pooled_softmax(qp, kp, want_scores=False, want_batch_mean=True)
        m, f = ops.coverage_mask(bms[l], force_sink_col=True, want_flags=True)
        torch.cuda.synchronize()
        if fused:
            assert _ulps(bm, bms[l]) <= 1
        else:
            assert torch.equal(bm, bms[l])
        assert torch.equal(m, masks[l])
        assert torch.equal(f, flags[l])


def _ulps(a: torch.Tensor, b: torch.Tensor) -> int:
    """Largest distance in units of the last place between two fp32 tensors
    of non-negative values."""
    ia = a.contiguous().view(torch.int32).long()
    ib = b.contiguous().view(torch.int32).long()
    return int((ia - ib).abs().max())


def test_pool_means_then_pooled_softmax_equals_pool_scores():
    """sa_pool_means followed by sa_pooled_softmax (the two halves, for hosts
    that pipeline them) gives sa_pool_scores' scores and batch mean (the
    fused kernel at this shape) within one ulp."""
    from sinkattn_b200 import ops

    g = torch.Generator().manual_seed(21)
    q = torch.randn(2, 3, 1000, 128, generator=g).bfloat16().cuda()
    k = torch.randn(2, 3, 1000, 128, generator=g).bfloat16().cuda()
    sc, bm = ops.pool_scores(q, k, want_scores=True, want_batch_mean=True)
    qp, kp = ops.pool_means(q, k)
    sc2, bm2 = ops.pooled_softmax(qp, kp, want_scores=True, want_batch_mean=True)
    torch.cuda.synchronize()
    assert sc.shape == sc2.shape == (2, 3, 8, 8) and bm2.shape == (3, 8, 8)
    assert _ulps(sc, sc2) <= 1 and _ulps(bm, bm2) <= 1


def test_calibration_pass_30_layers_vs_reference_rule(oracle):
    """cfg3 in full: the 30-layer pass (key block 0 forced, row totals summed
    on the device) against the reference rule applied to the same batch-mean
    scores with the reference's own fp32 row totals (CPU torch.sum, as
    _build_direct_mean_coverage_mask takes them on the calibrator's CPU
    tensors). Every row that differs must carry SA_ROW_NEAR_TARGET or
    SA_ROW_TIE_AT_CUT; the count of flagged and differing rows is reported.
    Layer 0's batch means are checked against the oracle's pooled scores."""
    from sinkattn_b200 import _lib, ops
    from tests.gen import wan_qk_layers_on_device

    layers = wan_qk_layers_on_device(30, torch.device("cuda"))
    masks, bms, flags = ops.calibration_pass(layers, force_sink_col=True, want_batch_mean=True,
                                             want_flags=True)
    torch.cuda.synchronize()
    q0, k0 = layers[0]
    ref0 = oracle.pooled_block_scores(q0[:, :2].float().cpu().numpy(),
                                      k0[:, :2].float().cpu().numpy()).mean(axis=0)
    np.testing.assert_allclose(bms[0, :2].cpu().numpy(), ref0, rtol=1e-4, atol=1e-7)
    del layers
    bms_c, masks_c, flags_c = bms.cpu(), masks.cpu().numpy(), flags.cpu().numpy()
    flagged = differing = 0
    for l in range(30):
        s = bms_c[l]
        res = oracle.coverage_mask(s.numpy(), row_total=s.sum(-1).numpy(), force_sink_col=True)
        diff = (masks_c[l] != res.mask).any(-1)
        fl = flags_c[l] & (_lib.SA_ROW_NEAR_TARGET | _lib.SA_ROW_TIE_AT_CUT)
        assert not (diff & (fl == 0)).any(), f"layer {l}: unflagged rows differ"
        flagged += int((fl != 0).sum())
        differing += int(diff.sum())
    print(f"30-layer pass: {30 * 12 * 256} rows, {flagged} flagged, {differing} differing "
          "(all flagged)")

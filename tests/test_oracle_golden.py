"""The CPU oracle against golden vectors produced by running the reference.

These pin the oracle before it is trusted as the GPU parity checker.
"""
from __future__ import annotations

import math
from pathlib import Path

import numpy as np
import pytest

from tests.conftest import from_bits, regen_input

POOL_CASES = ["pool_a", "pool_b", "pool_c"]
COV_CASES = ["cov_joint", "cov_peaky", "cov_text", "cov_video", "cov_ties", "cov_zero",
             "cov_nonsq", "cov_wide", "cov_sink"]


@pytest.mark.parametrize("case", POOL_CASES)
def test_pooled_scores_match_reference(golden, oracle, case):
    q = regen_input(golden, case, "q").float().numpy()
    k = regen_input(golden, case, "k").float().numpy()
    block = int(golden[f"{case}/block"])
    got = oracle.pooled_block_scores(q, k, block)
    want = golden[f"{case}/scores"]
    assert got.shape == want.shape
    np.testing.assert_allclose(got, want, rtol=2e-5, atol=2e-7)
    np.testing.assert_allclose(got.sum(-1), 1.0, atol=1e-5)


def _cov_args(golden, case):
    return dict(
        coverage=float(golden[f"{case}/coverage"]),
        keep_diagonal=bool(int(golden[f"{case}/keep_diagonal"])),
        text_blocks=int(golden[f"{case}/text_blocks"]),
        mode=str(golden[f"{case}/mode"]),
        force_sink_col=bool(int(golden[f"{case}/force_sink"])),
    )


@pytest.mark.parametrize("case", COV_CASES)
def test_coverage_mask_bit_exact_with_reference_totals(golden, oracle, case):
    scores = golden[f"{case}/scores"]
    want = golden[f"{case}/mask"]
    res = oracle.coverage_mask(scores, row_total=golden[f"{case}/total"],
                               row_selected=golden[f"{case}/selected"], **_cov_args(golden, case))
    diff_rows = np.argwhere((res.mask != want).any(-1))
    # torch's CPU sort is unstable: only rows whose cut splits equal scores may differ
    for h, i in diff_rows:
        assert res.tie_rows[h, i], f"{case}: row ({h},{i}) differs without a tie at the cut"
    if case != "cov_ties":
        assert diff_rows.size == 0


def test_coverage_ties_case_exercises_ties(golden, oracle):
    scores = golden["cov_ties/scores"]
    res = oracle.coverage_mask(scores, row_total=golden["cov_ties/total"],
                               row_selected=golden["cov_ties/selected"],
                               **_cov_args(golden, "cov_ties"))
    assert res.tie_rows.any()
    # tie rows keep the same number of blocks as the reference even when the
    # chosen members differ
    want = golden["cov_ties/mask"]
    np.testing.assert_array_equal(res.mask.sum(-1), want.sum(-1))


def test_coverage_zero_uses_empty_row_fallback(golden, oracle):
    res = oracle.coverage_mask(golden["cov_zero/scores"], row_total=golden["cov_zero/total"],
                               **_cov_args(golden, "cov_zero"))
    assert res.empty_rows.all()
    assert (res.mask.sum(-1) == 1).all()
    np.testing.assert_array_equal(res.mask, golden["cov_zero/mask"])


@pytest.mark.parametrize("case", ["cov_joint", "cov_text", "cov_nonsq"])
def test_coverage_mask_internal_totals_close(golden, oracle, case):
    """Without the reference's fp32 totals the oracle sums in fp64; decisions
    may flip only where the crossing sits within a few ulp of the target."""
    scores = golden[f"{case}/scores"]
    res = oracle.coverage_mask(scores, **_cov_args(golden, case))
    diff = (res.mask != golden[f"{case}/mask"]).any(-1)
    assert diff.mean() < 0.02


def test_dense_attention_matches_reference_dense_path(golden, oracle):
    q = regen_input(golden, "attn_dense", "q").float().numpy()
    k = regen_input(golden, "attn_dense", "k").float().numpy()
    v = regen_input(golden, "attn_dense", "v").float().numpy()
    nq, nk = math.ceil(q.shape[2] / 128), math.ceil(k.shape[2] / 128)
    mask = np.ones((1, 1, nq, nk), dtype=bool)
    out, lse = oracle.dense_masked_attention(q, k, v, mask)
    np.testing.assert_allclose(out, golden["attn_dense/out"], atol=2e-5, rtol=1e-4)
    np.testing.assert_allclose(lse, golden["attn_dense/lse"], atol=2e-5, rtol=1e-5)


def test_masked_attention_matches_reference_adapter(golden, oracle):
    q = regen_input(golden, "attn_sparse", "q").float().numpy()
    k = regen_input(golden, "attn_sparse", "k").float().numpy()
    v = regen_input(golden, "attn_sparse", "v").float().numpy()
    mask = golden["attn_sparse/mask"]
    out, lse = oracle.dense_masked_attention(q, k, v, mask)
    want = from_bits(golden["attn_sparse/out"])  # bf16 output of the reference adapter
    np.testing.assert_allclose(oracle.bf16_round(out), want, atol=1e-2, rtol=0)
    want_lse = from_bits(golden["attn_sparse/lse_bf16"])
    np.testing.assert_allclose(oracle.bf16_round(lse), want_lse, rtol=1e-2)


def test_wan_inner_attention_composition(golden, oracle):
    """Sink branch + pooled dynamic branch (gap 30, band 1) + adaptive mix,
    composed from oracle pieces the way WanSinkSparseInnerAttention.forward
    does (wanx/runtime/sink_sparse_wan.py:181-282)."""
    q = regen_input(golden, "attn_sparse", "q").float().numpy()
    k = regen_input(golden, "attn_sparse", "k").float().numpy()
    v = regen_input(golden, "attn_sparse", "v").float().numpy()
    mask = golden["attn_sparse/mask"].copy()
    gap = int(golden["wan_inner/sample_gap"])
    band = int(golden["wan_inner/band"])
    nq = mask.shape[-2]
    ii, jj = np.meshgrid(np.arange(nq), np.arange(mask.shape[-1]), indexing="ij")
    mask = mask | (np.abs(ii - jj) <= band)[None, None]
    o_s, l_s = oracle.dense_masked_attention(q, k, v, mask)
    # the reference rounds both branches to bf16 (q.dtype) before mixing
    o_s, l_s = oracle.bf16_round(o_s), oracle.bf16_round(l_s)
    kp = oracle.bf16_round(oracle.mean_pool_sequence_preserve_prefix(k, gap))
    vp = oracle.bf16_round(oracle.mean_pool_sequence_preserve_prefix(v, gap))
    dmask = np.ones((1, q.shape[1], nq, math.ceil(kp.shape[2] / 128)), dtype=bool)
    o_d, l_d = oracle.dense_masked_attention(q, kp, vp, dmask)
    o_d, l_d = oracle.bf16_round(o_d), oracle.bf16_round(l_d)
    mixed = oracle.mix_outputs(o_s, l_s, o_d, l_d, gap)
    want = from_bits(golden["wan_inner/out"])
    err = np.abs(mixed - want)
    assert err.max() < 2e-2
    assert err.mean() / np.abs(want).mean() < 1e-2


def test_kept_block_flops_counts_valid_area(oracle):
    mask = np.zeros((1, 1, 2, 3), dtype=bool)
    mask[0, 0, 1, 2] = True  # last row block (rows 128..199) x last col block (256..299)
    f = oracle.kept_block_flops(mask, 1, 1, 200, 300)
    assert f == 4 * 128 * (72 * 44)


@pytest.mark.parametrize("case", ["exact_a", "exact_b"])
def test_exact_block_mass_matches_reference(golden, oracle, case):
    q = regen_input(golden, case, "q").float().numpy()
    k = regen_input(golden, case, "k").float().numpy()
    got = oracle.exact_block_mass_scores(q, k)
    np.testing.assert_allclose(got, golden[f"{case}/scores"], rtol=1e-4, atol=1e-7)


@pytest.mark.parametrize("case", ["tri_a", "tri_b", "tri_c"])
def test_triton_max_restatement_matches_reference_kernel(oracle, case):
    """Pinned against outputs of the reference's Triton kernel run on a B200
    (tests/golden/make_golden_triton.py): bit-identical on these cases."""
    g = dict(np.load(Path(__file__).resolve().parent / "golden" / "triton_max.npz"))
    q = regen_input(g, case, "q").float().numpy()
    k = regen_input(g, case, "k").float().numpy()
    got = oracle.triton_max_pool_scores(q, k)
    np.testing.assert_array_equal(got, g[f"{case}/scores"])


def test_triton_max_pool_restatement_properties(oracle):
    """Rows are normalised (bf16 rounding aside), entries lie in [0, 1] and
    the diagonal-heavy input peaks on the diagonal."""
    rng = np.random.default_rng(0)
    q = oracle.bf16_round(rng.standard_normal((1, 1, 512, 128)).astype(np.float32))
    k = q.copy()
    s = oracle.triton_max_pool_scores(q, k)
    assert s.shape == (1, 1, 4, 4)
    assert np.all(s >= 0) and np.all(s <= 1)
    np.testing.assert_allclose(s.sum(-1), 1.0, atol=2e-2)
    assert np.all(np.argmax(s[0, 0], axis=1) == np.arange(4))


def test_qk_norm_rope_matches_reference(golden, oracle):
    """RMSNorm + rotary through the reference's own helpers (torch RMSNorm,
    fp64 complex rotary): the oracle equals them bit for bit here."""
    heads = int(golden["qkrope/heads"])
    for t in ("q", "k"):
        x = regen_input(golden, "qkrope", t).float().numpy()
        w = from_bits(golden[f"qkrope/w_{t}"])
        got = oracle.qk_norm_rope(x, w, float(golden["qkrope/eps"]), golden["qkrope/cos"],
                                  golden["qkrope/sin"], heads)
        want = from_bits(golden[f"qkrope/{t}_out"])
        d = oracle.bf16_ulp_distance(got, want)
        assert d.max() == 0, (d.max(), (d == 0).mean())

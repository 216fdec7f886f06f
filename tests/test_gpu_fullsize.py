"""Full-size parity of the attention kernels: every (b, h, query tile) of the
launches the benchmark times, compared with fp32 dense masked attention.

The per-unit fp32 reference runs on the GPU (tests/torch_ref.py), pinned
here against the numpy oracle on a small ragged case first. Tolerance (from
the benchmark contract), per 128-row query tile: max-abs 2e-2 and mean-rel
(mean |err| / mean |ref| over the tile) 1e-2 on the output; LSE within 2e-3
on every row, and empty rows (-inf) exactly where the reference has them.

Cases:
  * cfg2, the headline: Wan B=2, H=12, S=32768, column 0 | diagonal |
    Bernoulli(0.2) (rho ~ 0.21);
  * cfg2 with the reference coverage rule's mask (pool -> pooled softmax ->
    batch mean -> 0.85 coverage with key block 0 forced; rho ~ 0.84);
  * the ragged Wan length S = 32760 (last block 120 tokens);
  * cfg4, Z-Image: B=1, H=30, 16896 tokens = 132 blocks, coverage mask with
    the text rows and columns forced dense;
  * the Wan runtime's fused sink + pooled-dynamic forward at S = 32760
    (sink | band-1 mask, pooled K/V gap 30, +ln(gap) logit bias).
"""
from __future__ import annotations

import math

import numpy as np
import pytest
import torch

from tests.gen import cfg1_mask, wan_qk, zimg_qkv
from tests.torch_ref import compare_tiles, unit_attention

pytestmark = pytest.mark.gpu

MAX_ABS = 2e-2
MEAN_REL = 1e-2
LSE_ATOL = 2e-3


def _check_launch(q, k, v, mask, out, lse, what, extra=None, gap=None):
    """Compares every unit of a launch; returns the worst figures."""
    B, H = q.shape[0], q.shape[1]
    worst = {"max_abs": 0.0, "mean_rel": 0.0, "lse": 0.0}
    bias = 0.0 if gap is None else math.log(float(gap))
    for b in range(B):
        mb = mask[b if mask.shape[0] > 1 else 0]
        for h in range(H):
            ek = ev = None
            if extra is not None:
                ek, ev = extra[0][b, h], extra[1][b, h]
            ref, ref_lse = unit_attention(q[b, h], k[b, h], v[b, h], mb[h], extra_k=ek,
                                          extra_v=ev, extra_bias=bias)
            r = compare_tiles(out[b, h], lse[b, h], ref, ref_lse)
            assert r["lse_finite_mismatch"] == 0, (what, b, h, r)
            assert r["max_abs"] <= MAX_ABS, (what, b, h, r)
            assert r["mean_rel"] <= MEAN_REL, (what, b, h, r)
            assert r["lse"] <= LSE_ATOL, (what, b, h, r)
            for key in worst:
                worst[key] = max(worst[key], r[key])
    return worst


def test_gpu_reference_matches_oracle(oracle):
    """The GPU fp32 reference equals the numpy oracle to fp32 rounding on a
    ragged case with empty rows, and with extra biased keys."""
    g = torch.Generator().manual_seed(3)
    Sq, Sk, D = 1000, 777, 128
    q = torch.randn(1, 1, Sq, D, generator=g).bfloat16()
    k = torch.randn(1, 1, Sk, D, generator=g).bfloat16()
    v = torch.randn(1, 1, Sk, D, generator=g).bfloat16()
    nq, nk = math.ceil(Sq / 128), math.ceil(Sk / 128)
    m = torch.rand(1, 1, nq, nk, generator=g) < 0.4
    m[0, 0, 3] = False  # an empty query tile
    ref, ref_lse = oracle.dense_masked_attention(q.float().numpy(), k.float().numpy(),
                                                 v.float().numpy(), m.numpy())
    got, got_lse = unit_attention(q[0, 0].cuda(), k[0, 0].cuda(), v[0, 0].cuda(), m[0, 0].cuda(),
                                  row_chunk=384)
    np.testing.assert_allclose(got.cpu().numpy(), ref[0, 0], atol=2e-6, rtol=1e-5)
    assert np.array_equal(np.isfinite(got_lse.cpu().numpy()), np.isfinite(ref_lse[0, 0]))
    fin = np.isfinite(ref_lse[0, 0])
    np.testing.assert_allclose(got_lse.cpu().numpy()[fin], ref_lse[0, 0][fin], atol=2e-6)
    kp = torch.randn(1, 1, 40, D, generator=g).bfloat16()
    vp = torch.randn(1, 1, 40, D, generator=g).bfloat16()
    m2 = m.clone()
    m2[..., 0] = True
    ref2, ref2_lse = oracle.sink_dynamic_attention(q.float().numpy(), k.float().numpy(),
                                                   v.float().numpy(), m2.numpy(),
                                                   kp.float().numpy(), vp.float().numpy(), 30)
    got2, got2_lse = unit_attention(q[0, 0].cuda(), k[0, 0].cuda(), v[0, 0].cuda(),
                                    m2[0, 0].cuda(), extra_k=kp[0, 0].cuda(),
                                    extra_v=vp[0, 0].cuda(), extra_bias=math.log(30.0))
    np.testing.assert_allclose(got2.cpu().numpy(), ref2[0, 0], atol=2e-6, rtol=1e-5)
    np.testing.assert_allclose(got2_lse.cpu().numpy(), ref2_lse[0, 0], atol=2e-6)


@pytest.fixture(scope="module")
def wan_inputs():
    q, k, v = wan_qk(seed=0, device="cuda")
    return q, k, v


def test_wan_cfg2_rho21_every_tile(wan_inputs):
    """The benchmark's headline launch, all 2 x 12 x 256 query tiles."""
    from sinkattn_b200 import ops

    q, k, v = wan_inputs
    mask = cfg1_mask(12, 256, 256, seed=1).unsqueeze(0).expand(2, -1, -1, -1).contiguous().cuda()
    out, lse = ops.bsattn_fwd(q, k, v, mask)
    torch.cuda.synchronize()
    worst = _check_launch(q, k, v, mask, out, lse, "cfg2 rho~0.21")
    print("cfg2 rho~0.21 worst", worst)


def test_wan_cfg2_coverage_rule_every_tile(wan_inputs):
    """The benchmark's second figure: the mask the coverage rule builds from
    this layer's own Q/K (key block 0 forced), rho ~ 0.84."""
    from sinkattn_b200 import ops

    q, k, v = wan_inputs
    _, bm = ops.pool_scores(q, k, want_scores=False, want_batch_mean=True)
    cov, _ = ops.coverage_mask(bm, force_sink_col=True)
    mask = cov.unsqueeze(0).expand(2, -1, -1, -1).contiguous()
    density = float(mask.float().mean())
    assert 0.7 < density < 0.95
    out, lse = ops.bsattn_fwd(q, k, v, mask)
    torch.cuda.synchronize()
    worst = _check_launch(q, k, v, mask, out, lse, "cfg2 coverage")
    print("cfg2 coverage rho=%.3f worst" % density, worst)


def test_wan_ragged_32760_every_tile():
    """The real Wan token count: 32760 = 255 full blocks + 120 tokens."""
    from sinkattn_b200 import ops

    q, k, v = wan_qk(seed=2, S=32760, device="cuda")
    mask = cfg1_mask(12, 256, 256, seed=4).unsqueeze(0).expand(2, -1, -1, -1).contiguous().cuda()
    mask[:, :, :, 255] |= mask[:, :, :, 254]  # the ragged key block kept in more rows
    out, lse = ops.bsattn_fwd(q, k, v, mask)
    torch.cuda.synchronize()
    worst = _check_launch(q, k, v, mask, out, lse, "wan S=32760")
    print("wan S=32760 worst", worst)


def test_zimage_cfg4_every_tile():
    """cfg4 in full: coverage mask (key block 0 forced), then the text rows
    and columns forced dense as the Z-Image runtime does
    (zimg/runtime/sink_sparse_zimage.py:218-230)."""
    from sinkattn_b200 import ops

    q, k, v = zimg_qkv(seed=0, device="cuda")
    _, bm = ops.pool_scores(q, k, want_scores=False, want_batch_mean=True)
    cov, _ = ops.coverage_mask(bm, force_sink_col=True)
    nb = cov.shape[-1]
    assert nb == 132
    cov[:, :, nb - 4:] = True
    cov[:, nb - 4:, :] = True
    mask = cov.unsqueeze(0).contiguous()
    out, lse = ops.bsattn_fwd(q, k, v, mask)
    torch.cuda.synchronize()
    worst = _check_launch(q, k, v, mask, out, lse, "zimage cfg4")
    print("zimage cfg4 worst", worst)


def test_wan_runtime_fused_every_tile():
    """The Wan runtime default in one kernel: sink | band-1 mask over the
    32760 tokens, plus every pooled key of the gap-30 pooled K/V with the
    +ln(30) logit bias (the adaptive LSE mix as one softmax)."""
    from sinkattn_b200 import ops

    q, k, v = wan_qk(seed=5, S=32760, device="cuda")
    m = cfg1_mask(12, 256, 256, seed=1)
    ii = torch.arange(256)
    m = m | ((ii[:, None] - ii[None, :]).abs() <= 1)
    mask = m.unsqueeze(0).expand(2, -1, -1, -1).contiguous().cuda()
    kp = ops.mean_pool_seq(k, 30)
    vp = ops.mean_pool_seq(v, 30)
    assert kp.shape[2] == 1092
    out, lse = ops.sink_dynamic_attn(q, k, v, mask, kp, vp, 30, return_lse=True)
    torch.cuda.synchronize()
    worst = _check_launch(q, k, v, mask, out, lse, "wan runtime fused", extra=(kp, vp), gap=30)
    print("wan runtime fused worst", worst)

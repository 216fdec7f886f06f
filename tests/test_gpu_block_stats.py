"""GPU parity of the block-statistics kernel (sa_block_stats): the exact
block-mass mode against the reference's own outputs and the oracle, and the
block-maximum mode against the reference's Triton kernel outputs and the
oracle's restatement of it."""
from __future__ import annotations

import math
from pathlib import Path

import numpy as np
import pytest
import torch

from tests.conftest import regen_input

pytestmark = pytest.mark.gpu

TRITON_GOLDEN = Path(__file__).resolve().parent / "golden" / "triton_max.npz"


class _Cfg:
    block_size = 128

    def __init__(self, pooling_mode):
        self.pooling_mode = pooling_mode


def _randn(shape, seed, scale=1.0):
    g = torch.Generator().manual_seed(seed)
    return (torch.randn(*shape, generator=g) * scale).to(torch.bfloat16)


@pytest.mark.parametrize("case", ["exact_a", "exact_b"])
def test_exact_matches_reference_golden(golden, case):
    from sinkattn_b200 import ops

    q = regen_input(golden, case, "q").cuda()
    k = regen_input(golden, case, "k").cuda()
    got = ops.block_stats(q, k, mode="exact").cpu().numpy()
    want = golden[f"{case}/scores"]
    np.testing.assert_allclose(got, want, rtol=2e-3, atol=1e-6)
    np.testing.assert_allclose(got.sum(-1), 1.0, atol=1e-4)


@pytest.mark.parametrize("B,H,S,scale", [(1, 2, 1000, 1.0), (2, 1, 384, 3.0), (1, 1, 130, 1.0),
                                         (1, 1, 77, 2.0)])
def test_exact_matches_oracle(oracle, B, H, S, scale):
    from sinkattn_b200 import ops

    q = _randn((B, H, S, 128), 11 + S, scale)
    k = _randn((B, H, S, 128), 12 + S, scale)
    got = ops.block_stats(q.cuda(), k.cuda(), mode="exact").cpu().numpy()
    want = oracle.exact_block_mass_scores(q.float().numpy(), k.float().numpy())
    np.testing.assert_allclose(got, want, rtol=2e-3, atol=1e-6)


def test_exact_row_maximum_jump(oracle):
    """Key blocks whose logits exceed every earlier block's by more than 100
    in base 2 for the first 64 query rows and not for the others: the row
    maximum jumps late in the sweep, so the early blocks' masses are rescaled
    by factors far below the fp32 range of their own sums."""
    from sinkattn_b200 import ops

    S = 640
    g = torch.Generator().manual_seed(3)
    base = torch.randn(128, generator=g)
    q = torch.randn(1, 1, S, 128, generator=g)
    q[0, 0, :64] = base + 0.05 * torch.randn(64, 128, generator=g)
    k = torch.randn(1, 1, S, 128, generator=g)
    k[0, 0, 300] = 8.0 * base  # key block 2: logits ~1000 for the first 64 rows
    k[0, 0, 600] = 12.0 * base  # key block 4: a second jump
    q, k = q.to(torch.bfloat16), k.to(torch.bfloat16)
    got = ops.block_stats(q.cuda(), k.cuda(), mode="exact").cpu().numpy()
    want = oracle.exact_block_mass_scores(q.float().numpy(), k.float().numpy())
    assert np.isfinite(got).all()
    np.testing.assert_allclose(got, want, rtol=2e-3, atol=1e-6)


def test_negative_logits(oracle):
    """Every logit negative (positive Q against negative K), so each block's
    maximum is below zero: both modes against the oracle."""
    from sinkattn_b200 import ops

    g = torch.Generator().manual_seed(8)
    q = torch.randn(1, 2, 512, 128, generator=g).abs()
    k = -torch.randn(1, 2, 512, 128, generator=g).abs()
    q, k = q.to(torch.bfloat16), k.to(torch.bfloat16)
    qf, kf = q.float().numpy(), k.float().numpy()
    got = ops.block_stats(q.cuda(), k.cuda(), mode="max").cpu().numpy()
    want = oracle.triton_max_pool_scores(qf, kf)
    assert (got == want).mean() >= 0.97
    np.testing.assert_allclose(got, want, rtol=2 ** -6, atol=1e-6)
    got = ops.block_stats(q.cuda(), k.cuda(), mode="exact").cpu().numpy()
    np.testing.assert_allclose(got, oracle.exact_block_mass_scores(qf, kf), rtol=2e-3, atol=1e-6)


def test_exact_strided_layout(oracle):
    """[B,S,H,D] storage viewed as [B,H,S,D] (the Wan layout) needs no copy."""
    from sinkattn_b200 import ops

    B, H, S = 1, 3, 640
    qs = _randn((B, S, H, 128), 5).cuda()
    ks = _randn((B, S, H, 128), 6).cuda()
    q, k = qs.transpose(1, 2), ks.transpose(1, 2)
    got = ops.block_stats(q, k, mode="exact")
    ref = ops.block_stats(q.contiguous(), k.contiguous(), mode="exact")
    assert torch.equal(got, ref)


@pytest.mark.skipif(not TRITON_GOLDEN.exists(), reason="triton_max.npz not generated")
@pytest.mark.parametrize("case", ["tri_a", "tri_b", "tri_c"])
def test_max_matches_reference_triton_kernel(case):
    """Block maxima go through bf16 (R and Po) in both kernels; accumulation
    order in the two tensor-core GEMMs differs, so an entry may land one bf16
    step apart where a value sits on a rounding boundary."""
    from sinkattn_b200 import ops

    g = dict(np.load(TRITON_GOLDEN))
    q = regen_input(g, case, "q").cuda()
    k = regen_input(g, case, "k").cuda()
    got = ops.block_stats(q, k, mode="max").cpu().numpy()
    want = g[f"{case}/scores"]
    assert got.shape == want.shape
    exact = (got == want).mean()
    assert exact >= 0.97, f"only {exact:.3f} of entries bit-identical"
    np.testing.assert_allclose(got, want, rtol=2 ** -6, atol=1e-6)


@pytest.mark.parametrize("B,H,S", [(1, 2, 512), (2, 1, 1280), (1, 1, 1000)])
def test_max_matches_oracle(oracle, B, H, S):
    from sinkattn_b200 import ops

    q = _randn((B, H, S, 128), 21 + S)
    k = _randn((B, H, S, 128), 22 + S)
    got = ops.block_stats(q.cuda(), k.cuda(), mode="max").cpu().numpy()
    want = oracle.triton_max_pool_scores(q.float().numpy(), k.float().numpy())
    assert (got == want).mean() >= 0.97
    np.testing.assert_allclose(got, want, rtol=2 ** -6, atol=1e-6)


def test_drop_ins_dispatch_by_pooling_mode(oracle):
    from sinkattn_b200 import ops, reference_api as ra

    q = _randn((1, 2, 512, 128), 31).cuda()
    k = _randn((1, 2, 512, 128), 32).cuda()
    ex = ra._compute_exact_block_mass_scores(q, k, _Cfg("exact"))
    assert torch.equal(ex, ops.block_stats(q, k, mode="exact"))
    tr = ra._compute_pooled_qk_block_scores(q, k, k, _Cfg("triton"))
    assert torch.equal(tr, ops.block_stats(q, k, mode="max"))
    mean = ra._compute_pooled_qk_block_scores(q, k, k, _Cfg("mean"))
    want = oracle.pooled_block_scores(q.float().cpu().numpy(), k.float().cpu().numpy(), 128)
    np.testing.assert_allclose(mean.cpu().numpy(), want, rtol=1e-4, atol=1e-6)
    with pytest.raises(NotImplementedError):
        ra._compute_exact_block_mass_scores(q, k[:, :, :256], _Cfg("exact"))


def test_full_size_properties():
    """Wan-sized rows (the 32760 video tokens, one head; a ragged last block):
    exact-mode rows are probability vectors, max-mode rows are normalised
    bf16 vectors, both finite."""
    from sinkattn_b200 import ops
    from tests.gen import wan_qk

    q, k, _ = wan_qk(B=1, H=1, S=32760, seed=3, device="cuda")
    ex = ops.block_stats(q, k, mode="exact")
    mx = ops.block_stats(q, k, mode="max")
    torch.cuda.synchronize()
    nb = math.ceil(q.shape[2] / 128)
    assert ex.shape == mx.shape == (1, 1, nb, nb)
    assert torch.isfinite(ex).all() and torch.isfinite(mx).all()
    assert (ex >= 0).all() and (mx >= 0).all()
    torch.testing.assert_close(ex.sum(-1), torch.ones_like(ex.sum(-1)), atol=1e-4, rtol=0)
    torch.testing.assert_close(mx.sum(-1), torch.ones_like(mx.sum(-1)), atol=3e-2, rtol=0)

"""Host-side logic that needs no GPU: argument checks of the new entry points,
the rotary-table normalisation and RMSNorm detection of the Q/K producer
drop-in, the Z-Image calibrator's fixed block layout, and the score-mode
dispatch, and the CPU reference the benchmark times."""
from __future__ import annotations

import ctypes
import math

import numpy as np
import pytest
import torch


def _i64(*v):
    return (ctypes.c_int64 * 4)(*v)


def test_block_stats_validation_and_workspace(lib):
    from sinkattn_b200 import _lib

    st = _i64(128 * 256, 128 * 256, 128, 1)
    # head dim must be 128
    assert lib.sa_block_stats(16, 16, st, st, 1, 1, 256, 64, _lib.SA_STATS_EXACT, 0.0, 16, 16,
                              1 << 20, None, None) == _lib.SA_EINVAL
    # unknown mode
    assert lib.sa_block_stats(16, 16, st, st, 1, 1, 256, 128, 7, 0.0, 16, 16, 1 << 20, None,
                              None) == _lib.SA_EINVAL
    # missing workspace
    assert lib.sa_block_stats(16, 16, st, st, 1, 1, 256, 128, _lib.SA_STATS_MAX, 0.0, 16, None,
                              0, None, None) == _lib.SA_EINVAL
    assert "workspace" in lib.sa_last_error().decode()
    # too many key blocks (S > 131072)
    assert lib.sa_block_stats(16, 16, st, st, 1, 1, 131073, 128, _lib.SA_STATS_MAX, 0.0, 16, 16,
                              1 << 40, None, None) == _lib.SA_EINVAL
    assert lib.sa_block_stats_workspace_size(1, 1, 256, 9) == 0


def test_qk_norm_rope_validation(lib):
    from sinkattn_b200 import _lib

    # hidden must be a multiple of D
    assert lib.sa_qk_norm_rope(16, 16, 200, 200, 4, 4, 200, 128, None, None, 1, 1e-6, None, None,
                               0, 16, 16, 200, 200, None) == _lib.SA_EINVAL
    # cos without sin
    assert lib.sa_qk_norm_rope(16, 16, 256, 256, 4, 4, 256, 128, None, None, 1, 1e-6, 16, None,
                               64, 16, 16, 256, 256, None) == _lib.SA_EINVAL
    # misaligned row stride
    assert lib.sa_qk_norm_rope(16, 16, 260, 256, 4, 4, 256, 128, None, None, 1, 1e-6, None, None,
                               0, 16, 16, 256, 256, None) == _lib.SA_EINVAL
    # zero rows is a no-op
    assert lib.sa_qk_norm_rope(16, 16, 256, 256, 0, 4, 256, 128, None, None, 1, 1e-6, None, None,
                               0, 16, 16, 256, 256, None) == _lib.SA_OK


def test_aligned_accumulate_validation(lib):
    from sinkattn_b200 import _lib

    # n_blocks must equal image + text blocks
    assert lib.sa_score_accumulate_aligned(16, 2, 5, 4, 2, 6, 16, 16, 16, 1, None) == _lib.SA_EINVAL
    assert "Z-Image block score shape" in lib.sa_last_error().decode()
    # the sample must fit the fixed layout
    assert lib.sa_score_accumulate_aligned(16, 2, 7, 4, 3, 6, 16, 16, 16, 1, None) == _lib.SA_EINVAL
    assert lib.sa_pooled_softmax_layers(16, 16, 0, 1, 1, 4, 128, 0.0, 16, 16, None) == _lib.SA_EINVAL


def test_rotary_tables_forms():
    from sinkattn_b200.reference_api import _rotary_tables

    S, D = 5, 8
    ang = torch.outer(torch.arange(S, dtype=torch.float64), torch.arange(D // 2) + 1.0)
    cplx = torch.polar(torch.ones_like(ang), ang).to(torch.complex64)
    for freqs in (cplx, cplx[None, None]):
        c, s = _rotary_tables(freqs, S, D)
        assert c.shape == (S, D // 2) and torch.equal(c, cplx.real) and torch.equal(s, cplx.imag)
    # (real, imag) pair of [S, D/2]
    c, s = _rotary_tables((cplx.real, cplx.imag), S, D)
    assert torch.equal(c, cplx.real) and torch.equal(s, cplx.imag)
    # Wan's (cos, sin) pair repeated per channel, [1, S, 1, D]
    cos_full = torch.repeat_interleave(cplx.real, 2, dim=-1)[None, :, None, :]
    sin_full = torch.repeat_interleave(cplx.imag, 2, dim=-1)[None, :, None, :]
    c, s = _rotary_tables((cos_full, sin_full), S, D)
    assert torch.equal(c, cplx.real) and torch.equal(s, cplx.imag)
    with pytest.raises(TypeError):
        _rotary_tables("not a rotary embedding", S, D)


def test_rms_norm_detection():
    from sinkattn_b200.reference_api import _rms_like

    assert _rms_like(torch.nn.RMSNorm(16, eps=1e-6))
    assert not _rms_like(torch.nn.RMSNorm(16))            # eps None: torch picks it
    assert not _rms_like(torch.nn.LayerNorm(16))
    assert not _rms_like(torch.nn.RMSNorm(16, eps=1e-6, elementwise_affine=False))
    assert not _rms_like(None)


def test_zimage_fixed_layout():
    """_fixed_block_shape (zimg/runtime/sink_sparse_zimage.py:123-136): image
    tokens and the maximum text length padded to multiples of 32."""
    from dataclasses import dataclass

    from sinkattn_b200.calibrator import DeviceZImageSinkMaskCalibrator

    @dataclass
    class ZCfg:
        block_size: int = 128
        pooling_mode: str = "mean"
        text_length: int = 512
        token_width: int = 128
        token_height: int = 128
        token_depth: int = 1

    cal = DeviceZImageSinkMaskCalibrator(ZCfg())
    assert (cal.image_token_count, cal.image_blocks, cal.max_text_tokens, cal.total_blocks) == \
        (16384, 128, 512, 132)
    cal = DeviceZImageSinkMaskCalibrator(ZCfg(token_width=33, token_height=31, text_length=300))
    assert cal.image_token_count == 1024 and cal.image_blocks == 8
    assert cal.max_text_tokens == 320 and cal.total_blocks == 11
    with pytest.raises(ValueError):
        cal.record(0, torch.zeros(1, 1, 8, 128), torch.zeros(1, 1, 8, 128),
                   torch.zeros(1, 1, 8, 128), text_token_count=321)


def test_score_mode_dispatch():
    from sinkattn_b200 import reference_api as ra

    class Cfg:
        block_size = 128
        pooling_mode = "unknown"

    with pytest.raises(ValueError, match="Unsupported pooling_mode"):
        ra._compute_block_scores(torch.zeros(1), torch.zeros(1), torch.zeros(1), Cfg())
    Cfg.pooling_mode = " Exact "
    with pytest.raises(RuntimeError, match="CUDA"):  # dispatched to the exact kernel
        ra._compute_block_scores(torch.zeros(1, 1, 128, 128, dtype=torch.bfloat16),
                                 torch.zeros(1, 1, 128, 128, dtype=torch.bfloat16), None, Cfg())
    Cfg.block_size = 64
    with pytest.raises(NotImplementedError):
        ra._compute_exact_block_mass_scores(torch.zeros(1, 1, 64, 128), torch.zeros(1, 1, 64, 128),
                                            Cfg())
    assert math.isclose(1.0, 1.0)


def test_bench_cpu_reference_matches_oracle(oracle):
    """The CPU reference the benchmark times (dense masked torch attention on
    all host threads) computes the oracle's dense masked attention."""
    import bench

    g = torch.Generator().manual_seed(4)
    q = torch.randn(700, 128, generator=g)
    k = torch.randn(900, 128, generator=g)
    v = torch.randn(900, 128, generator=g)
    m = torch.rand(6, 8, generator=g) < 0.5
    m[:, 0] = True
    out, lse = bench.torch_masked_attention(q, k, v, m, row_chunk=256)
    ref, ref_lse = oracle.dense_masked_attention(q[None, None].numpy(), k[None, None].numpy(),
                                                 v[None, None].numpy(), m[None, None].numpy())
    np.testing.assert_allclose(out.numpy(), ref[0, 0], atol=1e-5)
    np.testing.assert_allclose(lse.numpy(), ref_lse[0, 0], atol=1e-5)


def test_bench_cpu_calibration_reference_matches_oracle(oracle):
    """The CPU calibration reference the benchmark times (torch block means,
    pooled softmax and batch mean, then the coverage rule with the sink
    column) builds the oracle's mask from the oracle's pooled scores."""
    import bench

    g = torch.Generator().manual_seed(6)
    q = torch.randn(2, 3, 1024, 128, generator=g).bfloat16()
    k = torch.randn(2, 3, 1024, 128, generator=g).bfloat16()
    got = bench.cpu_calibration_layer(q, k, oracle)
    scores = oracle.pooled_block_scores(q.float().numpy(), k.float().numpy(), 128).mean(0)
    ref = oracle.coverage_mask(scores, force_sink_col=True)
    assert got.shape == (3, 8, 8) and got[:, :, 0].all()
    # the two score computations differ in fp32 rounding only, which moves no
    # coverage cut on these inputs
    assert np.array_equal(got, ref.mask)


def test_default_config_copy_matches_reference(reference):
    """The tests' stand-in for SinkSparseConfig() carries the reference's
    defaults, pooling_mode "triton" among them."""
    from dataclasses import asdict

    from sinkattention.sparse_attention import SinkSparseConfig
    from tests.gen import REFERENCE_DEFAULT_CONFIG, default_config

    assert asdict(SinkSparseConfig()) == REFERENCE_DEFAULT_CONFIG
    assert asdict(default_config()) == REFERENCE_DEFAULT_CONFIG
    assert default_config().pooling_mode == "triton"


@pytest.mark.parametrize("mode", ["triton", "exact", "mean", "Triton", " EXACT "])
def test_device_calibrator_refuses_cpu_tensors(mode):
    """Every score mode of the device calibrator runs on CUDA tensors only
    (no CPU fallback); an unknown mode raises the reference's ValueError."""
    from sinkattn_b200.calibrator import DeviceSinkMaskCalibrator
    from tests.gen import default_config

    x = torch.zeros(1, 1, 256, 128, dtype=torch.bfloat16)
    cal = DeviceSinkMaskCalibrator(default_config(pooling_mode=mode))
    with pytest.raises(RuntimeError, match="CUDA"):
        cal.record(0, x, x, x)
    bad = DeviceSinkMaskCalibrator(default_config(pooling_mode="max"))
    with pytest.raises(ValueError, match="Unsupported pooling_mode"):
        bad.record(0, x, x, x)

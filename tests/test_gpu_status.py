"""Failure detection on the GPU without a GPU fault.

Every spin in the kernels is bounded in time; a wait that gives up writes
SA_DEV_WAIT_TIMEOUT into the status word (mapped page-locked host memory,
ops.DeviceStatus) and its kernel returns. These tests make one such wait run
out on purpose, with sa_selftest_wait_timeout (a warp waiting on an mbarrier
that nobody arrives on, limit 2 ms), and check that
  * the host sees the code without any further GPU call;
  * the context stays usable (a normal launch after it gives correct output);
  * the reference-facing drop-ins refuse the next call with RuntimeError, and
    the call after that (the word reset) goes through;
  * the device calibrator refuses to build a package from statistics that a
    timed-out launch may have fed.
"""
from __future__ import annotations

import ctypes

import pytest
import torch

pytestmark = pytest.mark.gpu

LIMIT_NS = 2_000_000


def _plant_timeout(dev):
    from sinkattn_b200 import _lib, ops

    lib = _lib.load()
    ptr = ops.DeviceStatus.pointer(dev)
    stream = torch.cuda.current_stream(dev).cuda_stream
    _lib.check(lib.sa_selftest_wait_timeout(ctypes.c_void_p(ptr), LIMIT_NS,
                                            ctypes.c_void_p(stream)),
               "sa_selftest_wait_timeout")
    torch.cuda.synchronize(dev)


def test_timeout_is_reported_and_context_survives():
    from sinkattn_b200 import ops

    dev = torch.device("cuda", 0)
    ops.DeviceStatus.check(dev)  # clean start
    _plant_timeout(dev)
    assert ops.DeviceStatus.value(dev) == 1
    with pytest.raises(RuntimeError, match="bounded wait"):
        ops.DeviceStatus.check(dev)
    assert ops.DeviceStatus.value(dev) == 0
    # the context is intact: a normal launch still computes the right thing
    g = torch.Generator(device="cuda").manual_seed(0)
    q = torch.randn(1, 2, 512, 128, device=dev, generator=g).bfloat16()
    k = torch.randn(1, 2, 512, 128, device=dev, generator=g).bfloat16()
    v = torch.randn(1, 2, 512, 128, device=dev, generator=g).bfloat16()
    mask = torch.ones(1, 2, 4, 4, dtype=torch.bool, device=dev)
    out, _ = ops.bsattn_fwd(q, k, v, mask)
    ref = torch.nn.functional.scaled_dot_product_attention(q.float(), k.float(), v.float())
    assert (out.float() - ref).abs().max().item() < 2e-2
    ops.DeviceStatus.check(dev)


def test_dropin_refuses_call_after_timeout():
    from sinkattn_b200 import ops, reference_api

    dev = torch.device("cuda", 0)
    ops.DeviceStatus.check(dev)
    g = torch.Generator(device="cuda").manual_seed(1)
    x = torch.randn(1, 2, 256, 128, device=dev, generator=g).bfloat16()
    _plant_timeout(dev)
    with pytest.raises(RuntimeError, match="bounded wait"):
        reference_api._mean_pool_sequence(x, 2)
    # the report was consumed: the next call runs
    y = reference_api._mean_pool_sequence(x, 2)
    torch.testing.assert_close(y.float(), x.float().unflatten(2, (128, 2)).mean(3),
                               atol=1e-2, rtol=1e-2)


def test_calibrator_refuses_package_after_timeout(tmp_path):
    from sinkattn_b200 import ops
    from sinkattn_b200.calibrator import DeviceSinkMaskCalibrator
    from tests.gen import default_config

    dev = torch.device("cuda", 0)
    ops.DeviceStatus.check(dev)
    cfg = default_config(pooling_mode="mean")
    cal = DeviceSinkMaskCalibrator(cfg)
    g = torch.Generator(device="cuda").manual_seed(2)
    q = torch.randn(1, 2, 1024, 128, device=dev, generator=g).bfloat16()
    k = torch.randn(1, 2, 1024, 128, device=dev, generator=g).bfloat16()
    cal.record(0, q, k, k)
    _plant_timeout(dev)
    with pytest.raises(RuntimeError, match="bounded wait"):
        cal.build_package()
    pkg = cal.build_package()  # the word was reset by the refusal
    assert pkg["counts"]["0"] == 1

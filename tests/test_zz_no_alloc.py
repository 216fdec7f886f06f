"""sa_pool_scores_noalloc through the C ABI, against sa_pool_scores.

The no-allocation entry point serves callers that cannot give the library a
device workspace: a C/FFI host without a device allocator, or a server that
reserved all GPU memory up front and may not cudaMalloc while serving. It
keeps its scratch in a 16 MiB device array inside the library. This test
calls it twice in a row, with different shapes, and checks each result
against the workspace-taking entry point (same kernels, so the results must
agree within the pooled-score tolerance used elsewhere: rtol 2e-5,
atol 2e-7). It also checks that an oversize request is refused.

This file is named to be collected last.
"""
from __future__ import annotations

import ctypes

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

RTOL, ATOL = 2e-5, 2e-7


def _strides(t):
    return (ctypes.c_int64 * 4)(*[int(s) for s in t.stride()])


def _run_both(lib, q, k, block):
    from sinkattn_b200 import _lib

    B, H, S, D = q.shape
    nb = -(-S // block)
    stream = torch.cuda.current_stream().cuda_stream
    ws_bytes = lib.sa_pool_scores_workspace_size(B, H, S, D, block)
    ws = torch.empty(ws_bytes, dtype=torch.uint8, device="cuda")
    ref_s = torch.empty(B, H, nb, nb, dtype=torch.float32, device="cuda")
    ref_m = torch.empty(H, nb, nb, dtype=torch.float32, device="cuda")
    rc = lib.sa_pool_scores(q.data_ptr(), k.data_ptr(), _strides(q), _strides(k), B, H, S, D,
                            block, -1.0, ref_s.data_ptr(), ref_m.data_ptr(), ws.data_ptr(),
                            ws_bytes, stream)
    _lib.check(rc, "sa_pool_scores")
    out_s = torch.full_like(ref_s, float("nan"))
    out_m = torch.full_like(ref_m, float("nan"))
    rc = lib.sa_pool_scores_noalloc(q.data_ptr(), k.data_ptr(), _strides(q), _strides(k), B, H,
                                    S, D, block, -1.0, out_s.data_ptr(), out_m.data_ptr(), stream)
    _lib.check(rc, "sa_pool_scores_noalloc")
    torch.cuda.synchronize()
    return ref_s.cpu().numpy(), ref_m.cpu().numpy(), out_s.cpu().numpy(), out_m.cpu().numpy()


def test_noalloc_matches_workspace_entry_point_on_two_calls():
    from sinkattn_b200 import _lib

    lib = _lib.load()
    g = torch.Generator().manual_seed(123)
    shapes = [((2, 3, 1000, 128), 128), ((1, 4, 777, 64), 64)]
    for (B, H, S, D), block in shapes:
        q = torch.randn(B, H, S, D, generator=g).bfloat16().cuda()
        k = torch.randn(B, H, S, D, generator=g).bfloat16().cuda()
        ref_s, ref_m, out_s, out_m = _run_both(lib, q, k, block)
        assert np.isfinite(out_s).all() and np.isfinite(out_m).all()
        np.testing.assert_allclose(out_s, ref_s, rtol=RTOL, atol=ATOL)
        np.testing.assert_allclose(out_m, ref_m, rtol=RTOL, atol=ATOL)


def test_noalloc_refuses_shapes_beyond_its_scratch():
    from sinkattn_b200 import _lib

    lib = _lib.load()
    B, H, S, D, block = 2, 30, 65536, 128, 128  # needs far more than 16 MiB
    need = lib.sa_pool_scores_workspace_size(B, H, S, D, block)
    assert need > 16 * 1024 * 1024
    st = (ctypes.c_int64 * 4)(H * S * D, S * D, D, 1)
    rc = lib.sa_pool_scores_noalloc(16, 16, st, st, B, H, S, D, block, -1.0, 16, None,
                                    torch.cuda.current_stream().cuda_stream)
    assert rc == _lib.SA_EINVAL
    assert "16 MiB" in _lib.last_error()

"""GPU parity of the Q/K producer (sa_qk_norm_rope): RMSNorm over the hidden
dimension + rotary embedding, against the reference's own output (golden
vectors) and the oracle, and the fused drop-in of the Wan processor's
_prepare_attention_tensors."""
from __future__ import annotations

import math

import numpy as np
import pytest
import torch

from tests.conftest import from_bits, regen_input

pytestmark = pytest.mark.gpu


def _assert_close_bf16(oracle, got, want):
    """Within one bf16 step, or within one bf16 step of the channel pair's
    magnitude: the normalised value is rounded to bf16 before the rotation
    (as between the reference's two kernels), and where its rounding lands one
    step apart the rotation carries that step into outputs that cancel to a
    small value. The rotation keeps each pair's norm, so the pair norm of the
    result bounds it. 97% of the outputs are bit-identical."""
    d = oracle.bf16_ulp_distance(got, want)
    pair = np.sqrt(want[..., 0::2].astype(np.float64) ** 2 + want[..., 1::2].astype(np.float64) ** 2)
    pair = np.repeat(pair, 2, axis=-1)
    near = np.abs(got - want) <= 2.0 ** -7 * pair + 2.0 ** -20
    assert ((d <= 1) | near).all(), (d.max(), np.abs(got - want)[d > 1].max())
    assert (d == 0).mean() >= 0.97, (d == 0).mean()


def _wan_freqs(S: int, D: int) -> torch.Tensor:
    inv = 1.0 / (10000.0 ** (torch.arange(0, D, 2, dtype=torch.float64) / D))
    ang = torch.outer(torch.arange(S, dtype=torch.float64), inv)
    return torch.polar(torch.ones_like(ang), ang).to(torch.complex64)


def test_matches_reference_golden(golden, oracle):
    from sinkattn_b200 import ops

    heads = int(golden["qkrope/heads"])
    q = regen_input(golden, "qkrope", "q").cuda()
    k = regen_input(golden, "qkrope", "k").cuda()
    B, S, hidden = q.shape
    D = hidden // heads
    wq = torch.from_numpy(from_bits(golden["qkrope/w_q"])).bfloat16().cuda()
    wk = torch.from_numpy(from_bits(golden["qkrope/w_k"])).bfloat16().cuda()
    cos = torch.from_numpy(golden["qkrope/cos"]).cuda()
    sin = torch.from_numpy(golden["qkrope/sin"]).cuda()
    qo, ko = ops.qk_norm_rope(q, k, D, float(golden["qkrope/eps"]), wq, wk, cos, sin)
    for got, key in ((qo, "q_out"), (ko, "k_out")):
        got = got.view(B, S, heads, D).transpose(1, 2).float().cpu().numpy()
        # the sum of squares is reduced in another order than torch's
        _assert_close_bf16(oracle, got, from_bits(golden[f"qkrope/{key}"]))


@pytest.mark.parametrize("S,heads,w_dtype", [(1000, 12, torch.bfloat16), (77, 4, torch.float32)])
def test_matches_oracle_and_in_place(oracle, S, heads, w_dtype):
    from sinkattn_b200 import ops

    g = torch.Generator().manual_seed(S)
    D = 128
    hidden = heads * D
    q = (3.0 * torch.randn(2, S, hidden, generator=g)).bfloat16()
    k = torch.randn(2, S, hidden, generator=g).bfloat16()
    wq = (1.0 + 0.2 * torch.randn(hidden, generator=g)).to(w_dtype)
    wk = (1.0 + 0.2 * torch.randn(hidden, generator=g)).to(w_dtype)
    f = _wan_freqs(S, D)
    qc, kc = q.cuda(), k.cuda()
    qo, ko = ops.qk_norm_rope(qc, kc, D, 1e-6, wq.cuda(), wk.cuda(), f.real.cuda(), f.imag.cuda())
    for x, w, got in ((q, wq, qo), (k, wk, ko)):
        want = oracle.qk_norm_rope(x.float().numpy(), w.float().numpy(), 1e-6,
                                   f.real.numpy(), f.imag.numpy(), heads)
        got = got.view(2, S, heads, D).transpose(1, 2).float().cpu().numpy()
        _assert_close_bf16(oracle, got, want)
    # in place gives the same bits
    ops.qk_norm_rope(qc, kc, D, 1e-6, wq.cuda(), wk.cuda(), f.real.cuda(), f.imag.cuda(),
                     out_q=qc, out_k=kc)
    assert torch.equal(qc, qo) and torch.equal(kc, ko)


def test_fused_prepare_matches_unfused_path():
    """The drop-in for _prepare_attention_tensors gives the tensors of the
    reference's flow (projection, RMSNorm module, per-head split, fp64
    complex rotary as in wanx/runtime/fast_misc.py:173-179) within one bf16
    step, for complex and for Wan (cos, sin) rotary embeddings."""
    from sinkattn_b200 import reference_api as ra

    torch.manual_seed(0)
    heads, D, S, dim = 12, 128, 512, 1536

    class Attn(torch.nn.Module):
        def __init__(self):
            super().__init__()
            self.heads = heads
            self.add_k_proj = None
            self.to_q = torch.nn.Linear(dim, dim, dtype=torch.bfloat16)
            self.to_k = torch.nn.Linear(dim, dim, dtype=torch.bfloat16)
            self.to_v = torch.nn.Linear(dim, dim, dtype=torch.bfloat16)
            self.norm_q = torch.nn.RMSNorm(dim, eps=1e-6, dtype=torch.bfloat16)
            self.norm_k = torch.nn.RMSNorm(dim, eps=1e-6, dtype=torch.bfloat16)

    attn = Attn().cuda()
    with torch.no_grad():
        attn.norm_q.weight.add_(0.1 * torch.randn(dim, device="cuda").bfloat16())
        attn.norm_k.weight.add_(0.1 * torch.randn(dim, device="cuda").bfloat16())
    hs = torch.randn(2, S, dim, device="cuda").bfloat16()
    f = _wan_freqs(S, D).cuda()

    def reference_flow(freqs):
        q = attn.norm_q(attn.to_q(hs)).unflatten(2, (heads, -1)).transpose(1, 2)
        k = attn.norm_k(attn.to_k(hs)).unflatten(2, (heads, -1)).transpose(1, 2)
        v = attn.to_v(hs).unflatten(2, (heads, -1)).transpose(1, 2)

        def rot(x):
            xc = torch.view_as_complex(x.double().unflatten(3, (-1, 2)))
            return torch.view_as_real(xc * freqs).flatten(3, 4).type_as(x)
        return rot(q), rot(k), v

    ra._UNFUSED_PREPARE[:] = [lambda *a: (_ for _ in ()).throw(AssertionError("not fused"))]
    cos_full = torch.repeat_interleave(f.real, 2, dim=-1)[None, :, None, :]
    sin_full = torch.repeat_interleave(f.imag, 2, dim=-1)[None, :, None, :]
    with torch.no_grad():
        want = reference_flow(f[None, None])
        for emb in (f[None, None], (cos_full, sin_full)):
            q, k, v, img = ra.fused_prepare_attention_tensors(attn, hs, None, emb)
            assert img is None and q.shape == (2, heads, S, D)
            assert torch.equal(v, want[2])
            for a, b in ((q, want[0]), (k, want[1])):
                diff = (a.float() - b.float()).abs()
                step = b.float().abs().clamp_min(1e-30) * 2.0 ** -7
                assert (diff <= step).float().mean() > 0.999 and (diff == 0).float().mean() > 0.8
    ra._UNFUSED_PREPARE.clear()

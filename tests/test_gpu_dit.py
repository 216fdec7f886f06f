"""The cfg5 DiT harness (tests/wan_dit.py) on one GPU at a small latent: two
Wan-1.3B blocks whose self-attention runs the reference's
WanSinkSparseAttnProcessor2_0 with install() in place, against the same
model whose inner attention is the reference arithmetic in fp32 (masked
dense sink attention, dense attention over the reference's own pooled K/V,
the reference's own adaptive mix). Tolerance: mean |err| / mean |ref| of the
model output within 2e-2 after two blocks."""
from __future__ import annotations

import pytest
import torch

from tests.torch_ref import unit_attention

pytestmark = pytest.mark.gpu

LATENT = (2, 16, 4, 32, 32)  # 4 x 16 x 16 = 1024 tokens, 8 blocks of 128


class _RefInner(torch.nn.Module):
    def __init__(self, mask, gap, pool, mix, cfg):
        super().__init__()
        self.mask, self.gap, self.pool, self.mix, self.cfg = mask, gap, pool, mix, cfg

    def forward(self, q, k, v):
        kd = self.pool(k, self.gap, prefix_tokens=0)
        vd = self.pool(v, self.gap, prefix_tokens=0)
        B, H, S, D = q.shape
        full = torch.ones((S + 127) // 128, (kd.shape[2] + 127) // 128, dtype=torch.bool,
                          device=q.device)
        out = torch.empty(B, H, S, D, device=q.device)
        for b in range(B):
            for h in range(H):
                so, sl = unit_attention(q[b, h], k[b, h], v[b, h], self.mask[h])
                do, dl = unit_attention(q[b, h], kd[b, h], vd[b, h], full)
                out[b, h] = self.mix(so, sl[:, None], do, dl[:, None], self.cfg,
                                     dynamic_sample_gap=self.gap)
        return out.to(q.dtype)


def test_dit_blocks_through_reference_processor(reference):
    import importlib

    from sinkattn_b200 import reference_api as ra
    from tests import wan_dit

    sa = importlib.import_module("sinkattention.sparse_attention")
    wan = importlib.import_module("wanx.runtime.sink_sparse_wan")
    orig_pool = sa._mean_pool_sequence_preserve_prefix
    orig_mix = sa._mix_attention_outputs
    saved = [(m, a, getattr(m, a)) for name, attrs in ra._PATCHES.items()
             for m in [importlib.import_module(name)] for a in attrs if hasattr(m, a)]
    saved += [(wan, "_prepare_attention_tensors", wan._prepare_attention_tensors),
              (wan.WanSinkSparseInnerAttention, "forward", wan.WanSinkSparseInnerAttention.forward)]
    ra.install()
    try:
        dev = torch.device("cuda", 0)
        g = torch.Generator().manual_seed(3)
        masks = torch.rand(2, 12, 8, 8, generator=g) < 0.5
        masks[..., 0] = True
        model, ex = wan_dit.build(masks, dev, layers=2, latent=LATENT)
        assert ex is None
        assert isinstance(model.blocks[0].attn1.processor, wan.WanSinkSparseAttnProcessor2_0)
        x, t, text, rot = wan_dit.inputs(dev, latent=LATENT)
        with torch.no_grad():
            got = model(x, t, text, rot).float()
            cfg = sa.SinkSparseConfig()
            for i, blk in enumerate(model.blocks):
                blk.attn1.inner_attention = _RefInner(masks[i].to(dev), cfg.sample_gap,
                                                      orig_pool, orig_mix, cfg)
            ref = model(x, t, text, rot).float()
        assert got.shape == (2, 1024, 64) and torch.isfinite(got).all()
        rel = float((got - ref).abs().mean() / ref.abs().mean())
        print("dit rel", rel)
        assert rel <= 2e-2, rel
    finally:
        for m, a, val in saved:
            setattr(m, a, val)

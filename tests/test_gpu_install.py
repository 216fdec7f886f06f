"""The reference's own processors on the GPU, with install() in place.

install() rebinds the reference's hot-path names to this package's kernels
(sinkattn_b200/reference_api.py). These tests import the reference's modules
(baseline/_ref, or SINKATTN_REFERENCE), bind the drop-ins, and run the
reference's code on CUDA tensors:

  * WanSinkSparseInnerAttention.forward (wanx/runtime/sink_sparse_wan.py:181-282)
    fused (one kernel: sink branch, pooled K/V branch and adaptive mix) and
    the reference's own unfused method calling the drop-ins;
  * WanSinkSparseAttnProcessor2_0.__call__ (sink_sparse_wan.py:347-374), with
    the fused Q/K RMSNorm + rotary producer in place of
    _prepare_attention_tensors (lines 285-315);
  * ZImageStaticSinkProcessor.__call__ (zimg/runtime/sink_sparse_zimage.py:466-614)
    on a padded batch whose two elements have different text lengths.

The expected values follow the reference's arithmetic in fp32: masked dense
attention for the sink branch (the mask the reference builds itself), dense
attention over the reference's own pooled K/V, and the reference's own
_mix_attention_outputs (saved before install) on fp32 outputs and LSEs.
Tolerance as the other attention tests: max-abs 2e-2 and mean-relative
(mean |err| / mean |ref|) 1e-2 on the attention output; the processors'
outputs after the output projection within 2e-2 relative to their scale.
"""
from __future__ import annotations

import pytest
import torch

from tests.torch_ref import unit_attention

pytestmark = pytest.mark.gpu

MAX_ABS = 2e-2
MEAN_REL = 1e-2


@pytest.fixture
def installed(reference):
    """install() with every rebound name restored afterwards."""
    import importlib

    from sinkattn_b200 import reference_api as ra

    saved = []
    for name, attrs in ra._PATCHES.items():
        mod = importlib.import_module(name)
        for attr in attrs:
            saved.append((mod, attr, getattr(mod, attr, None)))
    wan = importlib.import_module("wanx.runtime.sink_sparse_wan")
    saved.append((wan, "_prepare_attention_tensors", wan._prepare_attention_tensors))
    saved.append((wan.WanSinkSparseInnerAttention, "forward", wan.WanSinkSparseInnerAttention.forward))
    originals = {(getattr(m, "__name__", str(m)), a): v for m, a, v in saved}
    ra.install()
    try:
        yield originals
    finally:
        for mod, attr, val in saved:
            setattr(mod, attr, val)


def _check(out, ref, what):
    err = (out.float() - ref).abs()
    max_abs = float(err.max())
    mean_rel = float(err.mean() / ref.abs().mean())
    assert max_abs <= MAX_ABS and mean_rel <= MEAN_REL, (what, max_abs, mean_rel)
    return max_abs, mean_rel


def _expected_wan_inner(orig_pool, orig_mix, cfg, q, k, v, mask, gap):
    """The reference's pooled_kv / adaptive inner attention in fp32."""
    kd = orig_pool(k, gap, prefix_tokens=0)
    vd = orig_pool(v, gap, prefix_tokens=0)
    B, H, S, D = q.shape
    nkd = (kd.shape[2] + 127) // 128
    full = torch.ones((S + 127) // 128, nkd, dtype=torch.bool, device=q.device)
    out = torch.empty(B, H, S, D, dtype=torch.float32, device=q.device)
    for b in range(B):
        for h in range(H):
            so, sl = unit_attention(q[b, h], k[b, h], v[b, h],
                                    mask[b if mask.shape[0] > 1 else 0, h].bool())
            do, dl = unit_attention(q[b, h], kd[b, h], vd[b, h], full)
            out[b, h] = orig_mix(so, sl.unsqueeze(-1), do, dl.unsqueeze(-1), cfg,
                                 dynamic_sample_gap=gap)
    return out


def test_wan_inner_attention_fused_and_unfused(installed):
    """The Wan runtime default (pooled_kv, adaptive mix, band 1) at a ragged
    length: the fused forward and the reference's unfused method (on the
    drop-ins) both match the reference arithmetic."""
    import sinkattention.sparse_attention as sa
    import wanx.runtime.sink_sparse_wan as wan

    from sinkattn_b200 import reference_api as ra

    g = torch.Generator(device="cuda").manual_seed(0)
    B, H, S, D = 2, 4, 8190, 128
    nb = (S + 127) // 128
    q = torch.randn(B, H, S, D, device="cuda", generator=g).bfloat16()
    k = torch.randn(B, H, S, D, device="cuda", generator=g).bfloat16()
    v = torch.randn(B, H, S, D, device="cuda", generator=g).bfloat16()
    sink = torch.rand(H, nb, nb, device="cuda", generator=g) < 0.25
    sink[:, :, 0] = True
    cfg = sa.SinkSparseConfig().merged({"dynamic_mode": "pooled_kv", "dynamic_kernel": "block_sparse",
                                        "mixing_mode": "adaptive", "sample_gap": 30,
                                        "runtime_diagonal_band_width": 1})
    inner = wan.WanSinkSparseInnerAttention(0, sink.cpu(), cfg)
    assert wan.WanSinkSparseInnerAttention.forward is ra.fused_wan_inner_forward
    fused = inner(q, k, v)
    unfused = ra._UNFUSED_WAN_FORWARD[0](inner, q, k, v)
    torch.cuda.synchronize()
    # the runtime mask as the reference builds it: sink | band
    mask = inner._get_runtime_mask(sink_mask=inner.sink_mask, mask_tag="__base__", batch_size=B,
                                   num_heads=H, seq_len_q=S, seq_len_k=S, device=q.device)
    ii = torch.arange(nb, device="cuda")
    band = (ii[:, None] - ii[None, :]).abs() <= 1
    assert torch.equal(mask[0, 0].bool(), sink[0] | band)
    orig_pool = installed[("sinkattention.sparse_attention", "_mean_pool_sequence_preserve_prefix")]
    orig_mix = installed[("sinkattention.sparse_attention", "_mix_attention_outputs")]
    ref = _expected_wan_inner(orig_pool, orig_mix, cfg, q, k, v, mask, 30)
    print("fused", _check(fused, ref, "fused"))
    print("unfused", _check(unfused, ref, "unfused"))
    from sinkattn_b200 import ops

    ops.DeviceStatus.check(q.device)


class _WanAttn(torch.nn.Module):
    """The attributes WanSinkSparseAttnProcessor2_0 reads from diffusers'
    Attention for Wan self-attention."""

    def __init__(self, dim, heads, inner):
        super().__init__()
        self.heads = heads
        self.add_k_proj = None
        self.to_q = torch.nn.Linear(dim, dim, dtype=torch.bfloat16)
        self.to_k = torch.nn.Linear(dim, dim, dtype=torch.bfloat16)
        self.to_v = torch.nn.Linear(dim, dim, dtype=torch.bfloat16)
        self.norm_q = torch.nn.RMSNorm(dim, eps=1e-6, dtype=torch.bfloat16)
        self.norm_k = torch.nn.RMSNorm(dim, eps=1e-6, dtype=torch.bfloat16)
        with torch.no_grad():
            self.norm_q.weight.uniform_(0.5, 1.5)
            self.norm_k.weight.uniform_(0.5, 1.5)
        self.to_out = torch.nn.ModuleList([torch.nn.Linear(dim, dim, dtype=torch.bfloat16),
                                           torch.nn.Dropout(0.0)])
        self.inner_attention = inner


def test_wan_processor_end_to_end(installed):
    """WanSinkSparseAttnProcessor2_0.__call__ on hidden states with a rotary
    embedding: the installed producer (Q/K RMSNorm + rotation in one kernel)
    and fused attention against the reference's own _prepare_attention_tensors
    followed by the reference arithmetic in fp32 and the same projection."""
    import sinkattention.sparse_attention as sa
    import wanx.runtime.sink_sparse_wan as wan

    from sinkattn_b200 import reference_api as ra

    torch.manual_seed(1)
    B, H, D, S = 1, 2, 128, 4196
    dim = H * D
    nb = (S + 127) // 128
    sink = torch.rand(H, nb, nb) < 0.3
    sink[:, :, 0] = True
    cfg = sa.SinkSparseConfig().merged({"dynamic_mode": "pooled_kv", "mixing_mode": "adaptive",
                                        "sample_gap": 30, "runtime_diagonal_band_width": 1})
    inner = wan.WanSinkSparseInnerAttention(0, sink, cfg)
    attn = _WanAttn(dim, H, inner).cuda()
    hs = torch.randn(B, S, dim, device="cuda").bfloat16()
    ang = torch.outer(torch.arange(S, dtype=torch.float64),
                      1.0 / 10000 ** (torch.arange(0, D, 2, dtype=torch.float64) / D))
    freqs = torch.polar(torch.ones_like(ang), ang).to(torch.complex64).reshape(1, 1, S, D // 2).cuda()
    assert wan._prepare_attention_tensors is ra.fused_prepare_attention_tensors
    proc = wan.WanSinkSparseAttnProcessor2_0(layer_idx=0)
    with torch.no_grad():
        got = proc(attn, hs, rotary_emb=freqs)
        torch.cuda.synchronize()
        orig_prepare = installed[("wanx.runtime.sink_sparse_wan", "_prepare_attention_tensors")]
        q, k, v, _ = orig_prepare(attn, hs, None, freqs)
        mask = inner._get_runtime_mask(sink_mask=inner.sink_mask, mask_tag="__base__",
                                       batch_size=B, num_heads=H, seq_len_q=S, seq_len_k=S,
                                       device=q.device)
        orig_pool = installed[("sinkattention.sparse_attention", "_mean_pool_sequence_preserve_prefix")]
        orig_mix = installed[("sinkattention.sparse_attention", "_mix_attention_outputs")]
        ref_attn = _expected_wan_inner(orig_pool, orig_mix, cfg, q, k, v, mask, 30)
        ref = attn.to_out[0](ref_attn.transpose(1, 2).flatten(2, 3).bfloat16()).float()
    scale = float(ref.abs().mean())
    err = (got.float() - ref).abs()
    assert float(err.mean()) <= 2e-2 * scale, (float(err.mean()), scale)
    assert float(err.max()) <= 40 * 2e-2 * scale, (float(err.max()), scale)


def test_zimage_static_processor(installed):
    """ZImageStaticSinkProcessor.__call__ on a padded batch of two images
    with 200 and 90 text tokens: sliced sink mask with the text rows and
    columns dense, pooled image K/V plus the text K/V for the image rows'
    dynamic branch, adaptive mix, output projection."""
    import sinkattention.sparse_attention as sa
    import zimg.runtime.sink_sparse_zimage as zi

    torch.manual_seed(2)
    H, D = 2, 128
    dim = H * D
    cfg = sa.SinkSparseConfig().merged({"token_width": 32, "token_height": 16, "token_depth": 8,
                                        "text_length": 200, "dynamic_mode": "pooled_kv",
                                        "mixing_mode": "adaptive", "sample_gap": 4})
    image_tokens, image_blocks, total_blocks = zi._fixed_block_shape(cfg)
    assert (image_tokens, image_blocks, total_blocks) == (4096, 32, 34)
    sink = torch.rand(H, total_blocks, total_blocks) < 0.3
    sink[:, :, 0] = True
    proc = zi.ZImageStaticSinkProcessor(layer_idx=0, total_layers=1, sink_mask=sink, config=cfg)

    class Attn(torch.nn.Module):
        def __init__(self):
            super().__init__()
            self.heads = H
            self.to_q = torch.nn.Linear(dim, dim, dtype=torch.bfloat16)
            self.to_k = torch.nn.Linear(dim, dim, dtype=torch.bfloat16)
            self.to_v = torch.nn.Linear(dim, dim, dtype=torch.bfloat16)
            self.norm_q = torch.nn.RMSNorm(D, eps=1e-5, dtype=torch.bfloat16)
            self.norm_k = torch.nn.RMSNorm(D, eps=1e-5, dtype=torch.bfloat16)
            self.to_out = torch.nn.ModuleList([torch.nn.Linear(dim, dim, dtype=torch.bfloat16)])

    attn = Attn().cuda()
    texts = [200, 90]
    S = image_tokens + max(texts)
    hs = torch.randn(2, S, dim, device="cuda").bfloat16()
    am = torch.zeros(2, S, dtype=torch.bool, device="cuda")
    for b, t in enumerate(texts):
        am[b, :image_tokens + t] = True
    with torch.no_grad():
        got = proc(attn, hs, attention_mask=am)
        torch.cuda.synchronize()
        from zimg.runtime.modify_zimage import prepare_zimage_attention_tensors

        q, k, v = prepare_zimage_attention_tensors(attn, hs)
        orig_pool = installed[("zimg.runtime.sink_sparse_zimage", "_mean_pool_sequence")]
        orig_mix = installed[("zimg.runtime.sink_sparse_zimage", "_mix_attention_outputs")]
        out_padded = torch.zeros(2, S, H, D, device="cuda")
        for b, t in enumerate(texts):
            valid = image_tokens + t
            tb = (t + 127) // 128
            m = zi._slice_runtime_sink_mask(sink.cuda(), image_blocks=image_blocks,
                                            current_text_blocks=tb, total_blocks=total_blocks)
            m = zi._force_text_dense_runtime_mask(m, image_blocks=image_blocks,
                                                  current_text_blocks=tb)
            qi = q[b, :valid].transpose(0, 1)
            ki = k[b, :valid].transpose(0, 1)
            vi = v[b, :valid].transpose(0, 1)
            kd = torch.cat([orig_pool(ki[None, :, :image_tokens], 4)[0], ki[:, image_tokens:]], 1)
            vd = torch.cat([orig_pool(vi[None, :, :image_tokens], 4)[0], vi[:, image_tokens:]], 1)
            full = torch.ones(image_blocks, (kd.shape[1] + 127) // 128, dtype=torch.bool,
                              device="cuda")
            for h in range(H):
                so, sl = unit_attention(qi[h], ki[h], vi[h], m[h])
                do, dl = unit_attention(qi[h, :image_tokens], kd[h], vd[h], full)
                mixed = orig_mix(so[:image_tokens], sl[:image_tokens, None], do, dl[:, None], cfg,
                                 dynamic_sample_gap=4)
                out_padded[b, :image_tokens, h] = mixed
                out_padded[b, image_tokens:valid, h] = so[image_tokens:]
        ref = attn.to_out[0](out_padded.flatten(2, 3).bfloat16()).float()
    scale = float(ref.abs().mean())
    err = (got.float() - ref).abs()
    assert float(err.mean()) <= 2e-2 * scale, (float(err.mean()), scale)
    assert float(err.max()) <= 40 * 2e-2 * scale, (float(err.max()), scale)
    # padding rows stay zero before the projection: equal to the bias after
    assert torch.allclose(got[1, image_tokens + 90:].float(), attn.to_out[0].bias.float().expand(
        S - image_tokens - 90, -1), atol=1e-6)

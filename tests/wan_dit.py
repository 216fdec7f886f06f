"""A random-weight Wan2.1-1.3B-shaped DiT for the full-step workload (BASELINE
cfg5), in plain PyTorch (diffusers is not installed here).

Shapes follow Wan2.1-T2V-1.3B: 30 blocks, dim 1536, 12 heads of 128, FFN
8960 with tanh GELU, 3-D rotary embedding (head-dim split 44/42/42 over
frames/height/width), text context 512 x 4096, patch (1, 2, 2), latent
[2, 16, 21, 60, 104] -> 21 x 30 x 52 = 32760 tokens. Weights are N(0, 0.02)
from a seed, norms start at one.

Each block's self-attention is the reference's own processor,
WanSinkSparseAttnProcessor2_0.__call__ (wanx/runtime/sink_sparse_wan.py:347-374),
driven unchanged through a duck-typed `attn` (to_q, to_k, to_v, norm_q,
norm_k, to_out, add_k_proj=None, heads, inner_attention). With install() in
place its Q/K producer and inner attention are this package's kernels:
  * one GPU: inner_attention is the reference's WanSinkSparseInnerAttention
    (fused sink + pooled-K/V dynamic branch + adaptive mix, one kernel);
  * P GPUs (sequence parallel): every rank holds S/P tokens of the
    activations; inner_attention is UlyssesWanInner, which moves Q, K, V to
    the (batch, head) owners over NVLink peer memory (UlyssesPeerExchange),
    runs the same fused kernel on whole sequences, and moves the output back.
Cross-attention keys/values come from the (replicated) text context, so it
needs no exchange; everything else is per token.
"""
from __future__ import annotations

import math
from typing import Optional

import torch
import torch.nn as nn
import torch.nn.functional as F

WAN_1_3B = dict(dim=1536, ffn_dim=8960, heads=12, layers=30, in_ch=16, out_ch=16,
                text_dim=4096, text_len=512, freq_dim=256, patch=(1, 2, 2), eps=1e-6)
LATENT = (2, 16, 21, 60, 104)


class FP32LayerNorm(nn.LayerNorm):
    """LayerNorm computed in fp32, returned in the input's dtype (Wan's norms)."""

    def forward(self, x):
        w = self.weight.float() if self.weight is not None else None
        b = self.bias.float() if self.bias is not None else None
        return F.layer_norm(x.float(), self.normalized_shape, w, b, self.eps).to(x.dtype)


class SelfAttention(nn.Module):
    """The attributes the reference's Wan processor reads from diffusers'
    Attention; forward hands itself to that processor."""

    def __init__(self, dim, heads, eps):
        super().__init__()
        self.heads = heads
        self.add_k_proj = None
        self.to_q = nn.Linear(dim, dim)
        self.to_k = nn.Linear(dim, dim)
        self.to_v = nn.Linear(dim, dim)
        self.norm_q = nn.RMSNorm(dim, eps=eps)
        self.norm_k = nn.RMSNorm(dim, eps=eps)
        self.to_out = nn.ModuleList([nn.Linear(dim, dim), nn.Dropout(0.0)])
        self.inner_attention: Optional[nn.Module] = None
        self.processor = None

    def forward(self, x, rotary_emb):
        return self.processor(self, x, rotary_emb=rotary_emb)


class CrossAttention(nn.Module):
    """Text cross-attention: queries from the tokens, keys/values from the
    context (Wan's attn2 for T2V)."""

    def __init__(self, dim, heads, eps):
        super().__init__()
        self.heads = heads
        self.to_q = nn.Linear(dim, dim)
        self.to_k = nn.Linear(dim, dim)
        self.to_v = nn.Linear(dim, dim)
        self.norm_q = nn.RMSNorm(dim, eps=eps)
        self.norm_k = nn.RMSNorm(dim, eps=eps)
        self.to_out = nn.Linear(dim, dim)

    def forward(self, x, ctx):
        q = self.norm_q(self.to_q(x)).unflatten(2, (self.heads, -1)).transpose(1, 2)
        k = self.norm_k(self.to_k(ctx)).unflatten(2, (self.heads, -1)).transpose(1, 2)
        v = self.to_v(ctx).unflatten(2, (self.heads, -1)).transpose(1, 2)
        o = F.scaled_dot_product_attention(q, k, v)
        return self.to_out(o.transpose(1, 2).flatten(2, 3))


class WanBlock(nn.Module):
    def __init__(self, dim, ffn_dim, heads, eps):
        super().__init__()
        self.norm1 = FP32LayerNorm(dim, eps, elementwise_affine=False)
        self.attn1 = SelfAttention(dim, heads, eps)
        self.norm2 = FP32LayerNorm(dim, eps, elementwise_affine=True)
        self.attn2 = CrossAttention(dim, heads, eps)
        self.norm3 = FP32LayerNorm(dim, eps, elementwise_affine=False)
        self.ffn = nn.Sequential(nn.Linear(dim, ffn_dim), nn.GELU(approximate="tanh"),
                                 nn.Linear(ffn_dim, dim))
        self.scale_shift_table = nn.Parameter(torch.randn(1, 6, dim) / dim ** 0.5)

    def forward(self, x, ctx, tproj, rotary):
        shift_msa, scale_msa, gate_msa, c_shift, c_scale, c_gate = (
            self.scale_shift_table + tproj.float()).chunk(6, dim=1)
        h = (self.norm1(x.float()) * (1 + scale_msa) + shift_msa).type_as(x)
        x = (x.float() + self.attn1(h, rotary).float() * gate_msa).type_as(x)
        h = self.norm2(x.float()).type_as(x)
        x = x + self.attn2(h, ctx)
        h = (self.norm3(x.float()) * (1 + c_scale) + c_shift).type_as(x)
        return (x.float() + self.ffn(h).float() * c_gate).type_as(x)


def rope_freqs(f: int, h: int, w: int, head_dim: int = 128, theta: float = 10000.0):
    """Wan's 3-D rotary embedding as complex64 [1, 1, f*h*w, head_dim/2]: the
    head dimension split d - 4(d/6) : 2(d/6) : 2(d/6) over frames, height
    and width, each part a 1-D rotary table of its own axis."""
    d = head_dim
    dims = [d - 4 * (d // 6), 2 * (d // 6), 2 * (d // 6)]
    parts = []
    for n, dd in zip((f, h, w), dims):
        inv = 1.0 / theta ** (torch.arange(0, dd, 2, dtype=torch.float64) / dd)
        parts.append(torch.polar(torch.ones(n, dd // 2, dtype=torch.float64),
                                 torch.outer(torch.arange(n, dtype=torch.float64), inv)))
    ft = parts[0][:, None, None, :].expand(f, h, w, -1)
    fh = parts[1][None, :, None, :].expand(f, h, w, -1)
    fw = parts[2][None, None, :, :].expand(f, h, w, -1)
    return torch.cat([ft, fh, fw], dim=-1).reshape(1, 1, f * h * w, d // 2).to(torch.complex64)


def timestep_embedding(t: torch.Tensor, dim: int) -> torch.Tensor:
    half = dim // 2
    freqs = torch.exp(-math.log(10000.0) * torch.arange(half, device=t.device) / half)
    a = t.float()[:, None] * freqs[None]
    return torch.cat([torch.cos(a), torch.sin(a)], dim=-1)


class WanDiT(nn.Module):
    def __init__(self, cfg: dict = WAN_1_3B, layers: Optional[int] = None):
        super().__init__()
        c = dict(cfg)
        if layers is not None:
            c["layers"] = layers
        self.cfg = c
        dim, pt = c["dim"], c["patch"]
        self.patch_embedding = nn.Conv3d(c["in_ch"], dim, kernel_size=pt, stride=pt)
        self.text_embedding = nn.Sequential(nn.Linear(c["text_dim"], dim),
                                            nn.GELU(approximate="tanh"), nn.Linear(dim, dim))
        self.time_embedding = nn.Sequential(nn.Linear(c["freq_dim"], dim), nn.SiLU(),
                                            nn.Linear(dim, dim))
        self.time_projection = nn.Sequential(nn.SiLU(), nn.Linear(dim, 6 * dim))
        self.blocks = nn.ModuleList([WanBlock(dim, c["ffn_dim"], c["heads"], c["eps"])
                                     for _ in range(c["layers"])])
        self.norm_out = FP32LayerNorm(dim, c["eps"], elementwise_affine=False)
        self.out_table = nn.Parameter(torch.randn(1, 2, dim) / dim ** 0.5)
        self.proj_out = nn.Linear(dim, c["out_ch"] * math.prod(pt))

    @torch.no_grad()
    def init_weights(self, seed: int = 0):
        """Linear and conv weights N(0, 0.02), biases zero, norm scales one,
        drawn on the CPU from `seed` (the same model on every rank)."""
        g = torch.Generator().manual_seed(seed)
        for m in self.modules():
            if isinstance(m, (nn.Linear, nn.Conv3d)):
                m.weight.copy_(torch.randn(m.weight.shape, generator=g) * 0.02)
                m.bias.zero_()
            elif isinstance(m, (nn.RMSNorm, nn.LayerNorm)) and m.weight is not None:
                m.weight.fill_(1.0)
                if getattr(m, "bias", None) is not None:
                    m.bias.zero_()
        for blk in self.blocks:
            blk.scale_shift_table.copy_(torch.randn(1, 6, self.cfg["dim"], generator=g) * 0.02)
        self.out_table.copy_(torch.randn(1, 2, self.cfg["dim"], generator=g) * 0.02)

    def forward(self, latent, t, text, rotary, shard: Optional[tuple] = None):
        """latent [B, C, F, H, W], t [B], text [B, L, text_dim], rotary
        complex [1, 1, S, 64]. shard = (rank, world): this rank's S/world
        tokens only (the activations of a sequence-parallel run). Returns the
        tokens' output projection [B, S or S/world, C * 4]."""
        x = self.patch_embedding(latent).flatten(2).transpose(1, 2)
        if shard is not None:
            rank, world = shard
            Sr = x.shape[1] // world
            x = x[:, rank * Sr:(rank + 1) * Sr].contiguous()
            rotary = rotary[:, :, rank * Sr:(rank + 1) * Sr]
        temb = self.time_embedding(timestep_embedding(t, self.cfg["freq_dim"]).to(x.dtype))
        tproj = self.time_projection(temb).unflatten(1, (6, self.cfg["dim"]))
        ctx = self.text_embedding(text)
        for blk in self.blocks:
            x = blk(x, ctx, tproj, rotary)
        shift, scale = (self.out_table + temb.float().unsqueeze(1)).chunk(2, dim=1)
        x = (self.norm_out(x.float()) * (1 + scale) + shift).type_as(x)
        return self.proj_out(x)


class UlyssesWanInner(nn.Module):
    """The Wan inner attention of one layer under sequence parallelism.

    Called by the reference's processor with this rank's Q, K, V shards
    ([B, H, S/P, 128] views of the projections): the peer exchange moves
    them to the (batch, head) owners, each owner runs the Wan runtime's
    attention on whole sequences (sink mask + pooled K/V of gap `sample_gap`
    with the adaptive mix, one kernel: ops.sink_dynamic_attn), and the
    output rows come back to their sequence owners. Returns [B, H, S/P, 128]
    (a view of the exchange's output buffer, consumed by the processor's
    output projection before the next layer overwrites it)."""

    def __init__(self, exchange, sink_mask: torch.Tensor, sample_gap: int):
        super().__init__()
        self.exchange = exchange
        self.unit_masks = exchange.unit_masks(sink_mask.bool().unsqueeze(0))
        self.gap = int(sample_gap)

    def _units(self, q, k, v, mask, out):
        from sinkattn_b200 import ops

        kd = ops.mean_pool_seq(k, self.gap)
        vd = ops.mean_pool_seq(v, self.gap)
        ops.sink_dynamic_attn(q, k, v, mask, kd, vd, self.gap, out=out)
        return None

    def forward(self, q, k, v):
        out, _ = self.exchange(q.transpose(1, 2), k.transpose(1, 2), v.transpose(1, 2),
                               unit_masks=self.unit_masks, attn_fn=self._units)
        return out.transpose(1, 2)


def build(masks: torch.Tensor, device, layers: Optional[int] = None, seed: int = 0,
          world: int = 1, rank: int = 0, latent=LATENT, cfg: dict = WAN_1_3B):
    """The DiT in bf16 on `device` with every self-attention wired to the
    reference's Wan processor: masks bool [layers, H, nb, nb] (one sink mask
    per layer). install() must already be in place. Returns (model, exchange
    or None); the exchange (world > 1) must be closed by the caller."""
    import sinkattention.sparse_attention as sa
    import wanx.runtime.sink_sparse_wan as wan

    model = WanDiT(cfg, layers=layers)
    model.init_weights(seed)
    model = model.to(device=device, dtype=torch.bfloat16)
    L = len(model.blocks)
    _, _, f, h, w = latent
    pt = model.cfg["patch"]
    S = (f // pt[0]) * (h // pt[1]) * (w // pt[2])
    rcfg = sa.SinkSparseConfig()  # the Wan runtime default: pooled_kv, gap 30, adaptive
    exchange = None
    if world > 1:
        from sinkattn_b200.sharding import UlyssesPeerExchange

        exchange = UlyssesPeerExchange(latent[0], S, model.cfg["heads"], device=device)
    for i, blk in enumerate(model.blocks):
        blk.attn1.processor = wan.WanSinkSparseAttnProcessor2_0(layer_idx=i)
        m = masks[i % masks.shape[0]]
        if world > 1:
            blk.attn1.inner_attention = UlyssesWanInner(exchange, m.to(device), rcfg.sample_gap)
        else:
            blk.attn1.inner_attention = wan.WanSinkSparseInnerAttention(i, m.cpu(), rcfg)
    assert L == len(model.blocks)
    return model, exchange


def inputs(device, latent=LATENT, cfg: dict = WAN_1_3B, seed: int = 0):
    """Seeded latent [B, 16, F, H, W], timestep, text context and rotary table."""
    g = torch.Generator().manual_seed(seed)
    B, C, f, h, w = latent
    x = torch.randn(latent, generator=g).to(device=device, dtype=torch.bfloat16)
    t = torch.full((B,), 500.0, device=device)
    text = torch.randn(B, cfg["text_len"], cfg["text_dim"], generator=g).to(
        device=device, dtype=torch.bfloat16)
    pt = cfg["patch"]
    rot = rope_freqs(f // pt[0], h // pt[1], w // pt[2], cfg["dim"] // cfg["heads"]).to(device)
    return x, t, text, rot

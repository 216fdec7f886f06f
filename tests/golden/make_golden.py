"""Generate the golden vectors in tests/golden/ by running the REFERENCE.

Run in a container where the reference checkout is importable:

    python tests/golden/make_golden.py --reference /path/to/sinkattn

It imports the reference's own Python (sinkattention, wanx), runs its
functions on seeded inputs and stores inputs (where needed), outputs and
input digests in tests/golden/golden.npz. The tests and the GPU parity
checks read only that file; nothing at test time needs the reference.

Attention: the reference's block-sparse kernel is the external
Block-Sparse-Attention package, absent here, so the reference pipeline is run
with a dense-masked fp32 stand-in installed as block_sparse_attn_func. The
reference's adapter, mask caches, pooled dynamic branch and LSE mix then run
unchanged around it.
"""
from __future__ import annotations

import argparse
import math
import sys
from dataclasses import asdict
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE.parent.parent))

from tests.gen import cfg1_mask, digest  # noqa: E402


def bits(t: torch.Tensor) -> np.ndarray:
    return t.detach().cpu().contiguous().view(torch.int16).numpy().view(np.uint16)


def seeded_bf16(shape, seed) -> torch.Tensor:
    """Inputs are regenerated at test time from (shape, seed); the fixture
    stores their SHA-256 so a generator change is caught, not compared."""
    g = torch.Generator().manual_seed(seed)
    return torch.randn(*shape, generator=g).to(torch.bfloat16)


def pin_inputs(g: dict, name: str, **tensors_and_seeds) -> None:
    for key, (t, seed) in tensors_and_seeds.items():
        g[f"{name}/{key}_shape"] = np.array(t.shape)
        g[f"{name}/{key}_seed"] = np.array(seed)
        g[f"{name}/{key}_sha256"] = np.array(digest(t))


def fake_block_sparse_attn_func(q_unpad, k_unpad, v_unpad, cu_seqlens_q, cu_seqlens_k,
                                head_mask_type, streaming_info, base_blockmask, max_seqlen_q_,
                                max_seqlen_k_, p_dropout=0.0, deterministic=False,
                                softmax_scale=None, is_causal=False, exact_streaming=False,
                                return_attn_probs=False):
    """Dense masked fp32 attention with per-head masks (the stand-in)."""
    B = cu_seqlens_q.numel() - 1
    Sq, Sk = int(max_seqlen_q_), int(max_seqlen_k_)
    H, D = q_unpad.shape[1], q_unpad.shape[2]
    q = q_unpad.float().view(B, Sq, H, D).permute(0, 2, 1, 3)
    k = k_unpad.float().view(B, Sk, H, D).permute(0, 2, 1, 3)
    v = v_unpad.float().view(B, Sk, H, D).permute(0, 2, 1, 3)
    tok = base_blockmask.repeat_interleave(128, -2).repeat_interleave(128, -1)[..., :Sq, :Sk]
    sc = torch.matmul(q, k.transpose(-1, -2)) / math.sqrt(D)
    sc = sc.masked_fill(~tok, float("-inf"))
    lse = torch.logsumexp(sc, dim=-1)
    out = torch.matmul(torch.softmax(sc, dim=-1), v)
    out = out.permute(0, 2, 1, 3).reshape(B * Sq, H, D).to(q_unpad.dtype)
    if return_attn_probs:
        return out, lse, None
    return out


def main() -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True,
                    help="directory holding the reference's sinkattention/ (a checkout or an install)")
    ap.add_argument("--out", default=str(HERE / "golden.npz"))
    args = ap.parse_args()
    sys.path.insert(0, args.reference)
    import sinkattention.sparse_attention as sa
    from sinkattention.sparse_attention import SinkSparseConfig

    torch.set_num_threads(1)
    g: dict[str, np.ndarray] = {}

    # ---- pooled scores, mean mode (sparse_attention.py:118-142) -----------
    pool_cases = {
        "pool_a": dict(B=2, H=2, S=1000, D=128, block=128, seed=11),
        "pool_b": dict(B=1, H=2, S=384, D=64, block=128, seed=12),
        "pool_c": dict(B=1, H=1, S=300, D=128, block=64, seed=13),
    }
    for name, c in pool_cases.items():
        q = seeded_bf16((c["B"], c["H"], c["S"], c["D"]), c["seed"])
        k = seeded_bf16((c["B"], c["H"], c["S"], c["D"]), c["seed"] + 100)
        cfg = SinkSparseConfig(block_size=c["block"], pooling_mode="mean")
        out = sa._compute_pooled_qk_block_scores(q, k, k, cfg)
        pin_inputs(g, name, q=(q, c["seed"]), k=(k, c["seed"] + 100))
        g[f"{name}/block"] = np.array(c["block"])
        g[f"{name}/scores"] = out.numpy().astype(np.float32)

    # ---- exact block-mass scores (sparse_attention.py:145-227) --------------
    exact_cases = {
        "exact_a": dict(B=1, H=2, S=600, seed=51),
        "exact_b": dict(B=2, H=1, S=512, seed=52),
    }
    for name, c in exact_cases.items():
        q = seeded_bf16((c["B"], c["H"], c["S"], 128), c["seed"])
        k = seeded_bf16((c["B"], c["H"], c["S"], 128), c["seed"] + 100)
        cfg = SinkSparseConfig(pooling_mode="exact")
        out = sa._compute_exact_block_mass_scores(q.float(), k.float(), cfg)
        pin_inputs(g, name, q=(q, c["seed"]), k=(k, c["seed"] + 100))
        g[f"{name}/scores"] = out.numpy().astype(np.float32)

    # ---- Q/K producer: RMSNorm + rotary (wanx/runtime/sink_sparse_wan.py:300-315)
    # through the reference's own helpers with its default (non-Triton) path:
    # torch RMSNorm modules and the fp64 complex rotary (fast_misc.py:173-179).
    import wanx.runtime.fast_misc as fm

    S_r, H_r, D_r = 96, 2, 128
    hidden = H_r * D_r
    q_lin = seeded_bf16((1, S_r, hidden), 71)
    k_lin = seeded_bf16((1, S_r, hidden), 72)
    gw = torch.Generator().manual_seed(73)
    w_q = (1.0 + 0.25 * torch.randn(hidden, generator=gw)).to(torch.bfloat16)
    w_k = (1.0 + 0.25 * torch.randn(hidden, generator=gw)).to(torch.bfloat16)

    class _Attn:
        pass

    attn = _Attn()
    attn.norm_q = torch.nn.RMSNorm(hidden, eps=1e-6, dtype=torch.bfloat16)
    attn.norm_k = torch.nn.RMSNorm(hidden, eps=1e-6, dtype=torch.bfloat16)
    with torch.no_grad():
        attn.norm_q.weight.copy_(w_q)
        attn.norm_k.weight.copy_(w_k)
    # 1-D RoPE frequencies theta^(-2i/D), positions 0..S-1, complex64 [1,1,S,D/2]
    inv = 1.0 / (10000.0 ** (torch.arange(0, D_r, 2, dtype=torch.float64) / D_r))
    ang = torch.outer(torch.arange(S_r, dtype=torch.float64), inv)
    freqs = torch.polar(torch.ones_like(ang), ang).to(torch.complex64)[None, None]
    with torch.no_grad():
        qn, kn = fm.apply_fast_qk_norm(attn, q_lin, k_lin)
        qn = qn.unflatten(2, (H_r, -1)).transpose(1, 2)
        kn = kn.unflatten(2, (H_r, -1)).transpose(1, 2)
        qo, ko = fm.apply_fast_rotary_qk(qn, kn, freqs)
    pin_inputs(g, "qkrope", q=(q_lin, 71), k=(k_lin, 72))
    g["qkrope/w_q"] = bits(w_q)
    g["qkrope/w_k"] = bits(w_k)
    g["qkrope/eps"] = np.array(1e-6)
    g["qkrope/heads"] = np.array(H_r)
    g["qkrope/cos"] = freqs.real[0, 0].numpy().astype(np.float32)
    g["qkrope/sin"] = freqs.imag[0, 0].numpy().astype(np.float32)
    g["qkrope/q_out"] = bits(qo.contiguous())
    g["qkrope/k_out"] = bits(ko.contiguous())

    # ---- coverage masks (sparse_attention.py:268-376) ---------------------
    def softmax_scores(H, nq, nk, seed, temp):
        gen = torch.Generator().manual_seed(seed)
        return torch.softmax(torch.randn(H, nq, nk, generator=gen) * temp, dim=-1)

    def quantized_scores(H, nq, nk, seed):
        gen = torch.Generator().manual_seed(seed)
        x = torch.randint(0, 6, (H, nq, nk), generator=gen).float() / 64.0
        return x

    cov_cases = {
        "cov_joint": (softmax_scores(2, 64, 64, 21, 1.0), dict(keep_diagonal=True)),
        "cov_peaky": (softmax_scores(2, 64, 64, 22, 12.0), dict(keep_diagonal=True)),
        "cov_text": (softmax_scores(2, 40, 40, 23, 2.0),
                     dict(force_text_global_attention=True, text_length=512)),
        "cov_video": (softmax_scores(2, 40, 40, 23, 2.0),
                      dict(force_text_global_attention=True, text_length=512,
                           offline_text_video_coverage_mode="video_residual")),
        "cov_ties": (quantized_scores(2, 48, 48, 24), dict(keep_diagonal=False)),
        "cov_zero": (softmax_scores(1, 16, 16, 25, 1.0),
                     dict(keep_diagonal=False, offline_direct_coverage=0.0)),
        "cov_nonsq": (softmax_scores(1, 20, 70, 26, 1.5), dict(keep_diagonal=True)),
        "cov_wide": (softmax_scores(1, 4, 300, 27, 1.0), dict(keep_diagonal=True)),
        "cov_sink": (softmax_scores(2, 64, 64, 28, 1.0), dict(keep_diagonal=True)),
    }
    orig_required = sa._build_offline_required_mask
    for name, (scores, kw) in cov_cases.items():
        cfg = SinkSparseConfig(**kw)
        if name == "cov_sink":
            # the benchmark rule "always keep key-block 0": column 0 joins the
            # required set before the coverage step
            def with_sink(*, num_query_blocks, num_key_blocks, config, device):
                base = orig_required(num_query_blocks=num_query_blocks,
                                     num_key_blocks=num_key_blocks, config=config, device=device)
                req = torch.zeros(num_query_blocks, num_key_blocks, dtype=torch.bool)
                if base is not None:
                    req |= base
                req[:, 0] = True
                return req
            sa._build_offline_required_mask = with_sink
        try:
            mask = sa._build_direct_mean_coverage_mask(scores, cfg)
        finally:
            sa._build_offline_required_mask = orig_required
        H, nq, nk = scores.shape
        T = 0
        if cfg.force_text_global_attention and cfg.text_length > 0:
            T = min(math.ceil(cfg.text_length / cfg.block_size), nq, nk)
        video = cfg.offline_text_video_coverage_mode == "video_residual" and T > 0
        if video:
            total = torch.zeros(H, nq)
            total[:, T:] = scores[:, T:, T:].sum(dim=-1)
            sel = torch.zeros(H, nq)
        else:
            total = scores.sum(dim=-1)
            req = torch.zeros(nq, nk, dtype=torch.bool)
            if T > 0:
                req[:, :T] = True
                req[:T, :] = True
            if name == "cov_sink":
                req[:, 0] = True
            sel = (scores * req.float()).sum(dim=-1)
        g[f"{name}/scores"] = scores.numpy().astype(np.float32)
        g[f"{name}/mask"] = mask.numpy()
        g[f"{name}/total"] = total.numpy().astype(np.float32)
        g[f"{name}/selected"] = sel.numpy().astype(np.float32)
        g[f"{name}/coverage"] = np.array(cfg.offline_direct_coverage, dtype=np.float64)
        g[f"{name}/keep_diagonal"] = np.array(int(cfg.keep_diagonal))
        g[f"{name}/text_blocks"] = np.array(T)
        g[f"{name}/mode"] = np.array("video_residual" if video else "joint")
        g[f"{name}/force_sink"] = np.array(int(name == "cov_sink"))

    # ---- attention ---------------------------------------------------------
    # (1) the reference's own dense path with LSE on an all-true mask
    q = seeded_bf16((1, 1, 200, 128), 31)
    k = seeded_bf16((1, 1, 300, 128), 32)
    v = seeded_bf16((1, 1, 300, 128), 33)
    out, lse = sa._dense_short_attention_with_lse(q.float(), k.float(), v.float())
    pin_inputs(g, "attn_dense", q=(q, 31), k=(k, 32), v=(v, 33))
    g["attn_dense/out"] = out.numpy().astype(np.float32)
    g["attn_dense/lse"] = lse[..., 0].numpy().astype(np.float32)

    # (2) the reference's adapter with the stand-in kernel, masked, ragged
    sa.block_sparse_attn_func = fake_block_sparse_attn_func
    sa._HAS_BLOCK_SPARSE = True
    q = seeded_bf16((1, 2, 400, 128), 41)
    k = seeded_bf16((1, 2, 400, 128), 42)
    v = seeded_bf16((1, 2, 400, 128), 43)
    nb = math.ceil(400 / 128)
    mask = cfg1_mask(2, nb, nb, seed=44, p=0.3).unsqueeze(0)
    o_s, l_s = sa._block_sparse_attn(q, k, v, mask, return_lse=True)
    pin_inputs(g, "attn_sparse", q=(q, 41), k=(k, 42), v=(v, 43))
    g["attn_sparse/mask"] = mask.numpy()
    g["attn_sparse/out"] = bits(o_s.contiguous())
    g["attn_sparse/lse_bf16"] = bits(l_s[..., 0].contiguous())

    # (3) the Wan inner attention (sink + pooled dynamic branch + adaptive mix)
    from wanx.runtime.sink_sparse_wan import WanSinkSparseInnerAttention
    from wanx.runtime.inference import DEFAULT_SINK_RUNTIME_OVERRIDES
    cfg = SinkSparseConfig().merged(DEFAULT_SINK_RUNTIME_OVERRIDES)
    sink_mask = mask[0]
    inner = WanSinkSparseInnerAttention(0, sink_mask, cfg)
    mixed = inner(q, k, v)
    g["wan_inner/out"] = bits(mixed.contiguous())
    g["wan_inner/sample_gap"] = np.array(cfg.sample_gap)
    g["wan_inner/band"] = np.array(cfg.runtime_diagonal_band_width)
    g["wan_inner/config"] = np.array(repr(asdict(cfg)))

    g["_digest/cfg1_mask"] = np.array(digest(cfg1_mask()))
    np.savez_compressed(args.out, **g)
    size = Path(args.out).stat().st_size
    print(f"wrote {args.out}: {len(g)} arrays, {size / 1024:.0f} KiB")
    return 0


if __name__ == "__main__":
    sys.exit(main())

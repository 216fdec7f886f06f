"""Generate tests/golden/calib.npz by running the REFERENCE's own functions on
fixed inputs: the steps on either side of the kernels.

    python tests/golden/make_golden_calib.py --reference /path/to/sinkattn

- `_mean_pool_sequence_preserve_prefix` (sinkattention/sparse_attention.py:79-115):
  ragged lengths (replicate padding), a kept prefix, a prefix longer than the
  sequence, and a pool of 128.
- `_mix_attention_outputs` (sparse_attention.py:898-919) on bf16 outputs and
  bf16 LSE, as the reference's adapter returns them.
- `_adapt_block_mask_for_kernel` (sparse_attention.py:797-852): a coarse mask
  (256-token blocks, repeated onto 128 tiles), a fine one (32-token blocks,
  any-pooled), both with ragged lengths, and the identity at 128.
- `SinkMaskCalibrator` (sparse_attention.py:526-608): three generations of two
  layers, then `build_package`. The calibrator is fed fixed block scores by
  replacing `_compute_block_scores` in its module, so the statistics and masks
  are pinned apart from how the scores were made. The batch means it
  accumulated are captured from `_accumulate_score`.
- `ZImageSinkMaskCalibrator` (zimg/runtime/sink_sparse_zimage.py:140-186,
  248-366): four samples with 300, 100, 0 and 250 text tokens per layer
  (alignment into the fixed image-prefix/text-suffix layout, presence counts,
  presence-weighted statistics), then `build_package`.

Bulk bf16 inputs are regenerated at test time from (shape, seed) and checked
against stored SHA-256 digests; the small fp32 score inputs are stored as is.
Nothing at test time needs the reference.
"""
from __future__ import annotations

import argparse
import json
import sys
from dataclasses import asdict
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE.parent.parent))

from tests.golden.make_golden import bits, pin_inputs, seeded_bf16  # noqa: E402

MEAN_POOL_CASES = {
    "mpool_a": dict(shape=(1, 2, 1000, 128), seed=51, pool=30, prefix=0),
    "mpool_b": dict(shape=(1, 2, 1000, 128), seed=51, pool=30, prefix=77),
    "mpool_c": dict(shape=(1, 1, 100, 64), seed=52, pool=7, prefix=150),
    "mpool_d": dict(shape=(2, 1, 4100, 128), seed=53, pool=128, prefix=5),
}
MIX_CASE = dict(shape=(1, 2, 129, 64), seeds=(61, 62, 63, 64), sample_gap=30)
ADAPT_CASES = {
    "adapt_coarse": dict(source=256, Sq=1000, Sk=1300, heads=2, seed=91, p=0.3),
    "adapt_fine": dict(source=32, Sq=1000, Sk=700, heads=2, seed=92, p=0.05),
    "adapt_same": dict(source=128, Sq=1000, Sk=700, heads=2, seed=93, p=0.3),
}


def block_score_samples(gen: torch.Generator, B: int, H: int, n: int) -> torch.Tensor:
    """Row-stochastic fp32 block scores [B, H, n, n] (a softmax of random
    logits), the shape and value range of what the score modes return."""
    logits = torch.randn(B, H, n, n, generator=gen) * 2.0
    return torch.softmax(logits, dim=-1).float()


def main() -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True,
                    help="directory holding the reference's sinkattention/ (a checkout or an install)")
    ap.add_argument("--out", default=str(HERE / "calib.npz"))
    args = ap.parse_args()
    sys.path.insert(0, args.reference)
    import sinkattention.sparse_attention as sa
    import zimg.runtime.sink_sparse_zimage as zi
    from sinkattention.sparse_attention import SinkSparseConfig

    torch.set_num_threads(1)
    g: dict[str, np.ndarray] = {}

    # ---- sequence mean pooling with a kept prefix ---------------------------
    for name, c in MEAN_POOL_CASES.items():
        x = seeded_bf16(c["shape"], c["seed"])
        out = sa._mean_pool_sequence_preserve_prefix(x, c["pool"], prefix_tokens=c["prefix"])
        pin_inputs(g, name, x=(x, c["seed"]))
        g[f"{name}/pool"] = np.array(c["pool"])
        g[f"{name}/prefix"] = np.array(c["prefix"])
        g[f"{name}/out"] = bits(out.contiguous())

    # ---- adaptive LSE mix ----------------------------------------------------
    s1, s2, s3, s4 = MIX_CASE["seeds"]
    o_s = seeded_bf16(MIX_CASE["shape"], s1)
    o_d = seeded_bf16(MIX_CASE["shape"], s2)
    lse_shape = MIX_CASE["shape"][:3] + (1,)
    # LSE of the two branches: bf16 [B,H,S,1], as the adapter returns it
    # (sparse_attention.py:776); the dynamic branch's is lower by about ln(gap)
    l_s = (seeded_bf16(lse_shape, s3).float() * 2.0 + 6.0).to(torch.bfloat16)
    l_d = (seeded_bf16(lse_shape, s4).float() * 2.0 + 3.0).to(torch.bfloat16)
    cfg_mix = SinkSparseConfig(sample_gap=MIX_CASE["sample_gap"])
    mixed = sa._mix_attention_outputs(o_s, l_s, o_d, l_d, cfg_mix, MIX_CASE["sample_gap"])
    pin_inputs(g, "mix", o_s=(o_s, s1), o_d=(o_d, s2))
    g["mix/lse_s"] = bits(l_s.contiguous())
    g["mix/lse_d"] = bits(l_d.contiguous())
    g["mix/sample_gap"] = np.array(MIX_CASE["sample_gap"])
    g["mix/out"] = bits(mixed.contiguous())

    # ---- mask adaptation to the kernel's 128-token tiles ----------------------
    for name, c in ADAPT_CASES.items():
        gen = torch.Generator().manual_seed(c["seed"])
        nq = -(-c["Sq"] // c["source"])
        nk = -(-c["Sk"] // c["source"])
        src = torch.rand(1, c["heads"], nq, nk, generator=gen) < c["p"]
        out = sa._adapt_block_mask_for_kernel(src, source_block_size=c["source"],
                                              seq_len_q=c["Sq"], seq_len_k=c["Sk"])
        g[f"{name}/mask"] = src.numpy()
        g[f"{name}/source"] = np.array(c["source"])
        g[f"{name}/seq"] = np.array([c["Sq"], c["Sk"]])
        g[f"{name}/out"] = out.numpy()

    # ---- Wan calibrator: statistics, masks and package -----------------------
    gen = torch.Generator().manual_seed(71)
    wan_cfg = SinkSparseConfig(pooling_mode="mean", text_length=200,
                               force_text_global_attention=True)
    feed: list[torch.Tensor] = []
    sa_compute = sa._compute_block_scores
    sa._compute_block_scores = lambda q, k, v, config: feed.pop(0)
    captured: list[tuple[int, torch.Tensor]] = []
    cal = sa.SinkMaskCalibrator(wan_cfg)
    orig_acc = cal._accumulate_score

    def capture(layer_idx, scores):
        captured.append((layer_idx, scores.clone()))
        orig_acc(layer_idx, scores)

    cal._accumulate_score = capture
    try:
        for _step in range(3):
            for layer in (0, 1):
                feed.append(block_score_samples(gen, 2, 3, 9))
                cal.record(layer, torch.zeros(2), None, None)
        pkg = cal.build_package()
    finally:
        sa._compute_block_scores = sa_compute
    g["wan_cal/config"] = np.array(json.dumps(asdict(wan_cfg)))
    g["wan_cal/layers"] = np.array([lay for lay, _ in captured])
    g["wan_cal/scores"] = np.stack([s.numpy() for _, s in captured])
    for key in ("0", "1"):
        g[f"wan_cal/mean/{key}"] = pkg["mean_scores"][key].numpy()
        g[f"wan_cal/std/{key}"] = pkg["std_scores"][key].numpy()
        g[f"wan_cal/mask/{key}"] = pkg["sink_masks"][key].numpy()
        g[f"wan_cal/count/{key}"] = np.array(pkg["counts"][key])
    g["wan_cal/meta"] = np.array(json.dumps(pkg["meta"]))

    # ---- Z-Image calibrator: alignment, presence, statistics, masks -----------
    gen = torch.Generator().manual_seed(81)
    z_base = SinkSparseConfig(pooling_mode="mean", token_width=32, token_height=32,
                              token_depth=1, text_length=300)
    zcal = zi.ZImageSinkMaskCalibrator(z_base)
    texts = [300, 100, 0, 250]
    zfeed: list[torch.Tensor] = []
    samples: list[np.ndarray] = []
    zi_compute = zi._compute_block_scores
    zi._compute_block_scores = lambda q, k, v, config: zfeed.pop(0)
    try:
        for text in texts:
            for layer in (0, 1):
                n = zcal.image_blocks + -(-text // int(zcal.config.block_size))
                s = block_score_samples(gen, 1, 3, n)
                zfeed.append(s)
                samples.append(s[0].numpy())
                zcal.record(layer, torch.zeros(1), None, None, text_token_count=text)
        zpkg = zcal.build_package()
    finally:
        zi._compute_block_scores = zi_compute
    g["z_cal/config"] = np.array(json.dumps(asdict(zcal.config)))
    g["z_cal/texts"] = np.array(texts)
    g["z_cal/layout"] = np.array([zcal.image_token_count, zcal.image_blocks, zcal.total_blocks,
                                  zcal.max_text_tokens])
    for i, s in enumerate(samples):
        g[f"z_cal/scores/{i}"] = s
    for key in ("0", "1"):
        g[f"z_cal/mean/{key}"] = zpkg["mean_scores"][key].numpy()
        g[f"z_cal/std/{key}"] = zpkg["std_scores"][key].numpy()
        g[f"z_cal/mask/{key}"] = zpkg["sink_masks"][key].numpy()
        g[f"z_cal/presence/{key}"] = zcal.score_presence_sums[int(key)].numpy()
        g[f"z_cal/count/{key}"] = np.array(zpkg["counts"][key])
    g["z_cal/meta"] = np.array(json.dumps(zpkg["meta"]))

    np.savez_compressed(args.out, **g)
    size = Path(args.out).stat().st_size
    print(f"wrote {args.out}: {len(g)} arrays, {size / 1024:.0f} KiB")
    return 0


if __name__ == "__main__":
    sys.exit(main())

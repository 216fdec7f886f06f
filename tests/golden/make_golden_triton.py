"""Golden vectors for the block-maximum statistics, made by running the
REFERENCE's Triton kernel attn_with_pooling (sinkattention/pooling_kernel.py)
on a GPU, the way _compute_pooled_qk_block_scores calls it
(sinkattention/sparse_attention.py:124-135).

Run on a GPU machine where the reference package is importable:

    python tests/golden/make_golden_triton.py --reference <dir holding sinkattention/> \
        --out tests/golden/triton_max.npz

Only sequence lengths that are multiples of 128 are generated: for other
lengths the Triton kernel's block pointers run past the end of the head
(they carry no boundary check), so its output is not defined by the inputs.
Inputs are regenerated from (shape, seed) at test time; the file stores
their digests and the kernel's output.
"""
from __future__ import annotations

import argparse
import math
import sys
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE.parent.parent))

from tests.golden.make_golden import pin_inputs, seeded_bf16  # noqa: E402

CASES = {
    "tri_a": dict(B=1, H=2, S=512, qseed=71, kseed=171),
    "tri_b": dict(B=2, H=3, S=1024, qseed=72, kseed=172),
    "tri_c": dict(B=1, H=2, S=2048, qseed=73, kseed=73),  # k = q: diagonal-heavy
}


def main() -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True)
    ap.add_argument("--out", default=str(HERE / "triton_max.npz"))
    args = ap.parse_args()
    sys.path.insert(0, args.reference)
    from sinkattention.pooling_kernel import attn_with_pooling

    g = {}
    for name, c in CASES.items():
        shape = (c["B"], c["H"], c["S"], 128)
        q = seeded_bf16(shape, c["qseed"])
        k = seeded_bf16(shape, c["kseed"])
        _, pooled = attn_with_pooling(q.cuda(), k.cuda(), k.cuda(), False,
                                      1.0 / math.sqrt(q.size(-1)), 128)
        pin_inputs(g, name, q=(q, c["qseed"]), k=(k, c["kseed"]))
        g[f"{name}/scores"] = pooled.float().cpu().numpy()
    np.savez_compressed(args.out, **g)
    print(f"wrote {args.out}: {len(g)} arrays")
    return 0


if __name__ == "__main__":
    raise SystemExit(main())

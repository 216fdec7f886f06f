"""fp32 reference of the attention kernels on the GPU, for the full-size
parity tests (test infrastructure; the product never imports it).

The numpy oracle (oracle/sinkattn_oracle.py) defines the operation but takes
minutes per Wan-sized head on the host. This module computes the same dense
masked attention on the device so that every (b, h, query tile) of a full
launch can be compared:

    out = softmax(q k^T * scale + M) v,  M = -inf outside kept 128x128 blocks
    lse = log(sum exp(q k^T * scale + M))  (natural log)

with optional extra keys/values that every row sees with a constant logit
bias (the fused sink + pooled-dynamic branch: pooled K/V with +ln(gap)).

Precision. The two products run on TF32 tensor cores with operands that TF32
holds exactly, so the result is fp32 arithmetic up to summation order:
  * S = q k^T: q and k hold bf16 values (8 significant bits), which TF32 (11
    significant bits) represents exactly; every product is exact and the
    sums are fp32.
  * O = P v: v holds bf16 values (exact). P (fp32) is split P = P_hi + P_lo,
    P_hi = P with its 13 low mantissa bits cleared (exact in TF32) and
    P_lo = P - P_hi (exact in fp32, at most 2^-10 of P, and rounded by TF32
    to 2^-11 of itself), so the split adds about 2^-21 relative error.
Rows whose mask keeps no key give out 0 and lse -inf, as the kernel does.
The tests that use this module pin it against the numpy oracle first.
"""
from __future__ import annotations

import contextlib
import math
from typing import Iterator, Optional

import torch

BLOCK = 128


@contextlib.contextmanager
def tf32_matmul() -> Iterator[None]:
    prev = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = True
    try:
        yield
    finally:
        torch.backends.cuda.matmul.allow_tf32 = prev


def _split_mm(p: torch.Tensor, v: torch.Tensor) -> torch.Tensor:
    hi = (p.view(torch.int32) & ~0x1FFF).view(torch.float32)
    lo = p - hi
    return hi @ v + lo @ v


def unit_attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, block_mask: torch.Tensor,
                   scale: Optional[float] = None, extra_k: Optional[torch.Tensor] = None,
                   extra_v: Optional[torch.Tensor] = None, extra_bias: float = 0.0,
                   row_chunk: int = 4096) -> tuple[torch.Tensor, torch.Tensor]:
    """One (b, h) unit: q [Sq,D], k/v [Sk,D] (bf16-valued, any float dtype, on
    the GPU), block_mask bool [ceil(Sq/128), ceil(Sk/128)]; extra_k/extra_v
    [Se,D] seen by every row with logit bias extra_bias. Returns out fp32
    [Sq,D] and lse fp32 [Sq]."""
    Sq, D = q.shape
    Sk = k.shape[0]
    if scale is None:
        scale = 1.0 / math.sqrt(D)
    kf, vf = k.float(), v.float()
    ekf = None if extra_k is None else extra_k.float()
    evf = None if extra_v is None else extra_v.float()
    out = torch.empty(Sq, D, dtype=torch.float32, device=q.device)
    lse = torch.empty(Sq, dtype=torch.float32, device=q.device)
    col_mask = block_mask.repeat_interleave(BLOCK, dim=1)[:, :Sk]
    with tf32_matmul():
        for r0 in range(0, Sq, row_chunk):
            r1 = min(Sq, r0 + row_chunk)
            qf = q[r0:r1].float()
            s = (qf @ kf.T) * scale
            tok = col_mask[r0 // BLOCK:(r1 + BLOCK - 1) // BLOCK].repeat_interleave(BLOCK, dim=0)
            tok = tok[: r1 - r0]
            s.masked_fill_(~tok, float("-inf"))
            if ekf is not None:
                s = torch.cat([s, (qf @ ekf.T) * scale + extra_bias], dim=1)
            m = s.amax(dim=1, keepdim=True)
            empty = ~torch.isfinite(m)
            m = torch.where(empty, torch.zeros_like(m), m)
            p = torch.exp(s - m)
            del s
            l = p.sum(dim=1, keepdim=True)
            vv = vf if evf is None else torch.cat([vf, evf], dim=0)
            o = _split_mm(p, vv) / l
            del p
            lr = torch.log(l) + m
            o[empty[:, 0]] = 0.0
            lr[empty] = float("-inf")
            out[r0:r1] = o
            lse[r0:r1] = lr[:, 0]
    return out, lse


def compare_tiles(out: torch.Tensor, lse: torch.Tensor, ref: torch.Tensor,
                  ref_lse: torch.Tensor) -> dict:
    """Per 128-row query tile of one unit: max-abs error, mean-relative error
    (mean |err| / mean |ref| over the tile) and max LSE error (finite rows;
    rows the reference marks empty must be -inf). Returns the worst of each
    and their tiles."""
    Sq, D = ref.shape
    nq = (Sq + BLOCK - 1) // BLOCK
    pad = nq * BLOCK - Sq
    err = (out.float() - ref).abs()
    a = ref.abs()
    if pad:
        err = torch.cat([err, err.new_zeros(pad, D)])
        a = torch.cat([a, a.new_zeros(pad, D)])
    rows = torch.full((nq,), BLOCK, dtype=torch.float32, device=ref.device)
    rows[-1] = BLOCK - pad
    err_t = err.view(nq, BLOCK, D)
    max_abs = err_t.amax(dim=(1, 2))
    mean_rel = err_t.sum(dim=(1, 2)) / a.view(nq, BLOCK, D).sum(dim=(1, 2)).clamp_min(1e-30)
    fin = torch.isfinite(ref_lse)
    lse_bad = int((torch.isfinite(lse) != fin).sum())
    lerr = torch.where(fin, (lse - ref_lse).abs(), torch.zeros_like(ref_lse))
    if pad:
        lerr = torch.cat([lerr, lerr.new_zeros(pad)])
    lse_t = lerr.view(nq, BLOCK).amax(dim=1)
    return {"max_abs": float(max_abs.max()), "max_abs_tile": int(max_abs.argmax()),
            "mean_rel": float(mean_rel.max()), "mean_rel_tile": int(mean_rel.argmax()),
            "lse": float(lse_t.max()), "lse_tile": int(lse_t.argmax()),
            "lse_finite_mismatch": lse_bad, "tiles": nq}

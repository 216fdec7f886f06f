"""CPU oracle for the SinkAttention hot path — TEST INFRASTRUCTURE ONLY.

This module restates, in numpy, the reference algorithms that the CUDA
library replaces. It is the checker used by tests/, by
__graft_entry__.smoke() and by bench.py's CPU-baseline / reference arm. The
product path (sinkattn_b200) never imports it.

Pinning:
  * Pooling, pooled-score softmax and the coverage mask builder are pinned
    against golden vectors produced by importing the reference itself
    (tests/golden/make_golden.py -> tests/golden/*.npz).
  * Sequence mean pooling with a prefix, the adaptive mix, and both
    calibrators' statistics (including the Z-Image alignment) are pinned the
    same way (tests/golden/make_golden_calib.py -> tests/golden/calib.npz).
  * Attention: the reference obtains block-sparse attention from the external
    package mit-han-lab/Block-Sparse-Attention (unpinned, cloned at HEAD per
    README.md:26-33, absent here), so there is no reference output for masked
    attention. The dense-masked fp32 definition below is pinned against the
    reference's own dense path `_dense_short_attention_with_lse`
    (sinkattention/sparse_attention.py:870-895) on all-true masks and through
    the reference's WanSinkSparseInnerAttention with this oracle installed as
    block_sparse_attn_func (golden vectors); the masked case itself is
    "parity unpinned" beyond that definition.

Rounding facts reproduced (probed on CPU torch 2.11):
  * torch.cumsum on fp32 accumulates in fp64 and rounds every prefix to fp32.
  * coverage * total is an fp32 multiply (python float cast to fp32).
  * torch.sum's fp32 order is implementation-defined (vectorised cascade);
    callers that need bit-exact decisions pass the reference's own totals.
  * torch.sort on CPU is not stable; this oracle sorts stably (value
    descending, index ascending) and reports rows whose cut splits a tie.
"""
from __future__ import annotations

import math
from dataclasses import dataclass

import numpy as np

LN2 = math.log(2.0)


# ---------------------------------------------------------------------------
# bf16 helpers (inputs on the GPU are bf16; the reference upcasts with .float())
# ---------------------------------------------------------------------------
def bf16_round(x: np.ndarray) -> np.ndarray:
    """Round fp32 to the nearest bf16 (ties to even), returned as fp32."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    u = x.view(np.uint32).astype(np.uint64)
    lsb = (u >> 16) & 1
    r = ((u + 0x7FFF + lsb) >> 16) << 16
    out = r.astype(np.uint32).view(np.float32)
    nan = np.isnan(x)
    if nan.any():
        out = out.copy()
        out[nan] = np.nan
    return out


def bf16_bits(x: np.ndarray) -> np.ndarray:
    """fp32 values already on the bf16 grid -> uint16 bit patterns."""
    return (np.ascontiguousarray(x, dtype=np.float32).view(np.uint32) >> 16).astype(np.uint16)


def from_bf16_bits(b: np.ndarray) -> np.ndarray:
    return (b.astype(np.uint32) << 16).view(np.float32)


# ---------------------------------------------------------------------------
# Pooling and pooled scores
# ---------------------------------------------------------------------------
def mean_pool_sequence(x: np.ndarray, pool: int) -> np.ndarray:
    """_mean_pool_sequence (sinkattention/sparse_attention.py:88-94) with the
    replicate padding of _pad_to_multiple (lines 79-85). x: [B,H,S,D] fp32."""
    if pool <= 1:
        return x
    B, H, S, D = x.shape
    rem = S % pool
    if rem:
        pad = np.repeat(x[:, :, -1:, :], pool - rem, axis=2)
        x = np.concatenate([x, pad], axis=2)
    nb = x.shape[2] // pool
    return x.reshape(B, H, nb, pool, D).astype(np.float64).mean(axis=3).astype(np.float32)


def mean_pool_sequence_preserve_prefix(x: np.ndarray, pool: int, prefix: int = 0) -> np.ndarray:
    """_mean_pool_sequence_preserve_prefix (sparse_attention.py:97-115)."""
    if pool <= 1:
        return x
    S = x.shape[2]
    prefix = min(max(int(prefix), 0), S)
    if prefix <= 0:
        return mean_pool_sequence(x, pool)
    if prefix >= S:
        return x
    return np.concatenate([x[:, :, :prefix], mean_pool_sequence(x[:, :, prefix:], pool)], axis=2)


def softmax_lastdim(x: np.ndarray) -> np.ndarray:
    m = x.max(axis=-1, keepdims=True)
    e = np.exp((x - m).astype(np.float64))
    return (e / e.sum(axis=-1, keepdims=True)).astype(np.float32)


def pooled_block_scores(q: np.ndarray, k: np.ndarray, block: int = 128) -> np.ndarray:
    """_compute_pooled_qk_block_scores, pooling_mode="mean"
    (sparse_attention.py:138-142). q, k: [B,H,S,D] fp32 (bf16 values)."""
    D = q.shape[-1]
    qp = mean_pool_sequence(q.astype(np.float32), block)
    kp = mean_pool_sequence(k.astype(np.float32), block)
    logits = np.matmul(qp.astype(np.float64), np.swapaxes(kp, -1, -2).astype(np.float64))
    logits = (logits.astype(np.float32) * np.float32(1.0 / math.sqrt(D))).astype(np.float32)
    return softmax_lastdim(logits)


# ---------------------------------------------------------------------------
# Coverage mask builder
# ---------------------------------------------------------------------------
@dataclass
class CoverageResult:
    mask: np.ndarray        # bool [H, nq, nk]
    tie_rows: np.ndarray    # bool [H, nq]: cut separates equal scores
    empty_rows: np.ndarray  # bool [H, nq]: top-1 fallback used


def required_mask(nq: int, nk: int, text_blocks: int, force_sink_col: bool = False) -> np.ndarray:
    """_build_offline_required_mask (sparse_attention.py:241-265): the first
    `text_blocks` key columns and query rows are required. force_sink_col adds
    key column 0 (the "always keep key-block 0" rule of the benchmark config)."""
    req = np.zeros((nq, nk), dtype=bool)
    T = min(text_blocks, nq, nk) if text_blocks > 0 else 0
    if T > 0:
        req[:, :T] = True
        req[:T, :] = True
    if force_sink_col:
        req[:, 0] = True
    return req


def adapt_block_mask(mask: np.ndarray, source_block: int, seq_q: int, seq_k: int,
                     kernel_block: int = 128) -> np.ndarray:
    """_adapt_block_mask_for_kernel (sparse_attention.py:797-852): a bool
    mask [..., nq, nk] over `source_block`-token blocks, mapped onto the
    kernel's `kernel_block` tiles. A kernel tile is kept when any source block
    that overlaps it is kept: coarse blocks are repeated, fine blocks are
    any-pooled (absent blocks past the end count as not kept). The result has
    ceil(seq / kernel_block) tiles per side."""
    if source_block <= 0 or kernel_block <= 0:
        raise ValueError(f"Invalid block sizes: source={source_block}, kernel={kernel_block}")
    tq = -(-int(seq_q) // kernel_block)
    tk = -(-int(seq_k) // kernel_block)
    if source_block == kernel_block:
        if mask.shape[-2:] != (tq, tk):
            raise ValueError("Runtime block mask is already at kernel tile size but has the "
                             f"wrong shape: expected [..., {tq}, {tk}], got {list(mask.shape)}")
        return mask.copy()
    if source_block > kernel_block and source_block % kernel_block:
        raise ValueError("Cannot adapt a coarse Sink mask: source block size is not a "
                         "multiple of the kernel block size.")
    if source_block < kernel_block and kernel_block % source_block:
        raise ValueError("Cannot adapt a fine Sink mask: kernel block size is not a "
                         "multiple of the source block size.")
    nq, nk = mask.shape[-2:]
    out = np.zeros(mask.shape[:-2] + (tq, tk), dtype=bool)
    for i in range(tq):
        # source blocks overlapping kernel tile i: tokens [i*kb, (i+1)*kb)
        q0, q1 = i * kernel_block // source_block, -(-(i + 1) * kernel_block // source_block)
        for j in range(tk):
            k0, k1 = j * kernel_block // source_block, -(-(j + 1) * kernel_block // source_block)
            out[..., i, j] = mask[..., q0:min(q1, nq), k0:min(k1, nk)].any(axis=(-2, -1))
    return out


def _first_reach(cum32: np.ndarray, target: np.float32) -> int:
    hit = np.nonzero(cum32 >= target)[0]
    return int(hit[0]) if hit.size else -1


def coverage_mask(
    scores: np.ndarray,
    coverage: float = 0.85,
    keep_diagonal: bool = True,
    text_blocks: int = 0,
    mode: str = "joint",
    force_sink_col: bool = False,
    row_total: np.ndarray | None = None,
    row_selected: np.ndarray | None = None,
) -> CoverageResult:
    """_build_direct_mean_coverage_mask (sparse_attention.py:268-376).

    joint (lines 334-376) and video_residual (lines 286-332, only with
    text_blocks > 0, as line 286-290 requires). row_total / row_selected, when
    given, replace the fp32 row sums of lines 334 and 339 (video mode: the
    sum over columns >= T of line 301); otherwise they are fp64 sums rounded
    to fp32.
    """
    s = np.ascontiguousarray(scores, dtype=np.float32)
    H, nq, nk = s.shape
    cov = np.float32(min(max(float(coverage), 0.0), 1.0))
    T = min(text_blocks, nq, nk) if text_blocks > 0 else 0
    video = mode in ("video_residual", "video_residual_only", "residual_video") and T > 0
    req = required_mask(nq, nk, T, force_sink_col and not video)
    mask = np.zeros((H, nq, nk), dtype=bool)
    ties = np.zeros((H, nq), dtype=bool)
    empty = np.zeros((H, nq), dtype=bool)
    eps = np.float32(1e-6)
    for h in range(H):
        for i in range(nq):
            row = s[h, i]
            if T > 0 and i < T:
                mask[h, i, :] = True
                continue
            if video:
                cols = np.arange(T, nk)
                vals = row[T:]
                if row_total is not None:
                    total = np.float32(row_total[h, i])
                else:
                    total = np.float32(vals.astype(np.float64).sum())
                total = max(total, eps)
                target = np.float32(cov * total)
                keep = np.zeros(nk, dtype=bool)
                keep[:T] = True
                order = np.argsort(-vals.astype(np.float64), kind="stable")
                sv = vals[order]
                sv = np.where(np.isfinite(sv), sv, np.float32(0)).astype(np.float32)
                cum = np.cumsum(sv.astype(np.float64)).astype(np.float32)
                n_cand = nk - T
                if target > eps:
                    f = _first_reach(cum, target)
                    k = f + 1 if f >= 0 else n_cand
                else:
                    k = 0
                k = max(0, min(k, n_cand))
                keep[cols[order[:k]]] = True
                if 0 < k < n_cand and sv[k - 1] == sv[k]:
                    ties[h, i] = True
                if not keep.any():
                    keep[int(np.argmax(row))] = True
                    empty[h, i] = True
                mask[h, i] = keep
                continue
            r = req[i]
            if row_total is not None:
                total = np.float32(row_total[h, i])
            else:
                total = np.float32(row.astype(np.float64).sum())
            if row_selected is not None:
                selected = np.float32(row_selected[h, i])
            else:
                selected = np.float32((row.astype(np.float64) * r).sum())
            total = max(total, eps)
            target = np.float32(cov * total)
            resid = np.float32(max(np.float32(target - selected), np.float32(0.0)))
            cand = np.where(r, -np.inf, row.astype(np.float64))
            order = np.argsort(-cand, kind="stable")
            sv = row[order].astype(np.float32)
            sv = np.where(r[order], np.float32(0), sv)
            sv = np.where(np.isfinite(sv), sv, np.float32(0)).astype(np.float32)
            cum = np.cumsum(sv.astype(np.float64)).astype(np.float32)
            n_cand = int((~r).sum())
            if resid > eps:
                f = _first_reach(cum, resid)
                k = f + 1 if f >= 0 else n_cand
            else:
                k = 0
            k = max(0, min(k, nk))
            keep = r.copy()
            keep[order[:k]] = True
            if 0 < k < n_cand and sv[k - 1] == sv[k]:
                ties[h, i] = True
            if keep_diagonal and i < min(nq, nk):
                keep[i] = True
            if not keep.any():
                keep[order[0]] = True
                empty[h, i] = True
                if n_cand > 1 and sv[0] == sv[1]:
                    ties[h, i] = True
            mask[h, i] = keep
    return CoverageResult(mask=mask, tie_rows=ties, empty_rows=empty)


# ---------------------------------------------------------------------------
# Calibrator statistics
# ---------------------------------------------------------------------------
def accumulate(sum_: np.ndarray | None, sumsq: np.ndarray | None, x: np.ndarray):
    """SinkMaskCalibrator._accumulate_score (sparse_attention.py:537-549)."""
    x = x.astype(np.float32)
    if sum_ is None:
        return x.copy(), (x * x).astype(np.float32)
    return (sum_ + x).astype(np.float32), (sumsq + x * x).astype(np.float32)


def finalize(sum_: np.ndarray, sumsq: np.ndarray, count) -> tuple[np.ndarray, np.ndarray]:
    """_build_mean_and_masks (sparse_attention.py:563-566)."""
    mean = (sum_ / np.float32(count) if np.isscalar(count) else sum_ / count).astype(np.float32)
    second = (sumsq / np.float32(count) if np.isscalar(count) else sumsq / count).astype(np.float32)
    var = np.maximum(second - mean * mean, 0).astype(np.float32)
    return mean, np.sqrt(var).astype(np.float32)


def zimage_align(scores: np.ndarray, image_blocks: int, text_blocks: int,
                 total_blocks: int) -> tuple[np.ndarray, np.ndarray]:
    """_align_scores_image_text_suffix and _alignment_presence_mask
    (zimg/runtime/sink_sparse_zimage.py:140-186): one sample's scores
    [H, n, n], n = image_blocks + text_blocks, placed in the fixed
    [H, total, total] layout with the image blocks first and this sample's
    text blocks last; presence is 1 where a score landed, else 0."""
    H, n, _ = scores.shape
    if n != image_blocks + text_blocks or scores.shape[2] != n:
        raise ValueError("Unexpected Z-Image block score shape. "
                         f"Expected {image_blocks + text_blocks}x{image_blocks + text_blocks}, "
                         f"got {n}x{scores.shape[2]}.")
    src = np.concatenate([np.arange(image_blocks),
                          np.arange(image_blocks, image_blocks + text_blocks)])
    dst = np.concatenate([np.arange(image_blocks),
                          np.arange(total_blocks - text_blocks, total_blocks)])
    aligned = np.zeros((H, total_blocks, total_blocks), np.float32)
    presence = np.zeros_like(aligned)
    aligned[:, dst[:, None], dst[None, :]] = scores[:, src[:, None], src[None, :]]
    presence[:, dst[:, None], dst[None, :]] = 1.0
    return aligned, presence


def finalize_presence(sum_: np.ndarray, sumsq: np.ndarray,
                      presence: np.ndarray) -> tuple[np.ndarray, np.ndarray, np.ndarray]:
    """ZImageSinkMaskCalibrator.build_package's statistics
    (zimg/runtime/sink_sparse_zimage.py:330-334): presence counts raised to
    at least 1, then the presence-weighted mean and std. Returns (mean, std,
    clamped presence)."""
    pres = np.maximum(presence, np.float32(1.0)).astype(np.float32)
    mean, std = finalize(sum_, sumsq, pres)
    return mean, std, pres


# ---------------------------------------------------------------------------
# Attention
# ---------------------------------------------------------------------------
def dense_masked_attention(
    q: np.ndarray,
    k: np.ndarray,
    v: np.ndarray,
    block_mask: np.ndarray,
    scale: float | None = None,
    block: int = 128,
    head_mask_type: np.ndarray | None = None,
    row_chunk: int = 512,
) -> tuple[np.ndarray, np.ndarray]:
    """Dense masked attention, the definition of block_sparse_attn_func
    (called at sinkattention/sparse_attention.py:735-771): per (b, h),
    softmax(q k^T * scale + M) v where M is -inf outside kept 128x128 blocks.

    q [B,H,Sq,D], k/v [B,H,Sk,D] fp32; block_mask bool [Bm,Hm,nq,nk] (Bm 1 or B).
    head_mask_type None => head h uses mask head h; else value t>0 => mask
    head t-1, 0 => dense. Returns out fp32 [B,H,Sq,D] and natural-log
    lse fp32 [B,H,Sq]; rows with no kept block give out 0 and lse -inf.
    """
    B, H, Sq, D = q.shape
    Sk = k.shape[2]
    if scale is None:
        scale = 1.0 / math.sqrt(D)
    out = np.zeros((B, H, Sq, D), dtype=np.float32)
    lse = np.full((B, H, Sq), -np.inf, dtype=np.float32)
    for b in range(B):
        mb = block_mask[b if block_mask.shape[0] > 1 else 0]
        for h in range(H):
            if head_mask_type is None:
                bm = mb[h]
            elif int(head_mask_type[h]) > 0:
                bm = mb[int(head_mask_type[h]) - 1]
            else:
                bm = np.ones_like(mb[0])
            tok = np.repeat(np.repeat(bm, block, axis=0), block, axis=1)[:Sq, :Sk]
            kt = k[b, h].astype(np.float32).T
            for r0 in range(0, Sq, row_chunk):
                r1 = min(Sq, r0 + row_chunk)
                sc = (q[b, h, r0:r1].astype(np.float32) @ kt) * np.float32(scale)
                sc = np.where(tok[r0:r1], sc, -np.inf)
                m = sc.max(axis=-1, keepdims=True)
                ok = np.isfinite(m[:, 0])
                m = np.where(np.isfinite(m), m, 0)
                p = np.exp(sc - m)
                l = p.sum(axis=-1, keepdims=True)
                with np.errstate(invalid="ignore", divide="ignore"):
                    o = (p @ v[b, h].astype(np.float32)) / l
                    lr = (np.log(l[:, 0]) + m[:, 0]).astype(np.float32)
                o[~ok] = 0
                lr[~ok] = -np.inf
                out[b, h, r0:r1] = o
                lse[b, h, r0:r1] = lr
    return out, lse


def mix_outputs(sink_out, sink_lse, dyn_out, dyn_lse, sample_gap: int):
    """_mix_attention_outputs, adaptive (sparse_attention.py:898-919), in fp32.
    lse arrays [B,H,S] (natural log)."""
    lg = math.log(float(max(1, int(sample_gap))))
    ws = sink_lse.astype(np.float64)
    wd = dyn_lse.astype(np.float64) + lg
    m = np.maximum(ws, wd)
    es, ed = np.exp(ws - m), np.exp(wd - m)
    alpha = (es / (es + ed))[..., None]
    return (sink_out * alpha + dyn_out * (1 - alpha)).astype(np.float32)


def kept_block_flops(block_mask: np.ndarray, B: int, H: int, Sq: int, Sk: int, D: int = 128,
                     block: int = 128, head_mask_type=None) -> float:
    """Algorithmic FLOPs of masked attention: 4*D per kept (query, key) pair,
    counting valid rows x valid columns of every kept block."""
    nq = (Sq + block - 1) // block
    nk = (Sk + block - 1) // block
    rows = np.full(nq, block, dtype=np.int64)
    rows[-1] = Sq - (nq - 1) * block
    cols = np.full(nk, block, dtype=np.int64)
    cols[-1] = Sk - (nk - 1) * block
    area = np.outer(rows, cols)
    total = 0
    for b in range(B):
        mb = block_mask[b if block_mask.shape[0] > 1 else 0]
        for h in range(H):
            if head_mask_type is None:
                bm = mb[h]
            elif int(head_mask_type[h]) > 0:
                bm = mb[int(head_mask_type[h]) - 1]
            else:
                bm = np.ones_like(mb[0])
            total += int((area * bm[:nq, :nk]).sum())
    return 4.0 * D * total


def sink_dynamic_attention(q, k, v, block_mask, k_pool, v_pool, sample_gap: int,
                           scale: float | None = None, block: int = 128):
    """The Wan runtime's sink + pooled-K/V adaptive mix as one softmax
    (wanx/runtime/sink_sparse_wan.py:210-265 with _mix_attention_outputs,
    sparse_attention.py:898-919): per row, keys = kept sink keys plus every
    pooled key, pooled logits raised by ln(sample_gap). Exact algebra of
    alpha*o_s + (1-alpha)*o_d with alpha = e^{lse_s}/(e^{lse_s}+gap*e^{lse_d}).
    Returns (out [B,H,Sq,D], lse [B,H,Sq])."""
    B, H, Sq, D = q.shape
    Sk = k.shape[2]
    if scale is None:
        scale = 1.0 / math.sqrt(D)
    lg = math.log(float(max(1, int(sample_gap))))
    out = np.zeros((B, H, Sq, D), dtype=np.float32)
    lse = np.zeros((B, H, Sq), dtype=np.float32)
    for b in range(B):
        mb = block_mask[b if block_mask.shape[0] > 1 else 0]
        for h in range(H):
            tok = np.repeat(np.repeat(mb[h], block, axis=0), block, axis=1)[:Sq, :Sk]
            s1 = (q[b, h].astype(np.float64) @ k[b, h].astype(np.float64).T) * scale
            s1 = np.where(tok, s1, -np.inf)
            s2 = (q[b, h].astype(np.float64) @ k_pool[b, h].astype(np.float64).T) * scale + lg
            s = np.concatenate([s1, s2], axis=1)
            m = s.max(axis=1, keepdims=True)
            p = np.exp(s - m)
            l = p.sum(axis=1, keepdims=True)
            vv = np.concatenate([v[b, h], v_pool[b, h]], axis=0).astype(np.float64)
            out[b, h] = (p @ vv / l).astype(np.float32)
            lse[b, h] = (np.log(l[:, 0]) + m[:, 0]).astype(np.float32)
    return out, lse


def exact_block_mass_scores(q: np.ndarray, k: np.ndarray, block: int = 128) -> np.ndarray:
    """_compute_exact_block_mass_scores (sinkattention/sparse_attention.py:145-227):
    per query block, the mean over its rows of each key block's share of the
    row's softmax mass; row sums clamped at 1e-6 (line 224). [B,H,nq,nk]."""
    B, H, S, D = q.shape
    Sk = k.shape[2]
    scale = 1.0 / math.sqrt(D)
    nq, nk = -(-S // block), -(-Sk // block)
    out = np.zeros((B, H, nq, nk), dtype=np.float32)
    for b in range(B):
        for h in range(H):
            s = (q[b, h].astype(np.float64) @ k[b, h].astype(np.float64).T) * scale
            m = s.max(axis=1, keepdims=True)
            e = np.exp(s - m)
            rs = np.maximum(e.sum(axis=1, keepdims=True), 1e-6)
            pad = nk * block - Sk
            if pad:
                e = np.concatenate([e, np.zeros((S, pad))], axis=1)
            mass = e.reshape(S, nk, block).sum(axis=2) / rs
            for i in range(nq):
                out[b, h, i] = mass[i * block:min(S, (i + 1) * block)].mean(axis=0)
    return out


def triton_max_pool_scores(q: np.ndarray, k: np.ndarray, block: int = 128) -> np.ndarray:
    """The statistics of the Triton kernel attn_with_pooling
    (sinkattention/pooling_kernel.py:11-248):
      R[r,kb]  = bf16(max_{n in kb} (q_r . k_n) * qk_scale),
                 qk_scale = fp32(sm_scale) * fp32(1.44269504)   (lines 45-48, 161-162)
      m_r      = max over kb of the unrounded values             (line 46)
      Po[i,kb] = bf16(max_{r in block i} exp2(R[r,kb] - m_r))   (lines 65-75, l_i = 1)
      scores   = Po / sum(Po, -1) with bf16 tensors              (lines 243-244).
    Keys past S in the last block are masked (lines 34-41). For S not a
    multiple of `block` the Triton kernel also reads query rows past the end
    of the head; here those rows take no part in the column maxima."""
    B, H, S, D = q.shape
    nb = -(-S // block)
    pad = nb * block - S
    qk_scale = np.float32(np.float32(1.0 / math.sqrt(D)) * np.float32(1.44269504))
    out = np.zeros((B, H, nb, nb), dtype=np.float32)
    for b in range(B):
        for h in range(H):
            s = (q[b, h].astype(np.float64) @ k[b, h].astype(np.float64).T).astype(np.float32)
            if pad:
                s = np.concatenate([s, np.full((S, pad), -np.inf, np.float32)], axis=1)
            bmax = s.reshape(S, nb, block).max(axis=2)
            R = (bmax * qk_scale).astype(np.float32)
            m = R.max(axis=1, keepdims=True)
            Rb = bf16_round(R)
            x = np.exp2((Rb - m).astype(np.float64)).astype(np.float32)
            if pad:
                x = np.concatenate([x, np.zeros((pad, nb), np.float32)], axis=0)
            po = bf16_round(x.reshape(nb, block, nb).max(axis=1))
            tot = bf16_round(po.astype(np.float64).sum(axis=1, keepdims=True).astype(np.float32))
            out[b, h] = bf16_round((po / tot).astype(np.float32))
    return out


def qk_norm_rope(x: np.ndarray, w: np.ndarray, eps: float, cos: np.ndarray, sin: np.ndarray,
                 heads: int) -> np.ndarray:
    """The Wan Q/K producer (wanx/runtime/sink_sparse_wan.py:300-315): RMSNorm
    over the hidden dimension (fast_misc.py:306-340: y = x * rstd * w,
    rstd = 1/sqrt(mean(x^2) + eps)), rounded to bf16, split into heads, then
    the rotary product per channel pair (fast_misc.py:173-194: out_2i =
    y_2i cos - y_2i+1 sin, out_2i+1 = y_2i sin + y_2i+1 cos), rounded to bf16.
    x [B,S,hidden], w [hidden], cos/sin [S, D/2]; returns [B,H,S,D]."""
    xf = x.astype(np.float64)
    ms = (xf * xf).mean(axis=-1, keepdims=True)
    y = bf16_round((xf / np.sqrt(ms + eps) * w.astype(np.float64)).astype(np.float32))
    B, S, hidden = x.shape
    D = hidden // heads
    y = y.reshape(B, S, heads, D).transpose(0, 2, 1, 3).astype(np.float64)
    ye, yo = y[..., 0::2], y[..., 1::2]
    c = cos.astype(np.float64)[None, None]
    s = sin.astype(np.float64)[None, None]
    out = np.empty_like(y)
    out[..., 0::2] = ye * c - yo * s
    out[..., 1::2] = ye * s + yo * c
    return bf16_round(out.astype(np.float32))


def bf16_ulp_distance(a: np.ndarray, b: np.ndarray) -> np.ndarray:
    """Distance in bf16 steps between arrays of bf16-representable values."""
    def key(v):
        u = (np.ascontiguousarray(v, dtype=np.float32).view(np.uint32) >> 16).astype(np.int64)
        return np.where(u & 0x8000, 0x8000 - u, u)  # monotone integer order
    return np.abs(key(a) - key(b))

"""Drop-in replacements for the reference's hot-path entry points.

The reference (bb-2020-bb/sinkattn) reaches its kernels through a handful of
module-level names. This module provides same-named, same-signature
functions backed by libsinkattn, and install() binds them into the
reference's modules so the Wan and Z-Image processors run unchanged:

  sinkattention.sparse_attention.block_sparse_attn_func
      external Block-Sparse-Attention forward (sparse_attention.py:22-28, 735-771)
  sinkattention.sparse_attention._block_sparse_attn            (lines 710-776)
  sinkattention.sparse_attention._compute_pooled_qk_block_scores (lines 118-142)
  sinkattention.sparse_attention._compute_exact_block_mass_scores (lines 145-227)
  sinkattention.sparse_attention._build_direct_mean_coverage_mask (lines 268-376)
  sinkattention.sparse_attention._mean_pool_sequence_preserve_prefix (lines 97-115)
  sinkattention.sparse_attention._mix_attention_outputs        (lines 898-919)

Callers that imported a name into their own namespace are patched too
(wanx/runtime/sink_sparse_wan.py:10-26, zimg/runtime/sink_sparse_zimage.py:15-26).

Errors follow the reference: shape problems raise ValueError with the same
messages; kernel failures raise RuntimeError. Nothing here falls back to CPU
computation — CPU tensors raise.
"""
from __future__ import annotations

import math
import sys
from typing import Optional

import torch

from . import ops

# How head_mask_type is read by block_sparse_attn_func.
#   "per_head" (default): a mask with one slice per head is applied per head;
#       positive entries are ignored, 0 entries mark dense heads. This is the
#       per-head semantics the sink masks are calibrated with.
#   "upstream": the Block-Sparse-Attention reading — a positive entry t makes
#       the head use mask slice t-1 (so the reference's ones(H) would apply
#       slice 0 to every head), 0 = dense.
HEAD_MASK_TYPE_MODE = "per_head"

_BLOCK = 128


def _reports_device_failures(fn):
    """Checks, on entry, that no earlier kernel on the call's device
    reported a bounded wait that gave up (ops.DeviceStatus, read from host
    memory without synchronising) and raises RuntimeError if one did, so a
    stalled launch surfaces at the next call instead of passing on wrong
    outputs. Calls whose first tensor argument is not on a GPU go straight
    through (they raise their own error)."""
    import functools

    @functools.wraps(fn)
    def wrapper(*args, **kwargs):
        for a in args:
            if isinstance(a, torch.Tensor):
                if a.is_cuda:
                    ops.DeviceStatus.raise_if_set(a.device)
                break
        return fn(*args, **kwargs)

    return wrapper


def _hmt_host(head_mask_type: torch.Tensor) -> list[int]:
    # small int32 [H]; cached on the tensor's identity and version counter
    key = (head_mask_type.data_ptr(), head_mask_type._version, head_mask_type.numel())
    cached = _HMT_CACHE.get(key)
    if cached is None:
        cached = [int(x) for x in head_mask_type.detach().cpu().tolist()]
        _HMT_CACHE[key] = cached
    return cached


_HMT_CACHE: dict = {}


@_reports_device_failures
def block_sparse_attn_func(
    q_unpad,
    k_unpad,
    v_unpad,
    cu_seqlens_q,
    cu_seqlens_k,
    head_mask_type,
    streaming_info,
    base_blockmask,
    max_seqlen_q_,
    max_seqlen_k_,
    p_dropout=0.0,
    deterministic=False,
    softmax_scale=None,
    is_causal=False,
    exact_streaming=False,
    return_attn_probs=False,
):
    """Block-sparse attention forward with the upstream package's signature.

    q_unpad [total_q, H, D], k_unpad/v_unpad [total_k, H, D] (bf16, varlen
    packing described by cu_seqlens_*), base_blockmask bool
    [B, Hm, ceil(max_seqlen_q/128), ceil(max_seqlen_k/128)].
    Returns out [total_q, H, D], or (out, softmax_lse fp32 [B, H, max_seqlen_q],
    None) when return_attn_probs.
    """
    if p_dropout != 0.0:
        raise NotImplementedError("sinkattn_b200: dropout is not supported (forward inference only)")
    if is_causal:
        raise NotImplementedError("sinkattn_b200: causal masking is not supported")
    if exact_streaming:
        raise NotImplementedError("sinkattn_b200: streaming heads are not supported")
    total_q, H, D = q_unpad.shape
    total_k = k_unpad.shape[0]
    B = int(cu_seqlens_q.numel()) - 1
    Sq, Sk = int(max_seqlen_q_), int(max_seqlen_k_)
    hmt = None
    if HEAD_MASK_TYPE_MODE == "upstream":
        hv = _hmt_host(head_mask_type)
        if any(t < 0 for t in hv):
            raise NotImplementedError("sinkattn_b200: streaming heads (head_mask_type < 0)")
        hmt = head_mask_type.to(torch.int32)
    elif base_blockmask.shape[1] != H:
        # fewer mask slices than heads only makes sense with the mapping
        hv = _hmt_host(head_mask_type)
        if any(t < 0 for t in hv):
            raise NotImplementedError("sinkattn_b200: streaming heads (head_mask_type < 0)")
        hmt = head_mask_type.to(torch.int32)
    if total_q == B * Sq and total_k == B * Sk:
        # uniform batch: every sequence has the maximum length (the reference's case)
        q = q_unpad.view(B, Sq, H, D).permute(0, 2, 1, 3)
        k = k_unpad.view(B, Sk, H, D).permute(0, 2, 1, 3)
        v = v_unpad.view(B, Sk, H, D).permute(0, 2, 1, 3)
        out = torch.empty_like(q_unpad)
        out_v = out.view(B, Sq, H, D).permute(0, 2, 1, 3)
        _, lse = ops.bsattn_fwd(q, k, v, base_blockmask, softmax_scale=softmax_scale,
                                head_mask_type=hmt, return_lse=bool(return_attn_probs), out=out_v)
    else:
        # ragged varlen batch: one launch per sequence on its own slice
        cq = [int(x) for x in cu_seqlens_q.detach().cpu().tolist()]
        ck = [int(x) for x in cu_seqlens_k.detach().cpu().tolist()]
        out = torch.empty_like(q_unpad)
        lse = (torch.full((B, H, Sq), float("-inf"), dtype=torch.float32, device=q_unpad.device)
               if return_attn_probs else None)
        for b in range(B):
            sq, sk = cq[b + 1] - cq[b], ck[b + 1] - ck[b]
            if sq == 0:
                continue
            qb = q_unpad[cq[b]:cq[b + 1]].unsqueeze(0).permute(0, 2, 1, 3)
            kb = k_unpad[ck[b]:ck[b + 1]].unsqueeze(0).permute(0, 2, 1, 3)
            vb = v_unpad[ck[b]:ck[b + 1]].unsqueeze(0).permute(0, 2, 1, 3)
            mb = base_blockmask[b:b + 1, :, : math.ceil(sq / _BLOCK), : math.ceil(sk / _BLOCK)]
            ob = out[cq[b]:cq[b + 1]].unsqueeze(0).permute(0, 2, 1, 3)
            if sk == 0:
                ob.zero_()
                continue
            _, lb = ops.bsattn_fwd(qb, kb, vb, mb, softmax_scale=softmax_scale, head_mask_type=hmt,
                                   return_lse=bool(return_attn_probs), out=ob)
            if lse is not None:
                lse[b, :, :sq] = lb[0]
    if return_attn_probs:
        return out, lse, None
    return out


@_reports_device_failures
def _block_sparse_attn(
    q: torch.Tensor,
    k: torch.Tensor,
    v: torch.Tensor,
    block_mask: torch.Tensor,
    return_lse: bool = True,
) -> tuple[torch.Tensor, Optional[torch.Tensor]]:
    """sparse_attention.py:710-776 without the three transpose copies: the
    kernel reads the strided [B,H,S,D] views directly through TMA. Returns
    out as a [B,S,H,D]-contiguous tensor viewed [B,H,S,D] (the reference's
    layout) and lse [B,H,S,1] in q.dtype (line 776)."""
    B, H, Sq, D = q.shape
    if HEAD_MASK_TYPE_MODE == "upstream":
        # the reference passes ones(H): every head reads mask slice 0
        hmt = torch.ones(H, dtype=torch.int32, device=q.device)
    else:
        hmt = None
    out, lse = ops.bsattn_fwd(q, k, v, block_mask.contiguous(), head_mask_type=hmt,
                              return_lse=return_lse)
    if lse is None:
        return out, None
    return out, lse.unsqueeze(-1).to(device=q.device, dtype=q.dtype)


def _bf16(t: torch.Tensor) -> torch.Tensor:
    return t if t.dtype == torch.bfloat16 else t.to(torch.bfloat16)


@_reports_device_failures
def _compute_pooled_qk_block_scores(q, k, v, config) -> torch.Tensor:
    """sparse_attention.py:118-142, [B,H,nb,nb] fp32.

    pooling_mode "triton" (compared case-sensitively, as line 124 does) runs
    the block-maximum statistics of the reference's Triton kernel
    (pooling_kernel.py:11-248) on the tensor cores; any other mode gets the
    mean rule softmax(pool(q) pool(k)^T / sqrt(D)) of lines 138-142."""
    if config.pooling_mode == "triton":
        if int(config.block_size) != _BLOCK:
            raise NotImplementedError(
                f"triton pooling runs with block_size {_BLOCK} only, got {config.block_size}")
        return ops.block_stats(_bf16(q), _bf16(k), mode="max", scale=1.0 / math.sqrt(q.size(-1)))
    block = int(config.block_size)
    scores, _ = ops.pool_scores(_bf16(q), _bf16(k), block=block, scale=1.0 / math.sqrt(q.size(-1)))
    return scores


@_reports_device_failures
def _compute_exact_block_mass_scores(q, k, config) -> torch.Tensor:
    """sparse_attention.py:145-227: per query block, the mean over its rows of
    each key block's share of the row's softmax mass, [B,H,nq,nk] fp32, from
    one tensor-core pass per query tile instead of two chunked fp32 matmul
    sweeps per query block."""
    if int(config.block_size) != _BLOCK:
        raise NotImplementedError(
            f"exact block-mass scores run with block_size {_BLOCK} only, got {config.block_size}")
    if q.shape != k.shape:
        raise NotImplementedError(
            f"exact block-mass scores need q and k of one shape, got {tuple(q.shape)} and "
            f"{tuple(k.shape)}")
    return ops.block_stats(_bf16(q), _bf16(k), mode="exact", scale=1.0 / math.sqrt(q.size(-1)))


def _compute_block_scores(q, k, v, config) -> torch.Tensor:
    """sparse_attention.py:230-238: the calibration score mode dispatch over the
    drop-ins above."""
    pooling_mode = str(config.pooling_mode).strip().lower()
    if pooling_mode == "exact":
        return _compute_exact_block_mass_scores(q, k, config)
    if pooling_mode in {"triton", "mean"}:
        return _compute_pooled_qk_block_scores(q, k, v, config)
    raise ValueError(
        f"Unsupported pooling_mode: {config.pooling_mode}. Expected one of: exact, triton, mean.")


def _ceil_div(a: int, b: int) -> int:
    return (a + b - 1) // b


@_reports_device_failures
def _build_direct_mean_coverage_mask(mean_scores: torch.Tensor, config) -> torch.Tensor:
    """sparse_attention.py:268-376 on the GPU. The fp32 row totals (line 334,
    301) and selected sums (line 339) are taken with the same torch reduction
    on the same device as the reference, so the decisions are bit-identical;
    the sort, cumulative sums, cut and scatter run in the CUDA kernel. The
    mask is returned on the input's device."""
    if mean_scores.dim() != 3:
        raise ValueError(f"Expected [heads, blocks_q, blocks_k] scores, got {tuple(mean_scores.shape)}")
    H, nq, nk = mean_scores.shape
    coverage = min(max(float(config.offline_direct_coverage), 0.0), 1.0)
    mode = str(getattr(config, "offline_text_video_coverage_mode", "joint")).strip().lower()
    text_blocks = 0
    if bool(getattr(config, "force_text_global_attention", False)) and int(config.text_length) > 0:
        text_blocks = _ceil_div(int(config.text_length), int(config.block_size))
    T = min(text_blocks, nq, nk)
    scores = mean_scores.float()
    video = mode in {"video_residual", "video_residual_only", "residual_video"} and T > 0
    if video:
        row_total = torch.zeros(H, nq, dtype=torch.float32, device=scores.device)
        if nq - T > 0 and nk - T > 0:
            row_total[:, T:] = scores[:, T:, T:].sum(dim=-1)
        row_selected = None
    else:
        row_total = scores.sum(dim=-1)
        if T > 0:
            req = torch.zeros(nq, nk, dtype=torch.bool, device=scores.device)
            req[:, :T] = True
            req[:T, :] = True
            row_selected = (scores * req.unsqueeze(0).expand(H, -1, -1).float()).sum(dim=-1)
        else:
            row_selected = torch.zeros(H, nq, dtype=torch.float32, device=scores.device)
    dev = scores.device if scores.is_cuda else torch.device("cuda", torch.cuda.current_device())
    mask, _ = ops.coverage_mask(
        scores.to(dev), coverage=coverage, keep_diagonal=bool(config.keep_diagonal),
        text_blocks=T, mode="video_residual" if video else "joint",
        row_total=row_total.to(dev),
        row_selected=None if row_selected is None else row_selected.to(dev),
    )
    return mask if mean_scores.is_cuda else mask.to(mean_scores.device)


@_reports_device_failures
def _mean_pool_sequence_preserve_prefix(x: torch.Tensor, pool_size: int, *, prefix_tokens: int = 0):
    """sparse_attention.py:97-115 (bf16 in/out, fp32 accumulation)."""
    if pool_size <= 1:
        return x
    return ops.mean_pool_seq(x, int(pool_size), int(prefix_tokens))


@_reports_device_failures
def _mean_pool_sequence(x: torch.Tensor, pool_size: int):
    """sparse_attention.py:88-94 for bf16 tensors (Z-Image pooled branch)."""
    if pool_size <= 1:
        return x
    return ops.mean_pool_seq(x, int(pool_size), 0)


@_reports_device_failures
def _mix_attention_outputs(sink_out, sink_lse, dynamic_out, dynamic_lse, config, dynamic_sample_gap=None):
    """sparse_attention.py:898-919 (adaptive mode) as one fused kernel."""
    if config.mixing_mode != "adaptive":
        raise ValueError(f"Unsupported mixing_mode: {config.mixing_mode}")
    if sink_lse is None or dynamic_lse is None:
        raise ValueError("Adaptive Sink-Sparse mixing requires both sink_lse and dynamic_lse.")
    gap = config.sample_gap if dynamic_sample_gap is None else int(dynamic_sample_gap)
    return ops.mix_outputs(sink_out, sink_lse, dynamic_out, dynamic_lse, gap)


@_reports_device_failures
def fused_wan_inner_forward(self, q, k, v):
    """WanSinkSparseInnerAttention.forward (wanx/runtime/sink_sparse_wan.py:181-282)
    with the sink call, the pooled K/V dynamic call and the adaptive mix fused
    into one kernel (sa_sink_dynamic_attn_fwd).

    The runtime mask, timing sections and mask statistics are the reference
    method's own. Configurations other than the Wan default (dynamic_mode
    pooled_kv, adaptive mixing, block-sparse dynamic kernel) run the
    reference's unfused method, which uses the other drop-in functions.
    """
    from contextlib import nullcontext

    cfg = self.config
    mode, gap = self._resolve_dynamic_plan()
    fusable = (mode == "pooled_kv" and cfg.mixing_mode == "adaptive"
               and str(cfg.dynamic_kernel) in {"block_sparse", "auto"})
    if not fusable:
        return _UNFUSED_WAN_FORWARD[0](self, q, k, v)
    time_section = self.runtime_state.time_section if self.runtime_state is not None else None
    with (time_section("inner_total") if time_section is not None else nullcontext()):
        with (time_section("mask_prepare") if time_section is not None else nullcontext()):
            sink_mask_tag = "__base__"
            base_runtime_mask = self._get_runtime_mask(
                sink_mask=self.sink_mask, mask_tag=sink_mask_tag, batch_size=q.size(0),
                num_heads=q.size(1), seq_len_q=q.size(2), seq_len_k=k.size(2), device=q.device)
        with (time_section("comp_pool") if time_section is not None else nullcontext()):
            prefix_tokens = max(int(cfg.text_length), 0)
            k_dyn = _mean_pool_sequence_preserve_prefix(k, gap, prefix_tokens=prefix_tokens)
            v_dyn = _mean_pool_sequence_preserve_prefix(v, gap, prefix_tokens=prefix_tokens)
            dynamic_seq_len_k = int(k_dyn.size(2))
        with (time_section("sparse_main") if time_section is not None else nullcontext()):
            mixed_out, _ = ops.sink_dynamic_attn(q, k, v, base_runtime_mask, k_dyn, v_dyn, gap)
        if self.runtime_state is not None:
            with self.runtime_state.time_section("stats"):
                self.runtime_state.record_mask_stats(
                    layer_idx=self.layer_idx, sink_mask_tag=sink_mask_tag, dynamic_mode=mode,
                    dynamic_sample_gap=gap, base_runtime_mask=base_runtime_mask,
                    topup_mask=None, dynamic_seq_len_k=dynamic_seq_len_k,
                    total_seq_len_k=int(k.size(2)))
        return mixed_out


_UNFUSED_WAN_FORWARD: list = []


def _rotary_tables(freqs, S: int, D: int):
    """cos/sin fp32 [S, D/2] from the rotary embedding the Wan processor gets:
    a complex tensor [1,1,S,D/2] or [S,D/2] (wanx/runtime/fast_misc.py:711-720),
    a (real, imag) pair of [S,D/2] tensors, or Wan's (cos, sin) pair repeated
    per channel, [1,S,1,D], read at even and odd channels (fast_misc.py:145-170)."""
    if isinstance(freqs, torch.Tensor) and torch.is_complex(freqs):
        re, im = freqs.real, freqs.imag
    elif isinstance(freqs, (tuple, list)) and len(freqs) == 2:
        re, im = freqs
        if re.shape[-1] == D and re.numel() == S * D:
            re, im = re.reshape(S, D)[:, 0::2], im.reshape(S, D)[:, 1::2]
    else:
        raise TypeError(f"Unsupported rotary embedding type: {type(freqs)!r}")
    return re.reshape(S, D // 2).float(), im.reshape(S, D // 2).float()


def _rms_like(norm) -> bool:
    # the RMSNorm test of apply_fast_qk_norm (fast_misc.py:846-852)
    if norm is None or getattr(norm, "weight", None) is None or getattr(norm, "eps", None) is None:
        return False
    return "layernorm" not in norm.__class__.__name__.lower() and getattr(norm, "bias", None) is None


@_reports_device_failures
def fused_prepare_attention_tensors(attn, hidden_states, encoder_hidden_states=None,
                                    rotary_emb=None):
    """_prepare_attention_tensors (wanx/runtime/sink_sparse_wan.py:285-315) for
    self-attention with RMS-normalised Q/K and a rotary embedding: the Q/K
    RMSNorm and the rotation run as one kernel (sa_qk_norm_rope) on the
    projections' outputs. Q, K and V come back as [B,H,S,D] views of the
    [B,S,H*D] projections, the layout the attention kernel reads. Other
    configurations run the reference's own function."""
    norm_q, norm_k = getattr(attn, "norm_q", None), getattr(attn, "norm_k", None)
    fusable = (encoder_hidden_states is None and rotary_emb is not None
               and hidden_states.is_cuda and _rms_like(norm_q) and _rms_like(norm_k))
    if not fusable:
        return _UNFUSED_PREPARE[0](attn, hidden_states, encoder_hidden_states, rotary_emb)
    from contextlib import nullcontext

    timing = getattr(getattr(attn, "inner_attention", None), "timing", None)
    query = attn.to_q(hidden_states)
    key = attn.to_k(hidden_states)
    value = attn.to_v(hidden_states)
    if query.dtype != torch.bfloat16:
        return _UNFUSED_PREPARE[0](attn, hidden_states, encoder_hidden_states, rotary_emb)
    S = query.shape[1]
    D = query.shape[-1] // attn.heads
    with (timing.section("qk_norm") if timing is not None and timing.is_enabled else nullcontext()):
        cos, sin = _rotary_tables(rotary_emb, S, D)
        in_place = not (query.requires_grad or key.requires_grad)
        query, key = ops.qk_norm_rope(query, key, D, float(norm_q.eps), norm_q.weight,
                                      norm_k.weight, cos.to(query.device), sin.to(query.device),
                                      out_q=query if in_place else None,
                                      out_k=key if in_place else None)
    query = query.unflatten(2, (attn.heads, -1)).transpose(1, 2)
    key = key.unflatten(2, (attn.heads, -1)).transpose(1, 2)
    value = value.unflatten(2, (attn.heads, -1)).transpose(1, 2)
    return query, key, value, None


_UNFUSED_PREPARE: list = []


_PATCHES = {
    "sinkattention.sparse_attention": {
        "block_sparse_attn_func": block_sparse_attn_func,
        "_HAS_BLOCK_SPARSE": True,
        "_block_sparse_attn": _block_sparse_attn,
        "_compute_pooled_qk_block_scores": _compute_pooled_qk_block_scores,
        "_compute_exact_block_mass_scores": _compute_exact_block_mass_scores,
        "_build_direct_mean_coverage_mask": _build_direct_mean_coverage_mask,
        "_mean_pool_sequence_preserve_prefix": _mean_pool_sequence_preserve_prefix,
        "_mix_attention_outputs": _mix_attention_outputs,
    },
    "wanx.runtime.sink_sparse_wan": {
        "_block_sparse_attn": _block_sparse_attn,
        "_mean_pool_sequence_preserve_prefix": _mean_pool_sequence_preserve_prefix,
        "_mix_attention_outputs": _mix_attention_outputs,
    },
    "zimg.runtime.sink_sparse_zimage": {
        "_block_sparse_attn": _block_sparse_attn,
        "_build_direct_mean_coverage_mask": _build_direct_mean_coverage_mask,
        "_mean_pool_sequence": _mean_pool_sequence,
        "_mix_attention_outputs": _mix_attention_outputs,
    },
}


def install(modules: Optional[list[str]] = None, fused_dynamic: bool = True) -> list[str]:
    """Bind the replacements into the reference's modules (importing them if
    needed). Returns the list of patched module names. A module whose import
    fails with ImportError (a route whose dependencies are absent) is skipped,
    unless the caller named it in `modules`, in which case the error is
    raised. With fused_dynamic, WanSinkSparseInnerAttention.forward
    is replaced by fused_wan_inner_forward (one kernel for the sink branch, the
    pooled dynamic branch and their mix). In the Wan runtime the Q/K RMSNorm and
    rotary embedding become one kernel (fused_prepare_attention_tensors)."""
    import importlib

    patched = []
    for name, attrs in _PATCHES.items():
        if modules is not None and name not in modules:
            continue
        try:
            mod = sys.modules.get(name) or importlib.import_module(name)
        except ImportError:
            if modules is not None:
                raise
            continue
        for attr, val in attrs.items():
            setattr(mod, attr, val)
        if name == "wanx.runtime.sink_sparse_wan":
            orig = getattr(mod, "_prepare_attention_tensors", None)
            if orig is not None and orig is not fused_prepare_attention_tensors:
                _UNFUSED_PREPARE[:] = [orig]
                mod._prepare_attention_tensors = fused_prepare_attention_tensors
        if fused_dynamic and name == "wanx.runtime.sink_sparse_wan":
            cls = getattr(mod, "WanSinkSparseInnerAttention", None)
            if cls is not None and cls.forward is not fused_wan_inner_forward:
                _UNFUSED_WAN_FORWARD[:] = [cls.forward]
                cls.forward = fused_wan_inner_forward
        patched.append(name)
    return patched

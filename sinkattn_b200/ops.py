"""Tensor-level wrappers over libsinkattn (torch provides memory and streams).

Every function takes CUDA tensors, passes their data pointers and element
strides straight to the C ABI (no copies for any strided layout the kernels
accept) and launches on torch's current stream. CPU tensors are rejected:
there is no CPU path.
"""
from __future__ import annotations

import math
from typing import Optional

import torch

from . import _lib

BLOCK = 128


def _stream(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def _require_cuda(*ts: torch.Tensor) -> torch.device:
    dev = None
    for t in ts:
        if t is None:
            continue
        if not t.is_cuda:
            raise RuntimeError(
                "sinkattn_b200 runs on CUDA tensors only (got a tensor on "
                f"{t.device}); there is no CPU fallback"
            )
        if dev is None:
            dev = t.device
        elif t.device != dev:
            raise RuntimeError(f"tensors on different devices: {dev} and {t.device}")
    return dev


def _ptr(t: Optional[torch.Tensor]):
    return None if t is None else t.data_ptr()


def _bf16_view_ok(t: torch.Tensor) -> bool:
    if t.stride(-1) != 1:
        return False
    if any(s % 8 for s in t.stride()[:-1]):
        return False
    return t.data_ptr() % 16 == 0


def _as_kernel_layout(t: torch.Tensor) -> torch.Tensor:
    """Return t itself when its strides are TMA/16-byte compatible, else a
    contiguous copy (the only case where a copy is made)."""
    return t if _bf16_view_ok(t) else t.contiguous()


class DeviceStatus:
    """The status word kernels write when a bounded wait gives up, one per
    device, in mapped page-locked host memory (sa_status_create): kernels
    write it only on failure, and the host reads it at any time without
    synchronising. The reference-facing drop-ins call raise_if_set() on entry,
    so a failed launch is reported at the next call; check() synchronises
    first, for a verdict on every launch issued so far."""

    _words: dict[int, tuple[int, int]] = {}  # device -> (host address, device address)

    @classmethod
    def _word(cls, idx: int) -> tuple[int, int]:
        w = cls._words.get(idx)
        if w is None:
            lib = _lib.load()
            host = lib.sa_status_create()
            if not host:
                raise RuntimeError(f"sa_status_create failed: {_lib.last_error()}")
            dev_ptr = _lib.ctypes.c_void_p()
            _lib.check(lib.sa_status_device_pointer(host, _lib.ctypes.byref(dev_ptr)),
                       "sa_status_device_pointer")
            w = (int(host), int(dev_ptr.value))
            cls._words[idx] = w
        return w

    @staticmethod
    def _index(device: Optional[torch.device]) -> int:
        if device is None or device.index is None:
            return torch.cuda.current_device()
        return device.index

    @classmethod
    def pointer(cls, device: torch.device) -> int:
        """The address kernels on `device` write their status to."""
        return cls._word(cls._index(device))[1]

    @classmethod
    def value(cls, device: Optional[torch.device] = None) -> int:
        """The word as the host sees it now (no synchronisation)."""
        return int(_lib.ctypes.c_int32.from_address(cls._word(cls._index(device))[0]).value)

    @classmethod
    def raise_if_set(cls, device: Optional[torch.device] = None) -> None:
        """Raise RuntimeError (and reset the word) if a kernel already
        reported a failure; no synchronisation."""
        idxs = [cls._index(device)] if device is not None else list(cls._words)
        for idx in idxs:
            host = cls._word(idx)[0]
            rc = _lib.load().sa_check_status(host)
            if rc != _lib.SA_OK:
                raise RuntimeError(f"sinkattn_b200 on cuda:{idx}: {_lib.last_error()}")

    @classmethod
    def check(cls, device: Optional[torch.device] = None) -> None:
        """Synchronise and raise if any kernel on `device` (all devices used
        so far when None) reported a timeout."""
        idxs = [cls._index(device)] if device is not None else list(cls._words)
        for idx in idxs:
            torch.cuda.synchronize(idx)
            cls.raise_if_set(torch.device("cuda", idx))


def bsattn_fwd(
    q: torch.Tensor,
    k: torch.Tensor,
    v: torch.Tensor,
    block_mask: torch.Tensor,
    softmax_scale: Optional[float] = None,
    head_mask_type: Optional[torch.Tensor] = None,
    return_lse: bool = True,
    out: Optional[torch.Tensor] = None,
    lse: Optional[torch.Tensor] = None,
):
    """Block-sparse attention forward on [B,H,S,D] bf16 views (any strides).

    block_mask: bool [Bm,Hm,ceil(Sq/128),ceil(Sk/128)], Bm in {1,B}.
    head_mask_type: optional int32 [H] on the device (t>0 -> mask head t-1,
    0 -> dense); None -> mask head h for head h.
    Returns (out [B,H,Sq,D] bf16, lse fp32 [B,H,Sq] or None). `out` defaults to
    a [B,Sq,H,D]-contiguous buffer viewed as [B,H,Sq,D].
    """
    dev = _require_cuda(q, k, v, block_mask, head_mask_type)
    if q.dtype != torch.bfloat16 or k.dtype != torch.bfloat16 or v.dtype != torch.bfloat16:
        raise RuntimeError(f"bsattn_fwd expects bf16 q/k/v, got {q.dtype}/{k.dtype}/{v.dtype}")
    if q.dim() != 4 or k.dim() != 4 or v.dim() != 4:
        raise RuntimeError("bsattn_fwd expects 4-D [B,H,S,D] tensors")
    B, H, Sq, D = q.shape
    Sk = k.shape[2]
    if k.shape != (B, H, Sk, D) or v.shape != (B, H, Sk, D):
        raise RuntimeError(f"shape mismatch q{tuple(q.shape)} k{tuple(k.shape)} v{tuple(v.shape)}")
    nq, nk = math.ceil(Sq / BLOCK), math.ceil(Sk / BLOCK)
    if block_mask.dim() != 4 or block_mask.shape[-2:] != (nq, nk):
        raise RuntimeError(
            f"block_mask must be [B|1, Hm, {nq}, {nk}], got {tuple(block_mask.shape)}")
    if block_mask.shape[0] not in (1, B):
        raise RuntimeError(f"block_mask batch dim must be 1 or {B}")
    if block_mask.dtype not in (torch.bool, torch.uint8):
        raise RuntimeError(f"block_mask must be bool/uint8, got {block_mask.dtype}")
    Hm = block_mask.shape[1]
    if head_mask_type is not None:
        if head_mask_type.dtype != torch.int32 or head_mask_type.numel() != H:
            raise RuntimeError("head_mask_type must be int32 [H]")
        head_mask_type = head_mask_type.contiguous()
    q, k, v = _as_kernel_layout(q), _as_kernel_layout(k), _as_kernel_layout(v)
    if out is None:
        out = torch.empty((B, Sq, H, D), dtype=q.dtype, device=dev).permute(0, 2, 1, 3)
    elif not _bf16_view_ok(out):
        raise RuntimeError("out must have stride(-1)=1, 16-byte strides and alignment")
    if return_lse and lse is None:
        lse = torch.empty((B, H, Sq), dtype=torch.float32, device=dev)
    ms = list(block_mask.stride())
    if block_mask.shape[0] == 1:
        ms[0] = 0
    mstr = (_lib.ctypes.c_int64 * 4)(*ms)
    scale = -1.0 if softmax_scale is None else float(softmax_scale)
    lib = _lib.load()
    with torch.cuda.device(dev):
        rc = lib.sa_bsattn_fwd(
            q.data_ptr(), k.data_ptr(), v.data_ptr(),
            _lib.strides4(q), _lib.strides4(k), _lib.strides4(v),
            B, H, Sq, Sk, D,
            block_mask.data_ptr(), mstr, Hm,
            _ptr(head_mask_type), scale,
            out.data_ptr(), _lib.strides4(out),
            _ptr(lse) if return_lse else None,
            DeviceStatus.pointer(dev),
            _stream(dev),
        )
    _lib.check(rc, "sa_bsattn_fwd")
    return out, (lse if return_lse else None)


def sink_dynamic_attn(
    q: torch.Tensor,
    k: torch.Tensor,
    v: torch.Tensor,
    block_mask: torch.Tensor,
    k_pool: torch.Tensor,
    v_pool: torch.Tensor,
    sample_gap: int,
    softmax_scale: Optional[float] = None,
    head_mask_type: Optional[torch.Tensor] = None,
    return_lse: bool = False,
    out: Optional[torch.Tensor] = None,
):
    """Sink attention over the kept blocks of `block_mask` fused with dense
    attention over pooled keys/values (logits raised by ln(sample_gap)): the
    adaptive mix of the Wan runtime in one kernel. Shapes as bsattn_fwd;
    k_pool/v_pool [B,H,Sk_pool,D] bf16. Returns (out, lse or None)."""
    dev = _require_cuda(q, k, v, block_mask, k_pool, v_pool, head_mask_type)
    for t in (q, k, v, k_pool, v_pool):
        if t.dtype != torch.bfloat16 or t.dim() != 4:
            raise RuntimeError("sink_dynamic_attn expects 4-D bf16 tensors")
    B, H, Sq, D = q.shape
    Sk, Skp = k.shape[2], k_pool.shape[2]
    if k_pool.shape != (B, H, Skp, D) or v_pool.shape != (B, H, Skp, D):
        raise RuntimeError("k_pool / v_pool must be [B,H,Sk_pool,D]")
    nq, nk = math.ceil(Sq / BLOCK), math.ceil(Sk / BLOCK)
    if block_mask.dim() != 4 or block_mask.shape[-2:] != (nq, nk) or block_mask.shape[0] not in (1, B):
        raise RuntimeError(f"block_mask must be [B|1, Hm, {nq}, {nk}], got {tuple(block_mask.shape)}")
    if head_mask_type is not None:
        head_mask_type = head_mask_type.to(torch.int32).contiguous()
    q, k, v = _as_kernel_layout(q), _as_kernel_layout(k), _as_kernel_layout(v)
    k_pool, v_pool = _as_kernel_layout(k_pool), _as_kernel_layout(v_pool)
    if out is None:
        out = torch.empty((B, Sq, H, D), dtype=q.dtype, device=dev).permute(0, 2, 1, 3)
    lse = torch.empty((B, H, Sq), dtype=torch.float32, device=dev) if return_lse else None
    ms = list(block_mask.stride())
    if block_mask.shape[0] == 1:
        ms[0] = 0
    mstr = (_lib.ctypes.c_int64 * 4)(*ms)
    lib = _lib.load()
    with torch.cuda.device(dev):
        rc = lib.sa_sink_dynamic_attn_fwd(
            q.data_ptr(), k.data_ptr(), v.data_ptr(),
            _lib.strides4(q), _lib.strides4(k), _lib.strides4(v),
            B, H, Sq, Sk, D, block_mask.data_ptr(), mstr, block_mask.shape[1],
            _ptr(head_mask_type), k_pool.data_ptr(), v_pool.data_ptr(),
            _lib.strides4(k_pool), _lib.strides4(v_pool), Skp,
            math.log(float(max(1, int(sample_gap)))),
            -1.0 if softmax_scale is None else float(softmax_scale),
            out.data_ptr(), _lib.strides4(out), _ptr(lse),
            DeviceStatus.pointer(dev), _stream(dev),
        )
    _lib.check(rc, "sa_sink_dynamic_attn_fwd")
    return out, lse


def pool_scores_workspace_size(B: int, H: int, S: int, D: int, block: int = BLOCK) -> int:
    return int(_lib.load().sa_pool_scores_workspace_size(B, H, S, D, block))


def pool_scores_workspace(B: int, H: int, S: int, D: int, block: int = BLOCK,
                          device=None) -> torch.Tensor:
    """A workspace for pool_scores and calibration_layer (no clearing needed:
    the kernels' work counters carry a per-launch tag)."""
    need = pool_scores_workspace_size(B, H, S, D, block)
    return torch.empty(need, dtype=torch.uint8, device=device)


def _fused_calibration_ok(q: torch.Tensor, block: int) -> bool:
    B, H, S, D = q.shape
    return D == BLOCK and block == BLOCK and math.ceil(S / BLOCK) <= 256 and H <= 128


def pool_scores(
    q: torch.Tensor,
    k: torch.Tensor,
    block: int = BLOCK,
    scale: Optional[float] = None,
    want_scores: bool = True,
    want_batch_mean: bool = False,
    workspace: Optional[torch.Tensor] = None,
):
    """Mean-pooled block scores softmax(pool(q) pool(k)^T * scale).

    q, k: bf16 [B,H,S,D] (any strides with stride(-1)=1). Returns
    (scores fp32 [B,H,nb,nb] or None, batch_mean fp32 [H,nb,nb] or None).
    A given `workspace` (see pool_scores_workspace) may hold anything; calls
    sharing one must not overlap on the GPU.
    """
    dev = _require_cuda(q, k)
    if q.dtype != torch.bfloat16 or k.dtype != torch.bfloat16:
        raise RuntimeError("pool_scores expects bf16 q/k")
    if q.shape != k.shape or q.dim() != 4:
        raise RuntimeError("pool_scores expects q, k of equal shape [B,H,S,D]")
    B, H, S, D = q.shape
    nb = math.ceil(S / block)
    q, k = _as_kernel_layout(q), _as_kernel_layout(k)
    need = pool_scores_workspace_size(B, H, S, D, block)
    if workspace is None or workspace.numel() * workspace.element_size() < need:
        workspace = pool_scores_workspace(B, H, S, D, block, device=dev)
    scores = torch.empty((B, H, nb, nb), dtype=torch.float32, device=dev) if want_scores else None
    bmean = torch.empty((H, nb, nb), dtype=torch.float32, device=dev) if want_batch_mean else None
    sc = -1.0 if scale is None else float(scale)
    lib = _lib.load()
    with torch.cuda.device(dev):
        rc = lib.sa_pool_scores(
            q.data_ptr(), k.data_ptr(), _lib.strides4(q), _lib.strides4(k),
            B, H, S, D, block, sc, _ptr(scores), _ptr(bmean),
            workspace.data_ptr(), workspace.numel() * workspace.element_size(), _stream(dev),
        )
    _lib.check(rc, "sa_pool_scores")
    return scores, bmean


def pool_means(q: torch.Tensor, k: torch.Tensor, block: int = BLOCK,
               qp: Optional[torch.Tensor] = None, kp: Optional[torch.Tensor] = None):
    """Block means of bf16 q, k [B,H,S,D] -> fp32 [B,H,nb,D] each (first half
    of pool_scores)."""
    dev = _require_cuda(q, k)
    if q.dtype != torch.bfloat16 or k.dtype != torch.bfloat16 or q.shape != k.shape:
        raise RuntimeError("pool_means expects bf16 q, k of equal shape [B,H,S,D]")
    B, H, S, D = q.shape
    nb = math.ceil(S / block)
    q, k = _as_kernel_layout(q), _as_kernel_layout(k)
    if qp is None:
        qp = torch.empty((B, H, nb, D), dtype=torch.float32, device=dev)
    if kp is None:
        kp = torch.empty((B, H, nb, D), dtype=torch.float32, device=dev)
    lib = _lib.load()
    with torch.cuda.device(dev):
        rc = lib.sa_pool_means(q.data_ptr(), k.data_ptr(), _lib.strides4(q), _lib.strides4(k),
                               B, H, S, D, block, qp.data_ptr(), kp.data_ptr(), _stream(dev))
    _lib.check(rc, "sa_pool_means")
    return qp, kp


def pooled_softmax(qp: torch.Tensor, kp: torch.Tensor, scale: Optional[float] = None,
                   want_scores: bool = True, want_batch_mean: bool = False,
                   logits_ws: Optional[torch.Tensor] = None,
                   batch_mean_out: Optional[torch.Tensor] = None):
    """softmax(qp kp^T * scale) per batch from fp32 block means [B,H,nb,D]
    (second half of pool_scores). Returns (scores or None, batch_mean or None)."""
    dev = _require_cuda(qp, kp)
    B, H, nb, D = qp.shape
    if logits_ws is None or logits_ws.numel() < B * H * nb * nb:
        logits_ws = torch.empty(B * H * nb * nb, dtype=torch.float32, device=dev)
    scores = torch.empty((B, H, nb, nb), dtype=torch.float32, device=dev) if want_scores else None
    bmean = batch_mean_out
    if want_batch_mean and bmean is None:
        bmean = torch.empty((H, nb, nb), dtype=torch.float32, device=dev)
    sc = -1.0 if scale is None else float(scale)
    lib = _lib.load()
    with torch.cuda.device(dev):
        rc = lib.sa_pooled_softmax(qp.data_ptr(), kp.data_ptr(), B, H, nb, D, sc, _ptr(scores),
                                   _ptr(bmean) if want_batch_mean else None, logits_ws.data_ptr(),
                                   _stream(dev))
    _lib.check(rc, "sa_pooled_softmax")
    return scores, (bmean if want_batch_mean else None)


_STATS_MODES = {"exact": _lib.SA_STATS_EXACT, "max": _lib.SA_STATS_MAX}


def block_stats(q: torch.Tensor, k: torch.Tensor, mode: str = "exact",
                scale: Optional[float] = None, workspace: Optional[torch.Tensor] = None,
                out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """Block statistics of the full q k^T on the tensor cores, fp32 [B,H,nb,nb].

    mode "exact": mean over each query block's rows of the softmax mass each
    key block receives (the reference's exact pooling mode).
    mode "max": the block-maximum statistics of the reference's Triton
    pooling kernel, row-normalised with its bf16 rounding.
    q, k: bf16 [B,H,S,128] of equal shape (any strides with stride(-1)=1).
    """
    dev = _require_cuda(q, k)
    if mode not in _STATS_MODES:
        raise ValueError(f"block_stats mode must be one of {sorted(_STATS_MODES)}, got {mode!r}")
    if q.dtype != torch.bfloat16 or k.dtype != torch.bfloat16:
        raise RuntimeError("block_stats expects bf16 q/k")
    if q.shape != k.shape or q.dim() != 4:
        raise RuntimeError("block_stats expects q, k of equal shape [B,H,S,D]")
    B, H, S, D = q.shape
    nb = math.ceil(S / BLOCK)
    q, k = _as_kernel_layout(q), _as_kernel_layout(k)
    m = _STATS_MODES[mode]
    lib = _lib.load()
    need = int(lib.sa_block_stats_workspace_size(B, H, S, m))
    if need and (workspace is None or workspace.numel() * workspace.element_size() < need):
        workspace = torch.empty(need, dtype=torch.uint8, device=dev)
    if out is None:
        out = torch.empty((B, H, nb, nb), dtype=torch.float32, device=dev)
    sc = -1.0 if scale is None else float(scale)
    ws_bytes = 0 if not need else workspace.numel() * workspace.element_size()
    with torch.cuda.device(dev):
        rc = lib.sa_block_stats(q.data_ptr(), k.data_ptr(), _lib.strides4(q), _lib.strides4(k),
                                B, H, S, D, m, sc, out.data_ptr(),
                                workspace.data_ptr() if need else None, ws_bytes,
                                DeviceStatus.pointer(dev), _stream(dev))
    _lib.check(rc, "sa_block_stats")
    return out


def calibration_layer(
    q: torch.Tensor,
    k: torch.Tensor,
    scale: Optional[float] = None,
    want_scores: bool = False,
    want_batch_mean: bool = True,
    accumulate: Optional[tuple] = None,
    want_mask: bool = False,
    want_flags: bool = False,
    coverage: float = 0.85,
    keep_diagonal: bool = True,
    text_blocks: int = 0,
    mode: str = "joint",
    force_sink_col: bool = False,
    workspace: Optional[torch.Tensor] = None,
    scores_out: Optional[torch.Tensor] = None,
    batch_mean_out: Optional[torch.Tensor] = None,
    mask_out: Optional[torch.Tensor] = None,
    flags_out: Optional[torch.Tensor] = None,
) -> dict:
    """One calibration layer of the `mean` score mode in one launch
    (sa_calibration_layer): block means of q, k -> pooled logits -> softmax
    per batch element -> batch mean [-> running sums] [-> coverage mask].

    q, k: bf16 [B,H,S,128] (S <= 32768). accumulate: (sum, sumsq, first)
    with contiguous fp32 [H,nb,nb] accumulators. Returns a dict with the
    requested "scores" [B,H,nb,nb], "batch_mean" [H,nb,nb], "mask" bool
    [H,nb,nb] and "flags" int32 [H,nb]. The coverage mask uses row totals
    summed on the device (fp64, rounded); rows whose decision lies within
    2 ulp of the target carry SA_ROW_NEAR_TARGET in the flags."""
    dev = _require_cuda(q, k)
    if q.dtype != torch.bfloat16 or k.dtype != torch.bfloat16 or q.shape != k.shape or q.dim() != 4:
        raise RuntimeError("calibration_layer expects bf16 q, k of one shape [B,H,S,128]")
    B, H, S, D = q.shape
    nb = math.ceil(S / BLOCK)
    q, k = _as_kernel_layout(q), _as_kernel_layout(k)
    need = int(_lib.load().sa_calibration_layer_workspace_size(B, H, S))
    if workspace is None or workspace.numel() * workspace.element_size() < need:
        workspace = pool_scores_workspace(B, H, S, D, BLOCK, device=dev)
    out: dict = {}
    if want_scores or scores_out is not None:
        out["scores"] = scores_out if scores_out is not None else torch.empty(
            (B, H, nb, nb), dtype=torch.float32, device=dev)
    if want_batch_mean or batch_mean_out is not None:
        out["batch_mean"] = batch_mean_out if batch_mean_out is not None else torch.empty(
            (H, nb, nb), dtype=torch.float32, device=dev)
    if want_mask or mask_out is not None:
        out["mask"] = mask_out if mask_out is not None else torch.empty(
            (H, nb, nb), dtype=torch.bool, device=dev)
        if want_flags or flags_out is not None:
            out["flags"] = flags_out if flags_out is not None else torch.empty(
                (H, nb), dtype=torch.int32, device=dev)
    for name, t, dt in (("scores", out.get("scores"), torch.float32),
                        ("batch_mean", out.get("batch_mean"), torch.float32),
                        ("mask", out.get("mask"), torch.bool),
                        ("flags", out.get("flags"), torch.int32)):
        if t is not None and (t.dtype != dt or not t.is_contiguous() or t.device != dev):
            raise RuntimeError(f"calibration_layer: {name} must be contiguous {dt} on {dev}")
    acc_sum = acc_sumsq = None
    first = 0
    if accumulate is not None:
        acc_sum, acc_sumsq, first = accumulate
        for t in (acc_sum, acc_sumsq):
            if t.shape != (H, nb, nb) or t.dtype != torch.float32 or not t.is_contiguous():
                raise RuntimeError("calibration_layer: accumulators must be contiguous fp32 "
                                   f"[{H}, {nb}, {nb}]")
    mode_id = (_lib.SA_COVERAGE_VIDEO_RESIDUAL
               if str(mode).strip().lower() in {"video_residual", "video_residual_only",
                                                "residual_video"}
               else _lib.SA_COVERAGE_JOINT)
    lib = _lib.load()
    with torch.cuda.device(dev):
        rc = lib.sa_calibration_layer(
            q.data_ptr(), k.data_ptr(), _lib.strides4(q), _lib.strides4(k), B, H, S, D,
            -1.0 if scale is None else float(scale), _ptr(out.get("scores")),
            _ptr(out.get("batch_mean")), _ptr(acc_sum), _ptr(acc_sumsq), int(bool(first)),
            _ptr(out.get("mask")), _ptr(out.get("flags")), mode_id, float(coverage),
            int(bool(keep_diagonal)), int(text_blocks), int(bool(force_sink_col)),
            workspace.data_ptr(), workspace.numel() * workspace.element_size(),
            DeviceStatus.pointer(dev), _stream(dev))
    _lib.check(rc, "sa_calibration_layer")
    return out


_PASS_STREAMS: dict[int, tuple] = {}


def pooled_softmax_layers(qp: torch.Tensor, kp: torch.Tensor, scale: Optional[float] = None,
                          batch_means_out: Optional[torch.Tensor] = None,
                          logits_ws: Optional[torch.Tensor] = None) -> torch.Tensor:
    """Per-layer batch means of softmax(qp kp^T * scale) for L stacked layers:
    qp, kp fp32 [L,B,H,nb,D] contiguous -> fp32 [L,H,nb,nb]."""
    dev = _require_cuda(qp, kp)
    L, B, H, nb, D = qp.shape
    if kp.shape != qp.shape or not (qp.is_contiguous() and kp.is_contiguous()):
        raise RuntimeError("pooled_softmax_layers expects contiguous qp, kp of one shape")
    need = L * B * H * nb * nb
    if logits_ws is None or logits_ws.numel() < need:
        logits_ws = torch.empty(need, dtype=torch.float32, device=dev)
    out = batch_means_out
    if out is None:
        out = torch.empty((L, H, nb, nb), dtype=torch.float32, device=dev)
    sc = -1.0 if scale is None else float(scale)
    lib = _lib.load()
    with torch.cuda.device(dev):
        rc = lib.sa_pooled_softmax_layers(qp.data_ptr(), kp.data_ptr(), L, B, H, nb, D, sc,
                                          out.data_ptr(), logits_ws.data_ptr(), _stream(dev))
    _lib.check(rc, "sa_pooled_softmax_layers")
    return out


def calibration_pass(
    layers,
    block: int = BLOCK,
    coverage: float = 0.85,
    keep_diagonal: bool = True,
    text_blocks: int = 0,
    mode: str = "joint",
    force_sink_col: bool = False,
    want_batch_mean: bool = False,
    masks_out: Optional[torch.Tensor] = None,
    chunk: int = 3,
    head_groups: int = 1,
    want_flags: bool = False,
    workspace: Optional[torch.Tensor] = None,
    fused: Optional[bool] = None,
):
    """Pooling + pooled softmax + batch mean + coverage mask for a sequence of
    layers, each given as a (q, k) pair of bf16 [B,H,S,D] CUDA tensors.

    Several layers run a pipeline over layers (below), which overlaps each
    chunk's scores and masks with the next chunk's pooling; one layer at the
    calibration shapes (D = 128, block 128, at most 256 blocks) is one fused
    launch (sa_calibration_layer), whose score and mask work overlaps its own
    pooling. `fused` forces either choice (fused=True needs those shapes);
    with it, `chunk` and `head_groups` have no effect. The two agree to within
    one ulp on the batch means. The coverage masks use row totals summed on
    the device (fp64, rounded); with want_flags the SA_ROW_* flags of every
    row are returned too.

    The pipeline: the work goes in units of
    (layer, group of H/head_groups heads) and the
    units in chunks of `chunk`: every unit of a chunk is pooled back to back
    on one side stream (HBM-bound, one persistent TMA kernel per unit), then
    the chunk's pooled softmax and batch means (two launches for the whole
    chunk) and its coverage masks (one launch) run on a second side stream
    while the next chunk pools. head_groups > 1 lets a single layer overlap
    its own pooling with its scores and masks. The result is ordered on the
    caller's current stream. Returns (masks bool [L,H,nb,nb], batch means fp32
    [L,H,nb,nb] or None), plus flags int32 [L,H,nb] with want_flags."""
    layers = list(layers)
    if not layers:
        raise ValueError("calibration_pass needs at least one layer")
    q0, _ = layers[0]
    dev = _require_cuda(q0)
    B, H, S, D = q0.shape
    nb = math.ceil(S / block)
    L = len(layers)
    flags = torch.empty((L, H, nb), dtype=torch.int32, device=dev) if want_flags else None
    if fused is None:
        fused = L == 1 and _fused_calibration_ok(q0, block)
    elif fused and not _fused_calibration_ok(q0, block):
        raise ValueError("the fused calibration layer needs D = 128, block 128 and S <= 32768")
    if fused:
        masks = masks_out if masks_out is not None else torch.empty(
            (L, H, nb, nb), dtype=torch.bool, device=dev)
        bmeans = torch.empty((L, H, nb, nb), dtype=torch.float32, device=dev) \
            if want_batch_mean else None
        need = int(_lib.load().sa_calibration_layer_workspace_size(B, H, S))
        if workspace is None or workspace.numel() * workspace.element_size() < need:
            workspace = pool_scores_workspace(B, H, S, D, block, device=dev)
        for l, (q, k) in enumerate(layers):
            if q.shape != (B, H, S, D) or k.shape != (B, H, S, D):
                raise ValueError("all layers must share one [B,H,S,D] shape")
            calibration_layer(q, k, want_batch_mean=False,
                              batch_mean_out=None if bmeans is None else bmeans[l],
                              mask_out=masks[l], flags_out=None if flags is None else flags[l],
                              coverage=coverage, keep_diagonal=keep_diagonal,
                              text_blocks=text_blocks, mode=mode, force_sink_col=force_sink_col,
                              workspace=workspace)
        return (masks, bmeans, flags) if want_flags else (masks, bmeans)
    G = max(1, int(head_groups))
    if H % G:
        raise ValueError(f"head_groups ({G}) must divide the {H} heads")
    hg = H // G
    U = L * G  # units (layer, head group), in layer-major order
    C = max(1, min(int(chunk), U))
    idx = dev.index if dev.index is not None else torch.cuda.current_device()
    if idx not in _PASS_STREAMS:
        _PASS_STREAMS[idx] = (torch.cuda.Stream(dev), torch.cuda.Stream(dev))
    sp, sc = _PASS_STREAMS[idx]
    cur = torch.cuda.current_stream(dev)
    masks = masks_out if masks_out is not None else torch.empty(
        (L, H, nb, nb), dtype=torch.bool, device=dev)
    bmeans = torch.empty((L, H, nb, nb), dtype=torch.float32, device=dev) if want_batch_mean \
        else torch.empty((2, C, hg, nb, nb), dtype=torch.float32, device=dev)
    qp = torch.empty((2, C, B, hg, nb, D), dtype=torch.float32, device=dev)
    kp = torch.empty((2, C, B, hg, nb, D), dtype=torch.float32, device=dev)
    logits = torch.empty(C * B * hg * nb * nb, dtype=torch.float32, device=dev)
    pooled = [torch.cuda.Event() for _ in range(2)]
    consumed = [torch.cuda.Event() for _ in range(2)]
    # unit u covers rows [u*hg, (u+1)*hg) of the flattened [L*H] head rows
    mask_rows = masks.view(L * H, nb, nb)
    sp.wait_stream(cur)
    sc.wait_stream(cur)
    for ci, u0 in enumerate(range(0, U, C)):
        u1 = min(U, u0 + C)
        n = u1 - u0
        buf = ci % 2
        with torch.cuda.stream(sp):
            if ci >= 2:
                sp.wait_event(consumed[buf])
            for u in range(u0, u1):
                l, g = divmod(u, G)
                q, k = layers[l]
                if q.shape != (B, H, S, D) or k.shape != (B, H, S, D):
                    raise ValueError("all layers must share one [B,H,S,D] shape")
                hs = slice(g * hg, (g + 1) * hg)
                pool_means(q[:, hs], k[:, hs], block, qp=qp[buf, u - u0], kp=kp[buf, u - u0])
            pooled[buf].record(sp)
        with torch.cuda.stream(sc):
            sc.wait_event(pooled[buf])
            bm = (bmeans.view(L * H, nb, nb)[u0 * hg:u1 * hg].view(n, hg, nb, nb)
                  if want_batch_mean else bmeans[buf, :n])
            pooled_softmax_layers(qp[buf, :n], kp[buf, :n], batch_means_out=bm, logits_ws=logits)
            consumed[buf].record(sc)
            _, f = coverage_mask(bm.reshape(n * hg, nb, nb), coverage=coverage,
                                 keep_diagonal=keep_diagonal, text_blocks=text_blocks, mode=mode,
                                 force_sink_col=force_sink_col, out=mask_rows[u0 * hg:u1 * hg],
                                 want_flags=want_flags)
            if flags is not None:
                flags.view(L * H, nb)[u0 * hg:u1 * hg].copy_(f)
    cur.wait_stream(sp)
    cur.wait_stream(sc)
    for t in (qp, kp, logits, bmeans, masks):
        t.record_stream(sp)
        t.record_stream(sc)
    for q, k in layers:
        q.record_stream(sp)
        k.record_stream(sp)
    if flags is not None:
        flags.record_stream(sc)
        return masks, (bmeans if want_batch_mean else None), flags
    return masks, (bmeans if want_batch_mean else None)


def coverage_mask(
    scores: torch.Tensor,
    coverage: float = 0.85,
    keep_diagonal: bool = True,
    text_blocks: int = 0,
    mode: str = "joint",
    force_sink_col: bool = False,
    row_total: Optional[torch.Tensor] = None,
    row_selected: Optional[torch.Tensor] = None,
    want_flags: bool = False,
    out: Optional[torch.Tensor] = None,
):
    """Per-row minimal-coverage block mask from fp32 scores [H,nq,nk] (CUDA).

    Returns (mask bool [H,nq,nk], flags int32 [H,nq] or None). `out`, when
    given, is a contiguous bool [H,nq,nk] tensor the mask is written into."""
    dev = _require_cuda(scores, row_total, row_selected)
    if scores.dim() != 3:
        raise ValueError(f"Expected [heads, blocks_q, blocks_k] scores, got {tuple(scores.shape)}")
    if scores.dtype != torch.float32:
        scores = scores.float()
    if scores.stride(-1) != 1:
        scores = scores.contiguous()
    H, nq, nk = scores.shape
    mode_id = (_lib.SA_COVERAGE_VIDEO_RESIDUAL
               if str(mode).strip().lower() in {"video_residual", "video_residual_only", "residual_video"}
               else _lib.SA_COVERAGE_JOINT)
    for name, t in (("row_total", row_total), ("row_selected", row_selected)):
        if t is not None and (t.shape != (H, nq) or t.dtype != torch.float32):
            raise ValueError(f"{name} must be fp32 [H, nq]")
    row_total = None if row_total is None else row_total.contiguous()
    row_selected = None if row_selected is None else row_selected.contiguous()
    if out is not None:
        if out.shape != (H, nq, nk) or out.dtype != torch.bool or not out.is_contiguous():
            raise ValueError("out must be a contiguous bool [H, nq, nk] tensor")
        mask = out
    else:
        mask = torch.empty((H, nq, nk), dtype=torch.bool, device=dev)
    flags = torch.empty((H, nq), dtype=torch.int32, device=dev) if want_flags else None
    lib = _lib.load()
    with torch.cuda.device(dev):
        rc = lib.sa_coverage_mask(
            scores.data_ptr(), _lib.strides3(scores), H, nq, nk, mode_id, float(coverage),
            int(bool(keep_diagonal)), int(text_blocks), int(bool(force_sink_col)),
            _ptr(row_total), _ptr(row_selected), mask.data_ptr(), _ptr(flags), _stream(dev),
        )
    _lib.check(rc, "sa_coverage_mask")
    return mask, flags


def score_accumulate(x: torch.Tensor, sum_: torch.Tensor, sumsq: torch.Tensor, first: bool) -> None:
    dev = _require_cuda(x, sum_, sumsq)
    for t in (x, sum_, sumsq):
        if t.dtype != torch.float32 or not t.is_contiguous():
            raise RuntimeError("score_accumulate expects contiguous fp32 tensors")
    if x.numel() != sum_.numel() or x.numel() != sumsq.numel():
        raise RuntimeError("score_accumulate: size mismatch")
    lib = _lib.load()
    with torch.cuda.device(dev):
        rc = lib.sa_score_accumulate(x.data_ptr(), x.numel(), sum_.data_ptr(), sumsq.data_ptr(),
                                     int(bool(first)), _stream(dev))
    _lib.check(rc, "sa_score_accumulate")


def score_finalize(sum_: torch.Tensor, sumsq: torch.Tensor, count,
                   variance: bool = False) -> tuple[torch.Tensor, torch.Tensor]:
    """(mean, std) of running sums over `count` samples (a number or a per-
    element tensor); with variance=True the second result is the clamped
    variance instead of its square root."""
    dev = _require_cuda(sum_, sumsq)
    mean = torch.empty_like(sum_)
    std = torch.empty_like(sum_)
    cnt_t = count if isinstance(count, torch.Tensor) else None
    if cnt_t is not None:
        cnt_t = cnt_t.to(device=dev, dtype=torch.float32).contiguous()
    lib = _lib.load()
    with torch.cuda.device(dev):
        rc = lib.sa_score_finalize(sum_.data_ptr(), sumsq.data_ptr(), _ptr(cnt_t),
                                   float(count) if cnt_t is None else 0.0, sum_.numel(),
                                   mean.data_ptr(), std.data_ptr(), int(variance), _stream(dev))
    _lib.check(rc, "sa_score_finalize")
    return mean, std


def score_accumulate_aligned(scores: torch.Tensor, image_blocks: int, text_blocks: int,
                             total_blocks: int, sum_: torch.Tensor, sumsq: torch.Tensor,
                             presence: torch.Tensor, first: bool) -> None:
    """Place one sample's fp32 scores [H, n, n] (n = image + text blocks) into
    the fixed [H, T, T] layout and accumulate sum, sum of squares and presence
    there (the Z-Image calibrator's alignment)."""
    dev = _require_cuda(scores, sum_, sumsq, presence)
    if scores.dtype != torch.float32 or scores.dim() != 3 or scores.shape[1] != scores.shape[2]:
        raise ValueError(f"Expected [heads, blocks_q, blocks_k] scores, got {tuple(scores.shape)}")
    H, n = scores.shape[0], scores.shape[1]
    for t in (sum_, sumsq, presence):
        if t.shape != (H, total_blocks, total_blocks) or t.dtype != torch.float32 \
                or not t.is_contiguous():
            raise RuntimeError("aligned accumulators must be contiguous fp32 [H, T, T]")
    scores = scores.contiguous()
    lib = _lib.load()
    with torch.cuda.device(dev):
        rc = lib.sa_score_accumulate_aligned(scores.data_ptr(), H, n, int(image_blocks),
                                             int(text_blocks), int(total_blocks), sum_.data_ptr(),
                                             sumsq.data_ptr(), presence.data_ptr(), int(first),
                                             _stream(dev))
    if rc == _lib.SA_EINVAL and "Z-Image block score shape" in lib.sa_last_error().decode():
        raise ValueError(lib.sa_last_error().decode())
    _lib.check(rc, "sa_score_accumulate_aligned")


def score_finalize_presence(sum_: torch.Tensor, sumsq: torch.Tensor, presence: torch.Tensor,
                            variance: bool = False) -> tuple[torch.Tensor, torch.Tensor]:
    """Presence-weighted mean/std (or clamped variance with variance=True);
    presence is clamped to >= 1 in place."""
    dev = _require_cuda(sum_, sumsq, presence)
    if not (sum_.is_contiguous() and sumsq.is_contiguous() and presence.is_contiguous()):
        raise RuntimeError("score_finalize_presence expects contiguous tensors")
    mean = torch.empty_like(sum_)
    std = torch.empty_like(sum_)
    lib = _lib.load()
    with torch.cuda.device(dev):
        rc = lib.sa_score_finalize_presence(sum_.data_ptr(), sumsq.data_ptr(), presence.data_ptr(),
                                            sum_.numel(), mean.data_ptr(), std.data_ptr(),
                                            int(variance), _stream(dev))
    _lib.check(rc, "sa_score_finalize_presence")
    return mean, std


def qk_norm_rope(q: torch.Tensor, k: torch.Tensor, head_dim: int, eps: float,
                 w_q: Optional[torch.Tensor] = None, w_k: Optional[torch.Tensor] = None,
                 cos: Optional[torch.Tensor] = None, sin: Optional[torch.Tensor] = None,
                 out_q: Optional[torch.Tensor] = None, out_k: Optional[torch.Tensor] = None):
    """RMSNorm over the hidden dimension + rotary embedding for Q and K.

    q, k: bf16 [B, S, hidden] (the projections' outputs, stride(-1) = 1);
    w_q, w_k: [hidden] bf16 or fp32 (or None); cos, sin: fp32 [S, head_dim/2]
    (or None: no rotation). Returns (q, k) bf16 [B, S, hidden]; out_q/out_k
    may alias q/k (in place).
    """
    dev = _require_cuda(q, k, w_q, w_k, cos, sin)
    if q.dtype != torch.bfloat16 or k.dtype != torch.bfloat16 or q.dim() != 3 or q.shape != k.shape:
        raise RuntimeError("qk_norm_rope expects bf16 q, k of one shape [B, S, hidden]")
    B, S, hidden = q.shape

    def rows_view(t):
        if t.stride(-1) != 1 or t.stride(0) != S * t.stride(1):
            t = t.contiguous()
        return t

    q, k = rows_view(q), rows_view(k)
    if out_q is None:
        out_q = torch.empty((B, S, hidden), dtype=torch.bfloat16, device=dev)
    if out_k is None:
        out_k = torch.empty((B, S, hidden), dtype=torch.bfloat16, device=dev)
    for o in (out_q, out_k):
        if o.shape != (B, S, hidden) or o.dtype != torch.bfloat16 or o.stride(-1) != 1 \
                or o.stride(0) != S * o.stride(1):
            raise RuntimeError("qk_norm_rope outputs must be bf16 [B, S, hidden] with uniform rows")
    w_bf16 = 1
    if w_q is not None:
        if w_q.dtype == torch.bfloat16 and w_k.dtype == torch.bfloat16:
            w_q, w_k = w_q.contiguous(), w_k.contiguous()
        else:
            w_q, w_k = w_q.float().contiguous(), w_k.float().contiguous()
            w_bf16 = 0
        if w_q.numel() != hidden or w_k.numel() != hidden:
            raise RuntimeError(f"norm weights must have {hidden} elements")
    fs = 0
    if cos is not None:
        cos, sin = cos.float().contiguous(), sin.float().contiguous()
        if cos.shape != (S, head_dim // 2) or sin.shape != (S, head_dim // 2):
            raise ValueError(f"Rotary frequency shape mismatch: expected {(S, head_dim // 2)}, "
                             f"got {tuple(cos.shape)}")
        fs = cos.stride(0)
    lib = _lib.load()
    with torch.cuda.device(dev):
        rc = lib.sa_qk_norm_rope(q.data_ptr(), k.data_ptr(), q.stride(1), k.stride(1), B * S, S,
                                 hidden, int(head_dim), _ptr(w_q), _ptr(w_k), w_bf16, float(eps),
                                 _ptr(cos), _ptr(sin), fs, out_q.data_ptr(), out_k.data_ptr(),
                                 out_q.stride(1), out_k.stride(1), _stream(dev))
    _lib.check(rc, "sa_qk_norm_rope")
    return out_q, out_k


def mean_pool_seq(x: torch.Tensor, pool: int, prefix: int = 0) -> torch.Tensor:
    """_mean_pool_sequence_preserve_prefix on a bf16 [B,H,S,D] view."""
    dev = _require_cuda(x)
    if x.dtype != torch.bfloat16:
        raise RuntimeError("mean_pool_seq expects bf16")
    B, H, S, D = x.shape
    if pool <= 1:
        return x
    prefix = min(max(int(prefix), 0), S)
    if prefix >= S:
        return x
    out_rows = prefix + math.ceil((S - prefix) / pool)
    x = _as_kernel_layout(x)
    out = torch.empty((B, out_rows, H, D), dtype=x.dtype, device=dev).permute(0, 2, 1, 3)
    lib = _lib.load()
    with torch.cuda.device(dev):
        rc = lib.sa_mean_pool_seq(x.data_ptr(), _lib.strides4(x), B, H, S, D, int(pool), prefix,
                                  out.data_ptr(), _lib.strides4(out), _stream(dev))
    _lib.check(rc, "sa_mean_pool_seq")
    return out


def mix_outputs(sink_out, sink_lse, dyn_out, dyn_lse, sample_gap: int) -> torch.Tensor:
    """Adaptive LSE mix; lse tensors fp32 [B,H,S] (natural log)."""
    dev = _require_cuda(sink_out, sink_lse, dyn_out, dyn_lse)
    B, H, S, D = sink_out.shape
    sink_out, dyn_out = _as_kernel_layout(sink_out), _as_kernel_layout(dyn_out)
    sink_lse = sink_lse.reshape(B, H, S).float().contiguous()
    dyn_lse = dyn_lse.reshape(B, H, S).float().contiguous()
    out = torch.empty((B, S, H, D), dtype=sink_out.dtype, device=dev).permute(0, 2, 1, 3)
    lib = _lib.load()
    with torch.cuda.device(dev):
        rc = lib.sa_mix_outputs(sink_out.data_ptr(), _lib.strides4(sink_out), sink_lse.data_ptr(),
                                dyn_out.data_ptr(), _lib.strides4(dyn_out), dyn_lse.data_ptr(),
                                B, H, S, D, math.log(float(max(1, int(sample_gap)))),
                                out.data_ptr(), _lib.strides4(out), _stream(dev))
    _lib.check(rc, "sa_mix_outputs")
    return out

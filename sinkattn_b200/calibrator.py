"""Device-resident sink-mask calibrators.

Same interfaces and package format as the reference's SinkMaskCalibrator
(sinkattention/sparse_attention.py:526-608) and ZImageSinkMaskCalibrator
(zimg/runtime/sink_sparse_zimage.py:248-366): record(layer, q, k, v) per
self-attention call, then build_package() / save(). The difference is where
the statistics live: the reference takes every layer's scores to the host
(`.mean(dim=0).cpu()`, sparse_attention.py:581, sink_sparse_zimage.py:303)
and accumulates there; here the block scores, the Z-Image alignment and the
running sums stay on the GPU (sa_pool_scores / sa_block_stats,
sa_score_accumulate(_aligned)), and only the final mean/std/mask leave it.

The mean is sum / count in fp32 on the device, the same operations in the
same order as the reference's CPU accumulation; the std's square root is
taken on the host copy of the variance with torch.sqrt, the reference's own
CPU op; and masks are built by the drop-in _build_direct_mean_coverage_mask
on the host copy of the mean. All three equal the reference's bit for bit.
"""
from __future__ import annotations

from dataclasses import asdict
from pathlib import Path
from typing import Dict, Optional

import torch

from . import ops
from .reference_api import _build_direct_mean_coverage_mask, _compute_block_scores


class DeviceSinkMaskCalibrator:
    def __init__(self, config, device: Optional[torch.device] = None):
        self.config = config
        self.device = device
        self.current_step = -1
        self.score_sums: Dict[int, torch.Tensor] = {}
        self.score_sq_sums: Dict[int, torch.Tensor] = {}
        self.score_counts: Dict[int, int] = {}
        self._workspace: Optional[torch.Tensor] = None

    def reset_generation(self) -> None:
        self.current_step = -1

    @torch.no_grad()
    def record(self, layer_idx: int, q: torch.Tensor, k: torch.Tensor, v: torch.Tensor) -> None:
        """SinkMaskCalibrator.record (sparse_attention.py:575-582) on the device.

        The score mode is dispatched as _compute_block_scores does
        (sparse_attention.py:230-238): "exact" -> block masses of the full
        softmax, "triton" (the SinkSparseConfig default, compared
        case-sensitively as line 124 does) -> the Triton kernel's block maxima,
        "mean" (and a "triton" in another case, which line 124 sends to the
        torch path) -> the mean-pooled rule. The batch mean (line 580) stays on
        the device: torch's mean for the tensor-core statistics, as the
        reference takes it; the mean-pooled kernel forms it in its own epilogue.
        """
        if layer_idx == 0:
            self.current_step += 1
        mode = str(self.config.pooling_mode).strip().lower()
        if mode not in {"exact", "triton", "mean"}:
            raise ValueError(
                f"Unsupported pooling_mode: {self.config.pooling_mode}. Expected one of: "
                "exact, triton, mean.")
        ops._require_cuda(q, k)
        if mode == "exact" or self.config.pooling_mode == "triton":
            scores = _compute_block_scores(q, k, v, self.config)
            self._accumulate_score(layer_idx, scores.float().mean(dim=0))
            return
        B, H, S, D = q.shape
        block = int(self.config.block_size)
        need = ops.pool_scores_workspace_size(B, H, S, D, block)
        if self._workspace is None or self._workspace.numel() < need or \
                self._workspace.device != q.device:
            self._workspace = ops.pool_scores_workspace(B, H, S, D, block, device=q.device)
        qb = q if q.dtype == torch.bfloat16 else q.to(torch.bfloat16)
        kb = k if k.dtype == torch.bfloat16 else k.to(torch.bfloat16)
        if ops._fused_calibration_ok(qb, block):
            # one launch: scores, batch mean and the running sums
            first = layer_idx not in self.score_sums
            if first:
                nb = -(-S // block)
                self.score_sums[layer_idx] = torch.empty((H, nb, nb), dtype=torch.float32,
                                                         device=q.device)
                self.score_sq_sums[layer_idx] = torch.empty_like(self.score_sums[layer_idx])
                self.score_counts[layer_idx] = 0
            ops.calibration_layer(qb, kb, want_batch_mean=False,
                                  accumulate=(self.score_sums[layer_idx],
                                              self.score_sq_sums[layer_idx], first),
                                  workspace=self._workspace)
            self.score_counts[layer_idx] += 1
            return
        _, bmean = ops.pool_scores(qb, kb, block=block, want_scores=False,
                                   want_batch_mean=True, workspace=self._workspace)
        self._accumulate_score(layer_idx, bmean)

    def _accumulate_score(self, layer_idx: int, scores: torch.Tensor) -> None:
        """_accumulate_score (sparse_attention.py:537-549): adds one record's
        batch-mean scores [H, nq, nk] (fp32, on the GPU) to the layer's running
        sum and sum of squares, which stay on the GPU."""
        first = layer_idx not in self.score_sums
        if first:
            self.score_sums[layer_idx] = torch.empty_like(scores)
            self.score_sq_sums[layer_idx] = torch.empty_like(scores)
            self.score_counts[layer_idx] = 0
        ops.score_accumulate(scores, self.score_sums[layer_idx], self.score_sq_sums[layer_idx],
                             first=first)
        self.score_counts[layer_idx] += 1

    def _build_mean_and_masks(self, config=None):
        """_build_mean_and_masks (sparse_attention.py:551-573). Raises
        RuntimeError if any kernel that fed the statistics reported a bounded
        wait that gave up."""
        config = self.config if config is None else config
        for t in self.score_sums.values():
            ops.DeviceStatus.check(t.device)
            break
        mean_scores, std_scores, sink_masks, counts = {}, {}, {}, {}
        for layer_idx in sorted(self.score_sums.keys()):
            key = str(layer_idx)
            mean, var = ops.score_finalize(self.score_sums[layer_idx],
                                           self.score_sq_sums[layer_idx],
                                           self.score_counts[layer_idx], variance=True)
            mean_cpu = mean.cpu()
            mean_scores[key] = mean_cpu
            # the root with the reference's own CPU op (not correctly rounded
            # in every case), so the exported std carries the reference's bits
            std_scores[key] = torch.sqrt(var.cpu())
            sink_masks[key] = _build_direct_mean_coverage_mask(mean_cpu, config)
            counts[key] = int(self.score_counts[layer_idx])
        return mean_scores, std_scores, sink_masks, counts

    def build_package(self, include_scores: bool = True, config_override=None) -> dict:
        """build_package (sparse_attention.py:584-596): package format version 3."""
        export_config = self.config if config_override is None else config_override
        mean_scores, std_scores, sink_masks, counts = self._build_mean_and_masks(export_config)
        return {
            "version": 3,
            "config": asdict(export_config),
            "mean_scores": mean_scores if include_scores else {},
            "std_scores": std_scores if include_scores else {},
            "sink_masks": sink_masks,
            "counts": counts,
            "meta": {"route": "wanx_direct_coverage"},
        }

    def save(self, output_path: str, include_scores: bool = True, config_override=None) -> dict:
        package = self.build_package(include_scores=include_scores,
                                     config_override=config_override)
        out = Path(output_path)
        out.parent.mkdir(parents=True, exist_ok=True)
        torch.save(package, out)
        return package


def _pad_to_multiple(value: int, multiple: int = 32) -> int:
    return -(-int(value) // multiple) * multiple


def _zimg_config(config):
    """build_zimg_sink_config (zimg/runtime/sink_sparse_zimage.py:54-81) when the
    reference's Z-Image runtime is importable; otherwise the config as given,
    which must then already be a Z-Image config."""
    try:
        from zimg.runtime.sink_sparse_zimage import build_zimg_sink_config
    except ImportError:
        return config
    return build_zimg_sink_config(package_config=asdict(config))


class DeviceZImageSinkMaskCalibrator:
    """ZImageSinkMaskCalibrator with its statistics on the GPU.

    Every sample's scores [H, n, n] (n = image blocks + this sample's text
    blocks) are aligned into the fixed [H, T, T] layout, image blocks first and
    text blocks at the end, and accumulated with a presence count
    (sa_score_accumulate_aligned); the mean is presence-weighted
    (sa_score_finalize_presence). The fixed layout follows
    _fixed_block_shape: image tokens and the maximum text length are padded
    to multiples of 32 tokens (sink_sparse_zimage.py:30-35, 123-136)."""

    def __init__(self, config):
        self.config = _zimg_config(config)
        self.current_step = -1
        self.score_sums: Dict[int, torch.Tensor] = {}
        self.score_sq_sums: Dict[int, torch.Tensor] = {}
        self.score_presence_sums: Dict[int, torch.Tensor] = {}
        self.score_counts: Dict[int, int] = {}
        bs = int(self.config.block_size)
        self.image_token_count = _pad_to_multiple(
            int(self.config.token_width) * int(self.config.token_height)
            * int(self.config.token_depth))
        self.image_blocks = -(-self.image_token_count // bs)
        self.max_text_tokens = _pad_to_multiple(int(self.config.text_length))
        self.total_blocks = self.image_blocks + -(-self.max_text_tokens // bs)

    def reset_generation(self) -> None:
        self.current_step = -1

    @torch.no_grad()
    def record(self, layer_idx: int, q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, *,
               text_token_count: int) -> None:
        """ZImageSinkMaskCalibrator.record (sink_sparse_zimage.py:281-319)."""
        if layer_idx == 0:
            self.current_step += 1
        if text_token_count < 0:
            raise ValueError(f"Invalid Z-Image text token count: {text_token_count}")
        if text_token_count > self.max_text_tokens:
            raise ValueError(
                "Observed Z-Image text token count exceeds calibrated maximum. "
                f"Observed {text_token_count}, configured max {self.max_text_tokens}.")
        if q.size(0) != 1:
            raise ValueError("Z-Image calibration expects one sample at a time after "
                             "valid-token slicing.")
        scores = _compute_block_scores(q, k, v, self.config).detach().float()[0]
        current_text_blocks = -(-int(text_token_count) // int(self.config.block_size))
        first = layer_idx not in self.score_sums
        if first:
            shape = (scores.size(0), self.total_blocks, self.total_blocks)
            self.score_sums[layer_idx] = torch.empty(shape, dtype=torch.float32, device=q.device)
            self.score_sq_sums[layer_idx] = torch.empty_like(self.score_sums[layer_idx])
            self.score_presence_sums[layer_idx] = torch.empty_like(self.score_sums[layer_idx])
            self.score_counts[layer_idx] = 0
        ops.score_accumulate_aligned(scores, self.image_blocks, current_text_blocks,
                                     self.total_blocks, self.score_sums[layer_idx],
                                     self.score_sq_sums[layer_idx],
                                     self.score_presence_sums[layer_idx], first=first)
        self.score_counts[layer_idx] += 1

    @torch.no_grad()
    def build_package(self, include_scores: bool = True, config_override=None) -> dict:
        """build_package (sink_sparse_zimage.py:321-354): presence-weighted
        statistics, masks from the mean, package format version 3."""
        export_config = self.config if config_override is None else _zimg_config(config_override)
        for t in self.score_sums.values():
            ops.DeviceStatus.check(t.device)
            break
        mean_scores, std_scores, sink_masks, counts = {}, {}, {}, {}
        for layer_idx in sorted(self.score_sums.keys()):
            key = str(layer_idx)
            mean, var = ops.score_finalize_presence(self.score_sums[layer_idx],
                                                    self.score_sq_sums[layer_idx],
                                                    self.score_presence_sums[layer_idx],
                                                    variance=True)
            mean_cpu = mean.cpu()
            mean_scores[key] = mean_cpu
            std_scores[key] = torch.sqrt(var.cpu())
            sink_masks[key] = _build_direct_mean_coverage_mask(mean_cpu, export_config)
            counts[key] = int(self.score_counts[layer_idx])
        return {
            "version": 3,
            "config": asdict(export_config),
            "mean_scores": mean_scores if include_scores else {},
            "std_scores": std_scores if include_scores else {},
            "sink_masks": sink_masks,
            "counts": counts,
            "meta": {
                "route": "zimg_static_only",
                "text_layout": "image_prefix_text_suffix_aligned",
                "image_token_count": self.image_token_count,
                "max_text_token_count": self.max_text_tokens,
                "total_blocks": self.total_blocks,
            },
        }

    def save(self, output_path: str, include_scores: bool = True, config_override=None) -> dict:
        package = self.build_package(include_scores=include_scores,
                                     config_override=config_override)
        out = Path(output_path)
        out.parent.mkdir(parents=True, exist_ok=True)
        torch.save(package, out)
        return package

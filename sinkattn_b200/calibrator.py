"""Device-resident sink-mask calibrator.

Same interface and package format as the reference's SinkMaskCalibrator
(sinkattention/sparse_attention.py:526-608): record(layer, q, k, v) per
self-attention call, then build_package() / save(). The difference is where
the statistics live: the reference takes every layer's batch-mean scores to
the host (`.mean(dim=0).cpu()`, line 581) and accumulates sum and
sum-of-squares there; here the pooled scores, their batch mean and both
running sums stay on the GPU (sa_pool_scores + sa_score_accumulate), and only
the final mean/std/mask leave it.

The mean is sum / count in fp32 on the device, the same operations in the
same order as the reference's CPU accumulation, and masks are built by the
drop-in _build_direct_mean_coverage_mask on the host copy of the mean, so
they equal the reference's builder bit for bit.
"""
from __future__ import annotations

from dataclasses import asdict
from pathlib import Path
from typing import Dict, Optional

import torch

from . import ops
from .reference_api import _build_direct_mean_coverage_mask


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
        """SinkMaskCalibrator.record (sparse_attention.py:575-582) on the device."""
        if layer_idx == 0:
            self.current_step += 1
        mode = str(self.config.pooling_mode).strip().lower()
        if mode not in {"mean", "triton"}:
            raise NotImplementedError(
                f"DeviceSinkMaskCalibrator supports pooling_mode mean/triton, got {mode}")
        B, H, S, D = q.shape
        need = ops.pool_scores_workspace_size(B, H, S, D, int(self.config.block_size))
        if self._workspace is None or self._workspace.numel() < need or \
                self._workspace.device != q.device:
            self._workspace = torch.empty(need, dtype=torch.uint8, device=q.device)
        qb = q if q.dtype == torch.bfloat16 else q.to(torch.bfloat16)
        kb = k if k.dtype == torch.bfloat16 else k.to(torch.bfloat16)
        _, bmean = ops.pool_scores(qb, kb, block=int(self.config.block_size), want_scores=False,
                                   want_batch_mean=True, workspace=self._workspace)
        first = layer_idx not in self.score_sums
        if first:
            self.score_sums[layer_idx] = torch.empty_like(bmean)
            self.score_sq_sums[layer_idx] = torch.empty_like(bmean)
            self.score_counts[layer_idx] = 0
        ops.score_accumulate(bmean, self.score_sums[layer_idx], self.score_sq_sums[layer_idx],
                             first=first)
        self.score_counts[layer_idx] += 1

    def _build_mean_and_masks(self, config=None):
        """_build_mean_and_masks (sparse_attention.py:551-573)."""
        config = self.config if config is None else config
        mean_scores, std_scores, sink_masks, counts = {}, {}, {}, {}
        for layer_idx in sorted(self.score_sums.keys()):
            key = str(layer_idx)
            mean, std = ops.score_finalize(self.score_sums[layer_idx],
                                           self.score_sq_sums[layer_idx],
                                           self.score_counts[layer_idx])
            mean_cpu = mean.cpu()
            mean_scores[key] = mean_cpu
            std_scores[key] = std.cpu()
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

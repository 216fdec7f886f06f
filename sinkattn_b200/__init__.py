"""sinkattn_b200 — B200 (sm_100a) kernels for SinkAttention's hot path.

Two paths of the reference (bb-2020-bb/sinkattn) run here as hand-written
CUDA behind a C ABI (include/sinkattn.h, libsinkattn.so):

* block-sparse attention forward over kept 128x128 blocks (tcgen05 + TMEM +
  TMA), replacing the external block_sparse_attn_func;
* the calibration chain: mean pooling of Q/K, pooled-score softmax, batch
  mean / accumulation and the 0.85-coverage block-mask build.

``install()`` binds the drop-in functions of :mod:`sinkattn_b200.reference_api`
into the reference's modules; :mod:`sinkattn_b200.ops` is the tensor-level API.
"""
from . import ops
from ._lib import load as load_library
from .reference_api import (
    _block_sparse_attn,
    _build_direct_mean_coverage_mask,
    _compute_pooled_qk_block_scores,
    block_sparse_attn_func,
    install,
)

__all__ = [
    "ops",
    "load_library",
    "install",
    "block_sparse_attn_func",
    "_block_sparse_attn",
    "_compute_pooled_qk_block_scores",
    "_build_direct_mean_coverage_mask",
]

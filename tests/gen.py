"""Seeded synthetic inputs for the benchmark configurations.

The reference publishes no dataset for this path; these generators stand in
for real Wan / Z-Image activations with the shapes, sizes and value
distributions the benchmark configs state:

* cfg1: B=1, H=4, S=4096, D=128, Q/K/V ~ N(0,1) (torch CPU generator, seed 0);
  block mask [4,32,32] = column 0 | diagonal | Bernoulli(0.2) (seed 1).
* cfg2: Wan2.1 self-attention, B=2, H=12, D=128, S=32760 tokens (21x30x52)
  padded to 32768 (256 blocks). Q,K = N(0,1) + 0.5 * PE3D(t,h,w); V ~ N(0,1).
  Padding tokens (index >= 32760) carry noise only (PE = 0).
* cfg3: 30 layers of cfg2-style Q/K with seed = layer index.
* cfg4: Z-Image, B=1, H=30, 16384 image tokens (128x128) with 0.5 * PE2D plus
  512 text tokens (noise only): S = 16896 = 132 blocks.

PE3D splits the 128 channels into 42 (t) / 42 (h) / 44 (w); each group holds
sin then cos of position * 10000^(-2i/n) for i < n/2 (n = group width).
PE2D splits 64 (h) / 64 (w) the same way.
"""
from __future__ import annotations

import hashlib
import math

import numpy as np
import torch

WAN_T, WAN_H, WAN_W = 21, 30, 52
WAN_TOKENS = WAN_T * WAN_H * WAN_W  # 32760
WAN_S_PADDED = 32768
ZIMG_SIDE = 128
ZIMG_IMAGE_TOKENS = ZIMG_SIDE * ZIMG_SIDE  # 16384
ZIMG_TEXT_TOKENS = 512
ZIMG_S = ZIMG_IMAGE_TOKENS + ZIMG_TEXT_TOKENS  # 16896


def _sincos(pos: torch.Tensor, n: int) -> torch.Tensor:
    i = torch.arange(n // 2, dtype=torch.float64)
    freq = torch.pow(10000.0, -2.0 * i / n)
    ang = pos.to(torch.float64)[:, None] * freq[None, :]
    return torch.cat([torch.sin(ang), torch.cos(ang)], dim=1)


def pe3d(t: int = WAN_T, h: int = WAN_H, w: int = WAN_W, d: int = 128) -> torch.Tensor:
    """[t*h*w, d] float32, token order t-major then h then w."""
    assert d == 128
    tt, hh, ww = torch.meshgrid(torch.arange(t), torch.arange(h), torch.arange(w), indexing="ij")
    parts = [_sincos(tt.reshape(-1), 42), _sincos(hh.reshape(-1), 42), _sincos(ww.reshape(-1), 44)]
    return torch.cat(parts, dim=1).float()


def pe2d(h: int = ZIMG_SIDE, w: int = ZIMG_SIDE, d: int = 128) -> torch.Tensor:
    assert d == 128
    hh, ww = torch.meshgrid(torch.arange(h), torch.arange(w), indexing="ij")
    return torch.cat([_sincos(hh.reshape(-1), 64), _sincos(ww.reshape(-1), 64)], dim=1).float()


def randn(shape, seed: int, device="cpu", dtype=torch.float32) -> torch.Tensor:
    g = torch.Generator(device="cpu").manual_seed(int(seed))
    return torch.randn(*shape, generator=g, dtype=torch.float32).to(device=device, dtype=dtype)


def cfg1_mask(H: int = 4, nq: int = 32, nk: int = 32, seed: int = 1, p: float = 0.2) -> torch.Tensor:
    """Column 0 | diagonal | Bernoulli(p), bool [H, nq, nk]."""
    g = torch.Generator(device="cpu").manual_seed(int(seed))
    m = torch.rand(H, nq, nk, generator=g) < p
    m[:, :, 0] = True
    d = torch.arange(min(nq, nk))
    m[:, d, d] = True
    return m


def cfg1_inputs(device="cpu", dtype=torch.bfloat16, B=1, H=4, S=4096, D=128, seed=0):
    g = torch.Generator(device="cpu").manual_seed(int(seed))
    q = torch.randn(B, H, S, D, generator=g)
    k = torch.randn(B, H, S, D, generator=g)
    v = torch.randn(B, H, S, D, generator=g)
    nb = math.ceil(S / 128)
    mask = cfg1_mask(H, nb, nb, seed=1).unsqueeze(0)
    return (q.to(device=device, dtype=dtype), k.to(device=device, dtype=dtype),
            v.to(device=device, dtype=dtype), mask.to(device))


def wan_qk(seed: int = 0, B: int = 2, H: int = 12, S: int = WAN_S_PADDED, D: int = 128,
           amp: float = 0.5, device="cpu", dtype=torch.bfloat16, heads: slice | None = None):
    """cfg2 Q, K (and V) as [B,H,S,D]. PE is shared over batch and heads.
    Generated on the CPU with torch's generator, then moved to `device`."""
    g = torch.Generator(device="cpu").manual_seed(int(seed))
    pe = torch.zeros(S, D)
    n = min(S, WAN_TOKENS)
    pe[:n] = pe3d()[:n]
    q = torch.randn(B, H, S, D, generator=g)
    k = torch.randn(B, H, S, D, generator=g)
    v = torch.randn(B, H, S, D, generator=g)
    q += amp * pe
    k += amp * pe
    if heads is not None:
        q, k, v = q[:, heads], k[:, heads], v[:, heads]
    return (q.to(device=device, dtype=dtype), k.to(device=device, dtype=dtype),
            v.to(device=device, dtype=dtype))


def wan_qk_layers_on_device(n_layers: int, device, B: int = 2, H: int = 12,
                            S: int = WAN_S_PADDED, D: int = 128, amp: float = 0.5):
    """cfg3 timing inputs: Q, K per layer generated directly on the GPU with a
    CUDA generator seeded by the layer index (fast; a different random stream
    from the CPU generator used for the parity fixtures)."""
    pe = torch.zeros(S, D)
    n = min(S, WAN_TOKENS)
    pe[:n] = pe3d()[:n]
    pe = (amp * pe).to(device)
    out = []
    for layer in range(n_layers):
        g = torch.Generator(device=device).manual_seed(layer)
        q = torch.randn(B, H, S, D, generator=g, device=device).add_(pe).bfloat16()
        k = torch.randn(B, H, S, D, generator=g, device=device).add_(pe).bfloat16()
        out.append((q, k))
    return out


def zimg_qkv(seed: int = 0, H: int = 30, D: int = 128, amp: float = 0.5, device="cpu",
             dtype=torch.bfloat16):
    g = torch.Generator(device="cpu").manual_seed(int(seed))
    pe = torch.zeros(ZIMG_S, D)
    pe[:ZIMG_IMAGE_TOKENS] = pe2d()
    q = torch.randn(1, H, ZIMG_S, D, generator=g) + amp * pe
    k = torch.randn(1, H, ZIMG_S, D, generator=g) + amp * pe
    v = torch.randn(1, H, ZIMG_S, D, generator=g)
    return (q.to(device=device, dtype=dtype), k.to(device=device, dtype=dtype),
            v.to(device=device, dtype=dtype))


def digest(*arrays) -> str:
    """SHA-256 over the raw bytes of the given arrays/tensors (input pinning)."""
    h = hashlib.sha256()
    for a in arrays:
        if isinstance(a, torch.Tensor):
            a = a.detach().cpu()
            if a.dtype == torch.bfloat16:
                a = a.view(torch.int16)
            a = a.numpy()
        h.update(np.ascontiguousarray(a).tobytes())
    return h.hexdigest()


def config_from_json(text: str):
    """A dataclass instance carrying the fields and values of a stored
    SinkSparseConfig (JSON of its asdict()), for code that reads config
    attributes and calls asdict() on the config it was given."""
    import dataclasses
    import json

    data = json.loads(str(text))
    cls = dataclasses.make_dataclass("StoredSinkSparseConfig", list(data.keys()))
    return cls(**data)


# SinkSparseConfig() field defaults (sinkattention/sparse_attention.py:35-53),
# as asdict() gives them; tests/test_host_cpu.py checks this copy against the
# reference's dataclass when a reference checkout is importable.
REFERENCE_DEFAULT_CONFIG = {
    "block_size": 128, "sample_gap": 30, "token_width": 52, "token_height": 30,
    "token_depth": 21, "text_length": 0, "force_text_global_attention": False,
    "offline_text_video_coverage_mode": "joint", "keep_diagonal": True,
    "runtime_diagonal_band_width": 0, "pooling_mode": "triton", "dynamic_mode": "pooled_kv",
    "dynamic_kernel": "auto", "mixing_mode": "adaptive", "force_dense_steps": None,
    "force_dense_layers": None, "offline_direct_coverage": 0.85,
}


def default_config(**overrides):
    """A SinkSparseConfig stand-in with the reference's defaults (see
    REFERENCE_DEFAULT_CONFIG), fields overridden by keyword."""
    import json

    data = dict(REFERENCE_DEFAULT_CONFIG)
    data.update(overrides)
    return config_from_json(json.dumps(data))

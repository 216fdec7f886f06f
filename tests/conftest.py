"""Shared pytest set-up: the `gpu` marker, golden-vector access, oracle import."""
from __future__ import annotations

import os
import sys
from pathlib import Path

import numpy as np
import pytest
import torch

ROOT = Path(__file__).resolve().parent.parent
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))

from tests.gen import digest  # noqa: E402

GOLDEN = ROOT / "tests" / "golden" / "golden.npz"
CALIB_GOLDEN = ROOT / "tests" / "golden" / "calib.npz"


def _reference_dir() -> Path:
    """Where the reference's Python packages (sinkattention, wanx, zimg) are
    imported from by the tests that drive its own code: the directory named
    by the SINKATTN_REFERENCE environment variable, else the offline install
    under baseline/_ref. Tests that need it skip when it holds no package."""
    env = os.environ.get("SINKATTN_REFERENCE")
    return Path(env) if env else ROOT / "baseline" / "_ref"


REFERENCE_DIR = _reference_dir()


@pytest.fixture
def reference(monkeypatch):
    """Puts the reference's packages on sys.path for one test (skips when
    they are not available)."""
    if not (REFERENCE_DIR / "sinkattention").exists():
        pytest.skip(f"reference packages not found under {REFERENCE_DIR}")
    monkeypatch.syspath_prepend(str(REFERENCE_DIR))
    return REFERENCE_DIR


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA (B200) device")


def pytest_collection_modifyitems(config, items):
    if torch.cuda.is_available():
        return
    skip = pytest.mark.skip(reason="no CUDA device")
    for item in items:
        if "gpu" in item.keywords:
            item.add_marker(skip)


@pytest.fixture(scope="session")
def golden():
    return dict(np.load(GOLDEN, allow_pickle=False))


@pytest.fixture(scope="session")
def calib_golden():
    return dict(np.load(CALIB_GOLDEN, allow_pickle=False))


def regen_input(g: dict, case: str, key: str) -> torch.Tensor:
    """Regenerate a golden case's bf16 input from its seed and check the digest."""
    shape = tuple(int(x) for x in g[f"{case}/{key}_shape"])
    seed = int(g[f"{case}/{key}_seed"])
    gen = torch.Generator().manual_seed(seed)
    t = torch.randn(*shape, generator=gen).to(torch.bfloat16)
    want = str(g[f"{case}/{key}_sha256"])
    got = digest(t)
    assert got == want, (
        f"regenerated input {case}/{key} differs from the one the golden vectors were "
        f"made with (torch generator changed?): {got} != {want}")
    return t


def from_bits(a: np.ndarray) -> np.ndarray:
    return (a.astype(np.uint32) << 16).view(np.float32)


@pytest.fixture(scope="session")
def oracle():
    sys.path.insert(0, str(ROOT))
    from oracle import sinkattn_oracle

    return sinkattn_oracle


@pytest.fixture(scope="module")
def lib():
    """The C-ABI library (loading needs no GPU; entry points are only called
    with arguments they reject before any launch)."""
    from sinkattn_b200 import _lib

    return _lib.load()

"""CPU-only checks of the C-ABI boundary: the library loads, exports every
symbol include/sinkattn.h declares with the ctypes signature the header
gives, and rejects bad arguments on the host (before any CUDA call) with
SA_EINVAL and a message."""
from __future__ import annotations

import ctypes
import re
import subprocess
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent
HEADER = ROOT / "include" / "sinkattn.h"


def header_symbols() -> list[str]:
    text = HEADER.read_text()
    return sorted(set(re.findall(r"^SA_API\s+[\w\s\*]+?\b(sa_\w+)\s*\(", text, flags=re.M)))


def test_header_declares_symbols():
    syms = header_symbols()
    assert "sa_bsattn_fwd" in syms and "sa_coverage_mask" in syms and "sa_pool_scores" in syms


def test_library_exports_every_declared_symbol(lib):
    from sinkattn_b200 import _lib

    out = subprocess.run(["nm", "-D", "--defined-only", str(_lib.LIB_PATH)], capture_output=True,
                         text=True, check=True).stdout
    exported = {ln.split()[-1] for ln in out.splitlines() if " T " in ln}
    missing = [s for s in header_symbols() if s not in exported]
    assert not missing, f"declared but not exported: {missing}"
    for s in header_symbols():
        assert hasattr(lib, s)
    # the Python binding covers the same set
    assert sorted(_lib.exported_names()) == header_symbols()


def test_version(lib):
    assert lib.sa_version() == 1


def _i64(*v):
    return (ctypes.c_int64 * len(v))(*v)


def test_bsattn_rejects_bad_head_dim(lib):
    from sinkattn_b200 import _lib

    st = _i64(64 * 4 * 64, 64 * 64, 64, 1)
    rc = lib.sa_bsattn_fwd(16, 16, 16, st, st, st, 1, 4, 64, 64, 64, 16, _i64(0, 1, 1, 1), 4,
                           None, -1.0, 16, st, None, None, None)
    assert rc == _lib.SA_EINVAL
    assert "head dim must be 128" in _lib.last_error()


def test_bsattn_rejects_misaligned_stride(lib):
    from sinkattn_b200 import _lib

    st = _i64(128 * 3 * 100, 128, 3 * 128 + 4, 1)
    rc = lib.sa_bsattn_fwd(16, 16, 16, st, st, st, 1, 3, 100, 100, 128, 16, _i64(0, 1, 1, 1), 3,
                           None, -1.0, 16, st, None, None, None)
    assert rc == _lib.SA_EINVAL
    assert "stride" in _lib.last_error()


def test_bsattn_rejects_empty_and_null(lib):
    from sinkattn_b200 import _lib

    st = _i64(128 * 128, 128 * 128, 128, 1)
    rc = lib.sa_bsattn_fwd(16, 16, 16, st, st, st, 1, 1, 0, 128, 128, 16, _i64(0, 1, 1, 1), 1,
                           None, -1.0, 16, st, None, None, None)
    assert rc == _lib.SA_EINVAL
    rc = lib.sa_bsattn_fwd(None, 16, 16, st, st, st, 1, 1, 128, 128, 128, 16, _i64(0, 1, 1, 1), 1,
                           None, -1.0, 16, st, None, None, None)
    assert rc == _lib.SA_EINVAL and "null" in _lib.last_error()


def test_bsattn_rejects_mask_head_mismatch(lib):
    from sinkattn_b200 import _lib

    st = _i64(128 * 4 * 128, 128 * 128, 128, 1)
    rc = lib.sa_bsattn_fwd(16, 16, 16, st, st, st, 1, 4, 128, 128, 128, 16, _i64(0, 1, 1, 1), 2,
                           None, -1.0, 16, st, None, None, None)
    assert rc == _lib.SA_EINVAL and "head_mask_type" in _lib.last_error()


def test_pool_scores_workspace_and_validation(lib):
    from sinkattn_b200 import _lib

    B, H, S, D = 2, 12, 32768, 128
    nb = 256
    # work counters (one 128-byte line each, H + 5 of them, rounded to 256),
    # group flags (8 bytes per 16 block rows of each head, rounded to 256),
    # then pooled Q, K and logits in fp32 (sa_pool_scores) or pooled Q, K and
    # a batch-mean scratch (the fused calibration layer)
    ctr, flags = 2304, 1536  # 17 * 128 -> 2304; 12 heads * 16 groups * 8
    assert lib.sa_pool_scores_workspace_size(B, H, S, D, 128) == \
        ctr + flags + 4 * B * H * nb * (2 * D + nb)
    assert lib.sa_calibration_layer_workspace_size(B, H, S) == \
        ctr + flags + 4 * B * H * nb * 2 * D + 4 * H * nb * nb
    # 106 counter lines = 13568; 101 heads x 1 group x 8 bytes = 808 -> 1024
    assert lib.sa_calibration_layer_workspace_size(1, 101, 128) == \
        13568 + 1024 + 4 * 101 * 2 * 128 + 4 * 101
    assert lib.sa_pool_scores_workspace_size(0, H, S, D, 128) == 0
    st = _i64(H * S * D, S * D, D, 1)
    rc = lib.sa_pool_scores(16, 16, st, st, B, H, S, D, 128, -1.0, 16, None, 16, 8, None)
    assert rc == _lib.SA_EINVAL and "workspace" in _lib.last_error()
    rc = lib.sa_pool_scores(16, 16, st, st, B, H, S, D, 128, -1.0, None, None, 16, 1 << 40, None)
    assert rc == _lib.SA_EINVAL and "both NULL" in _lib.last_error()
    rc = lib.sa_pool_scores(16, 16, st, st, B, H, S, 100, 128, -1.0, 16, None, 16, 1 << 40, None)
    assert rc == _lib.SA_EINVAL


def test_calibration_layer_validation(lib):
    """sa_calibration_layer rejects what it cannot run before any launch."""
    from sinkattn_b200 import _lib

    B, H, S = 2, 12, 32768
    st = _i64(H * S * 128, S * 128, 128, 1)
    ws = 1 << 40

    def call(*, D=128, S=S, scores=16, acc=(None, None), mask=None, flags=None, mode=0,
             cov=0.85, text=0, ws_bytes=ws, strides=st, q=256):
        return lib.sa_calibration_layer(q, 256, strides, strides, B, H, S, D, -1.0, scores, None,
                                        acc[0], acc[1], 0, mask, flags, mode, cov, 1, text, 0,
                                        256, ws_bytes, None, None)

    assert call(D=64) == _lib.SA_EINVAL and "D must be 128" in _lib.last_error()
    assert call(S=32769) == _lib.SA_EINVAL and "256 blocks" in _lib.last_error()
    assert call(scores=None) == _lib.SA_EINVAL and "no output" in _lib.last_error()
    assert call(acc=(16, None)) == _lib.SA_EINVAL and "go together" in _lib.last_error()
    assert call(flags=16) == _lib.SA_EINVAL and "needs mask_out" in _lib.last_error()
    assert call(mode=5) == _lib.SA_EINVAL and "mode" in _lib.last_error()
    assert call(cov=float("nan")) == _lib.SA_EINVAL and "NaN" in _lib.last_error()
    assert call(text=-1) == _lib.SA_EINVAL
    assert call(strides=_i64(H * S * 128, S * 128, 100, 1)) == _lib.SA_EINVAL
    assert call(q=264) == _lib.SA_EINVAL and "aligned" in _lib.last_error()
    assert call(ws_bytes=1024) == _lib.SA_EINVAL and "workspace" in _lib.last_error()


def test_coverage_mask_validation(lib):
    from sinkattn_b200 import _lib

    st = (ctypes.c_int64 * 3)(5000 * 4, 5000, 1)
    rc = lib.sa_coverage_mask(16, st, 1, 4, 5000, 0, 0.85, 1, 0, 0, None, None, 16, None, None)
    assert rc == _lib.SA_EINVAL and "4096" in _lib.last_error()
    st = (ctypes.c_int64 * 3)(64, 8, 2)
    rc = lib.sa_coverage_mask(16, st, 1, 8, 8, 0, 0.85, 1, 0, 0, None, None, 16, None, None)
    assert rc == _lib.SA_EINVAL and "stride" in _lib.last_error()
    st = (ctypes.c_int64 * 3)(64, 8, 1)
    rc = lib.sa_coverage_mask(16, st, 1, 8, 8, 7, 0.85, 1, 0, 0, None, None, 16, None, None)
    assert rc == _lib.SA_EINVAL and "mode" in _lib.last_error()


def test_misc_validation(lib):
    from sinkattn_b200 import _lib

    assert lib.sa_score_accumulate(None, 4, 16, 16, 1, None) == _lib.SA_EINVAL
    assert lib.sa_score_finalize(16, None, None, 0.0, 4, 16, None, 0, None) == _lib.SA_EINVAL
    assert lib.sa_score_finalize_presence(16, 16, None, 4, 16, None, 0, None) == _lib.SA_EINVAL
    assert lib.sa_score_accumulate_aligned(16, 2, 5, 4, 2, 6, 16, 16, 16, 1, None) == _lib.SA_EINVAL
    st = _i64(8 * 8, 8 * 8, 8, 1)
    assert lib.sa_mean_pool_seq(16, st, 1, 1, 8, 12, 2, 0, 16, st, None) == _lib.SA_EINVAL


def test_ops_reject_cpu_tensors():
    """No CPU fallback: the tensor API refuses CPU tensors."""
    import torch

    from sinkattn_b200 import ops

    q = torch.zeros(1, 1, 128, 128, dtype=torch.bfloat16)
    m = torch.ones(1, 1, 1, 1, dtype=torch.bool)
    with pytest.raises(RuntimeError, match="CUDA"):
        ops.bsattn_fwd(q, q, q, m)
    with pytest.raises(RuntimeError, match="CUDA"):
        ops.pool_scores(q, q)
    with pytest.raises(RuntimeError, match="CUDA"):
        ops.coverage_mask(torch.rand(1, 4, 4))


def test_install_binds_dropins_into_reference(reference):
    """With the reference's packages importable, install() rebinds its hot-path
    names (including the fused Wan inner forward); the rebound functions
    refuse CPU tensors (no CPU fallback)."""
    import sys

    import torch

    import sinkattention.sparse_attention as sa
    import wanx.runtime.sink_sparse_wan as wan

    from sinkattn_b200 import reference_api as ra

    orig_forward = wan.WanSinkSparseInnerAttention.forward
    orig_prepare = wan._prepare_attention_tensors
    orig = {n: getattr(sa, n) for n in ("block_sparse_attn_func", "_block_sparse_attn",
                                        "_compute_pooled_qk_block_scores",
                                        "_build_direct_mean_coverage_mask")}
    try:
        patched = ra.install()
        assert "sinkattention.sparse_attention" in patched
        assert sa.block_sparse_attn_func is ra.block_sparse_attn_func
        assert sa._HAS_BLOCK_SPARSE is True
        assert wan._block_sparse_attn is ra._block_sparse_attn
        assert wan.WanSinkSparseInnerAttention.forward is ra.fused_wan_inner_forward
        cfg = sa.SinkSparseConfig().merged({"dynamic_mode": "pooled_kv", "dynamic_kernel": "block_sparse",
                                            "sample_gap": 30, "runtime_diagonal_band_width": 1})
        inner = wan.WanSinkSparseInnerAttention(0, torch.ones(2, 2, 2, dtype=torch.bool), cfg)
        x = torch.zeros(1, 2, 256, 128, dtype=torch.bfloat16)
        with pytest.raises(RuntimeError, match="CUDA"):
            inner(x, x, x)
        # the fused Q/K producer is bound, and hands CPU inputs to the
        # reference's own _prepare_attention_tensors unchanged
        assert wan._prepare_attention_tensors is ra.fused_prepare_attention_tensors
        assert ra._UNFUSED_PREPARE[0] is orig_prepare

        class Attn(torch.nn.Module):
            def __init__(self):
                super().__init__()
                self.heads = 2
                self.add_k_proj = None
                self.to_q = torch.nn.Linear(256, 256, dtype=torch.bfloat16)
                self.to_k = torch.nn.Linear(256, 256, dtype=torch.bfloat16)
                self.to_v = torch.nn.Linear(256, 256, dtype=torch.bfloat16)
                self.norm_q = torch.nn.RMSNorm(256, eps=1e-6, dtype=torch.bfloat16)
                self.norm_k = torch.nn.RMSNorm(256, eps=1e-6, dtype=torch.bfloat16)

        attn = Attn()
        hs = torch.randn(1, 8, 256).bfloat16()
        ang = torch.outer(torch.arange(8.0), torch.linspace(0.0, 1.0, 64))
        freqs = torch.polar(torch.ones_like(ang), ang)[None, None]
        with torch.no_grad():
            got = wan._prepare_attention_tensors(attn, hs, None, freqs)
            want = orig_prepare(attn, hs, None, freqs)
        for a, b in zip(got[:3], want[:3]):
            assert torch.equal(a, b)
    finally:
        wan._prepare_attention_tensors = orig_prepare
        wan.WanSinkSparseInnerAttention.forward = orig_forward
        for n, f in orig.items():
            setattr(sa, n, f)
        sa._HAS_BLOCK_SPARSE = orig["block_sparse_attn_func"] is not None
        for m in [m for m in list(sys.modules) if m.startswith(("wanx", "zimg", "sinkattention"))]:
            sys.modules.pop(m, None)


def header_signatures() -> dict[str, tuple[str, list[str]]]:
    """name -> (return type, parameter declarations) of every SA_API function."""
    text = HEADER.read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    text = re.sub(r"//[^\n]*", "", text)
    sigs = {}
    for m in re.finditer(r"^SA_API\s+([\w\s\*]+?)\b(sa_\w+)\s*\(([^)]*)\)\s*;", text, flags=re.M):
        params = " ".join(m.group(3).split())
        sigs[m.group(2)] = (m.group(1).strip(),
                            [] if params in ("", "void") else [p.strip() for p in params.split(",")])
    return sigs


# uint64_t and size_t are one ctypes type on LP64 (c_ulong)
_C_KINDS = {"int": "i32", "int32_t": "i32", "int64_t": "i64", "uint64_t": "size",
            "size_t": "size", "float": "f32"}


def _c_kind(decl: str, is_return: bool = False) -> str:
    decl = re.sub(r"\bconst\b", " ", decl)
    if "*" in decl or "[" in decl or "cudaStream_t" in decl:
        return "ptr"
    toks = decl.split()
    return _C_KINDS[toks[0] if is_return or len(toks) == 1 else " ".join(toks[:-1])]


def _ctypes_kind(t) -> str:
    return {ctypes.c_void_p: "ptr", ctypes.c_char_p: "ptr", ctypes.c_int: "i32",
            ctypes.c_int64: "i64", ctypes.c_size_t: "size", ctypes.c_float: "f32"}[t]


def test_ctypes_signatures_match_the_header():
    """Every entry point's ctypes declaration has the header's parameter count
    and kinds (pointer, int, int64, size_t, float) in order, so a call can
    never pass a misread argument to the library."""
    from sinkattn_b200 import _lib

    sigs = header_signatures()
    assert set(sigs) == set(header_symbols())
    assert set(sigs) == set(_lib._SIGNATURES), set(sigs) ^ set(_lib._SIGNATURES)
    for name, (ret, params) in sigs.items():
        res, args = _lib._SIGNATURES[name]
        assert _ctypes_kind(res) == _c_kind(ret, is_return=True), name
        want = [_c_kind(p) for p in params]
        got = [_ctypes_kind(a) for a in args]
        assert got == want, f"{name}: ctypes {got} != header {want}"


def test_install_skips_absent_routes_unless_named(monkeypatch):
    """A route whose module cannot be imported is skipped by install(), and
    raises when the caller asked for it by name."""
    from sinkattn_b200 import reference_api as ra

    monkeypatch.setattr(ra, "_PATCHES", {"sinkattn_absent_route.runtime": {"x": 1}})
    assert ra.install() == []
    with pytest.raises(ImportError):
        ra.install(modules=["sinkattn_absent_route.runtime"])


def test_status_word_check_and_selftest_validation(lib):
    """sa_check_status reads any host int32: a non-zero code is reported as
    SA_ETIMEOUT with a message and the word is reset; the self-test refuses a
    limit outside [1 us, 1 s] before it launches anything."""
    from sinkattn_b200 import _lib

    word = ctypes.c_int32(0)
    assert lib.sa_check_status(ctypes.addressof(word)) == _lib.SA_OK
    word.value = 1  # SA_DEV_WAIT_TIMEOUT, as a kernel writes it
    assert lib.sa_check_status(ctypes.addressof(word)) == _lib.SA_ETIMEOUT
    assert "bounded wait" in _lib.last_error()
    assert word.value == 0
    assert lib.sa_check_status(ctypes.addressof(word)) == _lib.SA_OK
    assert lib.sa_check_status(None) == _lib.SA_EINVAL
    assert lib.sa_status_destroy(None) == _lib.SA_OK
    assert lib.sa_selftest_wait_timeout(ctypes.addressof(word), 10, None) == _lib.SA_EINVAL
    assert "limit" in _lib.last_error()
    assert lib.sa_selftest_wait_timeout(ctypes.addressof(word), 2 * 10**9, None) == _lib.SA_EINVAL
    assert lib.sa_selftest_wait_timeout(None, 10**6, None) == _lib.SA_EINVAL


def test_ulysses_exchange_validation(lib):
    """The exchange entry points refuse what they cannot run before any
    launch."""
    from sinkattn_b200 import _lib

    st = _i64(*([4 * 3 * 128, 3 * 128, 128, 1] * 3))
    src = (ctypes.c_void_p * 3)(256, 256, 256)
    dst = (ctypes.c_void_p * 9)(*([512] * 9))

    def dispatch(T=3, D=128, P=2, rank=0, n_per=3, B=2, H=3):
        return lib.sa_ulysses_dispatch(T, src, st, B, 4, H, D, P, rank, n_per, dst, None)

    assert dispatch(D=64) == _lib.SA_EINVAL and "128" in _lib.last_error()
    assert dispatch(P=9) == _lib.SA_EINVAL and "ranks" in _lib.last_error()
    assert dispatch(rank=2) == _lib.SA_EINVAL and "rank" in _lib.last_error()
    assert dispatch(T=4) == _lib.SA_EINVAL and "tensors" in _lib.last_error()
    assert dispatch(n_per=2) == _lib.SA_EINVAL and "units" in _lib.last_error()
    bad = _i64(*([4 * 3 * 128, 3 * 128, 100, 1] * 3))
    assert lib.sa_ulysses_dispatch(3, src, bad, 2, 4, 3, 128, 2, 0, 3, dst, None) == _lib.SA_EINVAL
    assert lib.sa_ulysses_combine(256, None, 2, 4, 3, 128, 2, 0, 3, dst, dst, None) == \
        _lib.SA_EINVAL and "together" in _lib.last_error()
    assert lib.sa_ulysses_combine(256, None, 2, 4, 3, 128, 2, 5, 3, dst, None, None) == \
        _lib.SA_EINVAL
    for j0, j1 in ((2, 2), (0, 4), (-1, 1), (3, 2)):
        assert lib.sa_ulysses_dispatch_units(3, src, st, 2, 4, 3, 128, 2, 0, 3, j0, j1, dst,
                                             None) == _lib.SA_EINVAL
        assert "slots" in _lib.last_error()
        assert lib.sa_ulysses_combine_units(256, None, 2, 4, 3, 128, 2, 0, 3, j0, j1, dst, None,
                                            None) == _lib.SA_EINVAL
        assert "slots" in _lib.last_error()
    ptr = ctypes.c_void_p()
    assert lib.sa_ipc_alloc(0, ctypes.byref(ptr)) == _lib.SA_EINVAL
    assert lib.sa_ipc_get_handle(None, None) == _lib.SA_EINVAL
    assert lib.sa_ipc_free(None) == _lib.SA_OK and lib.sa_ipc_close(None) == _lib.SA_OK

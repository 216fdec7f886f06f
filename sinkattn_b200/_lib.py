"""ctypes binding of libsinkattn.so (the C ABI declared in include/sinkattn.h).

The library is loaded from this package directory. There is no fallback: if
the shared object is missing or a call fails, a RuntimeError is raised with
the library's own message.
"""
from __future__ import annotations

import ctypes
import os
import threading
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "libsinkattn.so"

SA_OK = 0
SA_EINVAL = -1
SA_EUNSUPPORTED = -2
SA_ETIMEOUT = -3
SA_ECUDA = -4

SA_DEV_OK = 0
SA_DEV_WAIT_TIMEOUT = 1

SA_COVERAGE_JOINT = 0
SA_COVERAGE_VIDEO_RESIDUAL = 1

SA_STATS_EXACT = 0
SA_STATS_MAX = 1

SA_ROW_TIE_AT_CUT = 1
SA_ROW_NEAR_TARGET = 2
SA_ROW_EMPTY_FALLBACK = 4

_c_i64_4 = ctypes.c_int64 * 4
_c_i64_3 = ctypes.c_int64 * 3
_vp = ctypes.c_void_p
_i = ctypes.c_int
_f = ctypes.c_float

# name -> (restype, argtypes); mirrors include/sinkattn.h
_SIGNATURES = {
    "sa_last_error": (ctypes.c_char_p, []),
    "sa_version": (_i, []),
    "sa_device_sm_count": (_i, []),
    "sa_bsattn_fwd": (
        _i,
        [_vp, _vp, _vp, _vp, _vp, _vp, _i, _i, _i, _i, _i, _vp, _vp, _i, _vp, _f, _vp, _vp,
         _vp, _vp, _vp],
    ),
    "sa_sink_dynamic_attn_fwd": (
        _i,
        [_vp, _vp, _vp, _vp, _vp, _vp, _i, _i, _i, _i, _i, _vp, _vp, _i, _vp, _vp, _vp, _vp, _vp,
         _i, _f, _f, _vp, _vp, _vp, _vp, _vp],
    ),
    "sa_pool_scores_workspace_size": (ctypes.c_size_t, [_i, _i, _i, _i, _i]),
    "sa_pool_scores": (
        _i,
        [_vp, _vp, _vp, _vp, _i, _i, _i, _i, _i, _f, _vp, _vp, _vp, ctypes.c_size_t, _vp],
    ),
    "sa_calibration_layer_workspace_size": (ctypes.c_size_t, [_i, _i, _i]),
    "sa_calibration_layer": (
        _i,
        [_vp, _vp, _vp, _vp, _i, _i, _i, _i, _f, _vp, _vp, _vp, _vp, _i, _vp, _vp, _i, _f, _i,
         _i, _i, _vp, ctypes.c_size_t, _vp, _vp],
    ),
    "sa_pool_means": (_i, [_vp, _vp, _vp, _vp, _i, _i, _i, _i, _i, _vp, _vp, _vp]),
    "sa_pooled_softmax_layers": (_i, [_vp, _vp, _i, _i, _i, _i, _i, _f, _vp, _vp, _vp]),
    "sa_pooled_softmax": (_i, [_vp, _vp, _i, _i, _i, _i, _f, _vp, _vp, _vp, _vp]),
    "sa_pool_scores_noalloc": (
        _i,
        [_vp, _vp, _vp, _vp, _i, _i, _i, _i, _i, _f, _vp, _vp, _vp],
    ),
    "sa_block_stats_workspace_size": (ctypes.c_size_t, [_i, _i, _i, _i]),
    "sa_block_stats": (
        _i,
        [_vp, _vp, _vp, _vp, _i, _i, _i, _i, _i, _f, _vp, _vp, ctypes.c_size_t, _vp, _vp],
    ),
    "sa_score_accumulate": (_i, [_vp, ctypes.c_int64, _vp, _vp, _i, _vp]),
    "sa_score_finalize": (_i, [_vp, _vp, _vp, _f, ctypes.c_int64, _vp, _vp, _i, _vp]),
    "sa_score_accumulate_aligned": (_i, [_vp, _i, _i, _i, _i, _i, _vp, _vp, _vp, _i, _vp]),
    "sa_score_finalize_presence": (_i, [_vp, _vp, _vp, ctypes.c_int64, _vp, _vp, _i, _vp]),
    "sa_qk_norm_rope": (
        _i,
        [_vp, _vp, ctypes.c_int64, ctypes.c_int64, _i, _i, _i, _i, _vp, _vp, _i, _f, _vp, _vp,
         ctypes.c_int64, _vp, _vp, ctypes.c_int64, ctypes.c_int64, _vp],
    ),
    "sa_coverage_mask": (
        _i,
        [_vp, _vp, _i, _i, _i, _i, _f, _i, _i, _i, _vp, _vp, _vp, _vp, _vp],
    ),
    "sa_mean_pool_seq": (_i, [_vp, _vp, _i, _i, _i, _i, _i, _i, _vp, _vp, _vp]),
    "sa_ipc_alloc": (_i, [ctypes.c_size_t, _vp]),
    "sa_ipc_free": (_i, [_vp]),
    "sa_ipc_get_handle": (_i, [_vp, _vp]),
    "sa_ipc_open_handle": (_i, [_vp, _vp]),
    "sa_ipc_close": (_i, [_vp]),
    "sa_ulysses_dispatch": (_i, [_i, _vp, _vp, _i, _i, _i, _i, _i, _i, _i, _vp, _vp]),
    "sa_ulysses_combine": (_i, [_vp, _vp, _i, _i, _i, _i, _i, _i, _i, _vp, _vp, _vp]),
    "sa_ulysses_dispatch_units": (_i, [_i, _vp, _vp, _i, _i, _i, _i, _i, _i, _i, _i, _i, _vp,
                                       _vp]),
    "sa_ulysses_combine_units": (_i, [_vp, _vp, _i, _i, _i, _i, _i, _i, _i, _i, _i, _vp, _vp,
                                      _vp]),
    "sa_status_create": (_vp, []),
    "sa_status_device_pointer": (_i, [_vp, _vp]),
    "sa_status_destroy": (_i, [_vp]),
    "sa_check_status": (_i, [_vp]),
    "sa_selftest_wait_timeout": (_i, [_vp, ctypes.c_uint64, _vp]),
    "sa_mix_outputs": (
        _i,
        [_vp, _vp, _vp, _vp, _vp, _vp, _i, _i, _i, _i, _f, _vp, _vp, _vp],
    ),
}

_lock = threading.Lock()
_lib: ctypes.CDLL | None = None


def exported_names() -> list[str]:
    return list(_SIGNATURES)


def load() -> ctypes.CDLL:
    """Load (once) and return the library with argtypes/restypes declared."""
    global _lib
    with _lock:
        if _lib is not None:
            return _lib
        if not LIB_PATH.exists():
            raise RuntimeError(
                f"sinkattn_b200: {LIB_PATH.name} is not built; run "
                "`python -m sinkattn_b200.build` (no CPU fallback exists)"
            )
        lib = ctypes.CDLL(os.fspath(LIB_PATH))
        for name, (res, args) in _SIGNATURES.items():
            fn = getattr(lib, name)
            fn.restype = res
            fn.argtypes = args
        _lib = lib
        return lib


def last_error() -> str:
    msg = load().sa_last_error()
    return msg.decode(errors="replace") if msg else ""


def check(rc: int, what: str) -> None:
    if rc != SA_OK:
        names = {SA_EINVAL: "SA_EINVAL", SA_EUNSUPPORTED: "SA_EUNSUPPORTED",
                 SA_ETIMEOUT: "SA_ETIMEOUT", SA_ECUDA: "SA_ECUDA"}
        raise RuntimeError(f"{what} failed ({names.get(rc, rc)}): {last_error()}")


def strides4(t) -> "ctypes.Array":
    st = t.stride()
    return _c_i64_4(*[int(x) for x in st])


def strides3(t) -> "ctypes.Array":
    st = t.stride()
    return _c_i64_3(*[int(x) for x in st])

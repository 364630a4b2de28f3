"""ctypes binding of the C ABI in include/dm3.h (libdm3.so, built for sm_100a).

The library is required: there is no CPU or eager-PyTorch fallback. Importing the package works
without it (so CPU-only tooling can inspect the API), but the first call raises a RuntimeError
naming the missing file.
"""

from __future__ import annotations

import ctypes
import os
import re
from pathlib import Path

PKG_DIR = Path(__file__).resolve().parent
LIB_PATH = Path(os.environ.get("DM3_LIB", PKG_DIR / "libdm3.so"))
HEADER = PKG_DIR.parent / "include" / "dm3.h"

DM3_OK, DM3_EINVAL, DM3_ECUDA, DM3_ETIMEOUT, DM3_ENOSPACE = 0, 1, 2, 3, 4

_p, _i, _i64, _sz, _u32p = ctypes.c_void_p, ctypes.c_int, ctypes.c_int64, ctypes.c_size_t, ctypes.POINTER(ctypes.c_uint32)

# name -> (restype, argtypes), in the order of include/dm3.h
SIGNATURES = {
    "dm3_last_error": (ctypes.c_char_p, []),
    "dm3_version": (ctypes.c_char_p, []),
    "dm3_fp8_gemv": (_i, [_p, _i, _i, _i, _p, _i64, _p, _i64, _i, _p, _i, _p, _i64, _i, _p]),
    "dm3_gemv_status": (_i, [_u32p, _p]),
    "dm3_fp8_gemv_gather": (_i, [_p, _i, _i, _i, _p, _i64, _i64, _p, _p, _i64, _i, _p, _i64, _i, _p]),
    "dm3_audio_head_workspace_bytes": (_sz, [_i]),
    "dm3_audio_head": (_i, [_p, _i, _p, _i64, _p, _i64, _i, _p, _i64, _i, _p, _p, _p, _i64, _p, _p, _i, _p, _sz, _p]),
    "dm3_direction_score": (_i, [_p, _p, _i, _p, _i64, _i64, _p, _p]),
    "dm3_fp8_gemm_workspace_bytes": (_sz, [_i, _i]),
    "dm3_fp8_gemm": (_i, [_p, _i, _i, _i, _p, _i64, _p, _i64, _i, _p, _i, _p, _i64, _i, _p, _sz, _p]),
    "dm3_moe_workspace_bytes": (_sz, [_i, _i, _i]),
    "dm3_moe_forward": (_i, [_p, _i, _i, _i, _p, _p, _i, _i, _p, _i64, _p, _i64, _p, _i64, _p, _i64, _i, _p, _p,
                             _sz, _p]),
    "dm3_moe_layer": (_i, [_p, _i, _i, _i, _p, _i, _i, _i, _i, _p, _p, _i64, _p, _i64, _p, _i64, _p, _i64, _i, _p,
                           _p, _p, _p, _i, _p, _p, _p, _p, _p, _p, _sz, _p]),
    "dm3_moe_status": (_i, [_p, _u32p, _p]),
    "dm3_moe_layer_noalloc": (_i, [_p, _i, _i, _i, _p, _i, _i, _i, _i, _p, _p, _i64, _p, _i64, _p, _i64, _p, _i64, _i,
                                   _p, _p, _p, _p, _i, _p, _p, _p, _p, _p, _p]),
    "dm3_moe_noalloc_status": (_i, [_u32p, _p]),
    "dm3_set_wait_limit_ns": (_i, [ctypes.c_uint64]),
    "dm3_moe_prefill_workspace_bytes": (_sz, [_i, _i, _i, _i, _i]),
    "dm3_moe_prefill": (_i, [_p, _i, _i, _i, _p, _i, _i, _i, _p, _p, _i64, _p, _i64, _p, _i64, _p, _i64, _i, _p, _p,
                             _p, _p, _i, _p, _p, _p, _p, _p, _p, _p, _p, _sz, _p]),
    "dm3_moe_grouped": (_i, [_p, _i, _i, _i, _p, _p, _i, _i, _p, _i64, _p, _i64, _p, _i64, _p, _i64, _i, _p, _p, _p,
                             _p, _sz, _p]),
    "dm3_route_workspace_bytes": (_sz, [_i, _i, _i, _i]),
    "dm3_route": (_i, [_p, _i, _i, _p, _i, _i, _i, _p, _p, _p, _p, _sz, _p]),
    "dm3_ep_arena_bytes": (_sz, [_i, _i, _i, _i]),
    "dm3_ep_alloc": (_i, [_sz, ctypes.POINTER(ctypes.c_void_p)]),
    "dm3_ep_free": (_i, [_p]),
    "dm3_ep_ipc_handle": (_i, [_p, _p]),
    "dm3_ep_ipc_open": (_i, [_p, ctypes.POINTER(ctypes.c_void_p)]),
    "dm3_ep_ipc_close": (_i, [_p]),
    "dm3_moe_prefill_ep_workspace_bytes": (_sz, [_i, _i, _i, _i, _i, _i]),
    "dm3_moe_prefill_ep": (_i, [_p, _i, _i, _i, _p, _i, _i, _i, _p, _p, _i64, _p, _i64, _p, _i64, _p, _i64, _i, _p,
                                _p, _p, _p, _i, _p, _p, _p, _p, _p, _i, _i, _i, _p, _p, _p, _sz, _p]),
    "dm3_ep_dispatch": (_i, [_p, _i, _i, _i, _p, _i, _i, _i, _p, _p, _p, _p, _i, _i, _i, _p, _p, _p, _sz, _p]),
    "dm3_ep_combine": (_i, [_p, _i, _i, _i, _p, _i, _i, _p, _i64, _p, _i64, _p, _i64, _p, _i64, _i, _p, _p, _p, _p,
                            _i, _p, _p, _p, _i, _i, _i, _p, _p, _sz, _p]),
    "dm3_moe_layer_ep": (_i, [_p, _i, _i, _i, _p, _i, _i, _i, _i, _p, _p, _i64, _p, _i64, _p, _i64, _p, _i64, _i, _p,
                              _p, _p, _p, _i, _p, _p, _p, _p, _p, _i, _i, _i, _p, _p, _sz, _p]),
    "dm3_last_launch_count": (_i, []),
}

_lib = None


def header_functions() -> list[str]:
    """Entry points declared in include/dm3.h (the ABI contract)."""
    text = HEADER.read_text()
    return re.findall(r"^\s*(?:const\s+)?(?:char\s*\*|int|size_t|void)\s+\**\s*(dm3_\w+)\s*\(", text, re.M)


def load():
    """Loads libdm3.so once and declares every signature; raises RuntimeError if it is missing."""
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            raise RuntimeError(
                f"drama3_b200: {LIB_PATH} is missing. Build it with `python -c \"import __graft_entry__ as g; "
                f"g.build()\"` (nvcc, sm_100a). There is no fallback implementation."
            )
        lib = ctypes.CDLL(str(LIB_PATH))
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(lib, name)
            fn.restype = res
            fn.argtypes = args
        _lib = lib
    return _lib


def check(rc: int, what: str) -> None:
    """Turns a non-zero status into a RuntimeError carrying dm3_last_error()."""
    if rc != DM3_OK:
        msg = load().dm3_last_error().decode(errors="replace")
        raise RuntimeError(f"{what} failed (status {rc}): {msg}")

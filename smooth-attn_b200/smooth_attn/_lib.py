"""ctypes binding of the C ABI in ``include/smooth_attn_b200.h``.

The shared library ``libsmooth_attn_b200.so`` sits next to this file (built
in-tree by ``smooth-attn_b200/build.py``).  There is no fallback: if the
library is missing or cannot be loaded, every kernel entry point raises
``RuntimeError``.
"""

from __future__ import annotations

import ctypes
import os
import threading
from pathlib import Path

LIB_PATH = Path(__file__).with_name("libsmooth_attn_b200.so")
# SA_DEBUG_LIB=1: the debug build (device-side index checks, build.py --debug)
DEBUG_LIB_PATH = Path(__file__).with_name("libsmooth_attn_b200_debug.so")

SA_OK = 0
SA_ERR_ARG = -1
SA_ERR_ALIGN = -2
SA_ERR_UNSUPPORTED = -3
SA_ERR_LAUNCH = -4
SA_ERR_TIMEOUT = -5
SA_ERR_CUDA = -6
SA_ERR_BOUNDS = -7

SA_F32, SA_F16, SA_BF16 = 0, 1, 2

_i64 = ctypes.c_int64
_int = ctypes.c_int
_f = ctypes.c_float
_p = ctypes.c_void_p
_i64p = ctypes.POINTER(ctypes.c_int64)

# name -> (restype, argtypes); mirrors include/smooth_attn_b200.h
SIGNATURES = {
    "sa_version": (_int, []),
    "sa_status_string": (ctypes.c_char_p, [_int]),
    "sa_last_cuda_error": (ctypes.c_char_p, []),
    "sa_device_status": (_int, [_int]),
    "sa_stream_status": (_int, [_p, _int]),
    "sa_probe_bounded_wait": (_int, [_i64, _p, _p]),
    "sa_debug_checks": (_int, []),
    "sa_copy_causal_bands": (_int, [_p, _p, _i64, _i64, _i64, _i64, _int, _i64p, _p]),
    "sa_host_zero_causal_tail": (_int, [_p, _i64, _i64, _i64, _i64, _int]),
    "sa_norm_fwd": (_int, [_p, _p, _p, _i64, _i64, _i64, _i64, _int, _int, _f, _f, _int, _p]),
    "sa_norm_bwd": (_int, [_p, _p, _p, _p, _i64, _i64, _i64, _i64, _i64, _int, _int, _int, _f, _f, _int, _p]),
    "sa_flash_fwd": (_int, [_p, _p, _p, _p, _p, _p, _i64, _i64, _i64, _i64, _i64,
                            _i64p, _i64p, _i64p, _i64p, _f, _i64, _int, _int, _p]),
    "sa_flash_bwd_workspace_size": (_i64, [_i64, _i64, _i64, _i64, _i64]),
    "sa_flash_bwd_noalloc_max_bytes": (_i64, []),
    "sa_flash_bwd_noalloc": (_int, [_p, _p, _p, _p, _p, _p, _p, _p, _p, _p,
                                    _i64, _i64, _i64, _i64, _i64,
                                    _i64p, _i64p, _i64p, _i64p, _i64p, _i64p, _i64p, _i64p,
                                    _f, _i64, _int, _int, _p]),
    "sa_flash_bwd": (_int, [_p, _p, _p, _p, _p, _p, _p, _p, _p, _p, _p, _i64,
                            _i64, _i64, _i64, _i64, _i64,
                            _i64p, _i64p, _i64p, _i64p, _i64p, _i64p, _i64p, _i64p,
                            _f, _i64, _int, _int, _int, _p]),
    "sa_flash_fwd_chunk": (_int, [_p, _p, _p, _p, _p, _p, _i64, _i64, _i64, _i64, _i64, _i64, _i64,
                                  _i64p, _i64p, _i64p, _i64p, _f, _i64, _int, _int, _p]),
    "sa_flash_bwd_chunk": (_int, [_p, _p, _p, _p, _p, _p, _p, _p, _p, _p, _p, _i64,
                                  _i64, _i64, _i64, _i64, _i64, _i64, _i64,
                                  _i64p, _i64p, _i64p, _i64p, _i64p, _i64p, _i64p, _i64p,
                                  _f, _i64, _int, _int, _int, _p]),
    "sa_out_proj": (_int, [_p, _p, _p, _i64, _i64, _i64, _i64, _i64, _i64, _int, _p]),
    "sa_rope_rotate": (_int, [_p, _p, _p, _p, _int, _i64, _i64, _i64, _i64, _i64p, _int, _p]),
    "sa_rope_flash_fwd_workspace_size": (_i64, [_i64, _i64, _i64, _i64, _i64]),
    "sa_rope_flash_fwd": (_int, [_p, _p, _p, _p, _p, _p, _p, _int, _p, _i64,
                                 _i64, _i64, _i64, _i64, _i64, _i64p, _i64p, _i64p, _i64p,
                                 _f, _i64, _int, _int, _p]),
    "sa_fp8_quantize": (_int, [_p, _p, _p, _i64, _i64, _i64, _int, _p, _p, _p, _p, _p, _p]),
    "sa_fp8_flash_fwd": (_int, [_p, _p, _p, _p, _p, _p, _i64, _i64, _i64, _i64, _i64,
                                _i64p, _i64p, _i64p, _i64p, _f, _i64, _p]),
    "sa_paged_decode_workspace_size": (_i64, [_i64, _i64, _i64, _i64, _i64, _i64, _int]),
    "sa_paged_decode": (_int, [_p, _p, _p, _p, _p, _p, _p, _i64,
                               _i64, _i64, _i64, _i64, _i64, _i64, _i64, _f, _int, _p]),
}

_lock = threading.Lock()
_lib = None


def load(path: Path | str | None = None):
    """Load (once) and return the ctypes library handle; raise if unavailable."""
    global _lib
    with _lock:
        if _lib is not None and path is None:
            return _lib
        if path is not None:
            p = Path(path)
        else:
            p = DEBUG_LIB_PATH if os.environ.get("SA_DEBUG_LIB", "") not in ("", "0") else LIB_PATH
        if not p.exists():
            raise RuntimeError(
                f"{p.name} is not built (expected at {p}); run `python smooth-attn_b200/build.py`. "
                "smooth_attn has no CPU or Triton fallback."
            )
        lib = ctypes.CDLL(str(p))
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(lib, name)
            fn.restype = res
            fn.argtypes = args
        if path is None:
            _lib = lib
        return lib


class KernelError(RuntimeError):
    pass


def check(status: int, what: str):
    """Map a C-ABI status to the reference's exception types."""
    if status == SA_OK:
        return
    lib = load()
    msg = lib.sa_status_string(status).decode()
    if status in (SA_ERR_ARG, SA_ERR_UNSUPPORTED, SA_ERR_ALIGN):
        raise ValueError(f"{what}: {msg}")
    detail = lib.sa_last_cuda_error().decode()
    raise KernelError(f"{what}: {msg} {detail}".strip())


def strides(t):
    return (ctypes.c_int64 * 4)(*t.stride())

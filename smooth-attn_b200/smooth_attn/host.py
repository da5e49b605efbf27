"""Causal squareplus normalization between pinned host buffers.

An addition to the reference's API (the reference only takes CUDA tensors):
``softplus_norm_causal_host_out(out, x, ...)`` normalizes the causal
``[..., L, L]`` matrices of the pinned CPU tensor ``x`` into the pinned CPU
tensor ``out`` on the GPU and returns once ``out`` is complete.

On this path PCIe, not HBM, sets the pace, so only what matters crosses it:

* up: the part of each row the causal kernel reads -- bands of 128 rows,
  columns up to the end of the band (about half of x);
* down: the same bands of the output, whose columns past each row's diagonal
  are exact zeros written by the kernel;
* the rest of ``out`` (the columns past each band, all zeros) is written by a
  host thread while the GPU works.

The matrices go through in ``slices`` slices over three CUDA streams (upload,
kernel, download), so both PCIe directions and the kernel overlap.  Device
buffers and streams are kept per (device, shape, dtype).
"""

from __future__ import annotations

import ctypes
import threading

import torch

from . import _lib
from .kernels import DEFAULT_FAMILY, softplus_norm_causal_triton_out

BAND = 128  # rows per copied band (a multiple of every dtype's 16-byte vector)
_SUPPORTED = (torch.float32, torch.float16, torch.bfloat16)
_state: dict = {}
_state_lock = threading.Lock()


def _bands(L: int, elem: int):
    """(first row, end row, copied columns) of each band."""
    vec = 16 // elem
    for r0 in range(0, L, BAND):
        r1 = min(L, r0 + BAND)
        yield r0, r1, min(L, -(-r1 // vec) * vec)


def causal_band_bytes(shape, dtype) -> int:
    """Bytes that one direction of ``softplus_norm_causal_host_out`` moves."""
    L = int(shape[-1])
    nmat = 1
    for d in shape[:-2]:
        nmat *= int(d)
    elem = torch.empty((), dtype=dtype).element_size()
    return sum((r1 - r0) * w for r0, r1, w in _bands(L, elem)) * elem * nmat


def _check(out, x):
    for name, t in (("x", x), ("out", out)):
        if not isinstance(t, torch.Tensor):
            raise TypeError(f"{name} must be a torch.Tensor")
    for name, t in (("x", x), ("out", out)):
        if t.device.type != "cpu" or not t.is_pinned():
            raise ValueError(f"{name} must be a pinned CPU tensor (torch.empty(..., pin_memory=True))")
        if not t.is_contiguous():
            raise ValueError(f"{name} must be contiguous")
    if x.dtype not in _SUPPORTED:
        raise ValueError(f"x dtype must be one of {_SUPPORTED}, got {x.dtype}")
    if out.shape != x.shape or out.dtype != x.dtype:
        raise ValueError("out must match x in shape and dtype")
    if x.dim() < 2 or x.shape[-1] != x.shape[-2]:
        raise ValueError("x must be [..., L, L]")


def _buffers(dev, nmat, L, dtype, nch):
    key = (dev, nmat, L, dtype, nch)
    with _state_lock:
        st = _state.get(key)
        if st is None:
            st = {
                "xd": torch.empty((nmat, L, L), device=dev, dtype=dtype),
                "od": torch.empty((nmat, L, L), device=dev, dtype=dtype),
                "s_in": torch.cuda.Stream(dev),
                "s_out": torch.cuda.Stream(dev),
                "ev_in": [torch.cuda.Event() for _ in range(nch)],
                "ev_c": [torch.cuda.Event() for _ in range(nch)],
            }
            _state[key] = st
    return st


def softplus_norm_causal_host_out(out, x, alpha=DEFAULT_FAMILY.alpha, theta=DEFAULT_FAMILY.theta,
                                  power=DEFAULT_FAMILY.power, *, family=None, device=None, slices=8):
    """``softplus_norm_causal_triton_out`` for pinned host ``x`` / ``out``; returns ``out``."""
    _check(out, x)
    L = x.shape[-1]
    nmat = x.numel() // (L * L) if L else 0
    if nmat == 0 or L == 0:
        return out
    dev = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
    elem = x.element_size()
    nch = slices if slices > 0 and nmat % slices == 0 else 1
    per = nmat // nch
    lib = _lib.load()
    xh, oh = x.view(nmat, L, L), out.view(nmat, L, L)

    # the all-zero columns past every band, on the host (native threads,
    # non-temporal stores), while the GPU works
    zero_status = []

    def zero_tail():
        zero_status.append(lib.sa_host_zero_causal_tail(ctypes.c_void_p(oh.data_ptr()), nmat, L, elem, BAND, 0))

    zt = threading.Thread(target=zero_tail, daemon=True)
    zt.start()
    try:
        _run_slices(lib, dev, xh, oh, nmat, L, elem, nch, per, alpha, theta, power, family)
    except BaseException:
        torch.cuda.synchronize(dev)  # no copy still in flight into out when the error surfaces
        raise
    finally:
        zt.join()  # never return (or raise) while the host thread still writes into out
    _lib.check(zero_status[0] if zero_status else _lib.SA_ERR_ARG, "sa_host_zero_causal_tail")
    return out


def _run_slices(lib, dev, xh, oh, nmat, L, elem, nch, per, alpha, theta, power, family):
    """Upload bands, run the kernel and download bands, slice by slice."""
    with torch.cuda.device(dev):
        st = _buffers(dev, nmat, L, xh.dtype, nch)
        xd, od, s_in, s_out = st["xd"], st["od"], st["s_in"], st["s_out"]
        cur = torch.cuda.current_stream(dev)
        s_in.wait_stream(cur)  # an earlier call's kernels are done with xd
        s_out.wait_stream(cur)
        for i in range(nch):
            a = i * per
            _lib.check(lib.sa_copy_causal_bands(ctypes.c_void_p(xd[a].data_ptr()), ctypes.c_void_p(xh[a].data_ptr()),
                                                per, L, elem, BAND, 1, None, ctypes.c_void_p(s_in.cuda_stream)),
                       "sa_copy_causal_bands")
            st["ev_in"][i].record(s_in)
            cur.wait_event(st["ev_in"][i])
            softplus_norm_causal_triton_out(od[a:a + per], xd[a:a + per], alpha, theta, power, family=family)
            st["ev_c"][i].record(cur)
            s_out.wait_event(st["ev_c"][i])
            _lib.check(lib.sa_copy_causal_bands(ctypes.c_void_p(oh[a].data_ptr()), ctypes.c_void_p(od[a].data_ptr()),
                                                per, L, elem, BAND, 0, None, ctypes.c_void_p(s_out.cuda_stream)),
                       "sa_copy_causal_bands")
        cur.wait_stream(s_out)
        s_out.synchronize()

"""Public API of smooth-attn, backed by hand-written sm_100a CUDA kernels.

Same names, signatures, argument meaning and exception types as the
reference package (NoSelection/smooth-attn ``src/smooth_attn/kernels.py``);
the ``*_triton*`` names are kept for drop-in compatibility although no Triton
is involved.  Every hot-path call validates on the host, then calls the C ABI
of ``libsmooth_attn_b200.so`` (``include/smooth_attn_b200.h``) on torch's
current CUDA stream.  There is no CPU or Triton fallback: on a machine
without the built library the kernel entry points raise ``RuntimeError``.
"""

from __future__ import annotations

import contextlib
import ctypes
import functools
import os
import math
import threading
from dataclasses import dataclass

import torch
import torch.nn.functional as F

from . import _lib

SUPPORTED_POWERS = (1, 2, 3)  # kernels.py:24
SUPPORTED_DTYPES = {  # kernels.py:25-29
    "fp32": torch.float32,
    "fp16": torch.float16,
    "bf16": torch.bfloat16,
}
EPS = 1e-12  # kernels.py:57
MAX_ROW_COLS = 4096  # kernels.py:236-240 (largest row the fused row kernels accept)
FLASH_HEAD_DIMS = (32, 64, 128)

_DTYPE_CODE = {torch.float32: _lib.SA_F32, torch.float16: _lib.SA_F16, torch.bfloat16: _lib.SA_BF16}
_CAUSAL_MASK_CACHE: dict = {}


@dataclass(frozen=True)
class FamilyConfig:
    """squareplus(alpha * (x - theta))^power / sum  (kernels.py:65-89)."""

    alpha: float = 2.0
    theta: float = 0.5
    power: int = 2

    def __post_init__(self):
        if self.power not in SUPPORTED_POWERS:
            raise ValueError(f"power must be one of {SUPPORTED_POWERS}, got {self.power}")

    @property
    def cache_key(self):
        return (float(self.alpha), float(self.theta), int(self.power))

    @property
    def kernel_kwargs(self):
        return {"ALPHA": float(self.alpha), "THETA": float(self.theta), "POWER": int(self.power)}

    @property
    def label(self):
        return f"squareplus({self.alpha:g} * (x - {self.theta:g}))^{self.power} / sum"


@dataclass(frozen=True)
class RowwiseBenchmarkResult:
    shape: tuple
    torch_softmax_us: float
    triton_softmax_us: float
    family_us: float


@dataclass(frozen=True)
class CausalBenchmarkResult:
    dtype: torch.dtype
    batch: int
    heads: int
    seq_len: int
    torch_softmax_us: float
    triton_softmax_us: float
    family_us: float
    softmax_err: float
    family_err: float
    softmax_sums_ok: bool
    family_sums_ok: bool
    softmax_meta: dict
    family_meta: dict


DEFAULT_FAMILY = FamilyConfig()
BENCH_ALPHA = DEFAULT_FAMILY.alpha
BENCH_THETA = DEFAULT_FAMILY.theta
BENCH_POWER = DEFAULT_FAMILY.power


# ---------------------------------------------------------------------------
# validation (error conventions of kernels.py:167-223)
# ---------------------------------------------------------------------------


def _resolve_family(alpha, theta, power, family):
    if family is None:
        return FamilyConfig(alpha=alpha, theta=theta, power=power)
    if (alpha, theta, power) != (DEFAULT_FAMILY.alpha, DEFAULT_FAMILY.theta, DEFAULT_FAMILY.power):
        raise ValueError("pass either family=... or alpha/theta/power overrides, not both")
    return family


def _validate_cuda_tensor(x, *, name):
    if not isinstance(x, torch.Tensor):
        raise TypeError(f"{name} must be a torch.Tensor")
    if not x.is_cuda:
        raise ValueError(f"{name} must be a CUDA tensor")
    if x.dtype not in SUPPORTED_DTYPES.values():
        raise ValueError(f"{name} dtype must be one of {tuple(SUPPORTED_DTYPES.values())}, got {x.dtype}")


def _check_cols(n_cols):
    if n_cols > MAX_ROW_COLS:
        raise ValueError(f"n_cols={n_cols} is too large for this fused row kernel")


def _prepare_rowwise_input(x):
    _validate_cuda_tensor(x, name="x")
    if x.ndim != 2:
        raise ValueError(f"row-wise kernels expect a 2D tensor, got shape {tuple(x.shape)}")
    return x if x.is_contiguous() else x.contiguous()


def _prepare_attention_input(x):
    _validate_cuda_tensor(x, name="x")
    if x.ndim < 2:
        raise ValueError("attention scores must have at least 2 dimensions")
    if x.shape[-1] != x.shape[-2]:
        raise ValueError("causal attention expects square score matrices on the last two dims")
    return x if x.is_contiguous() else x.contiguous()


def _prepare_output(out, reference):
    _validate_cuda_tensor(out, name="out")
    if out.shape != reference.shape:
        raise ValueError(f"out shape {tuple(out.shape)} must match input shape {tuple(reference.shape)}")
    if out.dtype != reference.dtype:
        raise ValueError(f"out dtype {out.dtype} must match input dtype {reference.dtype}")
    if out.device != reference.device:
        raise ValueError("out and input must live on the same CUDA device")
    if out.is_contiguous():
        return out, None
    return torch.empty_like(reference), out


def _finalize_output(kernel_out, user_out):
    if user_out is None:
        return kernel_out
    user_out.copy_(kernel_out)
    return user_out


def _stream(t):
    """torch's current stream on t's device, as the raw handle the C ABI takes
    (the raw lookup skips building a torch.cuda.Stream per call)."""
    return ctypes.c_void_p(torch._C._cuda_getCurrentRawStream(t.device.index))


def _on(device):
    """Make ``device`` current for a launch; no guard when it already is
    (the common case: entering torch.cuda.device costs microseconds per call)."""
    if device.index is None or device.index == torch.cuda.current_device():
        return contextlib.nullcontext()
    return torch.cuda.device(device)


def _is_winner_family(family):
    return family.cache_key == DEFAULT_FAMILY.cache_key


from torch._subclasses.fake_tensor import FakeTensor as _FakeTensor  # noqa: E402
from torch._subclasses.functional_tensor import FunctionalTensor as _FunctionalTensor  # noqa: E402
from torch.fx.experimental.proxy_tensor import get_proxy_mode as _get_proxy_mode  # noqa: E402

_TRACED_TYPES = (_FakeTensor, _FunctionalTensor)


def _tracing(*tensors):
    """True under torch.compile / make_fx / export: the kernels must then be
    reached through the torch.library ops in ``_ops.py`` (a ctypes launch
    is not traceable, and fake tensors have no data pointer)."""
    if torch.compiler.is_compiling() or _get_proxy_mode() is not None:
        return True
    return any(isinstance(t, _TRACED_TYPES) for t in tensors)


def _ops():
    return torch.ops.smooth_attn_b200


def _norm_meta(family, causal, rows, cols):
    variant = ("squareplus_winner" if _is_winner_family(family) else "squareplus_family") + "_b200"
    return {"variant": variant, "causal": bool(causal), "rows": rows, "cols": cols, "kernel": "sa_norm_fwd"}


# ---------------------------------------------------------------------------
# normalization forward / backward launchers
# ---------------------------------------------------------------------------


def _launch_norm_fwd(x2d, out2d, family, causal, rowsum=None):
    """x2d/out2d: contiguous [rows, cols] CUDA tensors of the same dtype."""
    if _tracing(x2d, out2d):
        rows, cols = x2d.shape
        _check_cols(cols)
        res, rs = _ops().norm_fwd(x2d, float(family.alpha), float(family.theta), int(family.power), bool(causal),
                                  rowsum is not None)
        out2d.copy_(res)
        if rowsum is not None:
            rowsum.copy_(rs)
        return _norm_meta(family, causal, rows, cols)
    return _norm_fwd_direct(x2d, out2d, family, causal, rowsum)


def _norm_fwd_direct(x2d, out2d, family, causal, rowsum=None):
    rows, cols = x2d.shape
    _check_cols(cols)
    with _on(x2d.device):
        st = _lib.load().sa_norm_fwd(
            x2d.data_ptr(), out2d.data_ptr(), rowsum.data_ptr() if rowsum is not None else None,
            rows, cols, max(x2d.stride(0), cols), max(out2d.stride(0), cols),
            _DTYPE_CODE[x2d.dtype], int(causal), float(family.alpha), float(family.theta), int(family.power),
            _stream(x2d),
        )
    _lib.check(st, "sa_norm_fwd")
    return _norm_meta(family, causal, rows, cols)


def _launch_norm_bwd(x2d, g2d, rowsum, dx2d, family, causal):
    if _tracing(x2d, g2d, rowsum, dx2d):
        assert causal
        _check_cols(x2d.shape[1])
        dx2d.copy_(_ops().norm_causal_bwd(x2d, g2d, rowsum, float(family.alpha), float(family.theta),
                                          int(family.power)))
        return
    _norm_bwd_direct(x2d, g2d, rowsum, dx2d, family, causal)


def _norm_bwd_direct(x2d, g2d, rowsum, dx2d, family, causal):
    rows, cols = x2d.shape
    _check_cols(cols)
    with _on(x2d.device):
        st = _lib.load().sa_norm_bwd(
            x2d.data_ptr(), g2d.data_ptr(), rowsum.data_ptr() if rowsum is not None else None, dx2d.data_ptr(),
            rows, cols, max(x2d.stride(0), cols), max(g2d.stride(0), cols), max(dx2d.stride(0), cols),
            _DTYPE_CODE[x2d.dtype], _DTYPE_CODE[g2d.dtype], int(causal),
            float(family.alpha), float(family.theta), int(family.power), _stream(x2d),
        )
    _lib.check(st, "sa_norm_bwd")


# ---------------------------------------------------------------------------
# row-wise normalization (kernels.py:985-1035)
# ---------------------------------------------------------------------------


def softplus_norm_triton(x, alpha=DEFAULT_FAMILY.alpha, theta=DEFAULT_FAMILY.theta, power=DEFAULT_FAMILY.power,
                         *, family=None, return_meta=False):
    family = _resolve_family(alpha, theta, power, family)
    x_row = _prepare_rowwise_input(x)
    _check_cols(x_row.shape[1])
    if _tracing(x_row):
        out, _ = _ops().norm_fwd(x_row, float(family.alpha), float(family.theta), int(family.power), False, False)
        meta = _norm_meta(family, False, *x_row.shape)
    else:
        out = torch.empty_like(x_row)
        meta = _launch_norm_fwd(x_row, out, family, causal=False)
    return (out, meta) if return_meta else out


def softplus_norm_triton_out(out, x, alpha=DEFAULT_FAMILY.alpha, theta=DEFAULT_FAMILY.theta,
                             power=DEFAULT_FAMILY.power, *, family=None, return_meta=False):
    family = _resolve_family(alpha, theta, power, family)
    x_row = _prepare_rowwise_input(x)
    kernel_out, user_out = _prepare_output(out, x_row)
    _check_cols(x_row.shape[1])
    meta = _launch_norm_fwd(x_row, kernel_out, family, causal=False)
    result = _finalize_output(kernel_out, user_out)
    return (result, meta) if return_meta else result


def sp2norm_triton(x, return_meta=False):
    return softplus_norm_triton(x, family=DEFAULT_FAMILY, return_meta=return_meta)


# ---------------------------------------------------------------------------
# causal normalization (kernels.py:1254-1297)
# ---------------------------------------------------------------------------


_FAST_CODES = {torch.float32: _lib.SA_F32, torch.float16: _lib.SA_F16, torch.bfloat16: _lib.SA_BF16}
_DEFAULT_ARGS = (float(DEFAULT_FAMILY.alpha), float(DEFAULT_FAMILY.theta), int(DEFAULT_FAMILY.power))


def _causal_out_fast(out, x):
    """Launch the default-family causal forward for plain contiguous CUDA
    tensors of one shape / dtype / device; None when the call needs the
    general path (tracing, other layouts, anything to validate or report)."""
    code = _FAST_CODES.get(x.dtype)
    if (code is None or not x.is_cuda or x.dim() < 2 or out.dtype is not x.dtype or out.shape != x.shape
            or not x.is_contiguous() or not out.is_contiguous() or out.device != x.device):
        return None
    L = x.shape[-1]
    if L != x.shape[-2] or L > MAX_ROW_COLS or L == 0 or torch.compiler.is_compiling() or _get_proxy_mode() is not None:
        return None
    dev = x.device.index
    if dev != torch.cuda.current_device():
        return None
    st = _lib.load().sa_norm_fwd(x.data_ptr(), out.data_ptr(), None, x.numel() // L, L, L, L, code, 1,
                                 *_DEFAULT_ARGS, ctypes.c_void_p(torch._C._cuda_getCurrentRawStream(dev)))
    _lib.check(st, "sa_norm_fwd")
    return out


def _causal_out(out, x_attn, family, rowsum=None):
    kernel_out, user_out = _prepare_output(out, x_attn)
    L = x_attn.shape[-1]
    _check_cols(L)
    meta = _launch_norm_fwd(x_attn.view(-1, L), kernel_out.view(-1, L), family, causal=True, rowsum=rowsum)
    return _finalize_output(kernel_out, user_out), meta


def softplus_norm_causal_triton(x, alpha=DEFAULT_FAMILY.alpha, theta=DEFAULT_FAMILY.theta,
                                power=DEFAULT_FAMILY.power, *, family=None, return_meta=False):
    family = _resolve_family(alpha, theta, power, family)
    x_attn = _prepare_attention_input(x)
    if _tracing(x_attn):
        L = x_attn.shape[-1]
        _check_cols(L)
        out, _ = _ops().norm_fwd(x_attn, float(family.alpha), float(family.theta), int(family.power), True, False)
        meta = _norm_meta(family, True, x_attn.numel() // max(L, 1), L)
        return (out, meta) if return_meta else out
    out = torch.empty_like(x_attn)
    return softplus_norm_causal_triton_out(out, x_attn, family=family, return_meta=return_meta)


def softplus_norm_causal_triton_out(out, x, alpha=DEFAULT_FAMILY.alpha, theta=DEFAULT_FAMILY.theta,
                                    power=DEFAULT_FAMILY.power, *, family=None, return_meta=False):
    if (family is None and not return_meta and type(x) is torch.Tensor and type(out) is torch.Tensor
            and alpha is DEFAULT_FAMILY.alpha and theta is DEFAULT_FAMILY.theta and power is DEFAULT_FAMILY.power):
        # the common call (default family, contiguous same-shape CUDA tensors) without the general
        # path's per-call objects; anything else, or any check failing, takes the general path
        # below with its full validation and error messages
        done = _causal_out_fast(out, x)
        if done is not None:
            return done
    family = _resolve_family(alpha, theta, power, family)
    x_attn = _prepare_attention_input(x)
    result, meta = _causal_out(out, x_attn, family)
    return (result, meta) if return_meta else result


class _SoftplusNormCausalAutogradFn(torch.autograd.Function):
    """kernels.py:1373-1398, but saving the fp32 row normalizer with x and
    running the fused CUDA backward directly on dY's own dtype (no fp32 copy)."""

    @staticmethod
    def forward(ctx, x, alpha, theta, power):
        family = FamilyConfig(alpha=float(alpha), theta=float(theta), power=int(power))
        x_attn = _prepare_attention_input(x)
        L = x_attn.shape[-1]
        if _tracing(x_attn):
            _check_cols(L)
            result, rowsum = _ops().norm_fwd(x_attn, family.alpha, family.theta, family.power, True, True)
        else:
            out = torch.empty_like(x_attn)
            rowsum = torch.empty(x_attn.numel() // max(L, 1), device=x_attn.device, dtype=torch.float32)
            result, _ = _causal_out(out, x_attn, family, rowsum=rowsum)
        ctx.family = family
        ctx.save_for_backward(x_attn, rowsum)
        return result

    @staticmethod
    def backward(ctx, grad_output):
        if not ctx.needs_input_grad[0]:
            return None, None, None, None
        x, rowsum = ctx.saved_tensors
        L = x.shape[-1]
        g = grad_output.contiguous()
        if _tracing(x, g, rowsum):
            f = ctx.family
            return _ops().norm_causal_bwd(x, g, rowsum, f.alpha, f.theta, f.power), None, None, None
        dx = torch.empty_like(x)
        _launch_norm_bwd(x.view(-1, L), g.view(-1, L), rowsum, dx.view(-1, L), ctx.family, causal=True)
        return dx, None, None, None


def softplus_norm_causal(x, alpha=DEFAULT_FAMILY.alpha, theta=DEFAULT_FAMILY.theta, power=DEFAULT_FAMILY.power,
                         *, family=None, implementation="triton"):
    family = _resolve_family(alpha, theta, power, family)
    if implementation == "triton":
        return _SoftplusNormCausalAutogradFn.apply(x, family.alpha, family.theta, family.power)
    if implementation == "eager":
        return softplus_norm_causal_eager(x.float(), family=family).to(x.dtype)
    raise ValueError("implementation must be 'triton' or 'eager'")


class SoftplusNormCausal(torch.nn.Module):
    def __init__(self, alpha=DEFAULT_FAMILY.alpha, theta=DEFAULT_FAMILY.theta, power=DEFAULT_FAMILY.power, *,
                 family=None, implementation="triton"):
        super().__init__()
        self.family = _resolve_family(alpha, theta, power, family)
        self.implementation = implementation

    def forward(self, x):
        return softplus_norm_causal(x, family=self.family, implementation=self.implementation)


# ---------------------------------------------------------------------------
# eager torch functions (public API of the reference, kernels.py:1328-1370,
# 2053-2084).  They are plain torch code on whatever device x lives on; they
# are the user-facing "eager" implementation, not a fallback of the kernels.
# ---------------------------------------------------------------------------


def _causal_mask(seq_len, device):
    key = (device.type, device.index, seq_len)
    if key not in _CAUSAL_MASK_CACHE:
        _CAUSAL_MASK_CACHE[key] = torch.triu(torch.ones(seq_len, seq_len, device=device, dtype=torch.bool), 1)
    return _CAUSAL_MASK_CACHE[key]


def _apply_family_activation_eager(arg):
    return 0.5 * (arg + torch.sqrt(arg * arg + 4.0))


def _family_y_eager(x, family):
    y = _apply_family_activation_eager(family.alpha * (x - family.theta))
    if family.power == 2:
        y = y * y
    elif family.power == 3:
        y = y * y * y
    return y


def softplus_norm_eager(x, alpha=DEFAULT_FAMILY.alpha, theta=DEFAULT_FAMILY.theta, power=DEFAULT_FAMILY.power, *,
                        family=None):
    family = _resolve_family(alpha, theta, power, family)
    y = _family_y_eager(x, family)
    return y / (y.sum(dim=-1, keepdim=True) + EPS)


def softplus_norm_causal_eager(x, alpha=DEFAULT_FAMILY.alpha, theta=DEFAULT_FAMILY.theta,
                               power=DEFAULT_FAMILY.power, *, family=None):
    family = _resolve_family(alpha, theta, power, family)
    y = _family_y_eager(x, family).masked_fill(_causal_mask(x.shape[-1], x.device), 0.0)
    return y / (y.sum(dim=-1, keepdim=True) + EPS)


def softmax_causal_eager(x):
    return F.softmax(x.masked_fill(_causal_mask(x.shape[-1], x.device), float("-inf")), dim=-1)


def sp2norm_flash_attention_eager(q, k, v, *, scale=None, window_size=0):
    B, H_q, T, D = q.shape
    H_kv = k.shape[1]
    if scale is None:
        scale = 1.0 / math.sqrt(D)
    if H_kv < H_q:
        g = H_q // H_kv
        k = k.unsqueeze(2).expand(B, H_kv, g, T, D).reshape(B, H_q, T, D)
        v = v.unsqueeze(2).expand(B, H_kv, g, T, D).reshape(B, H_q, T, D)
    s = torch.matmul(q.float(), k.float().transpose(-2, -1)) * scale
    arg = 2.0 * s - 1.0
    sp = 0.5 * (arg + torch.sqrt(arg * arg + 4.0))
    y = (sp * sp).masked_fill(_causal_mask(T, q.device), 0.0)
    if window_size > 0:
        pos = torch.arange(T, device=q.device)
        y = y.masked_fill(((pos[:, None] - pos[None, :]) >= window_size)[None, None], 0.0)
    attn = y / (y.sum(dim=-1, keepdim=True) + EPS)
    return torch.matmul(attn, v.float()).to(q.dtype)


# ---------------------------------------------------------------------------
# softmax baselines: comparison only, outside the hot path; backed by torch
# with the reference's validation (kernels.py:1233-1251, 1300-1325).
# ---------------------------------------------------------------------------


def softmax_triton(x, return_meta=False):
    x_row = _prepare_rowwise_input(x)
    out = torch.softmax(x_row, dim=-1)
    return (out, {"variant": "torch_softmax"}) if return_meta else out


def softmax_triton_out(out, x, return_meta=False):
    x_row = _prepare_rowwise_input(x)
    kernel_out, user_out = _prepare_output(out, x_row)
    torch.softmax(x_row, dim=-1, out=kernel_out)
    result = _finalize_output(kernel_out, user_out)
    return (result, {"variant": "torch_softmax"}) if return_meta else result


def softmax_causal_triton(x, return_meta=False):
    x_attn = _prepare_attention_input(x)
    out = softmax_causal_eager(x_attn.float()).to(x_attn.dtype)
    return (out, {"variant": "torch_softmax_causal"}) if return_meta else out


def softmax_causal_triton_out(out, x, return_meta=False):
    x_attn = _prepare_attention_input(x)
    kernel_out, user_out = _prepare_output(out, x_attn)
    kernel_out.copy_(softmax_causal_eager(x_attn.float()))
    result = _finalize_output(kernel_out, user_out)
    return (result, {"variant": "torch_softmax_causal"}) if return_meta else result


# ---------------------------------------------------------------------------
# fused squareplus flash attention (kernels.py:1912-2050)
# ---------------------------------------------------------------------------


def _flash_ready(t):
    """TMA needs unit dim stride and 16-byte aligned base/strides; copy otherwise."""
    es = t.element_size()
    ok = (t.stride(3) == 1 and t.data_ptr() % 16 == 0
          and all((s * es) % 16 == 0 for s in t.stride()[:3]))
    return t if ok else t.contiguous()


def _flash_check(q, k, v):
    for name, t in (("q", q), ("k", k), ("v", v)):
        _validate_cuda_tensor(t, name=name)
    if q.dtype not in (torch.bfloat16, torch.float16) or k.dtype != q.dtype or v.dtype != q.dtype:
        raise ValueError(f"flash attention needs bf16 or fp16 q/k/v of one dtype, got {q.dtype}/{k.dtype}/{v.dtype}")
    if q.shape[-1] not in FLASH_HEAD_DIMS:
        raise ValueError(f"head dim {q.shape[-1]} not supported (supported: {FLASH_HEAD_DIMS})")


def _sp2norm_flash_fwd(q, k, v, scale, n_kv_groups=1, window_size=0, use_fast_sqrt=True, with_residual=False):
    """Run the fused forward; return (o, row_sums) like kernels.py:1912-1931.

    with_residual=True also returns o_lo, the residual of o's 16-bit rounding
    (o + o_lo = the kernel's fp32 output to ~16 mantissa bits), which the
    backward uses for delta = rowsum(dO * o).
    """
    if _tracing(q, k, v):
        o, rs, o_lo = _ops().flash_fwd(q, k, v, float(scale), int(window_size), bool(use_fast_sqrt),
                                       bool(with_residual))
        return (o, rs, o_lo) if with_residual else (o, rs)
    return _flash_fwd_direct(q, k, v, scale, window_size, use_fast_sqrt, with_residual=with_residual)


def _flash_fwd_direct(q, k, v, scale, window_size, use_fast_sqrt, o=None, with_residual=False):
    B, H_q, T, D = q.shape
    H_kv = k.shape[1]
    if o is None:
        o = torch.empty_like(q)
        if not (o.stride(3) == 1 and all((s * o.element_size()) % 16 == 0 for s in o.stride()[:3])):
            o = torch.empty(q.shape, device=q.device, dtype=q.dtype)
    o_lo = torch.empty_strided(o.shape, o.stride(), device=o.device, dtype=o.dtype) if with_residual else None
    row_sums = torch.empty(B, H_q, T, device=q.device, dtype=torch.float32)
    if q.numel() == 0:
        return (o, row_sums, o_lo) if with_residual else (o, row_sums)
    with _on(q.device):
        st = _lib.load().sa_flash_fwd(
            q.data_ptr(), k.data_ptr(), v.data_ptr(), o.data_ptr(), _ptr(o_lo), row_sums.data_ptr(),
            B, H_q, H_kv, T, D, _lib.strides(q), _lib.strides(k), _lib.strides(v), _lib.strides(o),
            float(scale), int(window_size), int(not use_fast_sqrt), _DTYPE_CODE[q.dtype], _stream(q),
        )
    _lib.check(st, "sa_flash_fwd")
    return (o, row_sums, o_lo) if with_residual else (o, row_sums)


def _ptr(t):
    """Device pointer of an optional tensor (None or empty -> NULL)."""
    return t.data_ptr() if t is not None and t.numel() else None


def _match_strides(o_lo, o):
    """The C ABI reads o_lo with o's strides: copy it into that layout if needed."""
    if o_lo is None or not o_lo.numel() or o_lo.stride() == o.stride():
        return o_lo
    return torch.empty_strided(o.shape, o.stride(), device=o.device, dtype=o.dtype).copy_(o_lo)


def _deterministic(flag):
    """None follows torch.use_deterministic_algorithms(); otherwise the flag."""
    return torch.are_deterministic_algorithms_enabled() if flag is None else bool(flag)


def _sp2norm_flash_bwd(q, k, v, o, do, row_sums, scale, n_kv_groups=1, window_size=0, use_fast_sqrt=True,
                       o_lo=None, deterministic=None):
    """Run the fused backward; return (dq, dk, dv) like kernels.py:1934-1989.

    o_lo (optional): the forward's residual (``with_residual=True``).
    deterministic: dQ from the query-major kernel, bitwise reproducible
    (None: follow ``torch.use_deterministic_algorithms``)."""
    det = _deterministic(deterministic)
    if _tracing(q, k, v, o, do, row_sums):
        lo = o_lo if o_lo is not None else o.new_empty(0)
        return _ops().flash_bwd(q, k, v, o, lo, do, row_sums, float(scale), int(window_size), bool(use_fast_sqrt),
                                det)
    return _flash_bwd_direct(q, k, v, o, do, row_sums, scale, window_size, use_fast_sqrt, o_lo=o_lo,
                             deterministic=det)


def _flash_bwd_direct(q, k, v, o, do, row_sums, scale, window_size, use_fast_sqrt, o_lo=None, deterministic=False):
    B, H_q, T, D = q.shape
    H_kv = k.shape[1]
    do = _flash_ready(do)
    o_lo = _match_strides(o_lo, o)
    dq = torch.empty(q.shape, device=q.device, dtype=q.dtype)
    dk = torch.empty(k.shape, device=q.device, dtype=q.dtype)
    dv = torch.empty(v.shape, device=q.device, dtype=q.dtype)
    if q.numel() == 0:
        return dq, dk.zero_(), dv.zero_()
    lib = _lib.load()
    ws_bytes = int(lib.sa_flash_bwd_workspace_size(B, H_q, H_kv, T, D))
    ws = torch.empty(max(ws_bytes, 1), device=q.device, dtype=torch.uint8)
    with _on(q.device):
        st = lib.sa_flash_bwd(
            q.data_ptr(), k.data_ptr(), v.data_ptr(), o.data_ptr(), _ptr(o_lo), do.data_ptr(), row_sums.data_ptr(),
            dq.data_ptr(), dk.data_ptr(), dv.data_ptr(), ws.data_ptr(), ws_bytes,
            B, H_q, H_kv, T, D,
            _lib.strides(q), _lib.strides(k), _lib.strides(v), _lib.strides(o), _lib.strides(do),
            _lib.strides(dq), _lib.strides(dk), _lib.strides(dv),
            float(scale), int(window_size), int(not use_fast_sqrt), _DTYPE_CODE[q.dtype], int(bool(deterministic)),
            _stream(q),
        )
    _lib.check(st, "sa_flash_bwd")
    return dq, dk, dv


class _SP2NormFlashAttentionFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, q, k, v, scale, n_kv_groups, window_size, use_fast_sqrt, deterministic=None):
        if not _tracing(q, k, v):  # the traced op readies its inputs itself
            q, k, v = _flash_ready(q), _flash_ready(k), _flash_ready(v)
        train = any(ctx.needs_input_grad[:3])
        res = _sp2norm_flash_fwd(q, k, v, scale, n_kv_groups, window_size, use_fast_sqrt, with_residual=train)
        o, row_sums = res[0], res[1]
        ctx.save_for_backward(q, k, v, o, row_sums, res[2] if train else None)
        ctx.scale = scale
        ctx.n_kv_groups = n_kv_groups
        ctx.window_size = window_size
        ctx.use_fast_sqrt = use_fast_sqrt
        ctx.deterministic = deterministic
        return o

    @staticmethod
    def backward(ctx, grad_output):
        q, k, v, o, row_sums, o_lo = ctx.saved_tensors
        dq, dk, dv = _sp2norm_flash_bwd(q, k, v, o, grad_output, row_sums, ctx.scale, ctx.n_kv_groups,
                                        ctx.window_size, use_fast_sqrt=ctx.use_fast_sqrt, o_lo=o_lo,
                                        deterministic=ctx.deterministic)
        return dq, dk, dv, None, None, None, None, None


def sp2norm_flash_attention(q, k, v, *, scale=None, window_size=0, exact_math=False, deterministic=None):
    """Fused QK^T -> squareplus norm -> V without materializing the T x T scores.

    Supports autograd, GQA/MQA and sliding windows (kernels.py:2016-2050).
    q: [B, H_q, T, D]; k, v: [B, H_kv, T, D] (any strides); bf16 or fp16;
    D in {32, 64, 128}.  deterministic (an addition to the reference's
    signature; None follows ``torch.use_deterministic_algorithms``): compute
    dQ in the query-major kernel with a fixed summation order, so the
    backward is bitwise reproducible.
    """
    assert q.ndim == 4 and k.ndim == 4 and v.ndim == 4
    B, H_q, T, D = q.shape
    H_kv = k.shape[1]
    assert k.shape == (B, H_kv, T, D) and v.shape == (B, H_kv, T, D)
    assert H_q % H_kv == 0, f"H_q ({H_q}) must be divisible by H_kv ({H_kv})"
    _flash_check(q, k, v)
    if scale is None:
        scale = 1.0 / math.sqrt(D)
    return _SP2NormFlashAttentionFn.apply(q, k, v, scale, H_q // H_kv, window_size, not exact_math, deterministic)


def sp2norm_flash_attention_chunk(q, k, v, q_offset, *, scale=None, window_size=0, exact_math=False,
                                  return_residual=False):
    """Forward of a block of queries against a key prefix (``sa_flash_fwd_chunk``).

    q: [B, H_q, Tq, D] at global positions q_offset .. q_offset+Tq-1;
    k, v: [B, H_kv, Tk, D] at positions 0 .. Tk-1.  Same causal (and window)
    rule as ``sp2norm_flash_attention`` in global positions, so splitting a
    sequence into query chunks that each see their key prefix reproduces the
    whole forward.  The building block of context parallelism
    (``smooth_attn.parallel.context_parallel_attention``).  Returns
    (o [B, H_q, Tq, D], row_sums [B, H_q, Tq]), plus o_lo (the residual of
    o's rounding, for ``sp2norm_flash_attention_chunk_bwd``) when
    ``return_residual``.
    """
    assert q.ndim == 4 and k.ndim == 4 and v.ndim == 4
    B, H_q, Tq, D = q.shape
    H_kv, Tk = k.shape[1], k.shape[2]
    assert k.shape == (B, H_kv, Tk, D) and v.shape == (B, H_kv, Tk, D)
    assert H_q % H_kv == 0, f"H_q ({H_q}) must be divisible by H_kv ({H_kv})"
    _flash_check(q, k, v)
    if scale is None:
        scale = 1.0 / math.sqrt(D)
    if _tracing(q, k, v):
        o, rs, o_lo = _ops().flash_fwd_chunk(q, k, v, int(q_offset), float(scale), int(window_size),
                                             bool(exact_math), bool(return_residual))
        return (o, rs, o_lo) if return_residual else (o, rs)
    return _flash_fwd_chunk_direct(q, k, v, q_offset, scale, window_size, exact_math, return_residual)


def _flash_fwd_chunk_direct(q, k, v, q_offset, scale, window_size, exact_math, with_residual=False):
    B, H_q, Tq, D = q.shape
    H_kv, Tk = k.shape[1], k.shape[2]
    q, k, v = _flash_ready(q), _flash_ready(k), _flash_ready(v)
    o = torch.empty(q.shape, device=q.device, dtype=q.dtype)
    o_lo = torch.empty(q.shape, device=q.device, dtype=q.dtype) if with_residual else None
    row_sums = torch.empty(B, H_q, Tq, device=q.device, dtype=torch.float32)
    if q.numel() == 0:
        return (o, row_sums, o_lo) if with_residual else (o, row_sums)
    with _on(q.device):
        st = _lib.load().sa_flash_fwd_chunk(
            q.data_ptr(), k.data_ptr(), v.data_ptr(), o.data_ptr(), _ptr(o_lo), row_sums.data_ptr(),
            B, H_q, H_kv, Tq, Tk, int(q_offset), D, _lib.strides(q), _lib.strides(k), _lib.strides(v),
            _lib.strides(o), float(scale), int(window_size), int(bool(exact_math)), _DTYPE_CODE[q.dtype], _stream(q),
        )
    _lib.check(st, "sa_flash_fwd_chunk")
    return (o, row_sums, o_lo) if with_residual else (o, row_sums)


def sp2norm_flash_attention_chunk_bwd(q, k, v, o, do, row_sums, q_offset, *, scale=None, window_size=0,
                                      exact_math=False, o_lo=None, deterministic=None):
    """Backward of ``sp2norm_flash_attention_chunk`` (``sa_flash_bwd_chunk``).

    Returns (dq [B, H_q, Tq, D], dk, dv [B, H_kv, Tk, D]): dq is complete for
    the query block; dk / dv hold this block's contribution only (the
    context-parallel backward sums them over every rank's query blocks).
    o_lo (optional): the chunk forward's residual (``return_residual=True``).
    """
    D = q.shape[3]
    if scale is None:
        scale = 1.0 / math.sqrt(D)
    det = _deterministic(deterministic)
    if _tracing(q, k, v, o, do, row_sums):
        lo = o_lo if o_lo is not None else o.new_empty(0)
        return _ops().flash_bwd_chunk(q, k, v, o, lo, do, row_sums, int(q_offset), float(scale), int(window_size),
                                      bool(exact_math), det)
    return _flash_bwd_chunk_direct(q, k, v, o, do, row_sums, q_offset, scale, window_size, exact_math, o_lo, det)


def _flash_bwd_chunk_direct(q, k, v, o, do, row_sums, q_offset, scale, window_size, exact_math, o_lo=None,
                            deterministic=False):
    B, H_q, Tq, D = q.shape
    H_kv, Tk = k.shape[1], k.shape[2]
    q, k, v, o, do = (_flash_ready(t) for t in (q, k, v, o, do))
    o_lo = _match_strides(o_lo, o)
    dq = torch.empty(q.shape, device=q.device, dtype=q.dtype)
    dk = torch.empty(k.shape, device=q.device, dtype=q.dtype)
    dv = torch.empty(v.shape, device=q.device, dtype=q.dtype)
    if q.numel() == 0:
        return dq, dk.zero_(), dv.zero_()
    lib = _lib.load()
    ws_bytes = int(lib.sa_flash_bwd_workspace_size(B, H_q, H_kv, Tq, D))
    ws = torch.empty(max(ws_bytes, 1), device=q.device, dtype=torch.uint8)
    with _on(q.device):
        st = lib.sa_flash_bwd_chunk(
            q.data_ptr(), k.data_ptr(), v.data_ptr(), o.data_ptr(), _ptr(o_lo), do.data_ptr(), row_sums.data_ptr(),
            dq.data_ptr(), dk.data_ptr(), dv.data_ptr(), ws.data_ptr(), ws_bytes,
            B, H_q, H_kv, Tq, Tk, int(q_offset), D,
            _lib.strides(q), _lib.strides(k), _lib.strides(v), _lib.strides(o), _lib.strides(do),
            _lib.strides(dq), _lib.strides(dk), _lib.strides(dv),
            float(scale), int(window_size), int(bool(exact_math)), _DTYPE_CODE[q.dtype], int(bool(deterministic)),
            _stream(q),
        )
    _lib.check(st, "sa_flash_bwd_chunk")
    return dq, dk, dv


# ---------------------------------------------------------------------------
# forward-only entry points: RoPE, FP8, paged decode (kernels.py:2093-2829)
# ---------------------------------------------------------------------------


def precompute_rope_cos_sin(dim, seq_len, base=10000.0, device="cuda", dtype=torch.float32):
    """cos/sin tables for RoPE, each [T, D/2] (kernels.py:2093-2101)."""
    inv_freq = 1.0 / (base ** (torch.arange(0, dim, 2, device=device, dtype=torch.float32) / dim))
    t = torch.arange(seq_len, device=device, dtype=torch.float32)
    freqs = torch.outer(t, inv_freq)
    return freqs.cos().to(dtype), freqs.sin().to(dtype)


def _rope_tables(cos, sin, T, D, device):
    assert cos.shape == (T, D // 2) and sin.shape == (T, D // 2)
    if cos.dtype not in _DTYPE_CODE or sin.dtype != cos.dtype:
        cos, sin = cos.float(), sin.float()
    return cos.to(device).contiguous(), sin.to(device).contiguous()


def _rope_flash_fwd(q, k, v, cos, sin, scale, window_size, o=None):
    """Rotate q/k (sa_rope_flash_fwd) and run the tcgen05 forward; ``o`` may be
    a strided view to write into.  Returns (o, row_sums); row_sums is None
    under a tracer (the traced op returns o only)."""
    if _tracing(q, k, v, cos, sin):
        _flash_check(q, k, v)
        T, D = q.shape[2], q.shape[3]
        assert cos.shape == (T, D // 2) and sin.shape == (T, D // 2)
        res = _ops().rope_flash_fwd(q, k, v, cos, sin, float(scale), int(window_size))
        if o is None:
            return res, None
        o.copy_(res)
        return o, None
    return _rope_flash_fwd_direct(q, k, v, cos, sin, scale, window_size, o)


def _rope_flash_fwd_direct(q, k, v, cos, sin, scale, window_size, o=None):
    B, H_q, T, D = q.shape
    H_kv = k.shape[1]
    _flash_check(q, k, v)
    q, k, v = _flash_ready(q), _flash_ready(k), _flash_ready(v)
    cos, sin = _rope_tables(cos, sin, T, D, q.device)
    if o is None:
        o = torch.empty(q.shape, device=q.device, dtype=q.dtype)
    row_sums = torch.empty(B, H_q, T, device=q.device, dtype=torch.float32)
    if q.numel() == 0:
        return o, row_sums
    lib = _lib.load()
    nbytes = lib.sa_rope_flash_fwd_workspace_size(B, H_q, H_kv, T, D)
    ws = torch.empty(nbytes, device=q.device, dtype=torch.uint8)
    with _on(q.device):
        st = lib.sa_rope_flash_fwd(
            q.data_ptr(), k.data_ptr(), v.data_ptr(), o.data_ptr(), row_sums.data_ptr(),
            cos.data_ptr(), sin.data_ptr(), _DTYPE_CODE[cos.dtype], ws.data_ptr(), nbytes,
            B, H_q, H_kv, T, D, _lib.strides(q), _lib.strides(k), _lib.strides(v), _lib.strides(o),
            float(scale), int(window_size), 0, _DTYPE_CODE[q.dtype], _stream(q),
        )
    _lib.check(st, "sa_rope_flash_fwd")
    return o, row_sums


def sp2norm_rope_flash_attention(q, k, v, cos, sin, *, scale=None, window_size=0):
    """Fused RoPE + sp2norm flash attention forward (kernels.py:2373-2430).

    q: [B, H_q, T, D], k/v: [B, H_kv, T, D] un-rotated bf16 (or fp16);
    cos/sin: [T, D/2] tables from ``precompute_rope_cos_sin``.  q and k are
    rotated (rotate-half form, rounded to 16 bits) by one memory-bound pass,
    then the tcgen05 forward runs causal (optionally windowed) squareplus
    attention.  Returns o [B, H_q, T, D] in q's dtype.
    """
    assert q.ndim == 4 and k.ndim == 4 and v.ndim == 4
    B, H_q, T, D = q.shape
    H_kv = k.shape[1]
    assert H_q % H_kv == 0
    assert D % 2 == 0
    assert cos.shape == (T, D // 2) and sin.shape == (T, D // 2)
    if scale is None:
        scale = 1.0 / math.sqrt(D)
    return _rope_flash_fwd(q, k, v, cos, sin, scale, window_size)[0]


def sp2norm_rope_flash_attention_proj(q, k, v, w_o, cos, sin, *, scale=None, window_size=0):
    """Fused RoPE + sp2norm flash attention + output projection
    (kernels.py:2433-2490).

    w_o: [H_q, D, D_model].  The attention writes its output straight into a
    [B, T, H_q, D] buffer, so the projection summed over heads is one GEMM
    [B*T, H_q*D] @ [H_q*D, D_model] on tcgen05 tensor cores (``sa_out_proj``)
    with fp32 accumulation (the reference accumulates heads with bf16
    atomics).  Returns [B, T, D_model] bf16.
    """
    assert q.ndim == 4 and k.ndim == 4 and v.ndim == 4
    B, H_q, T, D = q.shape
    H_kv = k.shape[1]
    assert H_q % H_kv == 0
    assert D % 2 == 0
    assert w_o.shape[0] == H_q and w_o.shape[1] == D
    D_model = w_o.shape[2]
    if scale is None:
        scale = 1.0 / math.sqrt(D)
    o_bthd = torch.empty(B, T, H_q, D, device=q.device, dtype=q.dtype)
    _rope_flash_fwd(q, k, v, cos, sin, scale, window_size, o=o_bthd.permute(0, 2, 1, 3))
    w = w_o.to(device=q.device, dtype=q.dtype).reshape(H_q * D, D_model).contiguous()
    out = _out_proj(o_bthd.view(B * T, H_q * D), w)
    return out.view(B, T, D_model).to(torch.bfloat16)


def _out_proj(a, w):
    """a [M, K] @ w [K, N] -> [M, N] in a's dtype (``sa_out_proj``)."""
    if _tracing(a, w):
        return _ops().out_proj(a, w)
    return _out_proj_direct(a, w)


def _out_proj_direct(a, w):
    M, K = a.shape
    N = w.shape[1]
    out = torch.empty(M, N, device=a.device, dtype=a.dtype)
    if M == 0 or N == 0:
        return out
    if K == 0:
        return out.zero_()
    if a.stride(1) != 1 or (a.stride(0) * 2) % 16 or a.data_ptr() % 16:
        a = a.contiguous()
    if w.stride(1) != 1 or (w.stride(0) * 2) % 16 or w.data_ptr() % 16:
        w = w.contiguous()
    with _on(a.device):
        st = _lib.load().sa_out_proj(a.data_ptr(), w.data_ptr(), out.data_ptr(), M, K, N, a.stride(0), w.stride(0),
                                     out.stride(0), _DTYPE_CODE[a.dtype], _stream(a))
    _lib.check(st, "sa_out_proj")
    return out
def _fp8_quantize(q, k, v):
    """Per-tensor E4M3 quantization of q, k, v on the device (sa_fp8_quantize;
    the reference's _quantize_to_fp8, kernels.py:2592-2601, without its
    host synchronisation).  Returns (q8, k8, vq, scales): E4M3 bytes as
    uint8 tensors, v's quantized values as bf16, device float[3] scales."""
    q, k, v = q.contiguous(), k.contiguous(), v.contiguous()
    dev = q.device
    q8 = torch.empty(q.shape, device=dev, dtype=torch.uint8)
    k8 = torch.empty(k.shape, device=dev, dtype=torch.uint8)
    vq = torch.empty(v.shape, device=dev, dtype=torch.bfloat16)
    scales = torch.empty(3, device=dev, dtype=torch.float32)
    amax = torch.empty(3, device=dev, dtype=torch.int32)
    with _on(dev):
        st = _lib.load().sa_fp8_quantize(q.data_ptr(), k.data_ptr(), v.data_ptr(), q.numel(), k.numel(), v.numel(),
                                         _DTYPE_CODE[q.dtype], q8.data_ptr(), k8.data_ptr(), vq.data_ptr(),
                                         scales.data_ptr(), amax.data_ptr(), _stream(q))
    _lib.check(st, "sa_fp8_quantize")
    return q8, k8, vq, scales


def sp2norm_fp8_flash_attention(q, k, v, *, scale=None, window_size=0):
    """FP8 fused flash attention forward (kernels.py:2630-2673).

    q, k, v are quantized per tensor to E4M3 on the device; QK^T runs on FP8
    tensor cores (tcgen05 kind::f8f6f4) with the dequantization scales folded
    into the score scale, the squareplus activation in fp32, P.V on bf16
    tensor cores against v's quantized values, times v's scale.  Returns
    [B, H_q, T, D] bf16.
    """
    assert q.ndim == 4 and k.ndim == 4 and v.ndim == 4
    B, H_q, T, D = q.shape
    H_kv = k.shape[1]
    assert k.shape == (B, H_kv, T, D) and v.shape == (B, H_kv, T, D)
    assert H_q % H_kv == 0, f"H_q ({H_q}) must be divisible by H_kv ({H_kv})"
    if scale is None:
        scale = 1.0 / math.sqrt(D)
    for name, t in (("q", q), ("k", k), ("v", v)):
        _validate_cuda_tensor(t, name=name)
    if k.dtype != q.dtype or v.dtype != q.dtype:
        raise ValueError(f"q/k/v must share one dtype, got {q.dtype}/{k.dtype}/{v.dtype}")
    if D not in FLASH_HEAD_DIMS:
        raise ValueError(f"head dim {D} not supported (supported: {FLASH_HEAD_DIMS})")
    if _tracing(q, k, v):
        return _ops().fp8_flash_fwd(q, k, v, float(scale), int(window_size))
    return _fp8_flash_fwd_direct(q, k, v, scale, window_size)


def _fp8_flash_fwd_direct(q, k, v, scale, window_size):
    B, H_q, T, D = q.shape
    H_kv = k.shape[1]
    o = torch.empty(B, H_q, T, D, device=q.device, dtype=torch.bfloat16)
    if q.numel() == 0:
        return o
    q8, k8, vq, scales = _fp8_quantize(q, k, v)
    row_sums = torch.empty(B, H_q, T, device=q.device, dtype=torch.float32)
    with _on(q.device):
        st = _lib.load().sa_fp8_flash_fwd(
            q8.data_ptr(), k8.data_ptr(), vq.data_ptr(), o.data_ptr(), row_sums.data_ptr(), scales.data_ptr(),
            B, H_q, H_kv, T, D, _lib.strides(q8), _lib.strides(k8), _lib.strides(vq), _lib.strides(o),
            float(scale), int(window_size), _stream(q),
        )
    _lib.check(st, "sa_fp8_flash_fwd")
    return o


# ---------------------------------------------------------------------------
# paged-KV decode (kernels.py:2681-2829)
# ---------------------------------------------------------------------------

PAGED_HEAD_DIMS = (32, 64, 128, 256)
_paged_ws = {}  # (device index, stream handle) -> zero-ticketed workspace
_paged_ws_lock = threading.Lock()


def _paged_ws_size(B, H_q, H_kv, max_blocks, block_size, D, dtype_code, device_index):
    """sa_paged_decode_workspace_size, cached: it depends only on the shape,
    the device (its SM count) and the kernel choice (SA_PAGED_DECODE_KERNEL),
    and decode calls repeat one shape."""
    return _paged_ws_size_cached(B, H_q, H_kv, max_blocks, block_size, D, dtype_code, device_index,
                                 os.environ.get("SA_PAGED_DECODE_KERNEL"))


@functools.lru_cache(maxsize=256)
def _paged_ws_size_cached(B, H_q, H_kv, max_blocks, block_size, D, dtype_code, device_index, choice):
    return int(_lib.load().sa_paged_decode_workspace_size(B, H_q, H_kv, max_blocks, block_size, D, dtype_code))


def _paged_workspace(device, stream_handle, nbytes):
    """A workspace whose ticket words are zero (every completed call leaves
    them zero), reused per (device, stream) so calls on one stream never
    overlap on the GPU."""
    key = (device.index, stream_handle)
    with _paged_ws_lock:
        ws = _paged_ws.get(key)
        if ws is None or ws.numel() < nbytes:
            ws = torch.zeros(max(nbytes, 1 << 16), dtype=torch.uint8, device=device)
            _paged_ws[key] = ws
        return ws


def sp2norm_paged_attention(q, k_cache, v_cache, block_table, context_lens, *, scale=None, block_size=16):
    """Paged KV-cache sp2norm attention for autoregressive decode
    (kernels.py:2776-2829).

    q: [batch, H_q, 1, D]; k_cache, v_cache: [num_blocks, H_kv, block_size, D];
    block_table: [batch, max_blocks_per_seq] logical-to-physical page map;
    context_lens: [batch] cached tokens per sequence.  Returns the bf16
    [batch, H_q, D] output of sum_j y_j v_j / (sum_j y_j + 1e-12) with
    y_j = squareplus(2 (q . k_j) scale - 1)^2 over every cached token
    (no causal mask), computed by the sm_100a kernel ``sa_paged_decode``.
    """
    assert q.ndim == 4 and q.shape[2] == 1, "Decode: q must be [B, H, 1, D]"
    B, H_q, _, D = q.shape
    H_kv = k_cache.shape[1]
    assert H_q % H_kv == 0
    assert k_cache.shape[2] == block_size and v_cache.shape[2] == block_size
    max_blocks_per_seq = block_table.shape[1]
    if scale is None:
        scale = 1.0 / math.sqrt(D)
    for name, t in (("q", q), ("k_cache", k_cache), ("v_cache", v_cache)):
        _validate_cuda_tensor(t, name=name)
    if q.dtype not in (torch.bfloat16, torch.float16) or k_cache.dtype != q.dtype or v_cache.dtype != q.dtype:
        raise ValueError(f"paged decode needs bf16 or fp16 q/k_cache/v_cache of one dtype, "
                         f"got {q.dtype}/{k_cache.dtype}/{v_cache.dtype}")
    if D not in PAGED_HEAD_DIMS:
        raise ValueError(f"head dim {D} not supported (supported: {PAGED_HEAD_DIMS})")
    if k_cache.shape != v_cache.shape or k_cache.shape[3] != D:
        raise ValueError(f"k_cache {tuple(k_cache.shape)} / v_cache {tuple(v_cache.shape)} do not match D={D}")
    if _tracing(q, k_cache, v_cache, block_table, context_lens):
        return _ops().paged_decode(q, k_cache, v_cache, block_table, context_lens, float(scale), int(block_size))
    return _paged_decode_direct(q, k_cache, v_cache, block_table, context_lens, scale, block_size)


def _paged_decode_direct(q, k_cache, v_cache, block_table, context_lens, scale, block_size):
    B, H_q, _, D = q.shape
    H_kv = k_cache.shape[1]
    max_blocks_per_seq = block_table.shape[1]
    # (conversions only when needed: at batch 1 the host's per-call time, not
    # the kernel, paces back-to-back decode calls)
    if not q.is_contiguous():
        q = q.contiguous()
    if not k_cache.is_contiguous():
        k_cache = k_cache.contiguous()
    if not v_cache.is_contiguous():
        v_cache = v_cache.contiguous()
    dev = q.device
    if block_table.dtype is not torch.int32 or block_table.device != dev or not block_table.is_contiguous():
        block_table = block_table.to(device=dev, dtype=torch.int32).contiguous()
    if context_lens.dtype is not torch.int32 or context_lens.device != dev or not context_lens.is_contiguous():
        context_lens = context_lens.to(device=dev, dtype=torch.int32).contiguous()
    out = torch.empty(B, H_q, D, device=dev, dtype=torch.bfloat16)
    if out.numel() == 0:
        return out
    if max_blocks_per_seq == 0 or k_cache.shape[0] == 0:
        return out.zero_()
    lib = _lib.load()
    with _on(q.device):
        nbytes = _paged_ws_size(B, H_q, H_kv, max_blocks_per_seq, block_size, D, _DTYPE_CODE[q.dtype],
                                q.device.index)
        if nbytes < 0:
            _lib.check(int(nbytes), "sa_paged_decode_workspace_size")
        stream = _stream(q)
        ws = _paged_workspace(q.device, stream.value, nbytes) if nbytes > 0 else None
        st = lib.sa_paged_decode(
            q.data_ptr(), k_cache.data_ptr(), v_cache.data_ptr(), out.data_ptr(),
            block_table.data_ptr(), context_lens.data_ptr(),
            ws.data_ptr() if ws is not None else None, ws.numel() if ws is not None else 0,
            B, H_q, H_kv, k_cache.shape[0], block_size, max_blocks_per_seq, D, float(scale),
            _DTYPE_CODE[q.dtype], stream,
        )
    _lib.check(st, "sa_paged_decode")
    return out


# ---------------------------------------------------------------------------
# timing helpers (kernels.py:2832-2838)
# ---------------------------------------------------------------------------


def _median_cuda_us(fn, warmup=50, iters=200):
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    times = []
    for _ in range(iters):
        a = torch.cuda.Event(enable_timing=True)
        b = torch.cuda.Event(enable_timing=True)
        a.record()
        fn()
        b.record()
        b.synchronize()
        times.append(a.elapsed_time(b) * 1000.0)
    times.sort()
    return times[len(times) // 2]


def bench(fn, x=None, warmup=300, iters=1000):
    callback = (lambda: fn(x)) if x is not None else fn
    return _median_cuda_us(callback, warmup=warmup, iters=iters)


def bench_out(fn, out, x, warmup=300, iters=1000):
    return _median_cuda_us(lambda: fn(out, x), warmup=warmup, iters=iters)

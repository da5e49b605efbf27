"""``torch.library`` custom ops over the C ABI, so that ``torch.compile``
(and any other tracer: ``make_fx``, ``torch.export``) records each fused
kernel as one opaque node instead of breaking the graph at a ctypes call.

The reference's Triton kernels are traced by ``torch.compile`` as user
kernels; a ctypes launch is not traceable, so the public functions in
``kernels.py`` route through these ops whenever they run under a tracer
(``_tracing``) and call the C ABI directly otherwise (a custom-op dispatch
costs tens of microseconds, which would dominate the small decode calls).

Each op's real implementation is the direct launcher; its fake
implementation allocates outputs of the same shapes, dtypes and strides.
Outputs never alias inputs.  Ops (namespace ``smooth_attn_b200``):

* ``norm_fwd(x, alpha, theta, power, causal, with_rowsum) -> (out, rowsum)``
* ``norm_causal_bwd(x, g, rowsum, alpha, theta, power) -> dx``
* ``flash_fwd(q, k, v, scale, window_size, use_fast_sqrt, with_residual) -> (o, row_sums, o_lo)``
* ``flash_bwd(q, k, v, o, o_lo, do, row_sums, scale, window_size, use_fast_sqrt, deterministic) -> (dq, dk, dv)``
* ``flash_fwd_chunk(q, k, v, q_offset, scale, window_size, exact_math, with_residual) -> (o, row_sums, o_lo)``
* ``flash_bwd_chunk(q, k, v, o, o_lo, do, row_sums, q_offset, scale, window_size, exact_math, deterministic)
  -> (dq, dk, dv)``

``o_lo`` is the residual of o's 16-bit rounding (empty when not requested);
the backward ops take an empty ``o_lo`` for "none".
* ``rope_flash_fwd(q, k, v, cos, sin, scale, window_size) -> o``
* ``out_proj(a, w) -> a @ w`` (the RoPE projection GEMM)
* ``fp8_flash_fwd(q, k, v, scale, window_size) -> o``
* ``paged_decode(q, k_cache, v_cache, block_table, context_lens, scale, block_size) -> out``
"""

from __future__ import annotations

import torch
from torch import Tensor

from . import kernels as K

NS = "smooth_attn_b200"


def _rows(x: Tensor) -> int:
    L = x.shape[-1]
    return x.numel() // L if L else 0


# ------------------------------------------------------------------ norm


@torch.library.custom_op(f"{NS}::norm_fwd", mutates_args=(), device_types="cuda")
def norm_fwd(x: Tensor, alpha: float, theta: float, power: int, causal: bool,
             with_rowsum: bool) -> tuple[Tensor, Tensor]:
    x = x.contiguous()
    out = torch.empty(x.shape, device=x.device, dtype=x.dtype)
    rowsum = torch.empty(_rows(x) if with_rowsum else 0, device=x.device, dtype=torch.float32)
    if x.numel():
        L = x.shape[-1]
        fam = K.FamilyConfig(alpha=alpha, theta=theta, power=power)
        K._norm_fwd_direct(x.view(-1, L), out.view(-1, L), fam, causal, rowsum if with_rowsum else None)
    return out, rowsum


@norm_fwd.register_fake
def _(x, alpha, theta, power, causal, with_rowsum):
    return (torch.empty(x.shape, device=x.device, dtype=x.dtype),
            torch.empty(_rows(x) if with_rowsum else 0, device=x.device, dtype=torch.float32))


@torch.library.custom_op(f"{NS}::norm_causal_bwd", mutates_args=(), device_types="cuda")
def norm_causal_bwd(x: Tensor, g: Tensor, rowsum: Tensor, alpha: float, theta: float, power: int) -> Tensor:
    x, g, rowsum = x.contiguous(), g.contiguous(), rowsum.contiguous()
    dx = torch.empty(x.shape, device=x.device, dtype=x.dtype)
    if x.numel():
        L = x.shape[-1]
        fam = K.FamilyConfig(alpha=alpha, theta=theta, power=power)
        K._norm_bwd_direct(x.view(-1, L), g.view(-1, L), rowsum, dx.view(-1, L), fam, True)
    return dx


@norm_causal_bwd.register_fake
def _(x, g, rowsum, alpha, theta, power):
    return torch.empty(x.shape, device=x.device, dtype=x.dtype)


# ------------------------------------------------------------------ flash attention


@torch.library.custom_op(f"{NS}::flash_fwd", mutates_args=(), device_types="cuda")
def flash_fwd(q: Tensor, k: Tensor, v: Tensor, scale: float, window_size: int,
              use_fast_sqrt: bool, with_residual: bool) -> tuple[Tensor, Tensor, Tensor]:
    q, k, v = K._flash_ready(q), K._flash_ready(k), K._flash_ready(v)
    o = torch.empty(q.shape, device=q.device, dtype=q.dtype)
    res = K._flash_fwd_direct(q, k, v, scale, window_size, use_fast_sqrt, o=o, with_residual=with_residual)
    return res if with_residual else (res[0], res[1], q.new_empty(0))


@flash_fwd.register_fake
def _(q, k, v, scale, window_size, use_fast_sqrt, with_residual):
    B, H, T, _ = q.shape
    return (torch.empty(q.shape, device=q.device, dtype=q.dtype),
            torch.empty(B, H, T, device=q.device, dtype=torch.float32),
            torch.empty(q.shape if with_residual else (0,), device=q.device, dtype=q.dtype))


@torch.library.custom_op(f"{NS}::flash_bwd", mutates_args=(), device_types="cuda")
def flash_bwd(q: Tensor, k: Tensor, v: Tensor, o: Tensor, o_lo: Tensor, do: Tensor, row_sums: Tensor, scale: float,
              window_size: int, use_fast_sqrt: bool, deterministic: bool) -> tuple[Tensor, Tensor, Tensor]:
    q, k, v, o = (K._flash_ready(t) for t in (q, k, v, o))
    return K._flash_bwd_direct(q, k, v, o, do, row_sums.contiguous(), scale, window_size, use_fast_sqrt,
                               o_lo=o_lo if o_lo.numel() else None, deterministic=deterministic)


@flash_bwd.register_fake
def _(q, k, v, o, o_lo, do, row_sums, scale, window_size, use_fast_sqrt, deterministic):
    return tuple(torch.empty(t.shape, device=q.device, dtype=q.dtype) for t in (q, k, v))


@torch.library.custom_op(f"{NS}::flash_fwd_chunk", mutates_args=(), device_types="cuda")
def flash_fwd_chunk(q: Tensor, k: Tensor, v: Tensor, q_offset: int, scale: float, window_size: int,
                    exact_math: bool, with_residual: bool) -> tuple[Tensor, Tensor, Tensor]:
    res = K._flash_fwd_chunk_direct(q, k, v, q_offset, scale, window_size, exact_math, with_residual)
    return res if with_residual else (res[0], res[1], q.new_empty(0))


@flash_fwd_chunk.register_fake
def _(q, k, v, q_offset, scale, window_size, exact_math, with_residual):
    B, H, T, _ = q.shape
    return (torch.empty(q.shape, device=q.device, dtype=q.dtype),
            torch.empty(B, H, T, device=q.device, dtype=torch.float32),
            torch.empty(q.shape if with_residual else (0,), device=q.device, dtype=q.dtype))


@torch.library.custom_op(f"{NS}::flash_bwd_chunk", mutates_args=(), device_types="cuda")
def flash_bwd_chunk(q: Tensor, k: Tensor, v: Tensor, o: Tensor, o_lo: Tensor, do: Tensor, row_sums: Tensor,
                    q_offset: int, scale: float, window_size: int, exact_math: bool,
                    deterministic: bool) -> tuple[Tensor, Tensor, Tensor]:
    return K._flash_bwd_chunk_direct(q, k, v, o, do, row_sums.contiguous(), q_offset, scale, window_size,
                                     exact_math, o_lo if o_lo.numel() else None, deterministic)


@flash_bwd_chunk.register_fake
def _(q, k, v, o, o_lo, do, row_sums, q_offset, scale, window_size, exact_math, deterministic):
    return tuple(torch.empty(t.shape, device=q.device, dtype=q.dtype) for t in (q, k, v))


@torch.library.custom_op(f"{NS}::rope_flash_fwd", mutates_args=(), device_types="cuda")
def rope_flash_fwd(q: Tensor, k: Tensor, v: Tensor, cos: Tensor, sin: Tensor, scale: float,
                   window_size: int) -> Tensor:
    return K._rope_flash_fwd_direct(q, k, v, cos, sin, scale, window_size)[0]


@rope_flash_fwd.register_fake
def _(q, k, v, cos, sin, scale, window_size):
    return torch.empty(q.shape, device=q.device, dtype=q.dtype)


@torch.library.custom_op(f"{NS}::out_proj", mutates_args=(), device_types="cuda")
def out_proj(a: Tensor, w: Tensor) -> Tensor:
    return K._out_proj_direct(a, w)


@out_proj.register_fake
def _(a, w):
    return torch.empty(a.shape[0], w.shape[1], device=a.device, dtype=a.dtype)


@torch.library.custom_op(f"{NS}::fp8_flash_fwd", mutates_args=(), device_types="cuda")
def fp8_flash_fwd(q: Tensor, k: Tensor, v: Tensor, scale: float, window_size: int) -> Tensor:
    return K._fp8_flash_fwd_direct(q, k, v, scale, window_size)


@fp8_flash_fwd.register_fake
def _(q, k, v, scale, window_size):
    return torch.empty(q.shape, device=q.device, dtype=torch.bfloat16)


@torch.library.custom_op(f"{NS}::paged_decode", mutates_args=(), device_types="cuda")
def paged_decode(q: Tensor, k_cache: Tensor, v_cache: Tensor, block_table: Tensor, context_lens: Tensor,
                 scale: float, block_size: int) -> Tensor:
    return K._paged_decode_direct(q, k_cache, v_cache, block_table, context_lens, scale, block_size)


@paged_decode.register_fake
def _(q, k_cache, v_cache, block_table, context_lens, scale, block_size):
    B, H, _, D = q.shape
    return torch.empty(B, H, D, device=q.device, dtype=torch.bfloat16)

"""CPU oracle for the smooth-attn hot path (TEST INFRASTRUCTURE ONLY).

This module restates, in numpy, the reference's eager PyTorch algorithms for
squareplus normalization and squareplus flash attention.  It is the checker
the parity tests, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline
leg compare the CUDA kernels against.  Nothing in the product package imports
it; the product path has no CPU fallback.

Parity pinning: every function here is checked against golden vectors that
were produced by running the reference's own eager functions
(``src/smooth_attn/kernels.py`` in NoSelection/smooth-attn) on seeded inputs;
see ``tests/golden/gen_golden.py`` and ``tests/test_oracle_golden.py``.

Reference citations (file:line inside NoSelection/smooth-attn):
  * activation      ``src/smooth_attn/kernels.py:1328-1329``
  * row-wise norm   ``src/smooth_attn/kernels.py:1332-1346``
  * causal norm     ``src/smooth_attn/kernels.py:1349-1365``
  * causal bwd      ``src/smooth_attn/kernels.py:679-743`` (the closed form the
                    fused kernel uses; equals autograd of the eager causal norm)
  * flash eager     ``src/smooth_attn/kernels.py:2053-2084``
  * flash bwd       ``src/smooth_attn/kernels.py:1680-1909`` (closed form)
  * paged decode    ``src/smooth_attn/kernels.py:2681-2829`` and the decode
                    reference of ``tests/test_paged_attention.py:78-109``
  * RoPE            ``src/smooth_attn/kernels.py:2093-2101`` (tables),
                    ``:2147-2159`` (rotation), ``tests/test_rope_proj.py:15-30``
  * RoPE + W_o      ``src/smooth_attn/kernels.py:2354-2370`` and
                    ``tests/test_rope_proj.py:118-150``
  * FP8 attention   ``src/smooth_attn/kernels.py:2498-2673`` (quantization
                    ``:2592-2601``)
  * EPS             ``src/smooth_attn/kernels.py:57``

All arithmetic is float32 unless ``acc=np.float64`` is requested, matching the
reference's fp32 eager path.
"""

from __future__ import annotations

import math

import numpy as np

EPS = 1e-12  # kernels.py:57
SUPPORTED_POWERS = (1, 2, 3)  # kernels.py:24


def _as_f(x, acc):
    return np.asarray(x, dtype=acc)


def squareplus(arg, acc=np.float32):
    """sp(a) = 0.5 * (a + sqrt(a*a + 4))   (kernels.py:1328-1329)."""
    arg = _as_f(arg, acc)
    return acc(0.5) * (arg + np.sqrt(arg * arg + acc(4.0)))


def family_activation(x, alpha, theta, power, acc=np.float32):
    """y = sp(alpha*(x-theta))**power   (kernels.py:1340-1344)."""
    if power not in SUPPORTED_POWERS:
        raise ValueError(f"power must be one of {SUPPORTED_POWERS}, got {power}")
    x = _as_f(x, acc)
    y = squareplus(acc(alpha) * (x - acc(theta)), acc)
    if power == 2:
        y = y * y
    elif power == 3:
        y = y * y * y
    return y


def softplus_norm(x, alpha=2.0, theta=0.5, power=2, acc=np.float32):
    """Row-wise normalization over the last axis (kernels.py:1332-1346)."""
    y = family_activation(x, alpha, theta, power, acc)
    return y / (y.sum(axis=-1, keepdims=True) + acc(EPS))


def causal_mask(L):
    """True where column j is visible to row q, i.e. j <= q (kernels.py:226-233 masks j > q)."""
    return np.tril(np.ones((L, L), dtype=bool))


def softplus_norm_causal(x, alpha=2.0, theta=0.5, power=2, acc=np.float32, return_rowsum=False):
    """Causal normalization over the last two (square) axes (kernels.py:1349-1365).

    Returns ``out`` (and the normalizer ``S = sum_vis y + EPS`` per row when
    ``return_rowsum``), with exact zeros above the diagonal.
    """
    x = _as_f(x, acc)
    L = x.shape[-1]
    if x.shape[-2] != L:
        raise ValueError("causal attention expects square score matrices on the last two dims")
    y = family_activation(x, alpha, theta, power, acc)
    y = np.where(causal_mask(L), y, acc(0.0))
    s = y.sum(axis=-1, keepdims=True) + acc(EPS)
    out = y / s
    if return_rowsum:
        return out, s[..., 0]
    return out


def softplus_norm_causal_rows(x_rows, q0, alpha=2.0, theta=0.5, power=2, acc=np.float32):
    """Causal normalization of a block of rows of one [L, L] score matrix.

    x_rows: [n, L] holding query positions q0 .. q0+n-1; column j is visible
    to query q iff j <= q (the row test ``q_pos = row % L`` of kernels.py:585).
    """
    x_rows = _as_f(x_rows, acc)
    n, L = x_rows.shape
    q = np.arange(q0, q0 + n)[:, None]
    vis = np.arange(L)[None, :] <= q
    y = np.where(vis, family_activation(x_rows, alpha, theta, power, acc), acc(0.0))
    return y / (y.sum(axis=-1, keepdims=True) + acc(EPS))


def softplus_norm_causal_bwd(x, g, alpha=2.0, theta=0.5, power=2, acc=np.float32):
    """Gradient of ``sum(softplus_norm_causal(x) * g)`` w.r.t. x.

    Closed form used by the reference's fused backward (kernels.py:710-743):
      a = alpha (x - theta); sp = 0.5 (a + sqrt(a^2+4)); sp' = 0.5 (1 + a/sqrt(a^2+4))
      dy/dx = alpha * power * sp^(power-1) * sp'
      p = y / S;  dX = (dy/dx / S) * (g - sum_k g_k p_k); zero above the diagonal.
    """
    x = _as_f(x, acc)
    g = _as_f(g, acc)
    L = x.shape[-1]
    mask = causal_mask(L)
    a = acc(alpha) * (x - acc(theta))
    r = np.sqrt(a * a + acc(4.0))
    sp = acc(0.5) * (a + r)
    spp = acc(0.5) * (acc(1.0) + a / r)
    if power == 1:
        y = sp
        dydx = acc(alpha) * spp
    elif power == 2:
        y = sp * sp
        dydx = acc(alpha) * acc(2.0) * sp * spp
    elif power == 3:
        y = sp * sp * sp
        dydx = acc(alpha) * acc(3.0) * sp * sp * spp
    else:
        raise ValueError(f"power must be one of {SUPPORTED_POWERS}, got {power}")
    y = np.where(mask, y, acc(0.0))
    g = np.where(mask, g, acc(0.0))
    s = y.sum(axis=-1, keepdims=True) + acc(EPS)
    p = y / s
    dot = (g * p).sum(axis=-1, keepdims=True)
    dx = (dydx / s) * (g - dot)
    return np.where(mask, dx, acc(0.0))


def softplus_norm_bwd(x, g, alpha=2.0, theta=0.5, power=2, acc=np.float32):
    """Row-wise (non-causal) analogue of :func:`softplus_norm_causal_bwd`."""
    x = _as_f(x, acc)
    g = _as_f(g, acc)
    a = acc(alpha) * (x - acc(theta))
    r = np.sqrt(a * a + acc(4.0))
    sp = acc(0.5) * (a + r)
    spp = acc(0.5) * (acc(1.0) + a / r)
    y = sp ** power
    dydx = acc(alpha) * acc(power) * sp ** (power - 1) * spp
    s = y.sum(axis=-1, keepdims=True) + acc(EPS)
    dot = (g * (y / s)).sum(axis=-1, keepdims=True)
    return (dydx / s) * (g - dot)


def _expand_kv(k, n_q_heads):
    """GQA: query head h reads kv head h // (H_q // H_kv)  (kernels.py:1568, 2058-2062)."""
    h_kv = k.shape[1]
    if h_kv == n_q_heads:
        return k
    return np.repeat(k, n_q_heads // h_kv, axis=1)


def _flash_mask(T, window_size):
    m = causal_mask(T)
    if window_size > 0:
        pos = np.arange(T)
        m &= (pos[:, None] - pos[None, :]) < window_size  # kernels.py:2076-2079
    return m


def chunk_flash_attention(q, k, v, q_offset, scale=None, window_size=0, acc=np.float32):
    """Squareplus attention of a block of Tq queries at global positions
    q_offset .. q_offset+Tq-1 over keys 0 .. Tk-1 (same causal / window rule
    as kernels.py:2053-2084 in global positions).  With q_offset = 0 and
    Tq = Tk it is sp2norm_flash_attention; a sequence split into query
    chunks, each attending to the key prefix, reproduces the whole."""
    q = _as_f(q, acc)
    k = _expand_kv(_as_f(k, acc), q.shape[1])
    v = _expand_kv(_as_f(v, acc), q.shape[1])
    Tq, Tk, D = q.shape[-2], k.shape[-2], q.shape[-1]
    if scale is None:
        scale = 1.0 / math.sqrt(D)
    qp = np.arange(Tq)[:, None] + q_offset
    kp = np.arange(Tk)[None, :]
    m = kp <= qp
    if window_size > 0:
        m &= (qp - kp) < window_size
    s = np.matmul(q, np.swapaxes(k, -1, -2)) * acc(scale)
    a = acc(2.0) * s - acc(1.0)
    sp = acc(0.5) * (a + np.sqrt(a * a + acc(4.0)))
    y = np.where(m, sp * sp, acc(0.0))
    r = y.sum(axis=-1, keepdims=True) + acc(EPS)
    return np.matmul(y / r, v)


def sp2norm_flash_attention(q, k, v, scale=None, window_size=0, acc=np.float32, return_rowsum=False):
    """Eager squareplus attention (kernels.py:2053-2084).

    q: [B, H_q, T, D]; k, v: [B, H_kv, T, D].  Returns o [B, H_q, T, D] in ``acc``
    (and the normalizer R = sum_vis y + EPS, [B, H_q, T], when ``return_rowsum``).
    """
    q = _as_f(q, acc)
    k = _expand_kv(_as_f(k, acc), q.shape[1])
    v = _expand_kv(_as_f(v, acc), q.shape[1])
    T, D = q.shape[-2], q.shape[-1]
    if scale is None:
        scale = 1.0 / math.sqrt(D)
    s = np.matmul(q, np.swapaxes(k, -1, -2)) * acc(scale)
    a = acc(2.0) * s - acc(1.0)
    sp = acc(0.5) * (a + np.sqrt(a * a + acc(4.0)))
    y = sp * sp
    y = np.where(_flash_mask(T, window_size), y, acc(0.0))
    r = y.sum(axis=-1, keepdims=True) + acc(EPS)
    o = np.matmul(y / r, v)
    if return_rowsum:
        return o, r[..., 0]
    return o


def _flash_bwd_core(q, k_in, v_in, do, mask, scale, acc, emulate):
    """Closed-form flash backward over a boolean visibility mask [Tq, Tk].

    emulate=False: the reference's exact algebra in ``acc`` (kernels.py:1723-1909).
    emulate=True: the same algebra with the 16-bit rounding points of the
    B200 kernels (test infrastructure for telling operand rounding apart from
    defects): the forward's normalizer and output use y rounded to bf16
    (P.V multiplies bf16 y, as the reference does at kernels.py:1621, and the
    normalizer sums those same rounded y), dS is rounded to bf16 before the dQ
    / dK products and P = y / R before the dV product (the reference's
    rounding points, kernels.py:1776, 1894)."""
    B, Hq, Tq, D = q.shape
    Hkv, Tk = k_in.shape[1], k_in.shape[2]
    k = _expand_kv(k_in, Hq)
    v = _expand_kv(v_in, Hq)
    s = np.matmul(q, np.swapaxes(k, -1, -2)) * acc(scale)
    a = acc(2.0) * s - acc(1.0)
    rt = np.sqrt(a * a + acc(4.0))
    sp = acc(0.5) * (a + rt)
    spp = acc(0.5) * (acc(1.0) + a / rt)
    y = np.where(mask, sp * sp, acc(0.0))
    if emulate:
        yh = round_bf16(y).astype(acc)
        r = yh.sum(axis=-1, keepdims=True) + acc(EPS)
        o = np.matmul(yh / r, v)
    else:
        r = y.sum(axis=-1, keepdims=True) + acc(EPS)
        o = np.matmul(y / r, v)
    p = y / r
    delta = (do * o).sum(axis=-1, keepdims=True)
    dp = np.matmul(do, np.swapaxes(v, -1, -2))
    dy = np.where(mask, (dp - delta) / r, acc(0.0))
    ds = dy * acc(4.0) * sp * spp * acc(scale)
    if emulate:
        ds = round_bf16(ds).astype(acc)
        p = round_bf16(p).astype(acc)
    dq = np.matmul(ds, k)
    dk = np.matmul(np.swapaxes(ds, -1, -2), q)
    dv = np.matmul(np.swapaxes(p, -1, -2), do)
    if Hkv != Hq:
        g = Hq // Hkv
        dk = dk.reshape(B, Hkv, g, Tk, D).sum(axis=2)
        dv = dv.reshape(B, Hkv, g, Tk, D).sum(axis=2)
    return dq, dk, dv


def sp2norm_flash_attention_bwd(q, k, v, do, scale=None, window_size=0, acc=np.float32, emulate=False):
    """Gradients (dq, dk, dv) of ``sum(sp2norm_flash_attention(q,k,v) * do)``.

    Closed form of the reference's fused backward (kernels.py:1723-1909):
      delta = rowsum(dO * O); dP = dO V^T; dY = (dP - delta)/R;
      dS = dY * 4 sp sp' * scale;  dQ = dS K;  dK = dS^T Q;  dV = (y/R)^T dO
    GQA gradients of K/V are summed over the query heads of each group.
    ``emulate=True`` applies the 16-bit rounding points (see _flash_bwd_core).
    """
    q = _as_f(q, acc)
    T, D = q.shape[-2], q.shape[-1]
    if scale is None:
        scale = 1.0 / math.sqrt(D)
    return _flash_bwd_core(q, _as_f(k, acc), _as_f(v, acc), _as_f(do, acc), _flash_mask(T, window_size), scale,
                           acc, emulate)


def chunk_flash_attention_bwd(q, k, v, do, q_offset, scale=None, window_size=0, acc=np.float32, emulate=False):
    """Gradients of ``sum(chunk_flash_attention(q, k, v, q_offset) * do)``:
    dq for the query block, dk / dv for keys 0 .. Tk-1 (this block's
    contribution).  Same closed form as sp2norm_flash_attention_bwd with the
    mask in global positions."""
    q = _as_f(q, acc)
    Tq, D = q.shape[-2], q.shape[-1]
    Tk = np.shape(k)[-2]
    if scale is None:
        scale = 1.0 / math.sqrt(D)
    qp = np.arange(Tq)[:, None] + q_offset
    kp = np.arange(Tk)[None, :]
    mask = kp <= qp
    if window_size > 0:
        mask &= (qp - kp) < window_size
    return _flash_bwd_core(q, _as_f(k, acc), _as_f(v, acc), _as_f(do, acc), mask, scale, acc, emulate)


def paged_decode_attention(q, k_cache, v_cache, block_table, context_lens, scale=None, acc=np.float32):
    """Decode attention over a paged KV cache (kernels.py:2681-2829 and the
    reference's decode reference, tests/test_paged_attention.py:78-109).

    q: [B, H_q, 1, D]; k_cache, v_cache: [num_blocks, H_kv, block_size, D];
    block_table: [B, max_blocks] physical page of each logical page;
    context_lens: [B].  The single query of sequence b sees all of its
    context_lens[b] tokens (no causal mask).  Returns [B, H_q, D] in ``acc``:
      y = squareplus(2 s - 1)^2 with s = (q . k) * scale,
      o = sum(y v) / (sum(y) + 1e-12).
    """
    q = _as_f(q, acc)
    kc = _as_f(k_cache, acc)
    vc = _as_f(v_cache, acc)
    B, Hq, _, D = q.shape
    Hkv, bs = kc.shape[1], kc.shape[2]
    G = Hq // Hkv
    if scale is None:
        scale = 1.0 / math.sqrt(D)
    out = np.zeros((B, Hq, D), dtype=acc)
    for b in range(B):
        n = int(context_lens[b])
        pages = [int(block_table[b, i]) for i in range((n + bs - 1) // bs)]
        if not pages:
            continue
        k = np.concatenate([kc[pg] for pg in pages], axis=1)[:, :n]  # [Hkv, n, D]
        v = np.concatenate([vc[pg] for pg in pages], axis=1)[:, :n]
        for h in range(Hq):
            s = (k[h // G] @ q[b, h, 0]) * acc(scale)
            a = acc(2.0) * s - acc(1.0)
            sp = acc(0.5) * (a + np.sqrt(a * a + acc(4.0)))
            y = sp * sp
            out[b, h] = (y @ v[h // G]) / (y.sum() + acc(EPS))
    return out


def round_bf16(x):
    """Round float32 values to the nearest bfloat16 (ties to even), returned
    as float32 (what ``tensor.to(torch.bfloat16)`` does)."""
    u = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32)
    r = ((u + np.uint32(0x7FFF) + ((u >> np.uint32(16)) & np.uint32(1))) & np.uint32(0xFFFF0000)).astype(np.uint32)
    nan = np.isnan(np.asarray(x, dtype=np.float32))
    out = r.view(np.float32).copy()
    out[nan] = np.nan
    return out


def rope_tables(dim, seq_len, base=10000.0):
    """cos / sin tables [T, D/2] (kernels.py:2093-2101), float32."""
    inv_freq = (1.0 / (np.float32(base) ** (np.arange(0, dim, 2, dtype=np.float32) / np.float32(dim)))).astype(np.float32)
    t = np.arange(seq_len, dtype=np.float32)
    freqs = np.outer(t, inv_freq).astype(np.float32)
    return np.cos(freqs).astype(np.float32), np.sin(freqs).astype(np.float32)


def rope_rotate(x, cos, sin, to_bf16=True):
    """Rotate-half RoPE (tests/test_rope_proj.py:15-30, kernels.py:2147-2159):
    [x1 c - x2 s, x2 c + x1 s] in float32 with every product and sum rounded,
    then rounded to bf16 as the reference does before its QK^T dot."""
    x = np.asarray(x, dtype=np.float32)
    T, D = x.shape[-2], x.shape[-1]
    c = np.asarray(cos, dtype=np.float32)[:T]
    s = np.asarray(sin, dtype=np.float32)[:T]
    x1, x2 = x[..., : D // 2], x[..., D // 2:]
    out = np.concatenate([x1 * c - x2 * s, x2 * c + x1 * s], axis=-1).astype(np.float32)
    return round_bf16(out) if to_bf16 else out


def rope_flash_attention(q, k, v, cos, sin, scale=None, window_size=0):
    """RoPE on q and k, then squareplus flash attention
    (sp2norm_rope_flash_attention, kernels.py:2373-2430)."""
    return sp2norm_flash_attention(rope_rotate(q, cos, sin), rope_rotate(k, cos, sin), v, scale=scale,
                                   window_size=window_size)


def rope_flash_attention_proj(q, k, v, w_o, cos, sin, scale=None, window_size=0):
    """RoPE attention then the per-head output projection summed over heads
    (sp2norm_rope_flash_attention_proj, kernels.py:2433-2490): out[b, t] =
    sum_h bf16(o[b, h, t]) @ w_o[h], accumulated in float32."""
    o = round_bf16(rope_flash_attention(q, k, v, cos, sin, scale=scale, window_size=window_size))
    return np.einsum("bhtd,hdm->btm", o, np.asarray(w_o, dtype=np.float32)).astype(np.float32)


E4M3_MAX = 448.0  # kernels.py:2596


def round_e4m3(x):
    """Round float32 values (|x| <= 448) to the nearest E4M3 value, ties to
    even (3 mantissa bits, exponent bias 7, subnormal quantum 2^-9)."""
    x = np.asarray(x, dtype=np.float64)
    ax = np.abs(x)
    e = np.floor(np.log2(np.maximum(ax, 2.0 ** -9)))
    e = np.maximum(e, -6.0)  # below 2^-6 the spacing stays 2^-9
    q = 2.0 ** (e - 3)
    return (np.round(x / q) * q).astype(np.float32)


def quantize_fp8(x):
    """Per-tensor E4M3 quantization (kernels.py:2592-2601):
    scale = max(amax / 448, 1e-12) in float32, x8 = e4m3(clamp(x / scale)).
    Returns (x8 as float32 values, scale)."""
    x = np.asarray(x, dtype=np.float32)
    amax = np.float32(np.abs(x).max()) if x.size else np.float32(0)
    scale = np.maximum(np.float32(amax / np.float32(E4M3_MAX)), np.float32(1e-12)).astype(np.float32)
    xs = np.clip((x / scale).astype(np.float32), -E4M3_MAX, E4M3_MAX)
    return round_e4m3(xs), float(scale)


def fp8_flash_attention(q, k, v, scale=None, window_size=0):
    """FP8 squareplus attention forward (kernels.py:2498-2589, :2630-2673):
    scores = (q8 . k8) * (q_scale k_scale scale); y in float32; P = bf16(y);
    o = (P v8) v_scale / (sum y + EPS)."""
    q8, qs = quantize_fp8(q)
    k8, ks = quantize_fp8(k)
    v8, vs = quantize_fp8(v)
    T, D = q8.shape[-2], q8.shape[-1]
    if scale is None:
        scale = 1.0 / math.sqrt(D)
    sscale = np.float32(qs * ks * scale)  # the reference forms the product in double
    k8 = _expand_kv(k8, q8.shape[1])
    v8 = _expand_kv(v8, q8.shape[1])
    s = np.matmul(q8, np.swapaxes(k8, -1, -2)).astype(np.float32) * sscale
    a = s + s - np.float32(1.0)
    sp = np.float32(0.5) * (a + np.sqrt(a * a + np.float32(4.0)))
    y = np.where(_flash_mask(T, window_size), sp * sp, np.float32(0.0)).astype(np.float32)
    r = y.sum(axis=-1, keepdims=True) + np.float32(EPS)
    o = np.matmul(round_bf16(y), v8).astype(np.float32) * np.float32(vs)
    return o / r


def flash_flops(B, H, T, D, window_size=0, bwd=False):
    """Algorithmic FLOPs of causal squareplus attention.

    Visible (q,k) pairs are counted exactly (causal triangle, optionally clipped
    by the sliding window); forward = 2 GEMMs (QK^T, PV), backward = 5 GEMMs
    (QK^T recompute, dO V^T, dV, dK, dQ), each 2*D flops per visible pair.
    """
    if window_size and window_size < T:
        w = window_size
        vis = w * (w + 1) // 2 + (T - w) * w
    else:
        vis = T * (T + 1) // 2
    gemms = 5 if bwd else 2
    return 2 * D * vis * B * H * gemms

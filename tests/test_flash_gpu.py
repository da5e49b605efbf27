"""Parity of the tcgen05 fused squareplus attention (forward + backward) with
the numpy oracle and the committed golden vectors.  Mirrors the reference's
``tests/test_training_api.py:81-318`` (MHA, exact_math, non-contiguous
[B,T,H,D] inputs, GQA, sliding windows) plus head dims 32/64/128, fp16,
ragged sequence lengths and the BASELINE-size configs."""

from pathlib import Path

import numpy as np
import pytest
import torch

import smooth_attn as sa
from oracle import sa_oracle as O
from tests._util import assert_close, check_bf16_grads, np32, randn

pytestmark = pytest.mark.gpu
CUDA = "cuda"
G = np.load(Path(__file__).parent / "golden" / "golden.npz")

# bf16 outputs and gradients vs the fp32 oracle on the same (bf16-rounded)
# inputs, at the north-star tolerance: 2e-2 relative / 1e-2 absolute.  The
# kernel rounds the unnormalized y to bf16 before P.V like the reference
# (kernels.py:1621) and dS / P to bf16 before their MMAs (:1776, :1894); the
# backward forms delta = rowsum(dO * o) from the forward's fp32 output
# (o + o_lo).  Gradients are held to the tolerance element by element, with
# the one exception check_bf16_grads spells out (elements that the bf16
# operand rounding alone moves by more than half the tolerance).
FWD_TOL = dict(rtol=2e-2, atol=1e-2)
BWD_TOL = dict(rtol=2e-2, atol=1e-2)


@pytest.fixture(autouse=True)
def _need_cuda():
    if not torch.cuda.is_available():
        pytest.skip("CUDA required")


def _qkv(B, Hq, Hkv, T, D, seed, dtype=torch.bfloat16):
    q = randn((B, Hq, T, D), seed, dtype, CUDA)
    k = randn((B, Hkv, T, D), seed + 1, dtype, CUDA)
    v = randn((B, Hkv, T, D), seed + 2, dtype, CUDA)
    return q, k, v


def _fwd_ref(q, k, v, window=0):
    return O.sp2norm_flash_attention(np32(q), np32(k), np32(v), window_size=window, return_rowsum=True)


@pytest.mark.parametrize("D", [32, 64, 128])
@pytest.mark.parametrize("T", [1, 7, 64, 127, 128, 129, 300, 512])
def test_flash_fwd_matches_oracle(D, T):
    q, k, v = _qkv(2, 3, 3, T, D, seed=T + D)
    o = sa.sp2norm_flash_attention(q, k, v)
    ref, _ = _fwd_ref(q, k, v)
    assert not torch.isnan(o).any()
    assert_close(np32(o), ref, **FWD_TOL)


@pytest.mark.parametrize("T", [64, 128, 256, 512])
def test_flash_attention_matches_eager_reference_case(T):
    """reference tests/test_training_api.py:81-93"""
    q, k, v = _qkv(2, 4, 4, T, 32, seed=T)
    out_flash = sa.sp2norm_flash_attention(q, k, v)
    out_eager = sa.sp2norm_flash_attention_eager(q, k, v)
    torch.testing.assert_close(out_flash.float(), out_eager.float(), atol=1e-2, rtol=2e-2)


def test_flash_rowsum_saved():
    q, k, v = _qkv(1, 2, 2, 200, 64, seed=5)
    from smooth_attn.kernels import _sp2norm_flash_fwd

    o, rs = _sp2norm_flash_fwd(q, k, v, 1.0 / 8.0)
    _, ref_rs = _fwd_ref(q, k, v)
    # the kernel's normalizer sums the bf16-rounded y that P.V uses (the
    # reference sums the unrounded y): each term moves by at most one bf16
    # unit roundoff (2^-9), so the sums agree to 2 x 2^-9 relative
    assert_close(rs.cpu().numpy(), ref_rs, rtol=4e-3, atol=0)


@pytest.mark.parametrize("exact", [False, True])
def test_flash_exact_math(exact):
    q, k, v = _qkv(2, 4, 4, 256, 32, seed=9)
    o = sa.sp2norm_flash_attention(q, k, v, exact_math=exact)
    assert_close(np32(o), _fwd_ref(q, k, v)[0], **FWD_TOL)


def test_flash_fp16():
    q, k, v = _qkv(1, 2, 2, 192, 64, seed=3, dtype=torch.float16)
    o = sa.sp2norm_flash_attention(q, k, v)
    assert o.dtype == torch.float16
    assert_close(np32(o), _fwd_ref(q, k, v)[0], **FWD_TOL)


@pytest.mark.parametrize(("Hq", "Hkv"), [(8, 2), (8, 4), (4, 1)])
@pytest.mark.parametrize("T", [64, 128, 256])
def test_flash_gqa_fwd(Hq, Hkv, T):
    q, k, v = _qkv(2, Hq, Hkv, T, 32, seed=Hq * Hkv + T)
    o = sa.sp2norm_flash_attention(q, k, v)
    assert o.shape == q.shape
    assert_close(np32(o), _fwd_ref(q, k, v)[0], **FWD_TOL)


@pytest.mark.parametrize("W", [1, 32, 64, 100, 128, 129, 1000])
@pytest.mark.parametrize("T", [64, 256, 333])
def test_flash_window_fwd(W, T):
    q, k, v = _qkv(1, 2, 2, T, 64, seed=W + T)
    o = sa.sp2norm_flash_attention(q, k, v, window_size=W)
    assert_close(np32(o), _fwd_ref(q, k, v, W)[0], **FWD_TOL)


def test_flash_noncontiguous_fwd():
    """reference tests/test_training_api.py:110-125: [B,T,H,D].transpose(1,2) + GQA + window."""
    B, T, Hq, Hkv, D, W = 2, 128, 8, 2, 32, 32
    q = randn((B, T, Hq, D), 1, torch.bfloat16, CUDA).transpose(1, 2)
    k = randn((B, T, Hkv, D), 2, torch.bfloat16, CUDA).transpose(1, 2)
    v = randn((B, T, Hkv, D), 3, torch.bfloat16, CUDA).transpose(1, 2)
    assert not q.is_contiguous()
    o = sa.sp2norm_flash_attention(q, k, v, window_size=W)
    assert_close(np32(o), _fwd_ref(q, k, v, W)[0], **FWD_TOL)


@pytest.mark.parametrize("name", sorted({k.split("/")[0] for k in G.files if k.startswith("f_")}))
def test_flash_golden_fwd(name):
    q, k, v = (torch.from_numpy(G[f"{name}/{s}"]).to(torch.bfloat16).to(CUDA) for s in ("q", "k", "v"))
    w = int(G[f"{name}/window"])
    o = sa.sp2norm_flash_attention(q, k, v, window_size=w)
    assert_close(np32(o), G[f"{name}/o"], **FWD_TOL)


def test_flash_rejects_unsupported():
    q, k, v = _qkv(1, 1, 1, 16, 32, seed=1)
    with pytest.raises(ValueError):
        sa.sp2norm_flash_attention(q.float(), k.float(), v.float())
    q2 = randn((1, 1, 16, 48), 1, torch.bfloat16, CUDA)
    with pytest.raises(ValueError):
        sa.sp2norm_flash_attention(q2, q2, q2)


def test_flash_fwd_baseline_config4_slices():
    """[4,32,4096,128]: sampled heads equal the oracle; a rerun is bitwise identical."""
    q, k, v = _qkv(4, 32, 32, 4096, 128, seed=44)
    o = sa.sp2norm_flash_attention(q, k, v)
    for b, h in ((0, 0), (3, 31)):
        ref = O.sp2norm_flash_attention(np32(q[b:b + 1, h:h + 1]), np32(k[b:b + 1, h:h + 1]), np32(v[b:b + 1, h:h + 1]))
        assert_close(np32(o[b:b + 1, h:h + 1]), ref, **FWD_TOL)
    o2 = sa.sp2norm_flash_attention(q, k, v)
    assert torch.equal(o, o2)


def test_zz_flash_no_device_timeouts():
    from smooth_attn import _lib

    assert _lib.load().sa_device_status(1) == _lib.SA_OK


# ---- backward --------------------------------------------------------------


def _bwd_case(B, Hq, Hkv, T, D, W=0, seed=0, exact=False, dtype=torch.bfloat16, noncontig=False):
    if noncontig:
        q = randn((B, T, Hq, D), seed, dtype, CUDA).transpose(1, 2)
        k = randn((B, T, Hkv, D), seed + 1, dtype, CUDA).transpose(1, 2)
        v = randn((B, T, Hkv, D), seed + 2, dtype, CUDA).transpose(1, 2)
    else:
        q, k, v = _qkv(B, Hq, Hkv, T, D, seed, dtype)
    q, k, v = (t.detach().requires_grad_(True) for t in (q, k, v))
    do = randn((B, Hq, T, D), seed + 3, torch.float32, CUDA)
    o = sa.sp2norm_flash_attention(q, k, v, window_size=W, exact_math=exact)
    (o.float() * do).sum().backward()
    _check_grads((q.grad, k.grad, v.grad), q, k, v, do.to(dtype), window=W, dtype=dtype)


def _check_grads(got, q, k, v, do, window=0, dtype=torch.bfloat16):
    args = (np32(q), np32(k), np32(v), np32(do))
    ref = O.sp2norm_flash_attention_bwd(*args, window_size=window, acc=np.float64)
    emu = O.sp2norm_flash_attention_bwd(*args, window_size=window, emulate=True)
    for g, r, m in zip(got, ref, emu):
        assert g.dtype == dtype and g.shape == r.shape
        assert torch.isfinite(g.float()).all()
        check_bf16_grads(np32(g), r, m, **BWD_TOL)


@pytest.mark.parametrize("D", [32, 64, 128])
@pytest.mark.parametrize("T", [1, 5, 64, 128, 129, 257])
def test_flash_bwd_matches_oracle(D, T):
    _bwd_case(1, 2, 2, T, D, seed=T * 7 + D)


def test_flash_backward_reference_case():
    """reference tests/test_training_api.py:128-154 (eager softplus-norm on explicit scores)."""
    B, H, T, D = 1, 2, 64, 32
    scale = 1.0 / (D ** 0.5)
    q, k, v = (t.requires_grad_(True) for t in _qkv(B, H, H, T, D, seed=21))
    upstream = randn((B, H, T, D), 24, torch.float32, CUDA)
    (sa.sp2norm_flash_attention(q, k, v).float() * upstream).sum().backward()
    qr, kr, vr = (t.detach().clone().float().requires_grad_(True) for t in (q, k, v))
    attn = sa.softplus_norm_causal_eager(torch.matmul(qr, kr.transpose(-2, -1)) * scale)
    (torch.matmul(attn, vr) * upstream).sum().backward()
    emu = O.sp2norm_flash_attention_bwd(np32(q), np32(k), np32(v), np32(upstream), emulate=True)
    for got, ref, m in zip((q.grad, k.grad, v.grad), (qr.grad, kr.grad, vr.grad), emu):
        check_bf16_grads(np32(got), np32(ref), m, **BWD_TOL)


def test_flash_bwd_exact_math():
    _bwd_case(1, 2, 2, 64, 32, seed=31, exact=True)


@pytest.mark.parametrize(("Hq", "Hkv"), [(8, 2), (8, 4), (4, 1)])
def test_flash_bwd_gqa(Hq, Hkv):
    _bwd_case(1, Hq, Hkv, 64, 32, seed=40 + Hq + Hkv)
    _bwd_case(1, Hq, Hkv, 200, 64, seed=50 + Hq + Hkv)


@pytest.mark.parametrize("W", [32, 64, 130])
def test_flash_bwd_window(W):
    _bwd_case(1, 2, 2, 128, 32, W=W, seed=60 + W)
    _bwd_case(1, 2, 2, 300, 128, W=W, seed=70 + W)


def test_flash_bwd_gqa_window_noncontiguous():
    _bwd_case(1, 8, 2, 64, 32, W=32, seed=80)
    _bwd_case(1, 8, 2, 64, 32, W=32, seed=81, noncontig=True)


def test_flash_bwd_fp16():
    _bwd_case(1, 2, 2, 160, 64, seed=90, dtype=torch.float16)


@pytest.mark.parametrize("name", sorted({k.split("/")[0] for k in G.files if k.startswith("f_")}))
def test_flash_golden_bwd(name):
    q, k, v = (torch.from_numpy(G[f"{name}/{s}"]).to(torch.bfloat16).to(CUDA).requires_grad_(True)
               for s in ("q", "k", "v"))
    do = torch.from_numpy(G[f"{name}/do"]).to(CUDA)
    w = int(G[f"{name}/window"])
    (sa.sp2norm_flash_attention(q, k, v, window_size=w).float() * do).sum().backward()
    emu = O.sp2norm_flash_attention_bwd(np32(q), np32(k), np32(v), np32(do.to(torch.bfloat16)), window_size=w,
                                        emulate=True)
    for t, s, m in zip((q, k, v), ("dq", "dk", "dv"), emu):
        check_bf16_grads(np32(t.grad), G[f"{name}/{s}"], m, **BWD_TOL)


def test_flash_bwd_baseline_config4_slices():
    """[4,32,4096,128] fwd+bwd: sampled heads equal the oracle."""
    B, H, T, D = 4, 32, 4096, 128
    q, k, v = (t.requires_grad_(True) for t in _qkv(B, H, H, T, D, seed=444))
    do = randn((B, H, T, D), 448, torch.bfloat16, CUDA)
    sa.sp2norm_flash_attention(q, k, v).backward(do)
    for b, h in ((0, 5), (3, 31)):
        sl = (slice(b, b + 1), slice(h, h + 1))
        _check_grads((q.grad[sl], k.grad[sl], v.grad[sl]), q[sl], k[sl], v[sl], do[sl])


def test_zzz_flash_bwd_no_device_timeouts():
    from smooth_attn import _lib

    assert _lib.load().sa_device_status(1) == _lib.SA_OK


# ---- residual output and large grids -------------------------------------------


def test_flash_residual_is_rounding_of_fp32_output():
    """o_lo carries the part of the fp32 output that the bf16 o rounded away:
    |o_lo| <= half an ulp of o, and o + o_lo is closer to the oracle than o."""
    from smooth_attn.kernels import _sp2norm_flash_fwd

    q, k, v = _qkv(1, 4, 2, 300, 128, seed=17)
    o, rs, lo = _sp2norm_flash_fwd(q, k, v, 1.0 / 128 ** 0.5, with_residual=True)
    o0, _ = _sp2norm_flash_fwd(q, k, v, 1.0 / 128 ** 0.5)
    assert torch.equal(o, o0)  # the residual does not change o
    of, lf = o.float(), lo.float()
    assert (lf.abs() <= of.abs() * 2.0 ** -8 + 1e-30).all()
    ref, _ = _fwd_ref(q, k, v)
    err_hi = np.abs(np32(o) - ref).mean()
    err_hl = np.abs(np32(of + lf) - ref).mean()
    assert err_hl < err_hi


def test_flash_more_than_65535_heads():
    """B * H above the old 65535 grid limit: fwd and bwd run and sampled heads match."""
    B, H, T, D = 2, 33000, 5, 32
    q, k, v = (t.requires_grad_(True) for t in _qkv(B, H, H, T, D, seed=65))
    do = randn((B, H, T, D), 66, torch.bfloat16, CUDA)
    o = sa.sp2norm_flash_attention(q, k, v)
    o.backward(do)
    for b, h in ((0, 0), (1, 32999), (1, 16500)):
        sl = (slice(b, b + 1), slice(h, h + 1))
        ref = O.sp2norm_flash_attention(np32(q[sl]), np32(k[sl]), np32(v[sl]))
        assert_close(np32(o[sl]), ref, **FWD_TOL)
        _check_grads((q.grad[sl], k.grad[sl], v.grad[sl]), q[sl], k[sl], v[sl], do[sl])


# ---- deterministic dQ (query-major kernel) -----------------------------------


def _grads(q, k, v, do, W=0, det=None):
    q, k, v = (t.detach().requires_grad_(True) for t in (q, k, v))
    o = sa.sp2norm_flash_attention(q, k, v, window_size=W, deterministic=det)
    o.backward(do)
    return q.grad, k.grad, v.grad


@pytest.mark.parametrize(("Hq", "Hkv", "T", "D", "W"), [(2, 2, 1, 32, 0), (2, 2, 129, 64, 0), (4, 2, 300, 128, 0),
                                                        (8, 2, 256, 32, 64), (2, 1, 1024, 128, 0),
                                                        (2, 2, 333, 128, 100)])
def test_flash_bwd_deterministic_matches_oracle(Hq, Hkv, T, D, W):
    q, k, v = _qkv(1, Hq, Hkv, T, D, seed=T + D + Hq)
    do = randn((1, Hq, T, D), T + 5, torch.bfloat16, CUDA)
    got = _grads(q, k, v, do, W, det=True)
    _check_grads(got, q, k, v, do, window=W)
    # dK / dV come from the same key-major kernel either way: bitwise equal
    ref = _grads(q, k, v, do, W, det=False)
    assert torch.equal(got[1], ref[1]) and torch.equal(got[2], ref[2])


def test_flash_bwd_deterministic_is_bitwise_repeatable():
    q, k, v = _qkv(2, 8, 4, 4096, 128, seed=7)
    do = randn((2, 8, 4096, 128), 8, torch.bfloat16, CUDA)
    a = _grads(q, k, v, do, det=True)
    b = _grads(q, k, v, do, det=True)
    assert all(torch.equal(x, y) for x, y in zip(a, b))
    # torch.use_deterministic_algorithms selects the same path by default
    prev = torch.are_deterministic_algorithms_enabled()
    torch.use_deterministic_algorithms(True, warn_only=True)
    try:
        c = _grads(q, k, v, do)
    finally:
        torch.use_deterministic_algorithms(prev)
    assert torch.equal(a[0], c[0])


def test_flash_bwd_chunk_deterministic():
    from smooth_attn.kernels import sp2norm_flash_attention_chunk_bwd

    Tq, Tk, off = 200, 700, 500
    q = randn((1, 4, Tq, 128), 1, torch.bfloat16, CUDA)
    k = randn((1, 2, Tk, 128), 2, torch.bfloat16, CUDA)
    v = randn((1, 2, Tk, 128), 3, torch.bfloat16, CUDA)
    do = randn((1, 4, Tq, 128), 4, torch.bfloat16, CUDA)
    o, rs, lo = sa.sp2norm_flash_attention_chunk(q, k, v, off, window_size=96, return_residual=True)
    got = sp2norm_flash_attention_chunk_bwd(q, k, v, o, do, rs, off, window_size=96, o_lo=lo, deterministic=True)
    args = (np32(q), np32(k), np32(v), np32(do), off)
    ref = O.chunk_flash_attention_bwd(*args, window_size=96, acc=np.float64)
    emu = O.chunk_flash_attention_bwd(*args, window_size=96, emulate=True)
    for g, r, m in zip(got, ref, emu):
        check_bf16_grads(np32(g), r, m, **BWD_TOL)


@pytest.mark.parametrize(("Hq", "Hkv", "T", "D", "W"), [(4, 2, 200, 64, 0), (4, 1, 333, 128, 90)])
def test_flash_bwd_deterministic_exact_math(Hq, Hkv, T, D, W):
    """The deterministic kernels with IEEE sqrt (exact_math) against the oracle, and bitwise repeatable."""
    q, k, v = _qkv(1, Hq, Hkv, T, D, seed=T + 11)
    do = randn((1, Hq, T, D), T + 12, torch.bfloat16, CUDA)

    def grads():
        qq, kk, vv = (t.detach().requires_grad_(True) for t in (q, k, v))
        sa.sp2norm_flash_attention(qq, kk, vv, window_size=W, exact_math=True, deterministic=True).backward(do)
        return qq.grad, kk.grad, vv.grad

    a, b = grads(), grads()
    assert all(torch.equal(x, y) for x, y in zip(a, b))
    _check_grads(a, q, k, v, do, window=W)

"""Parity of the RoPE attention forward (``sa_rope_flash_fwd`` through
``sp2norm_rope_flash_attention``), the RoPE + output projection and the
standalone rotation (``sa_rope_rotate``) with the numpy oracle and the
committed golden vectors.  Mirrors the reference's ``tests/test_rope_proj.py``
(correctness at three shapes, GQA, sliding window, projection) plus head dim
128, ragged T, fp16, bf16 cos/sin tables, strided [B, T, H, D] inputs and the
C ABI's argument checks."""

import ctypes
from pathlib import Path

import numpy as np
import pytest
import torch

import smooth_attn as sa
from smooth_attn import _lib
from oracle import sa_oracle as O
from tests._util import assert_close, np32, randn

pytestmark = pytest.mark.gpu
CUDA = "cuda"
G = np.load(Path(__file__).parent / "golden" / "golden.npz")
FWD_TOL = dict(rtol=2e-2, atol=1e-2)  # bf16 attention output vs the fp32 oracle (as the flash tests)
PROJ_TOL = dict(rtol=2e-2, atol=1e-2)


@pytest.fixture(autouse=True)
def _need_cuda():
    if not torch.cuda.is_available():
        pytest.skip("CUDA required")


def _inputs(B, Hq, Hkv, T, D, seed, dtype=torch.bfloat16):
    q = randn((B, Hq, T, D), seed, dtype, CUDA)
    k = randn((B, Hkv, T, D), seed + 1, dtype, CUDA)
    v = randn((B, Hkv, T, D), seed + 2, dtype, CUDA)
    cos, sin = sa.precompute_rope_cos_sin(D, T, device=CUDA, dtype=torch.float32)
    return q, k, v, cos, sin


def _ref(q, k, v, cos, sin, window=0):
    return O.rope_flash_attention(np32(q), np32(k), np32(v), np32(cos), np32(sin), window_size=window)


@pytest.mark.parametrize("name", sorted({k.split("/")[0] for k in G.files if k.startswith("rope_")}))
def test_rope_golden(name):
    t = lambda s: torch.from_numpy(G[f"{name}/{s}"]).to(CUDA)
    q, k, v = (t(s).to(torch.bfloat16) for s in ("q", "k", "v"))
    cos, sin = t("cos"), t("sin")
    w = int(G[f"{name}/window"])
    o = sa.sp2norm_rope_flash_attention(q, k, v, cos, sin, window_size=w)
    assert_close(np32(o), G[f"{name}/o"], **FWD_TOL)
    if f"{name}/w_o" in G.files:
        out = sa.sp2norm_rope_flash_attention_proj(q, k, v, t("w_o").to(torch.bfloat16), cos, sin, window_size=w)
        assert out.dtype == torch.bfloat16
        assert_close(np32(out), G[f"{name}/proj"], **PROJ_TOL)


# tests/test_rope_proj.py:48-71 plus D=128 and ragged T
@pytest.mark.parametrize("B,H,T,D", [(1, 4, 64, 32), (2, 4, 128, 32), (2, 8, 256, 64), (1, 2, 300, 128),
                                     (2, 3, 77, 64), (1, 1, 1, 32)])
def test_rope_flash_correctness(B, H, T, D):
    q, k, v, cos, sin = _inputs(B, H, H, T, D, seed=B * 100 + T + D)
    o = sa.sp2norm_rope_flash_attention(q, k, v, cos, sin)
    assert o.shape == q.shape and o.dtype == q.dtype and not o.isnan().any()
    assert_close(np32(o), _ref(q, k, v, cos, sin), **FWD_TOL)


# tests/test_rope_proj.py:74-94
def test_rope_flash_gqa():
    q, k, v, cos, sin = _inputs(2, 8, 2, 128, 32, seed=5)
    o = sa.sp2norm_rope_flash_attention(q, k, v, cos, sin)
    assert o.shape == (2, 8, 128, 32)
    assert_close(np32(o), _ref(q, k, v, cos, sin), **FWD_TOL)


# tests/test_rope_proj.py:97-115
@pytest.mark.parametrize("W", [64, 1, 200])
def test_rope_flash_window(W):
    q, k, v, cos, sin = _inputs(2, 4, 4, 128 if W != 200 else 384, 32, seed=W)
    o = sa.sp2norm_rope_flash_attention(q, k, v, cos, sin, window_size=W)
    assert_close(np32(o), _ref(q, k, v, cos, sin, window=W), **FWD_TOL)


# tests/test_rope_proj.py:118-151 plus GQA and a wider model dim
@pytest.mark.parametrize("B,Hq,Hkv,T,D,DM", [(2, 4, 4, 64, 32, 128), (1, 8, 2, 200, 64, 512), (2, 4, 1, 130, 128, 256)])
def test_rope_proj_correctness(B, Hq, Hkv, T, D, DM):
    q, k, v, cos, sin = _inputs(B, Hq, Hkv, T, D, seed=DM + T)
    w_o = randn((Hq, D, DM), DM, torch.bfloat16, CUDA) * 0.02
    out = sa.sp2norm_rope_flash_attention_proj(q, k, v, w_o, cos, sin)
    assert out.shape == (B, T, DM) and out.dtype == torch.bfloat16 and not out.isnan().any()
    ref = O.rope_flash_attention_proj(np32(q), np32(k), np32(v), np32(w_o), np32(cos), np32(sin))
    assert_close(np32(out), ref, **PROJ_TOL)


def test_rope_fp16_bf16_tables_and_strided_inputs():
    B, H, T, D = 2, 4, 160, 64
    q, k, v, cos, sin = _inputs(B, H, H, T, D, seed=9, dtype=torch.float16)
    # [B, T, H, D] storage viewed as [B, H, T, D]
    qs, ks, vs = (x.transpose(1, 2).contiguous().transpose(1, 2) for x in (q, k, v))
    o = sa.sp2norm_rope_flash_attention(qs, ks, vs, cos.to(torch.bfloat16), sin.to(torch.bfloat16))
    ref = O.rope_flash_attention(np32(q), np32(k), np32(v), np32(cos.to(torch.bfloat16)),
                                 np32(sin.to(torch.bfloat16)))
    # fp16 rotation rounds to fp16 (finer than the reference's bf16)
    assert_close(np32(o), ref, **FWD_TOL)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_rope_rotate_bit_exact(dtype):
    """sa_rope_rotate reproduces the reference's eager rotation bit for bit
    (same fp32 rounding steps, then rounding to the 16-bit type)."""
    B, H, T, D = 2, 3, 50, 128
    x = randn((B, H, T, D), 1, dtype, CUDA) * 4
    cos, sin = sa.precompute_rope_cos_sin(D, T, device=CUDA)
    out = torch.empty_like(x)
    st = _lib.load().sa_rope_rotate(x.data_ptr(), out.data_ptr(), cos.data_ptr(), sin.data_ptr(), _lib.SA_F32,
                                    B, H, T, D, _lib.strides(x), _lib.SA_BF16 if dtype == torch.bfloat16 else _lib.SA_F16,
                                    ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    assert st == 0
    exp = O.rope_rotate(np32(x), np32(cos), np32(sin), to_bf16=False)
    exp = torch.from_numpy(exp).to(dtype).float().numpy()
    np.testing.assert_array_equal(np32(out), exp)


def test_rope_rejects_bad_arguments():
    q, k, v, cos, sin = _inputs(1, 2, 2, 64, 32, seed=3)
    with pytest.raises(AssertionError):
        sa.sp2norm_rope_flash_attention(q, k, v, cos[:32], sin[:32])
    with pytest.raises(ValueError):
        sa.sp2norm_rope_flash_attention(q.float(), k.float(), v.float(), cos, sin)
    ws = torch.empty(16, device=CUDA, dtype=torch.uint8)
    lib = _lib.load()
    st = lib.sa_rope_flash_fwd(q.data_ptr(), k.data_ptr(), v.data_ptr(), q.data_ptr(), None, cos.data_ptr(),
                               sin.data_ptr(), _lib.SA_F32, ws.data_ptr(), 16, 1, 2, 2, 64, 32, _lib.strides(q),
                               _lib.strides(k), _lib.strides(v), _lib.strides(q), 0.1, 0, 0, _lib.SA_BF16, None)
    assert st == _lib.SA_ERR_ARG  # workspace too small

"""Parity of the FP8 attention forward (``sa_fp8_quantize`` + ``sa_fp8_flash_fwd``
through ``sp2norm_fp8_flash_attention``) with the numpy oracle and the golden
quantization vectors.  Mirrors the reference's ``tests/test_fp8_flash.py``
(against eager attention at max error 0.3 / mean 0.02, sizes 64-512, GQA,
sliding window) and adds a tight comparison with the FP8 oracle (the same
quantized operands), head dims 64 and 128, ragged T and fp32 / fp16 inputs."""

from pathlib import Path

import numpy as np
import pytest
import torch

import smooth_attn as sa
from smooth_attn.kernels import _fp8_quantize
from oracle import sa_oracle as O
from tests._util import assert_close, np32, randn

pytestmark = pytest.mark.gpu
CUDA = "cuda"
G = np.load(Path(__file__).parent / "golden" / "golden.npz")
# same quantized operands: only accumulation order and bf16 output rounding differ
FP8_TOL = dict(rtol=2e-2, atol=1e-2)  # kernel vs the oracle on the same E4M3 inputs


@pytest.fixture(autouse=True)
def _need_cuda():
    if not torch.cuda.is_available():
        pytest.skip("CUDA required")


def _qkv(B, Hq, Hkv, T, D, seed, dtype=torch.bfloat16):
    return (randn((B, Hq, T, D), seed, dtype, CUDA), randn((B, Hkv, T, D), seed + 1, dtype, CUDA),
            randn((B, Hkv, T, D), seed + 2, dtype, CUDA))


def _e4m3(u8):
    return u8.view(torch.float8_e4m3fn).float()


@pytest.mark.parametrize("name", sorted({k.split("/")[0] for k in G.files if k.startswith("fp8_")}))
def test_fp8_quantize_golden(name):
    """The device quantizer reproduces the reference's _quantize_to_fp8 bit for bit."""
    x = torch.from_numpy(G[f"{name}/x"]).to(CUDA)
    x8, _, v8, scales = _fp8_quantize(x, x, x)
    ref = torch.from_numpy(G[f"{name}/x8"]).to(CUDA)
    assert torch.equal(_e4m3(x8), ref)
    assert torch.equal(v8.float(), ref)
    assert float(scales[0]) == float(np.float32(G[f"{name}/scale"]))
    assert torch.equal(scales, scales[:1].expand(3))


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16, torch.float32])
def test_fp8_quantize_matches_oracle(dtype):
    q, k, v = _qkv(2, 4, 2, 200, 64, seed=3, dtype=dtype)
    q8, k8, vq, scales = _fp8_quantize(q * 3, k, v * 0.01)
    for t, dev8, i in ((q * 3, _e4m3(q8), 0), (k, _e4m3(k8), 1), (v * 0.01, vq.float(), 2)):
        ref8, sc = O.quantize_fp8(np32(t))
        np.testing.assert_array_equal(np32(dev8), ref8)
        assert float(scales[i]) == float(np.float32(sc))


# tests/test_fp8_flash.py:10-31, :54-69 plus D 64/128 and ragged T
@pytest.mark.parametrize("B,H,T,D", [(2, 4, 128, 32), (2, 4, 64, 32), (2, 4, 256, 32), (2, 4, 512, 32),
                                     (1, 2, 300, 64), (1, 2, 257, 128), (2, 3, 77, 128)])
def test_fp8_matches_oracle_and_eager(B, H, T, D):
    q, k, v = _qkv(B, H, H, T, D, seed=T + D)
    o = sa.sp2norm_fp8_flash_attention(q, k, v)
    assert o.shape == q.shape and o.dtype == torch.bfloat16 and not o.isnan().any()
    assert_close(np32(o), O.fp8_flash_attention(np32(q), np32(k), np32(v)), **FP8_TOL)
    err = np.abs(np32(o) - O.sp2norm_flash_attention(np32(q), np32(k), np32(v)))
    assert err.max() < 0.3 and err.mean() < 0.02  # the reference's own bounds vs eager


# tests/test_fp8_flash.py:72-87
def test_fp8_gqa():
    q, k, v = _qkv(2, 8, 2, 128, 32, seed=8)
    o = sa.sp2norm_fp8_flash_attention(q, k, v)
    assert o.shape == (2, 8, 128, 32)
    assert_close(np32(o), O.fp8_flash_attention(np32(q), np32(k), np32(v)), **FP8_TOL)


# tests/test_fp8_flash.py:89-103
@pytest.mark.parametrize("W", [64, 1, 300])
def test_fp8_window(W):
    q, k, v = _qkv(2, 4, 4, 128 if W < 300 else 640, 64, seed=W)
    o = sa.sp2norm_fp8_flash_attention(q, k, v, window_size=W)
    assert_close(np32(o), O.fp8_flash_attention(np32(q), np32(k), np32(v), window_size=W), **FP8_TOL)


def test_fp8_scale_and_large_values():
    """Per-tensor scales absorb the magnitude of large inputs (x100 q and v,
    attention scale / 100): the result tracks the oracle on those inputs."""
    q, k, v = _qkv(1, 2, 2, 192, 64, seed=21)
    o1 = sa.sp2norm_fp8_flash_attention(q, k, v, scale=0.02)
    assert_close(np32(o1), O.fp8_flash_attention(np32(q), np32(k), np32(v), scale=0.02), **FP8_TOL)
    q2, v2 = q * 100, v * 100
    o2 = sa.sp2norm_fp8_flash_attention(q2, k, v2, scale=0.0002)
    ref2 = O.fp8_flash_attention(np32(q2), np32(k), np32(v2), scale=0.0002)
    assert_close(np32(o2), ref2, rtol=2e-2, atol=1.0)  # outputs ~100x larger: 1e-2 x 100


def test_fp8_rejects_bad_arguments():
    q, k, v = _qkv(1, 2, 2, 64, 48, seed=1)
    with pytest.raises(ValueError):
        sa.sp2norm_fp8_flash_attention(q, k, v)
    q, k, v = _qkv(1, 3, 2, 64, 32, seed=1)
    with pytest.raises(AssertionError):
        sa.sp2norm_fp8_flash_attention(q, k, v)

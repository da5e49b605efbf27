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
from tests._util import assert_close, np32, randn

pytestmark = pytest.mark.gpu
CUDA = "cuda"
G = np.load(Path(__file__).parent / "golden" / "golden.npz")

# bf16 attention output vs the fp32 oracle on the same (bf16-rounded) inputs.
# The kernel rounds the unnormalized y to bf16 before P.V exactly like the
# reference (kernels.py:1621), so the reference's own flash tolerance applies.
FWD_TOL = dict(rtol=5e-2, atol=2e-2)
BWD_TOL = dict(rtol=0.1, atol=5e-2)


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
    torch.testing.assert_close(out_flash.float(), out_eager.float(), atol=2e-2, rtol=5e-2)


def test_flash_rowsum_saved():
    q, k, v = _qkv(1, 2, 2, 200, 64, seed=5)
    from smooth_attn.kernels import _sp2norm_flash_fwd

    o, rs = _sp2norm_flash_fwd(q, k, v, 1.0 / 8.0)
    _, ref_rs = _fwd_ref(q, k, v)
    assert_close(rs.cpu().numpy(), ref_rs, rtol=2e-3, atol=0)


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

"""The output-projection GEMM of the RoPE attention (``sa_out_proj``) on its
own: ragged M / N / K, both 16-bit types, padded row strides, against an fp64
matmul of the same rounded inputs.  The reference fuses this product into its
attention kernel (``src/smooth_attn/kernels.py:2233-2370``) and checks it in
``tests/test_rope_proj.py:118-151`` at the end-to-end level, which
``tests/test_rope_gpu.py`` mirrors."""

import ctypes

import numpy as np
import pytest
import torch

from smooth_attn import _lib
from smooth_attn.kernels import _out_proj
from tests._util import assert_close, np32, randn

pytestmark = pytest.mark.gpu
TOL = dict(rtol=2e-2, atol=1e-2)


@pytest.fixture(autouse=True)
def _need_cuda():
    if not torch.cuda.is_available():
        pytest.skip("CUDA required")


@pytest.mark.parametrize(("M", "K", "N"), [(1, 64, 8), (127, 96, 264), (300, 4096, 520), (1024, 512, 256),
                                           (129, 32, 16), (4096, 4096, 1024)])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_out_proj_matches_fp64(M, K, N, dtype):
    a = randn((M, K), M + K, dtype, "cuda", scale=0.5)
    w = randn((K, N), K + N, dtype, "cuda", scale=0.05)
    out = _out_proj(a, w)
    assert out.dtype == dtype and out.shape == (M, N)
    ref = np32(a).astype(np.float64) @ np32(w).astype(np.float64)
    assert_close(np32(out), ref, **TOL)


def test_out_proj_padded_strides_and_determinism():
    a_full = randn((200, 160), 1, torch.bfloat16, "cuda")
    w_full = randn((128, 72), 2, torch.bfloat16, "cuda", scale=0.1)
    a, w = a_full[:, :128], w_full[:, :64]  # row strides 160 and 72 elements
    lib = _lib.load()
    out = torch.empty(200, 64, dtype=torch.bfloat16, device="cuda")
    st = lib.sa_out_proj(a.data_ptr(), w.data_ptr(), out.data_ptr(), 200, 128, 64, 160, 72, 64, _lib.SA_BF16,
                         ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    assert st == _lib.SA_OK
    ref = np32(a).astype(np.float64) @ np32(w).astype(np.float64)
    assert_close(np32(out), ref, **TOL)
    assert torch.equal(out, _out_proj(a, w))  # same bits through the Python path, run to run


def test_out_proj_rejects_bad_layouts():
    lib = _lib.load()
    x = torch.empty(64, 64, dtype=torch.bfloat16, device="cuda")
    assert lib.sa_out_proj(x.data_ptr(), x.data_ptr(), x.data_ptr(), 64, 64, 60, 64, 64, 64, _lib.SA_BF16,
                           None) == _lib.SA_ERR_ALIGN  # N % 8
    assert lib.sa_out_proj(x.data_ptr(), x.data_ptr(), x.data_ptr(), 64, 64, 64, 60, 64, 64, _lib.SA_BF16,
                           None) == _lib.SA_ERR_ALIGN  # lda < K
    assert lib.sa_out_proj(x.data_ptr(), x.data_ptr(), x.data_ptr(), 64, 64, 64, 64, 64, 64, _lib.SA_F32,
                           None) == _lib.SA_ERR_UNSUPPORTED

"""softplus_norm_causal_host_out: the causal norm between pinned host buffers
(only the bands the kernel reads / can write cross PCIe; the zero columns
past each band are written on the host).  The result must equal the device
path bit for bit, whatever the output buffer held before."""

import ctypes

import pytest
import torch

import smooth_attn as sa
from smooth_attn import _lib, host

pytestmark = pytest.mark.gpu


@pytest.fixture(autouse=True)
def _need_cuda():
    if not torch.cuda.is_available():
        pytest.skip("CUDA required")


@pytest.mark.parametrize(("shape", "dtype", "slices"), [((2, 3, 300, 300), torch.bfloat16, 3),
                                                        ((1, 2, 640, 640), torch.float32, 16),
                                                        ((2, 1, 129, 129), torch.float16, 2),
                                                        ((4, 2, 2048, 2048), torch.bfloat16, 8),
                                                        ((1, 1, 7, 7), torch.bfloat16, 1)])
def test_host_path_equals_device_path(shape, dtype, slices):
    g = torch.Generator().manual_seed(sum(shape))
    x = torch.randn(*shape, generator=g).to(dtype).pin_memory()
    out = torch.full(shape, float("nan"), dtype=dtype).pin_memory()  # every element must be overwritten
    for _ in range(2):  # the second call reuses the cached device buffers and streams
        sa.softplus_norm_causal_host_out(out, x, slices=slices)
        ref = sa.softplus_norm_causal_triton_out(torch.empty(shape, dtype=dtype, device="cuda"), x.cuda())
        assert torch.equal(out.cuda(), ref)
        out.fill_(float("nan"))


def test_band_copy_moves_the_counted_bytes():
    L, nmat = 300, 3
    x = torch.randn(nmat, L, L).to(torch.bfloat16).pin_memory()
    d = torch.zeros(nmat, L, L, dtype=torch.bfloat16, device="cuda")
    moved = ctypes.c_int64(0)
    st = _lib.load().sa_copy_causal_bands(ctypes.c_void_p(d.data_ptr()), ctypes.c_void_p(x.data_ptr()), nmat, L, 2,
                                          host.BAND, 1, ctypes.byref(moved),
                                          ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    _lib.check(st, "sa_copy_causal_bands")
    torch.cuda.synchronize()
    assert moved.value == host.causal_band_bytes(x.shape, x.dtype)
    for r0, r1, w in host._bands(L, 2):  # copied bands match, the rest is untouched
        assert torch.equal(d[:, r0:r1, :w].cpu(), x[:, r0:r1, :w])
        assert not d[:, r0:r1, w:].any()

"""The allocation-free backward entry point, called through the C ABI.

``sa_flash_bwd_noalloc`` serves callers that cannot allocate device memory
(a stream capture that must not allocate, a host framework that owns all GPU
memory, a latency-critical loop): its scratch is a fixed device array inside
the library instead of a caller workspace.  This test checks it against the
regular ``sa_flash_bwd`` (through the public API) on two calls in a row, so a
stale accumulator from the first call would show up in the second.  The file
is named to be collected last.
"""

import ctypes

import pytest
import torch

import smooth_attn as sa
from smooth_attn import _lib
from smooth_attn.kernels import _sp2norm_flash_fwd
from tests._util import randn

pytestmark = pytest.mark.gpu


@pytest.fixture(autouse=True)
def _need_cuda():
    if not torch.cuda.is_available():
        pytest.skip("CUDA required")


def _noalloc_bwd(q, k, v, o, do, rs, scale):
    lib = _lib.load()
    dq, dk, dv = torch.empty_like(q), torch.empty_like(k), torch.empty_like(v)
    B, Hq, T, D = q.shape
    st = lib.sa_flash_bwd_noalloc(
        q.data_ptr(), k.data_ptr(), v.data_ptr(), o.data_ptr(), do.data_ptr(), rs.data_ptr(),
        dq.data_ptr(), dk.data_ptr(), dv.data_ptr(), B, Hq, k.shape[1], T, D,
        _lib.strides(q), _lib.strides(k), _lib.strides(v), _lib.strides(o), _lib.strides(do),
        _lib.strides(dq), _lib.strides(dk), _lib.strides(dv),
        ctypes.c_float(scale), 0, 0, _lib.SA_BF16, ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    _lib.check(st, "sa_flash_bwd_noalloc")
    return dq, dk, dv


@pytest.mark.parametrize(("Hq", "Hkv", "T", "D"), [(4, 2, 256, 128), (2, 2, 200, 64)])
def test_noalloc_bwd_matches_allocating_entry_point_twice(Hq, Hkv, T, D):
    scale = 1.0 / D ** 0.5
    for call in range(2):
        q = randn((1, Hq, T, D), 10 + call, torch.bfloat16, "cuda")
        k = randn((1, Hkv, T, D), 20 + call, torch.bfloat16, "cuda")
        v = randn((1, Hkv, T, D), 30 + call, torch.bfloat16, "cuda")
        do = randn((1, Hq, T, D), 40 + call, torch.bfloat16, "cuda")
        o, rs = _sp2norm_flash_fwd(q, k, v, scale)
        ref = sa.kernels._sp2norm_flash_bwd(q, k, v, o, do, rs, scale)
        got = _noalloc_bwd(q, k, v, o, do, rs, scale)
        torch.cuda.synchronize()
        for g, r in zip(got, ref):
            # same kernels, different scratch: equal up to fp32 atomic ordering in dQ
            torch.testing.assert_close(g.float(), r.float(), rtol=0.1, atol=5e-2)


def test_noalloc_rejects_problem_larger_than_scratch():
    lib = _lib.load()
    cap = lib.sa_flash_bwd_noalloc_max_bytes()
    assert cap == 32 << 20
    B, Hq, T, D = 1, 64, 4096, 128  # needs 128 MiB of dQ accumulator
    assert lib.sa_flash_bwd_workspace_size(B, Hq, Hq, T, D) > cap
    x = torch.empty(1, device="cuda")
    s = (ctypes.c_int64 * 4)(Hq * T * D, T * D, D, 1)  # contiguous [B, Hq, T, D]; nothing is read
    st = lib.sa_flash_bwd_noalloc(*(x.data_ptr(),) * 9, B, Hq, Hq, T, D, *(s,) * 8,
                                  ctypes.c_float(0.1), 0, 0, _lib.SA_BF16, None)
    assert st == _lib.SA_ERR_ARG

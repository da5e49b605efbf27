"""The allocation-free backward entry point, called through the C ABI.

``sa_flash_bwd_noalloc`` serves callers that cannot allocate device memory:
code inside a CUDA-graph capture that must not allocate, plugins whose host
framework owns all GPU memory, or loops where an allocator call could stall.
Its scratch is a fixed device array inside the library instead of a caller
workspace.  This test checks, on two calls in a row (so a stale accumulator
left by the first call would show in the second):

* dK / dV equal the allocating ``sa_flash_bwd`` bit for bit (same kernels,
  no shared accumulator on that path), and dQ equals it up to the order of
  its fp32 atomic adds;
* all three gradients match the fp32 oracle at the bf16 tolerance;
* the call leaves the device's free memory unchanged.

The file is named to be collected last.
"""

import ctypes

import numpy as np
import pytest
import torch

import smooth_attn as sa
from oracle import sa_oracle as O
from smooth_attn import _lib
from smooth_attn.kernels import _sp2norm_flash_fwd
from tests._util import check_bf16_grads, np32, randn

pytestmark = pytest.mark.gpu


@pytest.fixture(autouse=True)
def _need_cuda():
    if not torch.cuda.is_available():
        pytest.skip("CUDA required")


def _noalloc_bwd(q, k, v, o, o_lo, do, rs, scale, dq, dk, dv):
    lib = _lib.load()
    B, Hq, T, D = q.shape
    st = lib.sa_flash_bwd_noalloc(
        q.data_ptr(), k.data_ptr(), v.data_ptr(), o.data_ptr(), o_lo.data_ptr(), do.data_ptr(), rs.data_ptr(),
        dq.data_ptr(), dk.data_ptr(), dv.data_ptr(), B, Hq, k.shape[1], T, D,
        _lib.strides(q), _lib.strides(k), _lib.strides(v), _lib.strides(o), _lib.strides(do),
        _lib.strides(dq), _lib.strides(dk), _lib.strides(dv),
        ctypes.c_float(scale), 0, 0, _lib.SA_BF16, ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    _lib.check(st, "sa_flash_bwd_noalloc")


@pytest.mark.parametrize(("Hq", "Hkv", "T", "D"), [(4, 2, 256, 128), (2, 2, 200, 64)])
def test_noalloc_bwd_matches_allocating_entry_point_twice(Hq, Hkv, T, D):
    scale = 1.0 / D ** 0.5
    for call in range(2):
        q = randn((1, Hq, T, D), 10 + call, torch.bfloat16, "cuda")
        k = randn((1, Hkv, T, D), 20 + call, torch.bfloat16, "cuda")
        v = randn((1, Hkv, T, D), 30 + call, torch.bfloat16, "cuda")
        do = randn((1, Hq, T, D), 40 + call, torch.bfloat16, "cuda")
        o, rs, lo = _sp2norm_flash_fwd(q, k, v, scale, with_residual=True)
        ref = sa.kernels._sp2norm_flash_bwd(q, k, v, o, do, rs, scale, o_lo=lo)
        got = tuple(torch.empty_like(t) for t in (q, k, v))
        if call == 1:  # after one call every kernel is loaded: the call itself must allocate nothing
            torch.cuda.synchronize()
            free0 = torch.cuda.mem_get_info()[0]
        _noalloc_bwd(q, k, v, o, lo, do, rs, scale, *got)
        torch.cuda.synchronize()
        if call == 1:
            assert torch.cuda.mem_get_info()[0] == free0
        assert torch.equal(got[1], ref[1]) and torch.equal(got[2], ref[2])
        # dQ: same partials, fp32 atomics in another order, then one bf16 rounding
        torch.testing.assert_close(got[0].float(), ref[0].float(), rtol=1e-2, atol=1e-2)
        args = (np32(q), np32(k), np32(v), np32(do))
        ref64 = O.sp2norm_flash_attention_bwd(*args, scale=scale, acc=np.float64)
        emu = O.sp2norm_flash_attention_bwd(*args, scale=scale, emulate=True)
        for g, r, m in zip(got, ref64, emu):
            check_bf16_grads(np32(g), r, m, rtol=2e-2, atol=1e-2)


def test_noalloc_rejects_problem_larger_than_scratch():
    lib = _lib.load()
    cap = lib.sa_flash_bwd_noalloc_max_bytes()
    assert cap == 32 << 20
    B, Hq, T, D = 1, 64, 4096, 128  # needs 128 MiB of dQ accumulator
    assert lib.sa_flash_bwd_workspace_size(B, Hq, Hq, T, D) > cap
    x = torch.empty(1, device="cuda")
    s = (ctypes.c_int64 * 4)(Hq * T * D, T * D, D, 1)  # contiguous [B, Hq, T, D]; nothing is read
    st = lib.sa_flash_bwd_noalloc(*(x.data_ptr(),) * 10, B, Hq, Hq, T, D, *(s,) * 8,
                                  ctypes.c_float(0.1), 0, 0, _lib.SA_BF16, None)
    assert st == _lib.SA_ERR_ARG
    # a size whose byte count overflows int64 is rejected, not wrapped
    big = 1 << 40
    assert lib.sa_flash_bwd_workspace_size(big, big, 1, 1024, 128) == 0
    st = lib.sa_flash_bwd_noalloc(*(x.data_ptr(),) * 10, big, big, 1, 1024, 128, *(s,) * 8,
                                  ctypes.c_float(0.1), 0, 0, _lib.SA_BF16, None)
    assert st == _lib.SA_ERR_ARG

"""Bounded device-side waits: a wait that runs out is recorded and reported,
and the kernel leaves normally (no trap, the context stays usable).

``sa_probe_bounded_wait`` launches one warp that waits, with the same bounded
mbarrier wait every kernel of the library uses, on a barrier that nothing
arrives on.  Nothing faults: the wait gives up after ~1 ms."""

import ctypes

import pytest
import torch

import smooth_attn as sa
from smooth_attn import _lib
from tests._util import randn

pytestmark = pytest.mark.gpu


@pytest.fixture(autouse=True)
def _need_cuda():
    if not torch.cuda.is_available():
        pytest.skip("CUDA required")


def test_expired_wait_reports_timeout_and_context_survives():
    lib = _lib.load()
    st = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    assert lib.sa_stream_status(st, 1) in (_lib.SA_OK, _lib.SA_ERR_TIMEOUT, _lib.SA_ERR_ARG)  # clear earlier state
    done = torch.zeros(1, dtype=torch.int32, device="cuda")
    assert lib.sa_probe_bounded_wait(1_000_000, done.data_ptr(), st) == _lib.SA_OK
    assert lib.sa_stream_status(st, 0) == _lib.SA_ERR_TIMEOUT
    assert int(done.item()) == 1  # the wait gave up and the kernel went on to its normal exit
    assert lib.sa_device_status(1) == _lib.SA_ERR_TIMEOUT  # device-wide view agrees; reset
    assert lib.sa_stream_status(st, 0) == _lib.SA_OK
    # the context is still usable: a regular launch runs and reports no timeout
    q = randn((1, 2, 64, 32), 1, torch.bfloat16, "cuda")
    o = sa.sp2norm_flash_attention(q, q, q)
    assert torch.isfinite(o.float()).all()
    assert lib.sa_stream_status(st, 0) == _lib.SA_OK


def test_probe_rejects_bad_limit():
    lib = _lib.load()
    done = torch.zeros(1, dtype=torch.int32, device="cuda")
    assert lib.sa_probe_bounded_wait(0, done.data_ptr(), None) == _lib.SA_ERR_ARG
    assert lib.sa_probe_bounded_wait(3_000_000_000, done.data_ptr(), None) == _lib.SA_ERR_ARG

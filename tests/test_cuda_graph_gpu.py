"""CUDA-graph capture of the public API: every path launches only on the
current stream, allocates through torch's caching allocator and never
synchronises the host, so it can be captured once and replayed with new
input data (a serving loop's decode step, a training step's attention).
Replays must give what an eager call on the same inputs gives."""

import gc

import pytest
import torch

import smooth_attn as sa
from tests._util import randn

pytestmark = pytest.mark.gpu
CUDA = "cuda"


@pytest.fixture(autouse=True)
def _need_cuda():
    if not torch.cuda.is_available():
        pytest.skip("CUDA required")


def _capture(fn):
    """Warm up on a side stream, then capture ``fn`` into a graph."""
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        for _ in range(2):
            fn()
    torch.cuda.current_stream().wait_stream(s)
    g = torch.cuda.CUDAGraph()
    # Garbage from earlier tests (graphs kept alive by reference cycles) must
    # not be collected mid-capture: destroying a graph frees its memory pool
    # (cudaFree), which invalidates the capture.  torch.cuda.graph no longer
    # collects before capturing by default, so collect here and keep the
    # collector off until the capture ends.  Thread-local mode: a CUDA call
    # from another thread of the process (a compile worker) must not
    # invalidate it either.
    gc.collect()
    gc.disable()
    try:
        with torch.cuda.graph(g, capture_error_mode="thread_local"):
            out = fn()
    finally:
        gc.enable()
    return g, out


@pytest.mark.parametrize("Hq,Hkv,D", [(32, 8, 128), (16, 16, 64), (8, 2, 256)])
def test_paged_decode_replay(Hq, Hkv, D):
    """Decode step with new queries and grown context lengths on each replay
    (tensor-core kernel for the GQA D=128 case, CUDA-core otherwise)."""
    B, BS, nb = 4, 16, 256
    q = randn((B, Hq, 1, D), 1, torch.bfloat16, CUDA)
    kc, vc = randn((nb, Hkv, BS, D), 2, torch.bfloat16, CUDA), randn((nb, Hkv, BS, D), 3, torch.bfloat16, CUDA)
    bt = torch.randperm(nb, device=CUDA).view(B, -1).to(torch.int32)
    cl = torch.tensor([1000, 5, 640, 17], device=CUDA, dtype=torch.int32)
    g, out = _capture(lambda: sa.sp2norm_paged_attention(q, kc, vc, bt, cl))
    for step in range(3):
        q.copy_(randn(q.shape, 10 + step, torch.bfloat16, CUDA))
        cl.add_(7)
        g.replay()
        torch.cuda.synchronize()
        assert torch.equal(out, sa.sp2norm_paged_attention(q, kc, vc, bt, cl))


def test_flash_fwd_bwd_graphed_callable():
    """torch.cuda.make_graphed_callables over the autograd flash attention:
    forward and backward graphs, replayed on fresh inputs."""
    shp = [(2, 8, 512, 128), (2, 2, 512, 128), (2, 2, 512, 128)]
    sample = [randn(s, i, torch.bfloat16, CUDA).requires_grad_(True) for i, s in enumerate(shp)]
    gc.collect()
    fn = torch.cuda.make_graphed_callables(lambda q, k, v: sa.sp2norm_flash_attention(q, k, v, window_size=300),
                                           tuple(sample))
    for step in range(2):
        ins = [randn(s, 20 + 3 * step + i, torch.bfloat16, CUDA).requires_grad_(True) for i, s in enumerate(shp)]
        ref = [t.detach().clone().requires_grad_(True) for t in ins]
        do = randn(shp[0], 50 + step, torch.bfloat16, CUDA)
        o = fn(*ins)
        (o * do).sum().backward()
        o_ref = sa.sp2norm_flash_attention(*ref, window_size=300)
        (o_ref * do).sum().backward()
        assert torch.equal(o, o_ref)
        # dK / dV are deterministic (summed in-CTA); dQ is added with fp32 atomics
        assert torch.equal(ins[1].grad, ref[1].grad) and torch.equal(ins[2].grad, ref[2].grad)
        torch.testing.assert_close(ins[0].grad, ref[0].grad, rtol=1e-2, atol=1e-2)


def test_norm_graphed_callable():
    x0 = randn((2, 8, 384, 384), 1, torch.bfloat16, CUDA).requires_grad_(True)
    gc.collect()
    fn = torch.cuda.make_graphed_callables(lambda x: sa.softplus_norm_causal(x), (x0,))
    x = randn(x0.shape, 2, torch.bfloat16, CUDA).requires_grad_(True)
    xr = x.detach().clone().requires_grad_(True)
    g = randn(x0.shape, 3, torch.bfloat16, CUDA)
    y = fn(x)
    (y * g).sum().backward()
    yr = sa.softplus_norm_causal(xr)
    (yr * g).sum().backward()
    assert torch.equal(y, yr) and torch.equal(x.grad, xr.grad)


def test_forward_only_paths_replay():
    B, H, T, D = 1, 4, 320, 64
    q, k, v = (randn((B, H, T, D), i, torch.bfloat16, CUDA) for i in range(3))
    cos, sin = sa.precompute_rope_cos_sin(D, T, device=CUDA)
    fns = [lambda: sa.sp2norm_rope_flash_attention(q, k, v, cos, sin),
           lambda: sa.sp2norm_fp8_flash_attention(q, k, v),
           lambda: sa.softplus_norm_triton(q[0, 0].float())]
    graphs = [_capture(f) for f in fns]
    q.copy_(randn(q.shape, 9, torch.bfloat16, CUDA) * 3)
    v.copy_(randn(v.shape, 8, torch.bfloat16, CUDA))
    for (g, out), f in zip(graphs, fns):
        g.replay()
        torch.cuda.synchronize()
        assert torch.equal(out, f())

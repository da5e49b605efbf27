"""``torch.compile`` over the public API on the GPU: full-graph compiled
forward and backward give the same results as the eager calls (both run the
same sm_100a kernels), and ``torch.library.opcheck`` validates every custom
op's schema and fake implementation against the real one."""

import pytest
import torch

import smooth_attn as sa
from tests._util import randn

pytestmark = pytest.mark.gpu
CUDA = "cuda"
OPS = torch.ops.smooth_attn_b200


@pytest.fixture(autouse=True)
def _need_cuda():
    if not torch.cuda.is_available():
        pytest.skip("CUDA required")
    torch._dynamo.reset()


def _grads(fn, *inputs, seed=7):
    ins = [t.detach().clone().requires_grad_(True) for t in inputs]
    out = fn(*ins)
    g = randn(out.shape, seed, out.dtype, CUDA)
    (out.float() * g.float()).sum().backward()
    return out.detach(), [t.grad for t in ins]


@pytest.mark.parametrize("backend", ["aot_eager", "inductor"])
def test_compiled_flash_fwd_bwd_matches_eager(backend):
    q = randn((2, 8, 384, 128), 1, torch.bfloat16, CUDA)
    k = randn((2, 2, 384, 128), 2, torch.bfloat16, CUDA)
    v = randn((2, 2, 384, 128), 3, torch.bfloat16, CUDA)

    def f(q, k, v):
        return sa.sp2norm_flash_attention(q, k, v, window_size=200) * 2.0

    o_e, g_e = _grads(f, q, k, v)
    o_c, g_c = _grads(torch.compile(f, backend=backend, fullgraph=True), q, k, v)
    assert torch.equal(o_e, o_c)
    for a, b in zip(g_e, g_c):
        torch.testing.assert_close(a, b, rtol=0, atol=0)


@pytest.mark.parametrize("backend", ["aot_eager", "inductor"])
def test_compiled_norm_fwd_bwd_matches_eager(backend):
    x = randn((2, 4, 256, 256), 4, torch.bfloat16, CUDA)

    def f(x):
        return sa.softplus_norm_causal(x) + 1.0

    o_e, (g_e,) = _grads(f, x)
    o_c, (g_c,) = _grads(torch.compile(f, backend=backend, fullgraph=True), x)
    assert torch.equal(o_e, o_c) and torch.equal(g_e, g_c)


def test_compiled_forward_only_paths_match_eager():
    B, Hq, Hkv, T, D = 1, 8, 2, 200, 64
    q, k, v = (randn((B, h, T, D), 10 + h, torch.bfloat16, CUDA) for h in (Hq, Hkv, Hkv))
    cos, sin = sa.precompute_rope_cos_sin(D, T, device=CUDA)
    qd = randn((3, Hq, 1, D), 5, torch.bfloat16, CUDA)
    kc, vc = randn((64, Hkv, 16, D), 6, torch.bfloat16, CUDA), randn((64, Hkv, 16, D), 7, torch.bfloat16, CUDA)
    bt = torch.randperm(64, device=CUDA)[:60].view(3, 20).to(torch.int32)
    cl = torch.tensor([300, 17, 1], device=CUDA, dtype=torch.int32)

    def f(q, k, v, cos, sin, qd, kc, vc, bt, cl):
        return (sa.sp2norm_rope_flash_attention(q, k, v, cos, sin), sa.sp2norm_fp8_flash_attention(q, k, v),
                sa.sp2norm_paged_attention(qd, kc, vc, bt, cl), sa.softplus_norm_triton(q[0, 0].float()))

    args = (q, k, v, cos, sin, qd, kc, vc, bt, cl)
    for a, b in zip(f(*args), torch.compile(f, backend="aot_eager", fullgraph=True)(*args)):
        assert torch.equal(a, b)


def test_opcheck_all_ops():
    q, k, v = (randn((1, h, 130, 64), h, torch.bfloat16, CUDA) for h in (4, 2, 2))
    o, rs, lo = OPS.flash_fwd(q, k, v, 0.125, 0, True, True)
    do = randn(q.shape, 9, torch.bfloat16, CUDA)
    x = randn((2, 96, 96), 3, torch.float32, CUDA)
    y, xr = OPS.norm_fwd(x, 2.0, 0.5, 2, True, True)
    cos, sin = sa.precompute_rope_cos_sin(64, 130, device=CUDA)
    qd = randn((2, 4, 1, 64), 5, torch.bfloat16, CUDA)
    kc, vc = randn((8, 2, 16, 64), 6, torch.bfloat16, CUDA), randn((8, 2, 16, 64), 7, torch.bfloat16, CUDA)
    bt = torch.arange(8, device=CUDA, dtype=torch.int32).view(2, 4)
    cl = torch.tensor([50, 64], device=CUDA, dtype=torch.int32)
    cases = [
        (OPS.norm_fwd, (x, 2.0, 0.5, 2, True, True)),
        (OPS.norm_fwd, (x.view(-1, 96), 2.0, 0.5, 3, False, False)),
        (OPS.norm_causal_bwd, (x, randn(x.shape, 8, torch.float32, CUDA), xr, 2.0, 0.5, 2)),
        (OPS.flash_fwd, (q, k, v, 0.125, 0, True, True)),
        (OPS.flash_fwd, (q, k, v, 0.125, 0, True, False)),
        (OPS.flash_bwd, (q, k, v, o, lo, do, rs, 0.125, 0, True, False)),
        (OPS.flash_bwd, (q, k, v, o, lo, do, rs, 0.125, 0, True, True)),
        (OPS.flash_bwd, (q, k, v, o, o.new_empty(0), do, rs, 0.125, 0, True, False)),
        (OPS.flash_fwd_chunk, (q[:, :, 64:], k, v, 64, 0.125, 0, False, True)),
        (OPS.flash_bwd_chunk, (q[:, :, 64:].contiguous(), k, v, o[:, :, 64:].contiguous(),
                               lo[:, :, 64:].contiguous(), do[:, :, 64:].contiguous(),
                               rs[:, :, 64:].contiguous(), 64, 0.125, 0, False, True)),
        (OPS.rope_flash_fwd, (q, k, v, cos, sin, 0.125, 0)),
        (OPS.out_proj, (q.view(-1, 64)[:192], randn((64, 40), 11, torch.bfloat16, CUDA))),
        (OPS.fp8_flash_fwd, (q, k, v, 0.125, 0)),
        (OPS.paged_decode, (qd, kc, vc, bt, cl, 0.125, 16)),
    ]
    for op, args in cases:
        torch.library.opcheck(op, args)

"""Tracing the public API without a GPU: under ``make_fx`` with fake CUDA
tensors every entry point must reach its ``torch.ops.smooth_attn_b200`` op
(never the ctypes launcher, which needs a data pointer), and each op's fake
implementation must give the shapes, dtypes and strides the API promises.
The compiled runs against the real kernels are in ``test_compile_gpu.py``."""

import pytest
import torch
from torch._subclasses.fake_tensor import FakeTensorMode
from torch.fx.experimental.proxy_tensor import make_fx

import smooth_attn as sa

OPS = torch.ops.smooth_attn_b200


@pytest.fixture
def fake():
    with FakeTensorMode() as m:
        yield m


def _t(*shape, dtype=torch.bfloat16):
    return torch.randn(*shape, device="cuda", dtype=dtype)


def _targets(g):
    return [str(n.target) for n in g.graph.nodes if n.op == "call_function"]


def _trace(fn, *args):
    return make_fx(fn, tracing_mode="fake")(*args)


def test_flash_and_norm_trace_to_custom_ops(fake):
    q, k, v = _t(2, 4, 256, 64), _t(2, 2, 256, 64), _t(2, 2, 256, 64)
    x = _t(2, 3, 128, 128)

    def f(q, k, v, x):
        return (sa.sp2norm_flash_attention(q, k, v, window_size=64), sa.softplus_norm_causal(x),
                sa.softplus_norm_causal_triton(x), sa.softplus_norm_triton(x.view(-1, 128)))

    g = _trace(f, q, k, v, x)
    t = _targets(g)
    assert t.count("smooth_attn_b200.flash_fwd.default") == 1
    assert t.count("smooth_attn_b200.norm_fwd.default") == 3
    outs = f(q, k, v, x)
    assert outs[0].shape == q.shape and outs[0].dtype == q.dtype
    assert all(o.shape == x.shape for o in outs[1:3]) and outs[3].shape == (6 * 128, 128)


def test_out_variants_trace_as_op_plus_copy(fake):
    x = _t(2, 64, 64, dtype=torch.float32)

    def f(x):
        out = torch.empty_like(x)
        return sa.softplus_norm_causal_triton_out(out, x)

    t = _targets(_trace(f, x))
    assert "smooth_attn_b200.norm_fwd.default" in t and "aten.copy_.default" in t


def test_forward_only_paths_trace(fake):
    B, Hq, Hkv, T, D = 2, 8, 2, 128, 64
    q, k, v = _t(B, Hq, T, D), _t(B, Hkv, T, D), _t(B, Hkv, T, D)
    cos, sin = _t(T, D // 2, dtype=torch.float32), _t(T, D // 2, dtype=torch.float32)
    w_o = _t(Hq, D, 256)
    qd = _t(B, Hq, 1, D)
    kc, vc = _t(40, Hkv, 16, D), _t(40, Hkv, 16, D)
    bt = torch.zeros(B, 20, dtype=torch.int32, device="cuda")
    cl = torch.full((B,), 300, dtype=torch.int32, device="cuda")

    def f(q, k, v, cos, sin, w_o, qd, kc, vc, bt, cl):
        return (sa.sp2norm_rope_flash_attention(q, k, v, cos, sin),
                sa.sp2norm_rope_flash_attention_proj(q, k, v, w_o, cos, sin),
                sa.sp2norm_fp8_flash_attention(q, k, v),
                sa.sp2norm_paged_attention(qd, kc, vc, bt, cl))

    args = (q, k, v, cos, sin, w_o, qd, kc, vc, bt, cl)
    t = _targets(_trace(f, *args))
    for op, n in (("rope_flash_fwd", 2), ("fp8_flash_fwd", 1), ("paged_decode", 1)):
        assert t.count(f"smooth_attn_b200.{op}.default") == n, (op, t)
    o_rope, o_proj, o_fp8, o_dec = f(*args)
    assert o_rope.shape == q.shape and o_proj.shape == (B, T, 256) and o_proj.dtype == torch.bfloat16
    assert o_fp8.shape == q.shape and o_fp8.dtype == torch.bfloat16
    assert o_dec.shape == (B, Hq, D) and o_dec.dtype == torch.bfloat16


def test_backward_ops_fake_shapes(fake):
    q, k, v = _t(1, 8, 96, 128, dtype=torch.float16), _t(1, 2, 96, 128, dtype=torch.float16), _t(1, 2, 96, 128,
                                                                                                   dtype=torch.float16)
    o, rs, lo = OPS.flash_fwd(q, k, v, 0.1, 0, True, True)
    assert o.shape == q.shape and o.is_contiguous() and rs.shape == (1, 8, 96) and rs.dtype == torch.float32
    assert lo.shape == o.shape and lo.dtype == o.dtype
    assert OPS.flash_fwd(q, k, v, 0.1, 0, True, False)[2].numel() == 0
    dq, dk, dv = OPS.flash_bwd(q, k, v, o, lo, torch.randn_like(o), rs, 0.1, 0, True, False)
    assert (dq.shape, dk.shape, dv.shape) == (q.shape, k.shape, v.shape)
    assert all(t.dtype == torch.float16 and t.is_contiguous() for t in (dq, dk, dv))
    x = _t(3, 50, 50)
    y, rsum = OPS.norm_fwd(x, 2.0, 0.5, 2, True, True)
    assert y.shape == x.shape and rsum.shape == (150,)
    assert OPS.norm_fwd(x, 2.0, 0.5, 2, True, False)[1].numel() == 0
    dx = OPS.norm_causal_bwd(x, torch.randn_like(x), rsum, 2.0, 0.5, 2)
    assert dx.shape == x.shape and dx.dtype == x.dtype


def test_chunk_paths_trace(fake):
    q, k, v = _t(1, 4, 128, 64), _t(1, 2, 384, 64), _t(1, 2, 384, 64)

    def f(q, k, v):
        o, rs = sa.sp2norm_flash_attention_chunk(q, k, v, 256)
        return (o, rs) + sa.kernels.sp2norm_flash_attention_chunk_bwd(q, k, v, o, torch.ones_like(o), rs, 256)

    t = _targets(_trace(f, q, k, v))
    assert "smooth_attn_b200.flash_fwd_chunk.default" in t and "smooth_attn_b200.flash_bwd_chunk.default" in t
    o, rs, dq, dk, dv = f(q, k, v)
    assert o.shape == q.shape and rs.shape == (1, 4, 128)
    assert (dq.shape, dk.shape, dv.shape) == (q.shape, k.shape, v.shape)


def test_validation_still_runs_under_tracing(fake):
    q = _t(1, 2, 64, 48)
    with pytest.raises(ValueError):
        _trace(lambda a: sa.sp2norm_flash_attention(a, a, a), q)
    with pytest.raises(ValueError):
        _trace(lambda a: sa.softplus_norm_causal(a), _t(2, 8, 4))

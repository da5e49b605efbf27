"""Parity of the CUDA normalization kernels (forward + fused backward) with the
numpy oracle and the committed golden vectors.  Mirrors the reference's
``tests/test_training_api.py:19-78`` plus odd sizes, all dtypes, all powers,
strided outputs and full-size (BASELINE config) property checks."""

from pathlib import Path

import numpy as np
import pytest
import torch

import smooth_attn as sa
from oracle import sa_oracle as O
from tests._util import TOL, assert_close, np32, randn

pytestmark = pytest.mark.gpu
CUDA = "cuda"
G = np.load(Path(__file__).parent / "golden" / "golden.npz")

FAMS = [sa.FamilyConfig(), sa.FamilyConfig(1.5, 0.25, 3), sa.FamilyConfig(0.7, -0.3, 1)]


@pytest.fixture(autouse=True)
def _need_cuda():
    if not torch.cuda.is_available():
        pytest.skip("CUDA required")


def _fwd_ref(x, fam):
    return O.softplus_norm_causal(np32(x), fam.alpha, fam.theta, fam.power)


@pytest.mark.parametrize("dtype", [torch.float32, torch.float16, torch.bfloat16])
@pytest.mark.parametrize("L", [1, 2, 3, 7, 8, 17, 64, 127, 128, 129, 256, 1000, 2048, 4096])
def test_causal_fwd_matches_oracle(dtype, L):
    B, H = (1, 1) if L >= 2048 else (2, 3)
    x = randn((B, H, L, L), seed=L, dtype=dtype, device=CUDA)
    out = torch.empty_like(x)
    y, meta = sa.softplus_norm_causal_triton_out(out, x, return_meta=True)
    assert y.data_ptr() == out.data_ptr()
    assert meta["variant"].startswith("squareplus_winner")
    ref = _fwd_ref(x, sa.DEFAULT_FAMILY)
    assert_close(np32(y), ref, **TOL[dtype])
    yn = np32(y)
    assert np.all(yn[..., ~O.causal_mask(L)] == 0.0), "upper triangle must be exact zeros"


@pytest.mark.parametrize("fam", FAMS, ids=["p2", "p3", "p1"])
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_causal_fwd_families(fam, dtype):
    x = randn((2, 2, 96, 96), seed=11, dtype=dtype, device=CUDA)
    y = sa.softplus_norm_causal_triton(x, family=fam)
    assert_close(np32(y), _fwd_ref(x, fam), **TOL[dtype])


# reference tests/test_training_api.py:36-60
@pytest.mark.parametrize(("seq_len", "family", "atol"), [
    (64, sa.FamilyConfig(), 5e-3), (512, sa.FamilyConfig(), 5e-3),
    (128, sa.FamilyConfig(alpha=1.5, theta=0.25, power=3), 7e-3)])
def test_causal_matches_eager_reference_case(seq_len, family, atol):
    x = randn((1, 2, seq_len, seq_len), seed=seq_len, dtype=torch.bfloat16, device=CUDA)
    out = torch.empty_like(x)
    y, meta = sa.softplus_norm_causal_triton_out(out, x, family=family, return_meta=True)
    ref = sa.softplus_norm_causal_eager(x.float(), family=family)
    torch.testing.assert_close(y.float(), ref, atol=atol, rtol=5e-2)
    torch.testing.assert_close(y.float().sum(-1), torch.ones_like(ref.sum(-1)), atol=atol, rtol=0.0)
    if family == sa.FamilyConfig():
        assert meta["variant"].startswith("squareplus_winner")


@pytest.mark.parametrize("name", sorted({k.split("/")[0] for k in G.files if k.startswith("c_")}))
def test_causal_golden(name):
    a, t, p = G[f"{name}/family"]
    fam = sa.FamilyConfig(float(a), float(t), int(p))
    dtype = torch.bfloat16 if name.endswith("bf16") else torch.float32
    x = torch.from_numpy(G[f"{name}/x"]).to(dtype).to(CUDA).requires_grad_(True)
    y = sa.softplus_norm_causal(x, family=fam)
    tol = TOL[dtype]
    assert_close(np32(y), G[f"{name}/out"], **tol)
    g = torch.from_numpy(G[f"{name}/g"]).to(CUDA)
    (y.float() * g).sum().backward()
    ref = G[f"{name}/dx"]
    if dtype == torch.float32:
        assert_close(np32(x.grad), ref, rtol=1e-5, atol=1e-6 * max(1.0, np.abs(ref).max()))
    else:
        assert_close(np32(x.grad), ref, rtol=2e-2, atol=1e-2)


@pytest.mark.parametrize("name", sorted({k.split("/")[0] for k in G.files if k.startswith("r_")}))
def test_rowwise_golden(name):
    a, t, p = G[f"{name}/family"]
    x = torch.from_numpy(G[f"{name}/x"]).to(CUDA)
    y = sa.softplus_norm_triton(x, alpha=float(a), theta=float(t), power=int(p))
    assert_close(np32(y), G[f"{name}/out"], **TOL[torch.float32])


@pytest.mark.parametrize("dtype", [torch.float32, torch.float16, torch.bfloat16])
@pytest.mark.parametrize("shape", [(1, 1), (3, 5), (64, 96), (256, 1024), (17, 2048), (9, 4096), (4, 4095)])
def test_rowwise_fwd(dtype, shape):
    x = randn(shape, seed=shape[1], dtype=dtype, device=CUDA)
    out = torch.empty_like(x)
    y = sa.softplus_norm_triton_out(out, x)
    assert_close(np32(y), O.softplus_norm(np32(x)), **TOL[dtype])


def test_rowwise_rejects_4d_and_wide():
    with pytest.raises(ValueError):
        sa.softplus_norm_triton(torch.zeros(2, 2, 4, 4, device=CUDA))
    with pytest.raises(ValueError, match="too large"):
        sa.softplus_norm_triton(torch.zeros(2, 4097, device=CUDA))


def test_out_validation_and_noncontiguous_out():
    x = randn((2, 2, 32, 32), seed=5, device=CUDA)
    with pytest.raises(ValueError):
        sa.softplus_norm_causal_triton_out(torch.empty(2, 2, 32, 31, device=CUDA), x)
    with pytest.raises(ValueError):
        sa.softplus_norm_causal_triton_out(torch.empty_like(x, dtype=torch.float16), x)
    base = torch.zeros(2, 2, 32, 64, device=CUDA)
    out = base[..., :32]  # non-contiguous
    y = sa.softplus_norm_causal_triton_out(out, x)
    assert y.data_ptr() == out.data_ptr()
    assert_close(np32(out), _fwd_ref(x, sa.DEFAULT_FAMILY), **TOL[torch.float32])
    assert torch.all(base[..., 32:] == 0)


def test_noncontiguous_input():
    xb = randn((2, 64, 64), seed=6, device=CUDA).transpose(-1, -2)
    assert not xb.is_contiguous()
    y = sa.softplus_norm_causal_triton(xb)
    assert_close(np32(y), _fwd_ref(xb.contiguous(), sa.DEFAULT_FAMILY), **TOL[torch.float32])


def test_output_canaries_untouched():
    """Kernel writes exactly rows*cols elements: canaries around the output survive."""
    L = 40
    x = randn((3, L, L), seed=8, dtype=torch.bfloat16, device=CUDA)
    buf = torch.full((3 * L * L + 64,), 7.0, device=CUDA, dtype=torch.bfloat16)
    out = buf[32:32 + 3 * L * L].view(3, L, L)
    sa.softplus_norm_causal_triton_out(out, x)
    assert torch.all(buf[:32] == 7.0) and torch.all(buf[-32:] == 7.0)


# ---- backward -----------------------------------------------------------


def _bwd_check(x, g, fam, dtype):
    xr = x.detach().clone().requires_grad_(True)
    y = sa.softplus_norm_causal(xr, family=fam)
    y.backward(g)
    ref = O.softplus_norm_causal_bwd(np32(x), np32(g), fam.alpha, fam.theta, fam.power)
    scale = max(1.0, float(np.abs(ref).max()))
    if dtype == torch.float32:
        assert_close(np32(xr.grad), ref, rtol=1e-5, atol=1e-6 * scale)
    else:
        assert_close(np32(xr.grad), ref, rtol=2e-2, atol=1e-2)
    assert xr.grad.dtype == x.dtype
    L = x.shape[-1]
    assert np.all(np32(xr.grad)[..., ~O.causal_mask(L)] == 0.0)


@pytest.mark.parametrize("dtype", [torch.float32, torch.float16, torch.bfloat16])
@pytest.mark.parametrize("L", [1, 5, 32, 129, 512, 2048])
def test_causal_bwd_matches_oracle(dtype, L):
    B, H = (1, 1) if L >= 2048 else (2, 2)
    x = randn((B, H, L, L), seed=100 + L, dtype=dtype, device=CUDA)
    g = randn((B, H, L, L), seed=200 + L, dtype=dtype, device=CUDA)
    _bwd_check(x, g, sa.DEFAULT_FAMILY, dtype)


@pytest.mark.parametrize("fam", FAMS, ids=["p2", "p3", "p1"])
def test_causal_bwd_families_fp32_grad(fam):
    x = randn((1, 2, 80, 80), seed=3, dtype=torch.bfloat16, device=CUDA)
    g = randn((1, 2, 80, 80), seed=4, dtype=torch.float32, device=CUDA)  # fp32 upstream on bf16 x
    _bwd_check(x, g, fam, torch.bfloat16)


# reference tests/test_training_api.py:63-78
def test_backward_matches_eager_reference():
    family = sa.FamilyConfig()
    x = randn((1, 2, 32, 32), seed=9, dtype=torch.bfloat16, device=CUDA).requires_grad_(True)
    upstream = randn((1, 2, 32, 32), seed=10, device=CUDA)
    (sa.softplus_norm_causal(x, family=family).float() * upstream).sum().backward()
    x_ref = x.detach().clone().requires_grad_(True)
    (sa.softplus_norm_causal_eager(x_ref.float(), family=family) * upstream).sum().backward()
    torch.testing.assert_close(x.grad.float(), x_ref.grad.float(), atol=5e-3, rtol=5e-2)


def test_module_and_mini_attention_example():
    """examples/mini_attention.py: SoftplusNormCausal -> @ V -> backward."""
    op = sa.SoftplusNormCausal(family=sa.FamilyConfig(alpha=2.0, theta=0.5, power=2))
    scores = randn((2, 8, 512, 512), seed=1, dtype=torch.bfloat16, device=CUDA).requires_grad_(True)
    values = randn((2, 8, 512, 64), seed=2, dtype=torch.bfloat16, device=CUDA)
    attn = op(scores)
    loss = (attn @ values).float().pow(2).mean()
    loss.backward()
    assert attn.shape == scores.shape and torch.isfinite(scores.grad.float()).all()


# ---- full-size BASELINE configs: size-independent properties --------------


def test_baseline_config2_full_size_properties():
    """bf16 [8,16,2048,2048]: rows sum to 1, exact-zero upper triangle, a sampled
    slice equals the oracle, and a second launch is bitwise identical."""
    x = randn((8, 16, 2048, 2048), seed=1234, dtype=torch.bfloat16, device=CUDA)
    out = torch.empty_like(x)
    sa.softplus_norm_causal_triton_out(out, x)
    sums = out.float().sum(-1)
    assert torch.allclose(sums, torch.ones_like(sums), atol=2e-2)
    upper = torch.triu(torch.ones(2048, 2048, dtype=torch.bool, device=CUDA), 1)
    assert int(out[:, :, upper].count_nonzero()) == 0
    assert_close(np32(out[3, 7]), _fwd_ref(x[3, 7], sa.DEFAULT_FAMILY), **TOL[torch.bfloat16])
    out2 = torch.empty_like(x)
    sa.softplus_norm_causal_triton_out(out2, x)
    assert torch.equal(out, out2)


def test_baseline_config3_bwd_slice_and_linearity():
    """bf16 [4,32,2048,2048] fwd+bwd: sampled slices match the oracle, and the
    backward is linear in dY (bwd(2 g) == 2 bwd(g) exactly in fp32 math)."""
    x = randn((4, 32, 2048, 2048), seed=77, dtype=torch.bfloat16, device=CUDA).requires_grad_(True)
    g = randn((4, 32, 2048, 2048), seed=78, dtype=torch.bfloat16, device=CUDA)
    y = sa.softplus_norm_causal(x)
    y.backward(g)
    for b, h in ((0, 0), (3, 31)):
        ref = O.softplus_norm_causal_bwd(np32(x[b, h]), np32(g[b, h]))
        assert_close(np32(x.grad[b, h]), ref, rtol=2e-2, atol=1e-2)
    gx = x.grad.clone()
    x.grad = None
    y = sa.softplus_norm_causal(x)
    y.backward(g * 2)
    assert torch.equal(x.grad, gx * 2)


def test_zz_no_device_timeouts_recorded():
    """No bounded device-side wait of the library gave up during this module."""
    from smooth_attn import _lib

    assert _lib.load().sa_device_status(1) == _lib.SA_OK

"""Parity of the sm_100a paged-KV decode kernel (``sa_paged_decode`` through
``sp2norm_paged_attention``) with the numpy oracle and the committed golden
vectors.  Mirrors the reference's ``tests/test_paged_attention.py`` (basic,
shuffled pages, GQA, variable context lengths, page sizes 8-64) and
``tests/test_paged_long_context.py`` (to 8K checked, 32K NaN/Inf-free), plus
head dims 32-256, fp16, non-power-of-two GQA groups, empty and ragged
contexts, NaN-filled unused page rows, split-KV ticket reuse and an
out-of-range page index."""

from pathlib import Path

import numpy as np
import pytest
import torch

import smooth_attn as sa
from smooth_attn import _lib
from oracle import sa_oracle as O
from tests._util import TOL, assert_close, np32, randn

pytestmark = pytest.mark.gpu
CUDA = "cuda"
G = np.load(Path(__file__).parent / "golden" / "golden.npz")


@pytest.fixture(autouse=True)
def _need_cuda():
    if not torch.cuda.is_available():
        pytest.skip("CUDA required")


def _paged(k, v, bs, seed, fill=0.0, spare=0):
    """Scatter contiguous [B, Hkv, T, D] K/V into shuffled pages of ``bs``
    rows (as the reference's _build_paged_kv_cache_shuffled does); unused
    rows and ``spare`` extra pages hold ``fill``."""
    B, Hkv, T, D = k.shape
    nps = (T + bs - 1) // bs
    total = B * nps + spare
    kc = torch.full((total, Hkv, bs, D), fill, dtype=k.dtype, device=k.device)
    vc = torch.full_like(kc, fill)
    perm = torch.randperm(total, generator=torch.Generator().manual_seed(seed))
    bt = torch.zeros(B, nps, dtype=torch.int32)
    for b in range(B):
        for blk in range(nps):
            phys = int(perm[b * nps + blk])
            bt[b, blk] = phys
            s, e = blk * bs, min(blk * bs + bs, T)
            kc[phys, :, : e - s] = k[b, :, s:e]
            vc[phys, :, : e - s] = v[b, :, s:e]
    cl = torch.full((B,), T, dtype=torch.int32)
    return kc, vc, bt.to(k.device), cl.to(k.device)


def _case(B, Hq, Hkv, T, D, bs, seed, dtype=torch.bfloat16, fill=0.0):
    q = randn((B, Hq, 1, D), seed, dtype, CUDA)
    k = randn((B, Hkv, T, D), seed + 1, dtype, CUDA)
    v = randn((B, Hkv, T, D), seed + 2, dtype, CUDA)
    kc, vc, bt, cl = _paged(k, v, bs, seed + 3, fill=fill)
    return q, kc, vc, bt, cl


def _ref(q, kc, vc, bt, cl, scale=None):
    return O.paged_decode_attention(np32(q), np32(kc), np32(vc), bt.cpu().numpy(), cl.cpu().numpy(), scale=scale)


def _check(out, ref, dtype=torch.bfloat16):
    assert out.dtype == torch.bfloat16
    assert torch.isfinite(out).all()
    assert_close(np32(out), ref, **TOL[dtype])


@pytest.mark.parametrize("name", sorted({k.split("/")[0] for k in G.files if k.startswith("p_")}))
def test_paged_golden(name):
    """Golden vectors of the reference's decode reference on shuffled pages."""
    t = lambda s, dt=torch.bfloat16: torch.from_numpy(G[f"{name}/{s}"]).to(CUDA, dt)
    q, kc, vc = t("q"), t("k_cache"), t("v_cache")
    bt, cl = t("block_table", torch.int32), t("context_lens", torch.int32)
    out = sa.sp2norm_paged_attention(q, kc, vc, bt, cl, block_size=kc.shape[2])
    _check(out, G[f"{name}/out"])


# tests/test_paged_attention.py:112-139 (basic) and :142-166 (shuffled)
@pytest.mark.parametrize("B,H,T,D,bs", [(1, 4, 64, 32, 16), (2, 4, 128, 32, 16), (2, 8, 256, 64, 16),
                                        (1, 4, 48, 32, 16), (4, 8, 256, 64, 16), (2, 4, 100, 128, 16)])
def test_paged_basic(B, H, T, D, bs):
    q, kc, vc, bt, cl = _case(B, H, H, T, D, bs, seed=B * 1000 + T + D)
    _check(sa.sp2norm_paged_attention(q, kc, vc, bt, cl, block_size=bs), _ref(q, kc, vc, bt, cl))


# tests/test_paged_attention.py:169-191 (GQA) plus non-power-of-two groups
@pytest.mark.parametrize("Hq,Hkv,D", [(8, 2, 32), (32, 8, 128), (12, 4, 64), (6, 1, 128), (16, 1, 128),
                                      (32, 2, 64), (24, 8, 256), (8, 8, 256), (20, 4, 32)])
def test_paged_gqa(Hq, Hkv, D):
    q, kc, vc, bt, cl = _case(2, Hq, Hkv, 160, D, 16, seed=Hq * 7 + Hkv + D)
    _check(sa.sp2norm_paged_attention(q, kc, vc, bt, cl, block_size=16), _ref(q, kc, vc, bt, cl))


# tests/test_paged_attention.py:194-226: sequences of different lengths
def test_paged_variable_context_lens():
    B, H, T, D, bs = 4, 4, 128, 32, 16
    q, kc, vc, bt, cl = _case(B, H, H, T, D, bs, seed=77)
    cl = torch.tensor([32, 64, 48, 128], dtype=torch.int32, device=CUDA)
    _check(sa.sp2norm_paged_attention(q, kc, vc, bt, cl, block_size=bs), _ref(q, kc, vc, bt, cl))


@pytest.mark.parametrize("lens", [[0, 1, 17, 5000], [1, 1, 1, 1], [4999, 0, 33, 2048]])
def test_paged_ragged_and_empty(lens):
    """Empty sequences give exact zeros (0 / 1e-12); partial last pages are
    masked; the long sequence splits over many CTAs while others are short."""
    B, H, Hkv, T, D, bs = 4, 8, 2, 5000, 128, 16
    q, kc, vc, bt, cl = _case(B, H, Hkv, T, D, bs, seed=sum(lens) % 1000, fill=float("nan"))
    cl = torch.tensor(lens, dtype=torch.int32, device=CUDA)
    out = sa.sp2norm_paged_attention(q, kc, vc, bt, cl, block_size=bs)
    ref = _ref(q, kc.nan_to_num(0.0), vc.nan_to_num(0.0), bt, cl)
    _check(out, ref)
    for b, n in enumerate(lens):
        if n == 0:
            assert (out[b] == 0).all()


# tests/test_paged_attention.py:229-251: page sizes
@pytest.mark.parametrize("bs", [8, 16, 32, 64, 128])
@pytest.mark.parametrize("D", [64, 128, 256])
def test_paged_block_sizes(bs, D):
    q, kc, vc, bt, cl = _case(2, 8, 4, 300, D, bs, seed=bs + D, fill=float("nan"))
    out = sa.sp2norm_paged_attention(q, kc, vc, bt, cl, block_size=bs)
    _check(out, _ref(q, kc.nan_to_num(0.0), vc.nan_to_num(0.0), bt, cl))


def test_paged_odd_block_size():
    """A page size that is not a power of two (rows per chunk divides it)."""
    q, kc, vc, bt, cl = _case(2, 4, 2, 200, 256, 24, seed=24, fill=float("nan"))
    out = sa.sp2norm_paged_attention(q, kc, vc, bt, cl, block_size=24)
    _check(out, _ref(q, kc.nan_to_num(0.0), vc.nan_to_num(0.0), bt, cl))


def test_paged_fp16_and_scale():
    q, kc, vc, bt, cl = _case(3, 8, 2, 333, 128, 16, seed=5, dtype=torch.float16)
    out = sa.sp2norm_paged_attention(q, kc, vc, bt, cl, scale=0.05, block_size=16)
    _check(out, _ref(q, kc, vc, bt, cl, scale=0.05), torch.float16)


# tests/test_paged_long_context.py:83-116: to 8K against the reference math
@pytest.mark.parametrize("T", [1024, 2048, 4096, 8192])
def test_paged_long_context(T):
    q, kc, vc, bt, cl = _case(1, 8, 2, T, 64, 16, seed=T)
    _check(sa.sp2norm_paged_attention(q, kc, vc, bt, cl, block_size=16), _ref(q, kc, vc, bt, cl))


# tests/test_paged_long_context.py:119-168: 16K-32K run without NaN/Inf
@pytest.mark.parametrize("T", [16384, 32768])
def test_paged_very_long_context(T):
    H, Hkv, D, bs = 32, 8, 128, 16
    nb = T // bs
    q = randn((1, H, 1, D), T, torch.bfloat16, CUDA)
    kc = randn((nb, Hkv, bs, D), T + 1, torch.bfloat16, CUDA)
    vc = randn((nb, Hkv, bs, D), T + 2, torch.bfloat16, CUDA)
    bt = torch.randperm(nb, generator=torch.Generator().manual_seed(T)).to(torch.int32).view(1, nb).to(CUDA)
    cl = torch.full((1,), T, dtype=torch.int32, device=CUDA)
    out = sa.sp2norm_paged_attention(q, kc, vc, bt, cl, block_size=bs)
    assert torch.isfinite(out).all() and out.float().norm() > 0
    _check(out, _ref(q, kc, vc, bt, cl))


def test_paged_split_tickets_reset():
    """Back-to-back split-KV calls on one stream reuse the ticket words; each
    call must leave them zero so the next combines correctly."""
    q, kc, vc, bt, cl = _case(1, 32, 8, 4096, 128, 16, seed=9)
    lib = _lib.load()
    assert lib.sa_paged_decode_workspace_size(1, 32, 8, bt.shape[1], 16, 128, _lib.SA_BF16) > 0  # splits
    ref = _ref(q, kc, vc, bt, cl)
    outs = [sa.sp2norm_paged_attention(q, kc, vc, bt, cl, block_size=16) for _ in range(5)]
    for o in outs:
        _check(o, ref)
        assert torch.equal(o, outs[0])


@pytest.mark.parametrize("B,T", [(64, 200), (300, 40), (7, 3000)])
def test_paged_many_sequences(B, T):
    """Many short sequences: CTA ranges hold several whole units and cut
    others, so both the direct and the combined output paths run."""
    q, kc, vc, bt, cl = _case(B, 32, 8, T, 128, 16, seed=B + T)
    _check(sa.sp2norm_paged_attention(q, kc, vc, bt, cl, block_size=16), _ref(q, kc, vc, bt, cl))


def test_paged_bad_page_index_reported():
    """A block_table entry outside the cache is read as page 0 (never out of
    bounds) and reported by sa_device_status as SA_ERR_ARG."""
    lib = _lib.load()
    lib.sa_device_status(1)
    q, kc, vc, bt, cl = _case(1, 4, 4, 64, 64, 16, seed=3)
    bt[0, 1] = kc.shape[0] + 100
    sa.sp2norm_paged_attention(q, kc, vc, bt, cl, block_size=16)
    assert lib.sa_device_status(1) == _lib.SA_ERR_ARG
    assert lib.sa_device_status(0) == _lib.SA_OK


@pytest.mark.parametrize("B,Hq,Hkv,T,bs", [(2, 32, 8, 1000, 16), (1, 16, 2, 4100, 8), (3, 12, 4, 517, 32),
                                           (1, 64, 4, 300, 64), (2, 8, 4, 129, 128), (4, 40, 2, 2222, 16)])
def test_paged_tensor_core_and_simt_kernels(monkeypatch, B, Hq, Hkv, T, bs):
    """bf16 D=128 GQA shapes run on the tensor-core kernel by default; the
    CUDA-core kernel (SA_PAGED_DECODE_KERNEL=simt) must agree, and both match
    the oracle (ragged last tiles, NaN-filled unused page rows, G up to 20)."""
    q, kc, vc, bt, cl = _case(B, Hq, Hkv, T, 128, bs, seed=B * T + bs, fill=float("nan"))
    cl = torch.tensor([max(1, T - 37 * i) for i in range(B)], dtype=torch.int32, device=CUDA)
    ref = _ref(q, kc.nan_to_num(0.0), vc.nan_to_num(0.0), bt, cl)
    out_tc = sa.sp2norm_paged_attention(q, kc, vc, bt, cl, block_size=bs)
    monkeypatch.setenv("SA_PAGED_DECODE_KERNEL", "simt")
    out_simt = sa.sp2norm_paged_attention(q, kc, vc, bt, cl, block_size=bs)
    _check(out_tc, ref)
    _check(out_simt, ref)
    assert (out_tc.float() - out_simt.float()).abs().max() <= 2e-2


def test_paged_rejects_bad_arguments():
    q, kc, vc, bt, cl = _case(1, 4, 4, 64, 64, 16, seed=4)
    with pytest.raises(AssertionError):
        sa.sp2norm_paged_attention(q.squeeze(2), kc, vc, bt, cl)
    with pytest.raises(AssertionError):
        sa.sp2norm_paged_attention(q, kc, vc, bt, cl, block_size=8)
    with pytest.raises(ValueError):
        sa.sp2norm_paged_attention(q.float(), kc.float(), vc.float(), bt, cl)
    q3, kc3, vc3, bt3, cl3 = _case(1, 4, 4, 64, 48, 16, seed=4)
    with pytest.raises(ValueError):
        sa.sp2norm_paged_attention(q3, kc3, vc3, bt3, cl3)
    # the C ABI rejects before launching
    st = _lib.load().sa_paged_decode(q.data_ptr(), kc.data_ptr(), vc.data_ptr(), q.data_ptr(), bt.data_ptr(),
                                     cl.data_ptr(), None, 0, 1, 4, 3, kc.shape[0], 16, bt.shape[1], 64,
                                     0.125, _lib.SA_BF16, None)
    assert st == _lib.SA_ERR_ARG

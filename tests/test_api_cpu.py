"""Host-side behaviour that needs no GPU: API surface, family config, the
reference's error conventions, the eager functions, and the C ABI library's
exported symbols."""

import ctypes
import re
from pathlib import Path

import numpy as np
import pytest
import torch

import smooth_attn as sa
from oracle import sa_oracle as O
from smooth_attn import _lib

ROOT = Path(__file__).resolve().parents[1]

REFERENCE_ALL = [
    "BENCH_ALPHA", "BENCH_POWER", "BENCH_THETA", "DEFAULT_FAMILY", "CausalBenchmarkResult", "FamilyConfig",
    "RowwiseBenchmarkResult", "SoftplusNormCausal", "bench", "bench_out", "benchmark_causal_suite",
    "benchmark_rowwise_suite", "main", "softmax_causal_eager", "softmax_causal_triton", "softmax_causal_triton_out",
    "softmax_triton", "softmax_triton_out", "softplus_norm_causal", "softplus_norm_causal_eager",
    "softplus_norm_causal_triton", "softplus_norm_causal_triton_out", "softplus_norm_eager", "softplus_norm_triton",
    "softplus_norm_triton_out", "sp2norm_flash_attention", "sp2norm_flash_attention_eager",
    "sp2norm_fp8_flash_attention", "sp2norm_rope_flash_attention", "sp2norm_rope_flash_attention_proj",
    "sp2norm_paged_attention", "precompute_rope_cos_sin", "sp2norm_triton",
]


def test_public_names_match_reference():
    assert sorted(sa.__all__) == sorted(REFERENCE_ALL)
    for name in REFERENCE_ALL:
        assert hasattr(sa, name), name


# tests/test_family_config.py of the reference
def test_family_config_rejects_bad_power():
    with pytest.raises(ValueError):
        sa.FamilyConfig(power=4)


def test_family_config_rejects_removed_activation_kwarg():
    with pytest.raises(TypeError):
        sa.FamilyConfig(activation="softplus")


def test_family_config_properties():
    f = sa.FamilyConfig(alpha=1.5, theta=0.25, power=3)
    assert f.cache_key == (1.5, 0.25, 3)
    assert f.kernel_kwargs == {"ALPHA": 1.5, "THETA": 0.25, "POWER": 3}
    assert f.label == "squareplus(1.5 * (x - 0.25))^3 / sum"
    assert sa.DEFAULT_FAMILY == sa.FamilyConfig(2.0, 0.5, 2)
    assert (sa.BENCH_ALPHA, sa.BENCH_THETA, sa.BENCH_POWER) == (2.0, 0.5, 2)


def test_family_and_overrides_conflict():
    x = torch.zeros(4, 4)
    with pytest.raises(ValueError, match="not both"):
        sa.softplus_norm_causal_eager(x, alpha=1.0, family=sa.DEFAULT_FAMILY)


@pytest.mark.parametrize("fn", [sa.softplus_norm_causal_triton, sa.softplus_norm_triton, sa.sp2norm_triton])
def test_non_tensor_raises_type_error(fn):
    with pytest.raises(TypeError):
        fn([[1.0]])


def test_cpu_tensor_raises_value_error():
    with pytest.raises(ValueError, match="CUDA"):
        sa.softplus_norm_causal_triton(torch.zeros(2, 4, 4))
    with pytest.raises(ValueError, match="CUDA"):
        sa.softplus_norm_causal_triton_out(torch.zeros(2, 4, 4), torch.zeros(2, 4, 4))
    with pytest.raises(ValueError, match="CUDA"):
        sa.softplus_norm_causal(torch.zeros(2, 4, 4))


def test_flash_asserts_shapes():
    q = torch.zeros(1, 4, 8, 32)
    with pytest.raises(AssertionError):
        sa.sp2norm_flash_attention(q, torch.zeros(1, 3, 8, 32), torch.zeros(1, 3, 8, 32))
    with pytest.raises(AssertionError):
        sa.sp2norm_flash_attention(q[0], q[0], q[0])
    with pytest.raises(ValueError, match="CUDA"):
        sa.sp2norm_flash_attention(q, q, q)


def test_bad_implementation():
    with pytest.raises(ValueError, match="implementation"):
        sa.softplus_norm_causal(torch.zeros(4, 4), implementation="cuda")


def test_extensions_refuse_host_tensors():
    """RoPE / FP8 / paged entry points exist under the reference's names and
    refuse CPU tensors (there is no CPU fallback)."""
    q = torch.zeros(1, 2, 64, 32, dtype=torch.bfloat16)
    cos, sin = sa.precompute_rope_cos_sin(32, 64, device="cpu")
    with pytest.raises(ValueError, match="CUDA"):
        sa.sp2norm_fp8_flash_attention(q, q, q)
    with pytest.raises(ValueError, match="CUDA"):
        sa.sp2norm_rope_flash_attention(q, q, q, cos, sin)
    with pytest.raises(ValueError, match="CUDA"):
        sa.sp2norm_rope_flash_attention_proj(q, q, q, torch.zeros(2, 32, 64), cos, sin)


def test_paged_decode_rejects_cpu_tensors():
    """The decode wrapper keeps the reference's shape asserts
    (kernels.py:2793-2797) and refuses host tensors (no CPU fallback)."""
    q = torch.zeros(1, 4, 1, 64, dtype=torch.bfloat16)
    kc = torch.zeros(4, 4, 16, 64, dtype=torch.bfloat16)
    bt = torch.zeros(1, 4, dtype=torch.int32)
    cl = torch.full((1,), 64, dtype=torch.int32)
    with pytest.raises(AssertionError):
        sa.sp2norm_paged_attention(q[:, :, 0], kc, kc, bt, cl)
    with pytest.raises(AssertionError):
        sa.sp2norm_paged_attention(q, kc, kc, bt, cl, block_size=8)
    with pytest.raises(ValueError, match="CUDA"):
        sa.sp2norm_paged_attention(q, kc, kc, bt, cl)


def test_eager_functions_match_oracle_cpu():
    x = torch.randn(2, 3, 33, 33, generator=torch.Generator().manual_seed(1))
    f = sa.FamilyConfig(1.5, 0.25, 3)
    np.testing.assert_allclose(sa.softplus_norm_causal_eager(x, family=f).numpy(),
                               O.softplus_norm_causal(x.numpy(), 1.5, 0.25, 3), rtol=1e-5, atol=1e-7)
    np.testing.assert_allclose(sa.softplus_norm_eager(x, family=f).numpy(),
                               O.softplus_norm(x.numpy(), 1.5, 0.25, 3), rtol=1e-5, atol=1e-7)
    y = sa.softplus_norm_causal(x, family=f, implementation="eager")
    assert y.dtype == x.dtype
    q = torch.randn(1, 4, 20, 32, generator=torch.Generator().manual_seed(2))
    k = torch.randn(1, 2, 20, 32, generator=torch.Generator().manual_seed(3))
    v = torch.randn(1, 2, 20, 32, generator=torch.Generator().manual_seed(4))
    np.testing.assert_allclose(sa.sp2norm_flash_attention_eager(q, k, v, window_size=5).numpy(),
                               O.sp2norm_flash_attention(q.numpy(), k.numpy(), v.numpy(), window_size=5),
                               rtol=1e-5, atol=1e-6)


def test_precompute_rope_cos_sin_cpu():
    cos, sin = sa.precompute_rope_cos_sin(8, 5, device="cpu")
    assert cos.shape == (5, 4) and sin.shape == (5, 4)
    np.testing.assert_allclose(cos[0].numpy(), 1.0)


def _header_symbols():
    text = "".join(p.read_text() for p in (ROOT / "include").glob("*.h"))
    return sorted(set(re.findall(r"^SA_API\s+[\w\s\*]+?\b(sa_\w+)\s*\(", text, flags=re.M)))


def test_c_abi_library_exports_every_header_symbol():
    syms = _header_symbols()
    assert "sa_norm_fwd" in syms and "sa_flash_bwd" in syms
    lib = _lib.load()  # loads without a GPU; no compute call is made here
    for s in syms:
        assert hasattr(lib, s), s
    assert set(syms) == set(_lib.SIGNATURES), "ctypes signatures out of sync with the header"
    assert lib.sa_version() >= 1
    assert lib.sa_status_string(_lib.SA_ERR_ARG) == b"invalid argument"
    assert lib.sa_debug_checks() == 0  # the release library has no device-side index checks


def test_debug_library_exports_every_header_symbol():
    """build.py --debug (run by the driver's build step) gives the same ABI with the checks compiled in."""
    if not _lib.DEBUG_LIB_PATH.exists():
        pytest.skip("debug library not built (python smooth-attn_b200/build.py --debug)")
    dbg = _lib.load(_lib.DEBUG_LIB_PATH)
    for s in _header_symbols():
        assert hasattr(dbg, s), s
    assert dbg.sa_debug_checks() == 1
    assert dbg.sa_status_string(_lib.SA_ERR_BOUNDS) == b"device-side index check failed (debug build)"


def test_c_abi_rejects_bad_arguments_before_launch():
    """Argument validation happens on the host and returns a status; no GPU needed."""
    lib = _lib.load()
    null = None
    # cols out of range / bad power / bad dtype / causal rows not a multiple of cols
    assert lib.sa_norm_fwd(null, null, null, 4, 5000, 5000, 5000, 0, 0, 2.0, 0.5, 2, null) == _lib.SA_ERR_ARG
    assert lib.sa_norm_fwd(null, null, null, 4, 4, 4, 4, 0, 0, 2.0, 0.5, 4, null) == _lib.SA_ERR_ARG
    assert lib.sa_norm_fwd(null, null, null, 4, 4, 4, 4, 7, 0, 2.0, 0.5, 2, null) == _lib.SA_ERR_UNSUPPORTED
    assert lib.sa_norm_fwd(null, null, null, 6, 4, 4, 4, 0, 1, 2.0, 0.5, 2, null) == _lib.SA_ERR_ARG
    assert lib.sa_norm_fwd(null, null, null, 4, 4, 4, 4, 0, 1, 2.0, 0.5, 2, null) == _lib.SA_ERR_ARG  # null ptr
    assert lib.sa_norm_fwd(null, null, null, 0, 4, 4, 4, 0, 1, 2.0, 0.5, 2, null) == _lib.SA_OK  # empty
    assert lib.sa_norm_bwd(null, null, null, null, 4, 4, 4, 4, 4, 0, 9, 1, 2.0, 0.5, 2, null) == _lib.SA_ERR_UNSUPPORTED
    with pytest.raises(ValueError):
        _lib.check(_lib.SA_ERR_ARG, "sa_norm_fwd")


def test_band_copy_rejects_bad_arguments_before_any_copy():
    lib = _lib.load()
    n = ctypes.c_int64(-1)
    assert lib.sa_copy_causal_bands(None, None, 2, 64, 2, 12, 1, ctypes.byref(n), None) == _lib.SA_ERR_ARG  # band % 8
    assert lib.sa_copy_causal_bands(None, None, 2, 64, 3, 128, 1, None, None) == _lib.SA_ERR_ARG  # element size
    assert lib.sa_copy_causal_bands(None, None, 2, 64, 2, 128, 1, None, None) == _lib.SA_ERR_ARG  # null pointers
    assert lib.sa_copy_causal_bands(None, None, 0, 64, 2, 128, 1, ctypes.byref(n), None) == _lib.SA_OK
    assert n.value == 0


def test_host_path_needs_pinned_cpu_tensors():
    from smooth_attn import host

    x = torch.randn(1, 16, 16)
    with pytest.raises(ValueError):
        sa.softplus_norm_causal_host_out(torch.empty_like(x), x)  # not pinned
    with pytest.raises(TypeError):
        sa.softplus_norm_causal_host_out(None, x)
    assert host.causal_band_bytes((8, 16, 2048, 2048), torch.bfloat16) == 570425344


@pytest.mark.parametrize(("L", "elem"), [(300, 2), (2048, 2), (129, 4), (7, 2)])
def test_host_zero_causal_tail_writes_exactly_the_tail(L, elem):
    """Host-only: zeros the columns past each 128-row band's copied width, nothing else."""
    from smooth_attn import host

    dt = np.uint16 if elem == 2 else np.uint32
    a = np.full((3, L, L), 0xABCD, dtype=dt)
    st = _lib.load().sa_host_zero_causal_tail(ctypes.c_void_p(a.ctypes.data), 3, L, elem, host.BAND, 3)
    assert st == _lib.SA_OK
    want = np.full((3, L, L), 0xABCD, dtype=dt)
    for r0, r1, w in host._bands(L, elem):
        want[:, r0:r1, w:] = 0
    assert np.array_equal(a, want)

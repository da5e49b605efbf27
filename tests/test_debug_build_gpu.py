"""The debug library (``build.py --debug``: device-side index checks that
count failures instead of trapping) on the GPU.

A child process with ``SA_DEBUG_LIB=1`` runs every kernel family on small,
ragged shapes: causal norm forward / backward (bulk and unaligned rows),
flash forward and both backwards (GQA, window, D = 64 / 128), paged decode
(tensor-core and CUDA-core kernels), RoPE attention with the output
projection, and the FP8 forward.  It checks that the debug library is the one
loaded, that no index check failed (``sa_device_status`` is SA_OK), and saves
the outputs; this process computes the same with the release library.  The
checks do not change the arithmetic, so the outputs must be bitwise equal
(dQ of the default backward, summed with fp32 atomics, up to the order of the
adds).
"""

import os
import subprocess
import sys
from pathlib import Path

import numpy as np
import pytest
import torch

from smooth_attn import _lib

pytestmark = pytest.mark.gpu
ROOT = Path(__file__).resolve().parents[1]


def run_all(out_path):
    import smooth_attn as sa

    dev = "cuda"
    res = {}

    def rnd(shape, seed, dtype=torch.bfloat16):
        g = torch.Generator().manual_seed(seed)
        return torch.randn(*shape, generator=g).to(dtype).to(dev)

    for L in (129, 256):
        x = rnd((2, 3, L, L), L).requires_grad_(True)
        y = sa.softplus_norm_causal(x)
        y.backward(rnd((2, 3, L, L), L + 1))
        res[f"norm_y_{L}"], res[f"norm_dx_{L}"] = y.detach(), x.grad
    for (Hq, Hkv, T, D, W) in ((4, 2, 300, 64, 0), (4, 4, 257, 128, 100), (4, 2, 384, 128, 0)):
        q, k, v = (rnd((1, h, T, D), T + h + D + i).requires_grad_(True) for i, h in enumerate((Hq, Hkv, Hkv)))
        do = rnd((1, Hq, T, D), T + 7)
        for det in (False, True):
            o = sa.sp2norm_flash_attention(q, k, v, window_size=W, deterministic=det)
            dq, dk, dv = torch.autograd.grad(o, (q, k, v), do)
            tag = f"{Hq}_{Hkv}_{T}_{D}_{W}_{int(det)}"
            res["o_" + tag], res["dq_" + tag], res["dk_" + tag], res["dv_" + tag] = o.detach(), dq, dk, dv
    B, Hq, Hkv, T, D, BS = 2, 8, 2, 200, 128, 16
    nb = B * ((T + BS - 1) // BS)
    qd = rnd((B, Hq, 1, D), 1)
    kc, vc = rnd((nb, Hkv, BS, D), 2), rnd((nb, Hkv, BS, D), 3)
    bt = torch.randperm(nb, generator=torch.Generator().manual_seed(4)).to(torch.int32).view(B, -1).to(dev)
    cl = torch.tensor([T, T - 37], dtype=torch.int32, device=dev)
    for kern in ("tc", "simt"):
        os.environ["SA_PAGED_DECODE_KERNEL"] = kern
        res["decode_" + kern] = sa.sp2norm_paged_attention(qd, kc, vc, bt, cl, block_size=BS)
    os.environ.pop("SA_PAGED_DECODE_KERNEL")
    T, D = 192, 64
    q, k, v = rnd((1, 4, T, D), 5), rnd((1, 4, T, D), 6), rnd((1, 4, T, D), 7)
    cos, sin = sa.precompute_rope_cos_sin(D, T, device=dev)
    w = rnd((4, D, 96), 8)
    res["rope_proj"] = sa.sp2norm_rope_flash_attention_proj(q, k, v, w, cos, sin)
    res["fp8"] = sa.sp2norm_fp8_flash_attention(q, k, v)
    torch.cuda.synchronize()
    lib = _lib.load()
    status = lib.sa_device_status(1)
    np.savez(out_path, debug=np.int32(lib.sa_debug_checks()), status=np.int32(status),
             **{kk: vv.float().cpu().numpy() for kk, vv in res.items()})


@pytest.fixture(autouse=True)
def _need_cuda():
    if not torch.cuda.is_available():
        pytest.skip("CUDA required")


def test_debug_library_runs_clean_and_matches_release(tmp_path):
    if not _lib.DEBUG_LIB_PATH.exists():
        pytest.fail("debug library missing: run python smooth-attn_b200/build.py --debug")
    out = tmp_path / "debug.npz"
    env = dict(os.environ, SA_DEBUG_LIB="1")
    code = (f"import sys; sys.path[:0] = [{str(ROOT / 'smooth-attn_b200')!r}, {str(ROOT)!r}]; "
            f"from tests.test_debug_build_gpu import run_all; run_all({str(out)!r})")
    r = subprocess.run([sys.executable, "-c", code], env=env, capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stderr[-3000:]
    dbg = np.load(out)
    assert int(dbg["debug"]) == 1, "the child did not load the debug library"
    assert int(dbg["status"]) == _lib.SA_OK, f"device status {int(dbg['status'])}: an index check failed"
    ref = tmp_path / "release.npz"
    run_all(ref)
    rel = np.load(ref)
    assert int(rel["debug"]) == 0
    for key in dbg.files:
        if key in ("debug", "status"):
            continue
        if key.startswith("dq_") and key.endswith("_0"):  # fp32 atomics: order of the adds
            np.testing.assert_allclose(dbg[key], rel[key], rtol=1e-2, atol=1e-2, err_msg=key)
        else:
            np.testing.assert_array_equal(dbg[key], rel[key], err_msg=key)

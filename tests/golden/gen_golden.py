"""Generate golden vectors from the reference's OWN eager implementation.

Run in a container that has the reference checkout (read-only) at
``$SMOOTH_ATTN_REF`` (default ``/root/reference``):

    python tests/golden/gen_golden.py

It imports ``smooth_attn`` from ``$SMOOTH_ATTN_REF/src`` and evaluates, on CPU
in float32 with seeded ``torch.Generator`` inputs:
  * ``softplus_norm_eager``               (kernels.py:1332-1346)
  * ``softplus_norm_causal_eager``        (kernels.py:1349-1365) + torch autograd
  * ``sp2norm_flash_attention_eager``     (kernels.py:2053-2084) + torch autograd
  * ``reference_decode_attention`` of the reference's paged tests
    (tests/test_paged_attention.py:78-109) on shuffled paged caches built by
    its ``_build_paged_kv_cache_shuffled`` (:43-75)
  * ``precompute_rope_cos_sin`` (kernels.py:2093-2101) with the RoPE tests'
    ``apply_rope_eager`` (tests/test_rope_proj.py:15-30) followed by
    ``sp2norm_flash_attention_eager``, and the per-head projection sum of
    tests/test_rope_proj.py:134-138
  * ``_quantize_to_fp8`` (kernels.py:2592-2601): E4M3 values and scales

and writes ``golden.npz`` next to this script.  The GPU box never runs this
script (the reference is not present there); the tests only read the
committed ``golden.npz``.  Inputs of bf16 cases are stored after rounding to
bf16 (as float32), so a consumer can rebuild the exact bf16 tensors.
"""

from __future__ import annotations

import os
import sys
from pathlib import Path

import numpy as np
import torch

REF = Path(os.environ.get("SMOOTH_ATTN_REF", "/root/reference"))
sys.path.insert(0, str(REF / "src"))

import smooth_attn as ref  # noqa: E402  (the reference package)

OUT = Path(__file__).with_name("golden.npz")


def randn(shape, seed, dtype=torch.float32):
    g = torch.Generator().manual_seed(seed)
    t = torch.randn(*shape, generator=g, dtype=torch.float32)
    return t.to(dtype).float()


def main():
    data = {}

    # --- causal norm, forward + autograd backward --------------------------
    causal_cases = [
        # name, shape, (alpha, theta, power), input dtype
        ("c_cfg1", (1, 2, 128, 128), (2.0, 0.5, 2), torch.float32),
        ("c_p3", (1, 2, 64, 64), (1.5, 0.25, 3), torch.float32),
        ("c_p1", (1, 1, 48, 48), (1.0, 0.0, 1), torch.float32),
        ("c_l1", (1, 1, 1, 1), (2.0, 0.5, 2), torch.float32),
        ("c_l7", (2, 1, 7, 7), (2.0, 0.5, 2), torch.float32),
        ("c_l17", (1, 3, 17, 17), (2.0, 0.5, 2), torch.float32),
        ("c_l129", (1, 1, 129, 129), (2.0, 0.5, 2), torch.float32),
        ("c_bf16", (1, 2, 64, 64), (2.0, 0.5, 2), torch.bfloat16),
        ("c_3d", (3, 40, 40), (2.0, 0.5, 2), torch.float32),
    ]
    for i, (name, shape, (a, t, p), dt) in enumerate(causal_cases):
        fam = ref.FamilyConfig(alpha=a, theta=t, power=p)
        x = randn(shape, 1000 + i, dt).requires_grad_(True)
        g = randn(shape, 2000 + i)
        y = ref.softplus_norm_causal_eager(x, family=fam)
        (y * g).sum().backward()
        data[f"{name}/x"] = x.detach().numpy()
        data[f"{name}/g"] = g.numpy()
        data[f"{name}/out"] = y.detach().numpy()
        data[f"{name}/dx"] = x.grad.numpy()
        data[f"{name}/family"] = np.array([a, t, p], dtype=np.float64)

    # --- row-wise norm forward ---------------------------------------------
    row_cases = [
        ("r_64x96", (64, 96), (2.0, 0.5, 2)),
        ("r_p3", (16, 250), (1.5, 0.25, 3)),
        ("r_odd", (5, 33), (0.7, -0.3, 1)),
    ]
    for i, (name, shape, (a, t, p)) in enumerate(row_cases):
        x = randn(shape, 3000 + i)
        y = ref.softplus_norm_eager(x, alpha=a, theta=t, power=p)
        data[f"{name}/x"] = x.numpy()
        data[f"{name}/out"] = y.numpy()
        data[f"{name}/family"] = np.array([a, t, p], dtype=np.float64)

    # --- flash attention, forward + autograd backward ----------------------
    flash_cases = [
        # name, B, Hq, Hkv, T, D, window
        ("f_mha", 1, 2, 2, 64, 32, 0),
        ("f_gqa_win", 1, 4, 2, 48, 32, 16),
        ("f_d64", 1, 1, 1, 80, 64, 0),
        ("f_d128", 1, 1, 1, 40, 128, 0),
    ]
    for i, (name, B, Hq, Hkv, T, D, W) in enumerate(flash_cases):
        q = randn((B, Hq, T, D), 4000 + i, torch.bfloat16).requires_grad_(True)
        k = randn((B, Hkv, T, D), 5000 + i, torch.bfloat16).requires_grad_(True)
        v = randn((B, Hkv, T, D), 6000 + i, torch.bfloat16).requires_grad_(True)
        do = randn((B, Hq, T, D), 7000 + i)
        o = ref.sp2norm_flash_attention_eager(q, k, v, window_size=W)
        (o * do).sum().backward()
        data[f"{name}/q"] = q.detach().numpy()
        data[f"{name}/k"] = k.detach().numpy()
        data[f"{name}/v"] = v.detach().numpy()
        data[f"{name}/do"] = do.numpy()
        data[f"{name}/o"] = o.detach().numpy()
        data[f"{name}/dq"] = q.grad.numpy()
        data[f"{name}/dk"] = k.grad.numpy()
        data[f"{name}/dv"] = v.grad.numpy()
        data[f"{name}/window"] = np.array(W)

    # --- paged-KV decode (reference decode reference of the paged tests) ---
    sys.path.insert(0, str(REF / "tests"))
    import test_paged_attention as tpa  # noqa: E402  (the reference's own test helpers)

    paged_cases = [
        # name, B, Hq, Hkv, T (per sequence), D, block_size
        ("p_basic", 2, 4, 4, 48, 32, 16),
        ("p_gqa", 2, 8, 2, 100, 64, 16),
        ("p_bs8", 1, 4, 4, 37, 128, 8),
    ]
    for i, (name, B, Hq, Hkv, T, D, BS) in enumerate(paged_cases):
        q = randn((B, Hq, 1, D), 8000 + i, torch.bfloat16).to(torch.bfloat16)
        k = randn((B, Hkv, T, D), 8100 + i, torch.bfloat16).to(torch.bfloat16)
        v = randn((B, Hkv, T, D), 8200 + i, torch.bfloat16).to(torch.bfloat16)
        torch.manual_seed(8300 + i)  # the shuffled builder draws a permutation
        kc, vc, bt, cl = tpa._build_paged_kv_cache_shuffled(k, v, block_size=BS)
        out = tpa.reference_decode_attention(q, k, v)
        data[f"{name}/q"] = q.float().numpy()
        data[f"{name}/k_cache"] = kc.float().numpy()
        data[f"{name}/v_cache"] = vc.float().numpy()
        data[f"{name}/block_table"] = bt.numpy()
        data[f"{name}/context_lens"] = cl.numpy()
        data[f"{name}/out"] = out.float().numpy()

    # --- RoPE attention and RoPE attention + output projection -------------
    import test_rope_proj as trp  # noqa: E402  (the reference's own test helpers)

    rope_cases = [
        # name, B, Hq, Hkv, T, D, window, D_model (0 = no projection)
        ("rope_mha", 1, 2, 2, 64, 32, 0, 0),
        ("rope_gqa_win", 2, 4, 2, 48, 64, 16, 0),
        ("rope_proj", 2, 4, 4, 40, 32, 0, 96),
    ]
    for i, (name, B, Hq, Hkv, T, D, W, DM) in enumerate(rope_cases):
        q = randn((B, Hq, T, D), 9000 + i, torch.bfloat16).to(torch.bfloat16)
        k = randn((B, Hkv, T, D), 9100 + i, torch.bfloat16).to(torch.bfloat16)
        v = randn((B, Hkv, T, D), 9200 + i, torch.bfloat16).to(torch.bfloat16)
        cos, sin = ref.precompute_rope_cos_sin(D, T, device="cpu", dtype=torch.float32)
        q_rot = trp.apply_rope_eager(q.float(), cos, sin).to(torch.bfloat16)
        k_rot = trp.apply_rope_eager(k.float(), cos, sin).to(torch.bfloat16)
        # fp32 eager attention on the (bf16-valued) rotated tensors pins the
        # oracle; the projection below follows the test, which projects the
        # bf16 eager output.
        o = ref.sp2norm_flash_attention_eager(q_rot.float(), k_rot.float(), v.float(), window_size=W)
        o_bf16 = ref.sp2norm_flash_attention_eager(q_rot, k_rot, v, window_size=W)
        data[f"{name}/q"] = q.float().numpy()
        data[f"{name}/k"] = k.float().numpy()
        data[f"{name}/v"] = v.float().numpy()
        data[f"{name}/cos"] = cos.numpy()
        data[f"{name}/sin"] = sin.numpy()
        data[f"{name}/q_rot"] = q_rot.float().numpy()
        data[f"{name}/k_rot"] = k_rot.float().numpy()
        data[f"{name}/o"] = o.float().numpy()
        data[f"{name}/window"] = np.array(W)
        if DM:
            w_o = randn((Hq, D, DM), 9300 + i, torch.bfloat16).to(torch.bfloat16) * 0.02
            proj = torch.zeros(B, T, DM, dtype=torch.float32)
            for h in range(Hq):  # tests/test_rope_proj.py:134-138
                proj += torch.matmul(o_bf16[:, h].float(), w_o[h].float())
            data[f"{name}/w_o"] = w_o.float().numpy()
            data[f"{name}/proj"] = proj.numpy()

    # --- FP8 per-tensor quantization (kernels.py:2592-2601) -----------------
    from smooth_attn.kernels import _quantize_to_fp8  # noqa: E402

    fp8_cases = [("fp8_bf16", (2, 4, 64, 32), torch.bfloat16, 1.0), ("fp8_f32", (1, 2, 48, 64), torch.float32, 7.5),
                 ("fp8_tiny", (1, 1, 16, 32), torch.float32, 1e-3)]
    for i, (name, shape, dt, mag) in enumerate(fp8_cases):
        x = (randn(shape, 9500 + i) * mag).to(dt)
        x8, sc = _quantize_to_fp8(x)
        data[f"{name}/x"] = x.float().numpy()
        data[f"{name}/x8"] = x8.float().numpy()
        data[f"{name}/scale"] = np.array(sc, dtype=np.float64)

    np.savez_compressed(OUT, **data)
    print(f"wrote {OUT} ({OUT.stat().st_size} bytes, {len(data)} arrays)")


if __name__ == "__main__":
    main()

"""Measured parity of the flash attention kernels against the fp64 oracle.

Not a test (pytest does not collect it): prints, per case, the largest
absolute error, the largest error relative to the tolerance
(|got - ref| / (atol + rtol |ref|), 2e-2 / 1e-2) and how many elements exceed
the plain tolerance (each of those must be explained by the reference's bf16
rounding of P / dS, which ``tests/_util.check_bf16_grads`` asserts).  Run on a
GPU box:

    python tests/parity_report.py
"""

import sys
from pathlib import Path

import numpy as np
import torch

ROOT = Path(__file__).resolve().parents[1]
for p in (str(ROOT / "smooth-attn_b200"), str(ROOT)):
    if p not in sys.path:
        sys.path.insert(0, p)

import smooth_attn as sa  # noqa: E402
from oracle import sa_oracle as O  # noqa: E402
from tests._util import np32, randn  # noqa: E402

RTOL, ATOL = 2e-2, 1e-2
CASES = [  # B, Hq, Hkv, T, D, window
    (2, 3, 3, 129, 32, 0), (2, 3, 3, 300, 64, 0), (2, 4, 2, 512, 128, 0), (1, 8, 2, 1024, 128, 0),
    (1, 4, 4, 777, 128, 100), (1, 2, 2, 2048, 128, 0),
]


def stats(got, ref):
    g, r = np.asarray(got, np.float64), np.asarray(ref, np.float64)
    err = np.abs(g - r)
    tol = ATOL + RTOL * np.abs(r)
    return err.max(), (err / tol).max(), int((err > tol).sum()), g.size


def main():
    print("| case B,Hq,Hkv,T,D,W | tensor | max abs err | max err / tol | elements over tol |")
    print("|---|---|---|---|---|")
    for i, (B, Hq, Hkv, T, D, W) in enumerate(CASES):
        q = randn((B, Hq, T, D), 100 + i, torch.bfloat16, "cuda").requires_grad_(True)
        k = randn((B, Hkv, T, D), 200 + i, torch.bfloat16, "cuda").requires_grad_(True)
        v = randn((B, Hkv, T, D), 300 + i, torch.bfloat16, "cuda").requires_grad_(True)
        do = randn((B, Hq, T, D), 400 + i, torch.bfloat16, "cuda")
        args = (np32(q), np32(k), np32(v))
        ref_o = O.sp2norm_flash_attention(*args, window_size=W, acc=np.float64)
        ref_g = O.sp2norm_flash_attention_bwd(*args, np32(do), window_size=W, acc=np.float64)
        name = f"{B},{Hq},{Hkv},{T},{D},{W}"
        for det in (False, True):
            q.grad = k.grad = v.grad = None
            o = sa.sp2norm_flash_attention(q, k, v, window_size=W, deterministic=det)
            o.backward(do)
            torch.cuda.synchronize()
            rows = [("o", o)] if not det else []
            rows += [(f"d{n}" + (" (det)" if det else ""), t.grad) for n, t in zip("qkv", (q, k, v))]
            for nm, t in rows:
                r = ref_o if nm == "o" else ref_g["qkv".index(nm[1])]
                a, rt, over, n = stats(np32(t), r)
                print(f"| {name} | {nm} | {a:.2e} | {rt:.3f} | {over} / {n} |")


if __name__ == "__main__":
    main()

"""Helpers shared by the test modules (seeded inputs, tolerances)."""

import numpy as np
import torch

# Tolerances against the fp32 oracle:
#   fp32 outputs: 1e-5 relative; bf16/fp16 outputs: 2e-2 relative / 1e-2 absolute.
TOL = {
    torch.float32: dict(rtol=1e-5, atol=1e-7),
    torch.float16: dict(rtol=2e-2, atol=1e-2),
    torch.bfloat16: dict(rtol=2e-2, atol=1e-2),
}


def randn(shape, seed, dtype=torch.float32, device="cpu", scale=1.0):
    g = torch.Generator().manual_seed(seed)
    t = torch.randn(*shape, generator=g, dtype=torch.float32) * scale
    return t.to(dtype).to(device)


def np32(t):
    return t.detach().float().cpu().numpy()


def assert_close(actual, expected, rtol, atol):
    a = np.asarray(actual, dtype=np.float64)
    e = np.asarray(expected, dtype=np.float64)
    np.testing.assert_allclose(a, e, rtol=rtol, atol=atol)

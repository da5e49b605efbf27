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


def check_bf16_grads(got, ref, emu, rtol=2e-2, atol=1e-2, max_frac=1e-3):
    """Element-wise criterion for 16-bit flash gradients against the fp32 oracle.

    Every element must be within ``atol + rtol * |ref|`` of the oracle, except
    where the kernel's own arithmetic, emulated on the CPU with the same bf16
    rounding points the reference prescribes (bf16 dS before dQ / dK, bf16 P
    before dV, bf16 y in P.V: ``emulate=True`` in the oracle), is itself more
    than half that tolerance away from the oracle; there the kernel must be
    within the tolerance of the emulation.  Such elements must also be rare
    (at most ``max_frac`` of the tensor).  Returns (worst ratio to the plain
    tolerance, number of elements outside it) for the record.
    """
    g = np.asarray(got, dtype=np.float64)
    r = np.asarray(ref, dtype=np.float64)
    m = np.asarray(emu, dtype=np.float64)
    tol = atol + rtol * np.abs(r)
    bad = np.abs(g - r) > tol
    explained = (np.abs(m - r) > 0.5 * tol) & (np.abs(g - m) <= atol + rtol * np.abs(m))
    unexplained = bad & ~explained
    ratio = float((np.abs(g - r) / tol).max()) if g.size else 0.0
    assert not unexplained.any(), (
        f"{int(unexplained.sum())} elements outside rtol={rtol} atol={atol} not explained by bf16 operand "
        f"rounding; worst ratio {ratio:.3f}")
    assert bad.sum() <= max(1, max_frac * g.size), f"{int(bad.sum())} of {g.size} elements outside the tolerance"
    return ratio, int(bad.sum())

"""Benchmark harness and CLI (``python -m smooth_attn``), mirroring the
reference's ``benchmark_rowwise_suite`` / ``benchmark_causal_suite`` /
``main`` (src/smooth_attn/kernels.py:2841-2925, 3052-3128).  Not on the hot
path; it times the CUDA kernels against torch softmax baselines.
"""

from __future__ import annotations

import argparse

import torch
import torch.nn.functional as F

from .kernels import (
    DEFAULT_FAMILY,
    SUPPORTED_DTYPES,
    CausalBenchmarkResult,
    FamilyConfig,
    RowwiseBenchmarkResult,
    bench,
    bench_out,
    softmax_causal_eager,
    softmax_causal_triton_out,
    softmax_triton_out,
    softplus_norm_causal,
    softplus_norm_causal_eager,
    softplus_norm_causal_triton_out,
    softplus_norm_triton_out,
)

DEFAULT_ROWWISE_SHAPES = ((256, 256), (1024, 1024), (4096, 512), (16384, 256), (128, 2048), (32768, 512))


def benchmark_rowwise_suite(family, shapes=None, warmup=50, iters=200):
    results = []
    for rows, cols in tuple(shapes or DEFAULT_ROWWISE_SHAPES):
        x = torch.randn(rows, cols, device="cuda")
        out_sm = torch.empty_like(x)
        out_fam = torch.empty_like(x)
        results.append(RowwiseBenchmarkResult(
            shape=(rows, cols),
            torch_softmax_us=bench(lambda z: F.softmax(z, dim=-1), x, warmup=warmup, iters=iters),
            triton_softmax_us=bench_out(softmax_triton_out, out_sm, x, warmup=warmup, iters=iters),
            family_us=bench_out(lambda o, z: softplus_norm_triton_out(o, z, family=family), out_fam, x,
                                warmup=warmup, iters=iters),
        ))
    return results


def benchmark_causal_suite(family, dtypes, lengths, batch=2, heads=8, warmup=50, iters=200):
    results = []
    for dtype in dtypes:
        for L in lengths:
            x = torch.randn(batch, heads, L, L, device="cuda", dtype=dtype)
            ref_sm = softmax_causal_eager(x.float())
            ref_fam = softplus_norm_causal_eager(x.float(), family=family)
            out_sm = torch.empty_like(x)
            out_fam = torch.empty_like(x)
            our_sm, sm_meta = softmax_causal_triton_out(out_sm, x, return_meta=True)
            our_fam, fam_meta = softplus_norm_causal_triton_out(out_fam, x, family=family, return_meta=True)
            atol = 1e-4 if dtype == torch.float32 else 5e-3
            results.append(CausalBenchmarkResult(
                dtype=dtype, batch=batch, heads=heads, seq_len=L,
                torch_softmax_us=bench(softmax_causal_eager, x, warmup=warmup, iters=iters),
                triton_softmax_us=bench_out(softmax_causal_triton_out, out_sm, x, warmup=warmup, iters=iters),
                family_us=bench_out(lambda o, z: softplus_norm_causal_triton_out(o, z, family=family), out_fam, x,
                                    warmup=warmup, iters=iters),
                softmax_err=(ref_sm - our_sm.float()).abs().max().item(),
                family_err=(ref_fam - our_fam.float()).abs().max().item(),
                softmax_sums_ok=torch.allclose(our_sm.float().sum(-1), torch.ones_like(ref_sm.sum(-1)), atol=atol),
                family_sums_ok=torch.allclose(our_fam.float().sum(-1), torch.ones_like(ref_fam.sum(-1)), atol=atol),
                softmax_meta=sm_meta, family_meta=fam_meta,
            ))
    return results


def validate_causal_backward(family, dtypes, seq_len=128, batch=2, heads=4):
    results = []
    for dtype in dtypes:
        x = torch.randn(batch, heads, seq_len, seq_len, device="cuda", dtype=dtype, requires_grad=True)
        upstream = torch.randn(batch, heads, seq_len, seq_len, device="cuda", dtype=torch.float32)
        (softplus_norm_causal(x, family=family).float() * upstream).sum().backward()
        g = x.grad.detach().clone()
        xr = x.detach().clone().requires_grad_(True)
        (softplus_norm_causal_eager(xr.float(), family=family) * upstream).sum().backward()
        results.append({
            "dtype": dtype,
            "max_abs_grad_err": (g.float() - xr.grad.float()).abs().max().item(),
            "grad_close": torch.allclose(g.float(), xr.grad.float(),
                                         atol=1e-4 if dtype == torch.float32 else 5e-3,
                                         rtol=1e-3 if dtype == torch.float32 else 5e-2),
        })
    return results


def parse_args(argv=None):
    p = argparse.ArgumentParser(description="smooth-attn B200 benchmark harness")
    p.add_argument("--mode", choices=("causal", "rowwise", "all"), default="causal")
    p.add_argument("--dtypes", default="bf16", help="comma-separated: fp32,fp16,bf16")
    p.add_argument("--lengths", default="128,256,512,1024")
    p.add_argument("--batch", type=int, default=2)
    p.add_argument("--heads", type=int, default=8)
    p.add_argument("--warmup", type=int, default=50)
    p.add_argument("--iters", type=int, default=200)
    p.add_argument("--alpha", type=float, default=DEFAULT_FAMILY.alpha)
    p.add_argument("--theta", type=float, default=DEFAULT_FAMILY.theta)
    p.add_argument("--power", type=int, default=DEFAULT_FAMILY.power)
    p.add_argument("--quick", action="store_true")
    p.add_argument("--check-backward", action="store_true")
    return p.parse_args(argv)


def main(argv=None):
    args = parse_args(argv)
    family = FamilyConfig(alpha=args.alpha, theta=args.theta, power=args.power)
    dtypes = [SUPPORTED_DTYPES[t.strip().lower()] for t in args.dtypes.split(",") if t.strip()]
    lengths = [int(t) for t in args.lengths.split(",") if t.strip()]
    if args.quick:
        lengths = lengths[:2]
        args.warmup, args.iters = min(args.warmup, 20), min(args.iters, 100)
    print(f"GPU: {torch.cuda.get_device_name()}  family: {family.label}")
    if args.mode in ("rowwise", "all"):
        for r in benchmark_rowwise_suite(family, warmup=args.warmup, iters=args.iters):
            print(f"rowwise {r.shape}: torch softmax {r.torch_softmax_us:8.1f} us  family {r.family_us:8.1f} us")
    if args.mode in ("causal", "all"):
        for r in benchmark_causal_suite(family, dtypes, lengths, args.batch, args.heads, args.warmup, args.iters):
            print(f"causal {str(r.dtype):15s} L={r.seq_len:5d}: softmax(eager) {r.torch_softmax_us:8.1f} us  "
                  f"family {r.family_us:8.1f} us  err {r.family_err:.2e}  sums_ok {r.family_sums_ok}")
    if args.check_backward:
        for row in validate_causal_backward(family, dtypes, seq_len=lengths[0], batch=min(args.batch, 2),
                                            heads=min(args.heads, 4)):
            print(f"backward {row['dtype']}: grad_close={row['grad_close']} max_abs_err={row['max_abs_grad_err']:.2e}")

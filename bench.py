"""Benchmark of the smooth-attn B200 hot path (one JSON line on rank 0).

Headline: causal squareplus normalization forward through
the out-buffer path, x bf16 [8,16,2048,2048] N(0,1), alpha=2, theta=0.5,
power=2 -> "causal-norm HBM GB/s" (algorithmic bytes: the visible triangle
read + the full output written).  A second workload object reports the fused
squareplus attention fwd+bwd TFLOP/s ([4,32,4096,128]).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

N > 1 runs under torchrun (one process per GPU, NCCL).  The work shards over
independent (batch, head) matrices with no collective on the data path: each
rank owns one full BASELINE-sized block of a global batch N times as large
("weak" scaling), and value = bytes (or FLOPs) of all ranks / max-over-ranks time.
Timing: CUDA events on the launching stream, W warm-up steps, barrier +
synchronize around the K timed steps, max over ranks.  Inputs are larger
than L2 (126 MB), so no flush is needed between steps.

The line's ``e2e`` runs the same workload from pinned host buffers through
``softplus_norm_causal_host_out`` (both PCIe transfers inside the timed
region), and ``flash_fwd_bwd`` (last in the line) also reports the
deterministic backward.

``--impl reference`` times the reference algorithm's CPU implementation (the
numpy oracle port, multi-threaded over matrices) on the host cores on a
bounded sample of the same workload.
"""

from __future__ import annotations

import argparse
import gc
import json
import os
import statistics
import subprocess
import sys
import threading
import time
from concurrent.futures import ThreadPoolExecutor
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT / "smooth-attn_b200"))
sys.path.insert(0, str(ROOT))

import numpy as np  # noqa: E402
import torch  # noqa: E402

NORM_CFG = dict(B=8, H=16, L=2048)  # BASELINE configs[1], largest L
FLASH_CFG = dict(B=4, H=32, T=4096, D=128)
METRIC = "causal-norm HBM GB/s"
# DRAM bytes (read + write) of one norm_fwd_bulk launch at [8,16,2048,2048]: ncu
# capture of the [2,16,2048,2048] case scaled by 4 (see profiles/).
NORM_TRAFFIC_BYTES = 4 * (138.446336e6 + 208.5952e6)


def norm_bytes(M, L, e=2, rowsum=False):
    """Algorithmic bytes of one causal-norm forward: the visible triangle read
    (L(L+1)/2 elements per matrix) + the full L*L output written."""
    return M * (e * L * (L + 1) // 2 + e * L * L) + (4 * M * L if rowsum else 0)


def peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return float(d["hbm_gbs"]), float(d["bf16_tflops"]), float(d.get("bf16_tflops_sustained", d["bf16_tflops"])), "measured"
    return 6650.0, 1590.0, 1400.0, "fallback"


class ClockSampler:
    """nvidia-smi clock / throttle sampling during the timed region."""

    def __init__(self, index):
        self.index = index
        self.proc = None
        self.lines = []

    def __enter__(self):
        q = ("timestamp,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.hw_slowdown,"
             "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
             "clocks_event_reasons.sw_power_cap")
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.index), f"--query-gpu={q}", "--format=csv,noheader,nounits",
                 "-lms", "50"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
            time.sleep(0.5)  # let nvidia-smi start before the timed region
        except (FileNotFoundError, OSError):
            self.proc = None
        self.t_start = time.time()
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append((time.time(), line.strip()))

    def __exit__(self, *exc):
        self.t_end = time.time()
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self):
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for t, ln in self.lines:
            parts = [p.strip() for p in ln.split(",")][1:]  # drop nvidia-smi's timestamp
            if len(parts) < 7 or not (self.t_start <= t <= self.t_end + 0.06):
                continue
            try:
                sm.append(float(parts[0]))
                mx = float(parts[1])
            except ValueError:
                continue
            for n, v in zip(names, parts[3:7]):
                if v.lower().startswith("active"):
                    reasons.add(n)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(sm)}


def dist_setup(n_gpus):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import torch.distributed as dist

        torch.cuda.set_device(local)
        dist.init_process_group("nccl", device_id=torch.device("cuda", local))
    else:
        torch.cuda.set_device(0)
    return world, rank, local


def barrier(world):
    if world > 1:
        import torch.distributed as dist

        dist.barrier()


def max_over_ranks(v, world):
    if world == 1:
        return v
    import torch.distributed as dist

    t = torch.tensor([v], device="cuda", dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def time_steps(fn, steps, world):
    """Time `steps` calls of fn with CUDA events on the current stream; max over ranks (ms)."""
    barrier(world)
    torch.cuda.synchronize()
    s = torch.cuda.current_stream()
    a = torch.cuda.Event(enable_timing=True)
    b = torch.cuda.Event(enable_timing=True)
    a.record(s)
    for _ in range(steps):
        fn()
    b.record(s)
    torch.cuda.synchronize()
    barrier(world)
    return max_over_ranks(a.elapsed_time(b), world)


def run_ours(args):
    import smooth_attn as sa
    from oracle import sa_oracle as O

    world, rank, local = dist_setup(args.gpus)
    hbm, tf_burst, tf_sus, peak_kind = peaks()
    if args.only == "flash":
        flash = run_flash(args, world, rank, tf_burst, tf_sus, peak_kind)
        if rank == 0:
            print(json.dumps({"metric": "fused squareplus-attn fwd+bwd TFLOP/s", "n_gpus": world, **flash}), flush=True)
        return
    if args.only == "cp":
        g = torch.Generator(device="cuda").manual_seed(99 + rank)
        shape = tuple(int(v) for v in args.shape.split(",")) if args.shape else CP_SHAPE
        res = extra_cp(shape, args.steps, world, rank, g, tf_sus)
        if rank == 0:
            print(json.dumps({"workload": "cp", "n_gpus": world, "steps": args.steps, **res}), flush=True)
        return
    if args.only in ("decode", "rope", "fp8"):  # one extension workload (profiling entry point)
        g = torch.Generator(device="cuda").manual_seed(777 + rank)
        shape = tuple(int(v) for v in args.shape.split(",")) if args.shape else None
        if args.only == "decode":
            res = extra_decode((shape,) if shape else DECODE_SHAPES, args.steps, world, g, hbm, O)
        elif args.only == "rope":
            res = extra_rope((shape,) if shape else ROPE_SHAPES, args.steps, world, g)
        else:
            res = extra_fp8((shape,) if shape else FP8_SHAPES, args.steps, world, g)
        if rank == 0:
            print(json.dumps({"workload": args.only, "n_gpus": world, "steps": args.steps, **res}), flush=True)
        return
    B, H, L = args.norm_batch, NORM_CFG["H"], NORM_CFG["L"]
    m_loc = B * H  # this rank's block of the global [N*B, H, L, L] batch
    M = m_loc * world
    gen = torch.Generator().manual_seed(1234 + rank)
    x = torch.randn(m_loc, L, L, generator=gen, dtype=torch.float32).to(torch.bfloat16).cuda()
    out = torch.empty_like(x)
    step = lambda: sa.softplus_norm_causal_triton_out(out, x)  # noqa: E731

    for _ in range(max(args.warmup, 3)):
        step()
    with ClockSampler(local) as clk:
        ms = time_steps(step, args.steps, world)
    ms_step = ms / args.steps
    bytes_all = norm_bytes(M, L)
    value = bytes_all / (ms_step * 1e-3) / 1e9
    achieved = norm_bytes(m_loc, L) / (ms_step * 1e-3) / 1e9  # per-GPU kernel achieved GB/s

    # parity rides along: a sampled matrix vs the oracle
    ref = O.softplus_norm_causal(x[0].float().cpu().numpy())
    err = float(np.abs(out[0].float().cpu().numpy() - ref).max())

    # e2e through the public API with pinned host buffers: every step uploads
    # the step's input from pinned host memory, runs the kernel and brings the
    # whole output back (softplus_norm_causal_host_out).  PCIe bounds this, so
    # only the bands of rows the causal kernel reads go up and only the bands it
    # can write nonzero come down (about half the bytes each way); the all-zero
    # columns past each band are written on the host while the GPU works.  The
    # matrices go in E2E_CHUNKS slices over upload / kernel / download streams.
    from smooth_attn import host as sa_host

    e2e_steps = max(1, min(args.steps, 5))
    xh = torch.empty(x.shape, dtype=x.dtype, pin_memory=True)
    xh.copy_(x)
    oh = torch.empty(x.shape, dtype=x.dtype, pin_memory=True)
    nch = E2E_CHUNKS if x.shape[0] % E2E_CHUNKS == 0 else 1
    band_bytes = sa_host.causal_band_bytes(x.shape, x.dtype)

    def e2e_step():
        sa.softplus_norm_causal_host_out(oh, xh, slices=nch)

    e2e_step()
    e2e_ok = bool(torch.equal(oh[:2].cuda(), out[:2]))  # the host path gives the device path's bits
    e2e_ms = time_steps(e2e_step, e2e_steps, world) / e2e_steps
    e2e_val = bytes_all / (e2e_ms * 1e-3) / 1e9

    flash = None
    if args.only == "all" and not args.skip_flash:
        flash = run_flash(args, world, rank, tf_burst, tf_sus, peak_kind)

    extra = None
    if args.only == "all" and not args.skip_extra:
        extra = run_extra(args, world, rank, hbm, tf_burst, tf_sus, peak_kind)
        if rank == 0:
            # the full per-shape records go to a file; the JSON line keeps a compact summary
            out_dir = ROOT / "gpurun_out"
            out_dir.mkdir(exist_ok=True)
            (out_dir / f"bench_other_configs_n{world}.json").write_text(json.dumps(extra, indent=1))
            extra = compact_extra(extra)

    long_ctx = None
    if args.only == "all" and not args.skip_extra:
        long_ctx = run_long_context(world, rank, tf_burst)

    cpu = None
    if rank == 0 and world == 1 and not args.skip_cpu:
        cpu = cpu_baseline(args.cpu_seconds)

    if rank == 0:
        line = {
            "metric": METRIC, "value": round(value, 1), "unit": "GB/s", "n_gpus": world, "steps": args.steps,
            "warmup": max(args.warmup, 3), "ms_per_step": round(ms_step, 4), "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "bf16", "data": "synthetic N(0,1), seeded",
            "config": {"workload": "causal squareplus norm fwd, out-buffer path (BASELINE configs[1], L=2048)",
                       "shape": [B, H, L, L], "alpha": 2.0, "theta": 0.5, "power": 2,
                       "parallelism": f"dp{world}: one [8,16,2048,2048] block of (b,h) matrices per GPU, no collective",
                       "l2": "inputs larger than L2 (1 GiB/step per GPU), no flush needed",
                       "max_abs_err_vs_oracle": err},
            "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": hbm, "unit": "GB/s",
                         "frac": round(achieved / hbm, 4), "traffic": args.traffic_bytes,
                         "peak_kind": f"{peak_kind} (MEASURED_PEAKS.json hbm_gbs)" if peak_kind == "measured" else "fallback",
                         "algorithmic_bytes_per_launch": norm_bytes(m_loc, L), "kernel": "sa::norm_fwd_bulk",
                         "traffic_source": "ncu dram bytes of one norm_fwd_bulk launch on bf16 [2,16,2048,2048], x4"},
            "e2e": {"value": round(e2e_val, 2), "unit": "GB/s", "h2d_bytes_per_step": band_bytes,
                    "d2h_bytes_per_step": band_bytes,
                    "path": f"softplus_norm_causal_host_out(pinned out, pinned x): the causal row bands the kernel "
                            f"reads go up and the bands it writes come down (cudaMemcpy3DAsync per 128-row band, "
                            f"{band_bytes} B each way of {x.numel() * 2}), the zero columns past the bands are "
                            f"written on the host; {nch} slices over upload / kernel / download streams",
                    "checked": e2e_ok},
            "gpu_launches": args.steps,
            "clocks": clk.summary(),
        }
        if cpu is not None:
            line["cpu_baseline"] = cpu
        if extra is not None:
            line["other_configs"] = extra
        if long_ctx is not None:
            line["long_context_fwd_strong"] = long_ctx
        if flash is not None:  # last: the second half of the metric survives a cut-off line tail
            line["flash_fwd_bwd"] = flash
        print(json.dumps(line), flush=True)


def run_flash(args, world, rank, tf_burst, tf_sus, peak_kind):
    """Fused squareplus attention fwd+bwd TFLOP/s at BASELINE configs[3]."""
    import smooth_attn as sa
    from oracle import sa_oracle as O

    B, H, T, D = (int(v) for v in args.flash_shape.split(","))
    b_loc = B * H  # this rank's block of (b,h) heads, laid out as [1, B*H, T, D]
    gen = torch.Generator().manual_seed(4321 + rank)
    mk = lambda: torch.randn(1, b_loc, T, D, generator=gen).to(torch.bfloat16).cuda().requires_grad_(True)  # noqa: E731
    q, k, v = mk(), mk(), mk()
    do = torch.randn(1, b_loc, T, D, generator=gen).to(torch.bfloat16).cuda()
    try:
        o = sa.sp2norm_flash_attention(q, k, v)
    except (ValueError, RuntimeError) as e:
        return {"unavailable": str(e)[:200]}

    det = bool(getattr(args, "deterministic", False))

    def step(det=det):
        o = sa.sp2norm_flash_attention(q, k, v, deterministic=det)
        torch.autograd.grad(o, (q, k, v), do)  # fresh dq/dk/dv, no .grad accumulation kernels

    for _ in range(max(args.warmup, 3)):
        step()
    # a seconds-long timed region (so the sustained peak is the right
    # denominator): as many steps as fill ~args.flash_seconds, at least 3
    probe = time_steps(step, 3, world) / 3
    steps = max(3, int(args.flash_seconds * 1e3 / probe))
    with ClockSampler(torch.cuda.current_device()) as clk:
        ms = time_steps(step, steps, world) / steps
    flops_all = world * (O.flash_flops(B, H, T, D) + O.flash_flops(B, H, T, D, bwd=True))
    flops_loc = O.flash_flops(1, b_loc, T, D) + O.flash_flops(1, b_loc, T, D, bwd=True)
    ach = flops_loc / (ms * 1e-3) / 1e12
    # forward-only timing for the roofline of the forward kernel (short region: burst peak)
    fsteps = max(3, steps // 3)
    fwd_ms = time_steps(lambda: sa.sp2norm_flash_attention(q.detach(), k.detach(), v.detach()), fsteps, world) / fsteps
    fwd_flops_loc = O.flash_flops(1, b_loc, T, D)
    # the bitwise-reproducible backward (query-major dQ) on the same inputs (short region)
    for _ in range(3):
        step(not det)
    other_ms = time_steps(lambda: step(not det), fsteps, world) / fsteps
    return {
        "metric": "fused squareplus-attn fwd+bwd TFLOP/s", "value": round(flops_all / (ms * 1e-3) / 1e12, 1),
        "unit": "TFLOP/s", "ms_per_step": round(ms, 3), "steps": steps,
        "timed_s": round(ms * steps * 1e-3, 2),
        "config": {"workload": "BASELINE configs[3]" if [B, H, T, D] == [4, 32, 4096, 128] else "custom",
                   "shape": [B, H, T, D], "dtype": "bf16", "causal": True,
                   "parallelism": f"dp{world}: one [{B},{H},{T},{D}] block of heads per GPU, no collective"},
        "roofline": {"bound": "tensor", "achieved": round(ach, 1), "peak": tf_sus, "unit": "TFLOP/s",
                     "frac": round(ach / tf_sus, 4), "peak_kind": f"{peak_kind} bf16_tflops_sustained",
                     "frac_of_burst": round(ach / tf_burst, 4), "burst_peak": tf_burst},
        "clocks": clk.summary(),
        "fwd_only": {"ms": round(fwd_ms, 3), "tflops": round(fwd_flops_loc / (fwd_ms * 1e-3) / 1e12, 1),
                     "frac_of_burst": round(fwd_flops_loc / (fwd_ms * 1e-3) / 1e12 / tf_burst, 4)},
        "deterministic": det,
        ("atomic_dq" if det else "deterministic_dq"): {
            "ms": round(other_ms, 3), "tflops": round(flops_loc / (other_ms * 1e-3) / 1e12, 1)},
    }


def run_long_context(world, rank, tf_burst):
    """BASELINE configs[4] as worded: ONE fixed [2,64,32768,128] forward whose
    128 (batch, head) units are split over the ranks (strong scaling, no
    collective on the data path).  After timing, the per-rank outputs are
    gathered over NCCL and, on rank 0, compared with the single-GPU forward of
    the whole problem (bitwise: each head runs the same kernel code either way)."""
    import smooth_attn as sa
    from oracle import sa_oracle as O
    from smooth_attn.parallel import gather_units, shard_units

    B, H, T, D = 2, 64, 32768, 128
    dev = torch.device("cuda")
    g = torch.Generator(device=dev).manual_seed(31337)  # the same full inputs on every rank
    q, k, v = (torch.randn(1, B * H, T, D, device=dev, generator=g).to(torch.bfloat16) for _ in range(3))
    start, count = shard_units(B * H, world, rank)
    ql, kl, vl = (t[:, start:start + count] for t in (q, k, v))
    f = lambda: sa.sp2norm_flash_attention(ql, kl, vl)  # noqa: E731
    for _ in range(2):
        f()
    steps = 3
    ms = time_steps(f, steps, world) / steps
    fl = O.flash_flops(B, H, T, D)
    res = {"config": "BASELINE configs[4]: bf16 [2,64,32768,128] causal forward, 128 (b,h) units split over "
                     f"{world} GPU(s), strong scaling, no collective", "units_per_rank": count,
           "ms": round(ms, 3), "TFLOP/s_all": round(fl / (ms * 1e-3) / 1e12, 1),
           "frac_of_burst_per_gpu": round(fl / (ms * 1e-3) / 1e12 / world / tf_burst, 3)}
    if world > 1:
        o_loc = f()[0]
        full = gather_units(o_loc, B * H)
        if rank == 0:
            ref = sa.sp2norm_flash_attention(q, k, v)[0]
            res["gathered_equals_single_gpu"] = bool(torch.equal(full, ref))
        del full
    del q, k, v
    torch.cuda.empty_cache()
    return res


def compact_extra(extra):
    """Short per-config numbers for the JSON line (full records go to a file)."""
    c = {}
    c["norm_L_sweep_GBs"] = {L: v["GB/s"] for L, v in extra["causal_norm_sweep"]["per_L"].items()}
    c["rowwise_fp32_GBs"] = extra["rowwise_fp32"]["GB/s"]
    c["norm_fwd_bwd_GBs"] = extra["causal_norm_fwd_bwd"]["GB/s"]
    c["norm_fwd_bwd_frac_hbm"] = extra["causal_norm_fwd_bwd"]["frac_hbm"]
    c["decode_GBs"] = {k.replace(" D=128 bs=16", ""): v["GB/s"] for k, v in extra["paged_decode"]["per_shape"].items()}
    c["rope_fwd_TFLOPs"] = {k: v["TFLOP/s"] for k, v in extra["rope_flash_fwd"]["per_shape"].items()}
    c["fp8_vs_bf16_fwd_TFLOPs"] = {k: [v["fp8"]["TFLOP/s"], v["bf16"]["TFLOP/s"]]
                                   for k, v in extra["fp8_flash_fwd"]["per_shape"].items()}
    c["out_proj_TFLOPs"] = {k: [v["tcgen05"]["TFLOP/s"], v["cublas"]["TFLOP/s"]]
                            for k, v in extra["out_proj"]["per_shape"].items()}
    if "config1_cpu" in extra:
        c["config1_cpu"] = extra["config1_cpu"]
    return c


def run_extra(args, world, rank, hbm, tf_burst, tf_sus, peak_kind):
    """The other BASELINE configs, one object each (parity spot-checks ride along).

    configs[1] sweep over L, configs[1] row-wise fp32, configs[2] causal norm
    forward + fused backward, plus the forward-only extensions: paged-KV decode at the reference's
    decode benchmark shapes (tests/test_paged_long_context.py:115-137) and
    RoPE attention at its RoPE benchmark shapes (tests/test_rope_proj.py:162-163).
    Inputs are generated on the device from seeded generators.
    """
    import smooth_attn as sa
    from oracle import sa_oracle as O

    dev = torch.device("cuda")
    g = torch.Generator(device=dev).manual_seed(777 + rank)
    out = {}

    def gbs(nbytes, ms):
        return round(nbytes / (ms * 1e-3) / 1e9, 1)

    # causal norm forward, bf16 [8,16,L,L], L swept
    sweep = {}
    for L in (128, 256, 512, 1024, 2048):
        x = torch.randn(8, 16, L, L, device=dev, generator=g).to(torch.bfloat16)
        o = torch.empty_like(x)
        n = max(20, 200 * 128 // L)
        for _ in range(3):
            sa.softplus_norm_causal_triton_out(o, x)
        ms = time_steps(lambda: sa.softplus_norm_causal_triton_out(o, x), n, world) / n
        b = norm_bytes(8 * 16, L)
        sweep[str(L)] = {"us": round(ms * 1e3, 2), "GB/s": gbs(b, ms), "frac_hbm": round(b / (ms * 1e-3) / 1e9 / hbm, 3),
                         "inputs_vs_L2": "larger" if x.numel() * 2 > 126e6 else "smaller (L2-resident, warm)"}
        del x, o
    out["causal_norm_sweep"] = {"config": "BASELINE configs[1]: bf16 [8,16,L,L] out-buffer path", "per_L": sweep}

    # configs[1] row-wise: fp32 [4,16,2048,2048] viewed [131072, 2048]
    x = torch.randn(131072, 2048, device=dev, generator=g)
    o = torch.empty_like(x)
    for _ in range(3):
        sa.softplus_norm_triton_out(o, x)
    ms = time_steps(lambda: sa.softplus_norm_triton_out(o, x), 50, world) / 50
    b = x.numel() * 8
    err = float((o[:4].cpu() - torch.from_numpy(O.softplus_norm(x[:4].cpu().numpy()))).abs().max())
    out["rowwise_fp32"] = {"config": "BASELINE configs[1] row-wise: fp32 [131072, 2048]", "ms": round(ms, 4),
                           "GB/s": gbs(b, ms), "frac_hbm": round(b / (ms * 1e-3) / 1e9 / hbm, 3),
                           "max_abs_err_vs_oracle": err}
    del x, o

    # causal norm forward + fused backward, bf16 [4,32,2048,2048]
    L, M = 2048, 4 * 32
    x = torch.randn(4, 32, L, L, device=dev, generator=g).to(torch.bfloat16).requires_grad_(True)
    dy = torch.randn(4, 32, L, L, device=dev, generator=g).to(torch.bfloat16)

    def fb():
        y = sa.softplus_norm_causal(x)
        torch.autograd.grad(y, x, dy)

    for _ in range(3):
        fb()
    ms = time_steps(fb, 20, world) / 20
    tri = L * (L + 1) // 2
    b = M * (2 * tri + 2 * L * L) + 4 * M * L + M * (2 * 2 * tri + 2 * L * L) + 4 * M * L
    out["causal_norm_fwd_bwd"] = {"config": "BASELINE configs[2]: bf16 [4,32,2048,2048] fwd + fused bwd (autograd)",
                                  "ms": round(ms, 4), "GB/s": gbs(b, ms),
                                  "frac_hbm": round(b / (ms * 1e-3) / 1e9 / hbm, 3), "algorithmic_bytes": b}
    del x, dy

    out["paged_decode"] = extra_decode(DECODE_SHAPES, 50, world, g, hbm, O)
    torch.cuda.empty_cache()
    out["rope_flash_fwd"] = extra_rope(ROPE_SHAPES, 20, world, g)
    torch.cuda.empty_cache()
    out["fp8_flash_fwd"] = extra_fp8(FP8_SHAPES, 20, world, g)
    torch.cuda.empty_cache()
    out["out_proj"] = extra_proj(PROJ_SHAPES, 20, world, g, tf_burst)
    torch.cuda.empty_cache()
    return out


# the reference's decode benchmark shapes (tests/test_paged_long_context.py:115-137), block 16
DECODE_SHAPES = ((1, 32, 8, 8192, 128, 16), (1, 32, 8, 32768, 128, 16), (8, 32, 8, 8192, 128, 16),
                 (32, 32, 8, 1024, 128, 16), (1, 12, 12, 32768, 64, 16), (8, 32, 32, 8192, 128, 16),
                 (64, 32, 8, 4096, 128, 16))
ROPE_SHAPES = ((2, 32, 1024, 128), (4, 12, 512, 64), (2, 32, 8192, 128))  # tests/test_rope_proj.py:162-163 + long
FP8_SHAPES = ((4, 8, 1024, 64), (2, 32, 8192, 128))  # tests/test_fp8_flash.py:126-127 + long
PROJ_SHAPES = ((2, 8192, 32, 128, 4096), (4, 2048, 32, 128, 4096))  # B, T, H, D, D_model of the RoPE projection
CP_SHAPE = (1, 32, 65536, 128)  # one long sequence split over the ranks (context parallelism)
E2E_CHUNKS = 8  # slices of the e2e step's batch (upload / compute / download pipeline)


def extra_cp(shape, steps, world, rank, g, tf_sus):
    """Context-parallel causal attention fwd+bwd over the ranks (strong scaling:
    one sequence, total work fixed): TFLOP/s of the whole job, K/V all-gather
    and dK/dV reduce-scatter inside the timed region."""
    import smooth_attn.parallel as par
    from oracle import sa_oracle as O

    B, H, T, D = shape
    dev = torch.device("cuda")
    w = max(world, 1)
    if T % (2 * w):
        raise SystemExit(f"T={T} must divide into 2*world chunks")
    loc = [torch.randn(B, H, T // w, D, device=dev, generator=g).to(torch.bfloat16).requires_grad_(True)
           for _ in range(3)]
    do = torch.randn(B, H, T // w, D, device=dev, generator=g).to(torch.bfloat16)
    if world > 1:
        step = lambda: torch.autograd.backward(par.context_parallel_attention(*loc), do)  # noqa: E731
    else:  # one rank: the plain single-GPU autograd forward + backward
        import smooth_attn as sa

        step = lambda: torch.autograd.backward(sa.sp2norm_flash_attention(*loc), do)  # noqa: E731
    for _ in range(2):
        step()
    ms = time_steps(step, steps, world) / steps
    fl = O.flash_flops(B, H, T, D) + O.flash_flops(B, H, T, D, bwd=True)
    return {"config": f"context-parallel fwd+bwd, bf16 [{B},{H},{T},{D}] split over {w} rank(s), "
                      "zig-zag chunks, NCCL all-gather K/V + reduce-scatter dK/dV", "scaling": "strong",
            "ms": round(ms, 3), "TFLOP/s_all": round(fl / (ms * 1e-3) / 1e12, 1),
            "TFLOP/s_per_gpu": round(fl / (ms * 1e-3) / 1e12 / w, 1),
            "frac_of_sustained_per_gpu": round(fl / (ms * 1e-3) / 1e12 / w / tf_sus, 3)}


def _gbs(nbytes, ms):
    return round(nbytes / (ms * 1e-3) / 1e9, 1)


def extra_decode(shapes, steps, world, g, hbm, O):
    """Paged-KV decode: GB/s of K+V bytes read, one public-API call per step,
    back to back; the B=1 T=8192 shape is spot-checked against the oracle."""
    import smooth_attn as sa

    dev = torch.device("cuda")
    dec = {}
    for B, Hq, Hkv, T, D, BS in shapes:
        nb = B * T // BS
        q = torch.randn(B, Hq, 1, D, device=dev, generator=g).to(torch.bfloat16)
        kc = torch.randn(nb, Hkv, BS, D, device=dev, generator=g).to(torch.bfloat16)
        vc = torch.randn(nb, Hkv, BS, D, device=dev, generator=g).to(torch.bfloat16)
        bt = torch.randperm(nb, device=dev, generator=g).to(torch.int32).view(B, -1)
        cl = torch.full((B,), T, dtype=torch.int32, device=dev)
        f = lambda: sa.sp2norm_paged_attention(q, kc, vc, bt, cl, block_size=BS)  # noqa: E731
        for _ in range(3):
            f()
        ms = time_steps(f, steps, world) / steps
        b = B * T * Hkv * D * 4
        key = f"B={B} H={Hq}/{Hkv} T={T} D={D} bs={BS}"
        dec[key] = {"us": round(ms * 1e3, 1), "GB/s": _gbs(b, ms), "frac_hbm": round(b / (ms * 1e-3) / 1e9 / hbm, 3),
                    "kv_bytes": b, "inputs_vs_L2": "larger" if b > 126e6 else "smaller (L2-resident, warm)",
                    "kernel": "tcgen05" if (Hq // Hkv >= 2 and D == 128) else "cuda-core"}
        if B <= 8:
            # the same call captured once in a CUDA graph and replayed, as a
            # serving loop would: what is left is the kernels' own latency
            side = torch.cuda.Stream()
            side.wait_stream(torch.cuda.current_stream())
            with torch.cuda.stream(side):
                for _ in range(2):
                    f()
            torch.cuda.current_stream().wait_stream(side)
            graph = torch.cuda.CUDAGraph()
            # no garbage collection mid-capture (a collected graph would free
            # its pool and invalidate this capture)
            gc.collect()
            gc.disable()
            try:
                with torch.cuda.graph(graph, capture_error_mode="thread_local"):
                    f()
            finally:
                gc.enable()
            for _ in range(3):
                graph.replay()
            ms_g = time_steps(graph.replay, steps, world) / steps
            dec[key]["graph_replay_us"] = round(ms_g * 1e3, 1)
            dec[key]["graph_replay_frac_hbm"] = round(b / (ms_g * 1e-3) / 1e9 / hbm, 3)
            del graph
        if B == 1 and T == 8192:
            o = f()
            ref = O.paged_decode_attention(q.float().cpu().numpy(), kc.float().cpu().numpy(),
                                           vc.float().cpu().numpy(), bt.cpu().numpy(), cl.cpu().numpy())
            dec[key]["max_abs_err_vs_oracle"] = float(np.abs(o.float().cpu().numpy() - ref).max())
        del q, kc, vc, bt, cl
    return {"config": "paged KV decode, bf16, shuffled pages, public API per call", "per_shape": dec}


def extra_rope(shapes, steps, world, g):
    """RoPE attention forward (rotation pass + tcgen05 forward), TFLOP/s of the attention."""
    import smooth_attn as sa
    from oracle import sa_oracle as O

    dev = torch.device("cuda")
    rope = {}
    for B, H, T, D in shapes:
        q, k, v = (torch.randn(B, H, T, D, device=dev, generator=g).to(torch.bfloat16) for _ in range(3))
        cos, sin = sa.precompute_rope_cos_sin(D, T, device=dev)
        f = lambda: sa.sp2norm_rope_flash_attention(q, k, v, cos, sin)  # noqa: E731
        for _ in range(3):
            f()
        ms = time_steps(f, steps, world) / steps
        fl = O.flash_flops(B, H, T, D)
        rope[f"B={B} H={H} T={T} D={D}"] = {"us": round(ms * 1e3, 1), "TFLOP/s": round(fl / (ms * 1e-3) / 1e12, 1)}
        del q, k, v
    return {"config": "RoPE + causal squareplus attention forward, bf16, public API per call", "per_shape": rope}


def extra_fp8(shapes, steps, world, g):
    """FP8 attention forward (device quantization + E4M3 QK^T forward) beside the bf16 forward."""
    import smooth_attn as sa
    from oracle import sa_oracle as O

    dev = torch.device("cuda")
    f8 = {}
    for B, H, T, D in shapes:
        q, k, v = (torch.randn(B, H, T, D, device=dev, generator=g).to(torch.bfloat16) for _ in range(3))
        fl = O.flash_flops(B, H, T, D)
        row = {}
        for name, fn in (("fp8", lambda: sa.sp2norm_fp8_flash_attention(q, k, v)),
                         ("bf16", lambda: sa.sp2norm_flash_attention(q, k, v))):
            for _ in range(3):
                fn()
            ms = time_steps(fn, steps, world) / steps
            row[name] = {"us": round(ms * 1e3, 1), "TFLOP/s": round(fl / (ms * 1e-3) / 1e12, 1)}
        f8[f"B={B} H={H} T={T} D={D}"] = row
        del q, k, v
    return {"config": "FP8 (E4M3 QK^T) causal squareplus attention forward incl. quantization, "
                      "public API per call; bf16 forward beside it", "per_shape": f8}


def extra_proj(shapes, steps, world, g, tf_burst):
    """RoPE attention output projection: [B*T, H*D] @ [H*D, D_model] on the
    tcgen05 GEMM (sa_out_proj), beside cuBLAS (torch.matmul) on the same
    operands for scale."""
    import smooth_attn.kernels as K

    dev = torch.device("cuda")
    res = {}
    for B, T, H, D, DM in shapes:
        a = torch.randn(B * T, H * D, device=dev, generator=g).to(torch.bfloat16)
        w = (torch.randn(H * D, DM, device=dev, generator=g) * 0.02).to(torch.bfloat16)
        fl = 2.0 * B * T * H * D * DM
        row = {}
        for name, fn in (("tcgen05", lambda: K._out_proj(a, w)), ("cublas", lambda: torch.matmul(a, w))):
            for _ in range(3):
                fn()
            ms = time_steps(fn, steps, world) / steps
            row[name] = {"us": round(ms * 1e3, 1), "TFLOP/s": round(fl / (ms * 1e-3) / 1e12, 1)}
        row["frac_of_burst"] = round(row["tcgen05"]["TFLOP/s"] / tf_burst, 3)
        res[f"M={B * T} K={H * D} N={DM}"] = row
        del a, w
    return {"config": "RoPE projection GEMM, bf16 operands, fp32 accumulation", "per_shape": res}


CPU_BLOCK_ROWS = 128  # CPU sample unit: a 128-row block of one [2048, 2048] causal matrix


def _block_bytes(q0, rows=CPU_BLOCK_ROWS, L=NORM_CFG["L"], e=2):
    """Algorithmic bytes of a row block: visible prefix of each row read + full rows written."""
    return e * sum(q + 1 for q in range(q0, q0 + rows)) + e * rows * L


def _cpu_norm_sample(seconds, threads, min_batches=1):
    """Time the oracle port on 128-row blocks of L=2048 causal matrices, one
    block per thread per batch, for ~`seconds` (at least `min_batches`).
    Returns (algorithmic bytes processed, seconds)."""
    from oracle import sa_oracle as O

    L = NORM_CFG["L"]
    rng = np.random.default_rng(0)
    nblk = L // CPU_BLOCK_ROWS
    work = [(rng.standard_normal((CPU_BLOCK_ROWS, L), dtype=np.float32), (i % nblk) * CPU_BLOCK_ROWS)
            for i in range(threads)]
    nbytes, batches = 0, 0
    t0 = time.perf_counter()
    with ThreadPoolExecutor(max_workers=threads) as ex:
        while True:
            list(ex.map(lambda w: O.softplus_norm_causal_rows(w[0], w[1]), work))
            nbytes += sum(_block_bytes(q0) for _, q0 in work)
            batches += 1
            if batches >= min_batches and time.perf_counter() - t0 > seconds:
                break
    return nbytes, time.perf_counter() - t0


def cpu_config1(reps=20):
    """BASELINE configs[0] timed in full on the host: causal squareplus norm of
    fp32 [2,8,128,128] N(0,1) scores (alpha 2, theta 0.5, power 2), forward and
    forward + eager autograd backward with an N(0,1) upstream gradient, through
    the reference's eager algorithm in torch (``softplus_norm_causal_eager``:
    the activation, the cached triu mask, masked_fill, the row sum + 1e-12,
    src/smooth_attn/kernels.py:1349-1365) on all host threads, and through the
    numpy port for comparison.  Median of ``reps`` runs after 3 warm-ups."""
    import smooth_attn as sa
    from oracle import sa_oracle as O

    torch.set_num_threads(os.cpu_count() or 1)
    g = torch.Generator().manual_seed(1234)
    x = torch.randn(2, 8, 128, 128, generator=g)
    dy = torch.randn(2, 8, 128, 128, generator=g)

    def med(fn):
        for _ in range(3):
            fn()
        ts = []
        for _ in range(reps):
            t0 = time.perf_counter()
            fn()
            ts.append(time.perf_counter() - t0)
        return round(statistics.median(ts) * 1e6, 1)

    def fwd_bwd():
        xr = x.clone().requires_grad_(True)
        sa.softplus_norm_causal_eager(xr).backward(dy)

    xn, dyn = x.numpy(), dy.numpy()
    return {"config": "BASELINE configs[0]: fp32 [2,8,128,128], alpha 2, theta 0.5, power 2",
            "torch_eager_fwd_us": med(lambda: sa.softplus_norm_causal_eager(x)),
            "torch_eager_fwd_bwd_us": med(fwd_bwd),
            "numpy_port_fwd_us": med(lambda: O.softplus_norm_causal(xn)),
            "numpy_port_fwd_bwd_us": med(lambda: (O.softplus_norm_causal(xn), O.softplus_norm_causal_bwd(xn, dyn))),
            "threads": torch.get_num_threads()}


def cpu_baseline(seconds=10.0):
    threads = os.cpu_count() or 1
    nbytes, dt = _cpu_norm_sample(seconds, threads)
    gbs = nbytes / dt / 1e9
    return {"value": round(gbs, 3), "unit": "GB/s", "cores": threads, "kind": "port",
            "sample": f"{nbytes / norm_bytes(1, NORM_CFG['L']):.1f} matrix-equivalents of [2048,2048] as 128-row "
                      f"blocks (numpy oracle, fp32 math, bf16-sized bytes), "
                      f"{dt:.1f} s, {threads} threads",
            "config1": cpu_config1()}


def run_reference(args):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    threads = os.cpu_count() or 1
    # whole run ~90 s whatever K is: per step one batch of blocks at minimum
    budget = min(20.0, 90.0 / max(1, args.steps + args.warmup))
    for _ in range(args.warmup):
        _cpu_norm_sample(budget, threads)
    vals = []
    t_all = time.perf_counter()
    for _ in range(args.steps):
        nbytes, dt = _cpu_norm_sample(budget, threads)
        vals.append(nbytes / dt / 1e9)
    t_all = time.perf_counter() - t_all
    v = statistics.median(vals)
    line = {
        "impl": "reference", "metric": METRIC, "value": round(v, 3), "unit": "GB/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic N(0,1), seeded",
        "config": {"workload": "causal squareplus norm fwd (BASELINE configs[1], L=2048), CPU port of the "
                               "reference eager algorithm", "shape": [8, 16, 2048, 2048]},
        "cpu_baseline": {"value": round(v, 3), "unit": "GB/s", "cores": threads, "kind": "port",
                         "sample": f"each step >= one batch of {threads} 128-row blocks of [2048,2048] causal "
                                   f"matrices (>= {budget:.2f} s); {args.steps} steps in {t_all:.1f} s; "
                                   f"median step"},
        "e2e": {"value": round(v, 3), "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    line["cpu_baseline"]["config1"] = cpu_config1()
    print(json.dumps(line), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=2000)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=("ours", "reference"), default="ours")
    ap.add_argument("--skip-flash", action="store_true")
    ap.add_argument("--only", choices=("all", "norm", "flash", "decode", "rope", "fp8", "cp"), default="all",
                    help="run one workload only (small-case profiling)")
    ap.add_argument("--shape", default=None,
                    help="with --only decode: B,Hq,Hkv,T,D,block_size; rope / fp8 / cp: B,H,T,D (one shape)")
    ap.add_argument("--norm-batch", type=int, default=NORM_CFG["B"],
                    help="B of the causal-norm workload [B,16,2048,2048] (BASELINE: 8)")
    ap.add_argument("--flash-shape", default=",".join(str(FLASH_CFG[k]) for k in "BHTD"),
                    help="B,H,T,D of the attention workload (BASELINE: 4,32,4096,128)")
    ap.add_argument("--skip-cpu", action="store_true")
    ap.add_argument("--deterministic", action="store_true",
                    help="flash fwd+bwd through the bitwise-reproducible backward (query-major dQ)")
    ap.add_argument("--skip-extra", action="store_true", help="skip the other BASELINE configs")
    ap.add_argument("--cpu-seconds", type=float, default=10.0)
    ap.add_argument("--flash-seconds", type=float, default=2.0,
                    help="length of the flash fwd+bwd timed region (seconds)")
    ap.add_argument("--traffic-bytes", type=float, default=NORM_TRAFFIC_BYTES,
                    help="ncu dram bytes per launch of the norm kernel, if measured")
    args = ap.parse_args()
    if args.impl == "reference":
        run_reference(args)
    else:
        try:
            run_ours(args)
        finally:  # every path, the single-workload ones included, leaves the process group cleanly
            import torch.distributed as dist

            if dist.is_available() and dist.is_initialized():
                dist.destroy_process_group()


if __name__ == "__main__":
    main()

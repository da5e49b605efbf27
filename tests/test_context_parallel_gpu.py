"""Context parallelism on the GPU: the query-chunk forward and backward
(``sa_flash_fwd_chunk`` / ``sa_flash_bwd_chunk``) against the oracle, chunks
that reproduce the full forward and backward, and — when two GPUs are
visible — two NCCL ranks running ``context_parallel_attention`` forward and
backward on zig-zag sequence blocks against the single-GPU autograd."""

import os
import socket

import numpy as np
import pytest
import torch

import smooth_attn as sa
from oracle import sa_oracle as O
from tests._util import assert_close, check_bf16_grads, np32, randn

pytestmark = pytest.mark.gpu
CUDA = "cuda"
FWD_TOL = dict(rtol=2e-2, atol=1e-2)  # bf16 attention output vs the fp32 oracle (as the flash tests)


@pytest.fixture(autouse=True)
def _need_cuda():
    if not torch.cuda.is_available():
        pytest.skip("CUDA required")


@pytest.mark.parametrize("Tq,Tk,off,D,window", [(128, 256, 128, 128, 0), (100, 300, 200, 64, 0),
                                                (256, 1000, 744, 128, 0), (64, 64, 0, 32, 0),
                                                (200, 700, 500, 128, 96), (130, 130, 0, 64, 17),
                                                (77, 900, 823, 128, 0)])
def test_chunk_forward_matches_oracle(Tq, Tk, off, D, window):
    q = randn((2, 4, Tq, D), Tq + off, torch.bfloat16, CUDA)
    k = randn((2, 2, Tk, D), Tk, torch.bfloat16, CUDA)
    v = randn((2, 2, Tk, D), Tk + 1, torch.bfloat16, CUDA)
    o, rs = sa.sp2norm_flash_attention_chunk(q, k, v, off, window_size=window)
    ref = O.chunk_flash_attention(np32(q), np32(k), np32(v), off, window_size=window)
    assert_close(np32(o), ref, **FWD_TOL)
    assert torch.isfinite(rs).all() and (rs > 0).all()


@pytest.mark.parametrize("T,chunks,window", [(1024, 4, 0), (2048, 8, 0), (1536, 6, 200)])
def test_chunks_reproduce_full_forward(T, chunks, window):
    q, k, v = (randn((1, h, T, 128), T + h, torch.bfloat16, CUDA) for h in (8, 2, 2))
    full = sa.sp2norm_flash_attention(q, k, v, window_size=window)
    C = T // chunks
    parts = [sa.sp2norm_flash_attention_chunk(q[:, :, c * C:(c + 1) * C].contiguous(), k[:, :, :(c + 1) * C],
                                              v[:, :, :(c + 1) * C], c * C, window_size=window)[0]
             for c in range(chunks)]
    got = torch.cat(parts, dim=2)
    assert (got.float() - full.float()).abs().max().item() <= 2e-2


BWD_TOL = dict(rtol=2e-2, atol=1e-2)  # the flash tests' backward tolerance


@pytest.mark.parametrize("Tq,Tk,off,D,window,Hq,Hkv", [(128, 256, 128, 128, 0, 4, 2), (100, 300, 200, 64, 0, 2, 2),
                                                       (256, 1000, 744, 128, 0, 4, 1), (64, 64, 0, 32, 0, 2, 2),
                                                       (200, 700, 500, 128, 96, 4, 2), (77, 900, 823, 64, 0, 2, 1),
                                                       (128, 1024, 896, 128, 50, 2, 2)])
def test_chunk_backward_matches_oracle(Tq, Tk, off, D, window, Hq, Hkv):
    """dq of the query block and its dk / dv contribution over the key prefix;
    with a window, keys no query of the block sees get exactly zero."""
    q = randn((1, Hq, Tq, D), Tq + off, torch.bfloat16, CUDA)
    k = randn((1, Hkv, Tk, D), Tk, torch.bfloat16, CUDA)
    v = randn((1, Hkv, Tk, D), Tk + 1, torch.bfloat16, CUDA)
    do = randn((1, Hq, Tq, D), 7, torch.bfloat16, CUDA)
    o, rs, lo = sa.sp2norm_flash_attention_chunk(q, k, v, off, window_size=window, return_residual=True)
    dq, dk, dv = sa.kernels.sp2norm_flash_attention_chunk_bwd(q, k, v, o, do, rs, off, window_size=window, o_lo=lo)
    args = (np32(q), np32(k), np32(v), np32(do), off)
    ref = O.chunk_flash_attention_bwd(*args, window_size=window, acc=np.float64)
    emu = O.chunk_flash_attention_bwd(*args, window_size=window, emulate=True)
    for g, r, m in zip((dq, dk, dv), ref, emu):
        check_bf16_grads(np32(g), r, m, **BWD_TOL)
    if window:
        first_seen = max(0, off - window + 1)
        assert (dk[:, :, :first_seen] == 0).all() and (dv[:, :, :first_seen] == 0).all()


def test_chunked_backward_reproduces_full_backward():
    """Chunk backwards summed over a split sequence equal the full backward's
    oracle gradients (dK / dV summed in fp32 over the chunks)."""
    T, chunks = 2048, 4
    q, k, v = (randn((1, h, T, 128), T + h, torch.bfloat16, CUDA) for h in (8, 2, 2))
    do = randn((1, 8, T, 128), 3, torch.bfloat16, CUDA)
    args = (np32(q), np32(k), np32(v), np32(do))
    ref = O.sp2norm_flash_attention_bwd(*args, acc=np.float64)
    emu = O.sp2norm_flash_attention_bwd(*args, emulate=True)
    C = T // chunks
    dk_acc = torch.zeros(k.shape, dtype=torch.float32, device=CUDA)
    dv_acc = torch.zeros_like(dk_acc)
    dqs = []
    for c in range(chunks):
        e = (c + 1) * C
        qc, doc = q[:, :, c * C:e].contiguous(), do[:, :, c * C:e].contiguous()
        o, rs, lo = sa.sp2norm_flash_attention_chunk(qc, k[:, :, :e], v[:, :, :e], c * C, return_residual=True)
        dq, dk, dv = sa.kernels.sp2norm_flash_attention_chunk_bwd(qc, k[:, :, :e], v[:, :, :e], o, doc, rs, c * C,
                                                                  o_lo=lo)
        dqs.append(dq)
        dk_acc[:, :, :e] += dk.float()
        dv_acc[:, :, :e] += dv.float()
    for g, r, m in zip((torch.cat(dqs, dim=2), dk_acc, dv_acc), ref, emu):
        check_bf16_grads(np32(g), r, m, **BWD_TOL)


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _cp_worker(rank, world, port, q):
    import torch.distributed as dist
    from datetime import timedelta

    from smooth_attn.parallel import _all_gather, context_parallel_attention, zigzag_merge, zigzag_split

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=60))
    try:
        g = torch.Generator().manual_seed(5)
        qf, kf, vf = (torch.randn(1, h, 4096, 128, generator=g).to(torch.bfloat16).cuda() for h in (16, 4, 4))
        dof = torch.randn(1, 16, 4096, 128, generator=g).to(torch.bfloat16).cuda()
        loc = [zigzag_split(t, world, rank).requires_grad_(True) for t in (qf, kf, vf)]
        o_local = context_parallel_attention(*loc)
        (o_local * zigzag_split(dof, world, rank)).sum().backward()
        o = zigzag_merge(_all_gather(o_local.detach()))
        grads = [zigzag_merge(_all_gather(t.grad)) for t in loc]
        full = [t.clone().requires_grad_(True) for t in (qf, kf, vf)]
        ref = sa.sp2norm_flash_attention(*full)
        (ref * dof).sum().backward()
        # allclose-style count of elements off by more than atol + rtol * |ref|
        # (bf16 gradients: the chunked dK/dV are sums of per-chunk bf16 partials)
        def bad(a, b, tol):
            a, b = a.detach().float(), b.detach().float()
            return int(((a - b).abs() > tol + tol * b.abs()).sum())

        nbad = bad(o, ref, 2e-2) + sum(bad(a, b.grad, 5e-2) for a, b in zip(grads, full))
        q.put((rank, "ok", nbad))
    except Exception as e:  # report, never hang
        q.put((rank, "error", repr(e)[:200]))
    finally:
        try:
            dist.destroy_process_group()
        except Exception:
            pass


def test_context_parallel_two_gpus_equals_single_gpu():
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    import torch.multiprocessing as mp

    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_cp_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=300)
        if p.is_alive():
            p.kill()
            pytest.fail("rank did not finish")
    res = sorted(q.get(timeout=5) for _ in range(2))
    assert [r[1] for r in res] == ["ok", "ok"], res
    assert all(r[2] == 0 for r in res), res

"""Context parallelism on the GPU: the query-chunk forward (``sa_flash_fwd_chunk``
through ``sp2norm_flash_attention_chunk``) against the oracle, chunks that
reproduce the full forward, and — when two GPUs are visible — two NCCL ranks
running ``context_parallel_attention`` on zig-zag sequence blocks against the
single-GPU forward."""

import os
import socket

import numpy as np
import pytest
import torch

import smooth_attn as sa
from oracle import sa_oracle as O
from tests._util import assert_close, np32, randn

pytestmark = pytest.mark.gpu
CUDA = "cuda"
FWD_TOL = dict(rtol=5e-2, atol=2e-2)  # bf16 attention output vs the fp32 oracle (as the flash tests)


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
        o_local = context_parallel_attention(*(zigzag_split(t, world, rank) for t in (qf, kf, vf)))
        o = zigzag_merge(_all_gather(o_local))
        ref = sa.sp2norm_flash_attention(qf, kf, vf)
        q.put((rank, "ok", float((o.float() - ref.float()).abs().max())))
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
    assert all(r[2] <= 2e-2 for r in res), res

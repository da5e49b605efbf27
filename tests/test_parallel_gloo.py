"""Host-side multi-rank logic on CPU: world-size-2 gloo ranks shard (batch,
head) units, compute their blocks, and the gathered result equals the
single-process result.  Also the block arithmetic and a rank failure seen by
the other rank as an error (never a hang)."""

import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from oracle import sa_oracle as O
from smooth_attn.parallel import gather_units, shard_heads, shard_kv_groups, shard_units


def test_shard_units_covers_everything_once():
    for n in (0, 1, 7, 8, 128, 129):
        for world in (1, 2, 3, 4, 8):
            seen = []
            for r in range(world):
                s, c = shard_units(n, world, r)
                seen.extend(range(s, s + c))
            assert seen == list(range(n))
    with pytest.raises(ValueError):
        shard_units(4, 2, 2)


def test_shard_kv_groups_keeps_gqa_groups_whole():
    q = torch.arange(2 * 8 * 3 * 4, dtype=torch.float32).reshape(2, 8, 3, 4)
    k = torch.arange(2 * 2 * 3 * 4, dtype=torch.float32).reshape(2, 2, 3, 4)
    qs, ks, vs = shard_kv_groups(q, k, k, world=4, rank=1)  # unit 1 = (b0, kv head 1)
    assert torch.equal(ks[0, 0], k[0, 1])
    assert torch.equal(qs[0], q[0, 4:8])


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _worker(rank, world, port, mode, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    from datetime import timedelta

    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=20))
    try:
        g = torch.Generator().manual_seed(0)
        x = torch.randn(3, 5, 12, 12, generator=g)  # 15 units: uneven split
        if mode == "fail" and rank == 1:
            raise RuntimeError("injected host-side failure on rank 1")
        local = shard_heads(x, world, rank)
        y_local = torch.from_numpy(O.softplus_norm_causal(local.numpy()))
        full = gather_units(y_local, 15)
        ref = O.softplus_norm_causal(x.reshape(15, 12, 12).numpy())
        q.put((rank, "ok", float(np.abs(full.numpy() - ref).max())))
    except Exception as e:  # report, never hang
        q.put((rank, "error", type(e).__name__))
    finally:
        try:
            dist.destroy_process_group()
        except Exception:
            pass


def _run(mode):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, mode, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
        if p.is_alive():
            p.kill()
            pytest.fail("rank did not finish")
    return sorted(q.get(timeout=5) for _ in range(2))


def test_gloo_world2_shard_compute_gather_equals_single_process():
    res = _run("ok")
    assert [r[1] for r in res] == ["ok", "ok"], res
    assert all(r[2] == 0.0 for r in res)


def test_gloo_world2_rank_failure_surfaces_as_error():
    res = _run("fail")
    assert res[1][1] == "error"  # the failing rank
    assert res[0][1] == "error"  # the survivor's collective errors out instead of hanging

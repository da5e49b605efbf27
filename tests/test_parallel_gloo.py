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
from smooth_attn.parallel import (
    _all_gather,
    context_parallel_attention,
    gather_units,
    shard_heads,
    shard_kv_groups,
    shard_units,
    zigzag_chunk_ids,
    zigzag_merge,
    zigzag_split,
)


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


def test_zigzag_split_merge_round_trip_and_balance():
    x = torch.arange(2 * 3 * 24 * 2, dtype=torch.float32).reshape(2, 3, 24, 2)
    for world in (1, 2, 3, 4):
        parts = [zigzag_split(x, world, r) for r in range(world)]
        assert torch.equal(zigzag_merge(parts), x)
        # causal work of a rank = key chunks seen by its two query chunks: equal for all ranks
        work = {sum(c + 1 for c in zigzag_chunk_ids(world, r)) for r in range(world)}
        assert work == {2 * world + 1}
    with pytest.raises(ValueError):
        zigzag_split(x, 5, 0)


@pytest.mark.parametrize("window", [0, 5, 40])
def test_oracle_query_chunks_reproduce_full_attention(window):
    """The restatement behind the chunk kernel: query chunks at their global
    offset against the key prefix give the full causal forward."""
    g = np.random.default_rng(3)
    q = g.standard_normal((1, 4, 48, 16)).astype(np.float32)
    k = g.standard_normal((1, 2, 48, 16)).astype(np.float32)
    v = g.standard_normal((1, 2, 48, 16)).astype(np.float32)
    full = O.sp2norm_flash_attention(q, k, v, window_size=window)
    C = 12
    parts = [O.chunk_flash_attention(q[:, :, c * C:(c + 1) * C], k[:, :, :(c + 1) * C], v[:, :, :(c + 1) * C],
                                     c * C, window_size=window) for c in range(4)]
    np.testing.assert_allclose(np.concatenate(parts, axis=2), full, rtol=1e-5, atol=1e-6)


def test_oracle_query_chunks_reproduce_full_backward():
    g = np.random.default_rng(4)
    q = g.standard_normal((1, 4, 48, 16)).astype(np.float32)
    k = g.standard_normal((1, 2, 48, 16)).astype(np.float32)
    v = g.standard_normal((1, 2, 48, 16)).astype(np.float32)
    do = g.standard_normal((1, 4, 48, 16)).astype(np.float32)
    rq, rk, rv = O.sp2norm_flash_attention_bwd(q, k, v, do, window_size=9)
    C = 12
    dk = np.zeros_like(k)
    dv = np.zeros_like(v)
    dqs = []
    for c in range(4):
        e = (c + 1) * C
        gq, gk, gv = O.chunk_flash_attention_bwd(q[:, :, c * C:e], k[:, :, :e], v[:, :, :e], do[:, :, c * C:e],
                                                 c * C, window_size=9)
        dqs.append(gq)
        dk[:, :, :e] += gk
        dv[:, :, :e] += gv
    for a, b in ((np.concatenate(dqs, axis=2), rq), (dk, rk), (dv, rv)):
        np.testing.assert_allclose(a, b, rtol=1e-4, atol=1e-5)


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
        if mode.startswith("cp"):
            # context parallelism: the gather / reorder / chunk / reduce-scatter
            # logic, forward and backward, with the chunk kernels replaced by
            # the oracle (CPU ranks, no GPU)
            import smooth_attn.kernels as K

            def chunk(qc, kp, vp, off, scale=None, window_size=0, return_residual=False):
                o = O.chunk_flash_attention(qc.numpy(), kp.numpy(), vp.numpy(), off, scale=scale,
                                            window_size=window_size)
                o = torch.from_numpy(o)
                res = (o, torch.ones(qc.shape[:3]))
                return res + (torch.zeros_like(o),) if return_residual else res

            def chunk_bwd(qc, kp, vp, o, do, sums, off, scale=None, window_size=0, o_lo=None):
                g = O.chunk_flash_attention_bwd(qc.detach().numpy(), kp.detach().numpy(), vp.detach().numpy(),
                                                do.numpy(), off, scale=scale, window_size=window_size)
                return tuple(torch.from_numpy(t) for t in g)

            K.sp2norm_flash_attention_chunk = chunk
            K.sp2norm_flash_attention_chunk_bwd = chunk_bwd
            window = int(mode[2:] or 0)
            g = torch.Generator().manual_seed(1)
            qf, kf, vf = (torch.randn(2, h, 40, 8, generator=g) for h in (4, 2, 2))
            dof = torch.randn(2, 4, 40, 8, generator=g)
            loc = [zigzag_split(t, world, rank).requires_grad_(True) for t in (qf, kf, vf)]
            o_local = context_parallel_attention(*loc, window_size=window)
            (o_local * zigzag_split(dof, world, rank)).sum().backward()
            o = zigzag_merge(_all_gather(o_local.detach()))
            grads = [zigzag_merge(_all_gather(t.grad)) for t in loc]
            ref = O.sp2norm_flash_attention(qf.numpy(), kf.numpy(), vf.numpy(), window_size=window)
            rg = O.sp2norm_flash_attention_bwd(qf.numpy(), kf.numpy(), vf.numpy(), dof.numpy(), window_size=window)
            err = max([float(np.abs(o.numpy() - ref).max())] +
                      [float(np.abs(a.numpy() - b).max()) for a, b in zip(grads, rg)])
            q.put((rank, "ok", err))
            return
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


@pytest.mark.parametrize("mode", ["cp", "cp7", "cp13"])
def test_gloo_world2_context_parallel_equals_single_process(mode):
    res = _run(mode)
    assert [r[1] for r in res] == ["ok", "ok"], res
    assert all(r[2] < 1e-5 for r in res), res

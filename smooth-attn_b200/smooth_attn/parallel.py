"""Multi-GPU plumbing for the smooth-attn path: one process per GPU.

The normalization and attention work is a set of independent units — score
matrices (batch, head) for the norm, (batch, kv-head) groups for attention
(GQA groups stay whole because a kv head's gradients sum over its query
heads).  Units are split into contiguous blocks, one per rank, and every
rank runs the single-GPU kernels on its block; there is no collective on the
data path.  ``gather_units`` collects the per-rank blocks (NCCL over NVLink on
GPUs, gloo on CPU) for validation only.

Context (sequence) parallelism for sequences too long for one GPU's block of
heads is the one exchange step: ``context_parallel_attention`` (below).
"""

from __future__ import annotations

import torch
import torch.distributed as dist


def shard_units(n_units: int, world: int, rank: int) -> tuple[int, int]:
    """Contiguous block of ``n_units`` owned by ``rank``: (start, count).

    Blocks differ in size by at most one unit; the first ``n_units % world``
    ranks take the larger blocks.
    """
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"bad rank {rank} for world size {world}")
    if n_units < 0:
        raise ValueError("n_units must be non-negative")
    base, extra = divmod(n_units, world)
    start = rank * base + min(rank, extra)
    return start, base + (1 if rank < extra else 0)


def shard_heads(x: torch.Tensor, world: int, rank: int, head_dim: int = 1) -> torch.Tensor:
    """This rank's block of the flattened (batch, head) units of ``x``.

    ``x`` is ``[B, H, ...]``; the result is ``[count, ...]`` (a view when possible).
    """
    B, H = x.shape[0], x.shape[head_dim]
    flat = x.reshape(B * H, *x.shape[2:])
    start, count = shard_units(B * H, world, rank)
    return flat[start:start + count]


def shard_kv_groups(q, k, v, world: int, rank: int):
    """Split attention inputs by (batch, kv-head) groups, keeping GQA groups whole.

    q: [B, Hq, T, D]; k, v: [B, Hkv, T, D].  Returns this rank's
    (q, k, v) as [1, n*G, T, D] / [1, n, T, D] blocks (n kv heads, G = Hq/Hkv).
    """
    B, Hq, T, D = q.shape
    Hkv = k.shape[1]
    G = Hq // Hkv
    start, count = shard_units(B * Hkv, world, rank)
    kq = k.reshape(B * Hkv, T, D)[start:start + count].unsqueeze(0)
    vq = v.reshape(B * Hkv, T, D)[start:start + count].unsqueeze(0)
    qq = q.reshape(B * Hkv, G, T, D)[start:start + count].reshape(1, count * G, T, D)
    return qq, kq, vq


def gather_units(local: torch.Tensor, n_units: int, group=None) -> torch.Tensor | None:
    """Concatenate every rank's block (leading dim = its unit count) on all ranks.

    Works with uneven blocks: blocks are padded to the largest one for the
    collective and trimmed afterwards.  Validation only; never on the hot path.
    """
    world = dist.get_world_size(group)
    counts = [shard_units(n_units, world, r)[1] for r in range(world)]
    top = max(counts)
    pad = torch.zeros((top,) + tuple(local.shape[1:]), dtype=local.dtype, device=local.device)
    pad[: local.shape[0]] = local
    if dist.get_backend(group) == "nccl":
        out = torch.empty((world * top,) + tuple(local.shape[1:]), dtype=local.dtype, device=local.device)
        dist.all_gather_into_tensor(out, pad, group=group)
        parts = list(out.split(top))
    else:
        parts = [torch.empty_like(pad) for _ in range(world)]
        dist.all_gather(parts, pad, group=group)
    return torch.cat([p[:c] for p, c in zip(parts, counts)])


# ---------------------------------------------------------------------------
# context parallelism: zig-zag sequence chunks, all-gathered K/V
# ---------------------------------------------------------------------------


def zigzag_chunk_ids(world: int, rank: int) -> tuple[int, int]:
    """The two of the 2*world sequence chunks held by ``rank``: (rank,
    2*world-1-rank).  Pairing an early chunk with a late one gives every rank
    the same causal work (chunk c sees c+1 key chunks)."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"bad rank {rank} for world size {world}")
    return rank, 2 * world - 1 - rank


def zigzag_split(x: torch.Tensor, world: int, rank: int, dim: int = 2) -> torch.Tensor:
    """This rank's two zig-zag chunks of the sequence dim of ``x``, concatenated."""
    T = x.shape[dim]
    if T % (2 * world):
        raise ValueError(f"sequence length {T} is not a multiple of 2*world = {2 * world}")
    chunks = x.chunk(2 * world, dim=dim)
    a, b = zigzag_chunk_ids(world, rank)
    return torch.cat([chunks[a], chunks[b]], dim=dim)


def zigzag_merge(parts, dim: int = 2) -> torch.Tensor:
    """Inverse of ``zigzag_split`` over all ranks: ``parts[r]`` is rank r's
    local tensor; returns the sequence in global order."""
    world = len(parts)
    chunks = [None] * (2 * world)
    for r, p in enumerate(parts):
        a, b = zigzag_chunk_ids(world, r)
        chunks[a], chunks[b] = p.chunk(2, dim=dim)
    return torch.cat(chunks, dim=dim)


def _all_gather(x: torch.Tensor, group=None) -> list:
    world = dist.get_world_size(group)
    x = x.contiguous()
    if dist.get_backend(group) == "nccl":
        out = torch.empty((world,) + tuple(x.shape), dtype=x.dtype, device=x.device)
        dist.all_gather_into_tensor(out, x, group=group)
        return list(out.unbind(0))
    parts = [torch.empty_like(x) for _ in range(world)]
    dist.all_gather(parts, x, group=group)
    return parts


def _reduce_scatter_zigzag(full: torch.Tensor, group=None, dim: int = 2) -> torch.Tensor:
    """Sum ``full`` (this rank's contribution over the whole sequence, in
    sequence order) over ranks and return this rank's two zig-zag chunks."""
    world = dist.get_world_size(group)
    rank = dist.get_rank(group)
    chunks = full.chunk(2 * world, dim=dim)
    blocks = [torch.cat([chunks[a], chunks[b]], dim=dim) for a, b in (zigzag_chunk_ids(world, r) for r in range(world))]
    if dist.get_backend(group) == "nccl":
        inp = torch.stack(blocks).contiguous()
        out = torch.empty_like(blocks[0])
        dist.reduce_scatter_tensor(out, inp, op=dist.ReduceOp.SUM, group=group)
        return out
    total = torch.stack(blocks).contiguous()  # gloo has no reduce_scatter: all-reduce, keep own block
    dist.all_reduce(total, op=dist.ReduceOp.SUM, group=group)
    return total[rank].clone()


def _key_span(c, C, window_size):
    """Keys [s0, e) that the queries of chunk c (positions c*C .. c*C+C-1) can
    see: the causal prefix, cut on the left by a sliding window.  The chunk
    kernels take keys from position 0, so callers pass the slice and the query
    offset c*C - s0 (relative positions keep the causal / window rule)."""
    e = (c + 1) * C
    s0 = max(0, c * C - window_size + 1) if window_size > 0 else 0
    return s0, e


def _cp_gather_kv(k, v, group):
    kv = torch.stack([k, v]).contiguous()
    return zigzag_merge(_all_gather(kv, group), dim=3)  # [2, B, Hkv, T, D] in sequence order


class _ContextParallelAttnFn(torch.autograd.Function):
    """Forward: all-gather K/V, chunk forwards.  Backward: all-gather K/V again,
    chunk backwards (dQ complete per local chunk, dK/dV contributions over the
    visible key prefix), then a reduce-scatter sums the dK/dV contributions of
    every rank into their owners' zig-zag chunks."""

    @staticmethod
    def forward(ctx, q, k, v, group, scale, window_size):
        from . import kernels

        world = dist.get_world_size(group)
        rank = dist.get_rank(group)
        C = q.shape[2] // 2
        full = _cp_gather_kv(k, v, group)
        train = any(ctx.needs_input_grad[:3])
        outs, sums, los = [], [], []
        for i, c in enumerate(zigzag_chunk_ids(world, rank)):
            qc = q[:, :, i * C:(i + 1) * C]
            s0, e = _key_span(c, C, window_size)
            res = kernels.sp2norm_flash_attention_chunk(qc, full[0, :, :, s0:e], full[1, :, :, s0:e], c * C - s0,
                                                        scale=scale, window_size=window_size, return_residual=train)
            outs.append(res[0])
            sums.append(res[1])
            if train:
                los.append(res[2])
        o = torch.cat(outs, dim=2)
        ctx.save_for_backward(q, k, v, o, torch.cat(sums, dim=2), torch.cat(los, dim=2) if train else None)
        ctx.group, ctx.scale, ctx.window_size = group, scale, window_size
        return o

    @staticmethod
    def backward(ctx, do):
        from . import kernels

        q, k, v, o, sums, o_lo = ctx.saved_tensors
        group = ctx.group
        world = dist.get_world_size(group)
        rank = dist.get_rank(group)
        C = q.shape[2] // 2
        full = _cp_gather_kv(k, v, group)
        T = full.shape[3]
        dk_full = torch.zeros(full.shape[1:], dtype=torch.float32, device=q.device)
        dv_full = torch.zeros_like(dk_full)
        dqs = []
        for i, c in enumerate(zigzag_chunk_ids(world, rank)):
            sl = slice(i * C, (i + 1) * C)
            s0, e = _key_span(c, C, ctx.window_size)
            dq, dk, dv = kernels.sp2norm_flash_attention_chunk_bwd(
                q[:, :, sl], full[0, :, :, s0:e], full[1, :, :, s0:e], o[:, :, sl], do[:, :, sl].contiguous(),
                sums[:, :, sl].contiguous(), c * C - s0, scale=ctx.scale, window_size=ctx.window_size,
                o_lo=None if o_lo is None else o_lo[:, :, sl])
            dqs.append(dq)
            dk_full[:, :, s0:e] += dk.float()
            dv_full[:, :, s0:e] += dv.float()
        assert dk_full.shape[2] == T
        dk_loc = _reduce_scatter_zigzag(dk_full, group).to(k.dtype)
        dv_loc = _reduce_scatter_zigzag(dv_full, group).to(v.dtype)
        return torch.cat(dqs, dim=2), dk_loc, dv_loc, None, None, None


def context_parallel_attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, *, group=None, scale=None,
                               window_size: int = 0) -> torch.Tensor:
    """Causal squareplus attention with the sequence split over ranks.

    q, k, v are this rank's zig-zag local blocks ``[B, H, 2C, D]`` (see
    ``zigzag_split``; the global length is T = 2·C·world).  Forward: K and V
    are all-gathered once (NCCL over NVLink on GPUs) and put back in sequence
    order; each of the rank's two query chunks runs the tcgen05 forward
    against its visible key prefix (``sp2norm_flash_attention_chunk`` with the
    chunk's global offset).  The squareplus normalizer is a plain sum, so no
    cross-rank max or rescale is needed: the result equals the single-GPU
    forward.  Backward (autograd): K/V are gathered again, each local chunk
    runs ``sp2norm_flash_attention_chunk_bwd``, dQ stays local and the dK/dV
    contributions are summed into their owners' chunks by one
    reduce-scatter.  Returns the rank's output in the zig-zag local layout.
    """
    if q.shape[2] % 2:
        raise ValueError("the local sequence block must hold two equal zig-zag chunks")
    return _ContextParallelAttnFn.apply(q, k, v, group, scale, window_size)

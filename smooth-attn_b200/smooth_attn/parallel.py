"""Multi-GPU plumbing for the smooth-attn path: one process per GPU.

The normalization and attention work is a set of independent units — score
matrices (batch, head) for the norm, (batch, kv-head) groups for attention
(GQA groups stay whole because a kv head's gradients sum over its query
heads).  Units are split into contiguous blocks, one per rank, and every
rank runs the single-GPU kernels on its block; there is no collective on the
data path.  ``gather_units`` collects the per-rank blocks (NCCL over NVLink on
GPUs, gloo on CPU) for validation only.
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

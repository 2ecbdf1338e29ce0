"""Independent partitions of the hot path across the GPUs of one node.

Each family splits into units that need nothing from one another: attention
by (batch, head), the GEMM by row blocks of A (M-tiles, B replicated), the row
family by rows. A rank computes its contiguous range of units on its own GPU;
there is no collective on the data path. ``gather`` reassembles a full result
on every rank (all_gather) only where a caller needs one, outside the timed
kernels. The reference is single-GPU (its README's "Apple Silicon is
single-GPU"), so this module has no reference counterpart.
"""
from __future__ import annotations

from typing import Optional, Sequence, Tuple

import torch


def unit_range(n_units: int, world: int, rank: int, align: int = 1) -> Tuple[int, int]:
    """Contiguous [start, stop) of ``n_units`` for ``rank`` of ``world``.

    Units are handed out in blocks of ``align`` (e.g. 128-row M-tiles) as evenly
    as possible; earlier ranks get the extra block when the count does not divide.
    """
    if world <= 0 or not 0 <= rank < world:
        raise ValueError(f"bad rank {rank} for world {world}")
    if n_units < 0 or align <= 0:
        raise ValueError("n_units must be >= 0 and align > 0")
    blocks = (n_units + align - 1) // align
    base, extra = divmod(blocks, world)
    b0 = rank * base + min(rank, extra)
    b1 = b0 + base + (1 if rank < extra else 0)
    return min(b0 * align, n_units), min(b1 * align, n_units)


def attention_shard(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, world: int,
                    rank: int) -> Tuple[torch.Tensor, torch.Tensor, torch.Tensor, Tuple[int, int]]:
    """This rank's (batch, head) units of [B, H, S, D] tensors, as [1, n, S, D] views.

    The (b, h) pairs are flattened b-major; views are taken without copies when the
    batch and head dimensions can be merged, else the slice is made contiguous.
    """
    B, H, S, D = q.shape
    lo, hi = unit_range(B * H, world, rank)

    def take(t):
        try:
            flat = t.view(B * H, S, D)
        except RuntimeError:
            flat = t.reshape(B * H, S, D)
        return flat[lo:hi].unsqueeze(0)

    return take(q), take(k), take(v), (lo, hi)


def gemm_shard(a: torch.Tensor, world: int, rank: int, tile: int = 128) -> Tuple[torch.Tensor, Tuple[int, int]]:
    """This rank's rows of A (whole 128-row M-tiles); B is used whole by every rank."""
    lo, hi = unit_range(a.shape[0], world, rank, align=tile)
    return a[lo:hi], (lo, hi)


def rows_shard(x: torch.Tensor, world: int, rank: int) -> Tuple[torch.Tensor, Tuple[int, int]]:
    lo, hi = unit_range(x.shape[0], world, rank)
    return x[lo:hi], (lo, hi)


def gather(local: torch.Tensor, ranges: Sequence[Tuple[int, int]], dim: int,
           group: Optional["torch.distributed.ProcessGroup"] = None) -> torch.Tensor:
    """All-gather the per-rank pieces (uneven sizes allowed) along ``dim``.

    ``ranges`` is every rank's [start, stop) in rank order (``unit_range`` for each
    rank). Pieces are padded to the largest one for the collective and trimmed.
    """
    import torch.distributed as dist
    world = dist.get_world_size(group)
    if len(ranges) != world:
        raise ValueError("need one range per rank")
    sizes = [b - a for a, b in ranges]
    mx = max(sizes) if sizes else 0
    local = local.movedim(dim, 0).contiguous()
    if local.shape[0] != sizes[dist.get_rank(group)]:
        raise ValueError("local piece does not match this rank's range")
    pad = torch.zeros((mx,) + tuple(local.shape[1:]), dtype=local.dtype, device=local.device)
    pad[: local.shape[0]] = local
    parts = [torch.empty_like(pad) for _ in range(world)]
    dist.all_gather(parts, pad, group=group)
    full = torch.cat([p[:n] for p, n in zip(parts, sizes)], dim=0)
    return full.movedim(0, dim)


def sharded_flash_attn(q, k, v, causal: bool = False, sm_scale: Optional[float] = None,
                       group=None, gather_output: bool = True):
    """Attention over this rank's (batch, head) units; optionally all-gather O.

    Every rank passes the full (or identically shaped) q/k/v; returns O for all
    units if ``gather_output`` else this rank's [1, n, S, D] piece.
    """
    import torch.distributed as dist
    from .ops import flash_attn_fwd
    world, rank = dist.get_world_size(group), dist.get_rank(group)
    B, H, S, D = q.shape
    ql, kl, vl, _ = attention_shard(q, k, v, world, rank)
    o = flash_attn_fwd(ql, kl, vl, causal=causal, sm_scale=sm_scale)
    if not gather_output:
        return o
    ranges = [unit_range(B * H, world, r) for r in range(world)]
    return gather(o[0], ranges, 0, group).view(B, H, S, D)

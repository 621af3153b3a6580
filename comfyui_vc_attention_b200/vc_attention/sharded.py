"""(batch, head)-sharded VC-Attention across the ranks of one node.

Every stage of the path is independent per (b, h) unit: the V-Smooth
permutation (grouping.py:160-186), the smooth-K mean (triton_attn.py:546),
the block statistics and the kernel grid (triton_attn.py:804) are all per
head.  Rank r of P therefore owns the contiguous unit range
[r*ceil(U/P), min(U, (r+1)*ceil(U/P))) of the flattened B*H axis, computes it
with the CUDA path, and, when the caller needs the whole tensor, one NCCL
all-gather assembles the (B, H, N, D) output.  There is no other exchange.

The all-gather moves equal slabs of ceil(U/P) units per rank into a padded
buffer; the padding units (when P does not divide U) are never read.
"""

from __future__ import annotations

from typing import Callable, Optional, Tuple

import torch

__all__ = ["shard_units", "vc_attention_sharded"]


def shard_units(units: int, world: int, rank: int) -> Tuple[int, int]:
    """Contiguous unit range [lo, hi) owned by ``rank``; empty for ranks past
    the end when ``world`` exceeds ``units``."""
    if world <= 0 or not 0 <= rank < world:
        raise ValueError(f"rank {rank} outside world {world}")
    per = -(-units // world)
    lo = min(units, rank * per)
    return lo, min(units, lo + per)


def _local_units(q, k, v, perm, lo, hi, compute):
    b, h, n, d = q.shape
    g = b * h
    ql = q.reshape(g, n, d)[lo:hi].unsqueeze(0)
    kl = k.reshape(g, n, d)[lo:hi].unsqueeze(0)
    vl = v.reshape(g, n, d)[lo:hi].unsqueeze(0)
    pl = None
    if perm is not None:
        pl = perm if perm.shape[0] == 1 else perm[lo:hi]
    return compute(ql, kl, vl, pl).reshape(hi - lo, n, d)


def vc_attention_sharded(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor,
                         perm: Optional[torch.Tensor] = None, cfg=None, scale: Optional[float] = None,
                         group=None, gather: bool = True,
                         compute: Optional[Callable] = None) -> torch.Tensor:
    """VC-Attention over this rank's (b, h) units, optionally all-gathered.

    q, k, v: (B, H, N, D), the same full tensors on every rank (views are
    sliced, not copied).  perm: (B*H, N) or (1, N) int32, or None.
    Returns the full (B, H, N, D) output on every rank when ``gather``, else
    this rank's (hi - lo, N, D) slab (unit range from :func:`shard_units`).
    ``compute`` (tests only) replaces the CUDA attention call; it receives
    (1, units, N, D) tensors and the matching permutation rows.
    """
    import torch.distributed as dist

    if compute is None:
        from .kernels.cuda_attn import vc_attention_cuda

        def compute(ql, kl, vl, pl):
            return vc_attention_cuda(ql, kl, vl, pl, cfg, scale)

    world = dist.get_world_size(group) if dist.is_initialized() else 1
    rank = dist.get_rank(group) if dist.is_initialized() else 0
    b, h, n, d = q.shape
    units = b * h
    lo, hi = shard_units(units, world, rank)
    per = -(-units // world)
    local = torch.zeros((per, n, d), dtype=q.dtype, device=q.device)
    if hi > lo:
        local[: hi - lo] = _local_units(q, k, v, perm, lo, hi, compute)
    if not gather:
        return local[: hi - lo]
    if world == 1:
        return local[:units].reshape(b, h, n, d)
    full = torch.empty((world * per, n, d), dtype=q.dtype, device=q.device)
    dist.all_gather_into_tensor(full, local, group=group)
    return full[:units].reshape(b, h, n, d)

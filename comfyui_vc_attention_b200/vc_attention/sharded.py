"""(batch, head)-sharded VC-Attention across the ranks of one node.

Every stage of the path is independent per (b, h) unit: the V-Smooth
permutation (grouping.py:160-186), the smooth-K mean (triton_attn.py:546),
the block statistics and the kernel grid (triton_attn.py:804) are all per
head.  So the units are dealt out to the ranks with no exchange, and only
when the caller needs the whole tensor do NCCL all-gathers assemble the
(B, H, N, D) output.

Two layouts:

* ``chunk=None``: rank r owns the contiguous range
  [r*ceil(U/P), min(U, (r+1)*ceil(U/P))) of the flattened B*H axis and one
  all-gather of equal padded slabs assembles the output after the compute.
* ``chunk=c``: the units are dealt in rounds of P*c, rank r taking units
  [i*P*c + r*c, i*P*c + (r+1)*c) of round i.  Round i's slabs then sit next to
  each other in the output, so its all-gather writes them in place, and it is
  issued asynchronously while round i+1 computes: the transfer overlaps the
  remaining heads and only the last round's gather is exposed.  The rank's
  units of all rounds are prepared in one call up front (a strided view of
  Q/K/V), so the rounds run only the attention kernel.  The attention CTA
  holds a whole SM (its registers), so an NCCL kernel runs only on SMs the
  attention leaves idle or as attention CTAs retire: a high-priority NCCL
  stream makes the waiting NCCL CTAs take those SMs first.

With ``transport="peer"`` (CUDA, chunked layout) the gather uses no SMs:
the full output lives in symmetric memory (every rank maps every other
rank's buffer), each round's attention writes straight into the rank's own
slice of it, and a copy stream pushes that slice into every peer's buffer
with device-to-device copies, which the copy engines carry over NVLink while
the next rounds compute.  One small NCCL all-reduce after the pushes tells
every rank that all slices have arrived.  The returned tensor is then that
persistent buffer (one per shape, dtype, device and group, held until the
process exits), which the next call of the same shape overwrites.

Padding units (past U) are never computed; their output rows are zeros in
the padded buffer and are never returned.
"""

from __future__ import annotations

from typing import Callable, List, Optional, Tuple

import torch

__all__ = ["shard_units", "rank_units", "vc_attention_sharded"]


def shard_units(units: int, world: int, rank: int) -> Tuple[int, int]:
    """Contiguous unit range [lo, hi) owned by ``rank``; empty for ranks past
    the end when ``world`` exceeds ``units``."""
    if world <= 0 or not 0 <= rank < world:
        raise ValueError(f"rank {rank} outside world {world}")
    per = -(-units // world)
    lo = min(units, rank * per)
    return lo, min(units, lo + per)


def rank_units(units: int, world: int, rank: int, chunk: Optional[int] = None) -> List[Tuple[int, int]]:
    """Unit ranges [lo, hi) owned by ``rank``, in output order: one range for
    ``chunk=None`` (:func:`shard_units`), else one per round of ``world * chunk``
    units (empty ranges of a partial last round left out)."""
    if chunk is None:
        lo, hi = shard_units(units, world, rank)
        return [(lo, hi)] if hi > lo else []
    if world <= 0 or not 0 <= rank < world:
        raise ValueError(f"rank {rank} outside world {world}")
    if chunk <= 0:
        raise ValueError("chunk must be positive")
    out = []
    for base in range(0, units, world * chunk):
        lo = min(units, base + rank * chunk)
        hi = min(units, lo + chunk)
        if hi > lo:
            out.append((lo, hi))
    return out


_ROUND_STREAMS = {}


def _round_streams(dev: torch.device):
    """Two compute streams per device for the rounds of the chunked layout
    (kept for the process: the caching allocator keeps freed blocks per stream)."""
    key = dev.index
    if key not in _ROUND_STREAMS:
        _ROUND_STREAMS[key] = (torch.cuda.Stream(dev), torch.cuda.Stream(dev))
    return _ROUND_STREAMS[key]


_COPY_STREAMS = {}
_PEER_BUFFERS = {}


def _copy_stream(dev: torch.device):
    """The stream that pushes a rank's round slices to its peers."""
    key = dev.index
    if key not in _COPY_STREAMS:
        _COPY_STREAMS[key] = torch.cuda.Stream(dev)
    return _COPY_STREAMS[key]


def _peer_output(shape, dtype, device, group):
    """(this rank's buffer, every rank's buffer as mapped here) of one output
    shape in symmetric memory, made once per (shape, dtype, device, group) by a
    rendezvous of all ranks of the group."""
    import os

    import torch.distributed as dist
    import torch.distributed._symmetric_memory as symm
    # plain peer mappings only: the pushes are copy-engine copies, and a
    # buffer bound to an NVLink multicast object is not needed (nor wanted
    # when a rank can end while its peers still hold the mapping)
    os.environ.setdefault("TORCH_SYMM_MEM_DISABLE_MULTICAST", "1")
    pg = group if group is not None else dist.group.WORLD
    key = (tuple(shape), dtype, device.index, pg.group_name)
    if key not in _PEER_BUFFERS:
        buf = symm.empty(*shape, dtype=dtype, device=device)
        hdl = symm.rendezvous(buf, pg)
        views = [buf if r == hdl.rank else hdl.get_buffer(r, tuple(shape), dtype) for r in range(hdl.world_size)]
        _PEER_BUFFERS[key] = (buf, views, hdl)
    return _PEER_BUFFERS[key][:2]


def _compute_units(q, k, v, perm, lo, hi, compute, dst, cfg=None, scale=None):
    """Attention of units [lo, hi), written to ``dst`` (hi - lo, N, D): by
    ``compute`` when given (tests), else by the CUDA kernels straight into
    ``dst``."""
    b, h, n, d = q.shape
    g = b * h
    ql = q.reshape(g, n, d)[lo:hi].unsqueeze(0)
    kl = k.reshape(g, n, d)[lo:hi].unsqueeze(0)
    vl = v.reshape(g, n, d)[lo:hi].unsqueeze(0)
    pl = None
    if perm is not None:
        pl = perm if perm.shape[0] == 1 else perm[lo:hi]
    if compute is None:
        from .kernels.cuda_attn import _attention_into
        _attention_into(ql, kl, vl, pl, cfg, scale, dst.unsqueeze(0))
    else:
        dst.copy_(compute(ql, kl, vl, pl).reshape(hi - lo, n, d))


def vc_attention_sharded(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor,
                         perm: Optional[torch.Tensor] = None, cfg=None, scale: Optional[float] = None,
                         group=None, gather: bool = True, chunk: Optional[int] = None,
                         compute: Optional[Callable] = None, overlap_rounds: bool = True,
                         transport: str = "nccl") -> torch.Tensor:
    """VC-Attention over this rank's (b, h) units, optionally all-gathered.

    q, k, v: (B, H, N, D), the same full tensors on every rank (views are
    sliced, not copied).  perm: (B*H, N) or (1, N) int32, or None.
    chunk: None (one contiguous range per rank, one gather after the
    compute) or units per rank per round (round-robin layout, each round's
    gather overlapping the next round's compute).
    Returns the full (B, H, N, D) output on every rank when ``gather``, else
    this rank's units stacked in output order, (units, N, D), as listed by
    :func:`rank_units`.  ``compute`` (tests only) replaces the CUDA
    attention call; it receives (1, units, N, D) tensors and the matching
    permutation rows.  In the chunked layout the rank's units are prepared
    once up front and each round runs the attention kernel into its slab;
    ``overlap_rounds`` runs consecutive rounds on two streams, so one
    round's last partial wave of attention CTAs shares the GPU with the next
    round's first; the NCCL kernels then get SMs only as attention CTAs
    retire, which is prompt when the process group's NCCL stream has high
    priority (``ProcessGroupNCCL.Options.is_high_priority_stream``).  Without
    it the rounds run in order on the caller's stream.
    ``transport``: "nccl" (an all-gather per round) or "peer" (CUDA tensors
    and the chunked layout with ``gather``: copy-engine pushes into the
    peers' symmetric-memory buffers, see the module notes; the result is a
    persistent buffer that the next call of the same shape overwrites).
    """
    import torch.distributed as dist

    if transport not in ("nccl", "peer"):
        raise ValueError(f"transport must be 'nccl' or 'peer', got {transport!r}")
    world = dist.get_world_size(group) if dist.is_initialized() else 1
    rank = dist.get_rank(group) if dist.is_initialized() else 0
    b, h, n, d = q.shape
    units = b * h
    if world == 1:
        chunk = None
    if chunk is None:
        lo, hi = shard_units(units, world, rank)
        per = -(-units // world)
        local = torch.empty((per, n, d), dtype=q.dtype, device=q.device)
        local[max(0, hi - lo):].zero_()
        if hi > lo:
            _compute_units(q, k, v, perm, lo, hi, compute, local[: hi - lo], cfg, scale)
        if not gather:
            return local[: hi - lo]
        if world == 1:
            return local[:units].reshape(b, h, n, d)
        full = torch.empty((world * per, n, d), dtype=q.dtype, device=q.device)
        dist.all_gather_into_tensor(full, local, group=group)
        return full[:units].reshape(b, h, n, d)

    rounds = -(-units // (world * chunk))
    peer = transport == "peer" and gather and q.is_cuda and compute is None
    if peer:
        full, views = _peer_output((rounds * world * chunk, n, d), q.dtype, q.device, group)
        cstream = _copy_stream(q.device)
    else:
        full = torch.empty((rounds * world * chunk, n, d), dtype=q.dtype, device=q.device) if gather else None
    mine = []
    works = []
    cur = torch.cuda.current_stream(q.device) if q.is_cuda else None
    streams = _round_streams(q.device) if (q.is_cuda and overlap_rounds) else None
    if streams is not None:
        for st in streams:
            st.wait_stream(cur)
    preps = _prepare_rounds(q, k, v, perm, cfg, scale, world, rank, chunk) if compute is None else None
    for i in range(rounds):
        base = i * world * chunk
        lo = min(units, base + rank * chunk)
        hi = min(units, lo + chunk)
        ctx = torch.cuda.stream(streams[i % 2]) if streams is not None else _nullctx()
        with ctx:
            if peer:
                slab = full[base + rank * chunk: base + (rank + 1) * chunk]
            else:
                slab = torch.empty((chunk, n, d), dtype=q.dtype, device=q.device)
            slab[max(0, hi - lo):].zero_()
            if hi > lo:
                if preps is None:
                    _compute_units(q, k, v, perm, lo, hi, compute, slab[: hi - lo], cfg, scale)
                else:
                    from .kernels.cuda_attn import _call_config, attention_prepared
                    # rounds overlap one another: no KV split of a round's last
                    # wave (each unit equals its single-GPU call bit for bit)
                    attention_prepared(preps(i), n, slab[: hi - lo].unsqueeze(0), scale if scale else d ** -0.5,
                                       _call_config(cfg, d), kv_split=1)
                mine.append(slab[: hi - lo])
            if peer:
                done = torch.cuda.Event()
                done.record()
            elif gather:
                # every rank issues every round, in the same order, with equal
                # slabs; NCCL orders the transfer after this round's compute
                works.append((dist.all_gather_into_tensor(full[base: base + world * chunk], slab, group=group,
                                                          async_op=True), slab))
        if peer:
            # push this round's slice into every peer's buffer (contiguous
            # device-to-device copies: copy engines over NVLink, no SMs)
            cstream.wait_event(done)
            with torch.cuda.stream(cstream):
                lo_r, hi_r = base + rank * chunk, base + (rank + 1) * chunk
                for r in range(world):
                    if r != rank:
                        views[r][lo_r:hi_r].copy_(slab)
    for w, _ in works:
        w.wait()
    if streams is not None:
        for st in streams:
            cur.wait_stream(st)
    if peer:
        # every rank's pushes are done once every rank has reached this
        # all-reduce (each enters it after its own copy stream drained)
        cur.wait_stream(cstream)
        flag = torch.zeros(1, dtype=torch.float32, device=q.device)
        dist.all_reduce(flag, group=group)
    if not gather:
        return torch.cat(mine, 0) if mine else torch.zeros((0, n, d), dtype=q.dtype, device=q.device)
    return full[:units].reshape(b, h, n, d)


def _prepare_rounds(q, k, v, perm, cfg, scale, world, rank, chunk):
    """Prepare this rank's units of every round up front, in one call for the
    full rounds (a strided (rounds, chunk, N, D) view of Q/K/V, no copy) and
    one for a partial last round: the prepare kernels then run on all of the
    rank's heads at once instead of a few heads per round, and the rounds run
    only the attention kernel.  Returns round index -> Prepared of that round."""
    from .kernels.cuda_attn import prepare_for, slice_prepared
    b, h, n, d = q.shape
    units = b * h
    span = world * chunk
    r_full = units // span
    out = {}
    if r_full:
        def rows(t):
            return t.reshape(units, n, d)[: r_full * span].view(r_full, world, chunk, n, d)[:, rank]
        pv = None
        if perm is not None:
            pv = (perm.expand(units, n) if perm.shape[0] == 1 else perm)[: r_full * span]
            pv = pv.view(r_full, world, chunk, n)[:, rank].reshape(r_full * chunk, n)
        p_all = prepare_for(rows(q), rows(k), rows(v), pv, cfg, scale)
        for i in range(r_full):
            out[i] = (p_all, i)
    lo = min(units, r_full * span + rank * chunk)
    hi = min(units, lo + chunk)
    if hi > lo:
        sl = [t.reshape(units, n, d)[lo:hi].unsqueeze(0) for t in (q, k, v)]
        pl = None if perm is None else (perm if perm.shape[0] == 1 else perm[lo:hi])
        out[r_full] = (prepare_for(*sl, pl, cfg, scale), 0)

    def get(i):
        p, j = out[i]
        return slice_prepared(p, j)
    return get


class _nullctx:
    def __enter__(self):
        return None

    def __exit__(self, *exc):
        return False

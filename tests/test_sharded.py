"""(batch, head) sharding and output all-gather (world size 2, gloo, CPU).

The attention call itself is replaced by a per-unit stand-in here: these
tests check the partition and the assembly, which are pure host logic; the
CUDA path is covered by the GPU parity tests."""

import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

from comfyui_vc_attention_b200.vc_attention.sharded import shard_units, vc_attention_sharded


def test_shard_units_cover_every_unit_once():
    for units in (1, 7, 56, 112):
        for world in (1, 2, 3, 4, 8):
            got = []
            for r in range(world):
                lo, hi = shard_units(units, world, r)
                assert 0 <= lo <= hi <= units
                got.extend(range(lo, hi))
            assert got == list(range(units))
    with pytest.raises(ValueError):
        shard_units(4, 2, 2)


def _stand_in(ql, kl, vl, pl):
    # depends on the unit's own data only (and on perm when given)
    out = ql + 2.0 * kl - vl
    if pl is not None:
        out = out + pl.to(out.dtype).reshape(1, -1, out.shape[2], 1)[:, : out.shape[1]] * 1e-3
    return out


def _worker(rank, world, port, b, h, n, d, with_perm, ret):
    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        g = torch.Generator().manual_seed(0)
        q = torch.randn(b, h, n, d, generator=g)
        k = torch.randn(b, h, n, d, generator=g)
        v = torch.randn(b, h, n, d, generator=g)
        perm = torch.stack([torch.randperm(n, generator=g) for _ in range(b * h)]).int() if with_perm else None
        full = vc_attention_sharded(q, k, v, perm, compute=_stand_in)
        ref = _stand_in(q.reshape(1, b * h, n, d), k.reshape(1, b * h, n, d), v.reshape(1, b * h, n, d),
                        perm).reshape(b, h, n, d)
        ok = torch.equal(full, ref)
        lo, hi = shard_units(b * h, world, rank)
        part = vc_attention_sharded(q, k, v, perm, compute=_stand_in, gather=False)
        ok = ok and part.shape[0] == hi - lo and torch.equal(part, ref.reshape(b * h, n, d)[lo:hi])
        ret[rank] = int(ok)
    finally:
        dist.destroy_process_group()


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


@pytest.mark.parametrize("b,h,with_perm", [(2, 3, True), (1, 5, False), (2, 4, True)])
def test_sharded_gather_matches_unsharded(b, h, with_perm):
    world = 2
    ctx = mp.get_context("spawn")
    ret = ctx.Array("i", [0] * world)
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, b, h, 16, 8, with_perm, ret)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    assert list(ret) == [1] * world

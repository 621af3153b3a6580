"""(batch, head) sharding and output all-gather (world size 2, gloo, CPU).

The attention call itself is replaced by a per-unit stand-in here: these
tests check the partition and the assembly, which are pure host logic; the
CUDA path is covered by the GPU parity tests."""

import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

from comfyui_vc_attention_b200.vc_attention.sharded import rank_units, shard_units, vc_attention_sharded


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


def test_rank_units_rounds_cover_every_unit_once():
    for units in (1, 7, 56, 112):
        for world in (1, 2, 3, 8):
            for chunk in (None, 1, 3, 14):
                got = []
                for r in range(world):
                    for lo, hi in rank_units(units, world, r, chunk):
                        assert 0 <= lo < hi <= units and (chunk is None or hi - lo <= chunk)
                        got.extend(range(lo, hi))
                assert sorted(got) == list(range(units))
    # round-robin: round i of world*chunk units, rank r at offset r*chunk
    assert rank_units(10, 2, 1, 2) == [(2, 4), (6, 8)]
    assert rank_units(10, 2, 0, 2) == [(0, 2), (4, 6), (8, 10)]


def _stand_in(ql, kl, vl, pl):
    # depends on the unit's own data only (and on perm when given)
    out = ql + 2.0 * kl - vl
    if pl is not None:
        out = out + pl.to(out.dtype).reshape(1, -1, out.shape[2], 1)[:, : out.shape[1]] * 1e-3
    return out


def _worker(rank, world, port, b, h, n, d, with_perm, ret, chunk=None, transport="nccl"):
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
        full = vc_attention_sharded(q, k, v, perm, compute=_stand_in, chunk=chunk, transport=transport)
        ref = _stand_in(q.reshape(1, b * h, n, d), k.reshape(1, b * h, n, d), v.reshape(1, b * h, n, d),
                        perm).reshape(b, h, n, d)
        ok = torch.equal(full, ref)
        part = vc_attention_sharded(q, k, v, perm, compute=_stand_in, gather=False, chunk=chunk,
                                    transport=transport)
        flat = ref.reshape(b * h, n, d)
        mine = [flat[lo:hi] for lo, hi in rank_units(b * h, world, rank, chunk)]
        want = torch.cat(mine, 0) if mine else flat[:0]
        ok = ok and part.shape == want.shape and torch.equal(part, want)
        ret[rank] = int(ok)
    finally:
        dist.destroy_process_group()


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


@pytest.mark.parametrize("b,h,with_perm,chunk,transport", [
    (2, 3, True, None, "nccl"), (1, 5, False, None, "nccl"), (2, 4, True, None, "nccl"),
    (2, 3, True, 1, "nccl"), (1, 5, False, 2, "nccl"), (2, 4, True, 3, "nccl"),
    # the copy-engine transport needs CUDA tensors: host tensors (and the
    # test stand-in) take the collective all-gather with the same layout
    (2, 4, True, 3, "peer")])
def test_sharded_gather_matches_unsharded(b, h, with_perm, chunk, transport):
    world = 2
    ctx = mp.get_context("spawn")
    ret = ctx.Array("i", [0] * world)
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, b, h, 16, 8, with_perm, ret, chunk, transport))
             for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    assert list(ret) == [1] * world


def test_unknown_transport_is_refused():
    q = torch.zeros(1, 2, 4, 8)
    with pytest.raises(ValueError, match="transport"):
        # checked before anything runs, with or without a process group
        import torch.distributed as dist
        assert not dist.is_initialized()
        vc_attention_sharded(q, q, q, None, compute=_stand_in, chunk=1, transport="ring")

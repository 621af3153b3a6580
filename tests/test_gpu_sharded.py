"""Multi-GPU (batch, head) sharding on real GPUs: the all-gathered output of
vc_attention_sharded equals single-GPU calls of every unit, bit for bit, with
the NCCL all-gathers and with the copy-engine pushes into symmetric memory
(twice in a row: the second call reuses the persistent buffer).

Runs as two spawned ranks over NCCL when two GPUs are visible; skipped
otherwise (the host-side partition logic is covered on CPU by
tests/test_sharded.py with gloo ranks).  NVLS is off (NCCL_NVLS_ENABLE=0) and
the process group has a short timeout, so a rank that fails ends the others'
collectives with an error instead of a wait.
"""

import os
import socket

import pytest
import torch

pytestmark = pytest.mark.gpu


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank, world, port, result_dir):
    import datetime

    import numpy as np
    import torch.distributed as dist

    from comfyui_vc_attention_b200.vc_attention.kernels.cuda_attn import (TritonConfig, attention_status,
                                                                          vc_attention_cuda)
    from comfyui_vc_attention_b200.vc_attention.sharded import vc_attention_sharded
    from oracle.inputs import make_qkv

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    dev = torch.device("cuda", rank)
    torch.cuda.set_device(dev)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=dev)
    ok = True
    msg = ""
    try:
        b, h, n, d = 2, 5, 1000, 128      # 10 units: uneven over 2 ranks in rounds of 3
        q, k, v = (torch.from_numpy(a).to(dev).to(torch.bfloat16) for a in make_qkv(b, h, n, d, seed=41))
        g = b * h
        perm = torch.stack([torch.from_numpy(np.random.default_rng(50 + i).permutation(n)) for i in range(g)])
        perm = perm.to(torch.int32).to(dev)
        cfg = TritonConfig(block_n=128, enable_expcast=True)
        for chunk, transport in ((None, "nccl"), (3, "nccl"), (3, "peer"), (3, "peer")):
            full = vc_attention_sharded(q, k, v, perm, cfg, d ** -0.5, gather=True, chunk=chunk,
                                        transport=transport)
            torch.cuda.synchronize()
            for u in range(g):
                ref = vc_attention_cuda(q.reshape(g, n, d)[u:u + 1].unsqueeze(0),
                                        k.reshape(g, n, d)[u:u + 1].unsqueeze(0),
                                        v.reshape(g, n, d)[u:u + 1].unsqueeze(0), perm[u:u + 1], cfg,
                                        d ** -0.5)
                if not torch.equal(ref.reshape(n, d), full.reshape(g, n, d)[u]):
                    ok = False
                    msg += f"chunk={chunk} {transport} unit {u} differs; "
        if attention_status() != (0, 0, 0):
            ok = False
            msg += "device status set; "
    except Exception as e:  # reported to the parent through the result file
        ok = False
        msg += f"{type(e).__name__}: {e}"
    finally:
        dist.barrier()
        dist.destroy_process_group()
    with open(os.path.join(result_dir, f"rank{rank}.txt"), "w") as f:
        f.write(("OK " if ok else "FAIL ") + msg)


def test_sharded_output_equals_single_gpu_on_two_gpus(tmp_path):
    if not torch.cuda.is_available() or torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    import torch.multiprocessing as mp
    mp.start_processes(_rank_main, args=(2, _free_port(), str(tmp_path)), nprocs=2, start_method="spawn",
                       join=True)
    for r in range(2):
        text = (tmp_path / f"rank{r}.txt").read_text()
        assert text.startswith("OK"), f"rank {r}: {text}"
